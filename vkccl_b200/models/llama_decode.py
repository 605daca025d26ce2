# SPDX-License-Identifier: Apache-2.0
"""Llama-3-70B-shaped tensor-parallel decode step (hidden 8192, 80 layers).

Per layer and rank (TP = n, bf16, random-init weights):

    qkv   = x_norm @ W_qkv^T          [B, (64 + 2 * 8) * 128 / n]   column parallel
    attn  = qkv[:, :8192 / n]           (stand-in for attention over the KV cache)
    part  = attn @ W_o^T              [B, 8192]   row parallel -> partial sums
    x, x_norm = AllReduce(part) + x, RMSNorm(...)          <- fused kernel
    h     = silu(x_norm W_g^T) * (x_norm W_u^T)  [B, 28672 / n]  column parallel
    part  = h @ W_d^T                 [B, 8192]   row parallel -> partial sums
    x, x_norm = AllReduce(part) + x, RMSNorm(...)          <- fused kernel

so every layer does two all-reduces of [B, 8192] fused with the residual add
and RMSNorm (eps 1e-5), as in vLLM's TP decode.  ``step`` runs the 80
layers with this library's GEMMs and ``vcclAllReduceAddRMSNorm``;
``step_nccl`` runs the same layers with cuBLAS, NCCL all-reduce and a torch
RMSNorm.  The attention core is replaced by a slice of the QKV projection,
identical in both paths, so the comparison isolates the TP communication
and the GEMMs.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from vkccl_b200.ops.fused import all_reduce_add_rms_norm
from vkccl_b200.ops.gemm import gemm_bf16, gemm_silu_mul, interleave_gate_up


@dataclass
class DecodeConfig:
    hidden: int = 8192
    intermediate: int = 28672
    heads: int = 64
    kv_heads: int = 8
    head_dim: int = 128
    layers: int = 80
    eps: float = 1e-5
    init_std: float = 0.02


class TPLlamaDecode:
    def __init__(self, comm, cfg: DecodeConfig = DecodeConfig(), seed: int = 0, device: str = "cuda"):
        self.comm, self.cfg = comm, cfg
        n, r = comm.nranks, comm.rank
        h = cfg.hidden
        self.qkv_out = (cfg.heads + 2 * cfg.kv_heads) * cfg.head_dim // n
        self.attn_out = h // n
        self.inter = cfg.intermediate // n
        g = torch.Generator(device=device).manual_seed(seed * 7919 + r)

        def w(rows, cols):
            return (torch.randn(rows, cols, generator=g, device=device) * cfg.init_std).bfloat16()

        self.layers = []
        for _ in range(cfg.layers):
            wg, wu = w(self.inter, h), w(self.inter, h)
            self.layers.append({
                "qkv": w(self.qkv_out, h),
                "o": w(h, self.attn_out),
                "gu": interleave_gate_up(wg, wu),
                "d": w(h, self.inter),
                "ln1": (1 + 0.02 * torch.randn(h, generator=g, device=device)).bfloat16(),
                "ln2": (1 + 0.02 * torch.randn(h, generator=g, device=device)).bfloat16(),
            })

    def step(self, x: torch.Tensor, x_norm: torch.Tensor, n_layers: int | None = None) -> torch.Tensor:
        """One decode step; x (residual) is updated in place, returns the final normed state."""
        c = self.comm
        for L in self.layers[:n_layers]:
            qkv = gemm_bf16(x_norm, L["qkv"])
            part = gemm_bf16(qkv[:, : self.attn_out].contiguous(), L["o"])
            x_norm = all_reduce_add_rms_norm(c, part, x, L["ln1"], self.cfg.eps)
            hid = gemm_silu_mul(x_norm, L["gu"])
            part = gemm_bf16(hid, L["d"])
            x_norm = all_reduce_add_rms_norm(c, part, x, L["ln2"], self.cfg.eps)
        return x_norm

    def step_nccl(self, x: torch.Tensor, x_norm: torch.Tensor, group=None, n_layers: int | None = None) -> torch.Tensor:
        import torch.distributed as dist

        n = self.comm.nranks

        def ar_norm(part, weight):
            if n > 1:
                dist.all_reduce(part, group=group)
            x.add_(part)
            xf = x.float()
            return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.cfg.eps) * weight.float()).bfloat16()

        for L in self.layers[:n_layers]:
            qkv = x_norm @ L["qkv"].T
            part = qkv[:, : self.attn_out] @ L["o"].T
            x_norm = ar_norm(part, L["ln1"])
            gu = (x_norm @ L["gu"].T).view(-1, self.inter // 16, 2, 16)
            hid = (torch.nn.functional.silu(gu[:, :, 0]) * gu[:, :, 1]).reshape(-1, self.inter)
            part = hid @ L["d"].T
            x_norm = ar_norm(part, L["ln2"])
        return x_norm
