# SPDX-License-Identifier: Apache-2.0
"""Llama-style tensor-parallel MLP layer on the fused kernels.

Sequence-parallel layout (Megatron SP): every rank holds x_shard = its
T/n rows of the [T, hidden] activations.  One layer is

    h       = silu(AllGather(x) @ W_gate^T) * (AllGather(x) @ W_up^T)   # [T, I/n]
    y_shard = ReduceScatter(h @ W_down^T)                               # [T/n, hidden]

and runs as two kernels of this library (plus a short local reduction):
``all_gather_gemm(..., silu_mul=True)`` (the gather is pulled by copy warps
inside the tcgen05 GEMM) and ``gemm_reduce_scatter`` (the GEMM epilogue
pushes tiles to their owners over NVLink).  ``forward_nccl`` is the
unfused NCCL + cuBLAS equivalent used as the comparison baseline.

The reference's only model is the toy TP MLP in its end-to-end test
(reference: python/tests/test_e2e_tp.py:60-92); this module is the
Llama-3-8B-shaped version of it on B200 kernels.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from vkccl_b200.ops.fused import all_gather_gemm, gemm_reduce_scatter
from vkccl_b200.ops.gemm import interleave_gate_up


@dataclass
class MLPConfig:
    hidden: int = 4096
    intermediate: int = 14336
    init_std: float = 0.02


class TPLlamaMLP:
    """One rank's shard of a Llama MLP layer (bf16, random init N(0, std))."""

    def __init__(self, comm, cfg: MLPConfig = MLPConfig(), seed: int = 0, device: str = "cuda"):
        self.comm = comm
        self.cfg = cfg
        n, r = comm.nranks, comm.rank
        if cfg.intermediate % (16 * n):
            raise ValueError("intermediate size must split into 16-row groups per rank")
        self.inter_shard = cfg.intermediate // n
        g = torch.Generator(device=device).manual_seed(seed * 1000 + r)
        std = cfg.init_std
        shape_gu = (self.inter_shard, cfg.hidden)
        self.w_gate = (torch.randn(shape_gu, generator=g, device=device) * std).bfloat16()
        self.w_up = (torch.randn(shape_gu, generator=g, device=device) * std).bfloat16()
        self.w_down = (torch.randn((cfg.hidden, self.inter_shard), generator=g, device=device) * std).bfloat16()
        self.w_gate_up = interleave_gate_up(self.w_gate, self.w_up)  # layout of the fused epilogue
        self._h = {}

    def forward(self, x_shard: torch.Tensor) -> torch.Tensor:
        """x_shard [T/n, hidden] -> y_shard [T/n, hidden] (stream-ordered)."""
        rows = x_shard.shape[0] * self.comm.nranks
        h = self._h.get(rows)
        if h is None:
            h = torch.empty((rows, self.inter_shard), dtype=torch.bfloat16, device=x_shard.device)
            self._h[rows] = h
        all_gather_gemm(self.comm, x_shard, self.w_gate_up, silu_mul=True, out=h)
        return gemm_reduce_scatter(self.comm, h, self.w_down)

    def forward_host(self, x_host: torch.Tensor, out_host: torch.Tensor | None = None,
                     groups: int = 1) -> torch.Tensor:
        """Host-to-host layer: pinned x_shard [T/n, hidden] in, y_shard out.

        The MLP treats tokens independently, so with groups > 1 the shard
        runs as that many token groups (the same split on every rank) and the
        PCIe copies of neighbouring groups overlap the layer's kernels
        (vkccl_b200.utils.host_pipeline).  Stream-ordered: synchronise the
        current stream before reading the result.
        """
        from vkccl_b200.utils.host_pipeline import run_rows

        if out_host is None:
            out_host = torch.empty((x_host.shape[0], self.cfg.hidden), dtype=torch.bfloat16,
                                   pin_memory=torch.cuda.is_available())
        return run_rows(self.forward, x_host, out_host, groups=groups, device=self.w_down.device)

    def forward_nccl(self, x_shard: torch.Tensor, group=None) -> torch.Tensor:
        """Same layer with torch.distributed (NCCL) collectives and cuBLAS GEMMs."""
        import torch.distributed as dist

        n = self.comm.nranks
        if n > 1:
            x = torch.empty((x_shard.shape[0] * n, x_shard.shape[1]), dtype=x_shard.dtype, device=x_shard.device)
            dist.all_gather_into_tensor(x, x_shard, group=group)
        else:
            x = x_shard
        h = torch.nn.functional.silu(x @ self.w_gate.T) * (x @ self.w_up.T)
        p = h @ self.w_down.T
        if n == 1:
            return p
        y = torch.empty((x_shard.shape[0], p.shape[1]), dtype=p.dtype, device=p.device)
        dist.reduce_scatter_tensor(y, p, group=group)
        return y

    def flops(self, tokens: int) -> float:
        """Multiply-add FLOPs of the whole layer (all ranks) for `tokens` rows."""
        c = self.cfg
        return 2.0 * tokens * c.hidden * c.intermediate * 3


def smoke_forward(comm) -> None:
    """Tiny forward through the fused path on cuda:0 (used by smoke())."""
    cfg = MLPConfig(hidden=512, intermediate=1024)
    mlp = TPLlamaMLP(comm, cfg, seed=1)
    x = torch.randn(64, cfg.hidden, device="cuda").bfloat16()
    y = mlp.forward(x)
    ref = mlp.forward_nccl(x)
    torch.cuda.synchronize()
    err = (y.float() - ref.float()).abs().max().item()
    scale = ref.float().abs().max().item() + 1e-6
    if not err <= 3e-2 * scale + 1e-2:
        raise AssertionError(f"smoke forward mismatch: {err} (scale {scale})")
