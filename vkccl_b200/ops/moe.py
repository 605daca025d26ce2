# SPDX-License-Identifier: Apache-2.0
"""Expert-parallel MoE dispatch / combine (stream-ordered on torch's current stream).

The reference offers only vcclAllToAll(v) for this (reference:
src/core/collectives.cc:708-740); routing, quantisation and the top-k sum
are fused into the transfers here.

moe_dispatch(comm, x, topk_weights, topk_ids, num_experts, capacity)
    Every (token, k) pair travels to the rank that owns expert topk_ids[t, k]
    (experts split evenly over ranks), quantised to fp8 e4m3 with one scale
    per 1x128 block on the way, and is dequantised to bf16 on arrival.
    Returns a MoeDispatch with the received rows (ordered by source rank,
    token, k), their routing weights, global expert ids and a device-side
    row count.
moe_combine(comm, dispatch, expert_out)
    The inverse: row i of expert_out (the expert's output for received row
    i) is scaled by its routing weight and travels back to its source,
    which sums the k rows of every token: out[t] = sum_k w[t,k] y(t,k).

The row count stays on the device; ``MoeDispatch.count()`` reads it (one
host synchronisation).  Buffers are sized by ``capacity`` (rows a rank may
receive, at least T * topk; the default is twice the average load); every
rank must pass the same capacity, hidden
size, topk and number of experts.  Call combine once per dispatch.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from vkccl_b200._lib import lib
from vkccl_b200.comm import _check


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


@dataclass
class MoeDispatch:
    recv_x: torch.Tensor       # [capacity, H] bf16; rows [0, count) are valid
    recv_meta: torch.Tensor    # [capacity, 4] int32: source rank, source token, k, local expert
    recv_w: torch.Tensor       # [capacity] f32 routing weights
    recv_count: torch.Tensor   # [1] int32 on the device
    tokens: int
    topk: int
    capacity: int
    num_experts: int
    rank: int
    experts_per_rank: int

    def count(self) -> int:
        return int(self.recv_count.item())

    def recv_ids(self) -> torch.Tensor:
        """Global expert id of every received row (capacity rows)."""
        return self.recv_meta[:, 3] + self.rank * self.experts_per_rank


def default_capacity(tokens: int, topk: int, nranks: int) -> int:
    """Room for twice the average load: with every rank routing T * topk
    pairs, a rank receives T * topk rows on average."""
    return max(2 * tokens * topk, 1) if nranks > 1 else max(tokens * topk, 1)


def moe_dispatch(comm, x: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor,
                 num_experts: Optional[int] = None, capacity: Optional[int] = None) -> MoeDispatch:
    if x.dtype != torch.bfloat16 or not x.is_cuda or x.dim() != 2 or not x.is_contiguous():
        raise ValueError("x must be a contiguous [T, H] bf16 CUDA tensor")
    t, h = x.shape
    if topk_ids.shape[0] != t or topk_weights.shape != topk_ids.shape:
        raise ValueError("topk_ids and topk_weights must be [T, topk]")
    topk = topk_ids.shape[1]
    n = comm.nranks
    num_experts = num_experts or n
    capacity = capacity or default_capacity(t, topk, n)
    ids = topk_ids.to(torch.int32).contiguous()
    w = topk_weights.to(torch.float32).contiguous()
    dev = x.device
    recv_x = torch.empty((capacity, h), dtype=torch.bfloat16, device=dev)
    recv_meta = torch.empty((capacity, 4), dtype=torch.int32, device=dev)
    recv_w = torch.empty((capacity,), dtype=torch.float32, device=dev)
    count = torch.zeros((1,), dtype=torch.int32, device=dev)
    _check(lib().vcclMoeDispatchFp8(x.data_ptr(), ids.data_ptr(), w.data_ptr(), recv_x.data_ptr(),
                                    recv_meta.data_ptr(), recv_w.data_ptr(), count.data_ptr(), t, h, topk,
                                    num_experts, capacity, comm._comm, _stream(x)),
           "vcclMoeDispatchFp8", comm._comm)
    return MoeDispatch(recv_x, recv_meta, recv_w, count, t, topk, capacity, num_experts, comm.rank,
                       num_experts // n)


def moe_combine(comm, d: MoeDispatch, expert_out: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    h = d.recv_x.shape[1]
    if (expert_out.dtype != torch.bfloat16 or not expert_out.is_cuda or not expert_out.is_contiguous()
            or expert_out.dim() != 2 or expert_out.shape[-1] != h):
        raise ValueError("expert_out must be a contiguous bf16 [rows, H] CUDA tensor in the received row order")
    if expert_out.shape[0] < d.capacity:
        # rows past the received count are never read, but the kernels index
        # up to the device-side count, so give them a capacity-sized buffer
        full = torch.empty((d.capacity, h), dtype=torch.bfloat16, device=expert_out.device)
        full[: expert_out.shape[0]].copy_(expert_out)
        expert_out = full
    if out is None:
        out = torch.empty((d.tokens, h), dtype=torch.bfloat16, device=expert_out.device)
    if out.dtype != torch.bfloat16 or not out.is_cuda or not out.is_contiguous() or tuple(out.shape) != (d.tokens, h):
        raise ValueError(f"out must be a contiguous bf16 CUDA tensor of shape {(d.tokens, h)}")
    _check(lib().vcclMoeCombine(expert_out.data_ptr(), d.recv_meta.data_ptr(), d.recv_w.data_ptr(),
                                d.recv_count.data_ptr(), out.data_ptr(), d.tokens, h, d.topk, d.capacity,
                                comm._comm, _stream(expert_out)),
           "vcclMoeCombine", comm._comm)
    return out


def quantize_dequantize_reference(x: torch.Tensor) -> torch.Tensor:
    """What a row looks like after dispatch: fp8 e4m3, one scale per 1x128 block.

    The kernels divide by the scale with IEEE division and round to the
    nearest e4m3 value with ties to even.  This reference runs on the CPU,
    whose division and fp8 cast do the same; torch's CUDA division is not
    correctly rounded, which moves exact ties (frequent here, since bf16
    inputs over amax / 448 often land on them) to the other neighbour.
    """
    t, h = x.shape
    xf = x.detach().cpu().float().view(t, h // 128, 128)
    amax = xf.abs().amax(dim=-1, keepdim=True)
    scale = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    q = (xf / scale).to(torch.float8_e4m3fn).float()
    return (q * scale).view(t, h).bfloat16().to(x.device)
