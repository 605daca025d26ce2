# SPDX-License-Identifier: Apache-2.0
"""Fused tensor-parallel collectives (stream-ordered on torch's current stream).

all_reduce_add_rms_norm(comm, partial, residual, weight, eps)
    residual += all_reduce(partial); returns RMSNorm(residual) * weight.
gemm_reduce_scatter(comm, a, w)
    row-parallel projection: reduce_scatter(a @ w^T) along rows, with the
    GEMM epilogue pushing tiles to their owner over NVLink.
all_gather_gemm(comm, x_shard, w, silu_mul=False)
    column-parallel projection of all_gather(x_shard) (optionally followed
    by silu(gate) * up), with the gather pulled by copy warps inside the
    GEMM kernel.
"""

from __future__ import annotations

import torch

from vkccl_b200._lib import lib
from vkccl_b200.comm import DataType, _check


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _shape(t: torch.Tensor, shape: tuple, name: str) -> None:
    """The kernels index by the shapes they are given: a tensor of another
    shape would be read or written past its end, so it is refused here."""
    if tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name} has shape {tuple(t.shape)}; expected {tuple(shape)}")


def _bf16(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda or t.dtype != torch.bfloat16 or not t.is_contiguous() or t.data_ptr() % 16:
        raise ValueError(f"{name} must be a contiguous, 16-byte aligned bf16 CUDA tensor")


def all_reduce_add_rms_norm(comm, partial: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                            eps: float = 1e-5, out: torch.Tensor | None = None) -> torch.Tensor:
    for t, nm in ((partial, "partial"), (residual, "residual"), (weight, "weight")):
        _bf16(t, nm)
    hidden = partial.shape[-1]
    rows = partial.numel() // hidden
    _shape(residual, partial.shape, "residual")
    _shape(weight, (hidden,), "weight")
    if out is None:
        out = torch.empty_like(partial)
    _bf16(out, "out")
    _shape(out, partial.shape, "out")
    _check(lib().vcclAllReduceAddRMSNorm(partial.data_ptr(), residual.data_ptr(), weight.data_ptr(),
                                         out.data_ptr(), rows, hidden, float(eps), int(DataType.BFLOAT16),
                                         comm._comm, _stream(partial)), "vcclAllReduceAddRMSNorm", comm._comm)
    return out


def gemm_reduce_scatter(comm, a: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    _bf16(a, "a")
    _bf16(w, "w")
    m, k = a.shape
    n = w.shape[0]
    _shape(w, (n, k), "w")
    if out is None:
        out = torch.empty((m // comm.nranks, n), dtype=torch.bfloat16, device=a.device)
    _bf16(out, "out")
    _shape(out, (m // comm.nranks, n), "out")
    _check(lib().vcclGemmReduceScatter(a.data_ptr(), w.data_ptr(), out.data_ptr(), m, n, k, comm._comm,
                                       _stream(a)), "vcclGemmReduceScatter", comm._comm)
    return out


def all_gather_gemm(comm, x_shard: torch.Tensor, w: torch.Tensor, silu_mul: bool = False,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    _bf16(x_shard, "x_shard")
    _bf16(w, "w")
    rows, k = x_shard.shape
    m = rows * comm.nranks
    n = w.shape[0]
    _shape(w, (n, k), "w")
    if out is None:
        out = torch.empty((m, n // 2 if silu_mul else n), dtype=torch.bfloat16, device=x_shard.device)
    _bf16(out, "out")
    _shape(out, (m, n // 2 if silu_mul else n), "out")
    _check(lib().vcclAllGatherGemm(x_shard.data_ptr(), w.data_ptr(), out.data_ptr(), m, n, k, 1 if silu_mul else 0,
                                   comm._comm, _stream(x_shard)), "vcclAllGatherGemm", comm._comm)
    return out
