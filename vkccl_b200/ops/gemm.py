# SPDX-License-Identifier: Apache-2.0
"""tcgen05 GEMM entry points (no library GEMM on these paths).

``gemm_bf16(a, w)``           a[M,K] @ w[N,K]^T -> [M,N] bf16
``gemm_silu_mul(a, w_gu)``    silu(a @ W_g^T) * (a @ W_u^T), w_gu from
                              ``interleave_gate_up(w_gate, w_up)``
"""

from __future__ import annotations

import torch

from vkccl_b200._lib import lib
from vkccl_b200.comm import _check


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _ok(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda or t.dtype != torch.bfloat16 or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous bf16 CUDA tensor")
    if t.data_ptr() % 16:
        raise ValueError(f"{name} must be 16-byte aligned")


def gemm_bf16(a: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    _ok(a, "a")
    _ok(w, "w")
    m, k = a.shape
    n = w.shape[0]
    if tuple(w.shape) != (n, k):
        raise ValueError(f"w has shape {tuple(w.shape)}; expected ({n}, {k})")
    if out is None:
        out = torch.empty((m, n), dtype=torch.bfloat16, device=a.device)
    _ok(out, "out")
    if tuple(out.shape) != (m, n):
        raise ValueError(f"out has shape {tuple(out.shape)}; expected ({m}, {n})")
    with torch.cuda.device(a.device):  # the library launches on the thread's current device
        _check(lib().vcclGemmBf16(a.data_ptr(), w.data_ptr(), out.data_ptr(), m, n, k, _stream(a)),
               "vcclGemmBf16")
    return out


def interleave_gate_up(w_gate: torch.Tensor, w_up: torch.Tensor) -> torch.Tensor:
    """[I,K] + [I,K] -> [2I,K] with gate/up rows interleaved in groups of 16."""
    i, k = w_gate.shape
    if i % 16:
        raise ValueError("intermediate size must be a multiple of 16")
    g = w_gate.reshape(i // 16, 16, k)
    u = w_up.reshape(i // 16, 16, k)
    return torch.stack([g, u], dim=1).reshape(2 * i, k).contiguous()


def gemm_silu_mul(a: torch.Tensor, w_gu: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    _ok(a, "a")
    _ok(w_gu, "w_gu")
    m, k = a.shape
    n = w_gu.shape[0]
    if tuple(w_gu.shape) != (n, k):
        raise ValueError(f"w_gu has shape {tuple(w_gu.shape)}; expected ({n}, {k})")
    if out is None:
        out = torch.empty((m, n // 2), dtype=torch.bfloat16, device=a.device)
    _ok(out, "out")
    if tuple(out.shape) != (m, n // 2):
        raise ValueError(f"out has shape {tuple(out.shape)}; expected ({m}, {n // 2})")
    with torch.cuda.device(a.device):
        _check(lib().vcclGemmSiluMul(a.data_ptr(), w_gu.data_ptr(), out.data_ptr(), m, n, k, _stream(a)),
               "vcclGemmSiluMul")
    return out
