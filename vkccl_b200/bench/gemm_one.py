# SPDX-License-Identifier: Apache-2.0
"""Run one tcgen05 GEMM shape a few times (for timing or an ncu capture).

    python -m vkccl_b200.bench.gemm_one --m 8192 --n 3584 --k 4096 [--silu] [--iters 3]

Prints the CUDA-event time of the last launch next to torch.matmul (cuBLAS)
and the achieved TFLOP/s.
"""

from __future__ import annotations

import argparse
import json

import torch

from vkccl_b200.ops.gemm import gemm_bf16, gemm_silu_mul


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--m", type=int, default=8192)
    ap.add_argument("--n", type=int, default=3584)
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--silu", action="store_true")
    ap.add_argument("--iters", type=int, default=3)
    a = ap.parse_args()
    a_ = torch.randn(a.m, a.k, device="cuda").bfloat16()
    w = (torch.randn(a.n, a.k, device="cuda") * 0.02).bfloat16()

    def ours():
        return gemm_silu_mul(a_, w) if a.silu else gemm_bf16(a_, w)

    def timed(fn):
        fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        best = 1e9
        for _ in range(a.iters):
            e0.record()
            fn()
            e1.record()
            e1.synchronize()
            best = min(best, e0.elapsed_time(e1) * 1000)
        return best

    t_ours = timed(ours)
    t_cublas = timed(lambda: a_ @ w.T)
    flops = 2.0 * a.m * a.n * a.k
    print(json.dumps({"m": a.m, "n": a.n, "k": a.k, "silu": a.silu, "ours_us": round(t_ours, 2),
                      "cublas_us": round(t_cublas, 2), "ours_tflops": round(flops / t_ours / 1e6, 1),
                      "cublas_tflops": round(flops / t_cublas / 1e6, 1)}))


if __name__ == "__main__":
    main()
