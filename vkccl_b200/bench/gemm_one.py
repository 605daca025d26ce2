# SPDX-License-Identifier: Apache-2.0
"""Run one tcgen05 GEMM shape a few times (for timing or an ncu capture).

    python -m vkccl_b200.bench.gemm_one --m 8192 --n 3584 --k 4096 [--silu] [--iters 3]

Prints the best CUDA-event time of one launch next to torch.matmul (cuBLAS)
and the achieved TFLOP/s.  With --graph, `iters` launches are captured in
one CUDA graph and the replay time is divided by `iters` (kernel time
without host launch overhead, inputs L2-warm), for both libraries.
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
    ap.add_argument("--graph", action="store_true")
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

    def graphed(fn):
        fn()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(a.iters):
                fn()
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        e1.synchronize()
        return e0.elapsed_time(e1) * 1000 / a.iters

    t_ours = (graphed if a.graph else timed)(ours)
    t_cublas = (graphed if a.graph else timed)(lambda: a_ @ w.T)
    flops = 2.0 * a.m * a.n * a.k
    print(json.dumps({"m": a.m, "n": a.n, "k": a.k, "silu": a.silu, "graph": a.graph, "ours_us": round(t_ours, 2),
                      "cublas_us": round(t_cublas, 2), "ours_tflops": round(flops / t_ours / 1e6, 1),
                      "cublas_tflops": round(flops / t_cublas / 1e6, 1)}))


if __name__ == "__main__":
    main()
