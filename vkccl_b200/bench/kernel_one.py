# SPDX-License-Identifier: Apache-2.0
"""Run one single-GPU kernel of the library a few times (for timing or an ncu capture).

    python -m vkccl_b200.bench.kernel_one moe --tokens 4096 --hidden 4096 [--iters 3]
    python -m vkccl_b200.bench.kernel_one rmsnorm --rows 128 --hidden 8192

moe:      MoE dispatch on a one-rank communicator (fp8 e4m3 1x128 quantise +
          dequantise of every (token, k) row: moeLocalDispatch), then combine.
rmsnorm:  residual add + RMSNorm on a one-rank communicator (addRmsNormLocal).

Prints the CUDA-event time of the fastest iteration and the achieved HBM
bandwidth of the algorithmic bytes.
"""

from __future__ import annotations

import argparse
import json

import torch

import vkccl_b200 as v


def timed(fn, iters):
    fn()
    torch.cuda.synchronize()
    best = 1e30
    for _ in range(iters):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        e1.synchronize()
        best = min(best, e0.elapsed_time(e1) * 1000)
    return best


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("kernel", choices=["moe", "rmsnorm"])
    ap.add_argument("--tokens", type=int, default=4096)
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--rows", type=int, default=128)
    ap.add_argument("--topk", type=int, default=2)
    ap.add_argument("--iters", type=int, default=3)
    a = ap.parse_args()
    torch.cuda.set_device(0)
    comm = v.Communicator(1, v.get_unique_id(), 0, cuda_device=0)
    g = torch.Generator(device="cuda").manual_seed(0)
    if a.kernel == "moe":
        from vkccl_b200.ops.moe import moe_combine, moe_dispatch

        x = torch.randn(a.tokens, a.hidden, device="cuda", generator=g).bfloat16()
        ids = torch.randint(0, 8, (a.tokens, a.topk), device="cuda", generator=g, dtype=torch.int32)
        w = torch.rand(a.tokens, a.topk, device="cuda", generator=g)
        state = {}

        def disp():
            state["d"] = moe_dispatch(comm, x, w, ids, num_experts=8)

        t = timed(disp, a.iters)
        d = state["d"]
        comb = timed(lambda: moe_combine(comm, d, d.recv_x), a.iters)
        rows = a.tokens * a.topk
        nbytes = a.tokens * a.hidden * 2 + rows * a.hidden * 2  # read x, write recv rows
        print(json.dumps({"kernel": "moe dispatch (1 rank)", "us": round(t, 2),
                          "GBps": round(nbytes / t / 1e3, 1), "combine_us": round(comb, 2)}))
    else:
        from vkccl_b200.ops.fused import all_reduce_add_rms_norm

        p = torch.randn(a.rows, a.hidden, device="cuda", generator=g).bfloat16()
        r = torch.randn(a.rows, a.hidden, device="cuda", generator=g).bfloat16()
        wt = torch.ones(a.hidden, device="cuda").bfloat16()
        t = timed(lambda: all_reduce_add_rms_norm(comm, p, r, wt, 1e-5), a.iters)
        nbytes = a.rows * a.hidden * 2 * 4  # read partial + residual, write residual + out
        print(json.dumps({"kernel": "add+rmsnorm (1 rank)", "us": round(t, 2), "GBps": round(nbytes / t / 1e3, 1)}))
    comm.destroy()


if __name__ == "__main__":
    main()
