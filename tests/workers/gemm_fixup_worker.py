# SPDX-License-Identifier: Apache-2.0
"""Decode-shaped GEMMs (split-K plans) written to a file, for comparing the
in-kernel split-K reduction (VCCL_GEMM_SPLIT_FIXUP=1) with the separate
reduction kernel: eager calls, repeated calls and CUDA-graph replays."""

import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))

from vkccl_b200.ops.gemm import gemm_bf16, gemm_silu_mul  # noqa: E402

SHAPES = [(1, 3584, 4096), (4, 4096, 1792), (8, 5120, 8192), (1, 28672, 8192), (3, 1024, 14336)]


def main(out_path):
    torch.cuda.set_device(0)
    results = {}
    for m, n, k in SHAPES:
        g = torch.Generator(device="cuda").manual_seed(m * 131 + n + k)
        a = torch.randn(m, k, device="cuda", generator=g).bfloat16()
        w = (torch.randn(n, k, device="cuda", generator=g) * 0.02).bfloat16()
        outs = [gemm_bf16(a, w) for _ in range(3)]  # repeated calls reuse the semaphores
        h = gemm_silu_mul(a, w)
        y = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=s):
                y.copy_(gemm_bf16(a, w))
        torch.cuda.current_stream().wait_stream(s)
        for _ in range(2):
            graph.replay()
        torch.cuda.synchronize()
        ref = a.float() @ w.float().T
        for o in outs + [y]:
            err = (o.float() - ref).abs().max().item()
            assert err <= 1e-2 * ref.abs().max().item() + 1e-3, f"{(m, n, k)}: err {err}"
            assert torch.equal(o, outs[0]), f"{(m, n, k)}: repeated call or graph replay differs"
        results[f"{m}x{n}x{k}"] = outs[0].cpu()
        results[f"{m}x{n}x{k}_silu"] = h.cpu()
        del graph
    torch.save(results, out_path)
    print("gemm fixup worker ok", flush=True)


if __name__ == "__main__":
    main(sys.argv[1])
