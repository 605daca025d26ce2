# SPDX-License-Identifier: Apache-2.0
"""Per-rank body of the fused tensor-parallel numerics test (run by torchrun).

Every rank builds the same seeded tensors, so each can compute the full
unsharded fp32 reference and check its own result.
"""

import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))

import vkccl_b200 as v  # noqa: E402
from vkccl_b200.ops.fused import all_gather_gemm, all_reduce_add_rms_norm, gemm_reduce_scatter  # noqa: E402
from vkccl_b200.ops.gemm import interleave_gate_up  # noqa: E402


def close(got, ref, rel, what):
    err = (got.float() - ref).abs().max().item()
    scale = ref.abs().max().item() + 1e-6
    if err > rel * scale + 1e-2:
        raise AssertionError(f"{what}: max err {err:.4g} vs scale {scale:.4g}")


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    comm = v.Communicator(world, v.get_unique_id(), rank, cuda_device=rank)
    g = torch.Generator(device="cuda")

    # --- all-reduce + residual + RMSNorm -------------------------------------
    H = 8192
    for rows in (1, 16, 128, 100):
        for rep in range(3):
            g.manual_seed(1000 + rows * 10 + rep)
            partials = [torch.randn(rows, H, device="cuda", generator=g).bfloat16() for _ in range(world)]
            residual = torch.randn(rows, H, device="cuda", generator=g).bfloat16()
            weight = (1 + 0.1 * torch.randn(H, device="cuda", generator=g)).bfloat16()
            x = residual.float() + sum(p.float() for p in partials)
            ref = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-5) * weight.float()
            res = residual.clone()
            out = all_reduce_add_rms_norm(comm, partials[rank], res, weight, 1e-5)
            torch.cuda.synchronize()
            close(res, x, 2e-2, f"residual rows={rows}")
            close(out, ref, 3e-2, f"rmsnorm rows={rows}")

    # --- GEMM + reduce-scatter -------------------------------------------------
    for (m, n_, k) in ((256 * world, 1024, 512), (128 * world, 4096, 1792), (8 * world, 512, 256)):
        for rep in range(3):
            g.manual_seed(2000 + m + rep)
            As = [torch.randn(m, k, device="cuda", generator=g).bfloat16() for _ in range(world)]
            Ws = [(torch.randn(n_, k, device="cuda", generator=g) * 0.05).bfloat16() for _ in range(world)]
            ref = sum(a.float() @ w.float().T for a, w in zip(As, Ws))
            per = m // world
            out = gemm_reduce_scatter(comm, As[rank], Ws[rank])
            torch.cuda.synchronize()
            close(out, ref[rank * per:(rank + 1) * per], 2e-2, f"gemm+rs m={m}")

    # --- all-gather + GEMM (plain and SiLU*mul) -------------------------------
    for (m, n_, k) in ((256 * world, 1024, 512), (64 * world, 3584, 4096), (4 * world, 512, 256)):
        for rep in range(3):
            g.manual_seed(3000 + m + rep)
            shards = [torch.randn(m // world, k, device="cuda", generator=g).bfloat16() for _ in range(world)]
            w = (torch.randn(n_, k, device="cuda", generator=g) * 0.05).bfloat16()
            xfull = torch.cat(shards).float()
            out = all_gather_gemm(comm, shards[rank], w)
            torch.cuda.synchronize()
            close(out, xfull @ w.float().T, 2e-2, f"ag+gemm m={m}")
            wg, wu = w[: n_ // 2], w[n_ // 2:]
            gu = interleave_gate_up(wg.contiguous(), wu.contiguous())
            out2 = all_gather_gemm(comm, shards[rank], gu, silu_mul=True)
            torch.cuda.synchronize()
            ref2 = torch.nn.functional.silu(xfull @ wg.float().T) * (xfull @ wu.float().T)
            close(out2, ref2, 3e-2, f"ag+gemm silu m={m}")

    # --- the bench's TP shard shapes (Llama-3-8B MLP, 8192 tokens, shards as at TP-8) -----
    # all-gather + gate/up GEMM: [8192 / n, 4096] shards x [3584, 4096] (SiLU*mul)
    # GEMM + reduce-scatter: [8192, 1792] x [4096, 1792] -> [8192 / n, 4096]
    T, HID, SH = 8192, 4096, 1792
    for rep in range(2):
        g.manual_seed(4000 + rep)
        shards = [torch.randn(T // world, HID, device="cuda", generator=g).bfloat16() for _ in range(world)]
        wg = (torch.randn(SH, HID, device="cuda", generator=g) * 0.02).bfloat16()
        wu = (torch.randn(SH, HID, device="cuda", generator=g) * 0.02).bfloat16()
        out = all_gather_gemm(comm, shards[rank], interleave_gate_up(wg, wu), silu_mul=True)
        torch.cuda.synchronize()
        xfull = torch.cat(shards).float()
        ref = torch.nn.functional.silu(xfull @ wg.float().T) * (xfull @ wu.float().T)
        close(out, ref, 3e-2, "ag+gemm silu at the bench shard shape")
        del xfull, ref, out
        As = [torch.randn(T, SH, device="cuda", generator=g).bfloat16() for _ in range(world)]
        Ws = [(torch.randn(HID, SH, device="cuda", generator=g) * 0.02).bfloat16() for _ in range(world)]
        per = T // world
        out = gemm_reduce_scatter(comm, As[rank], Ws[rank])
        torch.cuda.synchronize()
        ref = sum(a[rank * per:(rank + 1) * per].float() @ w.float().T for a, w in zip(As, Ws))
        close(out, ref, 2e-2, "gemm+rs at the bench shard shape")
        del As, Ws, out, ref

    # --- GEMM + reduce-scatter of changing shapes in a row (the CTA-pair path keeps
    # per-tile arrival counts across calls whose tiles differ), against fp32
    for m in (8192, 1024, 8192, 2048, 4096, 8192):
        if m % world or (m // world) % 128:
            continue
        g.manual_seed(5000 + m)
        As = [torch.randn(m, 512, device="cuda", generator=g).bfloat16() for _ in range(world)]
        Ws = [(torch.randn(4096, 512, device="cuda", generator=g) * 0.05).bfloat16() for _ in range(world)]
        per = m // world
        out = gemm_reduce_scatter(comm, As[rank], Ws[rank])
        torch.cuda.synchronize()
        ref = sum(a[rank * per:(rank + 1) * per].float() @ w.float().T for a, w in zip(As, Ws))
        close(out, ref, 2e-2, f"gemm+rs shape sequence m={m}")

    # --- shards of half a pair tile (128 rows per rank) with 56 column tiles: the shape whose
    # one-kernel tile walk could wait in a cycle at 8 ranks; it must take the two-kernel form
    m, n_w = 128 * world, 14336
    g.manual_seed(6000)
    As = [torch.randn(m, 512, device="cuda", generator=g).bfloat16() for _ in range(world)]
    Ws = [(torch.randn(n_w, 512, device="cuda", generator=g) * 0.05).bfloat16() for _ in range(world)]
    per = m // world
    out = gemm_reduce_scatter(comm, As[rank], Ws[rank])
    torch.cuda.synchronize()
    ref = sum(a[rank * per:(rank + 1) * per].float() @ w.float().T for a, w in zip(As, Ws))
    close(out, ref, 2e-2, f"gemm+rs half pair tiles m={m} n={n_w}")

    err = comm.async_error()
    comm.destroy()
    if err != 0:
        raise AssertionError(f"async error {err}")
    print(f"rank {rank}: fused ok", flush=True)


if __name__ == "__main__":
    main()
