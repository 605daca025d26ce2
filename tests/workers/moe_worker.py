# SPDX-License-Identifier: Apache-2.0
"""Per-rank body of the MoE dispatch/combine test (run by torchrun).

Every rank builds the same seeded inputs for all ranks, so each can compute
exactly which rows it must receive (source rank, token, k order), what they
look like after fp8 e4m3 1x128 quantisation, and what combine must return
for its own tokens.
"""

import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))

import vkccl_b200 as v  # noqa: E402
from vkccl_b200.ops.moe import moe_combine, moe_dispatch, quantize_dequantize_reference  # noqa: E402


def routing(g, T, E, topk):
    # uneven expert popularity: biased logits, top-k of a softmax
    bias = torch.linspace(0, 2, E, device="cuda")
    logits = torch.randn(T, E, device="cuda", generator=g) + bias
    p = torch.softmax(logits, dim=-1)
    w, ids = torch.topk(p, topk, dim=-1)
    return ids.to(torch.int32), (w / w.sum(-1, keepdim=True)).float()


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    comm = v.Communicator(world, v.get_unique_id(), rank, cuda_device=rank)
    g = torch.Generator(device="cuda")
    H = 1024
    e1 = max(world, 2)  # at least topk experts
    cases = [(256, 2, e1, 2048), (200, 2, 2 * world, 2048), (300, 1, world, 2048), (256, 2, e1, 4096)]
    for it, (T, topk, E, cap) in enumerate(cases):
        epr = E // world
        xs, idss, ws = [], [], []
        for s in range(world):
            g.manual_seed(5000 + 100 * it + s)
            xs.append(torch.randn(T, H, device="cuda", generator=g).bfloat16())
            ids, w = routing(g, T, E, topk)
            idss.append(ids)
            ws.append(w)
        d = moe_dispatch(comm, xs[rank], ws[rank], idss[rank], num_experts=E, capacity=cap)
        torch.cuda.synchronize()
        assert comm.async_error() == 0, comm.last_error()
        # expected rows on this rank
        exp_rows, exp_meta, exp_w = [], [], []
        for s in range(world):
            qdq = quantize_dequantize_reference(xs[s])
            for t in range(T):
                for k in range(topk):
                    e = int(idss[s][t, k])
                    if e // epr == rank:
                        exp_rows.append(qdq[t])
                        exp_meta.append((s, t, k, e % epr))
                        exp_w.append(float(ws[s][t, k]))
        n = d.count()
        assert n == len(exp_rows), (n, len(exp_rows))
        meta = d.recv_meta[:n].cpu().tolist()
        assert [tuple(m) for m in meta] == exp_meta, "row order / metadata"
        assert torch.allclose(d.recv_w[:n].cpu(), torch.tensor(exp_w)), "weights"
        if n:
            ref = torch.stack(exp_rows).float()
            got = d.recv_x[:n].float()
            err = (got - ref).abs()
            # identical arithmetic; allow a rare one-step rounding difference
            bad = err > 1e-3 * ref.abs().amax()
            if bad.float().mean().item() >= 1e-3:
                i, j = [int(a) for a in (bad.nonzero()[0])]
                s_, t_, k_, _ = exp_meta[i]
                blk = xs[s_][t_].float()[(j // 128) * 128:(j // 128 + 1) * 128]
                raise AssertionError(f"case {it}: {bad.float().mean().item():.4f} of elements differ; first at row {i} "
                                     f"col {j}: x={float(xs[s_][t_, j])} got={float(got[i, j])} ref={float(ref[i, j])} "
                                     f"amax={float(blk.abs().max())} got_row0={got[i, :4].tolist()} "
                                     f"ref_row0={ref[i, :4].tolist()} x_row0={xs[s_][t_, :4].float().tolist()}")
            assert err.max().item() <= 0.07 * ref.abs().max().item()
        # expert: row * (1 + local expert id), in bf16
        y = (d.recv_x.float() * (1 + d.recv_meta[:, 3:4].clamp(min=0).float())).bfloat16()
        out = moe_combine(comm, d, y)
        torch.cuda.synchronize()
        assert comm.async_error() == 0, comm.last_error()
        qdq = quantize_dequantize_reference(xs[rank]).float()
        exp = torch.zeros(T, H, device="cuda")
        for k in range(topk):
            e = idss[rank][:, k].long()
            yk = (qdq * (1 + (e % epr)).float()[:, None]).bfloat16().float()
            exp += (yk * ws[rank][:, k:k + 1]).bfloat16().float()
        err = (out.float() - exp).abs().max().item()
        assert err <= 1e-2 * exp.abs().max().item() + 1e-2, f"combine err {err}"
    comm.destroy()
    print("moe ok", flush=True)


if __name__ == "__main__":
    main()
