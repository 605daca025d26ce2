# SPDX-License-Identifier: Apache-2.0
"""Mixtral-8x7B-shaped expert-parallel dispatch / combine benchmark.

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m vkccl_b200.bench.moe [--tokens 4096]

Per rank: T tokens of hidden 4096 (bf16, seeded N(0,1)), top-2 routing from
seeded softmax logits with a per-expert bias (uneven counts), one expert per
GPU.  Times (CUDA events, after warm-up, max over ranks):

* vccl: vcclMoeDispatchFp8 (count exchange, fp8 e4m3 1x128 quantise while
  pushing over NVLink, dequantise on arrival) and vcclMoeCombine (weighted
  rows back to their sources, top-k sum).
* nccl: the usual torch.distributed path — sort pairs by destination,
  quantise to fp8 with the same block scales in PyTorch, exchange counts
  (host read of the split sizes), all_to_all_single of the fp8 rows and
  scales, dequantise; combine = all_to_all_single of the weighted bf16 rows
  back and an index_add top-k sum.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import torch
import torch.distributed as dist

import vkccl_b200 as v
from vkccl_b200.ops.moe import default_capacity, moe_combine, moe_dispatch


def routing(g, T, E, topk):
    bias = torch.linspace(0, 1, E, device="cuda")
    p = torch.softmax(torch.randn(T, E, device="cuda", generator=g) + bias, dim=-1)
    w, ids = torch.topk(p, topk, dim=-1)
    return ids.to(torch.int32), (w / w.sum(-1, keepdim=True)).float()


def quant(x):
    t, h = x.shape
    xf = x.float().view(t, h // 128, 128)
    amax = xf.abs().amax(-1, keepdim=True)
    s = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    return (xf / s).to(torch.float8_e4m3fn).view(t, h), s.view(t, h // 128)


def nccl_dispatch(x, ids, w, world, epr):
    T, H = x.shape
    topk = ids.shape[1]
    dest = (ids.long() // epr).view(-1)
    order = torch.argsort(dest, stable=True)
    tok = order // topk
    q, s = quant(x)
    send_q, send_s = q[tok], s[tok]
    send_meta = torch.stack([tok.int(), (order % topk).int(), ids.view(-1)[order]], dim=1)
    send_counts = torch.bincount(dest, minlength=world)
    recv_counts = torch.empty_like(send_counts)
    dist.all_to_all_single(recv_counts, send_counts)
    sc, rc = send_counts.tolist(), recv_counts.tolist()
    n = sum(rc)
    rq = torch.empty((n, H), dtype=torch.float8_e4m3fn, device=x.device)
    rs = torch.empty((n, H // 128), dtype=torch.float32, device=x.device)
    dist.all_to_all_single(rq.view(torch.uint8), send_q.view(torch.uint8), rc, sc)
    dist.all_to_all_single(rs, send_s, rc, sc)
    rx = (rq.float().view(n, H // 128, 128) * rs[..., None]).view(n, H).bfloat16()
    return rx, (order, sc, rc, w.view(-1)[order])


def nccl_combine(y, state, T, H, topk):
    order, sc, rc, wsorted = state
    back = torch.empty((sum(sc), H), dtype=torch.bfloat16, device=y.device)
    dist.all_to_all_single(back, y.contiguous(), sc, rc)
    out = torch.zeros((T, H), dtype=torch.float32, device=y.device)
    out.index_add_(0, order // topk, back.float() * wsorted[:, None])
    return out.bfloat16()


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=4096)
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--topk", type=int, default=2)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args()
    rank, world, local = (int(os.environ.get(k, d)) for k, d in (("RANK", 0), ("WORLD_SIZE", 1), ("LOCAL_RANK", 0)))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    raw = torch.zeros(v.UNIQUE_ID_BYTES, dtype=torch.uint8, device="cuda")
    if rank == 0:
        raw.copy_(torch.frombuffer(bytearray(v.get_unique_id().to_bytes()), dtype=torch.uint8).cuda())
    dist.broadcast(raw, 0)
    comm = v.Communicator(world, v.UniqueId.from_bytes(bytes(raw.cpu().numpy())), rank, cuda_device=local)
    T, H, topk, E = a.tokens, a.hidden, a.topk, world
    g = torch.Generator(device="cuda").manual_seed(77 + rank)
    x = torch.randn(T, H, device="cuda", generator=g).bfloat16()
    ids, w = routing(g, T, E, topk)
    cap = default_capacity(T, topk, world)

    def timed(fn):
        for _ in range(a.warmup):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        ts = []
        for _ in range(a.iters):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            dist.barrier()
            e0.record()
            fn()
            e1.record()
            e1.synchronize()
            ts.append(e0.elapsed_time(e1) * 1000)
        t = torch.tensor([sum(ts) / len(ts)], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    state = {}

    def vd():
        state["d"] = moe_dispatch(comm, x, w, ids, num_experts=E, capacity=cap)

    t_vd = timed(vd)
    d = state["d"]
    y = d.recv_x
    t_vc = timed(lambda: (vd(), moe_combine(comm, state["d"], y))) - t_vd
    nstate = {}

    def nd():
        nstate["r"] = nccl_dispatch(x, ids, w, world, E // world)

    t_nd = timed(nd)
    ry = nstate["r"][0]
    t_nc = timed(lambda: (nd(), nccl_combine(nstate["r"][0], nstate["r"][1], T, H, topk))) - t_nd
    del ry
    recv = d.count()
    rows = torch.tensor([recv], device="cuda")
    dist.all_reduce(rows, op=dist.ReduceOp.MAX)
    # Rooflines: the bytes each GPU must send over NVLink (pairs routed to other
    # ranks; fp8 row + scales + metadata on dispatch, bf16 row on combine) at
    # the measured 770 GB/s per direction.
    remote = (world - 1) / world * T * topk
    disp_us = remote * (H + H // 128 * 4 + 20) / 770e9 * 1e6
    comb_us = remote * H * 2 / 770e9 * 1e6
    if rank == 0:
        print(json.dumps({"bench": "moe_dispatch_combine", "n": world, "tokens_per_rank": T, "hidden": H,
                          "topk": topk, "experts": E, "capacity": cap, "max_rows_received": int(rows.item()),
                          "vccl_dispatch_us": round(t_vd, 1), "vccl_combine_us": round(t_vc, 1),
                          "nccl_dispatch_us": round(t_nd, 1), "nccl_combine_us": round(t_nc, 1),
                          "nvlink_roofline_us": {"dispatch": round(disp_us, 1), "combine": round(comb_us, 1)},
                          "roofline_fraction": {"dispatch": round(disp_us / t_vd, 3),
                                                "combine": round(comb_us / t_vc, 3)}}), flush=True)
    comm.destroy()
    dist.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
