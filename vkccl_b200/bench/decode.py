# SPDX-License-Identifier: Apache-2.0
"""Llama-3-70B TP decode-step benchmark (80 layers, hidden 8192, bf16).

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m vkccl_b200.bench.decode --batch 1,16,128

For each batch size B one decode step (80 layers, each with two all-reduces
of [B, 8192] fused with residual add + RMSNorm, plus the layer's TP GEMMs;
see vkccl_b200.models.llama_decode) is captured in a CUDA graph, as vLLM
runs decode, and replayed.  Reported: mean step time over --iters replays
(CUDA events, after warm-up, max over ranks) for this library and for the
same layers on cuBLAS + NCCL all-reduce + torch RMSNorm, plus the relative
difference between the two paths' hidden states after one layer and after
all layers (random weights make 80 layers amplify rounding differences).
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import torch
import torch.distributed as dist

import vkccl_b200 as v
from vkccl_b200.models.llama_decode import DecodeConfig, TPLlamaDecode


def graph_time(fn, iters: int, warmup: int) -> float:
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(warmup):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        g.replay()
    e1.record()
    e1.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) * 1000 / iters], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    del g
    return t.item()


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", default="1,16,128")
    ap.add_argument("--layers", type=int, default=80)
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
    model = TPLlamaDecode(comm, DecodeConfig(layers=a.layers), seed=0)
    # HBM roofline: every step streams this rank's weights once.
    wbytes = sum(t.numel() * t.element_size() for L in model.layers for t in L.values())
    hbm_gbs = 6463.7
    try:
        with open(os.path.join(os.environ.get("GRAFT_REPO_ROOT", "."), "MEASURED_PEAKS.json")) as f:
            hbm_gbs = float(json.load(f)["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        pass
    roof_us = wbytes / (hbm_gbs * 1e9) * 1e6
    out = {"bench": "llama70b_tp_decode_step", "n": world, "layers": a.layers,
           "weight_bytes_per_gpu": wbytes, "hbm_roofline_us": round(roof_us, 1), "results": {}}
    for b in (int(s) for s in a.batch.split(",")):
        g = torch.Generator(device="cuda").manual_seed(11 + b)  # same on every rank
        x0 = torch.randn(b, 8192, device="cuda", generator=g).bfloat16()
        xn0 = torch.randn(b, 8192, device="cuda", generator=g).bfloat16()
        def rel(a_, b_):
            return ((a_.float() - b_.float()).norm() / (b_.float().norm() + 1e-12)).item()

        xa, xb = x0.clone(), x0.clone()
        err1 = rel(model.step(xa, xn0, n_layers=1), model.step_nccl(xb, xn0, n_layers=1))
        xa, xb = x0.clone(), x0.clone()
        ya = model.step(xa, xn0)
        yb = model.step_nccl(xb, xn0)
        torch.cuda.synchronize()
        err = rel(ya, yb)
        xv, xr = x0.clone(), x0.clone()
        t_v = graph_time(lambda: model.step(xv, xn0), a.iters, a.warmup)
        t_n = graph_time(lambda: model.step_nccl(xr, xn0), a.iters, a.warmup)
        out["results"][str(b)] = {"vccl_us": round(t_v, 1), "nccl_cublas_us": round(t_n, 1),
                                  "speedup": round(t_n / t_v, 3), "roofline_fraction": round(roof_us / t_v, 3),
                                  "rel_diff_one_layer": err1, "rel_diff_final_state": err}
        if rank == 0:
            print(json.dumps({"batch": b, **out["results"][str(b)]}), flush=True)
    if rank == 0:
        print(json.dumps(out), flush=True)
    comm.destroy()
    dist.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
