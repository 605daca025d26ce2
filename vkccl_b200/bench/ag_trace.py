# SPDX-License-Identifier: Apache-2.0
"""Event timeline of the all-gather + GEMM kernel on every rank.

    VCCL_FUSED_TRACE=1 torchrun --nproc-per-node N --master-addr 127.0.0.1 \
        -m vkccl_b200.bench.ag_trace [--tokens 8192] [--calls 8] [--interleave]

Runs --calls back-to-back all_gather_gemm calls (Llama-3-8B gate/up shard,
SiLU*mul epilogue); with --interleave every call is followed by the
layer's GEMM + reduce-scatter, as inside the MLP.  After the last call
every rank reads its per-CTA trace and rank 0 prints, per rank, the
median and maximum over CTAs of each event time relative to that rank's
earliest kernel start (the GPUs' timers are not assumed to agree), plus
each call's device time.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

import vkccl_b200 as v
from vkccl_b200.models.llama_mlp import MLPConfig, TPLlamaMLP
from vkccl_b200.ops.fused import all_gather_gemm, gemm_reduce_scatter

EVENTS = ["start", "prev shard taken", "own slice staged"] + [f"pulled shard +{s}" for s in range(1, 8)] + \
         [f"released shard +{s}" for s in range(8)] + ["end"]


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--calls", type=int, default=8)
    ap.add_argument("--interleave", action="store_true")
    a = ap.parse_args()
    if os.environ.get("VCCL_FUSED_TRACE", "0") == "0":
        raise SystemExit("set VCCL_FUSED_TRACE=1")
    rank, world, local = (int(os.environ.get(k, d)) for k, d in (("RANK", 0), ("WORLD_SIZE", 1), ("LOCAL_RANK", 0)))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    raw = torch.zeros(v.UNIQUE_ID_BYTES, dtype=torch.uint8, device="cuda")
    if rank == 0:
        raw.copy_(torch.frombuffer(bytearray(v.get_unique_id().to_bytes()), dtype=torch.uint8).cuda())
    dist.broadcast(raw, 0)
    comm = v.Communicator(world, v.UniqueId.from_bytes(bytes(raw.cpu().numpy())), rank, cuda_device=local)
    mlp = TPLlamaMLP(comm, MLPConfig(4096, 14336), seed=0)
    x = torch.randn(a.tokens // world, 4096, device="cuda").bfloat16()
    h = torch.empty((a.tokens, mlp.inter_shard), dtype=torch.bfloat16, device="cuda")
    for _ in range(3):
        all_gather_gemm(comm, x, mlp.w_gate_up, silu_mul=True, out=h)
        gemm_reduce_scatter(comm, h, mlp.w_down)
    torch.cuda.synchronize()
    dist.barrier()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(a.calls)]
    for e0, e1 in ev:
        e0.record()
        all_gather_gemm(comm, x, mlp.w_gate_up, silu_mul=True, out=h)
        e1.record()
        if a.interleave:
            gemm_reduce_scatter(comm, h, mlp.w_down)
    torch.cuda.synchronize()
    times = [round(e0.elapsed_time(e1) * 1000, 1) for e0, e1 in ev]
    trace = comm.fused_trace()
    summary = {}
    if trace is not None:
        t = trace.astype(np.float64)
        t0 = t[:, 0].min()
        for i, name in enumerate(EVENTS):
            col = t[:, i]
            valid = col >= t0
            if valid.any():
                rel = (col[valid] - t0) / 1000.0
                summary[name] = [round(float(np.median(rel)), 1), round(float(rel.max()), 1)]
    gathered = [None] * world
    dist.all_gather_object(gathered, {"rank": rank, "call_us": times, "events_us_median_max": summary})
    if rank == 0:
        for g in gathered:
            print(json.dumps(g), flush=True)
    comm.destroy()
    dist.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
