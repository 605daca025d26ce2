# SPDX-License-Identifier: Apache-2.0
"""Event timeline of the GEMM + reduce-scatter kernels on every rank.

    VCCL_FUSED_TRACE=1 torchrun --nproc-per-node N --master-addr 127.0.0.1 \\
        -m vkccl_b200.bench.rs_trace [--tokens 8192] [--calls 8] [--interleave]

Runs --calls back-to-back gemm_reduce_scatter calls (Llama-3-8B down
projection shard: [T, 14336/N] x [14336/N, 4096]); with --interleave every
call follows the layer's all-gather + GEMM, as inside the MLP.  After the
last call each rank reads its per-CTA trace (fused/gemm_rs.cu, slots
20-27) and rank 0 prints, per rank: each call's device time, and the
median over CTAs of the wait for the previous call's slots, the time to push
every tile, one epilogue warp's push time per tile, the time to signal, and
for the reduction kernel, when every source's pushes had arrived and how long
the sum took (all in microseconds, relative to that rank's earliest GEMM
epilogue start; the GPUs' timers are not assumed to agree).
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

START, FREED, PUSH_NS, TILES, TILES_DONE, SIGNALLED, ARRIVED, REDUCED = range(20, 28)
REDUCE_BLOCKS = 64


def summarise(trace: np.ndarray) -> dict:
    t = trace.astype(np.float64)
    t0 = t[:, START].min()
    med = lambda col: round(float(np.median(col)), 2)  # noqa: E731
    tiles = np.maximum(t[:, TILES], 1)
    red = t[:REDUCE_BLOCKS]
    return {
        "freed_wait_us": med((t[:, FREED] - t[:, START]) / 1000),
        "tiles_us": med((t[:, TILES_DONE] - t[:, FREED]) / 1000),
        "push_per_tile_us": med(t[:, PUSH_NS] / tiles / 1000),
        "tiles_per_cta": med(t[:, TILES]),
        "signal_us": med((t[:, SIGNALLED] - t[:, TILES_DONE]) / 1000),
        "gemm_end_us": round(float((t[:, SIGNALLED].max() - t0) / 1000), 2),
        "reduce_arrived_us": med((red[:, ARRIVED] - t0) / 1000),
        "reduce_us": med((red[:, REDUCED] - red[:, ARRIVED]) / 1000),
    }


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
    h = torch.randn(a.tokens, mlp.inter_shard, device="cuda").bfloat16()
    for _ in range(3):
        all_gather_gemm(comm, x, mlp.w_gate_up, silu_mul=True, out=h)
        gemm_reduce_scatter(comm, h, mlp.w_down)
    torch.cuda.synchronize()
    dist.barrier()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(a.calls)]
    for e0, e1 in ev:
        if a.interleave:
            all_gather_gemm(comm, x, mlp.w_gate_up, silu_mul=True, out=h)
        e0.record()
        gemm_reduce_scatter(comm, h, mlp.w_down)
        e1.record()
    torch.cuda.synchronize()
    times = [round(e0.elapsed_time(e1) * 1000, 1) for e0, e1 in ev]
    trace = comm.fused_trace()
    summary = summarise(trace) if trace is not None else {}
    gathered = [None] * world
    dist.all_gather_object(gathered, {"rank": rank, "call_us": times, **summary})
    if rank == 0:
        for g in gathered:
            print(json.dumps(g), flush=True)
    comm.destroy()
    dist.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
