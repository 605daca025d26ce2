# SPDX-License-Identifier: Apache-2.0
"""Collective bandwidth sweep: vccl-b200 next to NCCL on the same GPUs.

Launch one process per GPU:

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m vkccl_b200.bench.collectives \
        --ops allreduce,allgather,reducescatter,broadcast --dtypes bf16,f32 -b 8 -e 1G

--host runs the host data plane (communicators without a device, CPU
tensors) next to torch.distributed's gloo backend, timed by the host clock;
it needs no GPU.

--window adds a "vcclwin" column: the same vccl call on buffers inside
registered windows (vcclMemAlloc memory mapped by every rank), which runs
the zero-copy kernels (all-reduce, all-gather, reduce-scatter, broadcast).  NCCL runs
on plain torch tensors in every column.

Every number is device time from CUDA events on the launching stream,
averaged over --iters launches captured in one CUDA graph (so host launch
overhead is excluded for both libraries), reported as the maximum over
ranks.  --eager times the same launches without a graph (what the
registration cache, VCCL_REG_CACHE=1, needs: captured calls stay staged).  busbw factors follow the reference bench (reference:
bench/vccl_bench.cc:147-152): 2(n-1)/n all-reduce, (n-1)/n all-gather and
reduce-scatter, 1 broadcast.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import torch
import torch.distributed as dist

from vkccl_b200 import comm as vc
from vkccl_b200.torch_comm import vccl_dtype

DT = {"bf16": torch.bfloat16, "f32": torch.float32, "f16": torch.float16}


def parse_size(s: str) -> int:
    mult = {"K": 1 << 10, "M": 1 << 20, "G": 1 << 30}
    if s[-1].upper() in mult:
        return int(float(s[:-1]) * mult[s[-1].upper()])
    return int(s)


def bus_factor(op: str, n: int) -> float:
    if op == "allreduce":
        return 2.0 * (n - 1) / n
    if op in ("allgather", "reducescatter"):
        return (n - 1) / n
    return 1.0


def make_call(lib: str, op: str, comm, send, recv, n):
    dt = vccl_dtype(send)
    if lib == "nccl":
        if op == "allreduce":
            return lambda: dist.all_reduce(recv)
        if op == "allgather":
            return lambda: dist.all_gather_into_tensor(recv, send)
        if op == "reducescatter":
            return lambda: dist.reduce_scatter_tensor(recv, send)
        return lambda: dist.broadcast(recv, 0)
    if op == "allreduce":
        return lambda: comm.all_reduce(send, recv, count=send.numel(), dtype=dt)
    if op == "allgather":
        return lambda: comm.all_gather(send, recv, sendcount=send.numel(), dtype=dt)
    if op == "reducescatter":
        return lambda: comm.reduce_scatter(send, recv, recvcount=recv.numel(), dtype=dt)
    return lambda: comm.broadcast(recv, 0, count=recv.numel(), dtype=dt)


def tuning_table(rows, world: int) -> str:
    """VCCL_TUNING_FILE rules from a sweep: for each all-reduce size, the
    fastest algorithm timed (vccl_<algo>_us columns); consecutive sizes with
    the same winner merge into one rule whose max_bytes is the largest size.
    The last rule has no size limit."""
    best = []
    for r in sorted((r for r in rows if r["op"] == "allreduce"), key=lambda r: r["bytes"]):
        algos = {k[len("vccl_"):-len("_us")]: v for k, v in r.items()
                 if k.startswith("vccl_") and k.endswith("_us") and k != "vccl_us"}
        if not algos:
            continue
        name = min(algos, key=algos.get)
        if best and best[-1][1] == name:
            best[-1] = (r["bytes"], name)
        else:
            best.append((r["bytes"], name))
    lines = ["# op ranks max_bytes algorithm  (measured by vkccl_b200.bench.collectives)"]
    for i, (size, name) in enumerate(best):
        lines.append(f"allreduce {world} {0 if i == len(best) - 1 else size} {name}")
    return "\n".join(lines) + "\n"


def time_graph(fn, iters: int, warmup: int) -> float:
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(warmup):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(iters):
            fn()
    g.replay()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    e1.synchronize()
    ms = e0.elapsed_time(e1) / iters
    del g
    return ms * 1000.0


def time_eager(fn, iters: int, warmup: int) -> float:
    """Mean device time per call of `iters` eager launches on the current
    stream (CUDA events around the loop, behind a short GPU lead so host
    launches stay ahead).  Used for paths that a graph capture would change:
    the registration cache (VCCL_REG_CACHE=1) keeps captured calls staged."""
    from vkccl_b200.utils.timing import gpu_lead

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    gpu_lead(5.0 + 0.2 * iters)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    e1.synchronize()
    return e0.elapsed_time(e1) / iters * 1000.0


def main_host(a) -> int:
    """--host: communicators without a device on CPU tensors (the host data plane), next to
    torch.distributed's gloo backend on the same tensors -- the CPU baseline the reference aims
    to beat.  Host clock over --iters calls, maximum over ranks."""
    import time

    os.environ["VCCL_NO_DEVICE"] = "1"
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    dist.init_process_group("gloo")
    raw = torch.zeros(vc.UNIQUE_ID_BYTES, dtype=torch.uint8)
    if rank == 0:
        raw.copy_(torch.frombuffer(bytearray(vc.get_unique_id().to_bytes()), dtype=torch.uint8))
    dist.broadcast(raw, 0)
    comm = vc.Communicator(world, vc.UniqueId.from_bytes(bytes(raw.numpy())), rank)
    lo, hi = parse_size(a.b), parse_size(a.e)
    rows = []
    for op in a.ops.split(","):
        for dname in a.dtypes.split(","):
            dt = DT[dname]
            es = torch.tensor([], dtype=dt).element_size()
            size = lo
            while size <= hi:
                count = max(1, size // es)
                if op in ("allgather", "reducescatter"):
                    count = max(1, count // world) * world
                if op == "allgather":
                    send, recv = torch.randn(count // world).to(dt), torch.empty(count, dtype=dt)
                elif op == "reducescatter":
                    send, recv = torch.randn(count).to(dt), torch.empty(count // world, dtype=dt)
                else:
                    send = torch.randn(count).to(dt)
                    recv = send.clone() if op == "broadcast" else torch.empty_like(send)
                row = {"op": op, "dtype": dname, "bytes": count * es, "n": world, "timing": "host clock"}
                for libname in ("vccl", "gloo"):
                    fn = make_call("nccl" if libname == "gloo" else "vccl", op, comm, send, recv, world)
                    try:
                        for _ in range(a.warmup):
                            fn()
                        dist.barrier()
                        t0 = time.perf_counter()
                        for _ in range(a.iters):
                            fn()
                        us = (time.perf_counter() - t0) / a.iters * 1e6
                    except RuntimeError as exc:  # an operation the backend lacks
                        row[libname + "_error"] = str(exc)[:80]
                        dist.barrier()
                        continue
                    t = torch.tensor([us], dtype=torch.float64)
                    dist.all_reduce(t, op=dist.ReduceOp.MAX)
                    us = t.item()
                    row[libname + "_us"] = round(us, 2)
                    row[libname + "_busbw"] = round(count * es / (us * 1e3) * bus_factor(op, world), 3)
                rows.append(row)
                if rank == 0:
                    print(json.dumps(row), flush=True)
                size = int(size * a.f)
    comm.destroy()
    if rank == 0 and a.out:
        with open(a.out, "w") as f:
            for r in rows:
                f.write(json.dumps(r) + "\n")
    dist.barrier()
    dist.destroy_process_group()
    return 0


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ops", default="allreduce,allgather,reducescatter,broadcast")
    ap.add_argument("--dtypes", default="bf16")
    ap.add_argument("-b", default="8")
    ap.add_argument("-e", default="256M")
    ap.add_argument("-f", type=float, default=4.0)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--libs", default="vccl,nccl")
    ap.add_argument("--algos", default="", help="also time these forced all-reduce algorithms")
    ap.add_argument("--out", default="")
    ap.add_argument("--tune-out", default="", help="write a VCCL_TUNING_FILE table from the --algos sweep")
    ap.add_argument("--window", action="store_true", help="also time vccl on registered-window buffers")
    ap.add_argument("--eager", action="store_true",
                    help="time eager launches instead of a CUDA graph (needed to see VCCL_REG_CACHE=1)")
    ap.add_argument("--host", action="store_true",
                    help="CPU tensors on communicators without a device, next to gloo (no GPU needed)")
    a = ap.parse_args()
    if a.host:
        return main_host(a)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    uid = vc.get_unique_id() if rank == 0 else None
    raw = torch.zeros(vc.UNIQUE_ID_BYTES, dtype=torch.uint8, device="cuda")
    if rank == 0:
        raw.copy_(torch.frombuffer(bytearray(uid.to_bytes()), dtype=torch.uint8))
    dist.broadcast(raw, 0)
    comm = vc.Communicator(world, vc.UniqueId.from_bytes(bytes(raw.cpu().numpy())), rank, cuda_device=local)
    rows = []
    lo, hi = parse_size(a.b), parse_size(a.e)
    wins = None
    if a.window:
        # two windows of the largest message, viewed as each size and dtype
        wbytes = (hi + 4096) // 16 * 16 + 16
        wsend, wrecv = vc.mem_alloc_tensor((wbytes,), torch.uint8), vc.mem_alloc_tensor((wbytes,), torch.uint8)
        wins = (wsend, wrecv, comm.window_register(wsend), comm.window_register(wrecv))
    for op in a.ops.split(","):
        for dname in a.dtypes.split(","):
            dt = DT[dname]
            es = torch.tensor([], dtype=dt).element_size()
            size = lo
            while size <= hi:
                count = max(1, size // es)
                if op in ("allgather", "reducescatter"):
                    per = max(1, count // world)
                    count = per * world
                if op == "allgather":
                    send = torch.randn(count // world, device="cuda").to(dt)
                    recv = torch.empty(count, device="cuda", dtype=dt)
                elif op == "reducescatter":
                    send = torch.randn(count, device="cuda").to(dt)
                    recv = torch.empty(count // world, device="cuda", dtype=dt)
                else:
                    send = torch.randn(count, device="cuda").to(dt)
                    recv = send.clone() if op == "broadcast" else torch.empty_like(send)
                row = {"op": op, "dtype": dname, "bytes": count * es, "n": world}
                variants = [(lib_, None) for lib_ in a.libs.split(",")]
                if wins is not None:
                    variants.append(("vcclwin", None))
                if op == "allreduce" and a.algos:
                    variants += [("vccl", algo) for algo in a.algos.split(",")]
                for libname, algo in variants:
                    if algo:
                        os.environ["VCCL_ALLREDUCE_ALGO"] = algo
                    if libname == "vcclwin":
                        ws = wins[0][: send.numel() * es].view(dt)
                        wr = wins[1][: recv.numel() * es].view(dt)
                        ws.copy_(send)
                        fn = make_call("vccl", op, comm, ws, wr, world)
                    else:
                        fn = make_call(libname, op, comm, send, recv, world)
                    us = (time_eager if a.eager else time_graph)(fn, a.iters, a.warmup)
                    os.environ.pop("VCCL_ALLREDUCE_ALGO", None)
                    if libname == "vccl" and comm.async_error() != 0:
                        raise RuntimeError(f"vccl async error during {op} {count * es} B: {comm.last_error()}")
                    t = torch.tensor([us], device="cuda")
                    dist.all_reduce(t, op=dist.ReduceOp.MAX)
                    us = t.item()
                    algbw = count * es / (us * 1e3)
                    key = libname + ("_" + algo if algo else "")
                    row[key + "_us"] = round(us, 2)
                    row[key + "_busbw"] = round(algbw * bus_factor(op, world), 2)
                rows.append(row)
                if rank == 0:
                    print(json.dumps(row), flush=True)
                size = int(size * a.f)
    if wins is not None:
        comm.window_deregister(wins[2])
        comm.window_deregister(wins[3])
        wins = None
    comm.destroy()
    if rank == 0 and a.tune_out:
        with open(a.tune_out, "w") as f:
            f.write(tuning_table(rows, world))
    if rank == 0 and a.out:
        with open(a.out, "w") as f:
            for r in rows:
                f.write(json.dumps(r) + "\n")
    dist.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
