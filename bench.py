# SPDX-License-Identifier: Apache-2.0
"""Flagship benchmark: Llama-3-8B-shaped tensor-parallel MLP layer.

    python bench.py --gpus N --steps K --warmup W            # this library
    python bench.py --impl reference --gpus N --steps K ...   # the reference

For N > 1 launch with torchrun (one process per GPU, 127.0.0.1 rendezvous).

Step = one sequence-parallel MLP layer at TP = N over T = --tokens tokens:
all-gather of the [T/N, 4096] activation shards fused into the gate/up
tcgen05 GEMM (+ SiLU*mul), then the down GEMM fused with the reduce-scatter.
Inputs are synthetic N(0,1) bf16 activations and random N(0, 0.02) weights
of the Llama-3-8B MLP (hidden 4096, intermediate 14336).

Metric (lower is better): layer latency in microseconds = mean device time
of exactly K steps (CUDA events around each step, L2 flushed with a 256 MiB
write between steps), max over ranks.  Also reported: the same layer with
NCCL + cuBLAS, the latency at other token counts, all-reduce bus bandwidth,
the end-to-end latency through the public API including the pinned H2D
copy of the input shard and the D2H read of the output shard, SM clocks
sampled during the timed region, and the kernel launch count.

The reference arm runs the reference library unmodified (built from
source into baseline/_ref): its VcclCommunicator all-gather /
reduce-scatter over TCP with torch CPU GEMMs, the reference's own way of
running this layer (its e2e TP test).  Host wall-clock, fp32 (CPU).
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time
from datetime import timedelta

ROOT = os.path.dirname(os.path.abspath(__file__))
HIDDEN, INTER = 4096, 14336
METRIC = "tp_mlp_layer_latency_us"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["vccl", "reference"], default="vccl")
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--sweep", default="1,32,512,8192", help="token counts also reported")
    ap.add_argument("--no-extras", action="store_true")
    return ap.parse_args()


def env_ranks():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def config(args, n, dtype, l2="flushed (256 MiB write) between timed steps"):
    return {
        "model": "Llama-3-8B MLP layer (hidden 4096, intermediate 14336), sequence-parallel tensor parallel",
        "global_batch": 1,
        "seq_len": args.tokens,
        "tokens_per_step": args.tokens,
        "parallelism": f"tp{n}",
        "dtype": dtype,
        "l2": l2,
    }


# ---------------------------------------------------------------------------
def run_vccl(args) -> int:
    import torch
    import torch.distributed as dist

    sys.path.insert(0, ROOT)
    os.environ.setdefault("VCCL_SOCKET_ADDR", "127.0.0.1")
    # host-side call counts per kernel path (no device work): which forms ran
    os.environ.setdefault("VCCL_PROF", "1")
    import vkccl_b200 as v
    from vkccl_b200.models.llama_mlp import MLPConfig, TPLlamaMLP
    from vkccl_b200.utils.timing import (ClockSampler, L2Flusher, NvmlClockSampler, bind_to_gpu_cpus,
                                         max_over_ranks, time_steps)

    rank, world, local = env_ranks()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    torch.cuda.set_device(local)
    # Host buffers on the GPU's NUMA node: the end-to-end copies then stay on one socket.
    numa_bound = bind_to_gpu_cpus(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=timedelta(seconds=300))
        raw = torch.zeros(v.UNIQUE_ID_BYTES, dtype=torch.uint8, device="cuda")
        if rank == 0:
            raw.copy_(torch.frombuffer(bytearray(v.get_unique_id().to_bytes()), dtype=torch.uint8).cuda())
        dist.broadcast(raw, 0)
        uid = v.UniqueId.from_bytes(bytes(raw.cpu().numpy()))
    else:
        uid = v.get_unique_id()
    comm = v.Communicator(world, uid, rank, cuda_device=local)
    mlp = TPLlamaMLP(comm, MLPConfig(HIDDEN, INTER), seed=0)
    flush = L2Flusher()
    gen = torch.Generator(device="cuda").manual_seed(1234 + rank)

    def shard(tokens):
        return torch.randn(tokens // world, HIDDEN, device="cuda", generator=gen).bfloat16()

    def measure(fn, steps, warmup, align_ranks=False):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        times = time_steps(fn, steps, flush, align_ranks)
        return max_over_ranks(sum(times) / len(times))

    # numerics: fused path vs NCCL + cuBLAS on the headline shape
    x = shard(args.tokens)
    y = mlp.forward(x)
    yr = mlp.forward_nccl(x)
    torch.cuda.synchronize()
    rel_err = ((y.float() - yr.float()).norm() / (yr.float().norm() + 1e-12)).item()
    rel_err = max_over_ranks(rel_err)

    # headline: exactly K timed steps, clocks sampled during them
    sampler = NvmlClockSampler(local)
    if not sampler.ok:
        sampler = ClockSampler(50)
    for _ in range(args.warmup):
        mlp.forward(x)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    if rank == 0:
        sampler.start()
    times = time_steps(lambda: mlp.forward(x), args.steps, flush)
    clocks = sampler.stop() if rank == 0 else {}
    value = max_over_ranks(sum(times) / len(times))
    # spread of the K timed steps (each statistic max over ranks): a single
    # slow step shows up here rather than only in the mean
    srt = sorted(times)
    step_stats = {"min": round(max_over_ranks(srt[0]), 2), "median": round(max_over_ranks(srt[len(srt) // 2]), 2),
                  "max": round(max_over_ranks(srt[-1]), 2)}
    if world > 1:
        # every rank's own mean: a slow rank stands out here
        mine = torch.tensor([sum(times) / len(times)], dtype=torch.float64, device="cuda")
        every = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(every, mine)
        step_stats["by_rank_mean"] = [round(float(t.item()), 2) for t in every]
    # Kernels of this library per step: the all-gather + GEMM kernel and the
    # GEMM + reduce-scatter kernel (one kernel on CTA pairs; the two-kernel
    # form adds its sum kernel); at one rank, the two GEMMs.  The L2 flush
    # between steps is torch's fill kernel, not counted.
    two_kernel_rs = os.environ.get("VCCL_RS_TWO_KERNELS", "0") != "0" or os.environ.get("VCCL_RS_TMA", "0") != "0"
    per_step_launches = 3 if world > 1 and two_kernel_rs else 2

    # end to end through the public API: pinned H2D input, forward, D2H output
    # (TPLlamaMLP.forward_host), the shard in 1 to 8 token groups whose copies
    # overlap the neighbouring groups' kernels; the fastest split is reported
    # with all the others.
    xh = x.cpu().pin_memory()
    yh = torch.empty(y.shape, dtype=y.dtype, pin_memory=True)
    e2e_by_groups, e2e_notes = {}, {}
    for g in (1, 2, 4, 8):
        if g == 1 or x.shape[0] >= 64 * g:
            try:
                e2e_by_groups[g] = measure(lambda g=g: mlp.forward_host(xh, yh, groups=g), args.steps, args.warmup)
            except Exception as exc:  # same shapes on every rank, so every rank takes this branch alike
                if g == 1:
                    raise
                e2e_notes[str(g)] = f"{type(exc).__name__}: {exc}"[:200]
    e2e_groups = min(e2e_by_groups, key=e2e_by_groups.get)
    e2e = e2e_by_groups[e2e_groups]
    mlp.forward_host(xh, yh, groups=e2e_groups)
    torch.cuda.synchronize()
    e2e_err = max_over_ranks(((yh.float() - y.cpu().float()).norm() / (y.cpu().float().norm() + 1e-12)).item())
    nccl_us = measure(lambda: mlp.forward_nccl(x), args.steps, args.warmup)

    extras = {}
    if not args.no_extras:
        sweep = {}
        for t in [int(s) for s in args.sweep.split(",") if s]:
            if t % world or t == args.tokens:
                continue
            xs = shard(t)
            sweep[str(t)] = {"vccl_us": round(measure(lambda: mlp.forward(xs), args.steps, args.warmup), 2),
                             "nccl_cublas_us": round(measure(lambda: mlp.forward_nccl(xs), args.steps, args.warmup), 2)}
        sweep[str(args.tokens)] = {"vccl_us": round(value, 2), "nccl_cublas_us": round(nccl_us, 2)}
        extras["latency_by_tokens"] = sweep
        extras["breakdown_us"] = breakdown(mlp, x, world, measure)
        if world > 1:
            extras["allreduce_busbw_GBps"] = allreduce_busbw(comm, world, measure, flush)
    flops = mlp.flops(args.tokens)
    try:
        paths = comm.prof_summary()
    except Exception:  # noqa: BLE001 - a diagnostic never fails the run
        paths = []
    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "us",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(value / 1000.0, 4),
            "steps_us": step_stats,
            "higher_is_better": False,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic N(0,1) activations, random N(0,0.02) weights",
            "config": {**config(args, world, "bf16"),
                       "host_cpus": "GPU-local NUMA cores (NVML affinity)" if numa_bound else "unrestricted"},
            "clocks": clocks,
            "e2e": {"value": round(e2e, 2), "unit": "us",
                    "h2d_bytes_per_step": x.numel() * x.element_size(),
                    "d2h_bytes_per_step": y.numel() * y.element_size(),
                    "api": "TPLlamaMLP.forward_host (pinned host in, pinned host out)",
                    "token_groups": e2e_groups,
                    "by_token_groups_us": {str(k): round(t, 2) for k, t in e2e_by_groups.items()},
                    **({"token_group_errors": e2e_notes} if e2e_notes else {}),
                    "rel_err_vs_device_forward": e2e_err},
            "gpu_launches": per_step_launches * args.steps,
            "nccl_cublas_us": round(nccl_us, 2),
            "speedup_vs_nccl_cublas": round(nccl_us / value, 3),
            "achieved_tflops": round(flops / (value * 1e-6) / 1e12, 1),
            "roofline": roofline(flops, args.tokens, world, value),
            "rel_err_vs_nccl_cublas": rel_err,
            # rank 0's calls per (operation, kernel path) over the whole run
            "paths": {f"{e['op']} / {e['algo']}": e["calls"] for e in paths},
            **extras,
        }
        print(json.dumps(line), flush=True)
    comm.destroy()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


NVLINK_GBS = 770.0  # measured peer copy, GB/s per direction per GPU


def measured_peaks():
    """bf16 burst and sustained TFLOP/s and HBM GB/s measured on this pool,
    or the stated fallback."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return {"burst": float(d["bf16_tflops"]), "sustained": float(d["bf16_tflops_sustained"]),
                "hbm": float(d["hbm_gbs"]), "src": "measured"}
    except (OSError, KeyError, ValueError):
        return {"burst": 1590.0, "sustained": 1400.0, "hbm": 6650.0, "src": "fallback"}


def roofline(flops, tokens, world, measured_us):
    """The layer's roofline on one GPU: the slower of its GEMM FLOPs at the
    bf16 peak and the bytes that must cross NVLink (all-gather in,
    reduce-scatter out: (n-1)/n of the [T, 4096] bf16 activations each way)
    at the measured per-direction link bandwidth.

    The headline fraction divides by the BURST GEMM peak: the timed region
    is K steps of a few milliseconds with an L2 flush between them, far
    shorter than the seconds-long loop the sustained figure comes from.  The
    fraction against the sustained (power-capped) peak is reported beside it.
    """
    pk = measured_peaks()
    link_bytes = (world - 1) / world * tokens * HIDDEN * 2 if world > 1 else 0.0
    link_us = link_bytes / (NVLINK_GBS * 1e9) * 1e6
    out = {"nvlink_us": round(link_us, 1), "peaks": pk["src"]}
    for name in ("burst", "sustained"):
        compute_us = flops / world / (pk[name] * 1e12) * 1e6
        bound = max(compute_us, link_us)
        if name == "burst":
            out.update(compute_us=round(compute_us, 1), bound="compute" if compute_us >= link_us else "nvlink",
                       fraction=round(bound / measured_us, 3))
        else:
            out.update(compute_us_sustained=round(compute_us, 1), fraction_sustained=round(bound / measured_us, 3))
    out["rule"] = "fraction: burst bf16 peak (short timed region); fraction_sustained: power-capped peak"
    return out


def breakdown(mlp, x, world, measure):
    """Each fused kernel alone, next to the same GEMM with no communication.

    Every step starts with the ranks aligned (device sync + barrier outside
    the timed region), as inside the layer where each fused kernel follows
    one that synchronised the ranks.
    """
    import torch

    from vkccl_b200.ops.fused import all_gather_gemm, gemm_reduce_scatter
    from vkccl_b200.ops.gemm import gemm_bf16, gemm_silu_mul

    rows = x.shape[0] * world
    xfull = torch.randn(rows, x.shape[1], device="cuda").bfloat16()
    h = torch.empty((rows, mlp.inter_shard), dtype=torch.bfloat16, device="cuda")
    out = {
        "ag_gemm_silu": measure(lambda: all_gather_gemm(mlp.comm, x, mlp.w_gate_up, silu_mul=True, out=h), 10, 3,
                                True),
        "gemm_silu_local": measure(lambda: gemm_silu_mul(xfull, mlp.w_gate_up, out=h), 10, 3, True),
        "gemm_rs": measure(lambda: gemm_reduce_scatter(mlp.comm, h, mlp.w_down), 10, 3, True),
        "gemm_local": measure(lambda: gemm_bf16(h, mlp.w_down), 10, 3, True),
        # the whole layer with the ranks aligned before every step: set against
        # the headline (steps back to back), it shows how much rank skew costs
        "layer_aligned": measure(lambda: mlp.forward(x), 10, 3, True),
    }
    return {k: round(v, 2) for k, v in out.items()}


def allreduce_busbw(comm, world, measure, flush):
    import torch
    import torch.distributed as dist

    from vkccl_b200.utils.timing import max_over_ranks

    out = {}
    for size in (1 << 20, 16 << 20, 256 << 20):
        a = torch.randn(size // 2, device="cuda").bfloat16()
        b = torch.empty_like(a)
        f = 2.0 * (world - 1) / world
        # the result this library gives against NCCL's on the same inputs
        # (before the timing loops, which reduce in place many times)
        comm.all_reduce(a, b)
        r = a.clone()
        dist.all_reduce(r)
        torch.cuda.synchronize()
        rel = max_over_ranks(((b.float() - r.float()).norm() / (r.float().norm() + 1e-12)).item())
        del r
        tv = measure(lambda: comm.all_reduce(a, b), 10, 3)
        if os.environ.get("VKCCL_BENCH_STEPS"):
            from vkccl_b200.utils.timing import time_steps

            steps = time_steps(lambda: comm.all_reduce(a, b), 10, flush)
            print(json.dumps({"rank": dist.get_rank(), "size": size, "steps_us": [round(t, 1) for t in steps]}),
                  file=sys.stderr, flush=True)
        tn = measure(lambda: dist.all_reduce(a), 10, 3)
        out[f"{size >> 20}MiB"] = {"vccl": round(size / (tv * 1e3) * f, 1), "nccl": round(size / (tn * 1e3) * f, 1),
                                   "rel_err_vs_nccl": round(rel, 5)}
    return out


# ---------------------------------------------------------------------------
def run_reference(args) -> int:
    ref = os.path.join(ROOT, "baseline", "_ref")
    lib = os.path.join(ref, "build", "libvccl.so")
    rank, world, _ = env_ranks()
    if not os.path.exists(lib) or not os.path.isdir(os.path.join(ref, "vccl")):
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "baseline/_ref not built (the reference's own "
                              "CMake build and its unmodified python package are expected there)"}))
        return 0
    os.environ["VCCL_LIBRARY"] = lib
    os.environ.setdefault("VCCL_SOCKET_ADDR", "127.0.0.1")
    os.environ.setdefault("GLOO_SOCKET_IFNAME", "lo")
    sys.path.insert(0, ref)
    import torch
    import torch.distributed as dist

    torch.set_num_threads(max(1, (os.cpu_count() or 8) // max(1, world)))
    if world > 1:
        dist.init_process_group("gloo", timeout=timedelta(seconds=600))
    else:
        import socket

        with socket.socket() as s:
            s.bind(("127.0.0.1", 0))
            port = s.getsockname()[1]
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1)
    from vccl.torch_comm import VcclCommunicator  # the reference's own communicator

    comm = VcclCommunicator(dist.group.WORLD)
    g = torch.Generator().manual_seed(rank)
    inter = INTER // world
    wg = torch.randn(inter, HIDDEN, generator=g) * 0.02
    wu = torch.randn(inter, HIDDEN, generator=g) * 0.02
    wd = torch.randn(HIDDEN, inter, generator=g) * 0.02
    x_shard = torch.randn(args.tokens // world, HIDDEN, generator=g)

    def step():
        x = comm.all_gather(x_shard, dim=0)
        h = torch.nn.functional.silu(x @ wg.T) * (x @ wu.T)
        return comm.reduce_scatter(h @ wd.T, dim=0)

    for _ in range(args.warmup):
        step()
    dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    us = (time.perf_counter() - t0) / args.steps * 1e6
    t = torch.tensor([us], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    us = t.item()
    if rank == 0:
        print(json.dumps({
            "impl": "reference",
            "metric": METRIC,
            "value": round(us, 1),
            "unit": "us",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(us / 1000.0, 3),
            "higher_is_better": False,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "fp32",
            "data": "synthetic N(0,1) activations, random N(0,0.02) weights",
            "config": config(args, world, "fp32 (reference host path: torch CPU GEMMs + vccl TCP collectives)",
                             l2="not applicable (host path)"),
            "timing": "host wall clock, mean of K steps, max over ranks (the reference has no device path)",
            # The reference's public path takes host tensors and returns host
            # tensors, so its end-to-end number is the same host-to-host step
            # time, with no device copies at all.
            "e2e": {"value": round(us, 1), "unit": "us", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0,
                    "api": "vccl.torch_comm.VcclCommunicator all_gather / reduce_scatter + torch CPU GEMMs "
                           "(host tensors in, host tensors out)"},
            "gpu_launches": 0,
        }), flush=True)
    comm.destroy()
    dist.destroy_process_group()
    return 0


def main() -> int:
    args = parse()
    if args.tokens % args.gpus:
        raise SystemExit("--tokens must be divisible by --gpus")
    return run_reference(args) if args.impl == "reference" else run_vccl(args)


if __name__ == "__main__":
    sys.exit(main())
