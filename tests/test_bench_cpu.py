# SPDX-License-Identifier: Apache-2.0
"""bench.py's reference arm and JSON contract, on the CPU.

The reference arm runs the reference library (its own build under
baseline/_ref) through its own VcclCommunicator over gloo with torch CPU
GEMMs; here on a small token count.  Skipped when that build is absent.
"""

import json
import os
import subprocess
import sys

import pytest

from conftest import ROOT, free_port


def _reference_built():
    return os.path.exists(os.path.join(ROOT, "baseline", "_ref", "build", "libvccl.so"))


@pytest.mark.skipif(not _reference_built(), reason="reference build not present")
@pytest.mark.parametrize("nranks", [1, 2])
def test_reference_arm_prints_contract_line(nranks):
    cmd = [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--gpus", str(nranks),
           "--tokens", "64", "--steps", "2", "--warmup", "1"]
    if nranks > 1:
        cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nranks}",
               "--master-addr=127.0.0.1", f"--master-port={free_port()}"] + cmd[1:]
    env = dict(os.environ, VCCL_SOCKET_ADDR="127.0.0.1")
    p = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stderr[-3000:]
    lines = [json.loads(line) for line in p.stdout.splitlines() if line.startswith("{")]
    assert len(lines) == 1
    d = lines[0]
    assert d["impl"] == "reference" and d["n_gpus"] == nranks and d["steps"] == 2 and d["warmup"] == 1
    assert d["metric"] == "tp_mlp_layer_latency_us" and d["value"] > 0 and d["higher_is_better"] is False
    # host tensors in and out: the end-to-end number is the step itself, with no device copies
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["unit"] == "us"
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0


def test_roofline_helper():
    import importlib.util

    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    b = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(b)
    flops = 2.0 * 8192 * 4096 * 14336 * 3
    r = b.roofline(flops, 8192, 8, 500.0)
    assert r["bound"] == "compute" and 0 < r["fraction"] < 1
    # burst peak headline, sustained beside it (a larger fraction: the sustained peak is lower)
    assert r["fraction_sustained"] > r["fraction"]
    assert r["nvlink_us"] > 0
    assert b.roofline(flops, 8192, 1, 500.0)["nvlink_us"] == 0


def test_collectives_bench_host_mode():
    """`vkccl_b200.bench.collectives --host` (CPU tensors on the host data plane next to gloo) runs
    without a GPU and prints one JSON row per operation and size with both libraries' times."""
    env = dict(os.environ, VCCL_SOCKET_ADDR="127.0.0.1", GLOO_SOCKET_IFNAME="lo", VCCL_DEBUG="ERROR")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={free_port()}", "-m", "vkccl_b200.bench.collectives",
           "--host", "--ops", "allreduce,allgather,reducescatter,broadcast", "--dtypes", "f32,bf16", "-b", "4K",
           "-e", "64K", "-f", "16", "--iters", "3", "--warmup", "1"]
    p = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert p.returncode == 0, p.stdout[-2000:] + p.stderr[-4000:]
    rows = [json.loads(line) for line in p.stdout.splitlines() if line.startswith("{")]
    assert len(rows) == 4 * 2 * 2, rows
    for r in rows:
        assert r["vccl_us"] > 0 and ("gloo_us" in r or "gloo_error" in r), r
