# SPDX-License-Identifier: Apache-2.0
"""Fused tensor-parallel kernels vs an unsharded fp32 PyTorch reference.

Runs tests/workers/fused_worker.py under torchrun with one rank per GPU
(all-reduce + residual + RMSNorm, GEMM + reduce-scatter, all-gather + GEMM
with and without SiLU*mul), three calls in a row per shape.
"""

import os
import subprocess
import sys

import pytest

from conftest import ROOT, free_port, gpu_count

pytestmark = pytest.mark.gpu


# small_m "0" forces the persistent fused kernels for every shape; the default
# runs shapes of up to 512 rows as collective + (split-K) GEMM.
@pytest.mark.parametrize("nranks,small_m", [(1, None), (2, None), (2, "0"), (4, None), (8, None), (8, "0")])
def test_fused_tp_ops(nranks, small_m):
    if gpu_count() < nranks:
        pytest.skip(f"needs {nranks} GPUs")
    port = free_port()
    env = dict(os.environ, VCCL_COMM_ID=f"127.0.0.1:{free_port()}", VCCL_SOCKET_ADDR="127.0.0.1",
               VCCL_TIMEOUT="30")
    if small_m is not None:
        env["VCCL_FUSED_SMALL_M"] = small_m
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nranks}",
           "--master-addr=127.0.0.1", f"--master-port={port}",
           os.path.join(ROOT, "tests", "workers", "fused_worker.py")]
    p = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=900)
    assert p.returncode == 0, p.stdout[-3000:] + p.stderr[-6000:]
    assert p.stdout.count("fused ok") == nranks


@pytest.mark.parametrize("nranks", [2, 4, 8])
def test_back_to_back_stress(nranks):
    """Unsynchronised streams of mixed collectives and graph replays."""
    if gpu_count() < nranks:
        pytest.skip(f"needs {nranks} GPUs")
    port = free_port()
    env = dict(os.environ, VCCL_COMM_ID=f"127.0.0.1:{free_port()}", VCCL_SOCKET_ADDR="127.0.0.1",
               VCCL_TIMEOUT="20")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nranks}",
           "--master-addr=127.0.0.1", f"--master-port={port}",
           os.path.join(ROOT, "tests", "workers", "stress_worker.py")]
    p = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=900)
    assert p.returncode == 0, p.stdout[-3000:] + p.stderr[-6000:]
    assert p.stdout.count("stress ok") == nranks
