# SPDX-License-Identifier: Apache-2.0
"""MoE dispatch (fp8 e4m3 1x128 quantised on the wire) and combine vs a
PyTorch reference, with uneven routing, 1 and 2 experts per rank, and a
capacity change that regrows the symmetric MoE region."""

import os
import subprocess
import sys

import pytest

from conftest import ROOT, free_port, gpu_count

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("nranks", [1, 2, 8])
def test_moe_dispatch_combine(nranks):
    if gpu_count() < nranks:
        pytest.skip(f"needs {nranks} GPUs")
    port = free_port()
    env = dict(os.environ, VCCL_COMM_ID=f"127.0.0.1:{free_port()}", VCCL_SOCKET_ADDR="127.0.0.1",
               VCCL_TIMEOUT="30")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nranks}",
           "--master-addr=127.0.0.1", f"--master-port={port}",
           os.path.join(ROOT, "tests", "workers", "moe_worker.py")]
    p = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stdout[-3000:] + p.stderr[-6000:]
    assert p.stdout.count("moe ok") == nranks
