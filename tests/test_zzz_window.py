# SPDX-License-Identifier: Apache-2.0
"""Zero-copy collectives on registered windows from Python: tensors on
vcclMemAlloc memory (mem_alloc_tensor), window_register, all-reduce /
all-gather / reduce-scatter in place on the peers' buffers."""

import os
import subprocess
import sys

import pytest

from conftest import ROOT, free_port, gpu_count

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("nranks", [1, 2, 4])
def test_window_collectives(nranks):
    if gpu_count() < nranks:
        pytest.skip(f"needs {nranks} GPUs")
    env = dict(os.environ, VCCL_SOCKET_ADDR="127.0.0.1", VCCL_TIMEOUT="30", GLOO_SOCKET_IFNAME="lo")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nranks}",
           "--master-addr=127.0.0.1", f"--master-port={free_port()}",
           os.path.join(ROOT, "tests", "workers", "window_worker.py")]
    p = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stdout[-3000:] + p.stderr[-6000:]
    assert p.stdout.count("window ok") == nranks
