# SPDX-License-Identifier: Apache-2.0
"""Registration cache from Python (VCCL_REG_CACHE=1): collectives on plain
PyTorch tensors run on windows the library registers on first use and
reuses afterwards (the NVLink form of the reference's per-call
registration cache, reference: src/core/comm.h:74-139)."""

import os
import subprocess
import sys

import pytest

from conftest import ROOT, free_port, gpu_count

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("nranks", [2, 4])
def test_registration_cache(nranks):
    if gpu_count() < nranks:
        pytest.skip(f"needs {nranks} GPUs")
    # VCCL_NVLS_MIN_RANKS above the rank count: all-reduce consults the cache only where the
    # staged NVLS kernel would not run
    env = dict(os.environ, VCCL_SOCKET_ADDR="127.0.0.1", VCCL_TIMEOUT="30", GLOO_SOCKET_IFNAME="lo",
               VCCL_REG_CACHE="1", VCCL_REG_CACHE_MIN=str(1 << 20), VCCL_NVLS_MIN_RANKS="8")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nranks}",
           "--master-addr=127.0.0.1", f"--master-port={free_port()}",
           os.path.join(ROOT, "tests", "workers", "reg_cache_worker.py")]
    p = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stdout[-3000:] + p.stderr[-6000:]
    assert p.stdout.count("reg cache ok") == nranks
