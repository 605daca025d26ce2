# SPDX-License-Identifier: Apache-2.0
"""GEMM + reduce-scatter with the TMA-store epilogue (VCCL_RS_TMA=1): the
fused worker's shapes at 256-wide tiles (the TMA path needs 64-column
passes) with the persistent fused kernels forced, against fp32 PyTorch."""

import os
import subprocess
import sys

import pytest

from conftest import ROOT, free_port, gpu_count

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("nranks", [2, 8])
def test_gemm_rs_tma_stores(nranks):
    if gpu_count() < nranks:
        pytest.skip(f"needs {nranks} GPUs")
    env = dict(os.environ, VCCL_COMM_ID=f"127.0.0.1:{free_port()}", VCCL_SOCKET_ADDR="127.0.0.1",
               VCCL_TIMEOUT="30", VCCL_RS_TMA="1", VCCL_GEMM_BN="256", VCCL_FUSED_SMALL_M="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nranks}",
           "--master-addr=127.0.0.1", f"--master-port={free_port()}",
           os.path.join(ROOT, "tests", "workers", "fused_worker.py")]
    p = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=900)
    assert p.returncode == 0, p.stdout[-3000:] + p.stderr[-6000:]
    assert p.stdout.count("fused ok") == nranks
