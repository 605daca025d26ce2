# SPDX-License-Identifier: Apache-2.0
"""Multi-process collective correctness on GPUs (native suite).

Runs csrc/tests/test_collectives.cc: the reference's fork-based matrix
ported to one GPU per rank, plus device-buffer sweeps over every algorithm,
kill-a-rank (device timeout) and InitAll.  With one GPU only the
single-rank configuration runs.
"""

import os
import subprocess

import pytest

from conftest import BIN, gpu_count

pytestmark = pytest.mark.gpu


def test_collectives_suite():
    n = gpu_count()
    if n == 0:
        pytest.skip("no GPU")
    env = dict(os.environ, VCCL_SOCKET_ADDR="127.0.0.1", VCCL_DEBUG="ERROR")
    p = subprocess.run([os.path.join(BIN, "test_collectives"), str(min(n, 8))], env=env, capture_output=True,
                       text=True, timeout=1200)
    print(p.stdout)
    assert p.returncode == 0, p.stdout + p.stderr[-4000:]
    assert "all tests passed" in p.stdout


def test_devbuf_demo():
    n = gpu_count()
    if n < 2:
        pytest.skip("needs 2 GPUs")
    p = subprocess.run([os.path.join(BIN, "vccl-devbuf-demo"), "--launch", "2"], capture_output=True, text=True,
                       timeout=300, env=dict(os.environ, VCCL_SOCKET_ADDR="127.0.0.1"))
    assert p.returncode == 0, p.stdout + p.stderr
    assert p.stdout.count(": OK") == 2


@pytest.mark.parametrize("route", ["memfd", "udmabuf"])
def test_dmabuf_registration(route):
    """Forked ranks (one GPU each) register a mappable fd (a memfd, or a dmabuf minted through
    /dev/udmabuf; skipped where the kernel lacks it) and run an all-reduce and an all-gather inside the
    mapping (reference: tests/test_dmabuf.cc)."""
    n = min(gpu_count(), 2)
    if n == 0:
        pytest.skip("no GPU")
    env = dict(os.environ, VCCL_SOCKET_ADDR="127.0.0.1", VCCL_DEBUG="ERROR", VCCL_TIMEOUT="30")
    p = subprocess.run([os.path.join(BIN, "test_dmabuf"), str(n), route], env=env, capture_output=True, text=True,
                       timeout=300)
    if p.returncode == 77:
        pytest.skip(p.stdout.strip()[-200:])
    assert p.returncode == 0, p.stdout + p.stderr[-4000:]
    assert f"dmabuf ({route}, {n} ranks): OK" in p.stdout
