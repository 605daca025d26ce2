# SPDX-License-Identifier: Apache-2.0
"""The native suite's extended mode (csrc/tests/test_collectives.cc,
`--extended`): the pipelined NVLS all-reduce, messages larger than the
staging region (multi-round two-shot / NVLS / pipelined NVLS) and the
zero-copy window collectives, a grouped Send/Recv whose ops sit on two
streams (the second stream must be ordered after the kernel), two all-reduces
on two streams where the second reads the first's output, with guard regions past every workspace that
each rank checks for out-of-bounds writes at the end, and vcclCommAbort from
another thread while a kernel waits for a rank that skipped the call.  Kept apart from the main matrix so that a
failure here cannot hide the main matrix's result under `pytest -x`."""

import os
import subprocess

import pytest

from conftest import BIN, gpu_count

pytestmark = pytest.mark.gpu


def test_collectives_extended():
    n = gpu_count()
    if n == 0:
        pytest.skip("no GPU")
    # VCCL_GUARDS: guard regions past every workspace, checked at the end of each rank
    env = dict(os.environ, VCCL_SOCKET_ADDR="127.0.0.1", VCCL_DEBUG="ERROR", VCCL_TIMEOUT="60", VCCL_GUARDS="1")
    p = subprocess.run([os.path.join(BIN, "test_collectives"), str(min(n, 8)), "--extended"], env=env,
                       capture_output=True, text=True, timeout=1200)
    print(p.stdout)
    assert p.returncode == 0, p.stdout + p.stderr[-4000:]
    assert "all tests passed" in p.stdout
