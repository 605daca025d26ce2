# SPDX-License-Identifier: Apache-2.0
"""Native control-plane suites (CPU; no GPU needed).

test_bootstrap: the reference's stray-client rendezvous test.
test_control:   lifecycle / split / ops / abort / host failure detection.
"""

import os
import subprocess

from conftest import BIN


def _run(name, timeout=300):
    env = dict(os.environ, VCCL_SOCKET_ADDR="127.0.0.1", VCCL_DEBUG="ERROR")
    p = subprocess.run([os.path.join(BIN, name)], env=env, capture_output=True, text=True, timeout=timeout)
    assert p.returncode == 0, p.stdout + p.stderr
    return p.stdout


def test_bootstrap_rejects_stray_client():
    assert "bootstrap-reject: OK" in _run("test_bootstrap")


def test_control_plane_suite():
    assert "control-plane: OK" in _run("test_control")
