# SPDX-License-Identifier: Apache-2.0
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
NATIVE = os.path.join(ROOT, "vkccl_b200", "_native")
BIN = os.path.join(NATIVE, "bin")

os.environ.setdefault("VCCL_SOCKET_ADDR", "127.0.0.1")
os.environ.setdefault("GLOO_SOCKET_IFNAME", "lo")
os.environ.setdefault("MASTER_ADDR", "127.0.0.1")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200)")
    config.addinivalue_line("markers", "multigpu: needs two or more GPUs")


def _ensure_built():
    lib = os.path.join(NATIVE, "libvccl.so")
    if not os.path.exists(lib):
        subprocess.run(["make", "-j8"], cwd=ROOT, check=True)


_ensure_built()


def gpu_count() -> int:
    try:
        import torch

        return torch.cuda.device_count() if torch.cuda.is_available() else 0
    except Exception:  # noqa: BLE001
        return 0


@pytest.fixture
def ngpu() -> int:
    return gpu_count()


def free_port() -> int:
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]
