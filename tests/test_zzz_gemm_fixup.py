# SPDX-License-Identifier: Apache-2.0
"""In-kernel split-K reduction (VCCL_GEMM_SPLIT_FIXUP=1): decode-shaped
GEMMs and GEMM + SiLU*mul must give the same bits as the separate reduction
kernel, call after call and under CUDA-graph replay."""

import os
import subprocess
import sys

import pytest
import torch

from conftest import ROOT, gpu_count

pytestmark = pytest.mark.gpu


def _run(tmp_path, fixup):
    out = str(tmp_path / f"gemm_{fixup}.pt")
    env = dict(os.environ, VCCL_GEMM_SPLIT_FIXUP=str(fixup))
    p = subprocess.run([sys.executable, os.path.join(ROOT, "tests", "workers", "gemm_fixup_worker.py"), out],
                       env=env, capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stdout[-3000:] + p.stderr[-4000:]
    return torch.load(out)


def test_split_fixup_matches_reduction_kernel(tmp_path):
    if gpu_count() == 0:
        pytest.skip("no GPU")
    plain = _run(tmp_path, 0)
    fused = _run(tmp_path, 1)
    assert plain.keys() == fused.keys()
    for key in plain:
        assert torch.equal(plain[key], fused[key]), key
