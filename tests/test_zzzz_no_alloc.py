# SPDX-License-Identifier: Apache-2.0
"""vcclGemmBf16NoAlloc, called through its exported C symbol.

Two calls in a row on the same stream must each match vcclGemmBf16 on the
same inputs (and the fp32 reference), for decode shapes that take the
split-K path through the fixed scratch and for a shape that does not.  A
shape whose split-K partials exceed the fixed scratch is rejected.  A warm
call changes no device memory figure, and an abandoned launch (its abort
word set from the host, no device fault) makes the next call fail once.

Named test_zz_* so it is collected last; it must pass alone too.
"""

import ctypes

import pytest
import torch

from conftest import gpu_count

pytestmark = pytest.mark.gpu

INTERNAL_ERROR = 3
INVALID_ARGUMENT = 4


def _lib():
    from vkccl_b200._lib import lib

    h = lib()
    fn = h.vcclGemmBf16NoAlloc
    fn.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 3 + [ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return h


def _call(fn, a, w, c):
    m, k = a.shape
    n = w.shape[0]
    return fn(a.data_ptr(), w.data_ptr(), c.data_ptr(), m, n, k, torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("m,n,k", [(1, 8192, 8192), (32, 4096, 1792), (200, 1536, 8192), (512, 1024, 1024)])
def test_no_alloc_matches_gemm(m, n, k):
    if gpu_count() == 0:
        pytest.skip("no GPU")
    h = _lib()
    g = torch.Generator(device="cuda").manual_seed(7 * m + n + k)
    a = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    w = (torch.randn(n, k, device="cuda", generator=g) * 0.02).bfloat16()
    ref_lib = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    assert _call(h.vcclGemmBf16, a, w, ref_lib) == 0
    outs = []
    for _ in range(2):
        c = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
        assert _call(h.vcclGemmBf16NoAlloc, a, w, c) == 0
        outs.append(c)
    torch.cuda.synchronize()
    ref = a.float() @ w.float().T
    scale = ref.abs().max().item() + 1e-6
    for c in outs:
        assert torch.isfinite(c.float()).all()
        assert (c.float() - ref_lib.float()).abs().max().item() <= 1e-2 * scale + 1e-3
        assert (c.float() - ref).abs().max().item() <= 1e-2 * scale + 1e-3


def test_no_alloc_rejects_oversized_scratch():
    if gpu_count() == 0:
        pytest.skip("no GPU")
    h = _lib()
    # 2 row tiles x 20 column tiles, K split 11 ways -> 256 x 2560 x 11 fp32 = 28.8 MB > 8 MiB.
    m, n, k = 256, 2560, 32768
    a = torch.zeros(m, k, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(n, k, dtype=torch.bfloat16, device="cuda")
    c = torch.zeros(m, n, dtype=torch.bfloat16, device="cuda")
    assert _call(h.vcclGemmBf16NoAlloc, a, w, c) == INVALID_ARGUMENT


def test_no_alloc_allocates_nothing_when_warm():
    if gpu_count() == 0:
        pytest.skip("no GPU")
    h = _lib()
    m, n, k = 8, 4096, 8192  # split-K: partials in the fixed scratch
    a = torch.randn(m, k, device="cuda").bfloat16()
    w = (torch.randn(n, k, device="cuda") * 0.02).bfloat16()
    c = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    assert _call(h.vcclGemmBf16NoAlloc, a, w, c) == 0  # first call: set-up
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        assert _call(h.vcclGemmBf16NoAlloc, a, w, c) == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0


def test_no_alloc_reports_abandoned_launch_once():
    if gpu_count() == 0:
        pytest.skip("no GPU")
    h = _lib()
    m, n, k = 4, 2048, 4096
    a = torch.randn(m, k, device="cuda").bfloat16()
    w = (torch.randn(n, k, device="cuda") * 0.02).bfloat16()
    c = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    assert _call(h.vcclGemmBf16NoAlloc, a, w, c) == 0
    torch.cuda.synchronize()
    assert h.vcclxNoAllocInjectAbort(torch.cuda.current_device()) == 0
    assert _call(h.vcclGemmBf16NoAlloc, a, w, c) == INTERNAL_ERROR
    assert _call(h.vcclGemmBf16NoAlloc, a, w, c) == 0  # the word was cleared
    torch.cuda.synchronize()
    ref = a.float() @ w.float().T
    assert (c.float() - ref).abs().max().item() <= 1e-2 * (ref.abs().max().item() + 1e-6) + 1e-3
