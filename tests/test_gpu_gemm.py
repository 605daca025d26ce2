# SPDX-License-Identifier: Apache-2.0
"""tcgen05 GEMM numerics vs a plain fp32 PyTorch reference."""

import pytest
import torch

from conftest import gpu_count

pytestmark = pytest.mark.gpu

SHAPES = [
    (128, 256, 64),
    (1, 3584, 4096),      # decode, gate/up shard
    (32, 4096, 1792),     # decode, down shard
    (300, 528, 200),      # ragged M and K
    (512, 3584, 4096),
    (2048, 4096, 1792),
]


def _ref(a, w):
    return (a.float() @ w.float().T)


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_gemm_bf16(m, n, k):
    if gpu_count() == 0:
        pytest.skip("no GPU")
    from vkccl_b200.ops.gemm import gemm_bf16

    g = torch.Generator(device="cuda").manual_seed(m * 7 + n + k)
    a = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    w = (torch.randn(n, k, device="cuda", generator=g) * 0.02).bfloat16()
    out = gemm_bf16(a, w)
    torch.cuda.synchronize()
    ref = _ref(a, w)
    err = (out.float() - ref).abs().max().item()
    scale = ref.abs().max().item() + 1e-6
    assert err <= 1e-2 * scale + 1e-3, f"max err {err} (scale {scale})"


@pytest.mark.parametrize("bn", [256, 128, 64, 32])
def test_gemm_all_tile_widths(bn, monkeypatch):
    if gpu_count() == 0:
        pytest.skip("no GPU")
    monkeypatch.setenv("VCCL_GEMM_BN", str(bn))
    from vkccl_b200.ops.gemm import gemm_bf16

    a = torch.randn(384, 1024, device="cuda").bfloat16()
    w = (torch.randn(768, 1024, device="cuda") * 0.02).bfloat16()
    out = gemm_bf16(a, w)
    ref = _ref(a, w)
    torch.cuda.synchronize()
    assert (out.float() - ref).abs().max().item() <= 1e-2 * ref.abs().max().item() + 1e-3


@pytest.mark.parametrize("m", [1, 32, 512])
def test_gemm_silu_mul(m):
    if gpu_count() == 0:
        pytest.skip("no GPU")
    from vkccl_b200.ops.gemm import gemm_silu_mul, interleave_gate_up

    k, inter = 4096, 1792
    a = torch.randn(m, k, device="cuda").bfloat16()
    wg = (torch.randn(inter, k, device="cuda") * 0.02).bfloat16()
    wu = (torch.randn(inter, k, device="cuda") * 0.02).bfloat16()
    out = gemm_silu_mul(a, interleave_gate_up(wg, wu))
    torch.cuda.synchronize()
    g = a.float() @ wg.float().T
    u = a.float() @ wu.float().T
    ref = torch.nn.functional.silu(g) * u
    err = (out.float() - ref).abs().max().item()
    assert err <= 2e-2 * ref.abs().max().item() + 1e-3, err


# Decode shapes (few output tiles) take the split-K path: fp32 partials per K
# split, summed by a second kernel.  Compared with the fp32 reference and
# with the same GEMM with split-K switched off.
@pytest.mark.parametrize("m,n,k", [(1, 8192, 8192), (64, 1024, 4096), (256, 1024, 8192), (17, 4096, 1792)])
def test_gemm_split_k(m, n, k, monkeypatch):
    if gpu_count() == 0:
        pytest.skip("no GPU")
    from vkccl_b200.ops.gemm import gemm_bf16

    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    a = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    w = (torch.randn(n, k, device="cuda", generator=g) * 0.02).bfloat16()
    out = gemm_bf16(a, w)
    monkeypatch.setenv("VCCL_GEMM_SPLITK", "0")
    plain = gemm_bf16(a, w)
    torch.cuda.synchronize()
    ref = _ref(a, w)
    scale = ref.abs().max().item() + 1e-6
    assert (out.float() - ref).abs().max().item() <= 1e-2 * scale + 1e-3
    assert (out.float() - plain.float()).abs().max().item() <= 1e-2 * scale + 1e-3


# The CTA-pair kernel (256 x 256 tiles over two SMs, tcgen05.mma.cta_group::2),
# forced with VCCL_GEMM_PAIR=2, against the fp32 reference and the one-SM
# kernel (VCCL_GEMM_PAIR=0); ragged M, N and K included, and shapes with too
# few pair tiles to fill the GPU, which split K on pairs.
PAIR_SHAPES = [(256, 256, 64), (512, 768, 1024), (1000, 1056, 776), (2048, 4096, 1792), (8192, 3584, 4096),
               # few pair tiles: split-K on pairs (2 and 4 splits), fp32 partials + reduction
               (512, 4096, 14336), (300, 2048, 8192)]


@pytest.mark.parametrize("m,n,k", PAIR_SHAPES)
@pytest.mark.parametrize("silu", [False, True])
def test_gemm_cta_pair(m, n, k, silu, monkeypatch):
    if gpu_count() == 0:
        pytest.skip("no GPU")
    from vkccl_b200.ops.gemm import gemm_bf16, gemm_silu_mul

    g = torch.Generator(device="cuda").manual_seed(m + 3 * n + 5 * k + silu)
    a = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    w = (torch.randn(n, k, device="cuda", generator=g) * 0.02).bfloat16()
    fn = gemm_silu_mul if silu else gemm_bf16
    outs = []
    for mode in ("2", "2", "0"):  # the pair kernel twice in a row, then the one-SM kernel
        monkeypatch.setenv("VCCL_GEMM_PAIR", mode)
        outs.append(fn(a, w))
    torch.cuda.synchronize()
    ref = _ref(a, w)
    if silu:  # W rows interleave gate and up in groups of 16
        r = ref.view(m, n // 32, 2, 16)
        ref = (torch.nn.functional.silu(r[:, :, 0]) * r[:, :, 1]).reshape(m, n // 2)
    scale = ref.abs().max().item() + 1e-6
    for out in outs:
        err = (out.float() - ref).abs().max().item()
        assert err <= 1e-2 * scale + 1e-3, f"max err {err} (scale {scale})"
    assert torch.equal(outs[0], outs[1])
