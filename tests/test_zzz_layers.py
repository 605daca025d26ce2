# SPDX-License-Identifier: Apache-2.0
"""Sequence-parallel linear layers (vkccl_b200.parallel) on one GPU against
plain fp32 PyTorch: ColumnParallelLinear with and without the SiLU*mul
pairing, RowParallelLinear, at a short (split-K) and a long input."""

import os

import pytest
import torch

from conftest import gpu_count

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("tokens", [8, 640])
def test_parallel_linear_layers(tokens):
    if gpu_count() == 0:
        pytest.skip("no GPU")
    os.environ.setdefault("VCCL_SOCKET_ADDR", "127.0.0.1")
    import vkccl_b200 as v
    from vkccl_b200.parallel import ColumnParallelLinear, RowParallelLinear

    torch.cuda.set_device(0)
    comm = v.Communicator(1, v.get_unique_id(), 0, cuda_device=0)
    try:
        g = torch.Generator(device="cuda").manual_seed(tokens)
        x = torch.randn(tokens, 512, device="cuda", generator=g).bfloat16()
        wg = (torch.randn(256, 512, device="cuda", generator=g) * 0.05).bfloat16()
        wu = (torch.randn(256, 512, device="cuda", generator=g) * 0.05).bfloat16()
        wd = (torch.randn(512, 256, device="cuda", generator=g) * 0.05).bfloat16()

        def close(got, ref, what):
            err = (got.float() - ref).abs().max().item()
            assert err <= 2e-2 * ref.abs().max().item() + 1e-3, f"{what}: err {err}"

        y = ColumnParallelLinear(comm, wg)(x)
        close(y, x.float() @ wg.float().T, "column")
        h = ColumnParallelLinear(comm, wg, up_weight=wu)(x)
        ref_h = torch.nn.functional.silu(x.float() @ wg.float().T) * (x.float() @ wu.float().T)
        close(h, ref_h, "column silu*mul")
        z = RowParallelLinear(comm, wd)(h)
        close(z, h.float() @ wd.float().T, "row")
        torch.cuda.synchronize()
    finally:
        comm.destroy()
