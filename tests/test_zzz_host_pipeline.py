# SPDX-License-Identifier: Apache-2.0
"""Host-to-host MLP layer (pinned in, pinned out, token groups overlapping
their copies with the kernels) against the device forward on one GPU."""

import os

import pytest
import torch

from conftest import gpu_count

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("groups", [1, 2, 4])
def test_forward_host_matches_device_forward(groups):
    if gpu_count() == 0:
        pytest.skip("no GPU")
    os.environ.setdefault("VCCL_SOCKET_ADDR", "127.0.0.1")
    import vkccl_b200 as v
    from vkccl_b200.models.llama_mlp import MLPConfig, TPLlamaMLP

    torch.cuda.set_device(0)
    comm = v.Communicator(1, v.get_unique_id(), 0, cuda_device=0)
    try:
        mlp = TPLlamaMLP(comm, MLPConfig(hidden=1024, intermediate=2048), seed=3)
        g = torch.Generator(device="cuda").manual_seed(5)
        x = torch.randn(1000, 1024, device="cuda", generator=g).bfloat16()
        ref = mlp.forward_nccl(x).float().cpu()
        xh = x.cpu().pin_memory()
        yh = torch.full((1000, 1024), float("nan"), dtype=torch.bfloat16).pin_memory()
        for _ in range(2):  # the second call reuses the side streams and cached buffers
            mlp.forward_host(xh, yh, groups=groups)
        torch.cuda.synchronize()
        err = (yh.float() - ref).abs().max().item()
        scale = ref.abs().max().item() + 1e-6
        assert err <= 3e-2 * scale + 1e-2, f"groups={groups}: max err {err} (scale {scale})"
    finally:
        comm.destroy()
