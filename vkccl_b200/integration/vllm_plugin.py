# SPDX-License-Identifier: Apache-2.0
"""vLLM plugin: run vLLM's tensor/expert-parallel communication on vkccl_b200.

The reference ships a patch to a vLLM fork that makes its platform return
vccl's communicator class (reference: integration/vllm-vulkan-vccl.patch,
integration/README.md).  vLLM loads "general plugins" from the
``vllm.general_plugins`` entry-point group in every process it starts, so
no patch is needed here: installing this package registers ``register``
(see pyproject.toml), which points the CUDA platform's device communicator
at ``vkccl_b200.torch_comm.VcclCommunicator``.  Set ``VKCCL_VLLM=0`` to keep
vLLM's own communicator.
"""

from __future__ import annotations

import os

COMMUNICATOR = "vkccl_b200.torch_comm.VcclCommunicator"


def register() -> bool:
    """Install the communicator on vLLM's CUDA platform; False if skipped."""
    if os.environ.get("VKCCL_VLLM", "1") == "0":
        return False
    try:
        from vllm.platforms import cuda as vllm_cuda
    except Exception:  # noqa: BLE001 - vLLM absent or not importable here
        return False
    vllm_cuda.CudaPlatform.get_device_communicator_cls = classmethod(lambda cls: COMMUNICATOR)
    return True
