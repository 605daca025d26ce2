# SPDX-License-Identifier: Apache-2.0
"""`vccl.torch_comm.VcclCommunicator` for vLLM, resolved to vkccl_b200's
device communicator (reference: python/vccl/torch_comm.py)."""

from vkccl_b200.torch_comm import VcclCommunicator  # noqa: F401

__all__ = ["VcclCommunicator"]
