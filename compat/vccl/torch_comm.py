# SPDX-License-Identifier: Apache-2.0
"""`vccl.torch_comm.VcclCommunicator` for vLLM, resolved to vkccl_b200's
device communicator (reference: python/vccl/torch_comm.py), with the
reference module's other names: its base class, its torch-dtype table and
its dtype helper (reference: python/vccl/torch_comm.py:70-88)."""

from vkccl_b200.comm import DataType
from vkccl_b200.torch_comm import _TORCH_TO_VCCL as _TORCH_DTYPE  # noqa: F401
from vkccl_b200.torch_comm import DeviceCommunicatorBase, VcclCommunicator, vccl_dtype  # noqa: F401


def _vccl_dtype(t):
    """The DataType of a torch tensor (TypeError for unsupported dtypes)."""
    return DataType(vccl_dtype(t))


__all__ = ["VcclCommunicator"]
