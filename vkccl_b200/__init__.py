# SPDX-License-Identifier: Apache-2.0
"""vkccl_b200: collective communication for NVIDIA B200 (NVLink 5 / NVSwitch).

The core is ``libvccl.so`` (C API in ``include/vccl.h``); this package binds
it with ctypes and adds torch integration:

* ``vkccl_b200.comm``       – Communicator, UniqueId, DataType, RedOp, groups
* ``vkccl_b200.torch_comm`` – vLLM ``VcclCommunicator`` device communicator
* ``vkccl_b200.ops``        – fused tensor-parallel kernels (GEMM+RS, AG+GEMM,
                              AR+residual+RMSNorm, MoE fp8 dispatch/combine)
* ``vkccl_b200.models``     – Llama / Mixtral shaped layers built on them
* ``vkccl_b200.parallel``   – process-group and sharding helpers
* ``vkccl_b200.utils``      – device timing and clock sampling
"""

from vkccl_b200._lib import UNIQUE_ID_BYTES, UniqueId, library_path
from vkccl_b200.comm import (
    Communicator,
    DataType,
    RedOp,
    VcclError,
    buffer_info,
    get_unique_id,
    group,
    group_end,
    group_start,
    init_all,
    mem_alloc,
    mem_alloc_tensor,
    mem_free,
    type_size,
    version,
)

__all__ = [
    "Communicator",
    "DataType",
    "RedOp",
    "UNIQUE_ID_BYTES",
    "UniqueId",
    "VcclError",
    "buffer_info",
    "get_unique_id",
    "group",
    "group_end",
    "group_start",
    "init_all",
    "library_path",
    "mem_alloc",
    "mem_alloc_tensor",
    "mem_free",
    "type_size",
    "version",
]
