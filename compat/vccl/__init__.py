# SPDX-License-Identifier: Apache-2.0
"""Drop-in `vccl` package name for code written against the reference's
Python bindings (reference: python/vccl/__init__.py).

Put this directory on PYTHONPATH (``PYTHONPATH=<repo>/compat``) and
``import vccl`` resolves to vkccl_b200: the same Communicator / UniqueId /
DataType / RedOp / VcclError / get_unique_id / group_start / group_end
names, backed by the NVLink library.  Buffers may be CUDA tensors (the
fast path, stream-ordered on torch's current stream) or host buffers
(numpy, CPU tensors, bytearrays), which are staged through the device; a
communicator without a device (VCCL_NO_DEVICE=1, or no GPU) moves host
buffers over TCP between the ranks, as the reference does.
"""

from vkccl_b200 import (  # noqa: F401
    UNIQUE_ID_BYTES,
    Communicator,
    DataType,
    RedOp,
    UniqueId,
    VcclError,
    get_unique_id,
    group,
    group_end,
    group_start,
    init_all,
    mem_alloc,
    mem_free,
    type_size,
    version,
)

from vkccl_b200.comm import buffer_info as _buffer_info_impl


def _buffer_info(obj, writable):
    """(address, bytes, DataType or None) of a buffer, the reference's helper
    signature (reference: python/vccl/__init__.py:186); refuses strided
    tensors with ValueError."""
    b = _buffer_info_impl(obj, writable)
    return b.addr, b.nbytes, b.dtype


__all__ = ["UNIQUE_ID_BYTES", "Communicator", "DataType", "RedOp", "UniqueId", "VcclError", "get_unique_id",
           "group", "group_end", "group_start", "init_all", "mem_alloc", "mem_free", "type_size", "version"]
