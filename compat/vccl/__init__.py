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

from vkccl_b200._lib import _declare, lib as _lib  # noqa: F401
from vkccl_b200.comm import _NAME_TO_TYPE as _DTYPE_NAMES  # noqa: F401
from vkccl_b200.comm import TYPE_SIZE as _TYPE_SIZE  # noqa: F401
from vkccl_b200.comm import _check as _check_impl
from vkccl_b200.comm import _pin_bootstrap_interface as _ensure_bootstrap_addr  # noqa: F401
from vkccl_b200.comm import buffer_info as _buffer_info_impl

# The reference's private helpers under their names (reference:
# python/vccl/__init__.py:61-92, 121-186, 220-243), for code that reached
# into them: the loaded library, its prototypes, the dtype tables (fp8
# added), the result check and the bootstrap-address default.


def _setup_prototypes(lib):
    """Declare this library's C prototypes on a ctypes handle."""
    _declare(lib)


def _check(result, what):
    """Raise VcclError for a non-success vcclResult_t."""
    _check_impl(result, what)


def _buffer_info(obj, writable):
    """(address, bytes, DataType or None) of a buffer, the reference's helper
    signature (reference: python/vccl/__init__.py:186); refuses strided
    tensors with ValueError."""
    b = _buffer_info_impl(obj, writable)
    return b.addr, b.nbytes, b.dtype


__all__ = ["UNIQUE_ID_BYTES", "Communicator", "DataType", "RedOp", "UniqueId", "VcclError", "get_unique_id",
           "group", "group_end", "group_start", "init_all", "mem_alloc", "mem_free", "type_size", "version"]
