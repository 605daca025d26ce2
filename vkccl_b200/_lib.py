# SPDX-License-Identifier: Apache-2.0
"""Loader and ctypes prototypes for libvccl.so.

The shared library is built in-tree (``make`` at the repository root) into
``vkccl_b200/_native/libvccl.so``; ``VCCL_LIBRARY`` overrides the path.  The
reference binding loads its library the same way (reference:
python/vccl/__init__.py:121-178); this one declares every entry point.
"""

from __future__ import annotations

import ctypes
import os
from typing import Optional

UNIQUE_ID_BYTES = 128

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB: Optional[ctypes.CDLL] = None


class UniqueId(ctypes.Structure):
    """Opaque 128-byte rendezvous id (``vcclUniqueId``)."""

    _fields_ = [("internal", ctypes.c_ubyte * UNIQUE_ID_BYTES)]

    def hex(self) -> str:
        return bytes(self.internal).hex()

    def to_bytes(self) -> bytes:
        return bytes(self.internal)

    @classmethod
    def from_bytes(cls, raw: bytes) -> "UniqueId":
        if len(raw) != UNIQUE_ID_BYTES:
            raise ValueError(f"unique id must be {UNIQUE_ID_BYTES} bytes, got {len(raw)}")
        uid = cls()
        ctypes.memmove(uid.internal, raw, UNIQUE_ID_BYTES)
        return uid

    @classmethod
    def from_hex(cls, s: str) -> "UniqueId":
        return cls.from_bytes(bytes.fromhex(s.strip()))


def library_path() -> str:
    env = os.environ.get("VCCL_LIBRARY")
    if env:
        return env
    return os.path.join(_HERE, "_native", "libvccl.so")


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        path = library_path()
        if not os.path.exists(path):
            raise OSError(
                f"libvccl.so not found at {path}; build it with `make -j` at the "
                "repository root (or set VCCL_LIBRARY)")
        handle = ctypes.CDLL(path)
        _declare(handle)
        _LIB = handle
    return _LIB


def _declare(h: ctypes.CDLL) -> None:
    c = ctypes
    P = c.c_void_p
    I = c.c_int
    Z = c.c_size_t
    ZP = c.POINTER(c.c_size_t)
    sig = {
        "vcclGetVersion": [c.POINTER(I)],
        "vcclGetUniqueId": [c.POINTER(UniqueId)],
        "vcclCommInitRank": [c.POINTER(P), I, UniqueId, I],
        "vcclCommInitRankConfig": [c.POINTER(P), I, UniqueId, I, P],
        "vcclCommInitAll": [c.POINTER(P), I, c.POINTER(I)],
        "vcclCommSplit": [P, I, I, c.POINTER(P), P],
        "vcclCommFinalize": [P],
        "vcclCommDestroy": [P],
        "vcclCommAbort": [P],
        "vcclCommGetAsyncError": [P, c.POINTER(I)],
        "vcclCommCount": [P, c.POINTER(I)],
        "vcclCommUserRank": [P, c.POINTER(I)],
        "vcclCommDevice": [P, c.POINTER(I)],
        "vcclAllGather": [P, P, Z, I, P],
        "vcclReduceScatter": [P, P, Z, I, I, P],
        "vcclAllReduce": [P, P, Z, I, I, P],
        "vcclReduce": [P, P, Z, I, I, I, P],
        "vcclBroadcast": [P, P, Z, I, I, P],
        "vcclBcast": [P, Z, I, I, P],
        "vcclGather": [P, P, Z, I, I, P],
        "vcclScatter": [P, P, Z, I, I, P],
        "vcclAllToAll": [P, P, Z, I, P],
        "vcclAllToAllv": [P, ZP, ZP, P, ZP, ZP, I, P],
        "vcclSend": [P, Z, I, I, P],
        "vcclRecv": [P, Z, I, I, P],
        "vcclAllGatherAsync": [P, P, Z, I, P, P],
        "vcclReduceScatterAsync": [P, P, Z, I, I, P, P],
        "vcclAllReduceAsync": [P, P, Z, I, I, P, P],
        "vcclReduceAsync": [P, P, Z, I, I, I, P, P],
        "vcclBroadcastAsync": [P, P, Z, I, I, P, P],
        "vcclGatherAsync": [P, P, Z, I, I, P, P],
        "vcclScatterAsync": [P, P, Z, I, I, P, P],
        "vcclAllToAllAsync": [P, P, Z, I, P, P],
        "vcclAllToAllvAsync": [P, ZP, ZP, P, ZP, ZP, I, P, P],
        "vcclSendAsync": [P, Z, I, I, P, P],
        "vcclRecvAsync": [P, Z, I, I, P, P],
        "vcclGroupStart": [],
        "vcclGroupEnd": [],
        "vcclRedOpCreatePreMulSum": [c.POINTER(I), P, I, I, P],
        "vcclRedOpDestroy": [I, P],
        "vcclMemAlloc": [c.POINTER(P), Z],
        "vcclMemFree": [P],
        "vcclCommRegister": [P, P, Z, c.POINTER(P)],
        "vcclCommDeregister": [P, P],
        "vcclCommRegisterDmaBuf": [P, I, c.c_uint64, Z, c.POINTER(P), c.POINTER(P)],
        "vcclCommWindowRegister": [P, P, Z, c.POINTER(P), I],
        "vcclCommWindowDeregister": [P, P],
        "vcclCommRegCacheFlush": [P],
        "vcclCommRegCacheStats": [P, c.POINTER(c.c_ulonglong)],
        "vcclTypeSize": [I],
        "vcclGetErrorString": [I],
        "vcclGetLastError": [P],
    }
    for name, args in sig.items():
        fn = getattr(h, name)
        fn.argtypes = args
        fn.restype = c.c_int
    h.vcclTypeSize.restype = c.c_size_t
    h.vcclGetErrorString.restype = c.c_char_p
    h.vcclGetLastError.restype = c.c_char_p
    _declare_extensions(h)


def _declare_extensions(h: ctypes.CDLL) -> None:
    """Fused tensor-parallel entry points (vccl_tp.h), when built."""
    c = ctypes
    P, I, Z, F = c.c_void_p, c.c_int, c.c_size_t, c.c_float
    ext = {
        "vcclAllReduceAddRMSNorm": [P, P, P, P, Z, Z, F, I, P, P],
        "vcclGemmBf16": [P, P, P, I, I, I, P],
        "vcclGemmBf16NoAlloc": [P, P, P, I, I, I, P],
        "vcclxFusedTrace": [P, P, P],
        "vcclxCheckGuards": [P, c.POINTER(c.c_ulonglong)],
        "vcclxBarrierBench": [P, I, I, I, c.POINTER(F)],
        "vcclxNoAllocInjectAbort": [I],
        "vcclxProfSummary": [P, c.c_char_p, Z],
        "vcclGemmSiluMul": [P, P, P, I, I, I, P],
        "vcclGemmReduceScatter": [P, P, P, I, I, I, P, P],
        "vcclAllGatherGemm": [P, P, P, I, I, I, I, P, P],
        "vcclMoeDispatchFp8": [P, P, P, P, P, P, P, I, I, I, I, I, P, P],
        "vcclMoeCombine": [P, P, P, P, P, I, I, I, I, P, P],
    }
    for name, args in ext.items():
        fn = getattr(h, name, None)
        if fn is not None:
            fn.argtypes = args
            fn.restype = c.c_int
