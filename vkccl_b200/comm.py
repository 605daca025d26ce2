# SPDX-License-Identifier: Apache-2.0
"""Python communicator over libvccl (ctypes).

Same surface as the reference binding (reference: python/vccl/__init__.py:
220-380: ``get_unique_id``, ``group_start/end``, ``Communicator`` with
all_reduce / all_gather / reduce_scatter / broadcast / send / recv /
register / register_dmabuf / deregister / destroy / handle), extended with
the calls that binding left out (reduce, gather, scatter, all_to_all(v),
split, init_all, abort, PreMulSum ops, mem_alloc) and with CUDA tensors.

Buffer rules:
  * CUDA tensors run stream-ordered on ``stream`` (default: torch's current
    stream), like NCCL; the call returns once the work is queued.
  * Host buffers (numpy arrays, bytearrays, CPU tensors, raw addresses) run
    host-blocking through the reference-named C calls; the library stages
    them through device memory.
"""

from __future__ import annotations

import ctypes
import enum
import os
from typing import Any, List, Optional, Sequence, Tuple

from vkccl_b200._lib import UNIQUE_ID_BYTES, UniqueId, lib


class DataType(enum.IntEnum):
    INT8 = 0
    UINT8 = 1
    INT32 = 2
    UINT32 = 3
    INT64 = 4
    UINT64 = 5
    FLOAT16 = 6
    FLOAT32 = 7
    FLOAT64 = 8
    BFLOAT16 = 9
    FLOAT8E4M3 = 10
    FLOAT8E5M2 = 11


class RedOp(enum.IntEnum):
    SUM = 0
    PROD = 1
    MAX = 2
    MIN = 3
    AVG = 4


TYPE_SIZE = {
    DataType.INT8: 1, DataType.UINT8: 1, DataType.INT32: 4, DataType.UINT32: 4,
    DataType.INT64: 8, DataType.UINT64: 8, DataType.FLOAT16: 2, DataType.FLOAT32: 4,
    DataType.FLOAT64: 8, DataType.BFLOAT16: 2, DataType.FLOAT8E4M3: 1, DataType.FLOAT8E5M2: 1,
}

_NAME_TO_TYPE = {
    "int8": DataType.INT8, "uint8": DataType.UINT8, "int32": DataType.INT32,
    "uint32": DataType.UINT32, "int64": DataType.INT64, "uint64": DataType.UINT64,
    "float16": DataType.FLOAT16, "half": DataType.FLOAT16, "float32": DataType.FLOAT32,
    "float": DataType.FLOAT32, "float64": DataType.FLOAT64, "double": DataType.FLOAT64,
    "bfloat16": DataType.BFLOAT16, "float8_e4m3fn": DataType.FLOAT8E4M3,
    "float8_e5m2": DataType.FLOAT8E5M2,
}


# torch dtype -> DataType (or None), filled on first sight of each dtype
_TORCH_DTYPE_TYPE: dict = {}


def _torch_type(dtype: Any) -> Optional[DataType]:
    try:
        return _TORCH_DTYPE_TYPE[dtype]
    except KeyError:
        t = _NAME_TO_TYPE.get(str(dtype).replace("torch.", ""))
        _TORCH_DTYPE_TYPE[dtype] = t
        return t


def _type_size(dt: int) -> int:
    size = TYPE_SIZE.get(dt)  # IntEnum keys: a plain int finds its member
    if size is None:
        raise ValueError(f"unknown vccl data type {dt}")
    return size


class VcclError(RuntimeError):
    def __init__(self, result: int, what: str, detail: str = ""):
        self.result = result
        msg = lib().vcclGetErrorString(result).decode()
        super().__init__(f"{what}: {msg}" + (f" ({detail})" if detail else ""))


def _check(result: int, what: str, comm: Optional[ctypes.c_void_p] = None) -> None:
    if result != 0:
        detail = lib().vcclGetLastError(comm).decode(errors="replace")
        raise VcclError(result, what, detail)


def version() -> int:
    v = ctypes.c_int()
    _check(lib().vcclGetVersion(ctypes.byref(v)), "vcclGetVersion")
    return v.value


def type_size(dt: int) -> int:
    return int(lib().vcclTypeSize(int(dt)))


class _Buf:
    __slots__ = ("addr", "nbytes", "dtype", "cuda", "device")

    def __init__(self, addr: int, nbytes: int, dtype: Optional[DataType], cuda: bool, device: int):
        self.addr, self.nbytes, self.dtype, self.cuda, self.device = addr, nbytes, dtype, cuda, device


def buffer_info(obj: Any, writable: bool) -> _Buf:
    """Address, size and element type of a buffer-like object."""
    if obj is None:
        return _Buf(0, 0, None, False, -1)
    if isinstance(obj, int):
        return _Buf(obj, 0, None, False, -1)
    data_ptr = getattr(obj, "data_ptr", None)
    if callable(data_ptr):  # torch tensor
        if not obj.is_contiguous():
            raise ValueError("vccl requires a contiguous tensor; call .contiguous() first")
        if obj.is_cuda:
            return _Buf(data_ptr(), obj.nbytes, _torch_type(obj.dtype), True, obj.get_device())
        if not obj.is_cpu:
            raise ValueError(f"unsupported tensor device '{obj.device}'")
        return _Buf(data_ptr(), obj.nbytes, _torch_type(obj.dtype), False, -1)
    iface = getattr(obj, "__array_interface__", None)
    if iface is not None:  # numpy
        addr, readonly = iface["data"]
        if writable and readonly:
            raise ValueError("buffer is read-only")
        return _Buf(addr, obj.nbytes, _NAME_TO_TYPE.get(obj.dtype.name), False, -1)
    view = memoryview(obj)
    if view.readonly:
        raise TypeError("read-only generic buffers are not supported; use numpy or torch")
    addr = ctypes.addressof((ctypes.c_char * 0).from_buffer(obj))
    return _Buf(addr, view.nbytes, None, False, -1)


def _pin_bootstrap_interface() -> None:
    """Advertise a routable address for the rendezvous socket.

    Same policy as the reference (reference: python/vccl/__init__.py:220-243):
    when neither VCCL_SOCKET_ADDR nor VCCL_SOCKET_IFNAME is set, use the
    default-route source address.  Single-host jobs may set
    VCCL_SOCKET_ADDR=127.0.0.1.
    """
    if os.environ.get("VCCL_SOCKET_ADDR") or os.environ.get("VCCL_SOCKET_IFNAME"):
        return
    import socket

    try:
        s = socket.socket(socket.AF_INET, socket.SOCK_DGRAM)
        s.connect(("10.255.255.255", 1))
        ip = s.getsockname()[0]
        s.close()
        if ip and not ip.startswith(("127.", "169.254.")):
            os.environ["VCCL_SOCKET_ADDR"] = ip
    except OSError:
        pass


def get_unique_id() -> UniqueId:
    _pin_bootstrap_interface()
    uid = UniqueId()
    _check(lib().vcclGetUniqueId(ctypes.byref(uid)), "vcclGetUniqueId")
    return uid


def group_start() -> None:
    _check(lib().vcclGroupStart(), "vcclGroupStart")


def group_end() -> None:
    _check(lib().vcclGroupEnd(), "vcclGroupEnd")


class group:
    """Context manager form of group_start/group_end."""

    def __enter__(self) -> "group":
        group_start()
        return self

    def __exit__(self, *exc: Any) -> None:
        group_end()


def mem_alloc(nbytes: int) -> int:
    p = ctypes.c_void_p()
    _check(lib().vcclMemAlloc(ctypes.byref(p), nbytes), "vcclMemAlloc")
    return p.value or 0


def mem_free(addr: int) -> None:
    _check(lib().vcclMemFree(ctypes.c_void_p(addr)), "vcclMemFree")


class _DeviceAlloc:
    """Owns one vcclMemAlloc allocation and exposes it through
    __cuda_array_interface__.  torch.as_tensor keeps this object alive for
    as long as the tensor's storage lives, so the memory is freed with the
    last view of the tensor."""

    def __init__(self, nbytes: int):
        self.addr = mem_alloc(nbytes)
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (self.addr, False),
                                         "version": 3, "strides": None}

    def __del__(self) -> None:
        if getattr(self, "addr", 0):
            try:
                mem_free(self.addr)
            except Exception:  # interpreter shutdown: the process is going away anyway
                pass
            self.addr = 0


def mem_alloc_tensor(shape: Sequence[int], dtype: Any, device: Any = None):
    """A torch tensor on `device` (default: the current CUDA device) backed by vcclMemAlloc
    memory (exportable, so it can be registered as a window).  Deregister any
    window on it before the last view of the tensor goes away."""
    import math

    import torch

    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    nbytes = max(1, math.prod(shape)) * torch.empty((), dtype=dtype).element_size()
    with torch.cuda.device(dev):  # vcclMemAlloc allocates on the current device; the caller's is restored
        raw = torch.as_tensor(_DeviceAlloc(nbytes), device=dev)
    return raw.view(dtype)[: math.prod(shape)].view(*shape)


class _Config(ctypes.Structure):
    _fields_ = [("size", ctypes.c_size_t), ("blocking", ctypes.c_int), ("splitShare", ctypes.c_int)]


class Communicator:
    """One rank's handle on a communicator.

    ``cuda_device`` (optional) is made current before the communicator is
    created; rank r then works on that GPU (``self.device``), and collectives
    take CUDA tensors (stream-ordered on torch's current stream) or host
    buffers (staged through the GPU).  Without a GPU, or with
    ``VCCL_NO_DEVICE=1`` (``self.device == -1``), the communicator moves host
    buffers (numpy arrays, CPU tensors, bytearrays) between its ranks over
    TCP, which may sit on different hosts.
    """

    def __init__(self, nranks: int, unique_id: Optional[UniqueId], rank: int,
                 cuda_device: Optional[int] = None, blocking: bool = True,
                 _handle: Optional[int] = None):
        self._comm = ctypes.c_void_p(_handle) if _handle is not None else ctypes.c_void_p()
        if _handle is None:
            _pin_bootstrap_interface()
            if cuda_device is not None:
                import torch

                # Makes the device's primary context current on this thread; the
                # library (its own static CUDA runtime) finds the device from it.
                torch.cuda.set_device(cuda_device)
            cfg = _Config(ctypes.sizeof(_Config), 1 if blocking else 0, 0)
            _check(lib().vcclCommInitRankConfig(ctypes.byref(self._comm), nranks, unique_id, rank,
                                                ctypes.byref(cfg)), "vcclCommInitRank")
        self.rank = rank
        self.nranks = nranks
        d = ctypes.c_int(-1)
        lib().vcclCommDevice(self._comm, ctypes.byref(d))
        self.device = d.value

    @property
    def handle(self) -> int:
        """Raw ``vcclComm_t`` as an int (for native callers); 0 after destroy."""
        return self._comm.value or 0

    # -- helpers ---------------------------------------------------------------
    def _resolve(self, buf: Any, count: Optional[int], dtype: Optional[int], writable: bool,
                 scale: int = 1) -> Tuple[_Buf, int, int]:
        b = buffer_info(buf, writable)
        dt = dtype if dtype is not None else b.dtype
        if dt is None:
            raise ValueError("dtype could not be inferred; pass dtype=")
        n = count
        if n is None:
            if b.nbytes == 0 and b.addr != 0:
                raise ValueError("count required when passing raw addresses")
            n = b.nbytes // _type_size(dt) // scale
        return b, int(n), int(dt)

    @staticmethod
    def _need(b: _Buf, elems: int, dt: int, what: str) -> None:
        """Refuse a buffer of known size that is too small for the call (a
        kernel would otherwise write or read past its end).  Raw addresses
        and absent buffers (non-root ranks) carry no size and are not checked."""
        need = int(elems) * _type_size(dt)
        if b.nbytes and b.nbytes < need:
            raise ValueError(f"{what} buffer holds {b.nbytes} bytes; the call needs {need}")

    def _stream(self, bufs: Sequence[_Buf], stream: Any) -> Optional[int]:
        """Stream handle for CUDA buffers, or None for the blocking host path."""
        cuda = [b for b in bufs if b.cuda]
        if not cuda:
            return None
        if stream is None:
            import torch

            # the buffers' device, which need not be the current one
            return torch.cuda.current_stream(cuda[0].device).cuda_stream
        if isinstance(stream, int):
            return stream
        return stream.cuda_stream

    def _op(self, op: Any) -> int:
        return int(op)

    # -- collectives -------------------------------------------------------------
    def all_reduce(self, send: Any, recv: Any = None, count: Optional[int] = None,
                   dtype: Optional[int] = None, op: Any = RedOp.SUM, stream: Any = None) -> None:
        if recv is None:
            recv = send
        s, n, dt = self._resolve(send, count, dtype, False)
        r, _, _ = self._resolve(recv, n, dt, True)
        self._need(r, n, dt, "receive")
        st = self._stream([s, r], stream)
        L = lib()
        if st is None:
            _check(L.vcclAllReduce(s.addr, r.addr, n, dt, self._op(op), self._comm), "vcclAllReduce", self._comm)
        else:
            _check(L.vcclAllReduceAsync(s.addr, r.addr, n, dt, self._op(op), self._comm, st),
                   "vcclAllReduceAsync", self._comm)

    def reduce(self, send: Any, recv: Any, root: int, count: Optional[int] = None,
               dtype: Optional[int] = None, op: Any = RedOp.SUM, stream: Any = None) -> None:
        s, n, dt = self._resolve(send, count, dtype, False)
        r = buffer_info(recv, True)
        self._need(r, n, dt, "receive")
        st = self._stream([s, r], stream)
        L = lib()
        if st is None:
            _check(L.vcclReduce(s.addr, r.addr, n, dt, self._op(op), root, self._comm), "vcclReduce", self._comm)
        else:
            _check(L.vcclReduceAsync(s.addr, r.addr, n, dt, self._op(op), root, self._comm, st),
                   "vcclReduceAsync", self._comm)

    def all_gather(self, send: Any, recv: Any, sendcount: Optional[int] = None,
                   dtype: Optional[int] = None, stream: Any = None) -> None:
        s, n, dt = self._resolve(send, sendcount, dtype, False)
        r, _, _ = self._resolve(recv, n, dt, True)
        self._need(r, n * self.nranks, dt, "receive")
        st = self._stream([s, r], stream)
        L = lib()
        if st is None:
            _check(L.vcclAllGather(s.addr, r.addr, n, dt, self._comm), "vcclAllGather", self._comm)
        else:
            _check(L.vcclAllGatherAsync(s.addr, r.addr, n, dt, self._comm, st), "vcclAllGatherAsync",
                   self._comm)

    def reduce_scatter(self, send: Any, recv: Any, recvcount: Optional[int] = None,
                       dtype: Optional[int] = None, op: Any = RedOp.SUM, stream: Any = None) -> None:
        r, n, dt = self._resolve(recv, recvcount, dtype, True)
        s, _, _ = self._resolve(send, n, dt, False)
        self._need(s, n * self.nranks, dt, "send")
        st = self._stream([s, r], stream)
        L = lib()
        if st is None:
            _check(L.vcclReduceScatter(s.addr, r.addr, n, dt, self._op(op), self._comm), "vcclReduceScatter",
                   self._comm)
        else:
            _check(L.vcclReduceScatterAsync(s.addr, r.addr, n, dt, self._op(op), self._comm, st),
                   "vcclReduceScatterAsync", self._comm)

    def broadcast(self, buf: Any, root: int, count: Optional[int] = None, dtype: Optional[int] = None,
                  recv: Any = None, stream: Any = None) -> None:
        b, n, dt = self._resolve(buf, count, dtype, True)
        r = b if recv is None else self._resolve(recv, n, dt, True)[0]
        self._need(r, n, dt, "receive")
        st = self._stream([b, r], stream)
        L = lib()
        if st is None:
            _check(L.vcclBroadcast(b.addr, r.addr, n, dt, root, self._comm), "vcclBroadcast", self._comm)
        else:
            _check(L.vcclBroadcastAsync(b.addr, r.addr, n, dt, root, self._comm, st), "vcclBroadcastAsync",
                   self._comm)

    def gather(self, send: Any, recv: Any, root: int, sendcount: Optional[int] = None,
               dtype: Optional[int] = None, stream: Any = None) -> None:
        s, n, dt = self._resolve(send, sendcount, dtype, False)
        r = buffer_info(recv, True)
        self._need(r, n * self.nranks, dt, "receive")
        st = self._stream([s, r], stream)
        L = lib()
        if st is None:
            _check(L.vcclGather(s.addr, r.addr, n, dt, root, self._comm), "vcclGather", self._comm)
        else:
            _check(L.vcclGatherAsync(s.addr, r.addr, n, dt, root, self._comm, st), "vcclGatherAsync", self._comm)

    def scatter(self, send: Any, recv: Any, root: int, recvcount: Optional[int] = None,
                dtype: Optional[int] = None, stream: Any = None) -> None:
        r, n, dt = self._resolve(recv, recvcount, dtype, True)
        s = buffer_info(send, False)
        self._need(s, n * self.nranks, dt, "send")
        st = self._stream([s, r], stream)
        L = lib()
        if st is None:
            _check(L.vcclScatter(s.addr, r.addr, n, dt, root, self._comm), "vcclScatter", self._comm)
        else:
            _check(L.vcclScatterAsync(s.addr, r.addr, n, dt, root, self._comm, st), "vcclScatterAsync",
                   self._comm)

    def all_to_all(self, send: Any, recv: Any, count: Optional[int] = None, dtype: Optional[int] = None,
                   stream: Any = None) -> None:
        s, n, dt = self._resolve(send, count, dtype, False, scale=self.nranks)
        r, _, _ = self._resolve(recv, n, dt, True)
        self._need(s, n * self.nranks, dt, "send")
        self._need(r, n * self.nranks, dt, "receive")
        st = self._stream([s, r], stream)
        L = lib()
        if st is None:
            _check(L.vcclAllToAll(s.addr, r.addr, n, dt, self._comm), "vcclAllToAll", self._comm)
        else:
            _check(L.vcclAllToAllAsync(s.addr, r.addr, n, dt, self._comm, st), "vcclAllToAllAsync", self._comm)

    def all_to_all_v(self, send: Any, sendcounts: Sequence[int], sdispls: Sequence[int], recv: Any,
                     recvcounts: Sequence[int], rdispls: Sequence[int], dtype: Optional[int] = None,
                     stream: Any = None) -> None:
        s = buffer_info(send, False)
        r = buffer_info(recv, True)
        dt = dtype if dtype is not None else (s.dtype if s.dtype is not None else r.dtype)
        if dt is None:
            raise ValueError("dtype could not be inferred; pass dtype=")
        for name, v in (("sendcounts", sendcounts), ("sdispls", sdispls), ("recvcounts", recvcounts),
                        ("rdispls", rdispls)):
            if len(v) != self.nranks:
                raise ValueError(f"{name} has {len(v)} entries; the communicator has {self.nranks} ranks")
        arr = ctypes.c_size_t * self.nranks
        sc, sd, rc, rd = (arr(*[int(x) for x in v]) for v in (sendcounts, sdispls, recvcounts, rdispls))
        self._need(s, max((sd[i] + sc[i] for i in range(self.nranks) if sc[i]), default=0), int(dt), "send")
        self._need(r, max((rd[i] + rc[i] for i in range(self.nranks) if rc[i]), default=0), int(dt), "receive")
        st = self._stream([s, r], stream)
        L = lib()
        if st is None:
            _check(L.vcclAllToAllv(s.addr, sc, sd, r.addr, rc, rd, int(dt), self._comm), "vcclAllToAllv",
                   self._comm)
        else:
            _check(L.vcclAllToAllvAsync(s.addr, sc, sd, r.addr, rc, rd, int(dt), self._comm, st),
                   "vcclAllToAllvAsync", self._comm)

    def send(self, buf: Any, peer: int, count: Optional[int] = None, dtype: Optional[int] = None,
             stream: Any = None) -> None:
        b, n, dt = self._resolve(buf, count, dtype, False)
        st = self._stream([b], stream)
        L = lib()
        if st is None:
            _check(L.vcclSend(b.addr, n, dt, peer, self._comm), "vcclSend", self._comm)
        else:
            _check(L.vcclSendAsync(b.addr, n, dt, peer, self._comm, st), "vcclSendAsync", self._comm)

    def recv(self, buf: Any, peer: int, count: Optional[int] = None, dtype: Optional[int] = None,
             stream: Any = None) -> None:
        b, n, dt = self._resolve(buf, count, dtype, True)
        st = self._stream([b], stream)
        L = lib()
        if st is None:
            _check(L.vcclRecv(b.addr, n, dt, peer, self._comm), "vcclRecv", self._comm)
        else:
            _check(L.vcclRecvAsync(b.addr, n, dt, peer, self._comm, st), "vcclRecvAsync", self._comm)

    # -- ops ---------------------------------------------------------------------
    def create_premul_sum(self, scalar: float, dtype: int = DataType.FLOAT32) -> int:
        """PreMulSum op: sum over ranks of scalar * input (float types)."""
        import struct

        dt = DataType(dtype)
        if dt == DataType.FLOAT32:
            raw = ctypes.c_float(scalar)
        elif dt == DataType.FLOAT64:
            raw = ctypes.c_double(scalar)
        elif dt == DataType.FLOAT16:
            raw = ctypes.c_uint16(struct.unpack("<H", struct.pack("<e", scalar))[0])
        elif dt == DataType.BFLOAT16:
            raw = ctypes.c_uint16(struct.unpack("<I", struct.pack("<f", scalar))[0] >> 16)
        else:
            raise ValueError("PreMulSum needs a float datatype")
        op = ctypes.c_int()
        _check(lib().vcclRedOpCreatePreMulSum(ctypes.byref(op), ctypes.byref(raw), int(dt), 1, self._comm),
               "vcclRedOpCreatePreMulSum", self._comm)
        return op.value

    def destroy_op(self, op: int) -> None:
        _check(lib().vcclRedOpDestroy(int(op), self._comm), "vcclRedOpDestroy", self._comm)

    # -- lifecycle -----------------------------------------------------------------
    def split(self, color: int, key: int) -> Optional["Communicator"]:
        out = ctypes.c_void_p()
        _check(lib().vcclCommSplit(self._comm, color, key, ctypes.byref(out), None), "vcclCommSplit", self._comm)
        if not out.value:
            return None
        n, r = ctypes.c_int(), ctypes.c_int()
        lib().vcclCommCount(out, ctypes.byref(n))
        lib().vcclCommUserRank(out, ctypes.byref(r))
        return Communicator(n.value, None, r.value, _handle=out.value)

    def abort(self) -> None:
        if self._comm:
            lib().vcclCommAbort(self._comm)

    def async_error(self) -> int:
        e = ctypes.c_int()
        _check(lib().vcclCommGetAsyncError(self._comm, ctypes.byref(e)), "vcclCommGetAsyncError")
        return e.value

    def finalize(self) -> None:
        _check(lib().vcclCommFinalize(self._comm), "vcclCommFinalize", self._comm)

    def fused_trace(self):
        """Per-CTA event times (ns) of the fused kernels, as a [ctas, 32]
        numpy array, when the communicator was created with
        VCCL_FUSED_TRACE=1; None otherwise.  Last all-gather + GEMM: 0 start,
        1 previous call's shard taken by every peer, 2 own slice staged, 3..9
        s-th peer shard pulled, 10..17 first tile of the s-th shard released,
        18 end.  Last GEMM + reduce-scatter: 20-27 (vkccl_b200.bench.rs_trace)."""
        import numpy as np

        out = np.zeros((256, 32), dtype=np.uint64)
        ctas = ctypes.c_int(0)
        r = lib().vcclxFusedTrace(self._comm, out.ctypes.data, ctypes.byref(ctas))
        if r != 0:
            return None
        return out[: ctas.value].copy()

    def check_guards(self) -> Optional[int]:
        """Bytes of this rank's debug guard regions that some kernel overwrote
        (communicator created with VCCL_GUARDS=1; synchronises the device),
        or None without guards."""
        bad = ctypes.c_ulonglong(0)
        if lib().vcclxCheckGuards(self._comm, ctypes.byref(bad)) != 0:
            return None
        return int(bad.value)

    def last_error(self) -> str:
        return lib().vcclGetLastError(self._comm).decode(errors="replace")

    # -- memory registration -----------------------------------------------------
    def register(self, buf: Any, nbytes: Optional[int] = None) -> ctypes.c_void_p:
        b = buffer_info(buf, True)
        h = ctypes.c_void_p()
        _check(lib().vcclCommRegister(self._comm, b.addr, nbytes or b.nbytes, ctypes.byref(h)),
               "vcclCommRegister", self._comm)
        return h

    def register_dmabuf(self, fd: int, nbytes: int, offset: int = 0) -> Tuple[int, ctypes.c_void_p]:
        ptr, h = ctypes.c_void_p(), ctypes.c_void_p()
        _check(lib().vcclCommRegisterDmaBuf(self._comm, fd, offset, nbytes, ctypes.byref(ptr), ctypes.byref(h)),
               "vcclCommRegisterDmaBuf", self._comm)
        return ptr.value or 0, h

    def deregister(self, handle: ctypes.c_void_p) -> None:
        _check(lib().vcclCommDeregister(self._comm, handle), "vcclCommDeregister", self._comm)

    # -- windows (zero-copy collectives) -----------------------------------------
    WIN_NO_MULTICAST = 0x1

    def window_register(self, buf: Any, nbytes: Optional[int] = None, flags: int = 0) -> ctypes.c_void_p:
        """Collective: map `buf` (the same size on every rank) into every rank.
        vcclMemAlloc memory (mem_alloc_tensor) is also bound to an NVLS
        multicast object; an ordinary CUDA tensor is shared by CUDA IPC.
        Collectives on buffers inside windows then read and write the peers'
        buffers in place; every rank must pass buffers at the same offsets of
        its windows.  Keep the memory alive (for a PyTorch tensor: the tensor,
        and no torch.cuda.empty_cache()) until window_deregister."""
        b = buffer_info(buf, True)
        h = ctypes.c_void_p()
        _check(lib().vcclCommWindowRegister(self._comm, b.addr, nbytes or b.nbytes, ctypes.byref(h), flags),
               "vcclCommWindowRegister", self._comm)
        return h

    def window_deregister(self, handle: ctypes.c_void_p) -> None:
        """Collective: undo window_register (before the memory is freed)."""
        _check(lib().vcclCommWindowDeregister(self._comm, handle), "vcclCommWindowDeregister", self._comm)

    # -- call profile (VCCL_PROF=1) ---------------------------------------------
    def prof_summary(self) -> list:
        """Per (operation, algorithm) this rank ran since the communicator was
        created with VCCL_PROF=1: dicts with op, algo, calls and bytes (count x
        type size summed).  Empty without VCCL_PROF."""
        buf = ctypes.create_string_buffer(1 << 16)
        _check(lib().vcclxProfSummary(self._comm, buf, len(buf)), "vcclxProfSummary", self._comm)
        out = []
        for line in buf.value.decode().splitlines():
            op, algo, calls, nbytes = line.split("\t")
            out.append({"op": op, "algo": algo, "calls": int(calls), "bytes": int(nbytes)})
        return out

    # -- registration cache (windows on demand; VCCL_REG_CACHE=1) -------------
    def reg_cache_flush(self) -> None:
        """Collective: drop every window the registration cache holds.  Call it
        on every rank before cached memory goes back to CUDA (for PyTorch
        tensors: before torch.cuda.empty_cache()); the peers keep cached
        allocations open until then."""
        _check(lib().vcclCommRegCacheFlush(self._comm), "vcclCommRegCacheFlush", self._comm)

    def reg_cache_stats(self) -> dict:
        """Counters of the registration cache: entries held, calls that
        consulted it on every rank, buffers reused, buffers registered,
        entries dropped, and its capacity."""
        out = (ctypes.c_ulonglong * 6)()
        _check(lib().vcclCommRegCacheStats(self._comm, out), "vcclCommRegCacheStats", self._comm)
        return dict(zip(("entries", "calls", "hits", "misses", "evictions", "capacity"), (int(v) for v in out)))

    def window(self, buf: Any, nbytes: Optional[int] = None, flags: int = 0) -> "_WindowScope":
        """`with comm.window(t): ...` registers `t` for the block (collective on
        entry and exit)."""
        return _WindowScope(self, buf, nbytes, flags)

    def destroy(self) -> None:
        if self._comm:
            lib().vcclCommDestroy(self._comm)
            self._comm = ctypes.c_void_p()

    def __enter__(self) -> "Communicator":
        return self

    def __exit__(self, *exc: Any) -> None:
        self.destroy()


class _WindowScope:
    def __init__(self, comm: "Communicator", buf: Any, nbytes: Optional[int], flags: int):
        self.comm, self.buf, self.nbytes, self.flags = comm, buf, nbytes, flags
        self.handle: Optional[ctypes.c_void_p] = None

    def __enter__(self) -> ctypes.c_void_p:
        self.handle = self.comm.window_register(self.buf, self.nbytes, self.flags)
        return self.handle

    def __exit__(self, *exc: Any) -> None:
        if self.handle is not None:
            self.comm.window_deregister(self.handle)
            self.handle = None


def init_all(ndev: int, devlist: Optional[Sequence[int]] = None) -> List[Communicator]:
    """vcclCommInitAll: ``ndev`` communicators in this process."""
    arr = (ctypes.c_void_p * ndev)()
    dl = (ctypes.c_int * ndev)(*devlist) if devlist is not None else None
    _check(lib().vcclCommInitAll(arr, ndev, dl), "vcclCommInitAll")
    return [Communicator(ndev, None, i, _handle=arr[i]) for i in range(ndev)]
