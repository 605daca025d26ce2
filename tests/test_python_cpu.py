# SPDX-License-Identifier: Apache-2.0
"""Python layer on the CPU (no GPU): bindings, control-plane communicators in
several processes, single-rank host collectives, and the host-side helpers of
the fused ops.

Multi-process cases run communicators without a device (VCCL_NO_DEVICE=1)
over the TCP bootstrap on 127.0.0.1, as the reference's Python suites run
their ranks as local processes (reference: python/tests/test_bindings.py);
tests/test_host_plane.py moves data between such ranks.
"""

import ctypes
import multiprocessing as mp
import os

import numpy as np
import pytest
import torch

from conftest import ROOT, free_port


def _env(port=None):
    os.environ["VCCL_NO_DEVICE"] = "1"
    os.environ["VCCL_SOCKET_ADDR"] = "127.0.0.1"
    os.environ.setdefault("VCCL_DEBUG", "ERROR")
    if port is not None:
        os.environ["VCCL_COMM_ID"] = f"127.0.0.1:{port}"


def test_metadata():
    import vkccl_b200 as v
    from vkccl_b200._lib import lib

    assert v.version() > 0
    sizes = {v.DataType.INT8: 1, v.DataType.UINT8: 1, v.DataType.INT32: 4, v.DataType.UINT32: 4,
             v.DataType.INT64: 8, v.DataType.UINT64: 8, v.DataType.FLOAT16: 2, v.DataType.FLOAT32: 4,
             v.DataType.FLOAT64: 8, v.DataType.BFLOAT16: 2}
    sizes[v.DataType.FLOAT8E4M3] = 1  # additions after the reference's ten types
    sizes[v.DataType.FLOAT8E5M2] = 1
    assert int(v.DataType.FLOAT8E4M3) == 10 and int(v.DataType.FLOAT8E5M2) == 11
    for dt, sz in sizes.items():
        assert v.type_size(dt) == sz
    for code in range(7):
        assert lib().vcclGetErrorString(code)


def test_unique_id_roundtrip():
    _env()
    import vkccl_b200 as v

    uid = v.get_unique_id()
    assert len(uid.to_bytes()) == v.UNIQUE_ID_BYTES
    assert v.UniqueId.from_hex(uid.hex()).to_bytes() == uid.to_bytes()
    assert v.UniqueId.from_bytes(uid.to_bytes()).hex() == uid.hex()
    with pytest.raises(ValueError):
        v.UniqueId.from_bytes(b"short")


def test_comm_id_derives_same_id():
    port = free_port()
    _env(port)
    import vkccl_b200 as v

    try:
        a, b = v.get_unique_id(), v.get_unique_id()
        assert a.to_bytes() == b.to_bytes()
    finally:
        os.environ.pop("VCCL_COMM_ID", None)


def _rank_body(rank, nranks, port, q):
    try:
        _env(port)
        import vkccl_b200 as v

        uid = v.get_unique_id()
        comm = v.Communicator(nranks, uid, rank)
        assert comm.rank == rank and comm.nranks == nranks
        # even / odd split, ranks ordered by key (reverse rank)
        sub = comm.split(rank % 2, nranks - rank)
        members = [r for r in range(nranks) if r % 2 == rank % 2]
        exp_rank = sorted(members, key=lambda r: nranks - r).index(rank)
        assert sub is not None and sub.nranks == len(members) and sub.rank == exp_rank, (sub.nranks, sub.rank)
        # NOCOLOR takes part and gets no communicator
        none = comm.split(-1 if rank == 0 else 0, rank)
        assert (none is None) == (rank == 0)
        op = comm.create_premul_sum(0.5, v.DataType.FLOAT32)
        comm.destroy_op(op)
        assert comm.async_error() == 0
        if none is not None:
            none.destroy()
        sub.destroy()
        comm.destroy()
        q.put((rank, "ok"))
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e)))


def test_control_plane_multiprocess():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    n = 3
    port = free_port()
    ps = [ctx.Process(target=_rank_body, args=(r, n, port, q)) for r in range(n)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(n))
    for p in ps:
        p.join(timeout=60)
    assert all(v == "ok" for v in res.values()), res


def test_single_rank_host_collectives():
    _env()
    import vkccl_b200 as v

    comm = v.Communicator(1, v.get_unique_id(), 0)
    try:
        x = np.arange(1, 1025, dtype=np.float32)
        y = np.empty_like(x)
        comm.all_reduce(x, y)
        assert np.array_equal(x, y)
        comm.all_reduce(x, y, op=v.RedOp.AVG)
        assert np.array_equal(x, y)
        op = comm.create_premul_sum(2.0, v.DataType.FLOAT32)
        comm.all_reduce(x, y, op=op)
        assert np.array_equal(2 * x, y)
        comm.destroy_op(op)
        g = np.empty_like(x)
        comm.all_gather(x, g)
        assert np.array_equal(x, g)
        t = torch.arange(64, dtype=torch.int32)
        comm.broadcast(t, 0)
        assert torch.equal(t, torch.arange(64, dtype=torch.int32))
    finally:
        comm.destroy()


def test_interleave_gate_up_layout():
    from vkccl_b200.ops.gemm import interleave_gate_up

    i, k = 64, 8
    wg = torch.arange(i * k, dtype=torch.float32).reshape(i, k)
    wu = -wg
    w = interleave_gate_up(wg, wu)
    assert w.shape == (2 * i, k)
    for blk in range(i // 16):
        assert torch.equal(w[32 * blk:32 * blk + 16], wg[16 * blk:16 * blk + 16])
        assert torch.equal(w[32 * blk + 16:32 * blk + 32], wu[16 * blk:16 * blk + 16])
    with pytest.raises(ValueError):
        interleave_gate_up(wg[:10], wu[:10])


def _e4m3_rne(v: np.ndarray) -> np.ndarray:
    """Round float32 values (|v| <= 448) to e4m3 with ties to even, from first principles."""
    out = np.zeros_like(v)
    a = np.abs(v).astype(np.float64)
    nz = a > 0
    e = np.floor(np.log2(np.where(nz, a, 1.0)))
    e = np.maximum(e, -6.0)            # subnormals share the smallest exponent
    step = 2.0 ** (e - 3)              # 3 mantissa bits
    q = a / step
    r = np.floor(q)
    frac = q - r
    r = np.where((frac > 0.5) | ((frac == 0.5) & (r % 2 == 1)), r + 1, r)
    out = np.sign(v) * np.minimum(r * step, 448.0)
    return out.astype(np.float32)


def test_fp8_block_quant_reference_is_round_to_nearest_even():
    from vkccl_b200.ops.moe import quantize_dequantize_reference

    g = torch.Generator().manual_seed(3)
    x = torch.randn(16, 512, generator=g).bfloat16()
    got = quantize_dequantize_reference(x).float().numpy()
    xf = x.float().numpy().reshape(16, 4, 128)
    amax = np.abs(xf).max(-1, keepdims=True)
    scale = np.where(amax > 0, amax / np.float32(448.0), np.float32(1.0)).astype(np.float32)
    q = _e4m3_rne((xf / scale).astype(np.float32))
    ref = torch.from_numpy((q * scale).reshape(16, 512)).bfloat16().float().numpy()
    assert np.array_equal(got, ref)


def test_moe_default_capacity():
    from vkccl_b200.ops.moe import default_capacity

    assert default_capacity(4096, 2, 8) == 16384  # twice the average load of T * topk rows
    assert default_capacity(4096, 2, 1) == 8192   # one rank receives exactly its own pairs
    assert default_capacity(0, 2, 8) == 1


def test_mlp_flops():
    from vkccl_b200.models.llama_mlp import MLPConfig

    cfg = MLPConfig(4096, 14336)
    assert cfg.hidden == 4096 and cfg.intermediate == 14336


def test_parallel_layout_and_buckets():
    from vkccl_b200.parallel import group_layout, plan_buckets

    assert [group_layout(8, r, 4) for r in (0, 3, 4, 7)] == [(0, 0, 0, 0), (0, 3, 3, 0), (1, 0, 0, 1), (1, 3, 3, 1)]
    with pytest.raises(ValueError):
        group_layout(8, 0, 3)
    f32, bf = torch.float32, torch.bfloat16
    # visited last to first; a dtype change or a full bucket closes it
    assert plan_buckets([10, 20, 1000, 5], [f32, f32, f32, bf], 200) == [[3], [2], [1, 0]]
    assert plan_buckets([4, 4, 4], [f32] * 3, 32) == [[2, 1], [0]]


def _groups_body(rank, nranks, port, q):
    try:
        _env(port)
        import vkccl_b200 as v
        from vkccl_b200.parallel import ParallelGroups

        comm = v.Communicator(nranks, v.get_unique_id(), rank)
        pg = ParallelGroups.build(comm, 2)
        assert (pg.tp.nranks, pg.tp.rank) == (2, rank % 2)
        assert (pg.dp.nranks, pg.dp.rank) == (nranks // 2, rank // 2)
        pg.destroy()
        comm.destroy()
        q.put((rank, "ok"))
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e)))


def test_parallel_groups_multiprocess():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    n = 4
    port = free_port()
    ps = [ctx.Process(target=_groups_body, args=(r, n, port, q)) for r in range(n)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(n))
    for p in ps:
        p.join(timeout=60)
    assert all(v == "ok" for v in res.values()), res


def test_compat_package_names():
    import importlib
    import sys

    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "compat"))
    try:
        sys.modules.pop("vccl", None)
        vccl = importlib.import_module("vccl")
        import vkccl_b200

        assert vccl.Communicator is vkccl_b200.Communicator
        for name in ("UniqueId", "DataType", "RedOp", "VcclError", "get_unique_id", "group_start", "group_end"):
            assert getattr(vccl, name) is getattr(vkccl_b200, name)
        assert vccl.UNIQUE_ID_BYTES == 128
        # the reference's private helpers (reference: python/vccl/__init__.py:61-92, 121-243)
        assert vccl._lib() is vkccl_b200._lib.lib()
        assert vccl._TYPE_SIZE[vccl.DataType.BFLOAT16] == 2 and vccl._DTYPE_NAMES["half"] == vccl.DataType.FLOAT16
        assert vccl._buffer_info(bytearray(8), True)[1] == 8
        assert callable(vccl._ensure_bootstrap_addr) and callable(vccl._setup_prototypes)
        try:
            vccl._check(4, "probe")  # vcclInvalidArgument
            raise AssertionError("no error raised")
        except vccl.VcclError as e:
            assert e.result == 4
        tc = importlib.import_module("vccl.torch_comm")
        assert tc.VcclCommunicator.__name__ == "VcclCommunicator"
        import torch

        assert tc._vccl_dtype(torch.zeros(1, dtype=torch.bfloat16)) == vccl.DataType.BFLOAT16
        assert tc._TORCH_DTYPE[torch.float32] == vccl.DataType.FLOAT32
        assert issubclass(tc.VcclCommunicator, tc.DeviceCommunicatorBase)
    finally:
        sys.path.pop(0)
        sys.modules.pop("vccl", None)
        sys.modules.pop("vccl.torch_comm", None)


def test_vllm_plugin_patches_cuda_platform(monkeypatch):
    import sys
    import types

    from vkccl_b200.integration import vllm_plugin

    class FakeCudaPlatform:
        @classmethod
        def get_device_communicator_cls(cls):
            return "vllm.distributed.device_communicators.cuda_communicator.CudaCommunicator"

    fake_cuda = types.ModuleType("vllm.platforms.cuda")
    fake_cuda.CudaPlatform = FakeCudaPlatform
    fake_platforms = types.ModuleType("vllm.platforms")
    fake_platforms.cuda = fake_cuda
    monkeypatch.setitem(sys.modules, "vllm.platforms", fake_platforms)
    monkeypatch.setitem(sys.modules, "vllm.platforms.cuda", fake_cuda)
    monkeypatch.setenv("VKCCL_VLLM", "0")
    assert vllm_plugin.register() is False
    monkeypatch.setenv("VKCCL_VLLM", "1")
    assert vllm_plugin.register() is True
    assert FakeCudaPlatform.get_device_communicator_cls() == "vkccl_b200.torch_comm.VcclCommunicator"


class _MirrorComm:
    """Stands in for a 2-rank vccl communicator whose peer holds the same
    tensors as this rank: all-gather repeats the local data, reduce-scatter
    returns twice this rank's chunk.  Enough to check the layout logic of
    VcclCommunicator (dims, padding, movedim) on the CPU."""

    def __init__(self, rank):
        self.rank = rank

    def all_gather(self, send, recv, sendcount=None, dtype=None):
        flat = send.reshape(-1)
        recv.view(2, -1).copy_(torch.stack([flat, flat]))

    def reduce_scatter(self, send, recv, recvcount=None, dtype=None):
        n = recv.numel()
        recv.reshape(-1).copy_(2 * send.reshape(-1)[self.rank * n:(self.rank + 1) * n])

    def all_reduce(self, send, recv=None, count=None, dtype=None):
        (send if recv is None else recv).mul_(2)


def _mirror_communicator(rank):
    from vkccl_b200.torch_comm import VcclCommunicator

    c = VcclCommunicator.__new__(VcclCommunicator)
    c.world_size, c.rank_in_group, c.vccl = 2, rank, _MirrorComm(rank)
    return c


@pytest.mark.parametrize("dim", [0, 1, 2, -1])
def test_torch_comm_gather_scatter_layouts(dim):
    g = torch.Generator().manual_seed(5)
    x = torch.randn(4, 6, 8, generator=g)
    for rank in (0, 1):
        c = _mirror_communicator(rank)
        assert torch.equal(c.all_gather(x, dim), torch.cat([x, x], dim))
        d = dim % 3
        chunk = x.chunk(2, d)[rank]
        assert torch.equal(c.reduce_scatter(x, dim), 2 * chunk)
        # uneven variant: both mirrored "ranks" send this rank's rows, padded to the largest size
        sizes = [3, 1]
        mine = x[: sizes[rank]]
        padded = torch.zeros((3,) + tuple(x.shape[1:]))
        padded[: sizes[rank]] = mine
        got = c.all_gatherv(mine, 0, sizes)
        assert torch.equal(got, torch.cat([padded[: sizes[0]], padded[: sizes[1]]], 0))
    y = torch.arange(12.0).reshape(6, 2)
    c = _mirror_communicator(0)
    assert torch.equal(c.reduce_scatterv(y, 0, [4, 2]), 2 * y[:4])


class _ThreadWorld:
    """n in-process "ranks" (threads) exchanging tensors, standing in for the
    library's all-to-all and send/recv to check the sequence-parallel
    layout logic on the CPU."""

    def __init__(self, n):
        import threading

        self.n = n
        self.barrier = threading.Barrier(n)
        self.blocks = [None] * n
        self.mail = {}
        self.cv = threading.Condition()


class _ThreadComm:
    def __init__(self, world, rank):
        self.w, self.rank, self.nranks = world, rank, world.n

    def all_to_all(self, send, recv, count=None, dtype=None):
        w = self.w
        w.blocks[self.rank] = send.reshape(w.n, -1).clone()
        w.barrier.wait()
        recv.view(w.n, -1).copy_(torch.stack([w.blocks[i][self.rank] for i in range(w.n)]))
        w.barrier.wait()

    def send(self, buf, peer, count=None, dtype=None):
        with self.w.cv:
            self.w.mail.setdefault((self.rank, peer), []).append(buf.clone())  # FIFO per (src, dst)
            self.w.cv.notify_all()

    def recv(self, buf, peer, count=None, dtype=None):
        with self.w.cv:
            assert self.w.cv.wait_for(lambda: self.w.mail.get((peer, self.rank)), timeout=30), "recv timed out"
            buf.copy_(self.w.mail[(peer, self.rank)].pop(0))


def _run_ranks(n, body):
    import threading

    world = _ThreadWorld(n)
    out, errs = [None] * n, []

    def run(r):
        try:
            out[r] = body(_ThreadComm(world, r))
        except Exception as e:  # noqa: BLE001
            errs.append(repr(e))

    ts = [threading.Thread(target=run, args=(r,)) for r in range(n)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(timeout=60)
    assert not errs, errs
    return out


@pytest.mark.parametrize("n", [1, 2, 4])
def test_ulysses_round_trip(n):
    from vkccl_b200.parallel.sequence import ulysses_heads_to_seq, ulysses_seq_to_heads

    S, H, D = 8 * n, 4 * n, 3
    full = torch.randn(S, H, D, generator=torch.Generator().manual_seed(1))
    s_loc, h_loc = S // n, H // n

    def body(c):
        mine = full[c.rank * s_loc:(c.rank + 1) * s_loc]
        heads = ulysses_seq_to_heads(c, mine)
        assert torch.equal(heads, full[:, c.rank * h_loc:(c.rank + 1) * h_loc])
        return ulysses_heads_to_seq(c, heads)

    outs = _run_ranks(n, body)
    for r in range(n):
        assert torch.equal(outs[r], full[r * s_loc:(r + 1) * s_loc])


def test_ring_pass_visits_every_block():
    from vkccl_b200.parallel.sequence import ring_pass, ring_schedule

    n = 4
    blocks = [torch.full((5,), float(r)) for r in range(n)]

    def body(c):
        held = blocks[c.rank]
        seen = [int(held[0])]
        for _ in range(n - 1):
            held = ring_pass(c, held)
            seen.append(int(held[0]))
        return seen

    outs = _run_ranks(n, body)
    for r in range(n):
        assert tuple(outs[r]) == ring_schedule(n, r)


def test_tuning_table_from_sweep():
    from vkccl_b200.bench.collectives import tuning_table

    rows = [
        {"op": "allreduce", "bytes": 4096, "vccl_us": 5, "vccl_ll_us": 5.0, "vccl_twoshot_us": 20.0},
        {"op": "allreduce", "bytes": 65536, "vccl_us": 6, "vccl_ll_us": 6.0, "vccl_twoshot_us": 21.0},
        {"op": "allreduce", "bytes": 4 << 20, "vccl_us": 20, "vccl_ll2_us": 20.0, "vccl_ll_us": 33.0},
        {"op": "allreduce", "bytes": 256 << 20, "vccl_us": 800, "vccl_nvls_us": 790.0, "vccl_twoshot_us": 900.0},
        {"op": "allgather", "bytes": 4096, "vccl_us": 8},
    ]
    lines = [ln for ln in tuning_table(rows, 8).splitlines() if not ln.startswith("#")]
    assert lines == ["allreduce 8 65536 ll", "allreduce 8 4194304 ll2", "allreduce 8 0 nvls"]


def test_buffer_info_validation():
    import vkccl_b200 as v

    t = torch.arange(12, dtype=torch.float32).reshape(3, 4)
    b = v.buffer_info(t, False)
    assert b.nbytes == 48 and b.dtype == v.DataType.FLOAT32 and not b.cuda
    with pytest.raises(ValueError):
        v.buffer_info(t.T, False)  # non-contiguous
    a = np.zeros(5, dtype=np.float64)
    assert v.buffer_info(a, True).dtype == v.DataType.FLOAT64
    ro = np.zeros(3)
    ro.setflags(write=False)
    with pytest.raises(ValueError):
        v.buffer_info(ro, True)
    assert v.buffer_info(bytearray(16), True).nbytes == 16
    assert v.buffer_info(None, False).addr == 0


def test_single_rank_count_and_dtype_rules():
    _env()
    import vkccl_b200 as v

    comm = v.Communicator(1, v.get_unique_id(), 0)
    try:
        x = bytearray(64)
        with pytest.raises(ValueError):
            comm.all_reduce(x)  # dtype cannot be inferred from a bytearray
        y = bytearray(64)
        comm.all_reduce(x, y, count=16, dtype=v.DataType.FLOAT32)
        with pytest.raises(ValueError):
            comm.all_reduce(12345, count=None, dtype=v.DataType.FLOAT32)  # raw address needs a count
        # buffers of known size that are too small are refused before any copy
        big, small = torch.arange(16, dtype=torch.float32), torch.zeros(8)
        with pytest.raises(ValueError, match="receive"):
            comm.all_reduce(big, small)
        with pytest.raises(ValueError, match="receive"):
            comm.all_gather(big, small)
        with pytest.raises(ValueError, match="send"):
            comm.reduce_scatter(small, big)
        with pytest.raises(ValueError, match="receive"):
            comm.all_to_all_v(big, [16], [0], small, [16], [0])
        with pytest.raises(ValueError, match="recvcounts"):
            comm.all_to_all_v(big, [16], [0], big, [], [0])
        comm.all_gather(small, big, sendcount=8)  # sizes that fit still run
        comm.all_to_all_v(big, [8], [8], small, [8], [0])
        assert torch.equal(small, big[8:])
    finally:
        comm.destroy()


def test_row_groups_and_host_pipeline():
    from vkccl_b200.utils.host_pipeline import row_groups, run_rows

    for rows in (1, 7, 8, 9, 64, 1000, 1024, 8192):
        for groups in (1, 2, 3, 4, 8):
            parts = row_groups(rows, groups)
            assert parts[0][0] == 0 and parts[-1][1] == rows
            assert all(p[1] == q[0] for p, q in zip(parts, parts[1:]))
            assert 1 <= len(parts) <= groups
            assert all((b - a) % 8 == 0 for a, b in parts[:-1])
            assert all(b > a for a, b in parts)
    assert row_groups(1024, 4) == [(0, 256), (256, 512), (512, 768), (768, 1024)]
    assert row_groups(0, 4) == []

    w = torch.randn(16, 5)
    x = torch.randn(100, 16)
    out = torch.empty(100, 5)
    calls = []

    def fn(t):
        calls.append(t.shape[0])
        return t @ w

    for g in (1, 3, 4):
        calls.clear()
        out.zero_()
        run_rows(fn, x, out, groups=g, device="cpu")
        torch.testing.assert_close(out, x @ w)
        assert sum(calls) == 100 and len(calls) == len(row_groups(100, g))
    with pytest.raises(ValueError):
        run_rows(fn, x, torch.empty(99, 5), groups=2, device="cpu")


def test_window_api_without_device():
    """Windows need the device data plane: a control-plane communicator
    refuses them with vcclInvalidUsage, and nothing leaks."""
    _env()
    import vkccl_b200 as v

    comm = v.Communicator(1, v.get_unique_id(), 0)
    try:
        buf = np.zeros(1024, dtype=np.float32)
        with pytest.raises(v.VcclError) as ei:
            comm.window_register(buf)
        assert ei.value.result == 5  # vcclInvalidUsage
        with pytest.raises(v.VcclError):
            comm.window_deregister(ctypes.c_void_p(0))
        with pytest.raises(v.VcclError):
            with comm.window(buf):
                pass
        assert comm.WIN_NO_MULTICAST == 1
        assert comm.check_guards() is None  # no device plane, no guard regions
        # The registration cache has nothing to hold without a device plane.
        comm.reg_cache_flush()
        assert comm.reg_cache_stats() == {"entries": 0, "calls": 0, "hits": 0, "misses": 0, "evictions": 0,
                                          "capacity": 16}
    finally:
        comm.destroy()


def test_registration_cache_capacity_from_env(monkeypatch):
    """The cache's capacity comes from VCCL_REG_CACHE_ENTRIES, else the reference's VCCL_MR_CACHE,
    else 16 (at least 2: a call's send and receive buffers)."""
    _env()
    import vkccl_b200 as v

    for env, want in (({"VCCL_MR_CACHE": "4"}, 4), ({"VCCL_MR_CACHE": "4", "VCCL_REG_CACHE_ENTRIES": "7"}, 7),
                      ({"VCCL_REG_CACHE_ENTRIES": "1"}, 2), ({}, 16)):
        for k in ("VCCL_MR_CACHE", "VCCL_REG_CACHE_ENTRIES"):
            monkeypatch.delenv(k, raising=False)
        for k, val in env.items():
            monkeypatch.setenv(k, val)
        comm = v.Communicator(1, v.get_unique_id(), 0)
        try:
            assert comm.reg_cache_stats()["capacity"] == want, env
        finally:
            comm.destroy()


def test_call_profile(monkeypatch):
    """VCCL_PROF=1: per (operation, algorithm) call counts and bytes, readable through
    prof_summary() and printed to stderr when the communicator is destroyed."""
    _env()
    import subprocess
    import sys
    import textwrap

    import vkccl_b200 as v

    monkeypatch.setenv("VCCL_PROF", "1")
    comm = v.Communicator(1, v.get_unique_id(), 0)
    try:
        a = np.arange(1000, dtype=np.float32)
        b = np.zeros_like(a)
        comm.all_reduce(a, b)
        comm.all_reduce(a, b)
        comm.broadcast(a, 0)
        prof = {(e["op"], e["algo"]): (e["calls"], e["bytes"]) for e in comm.prof_summary()}
        assert prof[("all-reduce", "host")] == (2, 8000)
        assert prof[("broadcast", "host")] == (1, 4000)
    finally:
        comm.destroy()
    monkeypatch.delenv("VCCL_PROF")
    comm = v.Communicator(1, v.get_unique_id(), 0)
    try:
        comm.all_reduce(np.ones(4, dtype=np.float32), np.zeros(4, dtype=np.float32))
        assert comm.prof_summary() == []
    finally:
        comm.destroy()
    code = textwrap.dedent("""
        import numpy as np, vkccl_b200 as v
        c = v.Communicator(1, v.get_unique_id(), 0)
        c.all_reduce(np.ones(256, dtype=np.float32), np.zeros(256, dtype=np.float32))
        c.destroy()
    """)
    p = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120,
                       env=dict(os.environ, VCCL_PROF="1"), cwd=ROOT)
    assert p.returncode == 0, p.stderr
    assert "[VCCL_PROF r0] all-reduce, host: 1 calls, 0.001 MiB" in p.stderr


def test_grad_buckets_single_rank_host():
    """GradBuckets on a one-rank control-plane communicator: average leaves
    the gradients as they are, PreMulSum scales them; host tensors use no window."""
    _env()
    import vkccl_b200 as v
    from vkccl_b200.parallel import GradBuckets

    comm = v.Communicator(1, v.get_unique_id(), 0)
    try:
        torch.manual_seed(0)
        params = [torch.nn.Parameter(torch.randn(n)) for n in (5, 300, 7, 64)]
        for p in params:
            p.grad = torch.randn_like(p)
        want = [p.grad.clone() for p in params]
        gb = GradBuckets(comm, params, bucket_bytes=1024)
        assert len(gb.plan) > 1
        gb.all_reduce()
        for p, w in zip(params, want):
            assert torch.equal(p.grad, w)
        gb.all_reduce(premul=0.5)
        for p, w in zip(params, want):
            torch.testing.assert_close(p.grad, 0.5 * w)
        assert gb._window is None
        gb.close()
    finally:
        comm.destroy()


def test_rs_trace_summary():
    """The GEMM + reduce-scatter trace reader on a synthetic trace."""
    from vkccl_b200.bench.rs_trace import summarise

    t = np.zeros((148, 32), dtype=np.uint64)
    t[:, 20], t[:, 21], t[:, 22], t[:, 23], t[:, 24], t[:, 25] = 1000, 3000, 50000, 7, 200000, 201000
    t[:64, 26], t[:64, 27] = 205000, 215000
    s = summarise(t)
    assert s["freed_wait_us"] == 2.0 and s["tiles_us"] == 197.0 and s["tiles_per_cta"] == 7.0
    assert abs(s["push_per_tile_us"] - 50 / 7) < 0.01 and s["reduce_us"] == 10.0 and s["gemm_end_us"] == 200.0


def test_single_rank_all_to_all_v_and_finalize():
    """all_to_all_v on a one-rank host communicator copies the block at the
    given displacements; finalize succeeds."""
    _env()
    import vkccl_b200 as v

    comm = v.Communicator(1, v.get_unique_id(), 0)
    try:
        x = np.arange(10, dtype=np.float32)
        y = np.full(12, -1.0, dtype=np.float32)
        comm.all_to_all_v(x, [4], [3], y, [4], [5])
        assert np.array_equal(y[5:9], x[3:7])
        assert np.all(y[:5] == -1) and np.all(y[9:] == -1)
        with pytest.raises(ValueError):
            comm.all_to_all_v(bytearray(8), [1], [0], bytearray(8), [1], [0])
        comm.finalize()
    finally:
        comm.destroy()


def test_bindings_declare_every_header_function():
    """Every function of include/vccl.h and include/vccl_tp.h has a ctypes
    prototype in vkccl_b200/_lib.py, and the built library exports it."""
    import re

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    hdr = "".join(open(os.path.join(root, "include", h)).read() for h in ("vccl.h", "vccl_tp.h", "vccl_x.h"))
    names = sorted(set(re.findall(r"\b(vccl[A-Za-z]\w*)\s*\(", hdr)))
    assert len(names) > 40
    src = open(os.path.join(root, "vkccl_b200", "_lib.py")).read()
    assert [n for n in names if f'"{n}"' not in src] == []
    from vkccl_b200._lib import lib

    h = lib()
    assert [n for n in names if not hasattr(h, n)] == []


def test_standalone_base_matches_vllm_base():
    """Without vLLM the communicator derives from a stand-in whose public
    methods are those of vLLM's DeviceCommunicatorBase; VcclCommunicator
    overrides every data-moving one."""
    import inspect

    from vkccl_b200.torch_comm import StandaloneCommunicatorBase, VcclCommunicator

    vbase = pytest.importorskip("vllm.distributed.device_communicators.base_device_communicator")
    base_methods = {m for m, _ in inspect.getmembers(vbase.DeviceCommunicatorBase, inspect.isfunction)
                    if not m.startswith("_")}
    ours = {m for m, _ in inspect.getmembers(VcclCommunicator, inspect.isfunction) if not m.startswith("_")}
    standalone = {m for m, _ in inspect.getmembers(StandaloneCommunicatorBase, inspect.isfunction)
                  if not m.startswith("_")}
    assert base_methods <= ours | standalone, sorted(base_methods - ours - standalone)
    for m in ("all_reduce", "all_gather", "all_gatherv", "reduce_scatter", "reduce_scatterv", "gather",
              "broadcast", "send", "recv", "batch_isend_irecv", "dispatch", "combine", "destroy"):
        assert m in VcclCommunicator.__dict__, m
    init_params = set(inspect.signature(vbase.DeviceCommunicatorBase.__init__).parameters)
    assert init_params <= set(inspect.signature(StandaloneCommunicatorBase.__init__).parameters)


def test_batch_isend_irecv_uses_group_ranks():
    """torch's P2POp holds the global rank in `peer` and the group's rank in
    `group_peer`; the communicator must address vccl ranks by the latter (a
    pipeline group of global ranks [0, 4] has vccl ranks 0 and 1)."""
    from types import SimpleNamespace

    import torch.distributed as dist

    from vkccl_b200.torch_comm import VcclCommunicator

    calls = []

    class Recorder:
        def send(self, t, peer, count, dtype):
            calls.append(("send", peer))

        def recv(self, t, peer, count, dtype):
            calls.append(("recv", peer))

    c = object.__new__(VcclCommunicator)
    c.vccl = Recorder()
    c.ranks = [0, 4]
    t = torch.zeros(4)
    ops = [SimpleNamespace(op=dist.isend, tensor=t, peer=4, group_peer=1),
           SimpleNamespace(op=dist.irecv, tensor=t, peer=4, group_peer=1),
           SimpleNamespace(op=dist.isend, tensor=t, peer=4)]  # no group_peer: global rank 4 -> group rank 1
    c.batch_isend_irecv(ops)
    assert calls == [("send", 1), ("recv", 1), ("send", 1)]
    with pytest.raises(ValueError):
        c.batch_isend_irecv([SimpleNamespace(op=dist.isend, tensor=t, peer=3)])
