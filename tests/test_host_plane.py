# SPDX-License-Identifier: Apache-2.0
"""Host data plane on the CPU: communicators without a device (VCCL_NO_DEVICE=1) and several
ranks in separate processes move host tensors over the TCP mesh (csrc/runtime/hostplane.cc).

The matrix follows the reference's collective suite (reference: tests/test_collectives.cc): every
operation, counts 1 / 7 / 1024 / 65539 (and a large all-reduce split into pieces), sum / prod /
max / min / avg / PreMulSum, integer and float types including bf16, fp16 and fp8, in place and
out of place, every root; grouped send / receive rings; all-to-all(v) with uneven counts.  The
oracle is computed on every rank from every rank's (deterministic) inputs, reducing in rank order
with the same accumulation types, so results must match bit for bit; all-reduce outputs are also
compared across ranks.  A rank that leaves early, and vcclCommAbort from another thread, end the
peers' calls with an error instead of a hang.
"""

import multiprocessing as mp
import os
import threading
import time

import pytest
import torch

from conftest import free_port

DTYPES = [torch.float32, torch.float64, torch.int32, torch.uint8, torch.int64, torch.float16, torch.bfloat16,
          torch.float8_e4m3fn, torch.float8_e5m2]
FLOATS = {torch.float32, torch.float64, torch.float16, torch.bfloat16, torch.float8_e4m3fn, torch.float8_e5m2}
COUNTS = [1, 7, 1024, 65539]


def _env(port):
    os.environ.update(VCCL_NO_DEVICE="1", VCCL_SOCKET_ADDR="127.0.0.1", VCCL_COMM_ID=f"127.0.0.1:{port}",
                      VCCL_DEBUG="ERROR", VCCL_TIMEOUT="30")


def _acc(dt):
    if dt in (torch.float16, torch.bfloat16, torch.float8_e4m3fn, torch.float8_e5m2):
        return torch.float32
    return dt


def _input(rank, count, dt, seed):
    """Small values: sums and products stay exact-ish and in range for every type."""
    g = torch.Generator().manual_seed(seed * 131 + rank)
    if dt in FLOATS:
        v = torch.randint(-8, 9, (count,), generator=g).float() / 4.0
        return v.to(dt)
    if dt == torch.uint8:
        return torch.randint(0, 4, (count,), generator=g).to(dt)
    return torch.randint(-3, 4, (count,), generator=g).to(dt)


def _oracle(xs, dt, op, n):
    """Reduction in rank order in the accumulation type, rounded once to `dt`."""
    acc_t = _acc(dt)
    parts = [x.to(acc_t) for x in xs]
    acc = parts[0].clone()
    for p in parts[1:]:
        if op in ("sum", "avg"):
            acc = acc + p
        elif op == "prod":
            acc = acc * p
        elif op == "max":
            acc = torch.maximum(acc, p)
        else:
            acc = torch.minimum(acc, p)
    if op == "avg":
        acc = acc / torch.tensor(n, dtype=acc_t)
    return acc.to(dt)


def _same(a, b):
    return torch.equal(a.view(torch.uint8) if a.element_size() == 1 else a, b.view(torch.uint8)
                       if b.element_size() == 1 else b)


def _matrix_body(rank, n, port, q):
    try:
        _env(port)
        os.environ["VCCL_PROF"] = "1"
        os.environ["VCCL_HOST_CHUNK"] = "4096"  # many pieces for the larger reductions
        os.environ["VCCL_HOST_BCAST_PIECE"] = "8192"  # ... and broadcasts
        import vkccl_b200 as v

        comm = v.Communicator(n, v.get_unique_id(), rank)
        R = v.RedOp
        seed = 0
        for dt in DTYPES:
            ops = ["sum", "prod", "max", "min"] + (["avg"] if dt in FLOATS else [])
            if dt in (torch.float32, torch.float64, torch.float16, torch.bfloat16):
                ops.append("premul")  # the op's scalar is given in the element type
            for op in ops:
                for count in COUNTS:
                    seed += 1
                    xs = [_input(r, count, dt, seed) for r in range(n)]
                    scalar = 0.5 + 0.25 * rank if op == "premul" else None
                    if op == "premul":
                        # each rank's own scalar: build the oracle from every rank's scaled input
                        acc_t = _acc(dt)
                        scaled = [(x.to(acc_t) * torch.tensor(0.5 + 0.25 * r, dtype=acc_t)).to(dt)
                                  for r, x in enumerate(xs)]
                        want = _oracle(scaled, dt, "sum", n)
                    else:
                        want = _oracle(xs, dt, op, n)
                    rop = {"sum": R.SUM, "prod": R.PROD, "max": R.MAX, "min": R.MIN, "avg": R.AVG}.get(op)
                    handle = None
                    if op == "premul":
                        handle = comm.create_premul_sum(scalar, int(v.comm._NAME_TO_TYPE[str(dt).split(".")[1]]))
                        rop = handle
                    for inplace in (False, True):
                        x = xs[rank].clone()
                        if inplace:
                            comm.all_reduce(x, op=rop)
                            got = x
                        else:
                            got = torch.empty_like(x)
                            comm.all_reduce(x, got, op=rop)
                        assert _same(got, want), f"all_reduce {dt} {op} n={count} inplace={inplace}"
                    if handle is not None:
                        comm.destroy_op(handle)
                    if count == 1024 and op in ("sum", "max"):
                        # reduce to every root; reduce-scatter; every rank's all-reduce output agrees
                        for root in range(n):
                            out = torch.empty_like(xs[rank])
                            comm.reduce(xs[rank].clone(), out, root, op=rop)
                            if rank == root:
                                assert _same(out, want), f"reduce {dt} {op} root={root}"
                        per = count
                        full = [_input(r, per * n, dt, seed + 1000) for r in range(n)]
                        rs_want = _oracle(full, dt, op, n)[rank * per:(rank + 1) * per]
                        rs_out = torch.empty(per, dtype=dt)
                        comm.reduce_scatter(full[rank].clone(), rs_out, op=rop)
                        assert _same(rs_out, rs_want), f"reduce_scatter {dt} {op}"
                        mine = torch.empty_like(xs[rank])
                        comm.all_reduce(xs[rank].clone(), mine, op=rop)
                        everyone = torch.empty(count * n, dtype=dt)
                        comm.all_gather(mine, everyone)
                        for r in range(n):
                            assert _same(everyone[r * count:(r + 1) * count], mine), "ranks disagree"
        # large all-reduce: the reduce-scatter + all-gather form in many pieces
        big = [_input(r, (1 << 20) + 3, torch.float32, 99) for r in range(n)]
        out = torch.empty_like(big[rank])
        comm.all_reduce(big[rank], out)
        assert torch.equal(out, _oracle(big, torch.float32, "sum", n)), "large all_reduce"
        # data movement: all-gather, broadcast, gather, scatter from every root
        for count in COUNTS:
            x = torch.arange(count, dtype=torch.int32) + 1000 * rank
            g = torch.empty(count * n, dtype=torch.int32)
            comm.all_gather(x, g)
            assert torch.equal(g, torch.cat([torch.arange(count, dtype=torch.int32) + 1000 * r for r in range(n)]))
            for root in range(n):
                b = torch.arange(count, dtype=torch.float64) * (rank + 1)
                comm.broadcast(b, root)
                assert torch.equal(b, torch.arange(count, dtype=torch.float64) * (root + 1)), "broadcast"
                gat = torch.full((count * n,), -1, dtype=torch.int32)
                comm.gather(x, gat, root)
                if rank == root:
                    assert torch.equal(gat, g), "gather"
                src = torch.arange(count * n, dtype=torch.int32) * (root + 1)
                sc = torch.empty(count, dtype=torch.int32)
                comm.scatter(src, sc, root)
                assert torch.equal(sc, src[rank * count:(rank + 1) * count]), "scatter"
        # all-to-all and all-to-all(v) with uneven counts (rank r sends r + p + 1 to p)
        a = torch.arange(8 * n, dtype=torch.int64) + 100 * rank
        b = torch.empty_like(a)
        comm.all_to_all(a, b)
        for p in range(n):
            assert torch.equal(b[p * 8:(p + 1) * 8], torch.arange(8, dtype=torch.int64) + 8 * rank + 100 * p)
        scn = [rank + p + 1 for p in range(n)]
        sdp = [sum(scn[:p]) for p in range(n)]
        rcn = [p + rank + 1 for p in range(n)]
        rdp = [sum(rcn[:p]) for p in range(n)]
        s = torch.arange(sum(scn), dtype=torch.int32) + 1000 * rank
        r = torch.full((sum(rcn),), -1, dtype=torch.int32)
        comm.all_to_all_v(s, scn, sdp, r, rcn, rdp)
        for p in range(n):
            # rank p sent me its block [sdp_p[rank], +scn_p[rank]) of arange + 1000 p
            p_sc = [p + k + 1 for k in range(n)]
            p_sd = sum(p_sc[:rank])
            assert torch.equal(r[rdp[p]:rdp[p] + rcn[p]],
                               torch.arange(p_sd, p_sd + p_sc[rank], dtype=torch.int32) + 1000 * p), "all_to_all_v"
        # grouped ring: send to the next rank, receive from the previous, in one group
        for count in (1, 4099, 300000):
            out = torch.arange(count, dtype=torch.float32) + rank
            inc = torch.empty(count, dtype=torch.float32)
            with v.group():
                comm.send(out, (rank + 1) % n)
                comm.recv(inc, (rank - 1) % n)
            assert torch.equal(inc, torch.arange(count, dtype=torch.float32) + (rank - 1) % n), "ring"
        # two messages to the same peer arrive in order
        if n >= 2 and rank < 2:
            peer = 1 - rank
            m1, m2 = torch.full((5,), 10 + rank), torch.full((7,), 20 + rank)
            r1, r2 = torch.empty(5, dtype=m1.dtype), torch.empty(7, dtype=m2.dtype)
            with v.group():
                comm.send(m1, peer)
                comm.send(m2, peer)
                comm.recv(r1, peer)
                comm.recv(r2, peer)
            assert torch.all(r1 == 10 + peer) and torch.all(r2 == 20 + peer), "ordered p2p"
        prof = {(e["op"], e["algo"]) for e in comm.prof_summary()}
        # small all-reduces go direct, large ones as reduce-scatter + all-gather
        assert ("all-reduce", "host TCP mesh, direct") in prof, prof
        assert ("all-reduce", "host TCP mesh, reduce-scatter + all-gather") in prof, prof
        assert ("send", "host TCP mesh") in prof and ("all-gather", "host TCP mesh") in prof, prof
        assert comm.async_error() == 0
        comm.destroy()
        q.put((rank, "ok", sorted(prof)))
    except Exception:  # noqa: BLE001
        import traceback

        q.put((rank, traceback.format_exc(), None))


def _run(body, n, timeout=600):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=body, args=(r, n, port, q)) for r in range(n)]
    for p in ps:
        p.start()
    res = {}
    try:
        for _ in range(n):
            r, status, extra = q.get(timeout=timeout)
            res[r] = (status, extra)
    finally:
        for p in ps:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return res


@pytest.mark.parametrize("n", [2, 3, 4])
def test_host_plane_matrix(n):
    res = _run(_matrix_body, n)
    bad = {r: s for r, (s, _) in res.items() if s != "ok"}
    assert not bad, bad


def _matrix_send_thread_body(rank, n, port, q):
    os.environ["VCCL_HOST_SEND_THREAD_MIN"] = "1"  # every batch that sends and receives hands its sends off
    _matrix_body(rank, n, port, q)


def test_host_plane_matrix_send_thread():
    """The same matrix with the sends of every two-way batch on the sender thread."""
    res = _run(_matrix_send_thread_body, 3)
    bad = {r: s for r, (s, _) in res.items() if s != "ok"}
    assert not bad, bad


def _forced_algo_body(rank, n, port, q):
    """VCCL_ALLREDUCE_ALGO on the host data plane: each family forced at sizes on both sides of
    the default threshold gives the same sums, and the call profile shows the forced path."""
    try:
        _env(port)
        os.environ["VCCL_PROF"] = "1"
        import vkccl_b200 as v

        comm = v.Communicator(n, v.get_unique_id(), rank)
        for algo, label in (("ring", "reduce-scatter + all-gather"), ("recdouble", "direct"),
                            ("twoshot", "reduce-scatter + all-gather"), ("oneshot", "direct")):
            os.environ["VCCL_ALLREDUCE_ALGO"] = algo
            for count in (7 * n, 5000, 1 << 17):
                x = torch.arange(count, dtype=torch.float32) % 17 + rank
                y = torch.empty_like(x)
                comm.all_reduce(x, y)
                want = (torch.arange(count, dtype=torch.float32) % 17) * n + n * (n - 1) // 2
                assert torch.equal(y, want), (algo, count)
            prof = {(e["op"], e["algo"]) for e in comm.prof_summary()}
            assert ("all-reduce", "host TCP mesh, " + label) in prof, (algo, prof)
        del os.environ["VCCL_ALLREDUCE_ALGO"]
        comm.destroy()
        q.put((rank, "ok", None))
    except Exception:  # noqa: BLE001
        import traceback

        q.put((rank, traceback.format_exc(), None))


def test_host_plane_forced_allreduce_algorithm():
    res = _run(_forced_algo_body, 3, timeout=300)
    assert all(s == "ok" for s, _ in res.values()), res


def _dead_peer_body(rank, n, port, q, count=1 << 16):
    try:
        _env(port)
        os.environ["VCCL_TIMEOUT"] = "20"
        import vkccl_b200 as v

        comm = v.Communicator(n, v.get_unique_id(), rank)
        x = torch.ones(1000)
        comm.all_reduce(x)  # the mesh exists and works
        if rank == 1:
            os._exit(0)  # leaves between steps, with nothing in flight
        t0 = time.time()
        try:
            comm.all_reduce(torch.ones(count))
            q.put((rank, "no error", None))
        except v.VcclError:
            q.put((rank, "ok", round(time.time() - t0, 2)))
    except Exception:  # noqa: BLE001
        import traceback

        q.put((rank, traceback.format_exc(), None))


def _dead_peer_send_thread_body(rank, n, port, q):
    os.environ["VCCL_HOST_SEND_THREAD_MIN"] = "4096"
    _dead_peer_body(rank, n, port, q, count=1 << 22)  # 16 MiB: more than the sockets hold


@pytest.mark.parametrize("body", [_dead_peer_body, _dead_peer_send_thread_body], ids=["one_thread", "send_thread"])
def test_host_plane_dead_peer(body):
    """A rank that exits ends its peers' next collective with an error (its streams close),
    also while the sender thread is moving a large message."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    n = 3
    port = free_port()
    ps = [ctx.Process(target=body, args=(r, n, port, q)) for r in range(n)]
    for p in ps:
        p.start()
    res = {}
    for _ in range(n - 1):
        r, status, extra = q.get(timeout=120)
        res[r] = (status, extra)
    for p in ps:
        p.join(timeout=30)
    assert set(res) == {0, 2} and all(s == "ok" for s, _ in res.values()), res
    assert all(t < 15 for _, t in res.values()), res


def _abort_body(rank, n, port, q, count=1 << 16):
    try:
        _env(port)
        import vkccl_b200 as v

        comm = v.Communicator(n, v.get_unique_id(), rank)
        comm.all_reduce(torch.ones(10))
        if rank == 0:
            # rank 1 never joins this call; abort from another thread unblocks it
            threading.Timer(0.5, comm.abort).start()
            t0 = time.time()
            try:
                comm.all_reduce(torch.ones(count))
                q.put((rank, "no error", None))
            except v.VcclError:
                q.put((rank, "ok", round(time.time() - t0, 2)))
        else:
            time.sleep(3)
            q.put((rank, "ok", None))
    except Exception:  # noqa: BLE001
        import traceback

        q.put((rank, traceback.format_exc(), None))


def _abort_send_thread_body(rank, n, port, q):
    os.environ["VCCL_HOST_SEND_THREAD_MIN"] = "4096"
    _abort_body(rank, n, port, q, count=1 << 22)  # the sender thread blocks on a full socket


@pytest.mark.parametrize("body", [_abort_body, _abort_send_thread_body], ids=["one_thread", "send_thread"])
def test_host_plane_abort_unblocks(body):
    res = _run(body, 2, timeout=120)
    assert all(s == "ok" for s, _ in res.values()), res
    assert res[0][1] < 10, res


def _vllm_comm_body(rank, n, port, q):
    """The reference's end-to-end TP layer (reference: python/tests/test_e2e_tp.py:60-92) through
    this library's VcclCommunicator on a CPU process group with CPU tensors."""
    try:
        _env(port)
        import torch.distributed as dist

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port + 1), GLOO_SOCKET_IFNAME="lo")
        dist.init_process_group("gloo", rank=rank, world_size=n)
        from vkccl_b200.torch_comm import VcclCommunicator

        comm = VcclCommunicator(dist.group.WORLD, device=torch.device("cpu"))
        T, H, I = 64, 32, 48
        g = torch.Generator().manual_seed(7)
        x = torch.randn(T, H, generator=g)
        wg, wu = torch.randn(I, H, generator=g) * 0.1, torch.randn(I, H, generator=g) * 0.1
        wd = torch.randn(H, I, generator=g) * 0.1
        shard, ish = T // n, I // n
        xs = x[rank * shard:(rank + 1) * shard]
        # column-parallel gate/up, row-parallel down, sequence-parallel activations
        xf = comm.all_gather(xs, dim=0)
        h = torch.nn.functional.silu(xf @ wg[rank * ish:(rank + 1) * ish].T) * (xf @ wu[rank * ish:(rank + 1) * ish].T)
        y = comm.reduce_scatter(h @ wd[:, rank * ish:(rank + 1) * ish].T, dim=0)
        ref = (torch.nn.functional.silu(x @ wg.T) * (x @ wu.T)) @ wd.T
        torch.testing.assert_close(y, ref[rank * shard:(rank + 1) * shard], rtol=1e-4, atol=1e-5)
        a = torch.full((5,), float(rank + 1))
        assert torch.equal(comm.all_reduce(a.clone()), torch.full((5,), float(n * (n + 1) // 2)))
        b = torch.arange(6, dtype=torch.float32) * (rank + 1)
        assert torch.equal(comm.broadcast(b.clone(), src=n - 1), torch.arange(6, dtype=torch.float32) * n)
        # the reference's staging-buffer cache contract (reference: python/tests/test_torch_comm.py:48-55):
        # one buffer per (role, shape, dtype), at a stable address, none added by repeated calls
        ptr = comm._buf("ar", a.shape, a.dtype).data_ptr()
        comm.all_reduce(a.clone())
        comm.all_reduce(a.clone())
        assert len(comm._buffers) == 1 and comm._buf("ar", a.shape, a.dtype).data_ptr() == ptr
        assert comm._buf("ag_out", (n, 5), torch.bfloat16).dtype == torch.bfloat16 and len(comm._buffers) == 2
        comm.destroy()
        assert not comm._buffers
        dist.destroy_process_group()
        q.put((rank, "ok", None))
    except Exception:  # noqa: BLE001
        import traceback

        q.put((rank, traceback.format_exc(), None))


@pytest.mark.parametrize("n", [2, 3])
def test_vllm_communicator_on_host_plane(n):
    res = _run(_vllm_comm_body, n, timeout=300)
    assert all(s == "ok" for s, _ in res.values()), res


def _distinct_addr_body(rank, n, port, q):
    """Every rank advertises its own address (127.0.0.1, .2, .3: distinct 'hosts' on loopback),
    so the mesh must connect to each rank's own endpoint."""
    try:
        _env(port)
        os.environ["VCCL_SOCKET_ADDR"] = f"127.0.0.{rank + 1}"
        import vkccl_b200 as v

        comm = v.Communicator(n, v.get_unique_id(), rank)
        x = torch.full((70000,), float(rank + 1))
        comm.all_reduce(x)
        assert torch.all(x == n * (n + 1) / 2)
        g = torch.empty(3 * n, dtype=torch.int64)
        comm.all_gather(torch.full((3,), rank), g)
        assert torch.equal(g, torch.arange(n).repeat_interleave(3))
        comm.destroy()
        q.put((rank, "ok", None))
    except Exception:  # noqa: BLE001
        import traceback

        q.put((rank, traceback.format_exc(), None))


def test_host_plane_ranks_on_distinct_addresses():
    res = _run(_distinct_addr_body, 3, timeout=120)
    assert all(s == "ok" for s, _ in res.values()), res


def _grad_buckets_body(rank, n, port, q):
    """Data parallelism on CPU: GradBuckets averages every parameter's gradient over the ranks
    (bucketed all-reduces on the host data plane)."""
    try:
        _env(port)
        import vkccl_b200 as v
        from vkccl_b200.parallel import GradBuckets

        comm = v.Communicator(n, v.get_unique_id(), rank)
        sizes = [1000, 3, 70000, 17]
        params = [torch.nn.Parameter(torch.zeros(s)) for s in sizes]

        def grads(r):
            g = torch.Generator().manual_seed(500 + r)
            return [torch.randn(s, generator=g) for s in sizes]

        for p, g in zip(params, grads(rank)):
            p.grad = g
        gb = GradBuckets(comm, params, bucket_bytes=64 << 10)
        gb.all_reduce()
        mean = [sum(gs) / n for gs in zip(*[grads(r) for r in range(n)])]
        for p, m in zip(params, mean):
            torch.testing.assert_close(p.grad, m, rtol=1e-5, atol=1e-6)
        gb.close()
        comm.destroy()
        q.put((rank, "ok", None))
    except Exception:  # noqa: BLE001
        import traceback

        q.put((rank, traceback.format_exc(), None))


def test_grad_buckets_on_host_plane():
    res = _run(_grad_buckets_body, 3, timeout=120)
    assert all(s == "ok" for s, _ in res.values()), res


def _sequence_body(rank, n, port, q):
    """Context / sequence parallelism on CPU ranks: the Ulysses all-to-all re-sharding round trip
    and the ring pass (grouped send / receive) of vkccl_b200.parallel.sequence over the host
    data plane."""
    try:
        _env(port)
        import vkccl_b200 as v
        from vkccl_b200.parallel.sequence import ring_pass, ring_schedule, ulysses_heads_to_seq, ulysses_seq_to_heads

        comm = v.Communicator(n, v.get_unique_id(), rank)
        S, H, D = 8 * n, 4 * n, 3
        full = torch.randn(S, H, D, generator=torch.Generator().manual_seed(1))
        s_loc, h_loc = S // n, H // n
        heads = ulysses_seq_to_heads(comm, full[rank * s_loc:(rank + 1) * s_loc].contiguous())
        assert torch.equal(heads, full[:, rank * h_loc:(rank + 1) * h_loc]), "seq -> heads"
        back = ulysses_heads_to_seq(comm, heads)
        assert torch.equal(back, full[rank * s_loc:(rank + 1) * s_loc]), "heads -> seq"
        held = torch.full((5,), float(rank))
        seen = [rank]
        for _ in range(n - 1):
            held = ring_pass(comm, held)
            seen.append(int(held[0]))
        assert tuple(seen) == ring_schedule(n, rank), seen
        comm.destroy()
        q.put((rank, "ok", None))
    except Exception:  # noqa: BLE001
        import traceback

        q.put((rank, traceback.format_exc(), None))


@pytest.mark.parametrize("n", [2, 4])
def test_sequence_parallel_on_host_plane(n):
    res = _run(_sequence_body, n, timeout=120)
    assert all(s == "ok" for s, _ in res.values()), res
