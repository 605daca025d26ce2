# SPDX-License-Identifier: Apache-2.0
"""Per-rank body of the VcclCommunicator GPU test (run by torchrun).

Mirrors the reference's torch communicator and end-to-end TP suites
(reference: python/tests/test_torch_comm.py, python/tests/test_e2e_tp.py) on
CUDA tensors: the gloo group only carries the unique id, the collectives run
on this library.  Every rank builds every rank's seeded inputs, so each can
compute the expected results locally.
"""

import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))

from vkccl_b200.ops.moe import quantize_dequantize_reference  # noqa: E402
from vkccl_b200.torch_comm import VcclCommunicator  # noqa: E402


def close(got, ref, tol, what):
    err = (got.float() - ref.float()).abs().max().item()
    scale = ref.float().abs().max().item() + 1e-6
    if err > tol * scale + 1e-5:
        raise AssertionError(f"{what}: max err {err:.4g} vs scale {scale:.4g}")


def per_rank(seed, n, shape, dtype=torch.float32):
    out = []
    for r in range(n):
        g = torch.Generator(device="cuda").manual_seed(seed * 100 + r)
        out.append(torch.randn(*shape, device="cuda", generator=g).to(dtype))
    return out


def main():
    dist.init_process_group("gloo")
    rank, n = dist.get_rank(), dist.get_world_size()
    torch.cuda.set_device(rank)
    comm = VcclCommunicator(dist.group.WORLD, device=torch.device("cuda", rank))

    # all_reduce (fp32 exact-ish, bf16 with tolerance), twice to reuse buffers
    for it, (dt, tol) in enumerate(((torch.float32, 1e-5), (torch.bfloat16, 3e-2), (torch.float32, 1e-5))):
        xs = per_rank(10 + it, n, (4099,), dt)
        got = comm.all_reduce(xs[rank].clone())
        close(got, sum(x.float() for x in xs), tol, f"all_reduce {dt}")

    # all_gather along dims 0, 1 and -1
    xs = per_rank(20, n, (3, 5, 7))
    for dim in (0, 1, -1):
        close(comm.all_gather(xs[rank], dim), torch.cat(xs, dim), 0, f"all_gather dim={dim}")

    # reduce_scatter along dims 0 and -1
    xs = per_rank(30, n, (4 * n, 6, 2 * n))
    total = sum(xs)
    for dim in (0, -1):
        close(comm.reduce_scatter(xs[rank], dim), total.chunk(n, dim)[rank], 1e-5, f"reduce_scatter dim={dim}")

    # broadcast from the last rank
    xs = per_rank(40, n, (1000,))
    t = xs[rank].clone()
    close(comm.broadcast(t, src=n - 1), xs[n - 1], 0, "broadcast")

    # gather to rank 0 along the last dim
    xs = per_rank(50, n, (2, 3))
    g = comm.gather(xs[rank], dst=0, dim=-1)
    if rank == 0:
        close(g, torch.cat(xs, -1), 0, "gather")
    else:
        assert g is None

    # pipeline-style send/recv ring and a batched exchange
    if n > 1:
        xs = per_rank(60, n, (257,))
        nxt, prv = (rank + 1) % n, (rank - 1) % n
        ops = [dist.P2POp(dist.isend, xs[rank], nxt), dist.P2POp(dist.irecv, torch.empty_like(xs[rank]), prv)]
        comm.batch_isend_irecv(ops)
        torch.cuda.synchronize()
        close(ops[1].tensor, xs[prv], 0, "batch_isend_irecv")
        if rank % 2 == 0:
            comm.send(xs[rank], nxt)
            got = comm.recv(xs[rank].shape, xs[rank].dtype, prv)
        else:
            got = comm.recv(xs[rank].shape, xs[rank].dtype, prv)
            comm.send(xs[rank], nxt)
        close(got, xs[prv], 0, "send/recv")

    # expert parallel dispatch / combine, two experts per rank
    comm.num_experts = 2 * n
    T, H, topk = 64, 256, 2
    xs = per_rank(70, n, (T, H), torch.bfloat16)
    ids, ws = [], []
    for r in range(n):
        gg = torch.Generator(device="cuda").manual_seed(7000 + r)
        p = torch.softmax(torch.randn(T, 2 * n, device="cuda", generator=gg), -1)
        w, i = torch.topk(p, topk, -1)
        ids.append(i.to(torch.int32))
        ws.append(w.float())
    recv_x, recv_w, recv_ids = comm.dispatch(xs[rank], ws[rank], ids[rank])
    expect_rows = sum(int(((i // 2) == rank).sum()) for i in ids)
    assert recv_x.shape[0] == expect_rows, (recv_x.shape, expect_rows)
    assert bool(((recv_ids // 2) == rank).all())
    out = comm.combine(recv_x.contiguous())
    ref = sum((quantize_dequantize_reference(xs[rank]).float() * ws[rank][:, k:k + 1]) for k in range(topk))
    close(out, ref, 2e-2, "dispatch/combine")

    # the reference's end-to-end TP layer: column-parallel W1 + GELU, row-parallel
    # W2 + all_reduce, LM head all_gather along the vocabulary
    HIDDEN, FFN, VOCAB, BATCH = 64, 128, 96, 5
    gg = torch.Generator(device="cuda").manual_seed(123)
    x = torch.randn(BATCH, HIDDEN, device="cuda", generator=gg)
    w1 = torch.randn(FFN, HIDDEN, device="cuda", generator=gg) * 0.1
    w2 = torch.randn(HIDDEN, FFN, device="cuda", generator=gg) * 0.1
    lm = torch.randn(VOCAB, HIDDEN, device="cuda", generator=gg) * 0.1
    f, v = FFN // n, VOCAB // n
    h = torch.nn.functional.gelu(x @ w1[rank * f:(rank + 1) * f].T)
    y = comm.all_reduce((h @ w2[:, rank * f:(rank + 1) * f].T).contiguous()) + x
    logits = comm.all_gather((y @ lm[rank * v:(rank + 1) * v].T).contiguous(), dim=-1)
    y_ref = torch.nn.functional.gelu(x @ w1.T) @ w2.T + x
    close(y, y_ref, 1e-4, "e2e tp hidden")
    close(logits, y_ref @ lm.T, 1e-4, "e2e tp logits")

    comm.destroy()
    dist.destroy_process_group()
    print(f"rank {rank}: torch_comm ok", flush=True)


if __name__ == "__main__":
    main()
