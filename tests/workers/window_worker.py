# SPDX-License-Identifier: Apache-2.0
"""Per-rank body of the window GPU test (run by torchrun): torch tensors on
vcclMemAlloc memory and from PyTorch's allocator, registered as windows,
through all-reduce, all-gather and reduce-scatter, and GradBuckets on its
registered bucket buffer, against locally computed results."""

import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))

import vkccl_b200 as v  # noqa: E402


def main():
    dist.init_process_group("gloo")
    rank, n = dist.get_rank(), dist.get_world_size()
    torch.cuda.set_device(rank)
    uid = [v.get_unique_id().to_bytes() if rank == 0 else None]
    dist.broadcast_object_list(uid, 0)
    comm = v.Communicator(n, v.UniqueId.from_bytes(uid[0]), rank, cuda_device=rank)
    count = 3 << 20  # past every LL threshold
    send = v.mem_alloc_tensor((count,), torch.bfloat16)
    recv = v.mem_alloc_tensor((count,), torch.bfloat16)
    ws = comm.window_register(send)
    wr = comm.window_register(recv)

    def inputs(r):
        g = torch.Generator(device="cuda").manual_seed(100 + r)
        return torch.randn(count, device="cuda", generator=g).bfloat16()

    total = sum(inputs(r).float() for r in range(n))
    send.copy_(inputs(rank))
    comm.all_reduce(send, recv)
    torch.cuda.synchronize()
    err = (recv.float() - total).abs().max().item()
    assert err <= 0.05 * total.abs().max().item(), f"window all_reduce err {err}"

    per = count // n
    comm.all_gather(send[:per], recv[: per * n])
    torch.cuda.synchronize()
    for r in range(n):
        assert torch.equal(recv[r * per:(r + 1) * per], inputs(r)[:per]), f"window all_gather block {r}"

    out = torch.empty(per, dtype=torch.bfloat16, device="cuda")
    comm.reduce_scatter(send[: per * n], out)
    torch.cuda.synchronize()
    want = total[rank * per:(rank + 1) * per]
    err = (out.float() - want).abs().max().item()
    assert err <= 0.05 * want.abs().max().item(), f"window reduce_scatter err {err}"

    # broadcast from the last rank into the receive window
    if rank == n - 1:
        recv[:per].copy_(inputs(rank)[:per])
    comm.broadcast(recv[:per], n - 1)  # in place
    torch.cuda.synchronize()
    assert torch.equal(recv[:per], inputs(n - 1)[:per]), "window broadcast"

    # all-to-all with equal blocks into the receive window
    comm.all_to_all(send[: per * n], recv[: per * n])
    torch.cuda.synchronize()
    for r in range(n):
        assert torch.equal(recv[r * per:(r + 1) * per], inputs(r)[rank * per:(rank + 1) * per]), f"all_to_all {r}"

    comm.window_deregister(ws)
    comm.window_deregister(wr)
    del send, recv

    # a tensor from PyTorch's own allocator (cudaMalloc): a window through CUDA IPC
    both = torch.empty(2 * count, dtype=torch.bfloat16, device="cuda")
    with comm.window(both):
        both[:count].copy_(inputs(rank))
        comm.all_reduce(both[:count], both[count:])
        torch.cuda.synchronize()
    err = (both[count:].float() - total).abs().max().item()
    assert err <= 0.05 * total.abs().max().item(), f"cudaMalloc window all_reduce err {err}"

    # data-parallel gradient buckets on one registered buffer
    from vkccl_b200.parallel import GradBuckets

    sizes = [1 << 20, 4099, 3 << 18, 77]
    params = [torch.nn.Parameter(torch.zeros(s, device="cuda")) for s in sizes]

    def grads(r):
        g = torch.Generator(device="cuda").manual_seed(500 + r)
        return [torch.randn(s, device="cuda", generator=g) for s in sizes]

    for p, g in zip(params, grads(rank)):
        p.grad = g
    gb = GradBuckets(comm, params, bucket_bytes=2 << 20)
    gb.all_reduce()
    torch.cuda.synchronize()
    assert gb._window is not None
    mean = [sum(gs) / n for gs in zip(*[grads(r) for r in range(n)])]
    for p, m in zip(params, mean):
        torch.testing.assert_close(p.grad, m, rtol=1e-5, atol=1e-6)
    gb.close()
    comm.destroy()
    dist.destroy_process_group()
    print(f"rank {rank}: window ok", flush=True)


if __name__ == "__main__":
    main()
