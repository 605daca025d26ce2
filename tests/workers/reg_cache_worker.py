# SPDX-License-Identifier: Apache-2.0
"""Per-rank body of the registration-cache GPU test (run by torchrun with
VCCL_REG_CACHE=1): collectives on plain PyTorch tensors register their
buffers as windows on first use and reuse them afterwards, a slice at one
offset reuses its tensor's window, a captured call stays on the staged
kernels, and a flush drops everything; every result is checked against
locally computed values and the cache counters against the expected
hits and registrations."""

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
    count = 3 << 20  # 6 MiB of bf16: past every LL threshold and VCCL_REG_CACHE_MIN

    def inputs(r, salt=0):
        g = torch.Generator(device="cuda").manual_seed(100 + r + 17 * salt)
        return torch.randn(count, device="cuda", generator=g).bfloat16()

    def close(got, want, what):
        err = (got.float() - want).abs().max().item()
        assert err <= 0.05 * want.abs().max().item(), f"{what}: err {err}"

    send = torch.empty(count, dtype=torch.bfloat16, device="cuda")
    recv = torch.empty(count, dtype=torch.bfloat16, device="cuda")
    assert comm.reg_cache_stats()["entries"] == 0

    # all-reduce twice: registered on the first call, reused on the second
    for salt in (0, 1):
        send.copy_(inputs(rank, salt))
        comm.all_reduce(send, recv)
        torch.cuda.synchronize()
        close(recv, sum(inputs(r, salt).float() for r in range(n)), f"all_reduce {salt}")
    st = comm.reg_cache_stats()
    assert st["misses"] == 2 and st["hits"] == 2 and st["entries"] == 2, st

    # all-gather into the cached receive tensor, reduce-scatter from the cached send tensor
    per = count // n
    send.copy_(inputs(rank))
    comm.all_gather(send[:per], recv[: per * n])
    torch.cuda.synchronize()
    for r in range(n):
        assert torch.equal(recv[r * per:(r + 1) * per], inputs(r)[:per]), f"all_gather block {r}"
    out = torch.empty(per, dtype=torch.bfloat16, device="cuda")
    comm.reduce_scatter(send[: per * n], out)
    torch.cuda.synchronize()
    total = sum(inputs(r).float() for r in range(n))
    close(out, total[rank * per:(rank + 1) * per], "reduce_scatter")
    st = comm.reg_cache_stats()
    assert st["misses"] == 2 and st["hits"] == 4, st

    # a slice at one offset on every rank reuses the tensor's window
    half = count // 2
    comm.all_reduce(send[half:], recv[half:])
    torch.cuda.synchronize()
    close(recv[half:], total[half:], "all_reduce on slices")
    st = comm.reg_cache_stats()
    assert st["misses"] == 2 and st["hits"] == 6, st

    # a call captured in a CUDA graph stays on the staged kernels
    calls_before = st["calls"]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            comm.all_reduce(send, recv)
    torch.cuda.current_stream().wait_stream(s)
    recv.zero_()
    graph.replay()
    torch.cuda.synchronize()
    close(recv, total, "captured all_reduce")
    st = comm.reg_cache_stats()
    assert st["calls"] == calls_before and st["hits"] == 6, st
    del graph

    # flush (collective) before memory goes back to CUDA, then register afresh
    comm.reg_cache_flush()
    st = comm.reg_cache_stats()
    assert st["entries"] == 0 and st["evictions"] == 2, st
    del send, recv, out
    torch.cuda.empty_cache()
    a = inputs(rank, 2)
    b = torch.empty_like(a)
    comm.all_reduce(a, b)
    torch.cuda.synchronize()
    close(b, sum(inputs(r, 2).float() for r in range(n)), "all_reduce after flush")
    st = comm.reg_cache_stats()
    assert st["misses"] == 4 and st["entries"] == 2, st

    err = comm.async_error()
    comm.reg_cache_flush()  # collective: no rank frees memory a peer still has open
    comm.destroy()
    dist.destroy_process_group()
    if err:
        raise AssertionError(f"async error {err}")
    print(f"rank {rank}: reg cache ok", flush=True)


if __name__ == "__main__":
    main()
