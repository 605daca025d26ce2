# SPDX-License-Identifier: Apache-2.0
"""Back-to-back stream-ordered collectives without host synchronisation.

Every call gets distinct input values, roots rotate, op kinds interleave and
sizes cross every algorithm threshold; the host only synchronises at the
end and then checks every output.  Then the same mix is captured in a CUDA
graph and replayed several times.  Catches slot-reuse races between
consecutive launches (a rank running ahead of its peers).
"""

import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))

import vkccl_b200 as v  # noqa: E402
from vkccl_b200.ops.fused import all_reduce_add_rms_norm  # noqa: E402

SIZES = [8, 1000, 16384, 65536, 262144, 1 << 20, 3 << 20]  # elements of bf16


def main():
    rank = int(os.environ["RANK"])
    n = int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    comm = v.Communicator(n, v.get_unique_id(), rank, cuda_device=rank)
    BF = int(v.DataType.BFLOAT16)

    def plan():
        """List of (kind, args, checker) for one round of calls."""
        calls = []
        it = 0
        for count in SIZES:
            for rep in range(3):
                it += 1
                base = float(it % 7)
                # all-reduce: rank r contributes (base + r) -> sum = n*base + n(n-1)/2
                x = torch.full((count,), base + rank, device="cuda", dtype=torch.bfloat16)
                y = torch.empty_like(x)
                calls.append(("ar", (x, y), n * base + n * (n - 1) / 2))
                # broadcast from a rotating root: value = 100 + root
                root = it % n
                b = torch.full((count,), 100.0 + root if rank == root else -1.0, device="cuda",
                               dtype=torch.bfloat16)
                calls.append(("bc", (b, root), 100.0 + root))
                # all-gather: block r holds (r + base)
                per = max(1, count // n)
                s = torch.full((per,), base + rank, device="cuda", dtype=torch.bfloat16)
                g = torch.empty(per * n, device="cuda", dtype=torch.bfloat16)
                calls.append(("ag", (s, g, per), base))
                # reduce-scatter: every rank contributes (base + r) everywhere
                rs_in = torch.full((per * n,), base + rank, device="cuda", dtype=torch.bfloat16)
                rs_out = torch.empty(per, device="cuda", dtype=torch.bfloat16)
                calls.append(("rs", (rs_in, rs_out, per), n * base + n * (n - 1) / 2))
        return calls

    def issue(calls):
        for kind, args, _ in calls:
            if kind == "ar":
                comm.all_reduce(args[0], args[1], dtype=BF)
            elif kind == "bc":
                comm.broadcast(args[0], args[1], dtype=BF)
            elif kind == "ag":
                comm.all_gather(args[0], args[1], sendcount=args[2], dtype=BF)
            else:
                comm.reduce_scatter(args[0], args[1], recvcount=args[2], dtype=BF)

    def check(calls, tag):
        for i, (kind, args, want) in enumerate(calls):
            if kind == "ar":
                got = args[1]
            elif kind == "bc":
                got = args[0]
            elif kind == "ag":
                got = args[1].view(n, -1) - torch.arange(n, device="cuda").view(n, 1).to(torch.bfloat16)
            else:
                got = args[1]
            ok = torch.all(got.float() == float(want)).item()
            if not ok:
                raise AssertionError(f"{tag}: call {i} ({kind}, {args[0].numel()} elems) wrong; "
                                     f"want {want}, got {got.float().unique()[:8].tolist()}")

    calls = plan()
    torch.cuda.synchronize()
    issue(calls)
    torch.cuda.synchronize()
    check(calls, "eager")

    # fused all-reduce + RMSNorm back to back
    H = 8192
    for rows in (1, 16, 128):
        outs = []
        for rep in range(5):
            p = torch.full((rows, H), 1.0 + rank + rep, device="cuda", dtype=torch.bfloat16)
            r = torch.zeros(rows, H, device="cuda", dtype=torch.bfloat16)
            w = torch.ones(H, device="cuda", dtype=torch.bfloat16)
            outs.append((all_reduce_add_rms_norm(comm, p, r, w), r, n * (1.0 + rep) + n * (n - 1) / 2))
        torch.cuda.synchronize()
        for o, r, want in outs:
            assert torch.all(r.float() == want).item(), f"norm residual rows={rows}"
            assert torch.allclose(o.float(), torch.ones_like(o.float()), atol=2e-2), f"norm out rows={rows}"

    # CUDA graph capture + replays
    calls = plan()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        issue(calls)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        issue(calls)
    for _ in range(4):
        graph.replay()
    torch.cuda.synchronize()
    check(calls, "graph")
    del graph

    err = comm.async_error()
    comm.destroy()
    if err:
        raise AssertionError(f"async error {err}")
    print(f"rank {rank}: stress ok", flush=True)


if __name__ == "__main__":
    main()
