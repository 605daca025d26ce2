# SPDX-License-Identifier: Apache-2.0
"""Sequence / context parallelism on the library's all-to-all and p2p kernels.

The reference has neither (it offers the primitives: all-to-all(v) and
grouped send/recv; reference: src/core/collectives.cc:708-740, :886-905);
these are the two standard ways to use them for long sequences.

* Ulysses: attention inputs sharded by sequence ([S/n, H, D] per rank) are
  re-sharded by heads ([S, H/n, D]) with one all-to-all, attention runs on
  full sequences for H/n heads, and a second all-to-all goes back.
* Ring attention: every rank keeps its query block and passes its key/value
  block around the ring, one neighbour exchange per step (``ring_pass``),
  so after n - 1 steps every query block has met every key/value block.

All calls are stream-ordered on torch's current stream for CUDA tensors.
"""

from __future__ import annotations

from typing import Tuple

import torch


def _vdt(t: torch.Tensor) -> int:
    from vkccl_b200.torch_comm import vccl_dtype

    return vccl_dtype(t)


def ulysses_seq_to_heads(comm, x: torch.Tensor) -> torch.Tensor:
    """[S/n, H, D] sequence shard -> [S, H/n, D] head shard (rank r keeps heads r*H/n ...)."""
    n = comm.nranks
    s_loc, h, d = x.shape
    if h % n:
        raise ValueError(f"{h} heads do not split over {n} ranks")
    hl = h // n
    # block j of the send buffer = my sequence chunk of head group j
    send = x.reshape(s_loc, n, hl, d).permute(1, 0, 2, 3).contiguous()
    recv = torch.empty_like(send)  # block i = rank i's sequence chunk of my head group
    comm.all_to_all(send, recv, count=send.numel() // n, dtype=_vdt(send))
    return recv.reshape(n * s_loc, hl, d)


def ulysses_heads_to_seq(comm, y: torch.Tensor) -> torch.Tensor:
    """Inverse of ulysses_seq_to_heads: [S, H/n, D] -> [S/n, H, D]."""
    n = comm.nranks
    s, hl, d = y.shape
    if s % n:
        raise ValueError(f"sequence length {s} does not split over {n} ranks")
    s_loc = s // n
    send = y.reshape(n, s_loc, hl, d).contiguous()  # block j = sequence chunk j of my heads
    recv = torch.empty_like(send)                   # block i = my sequence chunk of rank i's heads
    comm.all_to_all(send, recv, count=send.numel() // n, dtype=_vdt(send))
    return recv.permute(1, 0, 2, 3).reshape(s_loc, n * hl, d)


def ring_pass(comm, block: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Send `block` to rank r+1 and return the block of rank r-1 (one grouped exchange)."""
    from vkccl_b200.comm import group

    n, r = comm.nranks, comm.rank
    if out is None:
        out = torch.empty_like(block)
    if n == 1:
        out.copy_(block)
        return out
    src = block.contiguous()
    with group():
        comm.send(src, (r + 1) % n, count=src.numel(), dtype=_vdt(src))
        comm.recv(out, (r - 1) % n, count=out.numel(), dtype=_vdt(out))
    return out


def ring_schedule(n: int, rank: int) -> Tuple[int, ...]:
    """Owner of the key/value block a rank holds at each of the n ring steps."""
    return tuple((rank - s) % n for s in range(n))
