# SPDX-License-Identifier: Apache-2.0
"""Bucketed gradient all-reduce for data parallelism.

Gradients are packed (in reverse parameter order, the order backward
produces them) into flat buckets of about `bucket_bytes`, one dtype per
bucket; each bucket is all-reduced with the average (or a PreMulSum scale)
and unpacked.  The reference offers the primitives (avg, PreMulSum;
reference: src/core/collectives.cc:85-98, src/core/comm.cc:264-319) and
leaves bucketing to the caller; on NVLink, buckets of a few MiB keep each
all-reduce on the bandwidth-optimal algorithm while bounding launch count.
"""

from __future__ import annotations

from typing import Dict, List, Sequence

import torch


def plan_buckets(sizes: Sequence[int], dtypes: Sequence[torch.dtype], bucket_bytes: int) -> List[List[int]]:
    """Group parameter indices (visited last to first) into buckets.

    A bucket holds one dtype and closes once it reaches bucket_bytes; a
    tensor larger than bucket_bytes gets a bucket of its own.
    """
    buckets: List[List[int]] = []
    cur: List[int] = []
    cur_bytes = 0
    cur_dtype = None
    for i in reversed(range(len(sizes))):
        nbytes = sizes[i] * torch.tensor([], dtype=dtypes[i]).element_size()
        if cur and (dtypes[i] != cur_dtype or cur_bytes + nbytes > bucket_bytes):
            buckets.append(cur)
            cur, cur_bytes = [], 0
        cur.append(i)
        cur_bytes += nbytes
        cur_dtype = dtypes[i]
    if cur:
        buckets.append(cur)
    return buckets


class GradBuckets:
    """All-reduce the .grad of `params` over `comm` (average by default)."""

    def __init__(self, comm, params: Sequence[torch.nn.Parameter], bucket_bytes: int = 16 << 20):
        self.comm = comm
        self.params = [p for p in params if p.requires_grad]
        self.plan = plan_buckets([p.numel() for p in self.params], [p.dtype for p in self.params], bucket_bytes)
        self._flat: Dict[int, torch.Tensor] = {}

    def all_reduce(self, premul: float = 0.0) -> None:
        """Average gradients; with premul != 0, sum of premul * grad instead."""
        from vkccl_b200.comm import DataType, RedOp
        from vkccl_b200.torch_comm import vccl_dtype

        for b, idx in enumerate(self.plan):
            grads = [self.params[i].grad for i in idx]
            if any(g is None for g in grads):
                continue
            total = sum(g.numel() for g in grads)
            flat = self._flat.get(b)
            if flat is None or flat.numel() != total:
                flat = torch.empty(total, dtype=grads[0].dtype, device=grads[0].device)
                self._flat[b] = flat
            torch.cat([g.reshape(-1) for g in grads], out=flat)
            if premul:
                op = self.comm.create_premul_sum(premul, DataType(vccl_dtype(flat)))
                self.comm.all_reduce(flat, op=op)
                self.comm.destroy_op(op)
            else:
                self.comm.all_reduce(flat, op=RedOp.AVG)
            off = 0
            for g in grads:
                g.copy_(flat[off:off + g.numel()].view_as(g))
                off += g.numel()
