# SPDX-License-Identifier: Apache-2.0
"""Bucketed gradient all-reduce for data parallelism.

Gradients are packed (in reverse parameter order, the order backward
produces them) into flat buckets of about `bucket_bytes`, one dtype per
bucket; each bucket is all-reduced with the average (or a PreMulSum scale)
and unpacked.  The reference offers the primitives (avg, PreMulSum;
reference: src/core/collectives.cc:85-98, src/core/comm.cc:264-319) and
leaves bucketing to the caller; on NVLink, buckets of a few MiB keep each
all-reduce on the bandwidth-optimal algorithm while bounding launch count.

On CUDA the buckets are views of one buffer that every rank registers as a
window (the bucket plan, hence every offset, is the same on every rank), so
each bucket's all-reduce runs in place on the peers' buffers instead of
staging through the library's workspace.  `close()` deregisters it
(collective, like the registration on the first all_reduce).
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

    def __init__(self, comm, params: Sequence[torch.nn.Parameter], bucket_bytes: int = 16 << 20,
                 use_window: bool = True):
        self.comm = comm
        self.params = [p for p in params if p.requires_grad]
        self.plan = plan_buckets([p.numel() for p in self.params], [p.dtype for p in self.params], bucket_bytes)
        self._flat: Dict[int, torch.Tensor] = {}
        self.use_window = use_window
        self._window = None  # (backing uint8 tensor, handle)

    def _window_buffers(self, device: torch.device) -> None:
        """One registered buffer holding every bucket (256-byte aligned views)."""
        from vkccl_b200.comm import mem_alloc_tensor

        offsets, total = [], 0
        for idx in self.plan:
            p0 = self.params[idx[0]]
            nbytes = sum(self.params[i].numel() for i in idx) * p0.element_size()
            offsets.append((total, nbytes, p0.dtype))
            total += (nbytes + 255) // 256 * 256
        backing = mem_alloc_tensor((max(total, 256),), torch.uint8, device=device)
        handle = self.comm.window_register(backing)
        for b, (off, nbytes, dt) in enumerate(offsets):
            self._flat[b] = backing[off:off + nbytes].view(dt)
        self._window = (backing, handle)

    def close(self) -> None:
        """Deregister the bucket window (collective: every rank calls it)."""
        if self._window is not None:
            self.comm.window_deregister(self._window[1])
            self._window = None
            self._flat.clear()

    def all_reduce(self, premul: float = 0.0) -> None:
        """Average gradients; with premul != 0, sum of premul * grad instead."""
        from vkccl_b200.comm import DataType, RedOp
        from vkccl_b200.torch_comm import vccl_dtype

        dev = self.params[0].device if self.params else torch.device("cpu")
        if (self.use_window and self._window is None and dev.type == "cuda"
                and hasattr(self.comm, "window_register")):
            self._window_buffers(dev)
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
