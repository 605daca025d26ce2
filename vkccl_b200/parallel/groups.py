# SPDX-License-Identifier: Apache-2.0
"""Tensor- and data-parallel sub-communicators made with vcclCommSplit.

World rank r with tensor-parallel size t sits in TP group r // t (ranks
t*g .. t*g + t - 1, NVLink neighbours) at TP rank r % t, and in DP group
r % t at DP rank r // t.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple


def group_layout(world: int, rank: int, tp: int) -> Tuple[int, int, int, int]:
    """(tp_group, tp_rank, dp_group, dp_rank) of `rank`."""
    if tp < 1 or world % tp:
        raise ValueError(f"tensor-parallel size {tp} must divide world size {world}")
    return rank // tp, rank % tp, rank % tp, rank // tp


@dataclass
class ParallelGroups:
    world: object
    tp: object
    dp: Optional[object]
    tp_size: int
    dp_size: int

    @classmethod
    def build(cls, world_comm, tp_size: int) -> "ParallelGroups":
        """Collective over world_comm: every rank must call it with the same tp_size."""
        n, r = world_comm.nranks, world_comm.rank
        tg, trank, dg, drank = group_layout(n, r, tp_size)
        tp = world_comm.split(tg, trank)
        dp = world_comm.split(dg, drank) if n // tp_size > 1 else world_comm.split(-1, 0)
        return cls(world_comm, tp, dp, tp_size, n // tp_size)

    def destroy(self) -> None:
        for c in (self.tp, self.dp):
            if c is not None:
                c.destroy()
