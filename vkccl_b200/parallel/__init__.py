# SPDX-License-Identifier: Apache-2.0
"""Parallelism helpers on top of the communicator and the fused kernels.

* ``groups``  – split a world communicator into tensor- and data-parallel groups
* ``layers``  – column / row parallel linear layers (sequence parallel) on the
                fused all-gather+GEMM and GEMM+reduce-scatter kernels
* ``dp``      – bucketed gradient all-reduce (average or PreMulSum scaling)
* ``sequence``– Ulysses head/sequence re-sharding (all-to-all) and the ring
                key/value exchange of ring attention (grouped send/recv)

The reference ships only the primitives (all-reduce with avg / PreMulSum,
send/recv, all-to-all; reference: src/core/collectives.cc:505-555,
src/core/comm.cc:264-319); these helpers are the ways a training or serving
loop strings them together.
"""

from vkccl_b200.parallel.dp import GradBuckets, plan_buckets
from vkccl_b200.parallel.groups import ParallelGroups, group_layout
from vkccl_b200.parallel.layers import ColumnParallelLinear, RowParallelLinear
from vkccl_b200.parallel.sequence import ring_pass, ulysses_heads_to_seq, ulysses_seq_to_heads

__all__ = ["ColumnParallelLinear", "GradBuckets", "ParallelGroups", "RowParallelLinear", "group_layout",
           "plan_buckets", "ring_pass", "ulysses_heads_to_seq", "ulysses_seq_to_heads"]
