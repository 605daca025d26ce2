# SPDX-License-Identifier: Apache-2.0
"""Parallelism helpers on top of the communicator and the fused kernels.

* ``groups``  – split a world communicator into tensor- and data-parallel groups
* ``layers``  – column / row parallel linear layers (sequence parallel) on the
                fused all-gather+GEMM and GEMM+reduce-scatter kernels
* ``dp``      – bucketed gradient all-reduce (average or PreMulSum scaling)

The reference ships only the primitives (all-reduce with avg / PreMulSum,
send/recv, all-to-all; reference: src/core/collectives.cc:505-555,
src/core/comm.cc:264-319); these helpers are the ways a training or serving
loop strings them together.
"""

from vkccl_b200.parallel.dp import GradBuckets, plan_buckets
from vkccl_b200.parallel.groups import ParallelGroups, group_layout
from vkccl_b200.parallel.layers import ColumnParallelLinear, RowParallelLinear

__all__ = ["ColumnParallelLinear", "GradBuckets", "ParallelGroups", "RowParallelLinear", "group_layout",
           "plan_buckets"]
