# SPDX-License-Identifier: Apache-2.0
"""Sequence-parallel linear layers on the fused kernels.

ColumnParallelLinear: input rows sharded over ranks ([T/n, K] per rank),
weight rows sharded ([N/n, K]); y = AllGather(x) W^T, optionally followed by
silu(gate) * up with W holding interleaved gate/up rows.  One kernel
(all-gather pulled inside the tcgen05 GEMM; LL gather + split-K GEMM for
short inputs).

RowParallelLinear: input columns sharded ([T, K/n] per rank), weight columns
sharded ([N, K/n]); y_shard = ReduceScatter(x W^T) along rows ([T/n, N]).
The GEMM epilogue pushes tiles to their owners over NVLink.
"""

from __future__ import annotations

from typing import Optional

import torch

from vkccl_b200.ops.fused import all_gather_gemm, gemm_reduce_scatter
from vkccl_b200.ops.gemm import interleave_gate_up


class ColumnParallelLinear:
    def __init__(self, comm, weight: torch.Tensor, up_weight: Optional[torch.Tensor] = None):
        """weight: this rank's [N/n, K] rows; with up_weight the layer computes
        silu(x W^T) * (x U^T) and the two are stored interleaved."""
        self.comm = comm
        self.silu_mul = up_weight is not None
        self.weight = interleave_gate_up(weight, up_weight) if self.silu_mul else weight.contiguous()

    def __call__(self, x_shard: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        return all_gather_gemm(self.comm, x_shard, self.weight, silu_mul=self.silu_mul, out=out)


class RowParallelLinear:
    def __init__(self, comm, weight: torch.Tensor):
        """weight: this rank's [N, K/n] columns."""
        self.comm = comm
        self.weight = weight.contiguous()

    def __call__(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        return gemm_reduce_scatter(self.comm, x, self.weight, out=out)
