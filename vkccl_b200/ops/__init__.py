# SPDX-License-Identifier: Apache-2.0
"""Fused tensor-parallel operations on sm_100a kernels.

gemm   – tcgen05 GEMM and gate/up SiLU*mul GEMM
fused  – all-reduce + residual + RMSNorm, GEMM + reduce-scatter,
         all-gather + GEMM
moe    – expert-parallel dispatch (fp8 e4m3, 1x128 block scales) / combine
"""
