/* SPDX-License-Identifier: Apache-2.0
 *
 * vccl-b200 fused tensor-parallel operations (additions; no counterpart in
 * the reference C API).
 *
 * All calls are stream-ordered, take device pointers, and use bf16 row-major
 * tensors unless stated.  Weights follow torch.nn.Linear: W[out, in].
 */
#ifndef VCCL_TP_H_
#define VCCL_TP_H_

#include "vccl.h"

#ifdef __cplusplus
extern "C" {
#endif

/* C[M,N] = A[M,K] * W[N,K]^T on tcgen05 tensor cores (K % 8 == 0,
 * N % 16 == 0, 16-byte aligned pointers). */
vcclResult_t vcclGemmBf16(const void* A, const void* W, void* C, int M, int N, int K, vcclStream_t stream);

/* vcclGemmBf16 for callers that must not allocate device memory (no
 * counterpart in the reference).  Same arguments and results; the split-K
 * scratch of decode shapes lives in one fixed 8 MiB device array and the
 * abort word in a static host page instead of allocations.  A shape whose
 * split-K partials need more than 8 MiB returns vcclInvalidArgument.  The
 * first call on each device does set-up (resolves the array's address,
 * loads its module, maps the abort page); make it at start-up, before
 * device memory is reserved and before any stream capture.  A launch that
 * abandoned its tiles makes the next call return vcclInternalError.  Calls
 * that may overlap in time on one device (different streams or host
 * threads) share the array and race; calls on one stream are safe. */
vcclResult_t vcclGemmBf16NoAlloc(const void* A, const void* W, void* C, int M, int N, int K, vcclStream_t stream);

/* H[M,N/2] = silu(A W_g^T) * (A W_u^T), with W[N,K] holding gate and up rows
 * interleaved in groups of 16 (vcclInterleaveGateUp layout). */
vcclResult_t vcclGemmSiluMul(const void* A, const void* W, void* H, int M, int N, int K, vcclStream_t stream);

/* out = RMSNorm(residual + AllReduce(partial)) * weight, and residual is
 * updated in place to residual + AllReduce(partial).  Shapes [rows, hidden]. */
vcclResult_t vcclAllReduceAddRMSNorm(const void* partial, void* residual, const void* weight, void* out,
                                     size_t rows, size_t hidden, float eps, vcclDataType_t datatype,
                                     vcclComm_t comm, vcclStream_t stream);

/* Row-parallel GEMM fused with reduce-scatter over the communicator:
 * every rank computes P = A[M,K] W[N,K]^T, rows of P are owned by rank
 * (row / (M / nranks)); out[M/nranks, N] = sum over ranks of the owned rows.
 * Tiles are pushed to their owner over NVLink from the GEMM epilogue; with
 * M / nranks a multiple of 256 the owner's own tiles add the pushed ones in
 * the same kernel, otherwise a second kernel sums them.  Calls
 * with at most VCCL_FUSED_SMALL_M rows (default 512) run as a (split-K)
 * GEMM into scratch followed by the LL or push reduce-scatter.  Every rank
 * calls with the same M, N, K; M % nranks == 0, N % 16 == 0, K % 8 == 0. */
vcclResult_t vcclGemmReduceScatter(const void* A, const void* W, void* out, int M, int N, int K,
                                   vcclComm_t comm, vcclStream_t stream);

/* All-gather fused into a column-parallel GEMM: X_shard[M/nranks, K] per
 * rank, out = AllGather(X)[M,K] W[N,K]^T.  With siluMul != 0 the epilogue
 * applies silu(gate)*up (W interleaved as for vcclGemmSiluMul; out has N/2
 * columns).  Remote shards are pulled into local memory by copy warps while
 * the tensor cores work on the shards already present.  Calls with at most
 * VCCL_FUSED_SMALL_M rows run as an LL all-gather into scratch followed by a
 * (split-K) GEMM. */
vcclResult_t vcclAllGatherGemm(const void* xShard, const void* W, void* out, int M, int N, int K, int siluMul,
                               vcclComm_t comm, vcclStream_t stream);

/* Expert-parallel MoE dispatch with fp8 e4m3 1x128 block quantisation.
 * x[T,H] bf16, topkIds[T,topk] int32 (global expert ids), topkW[T,topk] f32,
 * experts split evenly over ranks.  Rows cross NVLink as e4m3 with one f32
 * scale (amax / 448) per 128 elements; recvX receives them dequantised to
 * bf16, the rows this rank's experts must process, in (source rank, token, k)
 * order; recvMeta[i] = {source rank, source token, k, local expert},
 * recvW[i] its routing weight; *recvCount is written on the device.
 * capacity bounds the rows a rank receives (and T * topk <= capacity); rows
 * past it are dropped and reported as an error.  Every rank passes the same
 * H, topk, numExperts and capacity.  H % 128 == 0, topk <= 8. */
vcclResult_t vcclMoeDispatchFp8(const void* x, const int* topkIds, const float* topkW, void* recvX, int* recvMeta,
                                float* recvW, int* recvCount, int T, int H, int topk, int numExperts, int capacity,
                                vcclComm_t comm, vcclStream_t stream);

/* Inverse of dispatch: expertOut[rows,H] (bf16, in the received row order)
 * is scaled by recvW on the expert rank, travels back to the source ranks,
 * and out[T,H] = sum_k topkW[t,k] * expertOut(t,k).  One combine per
 * dispatch. */
vcclResult_t vcclMoeCombine(const void* expertOut, const int* recvMeta, const float* recvW, const int* recvCount,
                            void* out, int T, int H, int topk, int capacity, vcclComm_t comm,
                            vcclStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* VCCL_TP_H_ */
