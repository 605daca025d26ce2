/* SPDX-License-Identifier: Apache-2.0
 * Diagnostic entry points of vkccl-b200 (not part of the reference API).
 * They synchronise the device and are meant for tools, tests and debugging,
 * not for the hot path. */
#ifndef VCCL_X_H_
#define VCCL_X_H_

#include "vccl.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Cross-GPU barrier latency: `iters` back-to-back block barriers over
 * `nblocks` blocks in one kernel, signalling variant `variant` (0: fence +
 * relaxed store / relaxed poll + fence, 1: release store / acquire poll,
 * 2: volatile store / poll, a timing floor only).  Every rank calls it with
 * the same arguments; *usPerBarrier receives the time per barrier. */
vcclResult_t vcclxBarrierBench(vcclComm_t comm, int iters, int nblocks, int variant, float* usPerBarrier);

/* Per-CTA event times (ns, %globaltimer) of the fused kernels, recorded when
 * the communicator was created with VCCL_FUSED_TRACE=1: *ctas rows of 32
 * slots.  Slots 0-18: the last all-gather + GEMM; 20-27: the last GEMM +
 * reduce-scatter.  vcclInvalidUsage without tracing. */
vcclResult_t vcclxFusedTrace(vcclComm_t comm, unsigned long long* out, int* ctas);

/* Bytes of this rank's guard regions (VCCL_GUARDS=1 at communicator
 * creation) no longer holding their fill pattern: out-of-bounds writes by
 * some kernel.  vcclInvalidUsage without guards. */
vcclResult_t vcclxCheckGuards(vcclComm_t comm, unsigned long long* badBytes);

/* Sets, from the host, the abort word of vcclGemmBf16NoAlloc on `device`:
 * the state a launch that abandoned its tiles (a pipeline wait ran out)
 * leaves behind.  The next vcclGemmBf16NoAlloc call on that device returns
 * vcclInternalError and clears it.  For tests of that error path. */
vcclResult_t vcclxNoAllocInjectAbort(int device);

/* The call profile of a communicator created with VCCL_PROF=1: one line per
 * (operation, algorithm or path) this rank ran, collectives and the fused
 * calls of vccl_tp.h alike, "op\talgorithm\tcalls\tbytes\n", bytes being
 * count x type size for collectives and the activation bytes (M x N or
 * M x K or T x H, bf16) for fused calls, summed over the calls.  The same lines are
 * printed to stderr when the communicator is destroyed.  Empty without
 * VCCL_PROF; vcclInvalidArgument when `len` is too small (the text is then
 * cut off). */
vcclResult_t vcclxProfSummary(vcclComm_t comm, char* buf, size_t len);

#ifdef __cplusplus
}
#endif

#endif /* VCCL_X_H_ */
