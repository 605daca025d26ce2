// SPDX-License-Identifier: Apache-2.0
// Work splits shared by the collective kernels and their host-side index
// tests (csrc/tests/test_coll_index.cc): which bytes or elements a block, a
// round or a rank's chunk covers.
#pragma once

#include <stddef.h>

namespace vccl {
namespace dev {

// Part `idx` of `parts` of [0, total), each part a multiple of `align`.
__host__ __device__ __forceinline__ void blockRange(size_t total, int parts, int idx, size_t align, size_t* lo,
                                                    size_t* hi) {
  size_t per = (total + parts - 1) / parts;
  per = (per + align - 1) / align * align;
  size_t a = per * static_cast<size_t>(idx);
  *lo = a < total ? a : total;
  size_t b = *lo + per;
  *hi = b < total ? b : total;
}

// Block `idx`'s part of a round of `m` units, split as a round of `full`
// units would be (full >= m).  Multi-round kernels split every round of a
// launch the same way, so block b only ever touches its own bytes of the
// staging region: a short last round must not hand block b bytes that a
// slower block b' (which block b never synchronises with) still reads.
__host__ __device__ __forceinline__ void roundRange(size_t full, size_t m, int parts, int idx, size_t align,
                                                    size_t* lo, size_t* hi) {
  blockRange(full, parts, idx, align, lo, hi);
  if (*hi > m) *hi = m;
  if (*lo > *hi) *lo = *hi;
}

// Per-rank chunk of the staged NVLS all-reduce, fixed for every round of a
// launch: a single round takes ceil(total / n) rounded up to 16 bytes (n
// chunks fit because the round size leaves 16 bytes per rank spare), longer
// messages full rounds of roundBytes / n rounded down to 16.
__host__ __device__ __forceinline__ size_t nvlsRoundChunk(size_t total, int n, size_t roundBytes) {
  if (total <= roundBytes) return ((total + n - 1) / n + 15) / 16 * 16;
  return roundBytes / n / 16 * 16;
}

// Per-rank chunk (units, a multiple of pk) when `count` units are split
// among n ranks (two-shot rounds, window all-reduce).
__host__ __device__ __forceinline__ size_t rankChunk(size_t count, int n, size_t pk) {
  return ((count + n - 1) / n + pk - 1) / pk * pk;
}

}  // namespace dev
}  // namespace vccl
