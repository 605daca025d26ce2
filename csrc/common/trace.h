// SPDX-License-Identifier: Apache-2.0
// Observability: NVTX ranges around every collective and fused-op launch
// (VCCL_NVTX=1; header-only NVTX v3, free when no profiler is attached) and
// an INFO log line the first time each (operation, algorithm, rank count) is
// chosen.  The reference's only tracing is per-step timing inside its verbs
// transport (reference: src/transport/verbs.cc:57-91).
#pragma once

#include <nvtx3/nvToolsExt.h>

#include <cstddef>

namespace vccl {

bool nvtxEnabled();

class TraceRange {
 public:
  explicit TraceRange(const char* name) : on_(nvtxEnabled()) {
    if (on_) nvtxRangePushA(name);
  }
  ~TraceRange() {
    if (on_) nvtxRangePop();
  }
  TraceRange(const TraceRange&) = delete;
  TraceRange& operator=(const TraceRange&) = delete;

 private:
  bool on_;
};

// Logs "<op>: <algo> (n ranks, first at <bytes> bytes)" once per triple.
void noteAlgorithm(const char* op, const char* algo, int nranks, size_t bytes);

}  // namespace vccl
