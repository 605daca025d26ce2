// SPDX-License-Identifier: Apache-2.0
#include "common/trace.h"

#include <mutex>
#include <set>
#include <string>
#include <tuple>

#include "common/env.h"
#include "common/log.h"

namespace vccl {

bool nvtxEnabled() {
  static const bool on = envLong("VCCL_NVTX", 0) != 0;
  return on;
}

void noteAlgorithm(const char* op, const char* algo, int nranks, size_t bytes) {
  static std::mutex mu;
  static std::set<std::tuple<std::string, std::string, int>> seen;
  std::lock_guard<std::mutex> g(mu);
  if (seen.emplace(op, algo, nranks).second)
    VINFO("%s: %s (%d ranks, first at %zu bytes)", op, algo, nranks, bytes);
}

}  // namespace vccl
