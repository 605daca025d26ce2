// SPDX-License-Identifier: Apache-2.0
// Measured algorithm tables (VCCL_TUNING_FILE): parsing and rule lookup,
// on the host.
#include <cstdio>
#include <string>

#include "runtime/tuning.h"

using namespace vccl;

namespace {
int gFail = 0;
#define EXPECT(c, ...)                                          \
  do {                                                          \
    if (!(c)) {                                                 \
      std::fprintf(stderr, "FAIL %s:%d: ", __FILE__, __LINE__); \
      std::fprintf(stderr, __VA_ARGS__);                        \
      std::fprintf(stderr, "\n");                               \
      gFail++;                                                  \
    }                                                           \
  } while (0)
}  // namespace

int main() {
  const std::string text =
      "# op ranks max_bytes algorithm\n"
      "allreduce 8 262144 ll\n"
      "allreduce 8 4194304 ll2   # trailing comment\n"
      "allreduce 0 0 twoshot\n"
      "\n"
      "broadcast 8 0 nvls\n"
      "allreduce eight 1 ll\n"          // malformed: ignored
      "allreduce 2 1024 ll extra\n";    // malformed: ignored
  const auto rules = parseTuning(text);
  EXPECT(rules.size() == 4, "parsed %zu rules", rules.size());
  EXPECT(tunedAlgorithm(rules, "allreduce", 8, 1024) == "ll", "small 8-rank all-reduce");
  EXPECT(tunedAlgorithm(rules, "allreduce", 8, 262144) == "ll", "boundary is inclusive");
  EXPECT(tunedAlgorithm(rules, "allreduce", 8, 262145) == "ll2", "next rule");
  EXPECT(tunedAlgorithm(rules, "allreduce", 8, 1 << 30) == "twoshot", "catch-all");
  EXPECT(tunedAlgorithm(rules, "allreduce", 4, 1024) == "twoshot", "rank count must match");
  EXPECT(tunedAlgorithm(rules, "broadcast", 8, 1 << 30) == "nvls", "0 bytes means no limit");
  EXPECT(tunedAlgorithm(rules, "broadcast", 2, 1024).empty(), "no rule");
  EXPECT(tunedAlgorithm(rules, "allgather", 8, 1024).empty(), "other op");
  EXPECT(loadTuningFile("/nonexistent/vccl-tuning").empty(), "missing file");
  std::printf("tuning: %s\n", gFail == 0 ? "OK" : "FAIL");
  return gFail == 0 ? 0 : 1;
}
