// SPDX-License-Identifier: Apache-2.0
// Measured algorithm tables: VCCL_TUNING_FILE names a text file of rules
//
//     # op        ranks  max_bytes  algorithm
//     allreduce   8      262144     ll
//     allreduce   8      4194304    ll2
//     allreduce   0      1099511627776  twoshot     (0 ranks: any rank count)
//     broadcast   8      0          pull           (0 bytes: no size limit)
//
// For a call, the first rule of its operation whose rank count matches
// (or is 0) and whose max_bytes is at least the message size (or is 0)
// names the algorithm; the built-in thresholds apply when no rule matches.
// `python -m vkccl_b200.bench.collectives --algos ... --tune-out FILE`
// writes such a file from a measured sweep.  The reference tunes with two
// environment thresholds per operation (reference:
// src/core/collectives.cc:263-271, :525-534).
#pragma once

#include <cstddef>
#include <string>
#include <vector>

namespace vccl {

struct TuningRule {
  std::string op;
  int nranks = 0;
  size_t maxBytes = 0;
  std::string algo;
};

// Parses `text` (the file's contents); malformed lines are skipped with a
// warning naming the line number.
std::vector<TuningRule> parseTuning(const std::string& text);
// Reads and parses a file; empty on error (logged).
std::vector<TuningRule> loadTuningFile(const char* path);
// The algorithm a table picks for (op, nranks, bytes), or "" if none.
std::string tunedAlgorithm(const std::vector<TuningRule>& rules, const char* op, int nranks, size_t bytes);

}  // namespace vccl
