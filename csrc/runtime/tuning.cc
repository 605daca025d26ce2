// SPDX-License-Identifier: Apache-2.0
#include "runtime/tuning.h"

#include <fstream>
#include <sstream>

#include "common/log.h"

namespace vccl {

std::vector<TuningRule> parseTuning(const std::string& text) {
  std::vector<TuningRule> rules;
  std::istringstream in(text);
  std::string line;
  int lineNo = 0;
  while (std::getline(in, line)) {
    lineNo++;
    const size_t hash = line.find('#');
    if (hash != std::string::npos) line.resize(hash);
    std::istringstream fields(line);
    TuningRule r;
    long long ranks = -1, bytes = -1;
    if (!(fields >> r.op)) continue;  // blank or comment
    std::string extra;
    if (!(fields >> ranks >> bytes >> r.algo) || (fields >> extra) || ranks < 0 || bytes < 0) {
      VWARN("tuning file line %d ignored: expected '<op> <ranks> <max_bytes> <algorithm>'", lineNo);
      continue;
    }
    r.nranks = static_cast<int>(ranks);
    r.maxBytes = static_cast<size_t>(bytes);
    rules.push_back(r);
  }
  return rules;
}

std::vector<TuningRule> loadTuningFile(const char* path) {
  std::ifstream f(path);
  if (!f) {
    VWARN("cannot read tuning file %s", path);
    return {};
  }
  std::stringstream ss;
  ss << f.rdbuf();
  std::vector<TuningRule> rules = parseTuning(ss.str());
  VINFO("tuning file %s: %zu rules", path, rules.size());
  return rules;
}

std::string tunedAlgorithm(const std::vector<TuningRule>& rules, const char* op, int nranks, size_t bytes) {
  for (const TuningRule& r : rules) {
    if (r.op != op) continue;
    if (r.nranks != 0 && r.nranks != nranks) continue;
    if (r.maxBytes != 0 && bytes > r.maxBytes) continue;
    return r.algo;
  }
  return std::string();
}

}  // namespace vccl
