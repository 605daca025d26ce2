// SPDX-License-Identifier: Apache-2.0
// Environment parsing and the watchdog budget: VCCL_TIMEOUT in seconds,
// default 60 as in the reference code (reference: src/util/deadline.h:10-56),
// plus the device-side budget derived from it.
#include "common/env.h"

#include <cstdlib>

namespace vccl {

long envLong(const char* name, long dflt) {
  const char* v = std::getenv(name);
  if (v == nullptr || *v == '\0') return dflt;
  char* end = nullptr;
  long x = std::strtol(v, &end, 10);
  return end == v ? dflt : x;
}

size_t envBytes(const char* name, size_t dflt) {
  const char* v = std::getenv(name);
  if (v == nullptr || *v == '\0') return dflt;
  char* end = nullptr;
  double x = std::strtod(v, &end);
  if (end == v || x < 0) return dflt;
  switch (*end) {
    case 'k': case 'K': x *= 1024.0; break;
    case 'm': case 'M': x *= 1024.0 * 1024.0; break;
    case 'g': case 'G': x *= 1024.0 * 1024.0 * 1024.0; break;
    default: break;
  }
  return static_cast<size_t>(x);
}

std::string envStr(const char* name, const char* dflt) {
  const char* v = std::getenv(name);
  return (v == nullptr || *v == '\0') ? std::string(dflt) : std::string(v);
}

int watchdogSeconds() { return static_cast<int>(envLong("VCCL_TIMEOUT", 60)); }

int connectWindowMs() {
  int s = watchdogSeconds();
  return (s <= 0 || s > 120) ? 120000 : s * 1000;
}

uint64_t deviceTimeoutNs() {
  long ms = envLong("VCCL_DEVICE_TIMEOUT_MS", -1);
  if (ms < 0) {
    int s = watchdogSeconds();
    // A disabled watchdog still gets a device bound: a GPU kernel that spins
    // forever would wedge the device for every other user.
    ms = (s <= 0) ? 600000L : static_cast<long>(s) * 1000L;
  }
  return static_cast<uint64_t>(ms) * 1000000ull;
}

Deadline::Deadline() : Deadline(watchdogSeconds()) {}

Deadline::Deadline(int seconds) : armed_(seconds > 0) {
  if (armed_) end_ = std::chrono::steady_clock::now() + std::chrono::seconds(seconds);
}

bool Deadline::expired() const {
  return armed_ && std::chrono::steady_clock::now() >= end_;
}

int Deadline::pollSliceMs() const {
  if (!armed_) return 1000;
  auto left = std::chrono::duration_cast<std::chrono::milliseconds>(
                  end_ - std::chrono::steady_clock::now()).count();
  if (left <= 0) return 0;
  return left > 1000 ? 1000 : static_cast<int>(left);
}

}  // namespace vccl
