// SPDX-License-Identifier: Apache-2.0
// Environment knobs and the watchdog deadline.
//
// VCCL_TIMEOUT (seconds, default 60 as in the reference code,
// reference: src/util/deadline.h:13-19; 0 disables) bounds every blocking
// host wait (sockets) and every device-side spin (flags, barriers).
#pragma once

#include <chrono>
#include <cstddef>
#include <cstdint>
#include <string>

namespace vccl {

long envLong(const char* name, long dflt);
size_t envBytes(const char* name, size_t dflt);  // accepts K/M/G suffixes
std::string envStr(const char* name, const char* dflt);

// Watchdog seconds; read on every call so tests may change it between comms.
int watchdogSeconds();
// Single connect() retry window in ms (watchdog capped to 120 s).
int connectWindowMs();
// Device-side spin budget in nanoseconds (VCCL_DEVICE_TIMEOUT_MS overrides).
uint64_t deviceTimeoutNs();

class Deadline {
 public:
  Deadline();
  explicit Deadline(int seconds);
  bool expired() const;
  // Milliseconds to pass to poll(): -1 = forever, else clamped to [0, 1000].
  int pollSliceMs() const;

 private:
  bool armed_;
  std::chrono::steady_clock::time_point end_;
};

}  // namespace vccl
