// SPDX-License-Identifier: Apache-2.0
// Logging and error propagation.
//
// Behaviour follows the reference's logger (reference: src/util/log.h:11-43):
// level from VCCL_DEBUG=NONE|ERROR|WARN|INFO|TRACE (default WARN), lines on
// stderr as "vccl [pid] LEVEL: msg", and the text of the calling thread's
// latest ERROR kept for vcclGetLastError.
#pragma once

#include "vccl.h"

namespace vccl {

enum class Level : int { None = 0, Error = 1, Warn = 2, Info = 3, Trace = 4 };

Level currentLevel();
void emit(Level lv, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
const char* threadLastError();
void setThreadLastError(const char* msg);

}  // namespace vccl

#define VLOG_AT(lv, ...)                                   \
  do {                                                     \
    if (static_cast<int>(::vccl::currentLevel()) >=        \
        static_cast<int>(::vccl::Level::lv))               \
      ::vccl::emit(::vccl::Level::lv, __VA_ARGS__);        \
    else if (::vccl::Level::lv == ::vccl::Level::Error)    \
      ::vccl::emit(::vccl::Level::None, __VA_ARGS__);      \
  } while (0)

#define VERR(...) VLOG_AT(Error, __VA_ARGS__)
#define VWARN(...) VLOG_AT(Warn, __VA_ARGS__)
#define VINFO(...) VLOG_AT(Info, __VA_ARGS__)
#define VTRACE(...) VLOG_AT(Trace, __VA_ARGS__)

// Return early with the failing result code.
#define VTRY(expr)                                                        \
  do {                                                                    \
    vcclResult_t vtry_res_ = (expr);                                      \
    if (vtry_res_ != vcclSuccess) {                                       \
      VTRACE("%s:%d: %s -> %s", __FILE__, __LINE__, #expr,                \
             vcclGetErrorString(vtry_res_));                              \
      return vtry_res_;                                                   \
    }                                                                     \
  } while (0)
