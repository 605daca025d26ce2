// SPDX-License-Identifier: Apache-2.0
// Logging: VCCL_DEBUG levels, "vccl [pid] LEVEL: msg" on stderr, and the
// thread-local text of the last error for vcclGetLastError (reference:
// src/util/log.cc:12-44, src/util/log.h:24-43).
#include "common/log.h"

#include <strings.h>
#include <unistd.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>

namespace vccl {
namespace {

Level parseLevel() {
  const char* v = std::getenv("VCCL_DEBUG");
  if (v == nullptr || *v == '\0') return Level::Warn;
  struct Named { const char* name; Level lv; };
  static const Named table[] = {{"NONE", Level::None},   {"ERROR", Level::Error},
                                {"WARN", Level::Warn},   {"INFO", Level::Info},
                                {"TRACE", Level::Trace}};
  for (const Named& n : table)
    if (strcasecmp(v, n.name) == 0) return n.lv;
  return Level::Warn;
}

thread_local char tLastError[1024];

}  // namespace

Level currentLevel() {
  static const Level lv = parseLevel();
  return lv;
}

void setThreadLastError(const char* msg) {
  std::snprintf(tLastError, sizeof(tLastError), "%s", msg ? msg : "");
}

const char* threadLastError() { return tLastError; }

// Level::None is used internally for ERROR lines whose printing is disabled:
// the text is still recorded for vcclGetLastError but nothing is written.
void emit(Level lv, const char* fmt, ...) {
  char line[1024];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(line, sizeof(line), fmt, ap);
  va_end(ap);
  if (lv == Level::Error || lv == Level::None) setThreadLastError(line);
  if (lv == Level::None) return;
  static const char* const kNames[] = {"NONE", "ERROR", "WARN", "INFO", "TRACE"};
  std::fprintf(stderr, "vccl [%d] %s: %s\n", static_cast<int>(getpid()),
               kNames[static_cast<int>(lv)], line);
}

}  // namespace vccl
