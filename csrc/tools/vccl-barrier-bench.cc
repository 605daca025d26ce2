// SPDX-License-Identifier: Apache-2.0
// vccl-barrier-bench: per-barrier latency of the cross-GPU block barrier for
// each signalling variant and grid size.  Diagnostic tool.
//   vccl-barrier-bench --launch N
#include <cuda_runtime.h>
#include <sys/wait.h>
#include <unistd.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "vccl.h"
#include "vccl_x.h"

static int runRank(int r, int n, const vcclUniqueId& id) {
  setvbuf(stdout, nullptr, _IOLBF, 0);
  cudaSetDevice(r);
  vcclComm_t c = nullptr;
  if (vcclCommInitRank(&c, n, id, r) != vcclSuccess) return 1;
  const char* names[] = {"fence+relaxed", "release/acquire", "volatile(no order)", "release/relaxed+fence"};
  for (int v = 0; v < 4; v++) {
    for (int g : {1, 8, 32, 64}) {
      float us = 0;
      vcclxBarrierBench(c, 200, g, v, &us);  // warm
      if (vcclxBarrierBench(c, 2000, g, v, &us) != vcclSuccess) return 2;
      if (r == 0) std::printf("variant %-24s blocks %3d : %7.3f us/barrier\n", names[v], g, us);
    }
  }
  vcclCommDestroy(c);
  return 0;
}

int main(int argc, char** argv) {
  int n = 2;
  for (int i = 1; i + 1 < argc; i++)
    if (std::strcmp(argv[i], "--launch") == 0) n = std::atoi(argv[i + 1]);
  setenv("VCCL_SOCKET_ADDR", "127.0.0.1", 0);
  vcclUniqueId id;
  if (vcclGetUniqueId(&id) != vcclSuccess) return 1;
  std::vector<pid_t> pids;
  for (int r = 0; r < n; r++) {
    pid_t p = fork();
    if (p == 0) _exit(runRank(r, n, id));
    pids.push_back(p);
  }
  int bad = 0;
  for (pid_t p : pids) {
    int st = 0;
    waitpid(p, &st, 0);
    if (!WIFEXITED(st) || WEXITSTATUS(st) != 0) bad++;
  }
  return bad ? 1 : 0;
}
