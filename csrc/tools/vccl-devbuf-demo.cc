// SPDX-License-Identifier: Apache-2.0
// vccl-devbuf-demo: all-gather inside externally exported device memory.
//
// Headless counterpart of the reference's Vulkan demo (reference:
// bench/vccl_vk_demo.cc:176-223), which exports device memory as an fd,
// registers it with vcclCommRegisterDmaBuf and all-gathers 1 Mi floats per
// rank inside it.  No graphics API is available on these machines, so the
// exporter here is the CUDA virtual memory API (cuMemCreate +
// cuMemExportToShareableHandle, POSIX fd); the registration and collective
// path is the same.  The fill and check are the demo's own arithmetic.
//
//   vccl-devbuf-demo --launch N
#include <cuda.h>
#include <cuda_runtime.h>
#include <sys/wait.h>
#include <unistd.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "vccl.h"

namespace {

template <typename F>
F entry(const char* name, int ver) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q{};
  cudaGetDriverEntryPointByVersion(name, &p, ver, cudaEnableDefault, &q);
  return reinterpret_cast<F>(p);
}

int runRank(int rank, int n, const vcclUniqueId& id) {
  cudaSetDevice(rank);
  cudaFree(nullptr);
  constexpr size_t kCount = 1 << 20;  // floats per rank
  auto memCreate = entry<decltype(&cuMemCreate)>("cuMemCreate", 10020);
  auto memExport = entry<decltype(&cuMemExportToShareableHandle)>("cuMemExportToShareableHandle", 10020);
  auto memGran = entry<decltype(&cuMemGetAllocationGranularity)>("cuMemGetAllocationGranularity", 10020);
  auto memRelease = entry<decltype(&cuMemRelease)>("cuMemRelease", 10020);
  CUmemAllocationProp prop;
  std::memset(&prop, 0, sizeof(prop));
  prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  prop.location.id = rank;
  prop.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  size_t gran = 0;
  memGran(&gran, &prop, CU_MEM_ALLOC_GRANULARITY_MINIMUM);
  const size_t bytes = (kCount * sizeof(float) * (n + 1) + gran - 1) / gran * gran;
  CUmemGenericAllocationHandle h = 0;
  int fd = -1;
  if (memCreate(&h, bytes, &prop, 0) != CUDA_SUCCESS ||
      memExport(&fd, h, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0) != CUDA_SUCCESS) {
    std::fprintf(stderr, "rank %d: exportable allocation failed\n", rank);
    return 1;
  }
  vcclComm_t comm = nullptr;
  if (vcclCommInitRank(&comm, n, id, rank) != vcclSuccess) return 1;
  void* ptr = nullptr;
  vcclMemHandle_t reg = nullptr;
  if (vcclCommRegisterDmaBuf(comm, fd, 0, bytes, &ptr, &reg) != vcclSuccess) {
    std::fprintf(stderr, "rank %d: registration failed: %s\n", rank, vcclGetLastError(comm));
    return 1;
  }
  close(fd);
  float* send = static_cast<float*>(ptr);
  float* recv = send + kCount;
  std::vector<float> host(kCount);
  for (size_t i = 0; i < kCount; i++) host[i] = static_cast<float>(rank * 7 + static_cast<int>(i % 13));
  cudaMemcpy(send, host.data(), kCount * sizeof(float), cudaMemcpyHostToDevice);
  if (vcclAllGather(send, recv, kCount, vcclFloat32, comm) != vcclSuccess) return 1;
  std::vector<float> all(kCount * n);
  cudaMemcpy(all.data(), recv, all.size() * sizeof(float), cudaMemcpyDeviceToHost);
  size_t bad = 0;
  for (int r = 0; r < n; r++)
    for (size_t i = 0; i < kCount; i++)
      if (all[r * kCount + i] != static_cast<float>(r * 7 + static_cast<int>(i % 13))) bad++;
  vcclCommDeregister(comm, reg);
  vcclCommDestroy(comm);
  memRelease(h);
  std::printf("rank %d: all-gather of %zu MiB in exported device memory: %s\n", rank,
              kCount * sizeof(float) * n >> 20, bad ? "FAIL" : "OK");
  return bad ? 1 : 0;
}

}  // namespace

int main(int argc, char** argv) {
  setvbuf(stdout, nullptr, _IOLBF, 0);
  int launch = 2;
  for (int i = 1; i + 1 < argc; i++)
    if (std::strcmp(argv[i], "--launch") == 0) launch = std::atoi(argv[i + 1]);
  setenv("VCCL_SOCKET_ADDR", "127.0.0.1", 0);
  vcclUniqueId id;
  if (vcclGetUniqueId(&id) != vcclSuccess) return 1;
  std::vector<pid_t> pids;
  for (int r = 0; r < launch; r++) {
    pid_t p = fork();
    if (p == 0) _exit(runRank(r, launch, id));
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
