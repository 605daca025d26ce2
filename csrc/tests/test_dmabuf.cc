// SPDX-License-Identifier: Apache-2.0
// Registration of dmabuf file descriptors, with collectives inside the
// mapping (reference: tests/test_dmabuf.cc:29-121).
//
// Two routes into vcclCommRegisterDmaBuf's CPU-mapping path:
//   udmabuf  a real dmabuf minted from a sealed memfd through /dev/udmabuf,
//            the kind of fd an exported graphics allocation is;
//   memfd    the memfd itself (a mappable fd that is not a CUDA export).
// Each rank registers its fd, writes its data through the returned pointer,
// runs an in-place all-reduce and an all-gather from the first half of the
// mapping into the second, and checks both on the host.  Ranks are forked
// processes with one GPU each; with VCCL_NO_DEVICE=1 they run on the CPU and
// move the mappings' bytes over the host data plane (TCP mesh), as the
// reference's ranks do over its TCP transport.
//
// Usage: test_dmabuf [nranks] [udmabuf|memfd]
// Exit: 0 pass, 1 fail, 77 skipped (/dev/udmabuf absent, or fewer GPUs than
// ranks for a device run).
#include <fcntl.h>
#include <linux/udmabuf.h>
#include <sys/ioctl.h>
#include <sys/mman.h>
#include <sys/wait.h>
#include <unistd.h>

#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "vccl.h"

namespace {

constexpr size_t kBytes = 96 * 4096;  // a multiple of the page size (udmabuf needs whole pages)
constexpr int kSkip = 77;

// A sealed memfd of kBytes; -1 on failure.
int makeMemfd() {
  int fd = memfd_create("vccl-dmabuf-test", MFD_ALLOW_SEALING);
  if (fd < 0) return -1;
  if (ftruncate(fd, kBytes) != 0 || fcntl(fd, F_ADD_SEALS, F_SEAL_SHRINK) != 0) {
    close(fd);
    return -1;
  }
  return fd;
}

// The fd a rank registers: a dmabuf over a memfd, or the memfd itself.
// -2 when /dev/udmabuf is absent.
int makeFd(bool udmabuf) {
  int memfd = makeMemfd();
  if (memfd < 0 || !udmabuf) return memfd;
  int dev = open("/dev/udmabuf", O_RDWR);
  if (dev < 0) {
    close(memfd);
    return -2;
  }
  struct udmabuf_create req;
  memset(&req, 0, sizeof(req));
  req.memfd = static_cast<__u32>(memfd);
  req.offset = 0;
  req.size = kBytes;
  int buf = ioctl(dev, UDMABUF_CREATE, &req);
  close(dev);
  close(memfd);
  return buf;
}

float arValue(int rank, size_t i) { return static_cast<float>((rank * 3 + static_cast<int>(i % 7)) % 11); }
float agValue(int rank, size_t i) { return static_cast<float>(rank * 512 + static_cast<int>(i % 257)); }

int rankMain(int rank, int n, const vcclUniqueId& id, bool udmabuf, bool useGpu) {
  if (useGpu && cudaSetDevice(rank) != cudaSuccess) return 1;
  vcclComm_t comm = nullptr;
  if (vcclCommInitRank(&comm, n, id, rank) != vcclSuccess) return 1;
  int fd = makeFd(udmabuf);
  if (fd == -2) {
    std::printf("rank %d: /dev/udmabuf not available: skipped\n", rank);
    vcclCommDestroy(comm);
    return kSkip;
  }
  if (fd < 0) {
    std::fprintf(stderr, "rank %d: cannot create the %s fd\n", rank, udmabuf ? "udmabuf" : "memfd");
    vcclCommDestroy(comm);
    return 1;
  }
  void* ptr = nullptr;
  vcclMemHandle_t handle = nullptr;
  vcclResult_t r = vcclCommRegisterDmaBuf(comm, fd, 0, kBytes, &ptr, &handle);
  close(fd);  // the registration keeps its own mapping
  if (r != vcclSuccess || ptr == nullptr) {
    std::fprintf(stderr, "rank %d: vcclCommRegisterDmaBuf: %s\n", rank, vcclGetErrorString(r));
    vcclCommDestroy(comm);
    return 1;
  }
  int bad = 0;
  float* data = static_cast<float*>(ptr);
  const size_t half = kBytes / sizeof(float) / 2;
  // in-place all-reduce over the first half
  for (size_t i = 0; i < half; i++) data[i] = arValue(rank, i);
  if (vcclAllReduce(data, data, half, vcclFloat32, vcclSum, comm) != vcclSuccess) bad++;
  for (size_t i = 0; i < half && bad < 4; i++) {
    float want = 0.0f;
    for (int p = 0; p < n; p++) want += arValue(p, i);
    if (data[i] != want) {
      std::fprintf(stderr, "rank %d: all-reduce [%zu] = %g, want %g\n", rank, i, data[i], want);
      bad++;
    }
  }
  // all-gather from the first half into the second
  const size_t per = half / n;
  for (size_t i = 0; i < per; i++) data[i] = agValue(rank, i);
  float* out = data + half;
  if (vcclAllGather(data, out, per, vcclFloat32, comm) != vcclSuccess) bad++;
  for (int p = 0; p < n; p++)
    for (size_t i = 0; i < per && bad < 8; i++)
      if (out[p * per + i] != agValue(p, i)) {
        std::fprintf(stderr, "rank %d: all-gather [%d][%zu] = %g, want %g\n", rank, p, i, out[p * per + i],
                     agValue(p, i));
        bad++;
      }
  if (vcclCommDeregister(comm, handle) != vcclSuccess) bad++;
  vcclCommDestroy(comm);
  return bad ? 1 : 0;
}

}  // namespace

int main(int argc, char** argv) {
  setenv("VCCL_SOCKET_ADDR", "127.0.0.1", 0);
  int n = argc > 1 ? std::atoi(argv[1]) : 1;
  const bool udmabuf = !(argc > 2 && std::strcmp(argv[2], "memfd") == 0);
  const char* nd = std::getenv("VCCL_NO_DEVICE");
  const bool useGpu = !(nd && std::atoi(nd) != 0);
  if (n < 1) n = 1;
  if (useGpu) {
    // Count GPUs in a child so this process never initialises CUDA before fork.
    int fds[2];
    if (pipe(fds) != 0) return 1;
    pid_t p = fork();
    if (p == 0) {
      int c = 0;
      if (cudaGetDeviceCount(&c) != cudaSuccess) c = 0;
      _exit(write(fds[1], &c, sizeof(c)) == sizeof(c) ? 0 : 1);
    }
    int ngpu = 0;
    if (read(fds[0], &ngpu, sizeof(ngpu)) != sizeof(ngpu)) ngpu = 0;
    waitpid(p, nullptr, 0);
    close(fds[0]);
    close(fds[1]);
    if (ngpu < n) {
      std::printf("needs %d GPUs, %d visible: skipped\n", n, ngpu);
      return kSkip;
    }
  }
  vcclUniqueId id;
  if (vcclGetUniqueId(&id) != vcclSuccess) return 1;
  std::vector<pid_t> kids;
  for (int r = 0; r < n; r++) {
    pid_t p = fork();
    if (p == 0) {
      const int rc = rankMain(r, n, id, udmabuf, useGpu);
      std::fflush(nullptr);
      _exit(rc);
    }
    kids.push_back(p);
  }
  int fails = 0, skips = 0;
  for (pid_t p : kids) {
    int st = 0;
    waitpid(p, &st, 0);
    if (WIFEXITED(st) && WEXITSTATUS(st) == kSkip) skips++;
    else if (!WIFEXITED(st) || WEXITSTATUS(st) != 0) fails++;
  }
  if (fails) {
    std::printf("dmabuf (%s, %d ranks): FAIL\n", udmabuf ? "udmabuf" : "memfd", n);
    return 1;
  }
  if (skips) return kSkip;
  std::printf("dmabuf (%s, %d ranks): OK\n", udmabuf ? "udmabuf" : "memfd", n);
  return 0;
}
