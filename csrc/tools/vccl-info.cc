// SPDX-License-Identifier: Apache-2.0
// vccl-info: survey of the GPUs, their NVLink peer access and NVLS
// (multicast) support, marking what the library will use.
//
// Replaces the reference's RDMA device / GID survey (reference:
// tools/vccl_info.cc:66-114) with the B200 data plane's equivalents: which
// devices exist, which pairs can map each other's memory over NVLink, and
// whether NVSwitch multicast objects (NVLS) can be created.
#include <arpa/inet.h>
#include <cuda.h>
#include <ifaddrs.h>
#include <netinet/in.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>

#include <string>

#include "common/net.h"

int main() {
  // The address this host advertises for the rendezvous and for the host
  // data plane (VCCL_SOCKET_ADDR, else VCCL_SOCKET_IFNAME, else the first
  // non-loopback IPv4).
  vccl::WireEndpoint ep{};
  if (vccl::localEndpoint(&ep) == vcclSuccess) {
    std::string addr = vccl::endpointString(ep);
    const size_t colon = addr.rfind(':');
    if (colon != std::string::npos) addr.resize(colon);  // no port is bound yet
    std::printf("bootstrap / host data plane address: %s\n", addr.c_str());
  }
  // The host's IPv4 interfaces (VCCL_SOCKET_IFNAME picks one, VCCL_SOCKET_ADDR
  // an address), as the reference's survey lists its network devices.
  ifaddrs* ifs = nullptr;
  if (getifaddrs(&ifs) == 0) {
    std::printf("IPv4 interfaces:");
    for (ifaddrs* i = ifs; i != nullptr; i = i->ifa_next) {
      if (i->ifa_addr == nullptr || i->ifa_addr->sa_family != AF_INET) continue;
      char buf[INET_ADDRSTRLEN] = {0};
      inet_ntop(AF_INET, &reinterpret_cast<sockaddr_in*>(i->ifa_addr)->sin_addr, buf, sizeof(buf));
      std::printf(" %s=%s", i->ifa_name, buf);
    }
    std::printf("\n");
    freeifaddrs(ifs);
  }
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
    std::printf("no CUDA devices visible: communicators move host buffers over the host data plane (TCP)\n");
    return 0;
  }
  using GetAttr = CUresult (*)(int*, CUdevice_attribute, CUdevice);
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q{};
  cudaGetDriverEntryPointByVersion("cuDeviceGetAttribute", &fn, 2000, cudaEnableDefault, &q);
  GetAttr getAttr = reinterpret_cast<GetAttr>(fn);
  int drv = 0, rt = 0;
  cudaDriverGetVersion(&drv);
  cudaRuntimeGetVersion(&rt);
  std::printf("CUDA driver %d, runtime %d, %d device(s)\n", drv, rt, n);
  for (int d = 0; d < n; d++) {
    cudaDeviceProp p;
    cudaGetDeviceProperties(&p, d);
    int mc = 0, vmm = 0, fd = 0;
    if (getAttr) {
      getAttr(&mc, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, d);
      getAttr(&vmm, CU_DEVICE_ATTRIBUTE_VIRTUAL_MEMORY_MANAGEMENT_SUPPORTED, d);
      getAttr(&fd, CU_DEVICE_ATTRIBUTE_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR_SUPPORTED, d);
    }
    std::printf("  [%d] %s sm_%d%d  %d SMs  %.1f GiB  bus %02x:%02x  VMM=%d posix-fd=%d multicast(NVLS)=%d\n", d,
                p.name, p.major, p.minor, p.multiProcessorCount, p.totalGlobalMem / 1073741824.0, p.pciBusID,
                p.pciDeviceID, vmm, fd, mc);
  }
  std::printf("peer access matrix (P = NVLink/P2P capable, A = native atomics):\n      ");
  for (int b = 0; b < n; b++) std::printf("%4d", b);
  std::printf("\n");
  bool allPeer = true;
  for (int a = 0; a < n; a++) {
    std::printf("  %2d: ", a);
    for (int b = 0; b < n; b++) {
      if (a == b) {
        std::printf("   -");
        continue;
      }
      int can = 0, atom = 0;
      cudaDeviceCanAccessPeer(&can, a, b);
      cudaDeviceGetP2PAttribute(&atom, cudaDevP2PAttrNativeAtomicSupported, a, b);
      allPeer &= can != 0;
      std::printf("  %c%c", can ? 'P' : '.', atom ? 'A' : ' ');
    }
    std::printf("\n");
  }
  const char* nvlsEnv = std::getenv("VCCL_NVLS_ENABLE");
  const bool nvlsOff = nvlsEnv && std::atoi(nvlsEnv) == 0;
  std::printf("vccl will use: %s peer-to-peer workspaces%s\n", allPeer ? "NVLink" : "(NOT all pairs P2P!)",
              nvlsOff ? ", NVLS disabled by VCCL_NVLS_ENABLE=0" : ", NVLS multicast when every rank supports it");
  return 0;
}
