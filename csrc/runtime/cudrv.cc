// SPDX-License-Identifier: Apache-2.0
#include "runtime/cudrv.h"

#include <cuda_runtime.h>

#include <mutex>

#include "common/log.h"

namespace vccl {
namespace {

template <typename Fn>
bool resolve(const char* name, int version, Fn* out) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q{};
  cudaError_t e = cudaGetDriverEntryPointByVersion(name, &p, version, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || p == nullptr) {
    cudaGetLastError();
    *out = nullptr;
    return false;
  }
  *out = reinterpret_cast<Fn>(p);
  return true;
}

}  // namespace

const DriverApi* driverApi() {
  static DriverApi api;
  static bool ok = false;
  static std::once_flag once;
  std::call_once(once, [] {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
      cudaGetLastError();
      return;
    }
    bool all = true;
    all &= resolve("cuMemCreate", 10020, &api.memCreate);
    all &= resolve("cuMemRelease", 10020, &api.memRelease);
    all &= resolve("cuMemMap", 10020, &api.memMap);
    all &= resolve("cuMemUnmap", 10020, &api.memUnmap);
    all &= resolve("cuMemAddressReserve", 10020, &api.memAddressReserve);
    all &= resolve("cuMemAddressFree", 10020, &api.memAddressFree);
    all &= resolve("cuMemSetAccess", 10020, &api.memSetAccess);
    all &= resolve("cuMemExportToShareableHandle", 10020, &api.memExport);
    all &= resolve("cuMemImportFromShareableHandle", 10020, &api.memImport);
    all &= resolve("cuMemGetAllocationGranularity", 10020, &api.memGranularity);
    all &= resolve("cuMemRetainAllocationHandle", 11000, &api.memRetain);
    all &= resolve("cuMemGetAddressRange", 3020, &api.memGetAddressRange);
    all &= resolve("cuDeviceGet", 2000, &api.deviceGet);
    all &= resolve("cuDeviceGetAttribute", 2000, &api.deviceGetAttribute);
    all &= resolve("cuGetErrorString", 6000, &api.getErrorString);
    all &= resolve("cuCtxGetDevice", 2000, &api.ctxGetDevice);
    // Optional pieces: multicast (NVLS) and tensor maps.
    resolve("cuMulticastCreate", 12010, &api.mcCreate);
    resolve("cuMulticastAddDevice", 12010, &api.mcAddDevice);
    resolve("cuMulticastBindMem", 12010, &api.mcBindMem);
    resolve("cuMulticastUnbind", 12010, &api.mcUnbind);
    resolve("cuMulticastGetGranularity", 12010, &api.mcGranularity);
    resolve("cuTensorMapEncodeTiled", 12000, &api.tensorMapEncodeTiled);
    resolve("cuPointerGetAttribute", 4000, &api.pointerGetAttribute);
    ok = all;
    if (!ok) VWARN("CUDA driver entry points missing; device data plane disabled");
  });
  return ok ? &api : nullptr;
}

const char* cuErrorText(CUresult r) {
  const DriverApi* d = driverApi();
  const char* s = nullptr;
  if (d && d->getErrorString) d->getErrorString(r, &s);
  return s ? s : "unknown CUDA driver error";
}

}  // namespace vccl
