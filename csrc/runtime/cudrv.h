// SPDX-License-Identifier: Apache-2.0
// CUDA driver API entry points, resolved at run time through the runtime's
// cudaGetDriverEntryPointByVersion.  Nothing links libcuda directly, so the
// library (and its control plane) also loads on hosts without a GPU driver.
#pragma once

#include <cuda.h>

namespace vccl {

struct DriverApi {
  decltype(&::cuMemCreate) memCreate;
  decltype(&::cuMemRelease) memRelease;
  decltype(&::cuMemMap) memMap;
  decltype(&::cuMemUnmap) memUnmap;
  decltype(&::cuMemAddressReserve) memAddressReserve;
  decltype(&::cuMemAddressFree) memAddressFree;
  decltype(&::cuMemSetAccess) memSetAccess;
  decltype(&::cuMemExportToShareableHandle) memExport;
  decltype(&::cuMemImportFromShareableHandle) memImport;
  decltype(&::cuMemGetAllocationGranularity) memGranularity;
  decltype(&::cuMemRetainAllocationHandle) memRetain;
  decltype(&::cuMemGetAddressRange) memGetAddressRange;
  decltype(&::cuMulticastCreate) mcCreate;
  decltype(&::cuMulticastAddDevice) mcAddDevice;
  decltype(&::cuMulticastBindMem) mcBindMem;
  decltype(&::cuMulticastUnbind) mcUnbind;
  decltype(&::cuMulticastGetGranularity) mcGranularity;
  decltype(&::cuDeviceGet) deviceGet;
  decltype(&::cuDeviceGetAttribute) deviceGetAttribute;
  decltype(&::cuTensorMapEncodeTiled) tensorMapEncodeTiled;
  decltype(&::cuGetErrorString) getErrorString;
  decltype(&::cuCtxGetDevice) ctxGetDevice;
  decltype(&::cuPointerGetAttribute) pointerGetAttribute;  // optional (registration cache)
};

// Null when no driver is present.
const DriverApi* driverApi();
const char* cuErrorText(CUresult r);

}  // namespace vccl
