// SPDX-License-Identifier: Apache-2.0
// Host side of the tcgen05 GEMM: tensor-map construction, tile-width
// selection and the plain / SiLU*mul entry points.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <utility>

#include "common/log.h"
#include "fused/gemm_launch.cuh"
#include "runtime/cudrv.h"
#include "vccl_tp.h"

namespace vccl {
namespace gemm {

bool makeMapKMajor(CUtensorMap* map, const void* base, int rows, int K, int boxRows) {
  const DriverApi* d = driverApi();
  if (d == nullptr || d->tensorMapEncodeTiled == nullptr) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (K % 8) != 0) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(boxRows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = d->tensorMapEncodeTiled(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                                       strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                       CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    VERR("cuTensorMapEncodeTiled failed: %s", cuErrorText(r));
    return false;
  }
  return true;
}

int smCount() {
  static int n = [] {
    int dev = 0, c = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev);
    return c;
  }();
  return n;
}

int pickBNWaves(int M, int N, int sms) {
  const int tm = (M + kBM - 1) / kBM;
  double best = 0.0;
  int bestBn = 256;
  for (int bn : {256, 128, 64, 32}) {
    const int tiles = tm * ((N + bn - 1) / bn);
    const int waves = (tiles + sms - 1) / sms;
    // A narrower tile re-reads its A rows once more per column tile and
    // runs shorter MMA chains; charge it a little per halving.
    const double charge = bn >= 256 ? 1.0 : bn == 128 ? 1.05 : bn == 64 ? 1.15 : 1.35;
    const double cost = static_cast<double>(waves) * bn * charge;
    if (bn == 256 || cost < best - 1e-9) {
      best = cost;
      bestBn = bn;
    }
  }
  return bestBn;
}

int pairGroupRows(int K) {
  static const long env = envLongGemm("VCCL_GEMM_GROUP");
  if (env > 0 && env <= 64) return static_cast<int>(env);
  // Measured on B200 (gemm_one): 16 pair rows for K = 4096 (8192 x 28672:
  // 1194 us against 1213 / 1234 us with 12 / 8), 8 for K = 14336 (8192 x
  // 4096: 642 us against 649 / 660 us with 16 / 4).  A pair row's A strip
  // is 256 x K x 2 bytes; longer strips want smaller groups.
  return K <= 8192 ? 16 : 8;
}

int pairMode() {
  // Read per call (tests switch it): unset or 1 = by cost, 0 = off, 2 = always.
  const char* v = std::getenv("VCCL_GEMM_PAIR");
  if (v == nullptr || v[0] == '\0') return 1;
  return v[0] == '0' ? 0 : v[0] == '2' ? 2 : 1;
}

int pairMaxClusters(const void* kernel, int smemBytes, int threads) {
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find({dev, kernel});
  if (it != cache.end()) return it->second;
  // The occupancy query sees the kernel's shared-memory limit, so raise it first.
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smemBytes) != cudaSuccess) {
    VWARN("GEMM on CTA pairs: cannot raise the shared-memory limit on device %d; one-SM tiles only", dev);
    cudaGetLastError();
    cache[{dev, kernel}] = 0;
    return 0;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(smCount()), 1, 1);
  cfg.blockDim = dim3(static_cast<unsigned>(threads), 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(smemBytes);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  const cudaError_t e = cudaOccupancyMaxActiveClusters(&n, kernel, &cfg);
  if (e != cudaSuccess) {
    VWARN("GEMM on CTA pairs: occupancy query failed on device %d (%s); one-SM tiles only", dev,
          cudaGetErrorString(e));
    cudaGetLastError();
    n = 0;
  }
  VINFO("GEMM on CTA pairs: %d pairs co-resident on device %d", n, dev);
  cache[{dev, kernel}] = n;
  return n;
}

int pickBN(int M, int N) {
  const int sms = smCount();
  static const bool byWaves = envLongGemm("VCCL_GEMM_PICK_WAVES") != 0;
  if (byWaves) return pickBNWaves(M, N, sms);
  const int tm = (M + kBM - 1) / kBM;
  for (int bn : {256, 128, 64}) {
    const int tiles = tm * ((N + bn - 1) / bn);
    if (tiles >= sms) return bn;
  }
  return 32;
}

// Decode shapes (at most two 128-row tiles) stream the weights once; their
// time is set by how evenly the work spreads over the SMs.  Split K so that
// tiles x splits fills whole waves of the persistent grid, keeping at least
// 4 k-blocks per split and the fp32 partials below a quarter of the weight
// bytes (M x N x splits x 4 <= N x K x 2 / 4).
SplitPlan planSplitK(int M, int N, int K) {
  const int sms = smCount();
  const int tilesM = (M + kBM - 1) / kBM;
  if (tilesM > 2) return {0, 1};
  const int numK = (K + kBK - 1) / kBK;
  const int tiles = tilesM * ((N + 127) / 128);
  int maxS = numK / 4;
  if (maxS > 16) maxS = 16;
  const int byPartials = K / (8 * M);
  if (maxS > byPartials) maxS = byPartials;
  auto waste = [&](int s) {
    const int units = tiles * s;
    const int waves = (units + sms - 1) / sms;
    return static_cast<double>(waves) * sms / units;
  };
  int best = 1;
  double bestWaste = waste(1);
  for (int s = 2; s <= maxS; s++) {
    const double w = waste(s);
    if (w < bestWaste - 0.03) {
      best = s;
      bestWaste = w;
    }
  }
  if (best < 2) return {0, 1};
  return {128, best};
}

namespace {
__global__ void __launch_bounds__(256) splitReduceKernel(const float4* ws, int splits, size_t n4, size_t stride4,
                                                         uint2* out, const volatile int* abortWord) {
  // The GEMM that wrote the partials abandoned its tiles: the partials are
  // stale, so the output is poisoned with NaN instead of summed.
  const bool poison = abortWord != nullptr && *abortWord != 0;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    if (poison) {
      out[i] = make_uint2(0x7fc07fc0u, 0x7fc07fc0u);
      continue;
    }
    float4 a = ws[i];
    for (int sp = 1; sp < splits; sp++) {
      const float4 b = ws[sp * stride4 + i];
      a.x += b.x;
      a.y += b.y;
      a.z += b.z;
      a.w += b.w;
    }
    out[i] = make_uint2(packBf16(a.x, a.y), packBf16(a.z, a.w));
  }
}

// Partials hold gate and up columns interleaved in groups of 16 (see
// EpiSiluMul); out[m][j] = silu(gate) * up with j = 16 g + w taking gate
// column 32 g + w and up column 32 g + 16 + w.  Four outputs per thread.
__global__ void __launch_bounds__(256) splitReduceSiluKernel(const float* ws, int splits, int M, int N,
                                                             size_t stride, uint2* out) {
  const int half = N / 2;
  const size_t n4 = static_cast<size_t>(M) * half / 4;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t o = i * 4;
    const int m = static_cast<int>(o / half), j = static_cast<int>(o % half);
    const size_t gcol = static_cast<size_t>(m) * N + (j / 16) * 32 + (j % 16);
    float4 g = *reinterpret_cast<const float4*>(ws + gcol);
    float4 u = *reinterpret_cast<const float4*>(ws + gcol + 16);
    for (int sp = 1; sp < splits; sp++) {
      const float4 g2 = *reinterpret_cast<const float4*>(ws + sp * stride + gcol);
      const float4 u2 = *reinterpret_cast<const float4*>(ws + sp * stride + gcol + 16);
      g.x += g2.x, g.y += g2.y, g.z += g2.z, g.w += g2.w;
      u.x += u2.x, u.y += u2.y, u.z += u2.z, u.w += u2.w;
    }
    auto f = [](float x, float y) { return x / (1.0f + __expf(-x)) * y; };
    out[i] = make_uint2(packBf16(f(g.x, u.x), f(g.y, u.y)), packBf16(f(g.z, u.z), f(g.w, u.w)));
  }
}
}  // namespace

cudaError_t launchSplitReduceSilu(const float* ws, int splits, int M, int N, void* out, cudaStream_t st) {
  const size_t n4 = static_cast<size_t>(M) * (N / 2) / 4;
  size_t blocks = (n4 + 255) / 256;
  if (blocks > static_cast<size_t>(smCount()) * 4) blocks = static_cast<size_t>(smCount()) * 4;
  if (blocks == 0) blocks = 1;
  splitReduceSiluKernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(ws, splits, M, N,
                                                                       static_cast<size_t>(M) * N,
                                                                       static_cast<uint2*>(out));
  return cudaGetLastError();
}

cudaError_t launchSplitReduce(const float* ws, int splits, size_t elems, void* out, cudaStream_t st,
                              const volatile int* abortWord) {
  const size_t n4 = elems / 4;
  size_t blocks = (n4 + 255) / 256;
  if (blocks > static_cast<size_t>(smCount()) * 4) blocks = static_cast<size_t>(smCount()) * 4;
  if (blocks == 0) blocks = 1;
  splitReduceKernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(reinterpret_cast<const float4*>(ws), splits, n4,
                                                                   n4, static_cast<uint2*>(out), abortWord);
  return cudaGetLastError();
}

// Split-K scratch, cached per (device, stream) so steady-state calls
// allocate nothing: calls on one stream are ordered, and calls on different
// streams use different buffers.  A call that needs more than the cached
// size waits for its stream, frees the old buffer and allocates a larger one.
// At most kCachedStreams streams per device get a cached buffer (nothing
// tells the library when a stream is destroyed, so the cache must not grow
// with every stream a program ever creates); calls on other streams use a
// stream-ordered allocation, as while capturing.  nullptr means "not cached".
// Not used while the stream is being captured (see vcclGemmBf16).
constexpr size_t kCachedStreams = 16;

float* splitScratch(cudaStream_t st, size_t bytes) {
  static std::mutex mu;
  static std::map<std::pair<int, cudaStream_t>, std::pair<void*, size_t>> cache;
  static std::map<int, size_t> perDevice;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find({dev, st});
  if (it == cache.end()) {
    if (perDevice[dev] >= kCachedStreams) return nullptr;
    perDevice[dev]++;
    it = cache.emplace(std::make_pair(dev, st), std::make_pair(nullptr, size_t{0})).first;
  }
  auto& e = it->second;
  if (e.second < bytes) {
    if (e.first != nullptr) {
      cudaStreamSynchronize(st);
      cudaFree(e.first);
      e = {nullptr, 0};
    }
    const size_t sz = (bytes + (1u << 20) - 1) / (1u << 20) * (1u << 20);
    void* p = nullptr;
    if (cudaMalloc(&p, sz) != cudaSuccess) return nullptr;
    e = {p, sz};
  }
  return static_cast<float*>(e.first);
}

bool splitFixupEnabled() {
  // On by default: measured on B200, the in-kernel reduction saves the second
  // kernel of a decode GEMM (1 x 7168 x 8192 + SiLU*mul: 45.8 vs 48.8 us) with
  // the same bits; VCCL_GEMM_SPLIT_FIXUP=0 keeps the separate reduction.
  static const bool on = [] {
    const char* v = std::getenv("VCCL_GEMM_SPLIT_FIXUP");
    return v == nullptr || v[0] != '0';
  }();
  return on;
}

// Fix-up semaphores, cached per (device, stream) like the scratch; zeroed
// once, and every call leaves them at zero.
uint32_t* splitSems(cudaStream_t st) {
  static std::mutex mu;
  static std::map<std::pair<int, cudaStream_t>, uint32_t*> cache;
  static std::map<int, size_t> perDevice;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find({dev, st});
  if (it == cache.end()) {
    if (perDevice[dev] >= kCachedStreams) return nullptr;
    perDevice[dev]++;
    it = cache.emplace(std::make_pair(dev, st), nullptr).first;
  }
  uint32_t*& p = it->second;
  if (p == nullptr) {
    void* q = nullptr;
    if (cudaMalloc(&q, kSemSlots * sizeof(uint32_t)) != cudaSuccess) return nullptr;
    if (cudaMemset(q, 0, kSemSlots * sizeof(uint32_t)) != cudaSuccess) {
      cudaFree(q);
      return nullptr;
    }
    p = static_cast<uint32_t*>(q);
  }
  return p;
}

bool acquireScratch(cudaStream_t st, size_t bytes, Scratch* out) {
  out->p = nullptr;
  out->async = false;
  out->st = st;
  out->sems = nullptr;
  out->semsAsync = false;
  if (bytes == 0) return true;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  cudaStreamIsCapturing(st, &cap);
  if (cap != cudaStreamCaptureStatusNone) {
    // While the stream is captured into a CUDA graph nothing may be
    // allocated synchronously; a stream-ordered allocation becomes a memory
    // node of the graph.
    if (cudaMallocAsync(&out->p, bytes, st) != cudaSuccess) return false;
    out->async = true;
    if (splitFixupEnabled()) {
      void* q = nullptr;
      if (cudaMallocAsync(&q, kSemSlots * sizeof(uint32_t), st) == cudaSuccess) {
        if (cudaMemsetAsync(q, 0, kSemSlots * sizeof(uint32_t), st) == cudaSuccess) {
          out->sems = static_cast<uint32_t*>(q);
          out->semsAsync = true;
        } else {
          cudaFreeAsync(q, st);
        }
      }
    }
    return true;
  }
  out->p = splitScratch(st, bytes);
  if (out->p == nullptr) {
    // Not a cached stream (or its allocation failed): a stream-ordered
    // allocation released after the call.
    if (cudaMallocAsync(&out->p, bytes, st) != cudaSuccess) {
      out->p = nullptr;
      return false;
    }
    out->async = true;
    return true;  // no fix-up semaphores: the reduction kernel runs
  }
  if (splitFixupEnabled()) out->sems = splitSems(st);
  return true;
}

void releaseScratch(const Scratch& s) {
  if (s.async && s.p != nullptr) cudaFreeAsync(s.p, s.st);
  if (s.semsAsync && s.sems != nullptr) cudaFreeAsync(s.sems, s.st);
}

SplitPlan planFor(int M, int N, int K, int bnOverride, bool allowSplit) {
  const char* sk = std::getenv("VCCL_GEMM_SPLITK");
  if (!allowSplit || bnOverride > 0 || (sk && sk[0] == '0')) return {0, 1};
  // VCCL_GEMM_SPLITS=s forces s K splits of 128-wide tiles on decode shapes
  // (for measurements; 1 = no split).
  const long forced = envLongGemm("VCCL_GEMM_SPLITS");
  if (forced > 0 && (M + kBM - 1) / kBM <= 2) {
    const int numK = (K + kBK - 1) / kBK;
    const int sp = static_cast<int>(forced < numK ? forced : numK);
    return sp > 1 ? SplitPlan{128, sp} : SplitPlan{0, 1};
  }
  return planSplitK(M, N, K);
}

PairPlan planPair(int M, int N, int K, int bnOverride, int pairs) {
  const int mode = pairMode();
  if (mode == 0 || bnOverride > 0 || M < kPairBM || N < kPairBN || pairs <= 0) return {false, 1};
  const int tiles = ((M + kPairBM - 1) / kPairBM) * ((N + kPairBN - 1) / kPairBN);
  const int nk = (K + kBK - 1) / kBK;
  const char* sk = std::getenv("VCCL_GEMM_SPLITK");
  const bool splitOk = !(sk && sk[0] == '0');
  // Time model (us), B200: a pair does a 256 x 256 x K tile in about
  // 2 * 256 * 256 * K / 21.6e12 s (1.6 PFLOP/s over 74 pairs); partials cost
  // their write and read at ~6 TB/s plus a launch.
  const double wave = 2.0 * kPairBM * kPairBN * K / 21.6e6;
  double best = 1e30;
  int bestS = 1;
  for (int sp = 1; sp <= 4; sp++) {
    if (sp > 1 && (!splitOk || nk / sp < 8)) break;
    const int waves = (tiles * sp + pairs - 1) / pairs;
    double t = waves * wave / sp;
    if (sp > 1) t += 2.0 * M * N * 4.0 * sp / 6.0e6 + 3.0;
    if (t < best * 0.97) {  // a split must win clearly
      best = t;
      bestS = sp;
    }
  }
  if (mode == 2) return {true, bestS};
  // The one-SM kernel at its tile width, its own split-K only for decode
  // shapes.  Its time per wave against the ideal, measured on B200
  // (gemm_one): 1.18x with 256-wide tiles (8192 x 28672 x 4096), 1.38x with
  // 128 (1024 x 4096 x 14336), 2.1x with 64 (512 x 4096 x 14336); narrower
  // tiles re-read A from shared memory for fewer columns per MMA.
  const int sms = smCount();
  const int bn = pickBN(M, N);
  const double charge = bn >= 256 ? 1.18 : bn == 128 ? 1.38 : bn == 64 ? 2.1 : 3.0;
  const int tiles1 = ((M + kBM - 1) / kBM) * ((N + bn - 1) / bn);
  const double wave1 = 2.0 * kBM * bn * K / (1.6e15 / sms) * 1e6 * charge;
  const double t1 = ((tiles1 + sms - 1) / sms) * wave1;
  return {best <= t1, bestS};
}

size_t gemmAutoScratchBytes(int M, int N, int K, int bnOverride, bool allowSplit) {
  const SplitPlan plan = planFor(M, N, K, bnOverride, allowSplit);
  if (plan.splits > 1) return static_cast<size_t>(M) * N * plan.splits * sizeof(float);
  if (!allowSplit) return 0;
  // Either epilogue's pair instance: the plans agree (same shape), only the
  // occupancy could differ, and both are one CTA per SM.
  const PairPlan pp = planPair(M, N, K, bnOverride, pairClustersFor<EpiStore>());
  return pp.use && pp.splits > 1 ? static_cast<size_t>(M) * N * pp.splits * sizeof(float) : 0;
}

cudaError_t gemmAuto(const void* A, const void* W, void* C, int M, int N, int K, bool siluMul, cudaStream_t st,
                     int bnOverride, bool allowSplit, float* ws, uint32_t* sems) {
  const SplitPlan plan = planFor(M, N, K, bnOverride, allowSplit);
  if (plan.splits > 1) {
    if (ws == nullptr) return cudaErrorInvalidValue;
    const size_t elems = static_cast<size_t>(M) * N;
    EpiPartialF32 epi{ws, N, elems};
    const int tiles = ((M + kBM - 1) / kBM) * ((N + plan.bn - 1) / plan.bn);
    if (sems != nullptr && M <= kFixupMaxRows && tiles * 4 <= kSemSlots) {
      auto* out = static_cast<__nv_bfloat16*>(C);
      if (siluMul) return launchGemm(A, W, M, N, K, EpiSplitFixup<true>{epi, sems, out}, NoHooks{}, st, plan.bn, 0,
                                     plan.splits);
      return launchGemm(A, W, M, N, K, EpiSplitFixup<false>{epi, sems, out}, NoHooks{}, st, plan.bn, 0,
                        plan.splits);
    }
    cudaError_t e = launchGemm(A, W, M, N, K, epi, NoHooks{}, st, plan.bn, 0, plan.splits);
    if (e != cudaSuccess) return e;
    return siluMul ? launchSplitReduceSilu(ws, plan.splits, M, N, C, st)
                   : launchSplitReduce(ws, plan.splits, elems, C, st);
  }
  // VCCL_GEMM_PAIR=2 demands the pair kernel for every shape it covers and
  // fails (instead of falling back) where the device cannot run it.
  const bool forcePair = pairMode() == 2 && M >= kPairBM && N >= kPairBN && bnOverride <= 0;
  const PairPlan pp = planPair(M, N, K, bnOverride, pairClustersFor<EpiStore>());
  if (pp.use && pp.splits > 1 && allowSplit) {
    // Split-K on pairs: fp32 partials, then the (SiLU*mul) reduction.
    if (ws == nullptr) return cudaErrorInvalidValue;
    const size_t elems = static_cast<size_t>(M) * N;
    EpiPartialF32 epi{ws, N, elems};
    cudaError_t e = launchGemmPair(A, W, M, N, K, epi, st, nullptr, PairNoHooks{}, 0, pp.splits);
    if (e == cudaErrorNotSupported && !forcePair) {
      e = cudaSuccess;  // fall through to the one-SM kernel below
    } else {
      if (e != cudaSuccess) return e;
      return siluMul ? launchSplitReduceSilu(ws, pp.splits, M, N, C, st) : launchSplitReduce(ws, pp.splits, elems, C, st);
    }
  }
  if (siluMul) {
    EpiSiluMul epi{static_cast<__nv_bfloat16*>(C), N / 2};
    if (pp.use) {
      const cudaError_t e = launchGemmPair(A, W, M, N, K, epi, st);
      if (e != cudaErrorNotSupported || forcePair) return e;
    } else if (forcePair) {
      return cudaErrorNotSupported;
    }
    return launchGemm(A, W, M, N, K, epi, NoHooks{}, st, bnOverride, 0);
  }
  EpiStore epi{static_cast<__nv_bfloat16*>(C), N};
  if (pp.use) {
    const cudaError_t e = launchGemmPair(A, W, M, N, K, epi, st);
    if (e != cudaErrorNotSupported || forcePair) return e;
  } else if (forcePair) {
    return cudaErrorNotSupported;
  }
  return launchGemm(A, W, M, N, K, epi, NoHooks{}, st, bnOverride, 0);
}

// One abort flag per device in pinned, mapped host memory: a GEMM that
// abandons its tiles (a pipeline wait ran out) sets it, and the next GEMM
// call on that device reads it without synchronising.
namespace {
std::mutex gFlagMu;
int* gHostFlags[64] = {};
int* gDevFlags[64] = {};

int currentDevice() {
  int dev = 0;
  cudaGetDevice(&dev);
  return dev & 63;
}
}  // namespace

int* errorFlag() {
  const int dev = currentDevice();
  std::lock_guard<std::mutex> lock(gFlagMu);
  if (gDevFlags[dev] == nullptr) {
    int* h = nullptr;
    if (cudaHostAlloc(reinterpret_cast<void**>(&h), sizeof(int) * 16, cudaHostAllocMapped | cudaHostAllocPortable) !=
        cudaSuccess)
      return nullptr;
    memset(h, 0, sizeof(int) * 16);
    int* d = nullptr;
    if (cudaHostGetDevicePointer(reinterpret_cast<void**>(&d), h, 0) != cudaSuccess) return nullptr;
    gHostFlags[dev] = h;
    gDevFlags[dev] = d;
  }
  return gDevFlags[dev];
}

bool takeAbortFlag() {
  const int dev = currentDevice();
  std::lock_guard<std::mutex> lock(gFlagMu);
  volatile int* h = gHostFlags[dev];
  if (h == nullptr || *h == 0) return false;
  *h = 0;
  return true;
}

vcclResult_t gemmWithScratch(const char* what, const void* A, const void* W, void* C, int M, int N, int K,
                             bool siluMul, cudaStream_t st) {
  const int bnEnv = static_cast<int>(envLongGemm("VCCL_GEMM_BN"));
  // Decode shapes split K across more CTAs; the fp32 partials live in
  // per-stream scratch (a graph memory node while the stream is captured).
  Scratch sc;
  const size_t bytes = gemmAutoScratchBytes(M, N, K, bnEnv, true);
  if (!acquireScratch(st, bytes, &sc)) {
    VERR("%s: cannot allocate %zu bytes of split-K scratch", what, bytes);
    return vcclSystemError;
  }
  cudaError_t e = gemmAuto(A, W, C, M, N, K, siluMul, st, bnEnv, true, static_cast<float*>(sc.p), sc.sems);
  releaseScratch(sc);
  if (e != cudaSuccess) {
    VERR("%s: %s", what, cudaGetErrorString(e));
    return launchResult(e);
  }
  return vcclSuccess;
}

}  // namespace gemm
}  // namespace vccl

using namespace vccl;

extern "C" {

namespace {
vcclResult_t gemmEntry(const char* what, const void* A, const void* W, void* C, int M, int N, int K, bool siluMul,
                       vcclStream_t stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (gemm::takeAbortFlag()) {
    VERR("%s: an earlier GEMM on this device abandoned its tiles (a pipeline wait ran out); its output is invalid",
         what);
    return vcclInternalError;
  }
  return gemm::gemmWithScratch(what, A, W, C, M, N, K, siluMul, st);
}
}  // namespace

vcclResult_t vcclGemmBf16(const void* A, const void* W, void* C, int M, int N, int K, vcclStream_t stream) {
  if (!A || !W || !C || M <= 0 || N <= 0 || K <= 0 || (N % 16) != 0 || (K % 8) != 0) return vcclInvalidArgument;
  return gemmEntry("vcclGemmBf16", A, W, C, M, N, K, false, stream);
}

vcclResult_t vcclGemmSiluMul(const void* A, const void* W, void* H, int M, int N, int K, vcclStream_t stream) {
  if (!A || !W || !H || M <= 0 || N <= 0 || K <= 0 || (N % 32) != 0 || (K % 8) != 0) return vcclInvalidArgument;
  return gemmEntry("vcclGemmSiluMul", A, W, H, M, N, K, true, stream);
}

}  // extern "C"
