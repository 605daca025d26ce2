/* SPDX-License-Identifier: Apache-2.0
 *
 * vccl-b200 — collective communication for NVIDIA B200 over NVLink 5 / NVSwitch.
 *
 * API-compatible with the vccl C API (reference: include/vccl.h): every
 * function, enum value and struct layout of that header is kept so existing
 * callers (C, ctypes, Rust FFI) relink unchanged.  What changes is the data
 * plane: buffers may live in device memory, and every collective is a CUDA
 * kernel that moves data with peer-to-peer and NVLS multimem loads/stores
 * over NVLink between the ranks' symmetric workspaces.
 *
 * Semantics of the reference-named calls (vcclAllReduce, ...): host-blocking.
 * The work is ordered after everything already queued on the device's legacy
 * default stream and the call returns when the result is in recvbuff.  Both
 * device pointers and host pointers are accepted; host buffers are staged
 * through device memory.  The *Async variants (additions) take a CUDA stream,
 * accept device pointers only, and return immediately (NCCL semantics).
 * The kernels of one communicator run one after another in issue order even
 * when the calls name different streams (a call on a new stream waits for
 * the communicator's previous call; not applied inside CUDA-graph capture).
 */
#ifndef VCCL_H_
#define VCCL_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VCCL_MAJOR 0
#define VCCL_MINOR 2
#define VCCL_PATCH 0
#define VCCL_VERSION_CODE (VCCL_MAJOR * 10000 + VCCL_MINOR * 100 + VCCL_PATCH)

#define VCCL_UNIQUE_ID_BYTES 128
typedef struct {
  char internal[VCCL_UNIQUE_ID_BYTES];
} vcclUniqueId;

typedef struct vcclComm* vcclComm_t;

/* A CUDA stream (cudaStream_t / CUstream), spelled without CUDA headers. */
typedef struct CUstream_st* vcclStream_t;

typedef enum {
  vcclSuccess = 0,
  vcclUnhandledError = 1,
  vcclSystemError = 2,
  vcclInternalError = 3,
  vcclInvalidArgument = 4,
  vcclInvalidUsage = 5,
  vcclRemoteError = 6,
  vcclNumResults = 7
} vcclResult_t;

typedef enum {
  vcclInt8 = 0,
  vcclUint8 = 1,
  vcclInt32 = 2,
  vcclUint32 = 3,
  vcclInt64 = 4,
  vcclUint64 = 5,
  vcclFloat16 = 6,
  vcclFloat32 = 7,
  vcclFloat64 = 8,
  vcclBfloat16 = 9,
  /* Additions (same values as NCCL >= 2.24). */
  vcclFloat8e4m3 = 10,
  vcclFloat8e5m2 = 11,
  vcclNumTypes = 12
} vcclDataType_t;

typedef enum {
  vcclSum = 0,
  vcclProd = 1,
  vcclMax = 2,
  vcclMin = 3,
  vcclAvg = 4,
  vcclNumOps = 5
  /* Values >= vcclNumOps are communicator-local PreMulSum ops. */
} vcclRedOp_t;

typedef enum {
  vcclScalarDevice = 0,
  vcclScalarHostImmediate = 1
} vcclScalarResidence_t;

/* Communicator configuration.  `blocking` is honoured: with blocking=0 the
 * reference-named collectives do not wait for completion (they behave like
 * the *Async variants on the legacy default stream). */
typedef struct {
  size_t size;
  int blocking;
  int splitShare;
} vcclConfig_t;

#define VCCL_CONFIG_INITIALIZER { sizeof(vcclConfig_t), 1, 0 }

#define VCCL_SPLIT_NOCOLOR (-1)

vcclResult_t vcclGetVersion(int* version);

/* Create a unique id.  Must be called by the process that will be rank 0
 * (it binds the rendezvous socket), unless VCCL_COMM_ID=<ip>:<port> is set,
 * in which case every rank may derive the same id locally. */
vcclResult_t vcclGetUniqueId(vcclUniqueId* uniqueId);

/* Collectively create a communicator.  Rank r binds to the current CUDA
 * device of the calling thread (cudaSetDevice before the call); every rank
 * of a device communicator must sit in one NVSwitch domain.  Without a
 * visible CUDA device (or with VCCL_NO_DEVICE=1) the communicator moves host
 * buffers: the blocking collectives and send/recv run over a TCP mesh
 * between the ranks, which may sit on different hosts, with the reductions
 * on the CPU; the stream-ordered (*Async) calls return vcclInvalidUsage. */
vcclResult_t vcclCommInitRank(vcclComm_t* comm, int nranks,
                              vcclUniqueId commId, int rank);
vcclResult_t vcclCommInitRankConfig(vcclComm_t* comm, int nranks,
                                    vcclUniqueId commId, int rank,
                                    vcclConfig_t* config);

/* ndev communicators in this process, comm i on device devlist[i] (or i when
 * devlist is NULL).  Collectives on them must be issued inside a group. */
vcclResult_t vcclCommInitAll(vcclComm_t* comms, int ndev, const int* devlist);

vcclResult_t vcclCommSplit(vcclComm_t comm, int color, int key,
                           vcclComm_t* newcomm, vcclConfig_t* config);
vcclResult_t vcclCommFinalize(vcclComm_t comm);
vcclResult_t vcclCommDestroy(vcclComm_t comm);
vcclResult_t vcclCommAbort(vcclComm_t comm);
vcclResult_t vcclCommGetAsyncError(vcclComm_t comm, vcclResult_t* asyncError);
vcclResult_t vcclCommCount(const vcclComm_t comm, int* count);
vcclResult_t vcclCommUserRank(const vcclComm_t comm, int* rank);
/* CUDA device ordinal bound to this communicator (-1 for a communicator
 * without a device, which moves host buffers; the reference always reports 0). */
vcclResult_t vcclCommDevice(const vcclComm_t comm, int* device);

/* ── Collectives (reference semantics, host-blocking) ─────────────────── */
vcclResult_t vcclAllGather(const void* sendbuff, void* recvbuff,
                           size_t sendcount, vcclDataType_t datatype,
                           vcclComm_t comm);
vcclResult_t vcclReduceScatter(const void* sendbuff, void* recvbuff,
                               size_t recvcount, vcclDataType_t datatype,
                               vcclRedOp_t op, vcclComm_t comm);
vcclResult_t vcclAllReduce(const void* sendbuff, void* recvbuff, size_t count,
                           vcclDataType_t datatype, vcclRedOp_t op,
                           vcclComm_t comm);
vcclResult_t vcclReduce(const void* sendbuff, void* recvbuff, size_t count,
                        vcclDataType_t datatype, vcclRedOp_t op, int root,
                        vcclComm_t comm);
vcclResult_t vcclBroadcast(const void* sendbuff, void* recvbuff, size_t count,
                           vcclDataType_t datatype, int root, vcclComm_t comm);
vcclResult_t vcclBcast(void* buff, size_t count, vcclDataType_t datatype,
                       int root, vcclComm_t comm);
vcclResult_t vcclGather(const void* sendbuff, void* recvbuff,
                        size_t sendcount, vcclDataType_t datatype, int root,
                        vcclComm_t comm);
vcclResult_t vcclScatter(const void* sendbuff, void* recvbuff,
                         size_t recvcount, vcclDataType_t datatype, int root,
                         vcclComm_t comm);
vcclResult_t vcclAllToAll(const void* sendbuff, void* recvbuff, size_t count,
                          vcclDataType_t datatype, vcclComm_t comm);
vcclResult_t vcclAllToAllv(const void* sendbuff, const size_t sendcounts[],
                           const size_t sdispls[], void* recvbuff,
                           const size_t recvcounts[], const size_t rdispls[],
                           vcclDataType_t datatype, vcclComm_t comm);
vcclResult_t vcclSend(const void* sendbuff, size_t count,
                      vcclDataType_t datatype, int peer, vcclComm_t comm);
vcclResult_t vcclRecv(void* recvbuff, size_t count, vcclDataType_t datatype,
                      int peer, vcclComm_t comm);

/* ── Stream-ordered variants (additions; device pointers only) ─────────── */
vcclResult_t vcclAllGatherAsync(const void* sendbuff, void* recvbuff,
                                size_t sendcount, vcclDataType_t datatype,
                                vcclComm_t comm, vcclStream_t stream);
vcclResult_t vcclReduceScatterAsync(const void* sendbuff, void* recvbuff,
                                    size_t recvcount, vcclDataType_t datatype,
                                    vcclRedOp_t op, vcclComm_t comm,
                                    vcclStream_t stream);
vcclResult_t vcclAllReduceAsync(const void* sendbuff, void* recvbuff,
                                size_t count, vcclDataType_t datatype,
                                vcclRedOp_t op, vcclComm_t comm,
                                vcclStream_t stream);
vcclResult_t vcclReduceAsync(const void* sendbuff, void* recvbuff,
                             size_t count, vcclDataType_t datatype,
                             vcclRedOp_t op, int root, vcclComm_t comm,
                             vcclStream_t stream);
vcclResult_t vcclBroadcastAsync(const void* sendbuff, void* recvbuff,
                                size_t count, vcclDataType_t datatype,
                                int root, vcclComm_t comm,
                                vcclStream_t stream);
vcclResult_t vcclGatherAsync(const void* sendbuff, void* recvbuff,
                             size_t sendcount, vcclDataType_t datatype,
                             int root, vcclComm_t comm, vcclStream_t stream);
vcclResult_t vcclScatterAsync(const void* sendbuff, void* recvbuff,
                              size_t recvcount, vcclDataType_t datatype,
                              int root, vcclComm_t comm, vcclStream_t stream);
vcclResult_t vcclAllToAllAsync(const void* sendbuff, void* recvbuff,
                               size_t count, vcclDataType_t datatype,
                               vcclComm_t comm, vcclStream_t stream);
vcclResult_t vcclAllToAllvAsync(const void* sendbuff, const size_t sendcounts[],
                                const size_t sdispls[], void* recvbuff,
                                const size_t recvcounts[],
                                const size_t rdispls[],
                                vcclDataType_t datatype, vcclComm_t comm,
                                vcclStream_t stream);
vcclResult_t vcclSendAsync(const void* sendbuff, size_t count,
                           vcclDataType_t datatype, int peer, vcclComm_t comm,
                           vcclStream_t stream);
vcclResult_t vcclRecvAsync(void* recvbuff, size_t count,
                           vcclDataType_t datatype, int peer, vcclComm_t comm,
                           vcclStream_t stream);

/* ── Group semantics ─────────────────────────────────────────────────────
 * Calls between vcclGroupStart and the outermost vcclGroupEnd are queued.
 * At vcclGroupEnd each communicator's queue is launched in issue order;
 * every maximal run of consecutive Send/Recv on one communicator becomes one
 * kernel in which all of its transfers progress together, so a send+recv
 * pair with the same peer cannot deadlock.  Communicators on different
 * devices progress concurrently.  Groups nest. */
vcclResult_t vcclGroupStart(void);
vcclResult_t vcclGroupEnd(void);

/* ── Custom reduction ops ─────────────────────────────────────────────── */
vcclResult_t vcclRedOpCreatePreMulSum(vcclRedOp_t* op, void* scalar,
                                      vcclDataType_t datatype,
                                      vcclScalarResidence_t residence,
                                      vcclComm_t comm);
vcclResult_t vcclRedOpDestroy(vcclRedOp_t op, vcclComm_t comm);

/* ── Memory ──────────────────────────────────────────────────────────────
 * Device memory on the current CUDA device, allocated with the CUDA virtual
 * memory API as an exportable (POSIX fd) allocation, so it can be shared
 * with peers.  Without a CUDA device this falls back to page-aligned host
 * memory, as in the reference. */
vcclResult_t vcclMemAlloc(void** ptr, size_t size);
vcclResult_t vcclMemFree(void* ptr);

/* ── Threading contract ──────────────────────────────────────────────────
 * One collective (or one group) per communicator at a time.  Register and
 * Deregister are internally synchronised but must not overlap a collective
 * on the same communicator.  vcclCommAbort is safe from any thread at any
 * time: kernels of the communicator poll a host-mapped abort word and
 * return with an error. */

typedef void* vcclMemHandle_t;

/* Record a buffer with the communicator.  Collectives whose buffers are
 * registered skip pointer-kind probing; host buffers are pinned
 * (cudaHostRegister) so staging copies run at full PCIe speed. */
vcclResult_t vcclCommRegister(vcclComm_t comm, void* buff, size_t bytes,
                              vcclMemHandle_t* handle);
vcclResult_t vcclCommDeregister(vcclComm_t comm, vcclMemHandle_t handle);

/* Import an externally exported buffer and register it.  Accepted fds:
 * a CUDA VMM POSIX-fd export (cuMemExportToShareableHandle), an opaque fd
 * from another API's external-memory export, or a CPU-mappable dmabuf
 * (udmabuf/memfd).  *ptr receives the address to pass to collectives
 * (device address for the first two, a host mapping for the last).
 * vccl does not take ownership of fd. */
vcclResult_t vcclCommRegisterDmaBuf(vcclComm_t comm, int fd, uint64_t offset,
                                    size_t bytes, void** ptr,
                                    vcclMemHandle_t* handle);

/* ── Windows (an addition: zero-copy collectives) ───────────────────────
 * Collective: every rank calls it, in the same order, with a buffer of the
 * same `size` that lies inside a vcclMemAlloc device allocation (or, on
 * every rank alike, inside plain cudaMalloc memory: opened by CUDA IPC, or
 * used directly between ranks of one process, no multicast).  Every rank then maps every peer's
 * buffer, and for vcclMemAlloc memory on a node that supports NVLS the
 * buffers are also bound to one multicast object (unless flags has
 * VCCL_WIN_NO_MULTICAST).  All-reduce with both buffers in windows,
 * all-gather, broadcast and all-to-all(v) with the receive buffer in a
 * window and reduce-scatter with the send buffer in a window
 * then read and write the peers' buffers in place (no staging copies).  Rule for those calls: every rank passes
 * buffers at the same offsets of its windows and the same count; calls
 * that break it fail with vcclInvalidUsage on every rank and move no data.
 * Deregister is collective as well and must precede vcclMemFree. */
typedef void* vcclWindow_t;
#define VCCL_WIN_NO_MULTICAST 0x1
vcclResult_t vcclCommWindowRegister(vcclComm_t comm, void* buff, size_t size,
                                    vcclWindow_t* win, int flags);
vcclResult_t vcclCommWindowDeregister(vcclComm_t comm, vcclWindow_t win);

/* ── Registration cache (an addition: windows on demand) ──────────────────
 * With VCCL_REG_CACHE=1 on every rank, all-reduce, all-gather,
 * reduce-scatter and broadcast on plain cudaMalloc buffers (PyTorch
 * tensors) of at least VCCL_REG_CACHE_MIN bytes (window extent; default
 * 64 MiB) register their buffers as windows the first time and reuse them
 * afterwards, so those calls run the zero-copy window kernels without
 * vcclCommWindowRegister.  Each such call costs one small host allgather
 * among the ranks (tens of microseconds over the bootstrap's TCP sockets,
 * more with more ranks), which decides, alike on every rank, whether every rank
 * holds the same cached windows; registering costs a window registration,
 * and dropping an entry (LRU beyond VCCL_REG_CACHE_ENTRIES entries, or
 * an allocation replaced at the same address) synchronizes the device.
 * VCCL_REG_CACHE_ENTRIES defaults to VCCL_MR_CACHE, else 16.
 * Calls inside a stream capture stay on the staged kernels.  Peers keep the
 * cached allocations open: drop the cache (collective) before freeing
 * cached memory back to CUDA (torch.cuda.empty_cache()); vcclCommDestroy
 * drops it as well, together on every rank.
 * Stats: out[0] entries, [1] calls that consulted the cache on every rank,
 * [2] buffers reused, [3] buffers registered, [4] entries dropped,
 * [5] capacity. */
vcclResult_t vcclCommRegCacheFlush(vcclComm_t comm);
vcclResult_t vcclCommRegCacheStats(vcclComm_t comm, unsigned long long out[6]);

const char* vcclGetErrorString(vcclResult_t result);
const char* vcclGetLastError(vcclComm_t comm);
size_t vcclTypeSize(vcclDataType_t datatype);

#ifdef __cplusplus
}
#endif

#endif /* VCCL_H_ */
