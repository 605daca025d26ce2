// SPDX-License-Identifier: Apache-2.0
// Host data plane: collectives on host memory over TCP, for communicators
// without a device (VCCL_NO_DEVICE=1, or a host with no GPU) whose ranks
// may sit on different hosts.
//
// The device communicators move data with NVLink kernels and need every
// rank on one NVSwitch domain.  The reference's only data path is the host
// one (TCP or RoCE between hosts, reductions on the CPU; reference:
// src/transport/tcp.cc, src/core/collectives.cc); this plane keeps that
// capability for host tensors.  Its design is a full mesh of TCP streams
// (one per rank pair) driven by one progress loop over all of them, and
// every collective is a set of concurrent point-to-point transfers over the
// mesh rather than a ring:
//
//  * all-gather, gather, scatter, all-to-all(v): every rank sends its
//    blocks to every destination at once (each stream carries exactly the
//    bytes that must cross it);
//  * broadcast: small messages go from the root to every rank; large ones
//    in pieces, the root handing each receiver one block of a piece (every
//    byte leaves the root once) and the receivers exchanging their blocks;
//  * reduce-scatter: every rank sends each owner its copy of the owner's
//    block, and the owner reduces the n contributions in rank order;
//  * all-reduce: reduce-scatter, then all-gather of the reduced blocks (or,
//    while (n - 1) x the message is at most VCCL_HOST_AR_DIRECT bytes, every
//    rank sends the whole message to every peer and reduces all n copies in
//    rank order);
//  * reduce: every rank sends to the root, which reduces in rank order;
//  * a group of sends and receives runs in one progress loop.
//
// Every element is reduced by one rank, in rank order, with 16- and 8-bit
// floats accumulated in fp32, so every rank ends with the same bits.
// Large messages go in pieces (VCCL_HOST_CHUNK bytes per peer): the
// reduction buffers stay bounded, and the next piece is on the wire while the
// current one is reduced.  A batch that sends and receives many bytes hands
// its sends to a sender thread, so the kernel's socket copies run on two
// cores.  Waits honour VCCL_TIMEOUT and vcclCommAbort; a peer that closes
// its stream fails the call.
#pragma once

#include <atomic>
#include <condition_variable>
#include <cstddef>
#include <cstdint>
#include <deque>
#include <memory>
#include <mutex>
#include <thread>
#include <vector>

#include "vccl.h"

namespace vccl {

class Bootstrap;

// One transfer of a progress loop: `bytes` from `buf` to `peer` (send) or
// from `peer` into `buf` (receive).  Transfers to (from) one peer leave
// (arrive) in list order.
struct HostXfer {
  bool send;
  int peer;
  char* buf;
  size_t bytes;
};

// Host-side reduction arguments of one call.
struct HostRed {
  vcclDataType_t dt;
  int kind;      // sum / prod / max / min (the device RedKind values)
  bool avg;      // divide the sum by the rank count (float types)
  bool premul;   // every rank scales its own contribution by its `scalar` before sending
  double scalar;
};

class HostPlane {
 public:
  // Collective: every rank of `bs` calls it; builds the mesh.
  static vcclResult_t create(Bootstrap* bs, std::unique_ptr<HostPlane>* out);
  ~HostPlane();

  int rank() const { return rank_; }
  int nranks() const { return n_; }

  // Runs every transfer of `xs` to completion, all streams progressing at
  // once.  Self transfers are not allowed (copy locally instead).
  vcclResult_t run(const std::vector<HostXfer>& xs);

  vcclResult_t allReduce(const char* send, char* recv, size_t count, const HostRed& r);
  vcclResult_t reduceScatter(const char* send, char* recv, size_t recvCount, const HostRed& r);
  vcclResult_t allGather(const char* send, char* recv, size_t bytes);
  vcclResult_t broadcast(const char* send, char* recv, size_t bytes, int root);
  vcclResult_t reduce(const char* send, char* recv, size_t count, const HostRed& r, int root);
  vcclResult_t gather(const char* send, char* recv, size_t bytes, int root);
  vcclResult_t scatter(const char* send, char* recv, size_t bytes, int root);
  // Counts and displacements in bytes.
  vcclResult_t allToAllv(const char* send, const size_t* sc, const size_t* sd, char* recv, const size_t* rc,
                         const size_t* rd);

  // Unblocks every wait (vcclCommAbort); later calls fail.
  void abort();

  // How the latest collective moved its data (for the call profile).
  const char* path() const { return path_; }

 private:
  HostPlane(int rank, int n) : rank_(rank), n_(n) {}

  // Transfers in progress: run() starts a batch and finishes it; reductions
  // in pieces start the next piece's batch (its first bytes go out, the
  // sockets take the rest as they drain) before reducing the current piece.
  struct Batch {
    struct PeerQ {
      std::deque<const HostXfer*> sends, recvs;
      size_t soff = 0, roff = 0;
    };
    std::vector<PeerQ> q;
    size_t pending = 0;
    // The sends of a large batch, handed to the sender thread (null: this
    // thread moves them with the receives).
    std::unique_ptr<Batch> out;
  };
  vcclResult_t start(const std::vector<HostXfer>& xs, Batch* b);
  vcclResult_t finish(Batch* b);
  // The progress loop of one batch (this thread or the sender thread).
  vcclResult_t drive(Batch* b);
  // One non-blocking pass over every stream of the batch.
  vcclResult_t pass(Batch* b, bool* moved);
  // Pieces 0..pieces-1: xfers(k, slot, &xs) lists piece k's transfers into
  // buffer `slot` (0 or 1), reduce(k, slot) reduces it.
  template <typename X, typename R>
  vcclResult_t pipelined(size_t pieces, X xfers, R reduce);

  int rank_;
  int n_;
  const char* path_ = "host TCP mesh";
  std::vector<int> fd_;  // stream to each peer ([rank_] = -1)
  std::atomic<bool> aborted_{false};
  size_t chunk_ = 8u << 20;      // per-peer piece of a reduction (VCCL_HOST_CHUNK)
  // All-reduce whose whole message to every peer, (n - 1) x bytes, is at
  // most this: direct exchange (VCCL_HOST_AR_DIRECT).
  size_t directMax_ = 128u << 10;
  int spinUs_ = 50;               // retry without sleeping this long before poll() (VCCL_HOST_SPIN_US)
  // Reduction buffers kept across calls (a fresh allocation per call would
  // page-fault its way through every byte): [0] and [1] receive alternate
  // pieces, [2] holds a pre-multiplied copy of the input.
  std::vector<char> scratch_[3];
  char* scratch(int i, size_t bytes) {
    if (scratch_[i].size() < bytes) scratch_[i].resize(bytes);
    return scratch_[i].data();
  }
  size_t bcastDirect_ = 16u << 10;  // broadcast up to this: root to every rank (VCCL_HOST_BCAST_DIRECT)
  size_t bcastPiece_ = 1u << 20;    // ... above: per-receiver block of one piece (VCCL_HOST_BCAST_PIECE)

  // Sender thread: a batch that sends at least sendThreadMin_ bytes
  // (VCCL_HOST_SEND_THREAD_MIN; 0: never) hands its sends to it, so the
  // kernel's copies of outgoing bytes run on another core while this thread
  // receives and reduces.  One batch at a time (finish() waits for it).
  size_t sendThreadMin_ = 8u << 20;
  std::thread sender_;
  std::mutex sMu_;
  std::condition_variable sCv_, sDoneCv_;
  Batch* job_ = nullptr;
  bool jobDone_ = true;
  bool stop_ = false;
  vcclResult_t jobRes_ = vcclSuccess;
  void senderLoop();
  bool ensureSender();  // starts the thread once; false (and no hand-offs) if it cannot
  void handOff(Batch* sends);
  vcclResult_t waitHandOff();
};

// out = reduce over the contributions src[0..] in that order (count
// elements each): fp32 accumulation for 16- and 8-bit floats, avg divides
// by src.size() before the final rounding.  Pre-multiplication is applied
// before the data leaves its rank (hostScale), not here.
void hostReduce(char* out, const std::vector<const char*>& src, size_t count, const HostRed& r);
// out = in * scalar, rounded to the element type (float types).
void hostScale(char* out, const char* in, size_t count, vcclDataType_t dt, double scalar);

}  // namespace vccl
