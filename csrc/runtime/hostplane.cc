// SPDX-License-Identifier: Apache-2.0
// Host data plane over a TCP mesh (see hostplane.h).
#include "runtime/hostplane.h"

#include <arpa/inet.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <errno.h>
#include <poll.h>
#include <sys/socket.h>

#include <sched.h>

#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <exception>

#include "common/env.h"
#include "common/log.h"
#include "common/net.h"
#include "control/bootstrap.h"
#include "kernels/dtypes.cuh"

namespace vccl {

namespace {

#ifndef MSG_NOSIGNAL
#define MSG_NOSIGNAL 0
#endif

// Storage type S reduced in accumulation type A.
template <typename S>
struct Elem {
  using A = S;
  static A in(S v) { return v; }
  static S out(A v) { return v; }
};
template <>
struct Elem<__half> {
  using A = float;
  static A in(__half v) { return __half2float(v); }
  static __half out(A v) { return __float2half_rn(v); }
};
template <>
struct Elem<__nv_bfloat16> {
  using A = float;
  static A in(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __nv_bfloat16 out(A v) { return __float2bfloat16_rn(v); }
};
template <>
struct Elem<__nv_fp8_e4m3> {
  using A = float;
  static A in(__nv_fp8_e4m3 v) { return static_cast<float>(v); }
  static __nv_fp8_e4m3 out(A v) { return __nv_fp8_e4m3(v); }
};
template <>
struct Elem<__nv_fp8_e5m2> {
  using A = float;
  static A in(__nv_fp8_e5m2 v) { return static_cast<float>(v); }
  static __nv_fp8_e5m2 out(A v) { return __nv_fp8_e5m2(v); }
};

// acc[i] = acc[i] (op) x[i] over a block, one operation per loop so the
// compiler vectorises it.
template <typename S, typename A>
void foldBlock(A* acc, const S* x, size_t m, int kind) {
  using E = Elem<S>;
  switch (kind) {
    case dev::kProd:
      for (size_t i = 0; i < m; i++) acc[i] = static_cast<A>(acc[i] * E::in(x[i]));
      break;
    case dev::kMax:
      for (size_t i = 0; i < m; i++) {
        const A v = E::in(x[i]);
        acc[i] = acc[i] < v ? v : acc[i];
      }
      break;
    case dev::kMin:
      for (size_t i = 0; i < m; i++) {
        const A v = E::in(x[i]);
        acc[i] = v < acc[i] ? v : acc[i];
      }
      break;
    default:
      for (size_t i = 0; i < m; i++) acc[i] = static_cast<A>(acc[i] + E::in(x[i]));
      break;
  }
}

template <typename S>
void reduceT(char* out, const std::vector<const char*>& src, size_t count, const HostRed& r) {
  using E = Elem<S>;
  using A = typename E::A;
  const size_t n = src.size();
  S* o = reinterpret_cast<S*>(out);
  // Block by block: every contribution of a block is read into the
  // accumulator before the block is written (the output may be one of the
  // contributions, in place); per element the order is rank order.
  constexpr size_t kBlock = 2048;
  A acc[kBlock];
  for (size_t b = 0; b < count; b += kBlock) {
    const size_t m = count - b < kBlock ? count - b : kBlock;
    const S* s0 = reinterpret_cast<const S*>(src[0]) + b;
    for (size_t i = 0; i < m; i++) acc[i] = E::in(s0[i]);
    for (size_t p = 1; p < n; p++) foldBlock<S, A>(acc, reinterpret_cast<const S*>(src[p]) + b, m, r.kind);
    if (r.avg)
      for (size_t i = 0; i < m; i++) acc[i] = static_cast<A>(acc[i] / static_cast<A>(n));
    for (size_t i = 0; i < m; i++) o[b + i] = E::out(acc[i]);
  }
}

template <typename S>
void scaleT(char* out, const char* in, size_t count, double scalar) {
  using E = Elem<S>;
  using A = typename E::A;
  const S* x = reinterpret_cast<const S*>(in);
  S* o = reinterpret_cast<S*>(out);
  for (size_t i = 0; i < count; i++) o[i] = E::out(static_cast<A>(E::in(x[i]) * static_cast<A>(scalar)));
}

template <template <typename> class F, typename... Args>
void byType(vcclDataType_t dt, Args&&... args) {
  switch (dt) {
    case vcclInt8: F<int8_t>::run(args...); break;
    case vcclUint8: F<uint8_t>::run(args...); break;
    case vcclInt32: F<int32_t>::run(args...); break;
    case vcclUint32: F<uint32_t>::run(args...); break;
    case vcclInt64: F<int64_t>::run(args...); break;
    case vcclUint64: F<uint64_t>::run(args...); break;
    case vcclFloat16: F<__half>::run(args...); break;
    case vcclFloat32: F<float>::run(args...); break;
    case vcclFloat64: F<double>::run(args...); break;
    case vcclBfloat16: F<__nv_bfloat16>::run(args...); break;
    case vcclFloat8e4m3: F<__nv_fp8_e4m3>::run(args...); break;
    case vcclFloat8e5m2: F<__nv_fp8_e5m2>::run(args...); break;
    default: break;
  }
}

template <typename S>
struct ReduceF {
  static void run(char* out, const std::vector<const char*>& src, size_t count, const HostRed& r) {
    reduceT<S>(out, src, count, r);
  }
};
template <typename S>
struct ScaleF {
  static void run(char* out, const char* in, size_t count, double scalar) { scaleT<S>(out, in, count, scalar); }
};

size_t ceilDiv(size_t a, size_t b) { return (a + b - 1) / b; }

}  // namespace

void hostReduce(char* out, const std::vector<const char*>& src, size_t count, const HostRed& r) {
  byType<ReduceF>(r.dt, out, src, count, r);
}

void hostScale(char* out, const char* in, size_t count, vcclDataType_t dt, double scalar) {
  byType<ScaleF>(dt, out, in, count, scalar);
}

// ---- mesh --------------------------------------------------------------------

vcclResult_t HostPlane::create(Bootstrap* bs, std::unique_ptr<HostPlane>* out) {
  const int n = bs->nranks(), me = bs->rank();
  std::unique_ptr<HostPlane> hp(new HostPlane(me, n));
  hp->fd_.assign(n, -1);
  hp->chunk_ = envBytes("VCCL_HOST_CHUNK", 8u << 20);
  if (hp->chunk_ < 4096) hp->chunk_ = 4096;
  // 128 KiB sent per rank: paired runs put the crossover with reduce-scatter
  // + all-gather near 16 KiB messages at 8 ranks and 16-32 KiB at 4.
  hp->directMax_ = envBytes("VCCL_HOST_AR_DIRECT", 128u << 10);
  hp->spinUs_ = static_cast<int>(envLong("VCCL_HOST_SPIN_US", 50));
  hp->bcastDirect_ = envBytes("VCCL_HOST_BCAST_DIRECT", 16u << 10);
  hp->bcastPiece_ = envBytes("VCCL_HOST_BCAST_PIECE", 1u << 20);
  // 8 MiB: paired runs of 16 and 64 MiB all-reduce and reduce-scatter at 4
  // and 8 ranks measured the two-core form 10-25 % faster; smaller batches
  // gain less than the hand-off costs.
  hp->sendThreadMin_ = envBytes("VCCL_HOST_SEND_THREAD_MIN", 8u << 20);
  // Every rank listens, then the ranks exchange endpoints: a rank connects to
  // every higher rank (connections complete into the peer's backlog, so the
  // order cannot deadlock) and accepts every lower one.
  int lfd = -1;
  uint16_t port = 0;
  WireEndpoint mine{};
  bool ok = tcpListen(0, &lfd, &port) == vcclSuccess && localEndpoint(&mine) == vcclSuccess;
  mine.portBE = htons(port);
  struct Entry {
    WireEndpoint ep;
    int32_t ok;
  };
  std::vector<Entry> all(n);
  all[me] = Entry{mine, ok ? 1 : 0};
  vcclResult_t res = bs->allGather(all.data(), sizeof(Entry));
  if (res != vcclSuccess) {
    closeFd(lfd);
    return res;
  }
  for (const Entry& e : all) ok = ok && e.ok != 0;
  if (!ok) {
    closeFd(lfd);
    VERR("host data plane: a rank could not open its listening socket");
    return vcclSystemError;
  }
  for (int p = me + 1; p < n && res == vcclSuccess; p++) {
    int fd = -1;
    res = tcpConnect(all[p].ep, connectWindowMs(), &fd);
    const int32_t who = me;
    if (res == vcclSuccess) res = sendFull(fd, &who, sizeof(who));
    hp->fd_[p] = fd;
  }
  for (int k = 0; k < me && res == vcclSuccess; k++) {
    int fd = -1;
    res = tcpAccept(lfd, nullptr, &fd);
    int32_t who = -1;
    if (res == vcclSuccess) res = recvFull(fd, &who, sizeof(who));
    if (res == vcclSuccess && (who < 0 || who >= me || hp->fd_[who] >= 0)) {
      VERR("host data plane: unexpected connection (rank %d) on rank %d", who, me);
      res = vcclSystemError;
    }
    if (res == vcclSuccess) {
      hp->fd_[who] = fd;
    } else {
      closeFd(fd);
    }
  }
  closeFd(lfd);
  // Every rank learns whether every mesh link came up.
  const bool meshOk = everyone(bs, res == vcclSuccess);
  if (!meshOk) return res != vcclSuccess ? res : vcclSystemError;
  VINFO("host data plane: TCP mesh of %d ranks ready", n);
  *out = std::move(hp);
  return vcclSuccess;
}

HostPlane::~HostPlane() {
  if (sender_.joinable()) {
    {
      std::lock_guard<std::mutex> g(sMu_);
      stop_ = true;
    }
    sCv_.notify_one();
    sender_.join();
  }
  for (int fd : fd_) closeFd(fd);
}

void HostPlane::senderLoop() {
  std::unique_lock<std::mutex> lk(sMu_);
  for (;;) {
    sCv_.wait(lk, [&] { return stop_ || job_ != nullptr; });
    if (stop_) return;
    Batch* j = job_;
    lk.unlock();
    const vcclResult_t r = drive(j);
    lk.lock();
    job_ = nullptr;
    jobRes_ = r;
    jobDone_ = true;
    sDoneCv_.notify_all();
  }
}

bool HostPlane::ensureSender() {
  if (sender_.joinable()) return true;
  try {
    sender_ = std::thread([this] { senderLoop(); });
    return true;
  } catch (const std::exception& e) {
    VWARN("host data plane: no sender thread (%s); sends stay on the calling thread", e.what());
    sendThreadMin_ = 0;
    return false;
  }
}

void HostPlane::handOff(Batch* sends) {
  {
    std::lock_guard<std::mutex> g(sMu_);
    job_ = sends;
    jobDone_ = false;
  }
  sCv_.notify_one();
}

vcclResult_t HostPlane::waitHandOff() {
  std::unique_lock<std::mutex> lk(sMu_);
  sDoneCv_.wait(lk, [&] { return jobDone_; });
  return jobRes_;
}

void HostPlane::abort() {
  aborted_.store(true);
  for (int fd : fd_)
    if (fd >= 0) shutdownFd(fd);
}

// ---- progress loop ---------------------------------------------------------

vcclResult_t HostPlane::start(const std::vector<HostXfer>& xs, Batch* b) {
  b->q.assign(n_, Batch::PeerQ{});
  b->pending = 0;
  b->out.reset();
  size_t sendBytes = 0, recvBytes = 0;
  for (const HostXfer& x : xs) {
    if (x.peer < 0 || x.peer >= n_ || x.peer == rank_ || fd_[x.peer] < 0) {
      VERR("host data plane: transfer with invalid peer %d", x.peer);
      return vcclInternalError;
    }
    (x.send ? sendBytes : recvBytes) += x.bytes;
  }
  // Only a batch that also receives gains: its sends and receives then
  // copy on two cores at once.
  const bool split = sendThreadMin_ > 0 && sendBytes >= sendThreadMin_ && recvBytes > 0 && ensureSender();
  if (split) {
    b->out.reset(new Batch);
    b->out->q.assign(n_, Batch::PeerQ{});
  }
  for (const HostXfer& x : xs) {
    if (x.bytes == 0) continue;
    Batch* to = x.send && split ? b->out.get() : b;
    (x.send ? to->q[x.peer].sends : to->q[x.peer].recvs).push_back(&x);
    to->pending++;
  }
  if (split) handOff(b->out.get());
  bool moved = false;
  const vcclResult_t r = b->pending ? pass(b, &moved) : vcclSuccess;
  if (r != vcclSuccess && split) {
    // The caller's buffers must outlive the sender thread's use of them.
    abort();
    (void)waitHandOff();
    b->out.reset();
  }
  return r;
}

vcclResult_t HostPlane::pass(Batch* b, bool* moved) {
  if (aborted_.load()) {
    VERR("host data plane: communicator aborted");
    return vcclSystemError;
  }
  for (int p = 0; p < n_ && b->pending > 0; p++) {
    Batch::PeerQ& pq = b->q[p];
    // Send as much as the socket takes, then take what has arrived.
    while (!pq.sends.empty()) {
      const HostXfer* x = pq.sends.front();
      const ssize_t k = ::send(fd_[p], x->buf + pq.soff, x->bytes - pq.soff, MSG_DONTWAIT | MSG_NOSIGNAL);
      if (k > 0) {
        *moved = true;
        pq.soff += static_cast<size_t>(k);
        if (pq.soff == x->bytes) {
          pq.sends.pop_front();
          pq.soff = 0;
          b->pending--;
        }
        continue;
      }
      if (k < 0 && errno == EINTR) continue;
      if (k < 0 && (errno == EAGAIN || errno == EWOULDBLOCK)) break;
      VERR("host data plane: send to rank %d failed: %s", p, k == 0 ? "no progress" : strerror(errno));
      return vcclSystemError;
    }
    while (!pq.recvs.empty()) {
      const HostXfer* x = pq.recvs.front();
      const ssize_t k = ::recv(fd_[p], x->buf + pq.roff, x->bytes - pq.roff, MSG_DONTWAIT);
      if (k > 0) {
        *moved = true;
        pq.roff += static_cast<size_t>(k);
        if (pq.roff == x->bytes) {
          pq.recvs.pop_front();
          pq.roff = 0;
          b->pending--;
        }
        continue;
      }
      if (k == 0) {
        VERR("host data plane: rank %d closed its stream", p);
        return vcclSystemError;
      }
      if (errno == EINTR) continue;
      if (errno == EAGAIN || errno == EWOULDBLOCK) break;
      VERR("host data plane: recv from rank %d failed: %s", p, strerror(errno));
      return vcclSystemError;
    }
  }
  return vcclSuccess;
}

vcclResult_t HostPlane::finish(Batch* b) {
  vcclResult_t r = drive(b);
  if (b->out) {
    // A failed receive side stops the sends too (the streams are broken);
    // either way the sender thread is done with the caller's buffers on return.
    if (r != vcclSuccess) abort();
    const vcclResult_t rs = waitHandOff();
    b->out.reset();
    if (r == vcclSuccess) r = rs;
  }
  return r;
}

vcclResult_t HostPlane::drive(Batch* b) {
  Deadline dl;
  std::vector<pollfd> pfd;
  std::vector<int> who;
  const auto spin = std::chrono::microseconds(spinUs_);
  auto idleSince = std::chrono::steady_clock::now();
  while (b->pending > 0) {
    bool moved = false;
    VTRY(pass(b, &moved));
    if (b->pending == 0) break;
    if (moved) {
      idleSince = std::chrono::steady_clock::now();
      continue;
    }
    // Nothing moved: keep trying for a short while (an answer is often
    // microseconds away, and a sleep in poll() costs a wake-up), then wait
    // until some stream can move.
    if (std::chrono::steady_clock::now() - idleSince < spin) {
      sched_yield();
      continue;
    }
    pfd.clear();
    who.clear();
    for (int p = 0; p < n_; p++) {
      short ev = 0;
      if (!b->q[p].sends.empty()) ev |= POLLOUT;
      if (!b->q[p].recvs.empty()) ev |= POLLIN;
      if (ev) {
        pfd.push_back(pollfd{fd_[p], ev, 0});
        who.push_back(p);
      }
    }
    const int rc = ::poll(pfd.data(), pfd.size(), dl.pollSliceMs());
    if (rc < 0 && errno != EINTR) {
      VERR("host data plane: poll failed: %s", strerror(errno));
      return vcclSystemError;
    }
    for (size_t i = 0; rc > 0 && i < pfd.size(); i++) {
      // A closed or failed stream with nothing left to read is an error; with
      // data pending, the next pass reads it and then sees the close.
      if ((pfd[i].revents & (POLLERR | POLLNVAL)) != 0) {
        VERR("host data plane: stream to rank %d failed", who[i]);
        return vcclSystemError;
      }
    }
    if (rc == 0 && dl.expired()) {
      VERR("host data plane: timed out after VCCL_TIMEOUT=%ds", watchdogSeconds());
      return vcclSystemError;
    }
  }
  return vcclSuccess;
}

vcclResult_t HostPlane::run(const std::vector<HostXfer>& xs) {
  Batch b;
  VTRY(start(xs, &b));
  return finish(&b);
}

template <typename X, typename R>
vcclResult_t HostPlane::pipelined(size_t pieces, X xfers, R reduce) {
  if (pieces == 0) return vcclSuccess;
  std::vector<HostXfer> xs[2];
  Batch b[2];
  xfers(size_t{0}, 0, &xs[0]);
  VTRY(start(xs[0], &b[0]));
  VTRY(finish(&b[0]));
  for (size_t k = 0; k < pieces; k++) {
    const int s = static_cast<int>(k % 2), t = 1 - s;
    if (k + 1 < pieces) {
      xs[t].clear();
      xfers(k + 1, t, &xs[t]);
      VTRY(start(xs[t], &b[t]));
    }
    reduce(k, s);
    if (k + 1 < pieces) VTRY(finish(&b[t]));
  }
  return vcclSuccess;
}

// ---- collectives -----------------------------------------------------------

vcclResult_t HostPlane::allGather(const char* send, char* recv, size_t bytes) {
  path_ = "host TCP mesh";
  if (bytes == 0) return vcclSuccess;
  char* mine = recv + rank_ * bytes;
  if (mine != send) memmove(mine, send, bytes);
  std::vector<HostXfer> xs;
  for (int p = 0; p < n_; p++) {
    if (p == rank_) continue;
    xs.push_back({true, p, mine, bytes});
    xs.push_back({false, p, recv + p * bytes, bytes});
  }
  return run(xs);
}

vcclResult_t HostPlane::broadcast(const char* send, char* recv, size_t bytes, int root) {
  path_ = "host TCP mesh";
  if (bytes == 0) return vcclSuccess;
  const int m = n_ - 1;  // ranks that receive
  if (rank_ == root && recv != send) memmove(recv, send, bytes);
  if (bytes <= bcastDirect_ || m < 2) {
    // Small: the root sends the whole message to every rank.
    std::vector<HostXfer> xs;
    if (rank_ == root) {
      for (int p = 0; p < n_; p++)
        if (p != root) xs.push_back({true, p, recv, bytes});
    } else {
      xs.push_back({false, root, recv, bytes});
    }
    return run(xs);
  }
  path_ = "host TCP mesh, pieces";
  // Large: in pieces, the root hands receiver j the j-th block of each piece
  // (it sends every byte once), and the receivers exchange their blocks
  // among themselves; while they exchange one piece, the root's next piece
  // is already on its way into their sockets.
  const size_t piece = std::max<size_t>(bcastPiece_, 4096) * m;
  auto block = [&](size_t off, size_t len, int j, size_t* bo, size_t* bl) {
    const size_t b = ceilDiv(len, m);
    const size_t lo = std::min(len, static_cast<size_t>(j) * b), hi = std::min(len, static_cast<size_t>(j + 1) * b);
    *bo = off + lo;
    *bl = hi - lo;
  };
  auto receiver = [&](int j) { return (root + 1 + j) % n_; };
  if (rank_ == root) {
    std::vector<HostXfer> xs;
    for (size_t off = 0; off < bytes; off += piece) {
      const size_t len = std::min(piece, bytes - off);
      for (int j = 0; j < m; j++) {
        size_t bo = 0, bl = 0;
        block(off, len, j, &bo, &bl);
        xs.push_back({true, receiver(j), recv + bo, bl});
      }
    }
    return run(xs);
  }
  const int me = (rank_ - root - 1 + n_) % n_;
  for (size_t off = 0; off < bytes; off += piece) {
    const size_t len = std::min(piece, bytes - off);
    size_t mo = 0, ml = 0;
    block(off, len, me, &mo, &ml);
    VTRY(run({{false, root, recv + mo, ml}}));
    std::vector<HostXfer> xs;
    for (int j = 0; j < m; j++) {
      if (j == me) continue;
      size_t bo = 0, bl = 0;
      block(off, len, j, &bo, &bl);
      xs.push_back({true, receiver(j), recv + mo, ml});
      xs.push_back({false, receiver(j), recv + bo, bl});
    }
    VTRY(run(xs));
  }
  return vcclSuccess;
}

vcclResult_t HostPlane::gather(const char* send, char* recv, size_t bytes, int root) {
  path_ = "host TCP mesh";
  if (bytes == 0) return vcclSuccess;
  std::vector<HostXfer> xs;
  if (rank_ == root) {
    if (recv + root * bytes != send) memmove(recv + root * bytes, send, bytes);
    for (int p = 0; p < n_; p++)
      if (p != root) xs.push_back({false, p, recv + p * bytes, bytes});
  } else {
    xs.push_back({true, root, const_cast<char*>(send), bytes});
  }
  return run(xs);
}

vcclResult_t HostPlane::scatter(const char* send, char* recv, size_t bytes, int root) {
  path_ = "host TCP mesh";
  if (bytes == 0) return vcclSuccess;
  std::vector<HostXfer> xs;
  if (rank_ == root) {
    if (recv != send + root * bytes) memmove(recv, send + root * bytes, bytes);
    for (int p = 0; p < n_; p++)
      if (p != root) xs.push_back({true, p, const_cast<char*>(send + p * bytes), bytes});
  } else {
    xs.push_back({false, root, recv, bytes});
  }
  return run(xs);
}

vcclResult_t HostPlane::allToAllv(const char* send, const size_t* sc, const size_t* sd, char* recv,
                                  const size_t* rc, const size_t* rd) {
  path_ = "host TCP mesh";
  // A receive range that overlaps the send buffer would be overwritten
  // before it leaves: send from a copy then.
  size_t sEnd = 0, rEnd = 0;
  for (int p = 0; p < n_; p++) {
    sEnd = std::max(sEnd, sd[p] + sc[p]);
    rEnd = std::max(rEnd, rd[p] + rc[p]);
  }
  std::vector<char> copy;
  if (send < recv + rEnd && recv < send + sEnd) {
    copy.assign(send, send + sEnd);
    send = copy.data();
  }
  if (sc[rank_] > 0) memmove(recv + rd[rank_], send + sd[rank_], sc[rank_]);
  std::vector<HostXfer> xs;
  for (int s = 1; s < n_; s++) {
    const int to = (rank_ + s) % n_, from = (rank_ - s + n_) % n_;
    xs.push_back({true, to, const_cast<char*>(send + sd[to]), sc[to]});
    xs.push_back({false, from, recv + rd[from], rc[from]});
  }
  return run(xs);
}

vcclResult_t HostPlane::reduceScatter(const char* send, char* recv, size_t recvCount, const HostRed& r) {
  path_ = "host TCP mesh";
  const size_t es = vcclTypeSize(r.dt);
  if (recvCount == 0) return vcclSuccess;
  const size_t cb = recvCount * es;
  if (r.premul) {
    char* scaled = scratch(2, cb * n_);
    hostScale(scaled, send, recvCount * n_, r.dt, r.scalar);
    send = scaled;
  }
  const size_t pe = std::max<size_t>(1, chunk_ / es);
  const size_t ps = std::min(pe, recvCount);  // elements of one peer's piece in a buffer
  char* tmp[2] = {scratch(0, ps * es * n_), scratch(1, ps * es * n_)};
  std::vector<const char*> src(n_);
  auto len = [&](size_t k) { return std::min(pe, recvCount - k * pe); };
  return pipelined(
      ceilDiv(recvCount, pe),
      [&](size_t k, int slot, std::vector<HostXfer>* xs) {
        const size_t off = k * pe, m = len(k);
        for (int p = 0; p < n_; p++) {
          if (p == rank_) continue;
          xs->push_back({true, p, const_cast<char*>(send + p * cb + off * es), m * es});
          xs->push_back({false, p, tmp[slot] + p * ps * es, m * es});
        }
      },
      [&](size_t k, int slot) {
        const size_t off = k * pe, m = len(k);
        for (int p = 0; p < n_; p++) src[p] = p == rank_ ? send + rank_ * cb + off * es : tmp[slot] + p * ps * es;
        hostReduce(recv + off * es, src, m, r);
      });
}

vcclResult_t HostPlane::reduce(const char* send, char* recv, size_t count, const HostRed& r, int root) {
  path_ = "host TCP mesh";
  const size_t es = vcclTypeSize(r.dt);
  if (count == 0) return vcclSuccess;
  if (r.premul) {
    char* scaled = scratch(2, count * es);
    hostScale(scaled, send, count, r.dt, r.scalar);
    send = scaled;
  }
  const size_t pe = std::max<size_t>(1, chunk_ / es);
  if (rank_ != root) {
    std::vector<HostXfer> xs{{true, root, const_cast<char*>(send), count * es}};
    return run(xs);
  }
  const size_t ps = std::min(pe, count);
  char* tmp[2] = {scratch(0, ps * es * n_), scratch(1, ps * es * n_)};
  std::vector<const char*> src(n_);
  auto len = [&](size_t k) { return std::min(pe, count - k * pe); };
  return pipelined(
      ceilDiv(count, pe),
      [&](size_t k, int slot, std::vector<HostXfer>* xs) {
        for (int p = 0; p < n_; p++)
          if (p != rank_) xs->push_back({false, p, tmp[slot] + p * ps * es, len(k) * es});
      },
      [&](size_t k, int slot) {
        const size_t off = k * pe;
        for (int p = 0; p < n_; p++) src[p] = p == rank_ ? send + off * es : tmp[slot] + p * ps * es;
        hostReduce(recv + off * es, src, len(k), r);
      });
}

vcclResult_t HostPlane::allReduce(const char* send, char* recv, size_t count, const HostRed& r) {
  path_ = "host TCP mesh";
  const size_t es = vcclTypeSize(r.dt);
  if (count == 0) return vcclSuccess;
  const size_t bytes = count * es;
  if (r.premul) {
    char* scaled = scratch(2, bytes);
    hostScale(scaled, send, count, r.dt, r.scalar);
    send = scaled;
  }
  std::vector<const char*> src(n_);
  bool direct = bytes * static_cast<size_t>(n_ - 1) <= directMax_;
  // VCCL_ALLREDUCE_ALGO forces the path, read on every call as on the device
  // (every rank sets it alike): ring / twoshot -> reduce-scatter + all-gather,
  // recdouble / oneshot / ll -> direct (the reference's two families under
  // its own names, reference: src/core/collectives.cc:525-534).
  if (const char* f = std::getenv("VCCL_ALLREDUCE_ALGO")) {
    if (std::strcmp(f, "ring") == 0 || std::strcmp(f, "twoshot") == 0) direct = false;
    else if (std::strcmp(f, "recdouble") == 0 || std::strcmp(f, "oneshot") == 0 || std::strcmp(f, "ll") == 0)
      direct = true;
  }
  if (direct || count < static_cast<size_t>(n_)) {
    // Small: every rank sends the whole message to every peer and reduces
    // the n copies in rank order.
    path_ = "host TCP mesh, direct";
    char* tmp = scratch(0, bytes * n_);
    std::vector<HostXfer> xs;
    for (int p = 0; p < n_; p++) {
      if (p == rank_) continue;
      xs.push_back({true, p, const_cast<char*>(send), bytes});
      xs.push_back({false, p, tmp + p * bytes, bytes});
    }
    VTRY(run(xs));
    for (int p = 0; p < n_; p++) src[p] = p == rank_ ? send : tmp + p * bytes;
    hostReduce(recv, src, count, r);
    return vcclSuccess;
  }
  // Large: rank q owns elements [q * bc, (q + 1) * bc) (the last block may be
  // shorter); reduce-scatter in pieces, then all-gather of the owned blocks.
  path_ = "host TCP mesh, reduce-scatter + all-gather";
  const size_t bc = ceilDiv(count, n_);
  auto blkOff = [&](int q) { return std::min(static_cast<size_t>(q) * bc, count); };
  auto blkLen = [&](int q) { return std::min(static_cast<size_t>(q + 1) * bc, count) - blkOff(q); };
  const size_t pe = std::max<size_t>(1, chunk_ / es);
  const size_t ps = std::min(pe, bc);  // elements of one peer's piece in a buffer
  char* tmp[2] = {scratch(0, ps * es * n_), scratch(1, ps * es * n_)};
  auto len = [&](int q, size_t off) { return blkLen(q) > off ? std::min(pe, blkLen(q) - off) : size_t{0}; };
  VTRY(pipelined(
      ceilDiv(bc, pe),
      [&](size_t k, int slot, std::vector<HostXfer>* xs) {
        const size_t off = k * pe, mine = len(rank_, off);
        for (int p = 0; p < n_; p++) {
          if (p == rank_) continue;
          xs->push_back({true, p, const_cast<char*>(send + (blkOff(p) + off) * es), len(p, off) * es});
          xs->push_back({false, p, tmp[slot] + p * ps * es, mine * es});
        }
      },
      [&](size_t k, int slot) {
        const size_t off = k * pe, mine = len(rank_, off);
        if (mine == 0) return;
        for (int p = 0; p < n_; p++)
          src[p] = p == rank_ ? send + (blkOff(rank_) + off) * es : tmp[slot] + p * ps * es;
        hostReduce(recv + (blkOff(rank_) + off) * es, src, mine, r);
      }));
  std::vector<HostXfer> xs;
  for (int p = 0; p < n_; p++) {
    if (p == rank_) continue;
    xs.push_back({true, p, recv + blkOff(rank_) * es, blkLen(rank_) * es});
    xs.push_back({false, p, recv + blkOff(p) * es, blkLen(p) * es});
  }
  return run(xs);
}

}  // namespace vccl
