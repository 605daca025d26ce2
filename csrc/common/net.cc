// SPDX-License-Identifier: Apache-2.0
// Sockets for the control plane: advertised address choice, listen /
// connect with retry, exact-size send and receive, and descriptor passing
// over Unix sockets (reference: src/util/socket.cc:89-339 for the TCP part;
// the SCM_RIGHTS part has no counterpart there).
#include "common/net.h"

#include <arpa/inet.h>
#include <errno.h>
#include <fcntl.h>
#include <ifaddrs.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <poll.h>
#include <sys/un.h>
#include <unistd.h>

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <thread>

#include "common/env.h"
#include "common/log.h"

namespace vccl {
namespace {

constexpr uint16_t kFamV4 = 1;
constexpr uint16_t kFamV6 = 2;

#ifdef MSG_NOSIGNAL
constexpr int kNoSig = MSG_NOSIGNAL;
#else
constexpr int kNoSig = 0;
#endif

void tuneTcp(int fd) {
  int on = 1;
  setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &on, sizeof(on));
}

bool aborted(const std::atomic<bool>* f) {
  return f != nullptr && f->load(std::memory_order_relaxed);
}

// Wait until fd is ready for `events` or the deadline/abort fires.
vcclResult_t waitReady(int fd, short events, const Deadline& dl,
                       const std::atomic<bool>* abortFlag, const char* what) {
  for (;;) {
    if (aborted(abortFlag)) {
      VERR("%s: communicator aborted", what);
      return vcclSystemError;
    }
    pollfd p{fd, events, 0};
    int rc = poll(&p, 1, dl.pollSliceMs());
    if (rc > 0) return vcclSuccess;
    if (rc < 0 && errno != EINTR) {
      VERR("%s: poll failed: %s", what, strerror(errno));
      return vcclSystemError;
    }
    if (dl.expired()) {
      VERR("%s: timed out after VCCL_TIMEOUT=%ds", what, watchdogSeconds());
      return vcclSystemError;
    }
  }
}

socklen_t toSockaddr(const WireEndpoint& ep, sockaddr_storage* ss) {
  memset(ss, 0, sizeof(*ss));
  if (ep.family == kFamV6) {
    auto* s6 = reinterpret_cast<sockaddr_in6*>(ss);
    s6->sin6_family = AF_INET6;
    s6->sin6_port = ep.portBE;
    memcpy(&s6->sin6_addr, ep.addr, 16);
    return sizeof(sockaddr_in6);
  }
  auto* s4 = reinterpret_cast<sockaddr_in*>(ss);
  s4->sin_family = AF_INET;
  s4->sin_port = ep.portBE;
  memcpy(&s4->sin_addr, ep.addr, 4);
  return sizeof(sockaddr_in);
}

sockaddr_un abstractAddr(const std::string& name, socklen_t* len) {
  sockaddr_un a;
  memset(&a, 0, sizeof(a));
  a.sun_family = AF_UNIX;
  // Leading NUL = Linux abstract namespace.
  size_t n = std::min(name.size(), sizeof(a.sun_path) - 2);
  memcpy(a.sun_path + 1, name.data(), n);
  *len = static_cast<socklen_t>(offsetof(sockaddr_un, sun_path) + 1 + n);
  return a;
}

}  // namespace

std::string endpointString(const WireEndpoint& ep) {
  char host[INET6_ADDRSTRLEN] = "?";
  inet_ntop(ep.family == kFamV6 ? AF_INET6 : AF_INET, ep.addr, host, sizeof(host));
  char out[INET6_ADDRSTRLEN + 8];
  std::snprintf(out, sizeof(out), "%s:%u", host, endpointPort(ep));
  return out;
}

uint16_t endpointPort(const WireEndpoint& ep) { return ntohs(ep.portBE); }

vcclResult_t parseEndpoint(const char* hostPort, WireEndpoint* out) {
  memset(out, 0, sizeof(*out));
  const char* colon = hostPort ? strrchr(hostPort, ':') : nullptr;
  if (colon == nullptr || colon == hostPort) return vcclInvalidArgument;
  std::string host(hostPort, colon - hostPort);
  if (host.size() > 2 && host.front() == '[' && host.back() == ']')
    host = host.substr(1, host.size() - 2);
  long port = std::strtol(colon + 1, nullptr, 10);
  if (port <= 0 || port > 65535) return vcclInvalidArgument;
  out->portBE = htons(static_cast<uint16_t>(port));
  if (inet_pton(AF_INET, host.c_str(), out->addr) == 1) {
    out->family = kFamV4;
    return vcclSuccess;
  }
  if (inet_pton(AF_INET6, host.c_str(), out->addr) == 1) {
    out->family = kFamV6;
    return vcclSuccess;
  }
  return vcclInvalidArgument;
}

vcclResult_t localEndpoint(WireEndpoint* out) {
  memset(out, 0, sizeof(*out));
  std::string forced = envStr("VCCL_SOCKET_ADDR", "");
  if (!forced.empty()) {
    if (inet_pton(AF_INET, forced.c_str(), out->addr) == 1) {
      out->family = kFamV4;
      return vcclSuccess;
    }
    if (inet_pton(AF_INET6, forced.c_str(), out->addr) == 1) {
      out->family = kFamV6;
      return vcclSuccess;
    }
    VERR("VCCL_SOCKET_ADDR='%s' is not an IP address", forced.c_str());
    return vcclInvalidArgument;
  }
  std::string ifname = envStr("VCCL_SOCKET_IFNAME", "");
  ifaddrs* list = nullptr;
  if (getifaddrs(&list) != 0) {
    VERR("getifaddrs failed: %s", strerror(errno));
    return vcclSystemError;
  }
  const sockaddr_in* pick = nullptr;
  const sockaddr_in* loop = nullptr;
  for (ifaddrs* it = list; it != nullptr; it = it->ifa_next) {
    if (it->ifa_addr == nullptr || it->ifa_addr->sa_family != AF_INET) continue;
    const auto* s4 = reinterpret_cast<const sockaddr_in*>(it->ifa_addr);
    if (!ifname.empty()) {
      if (ifname == it->ifa_name) { pick = s4; break; }
      continue;
    }
    bool isLoop = (ntohl(s4->sin_addr.s_addr) >> 24) == 127;
    if (isLoop) {
      if (loop == nullptr) loop = s4;
    } else if (pick == nullptr) {
      pick = s4;
    }
  }
  if (pick == nullptr) pick = loop;
  vcclResult_t res = vcclSuccess;
  if (pick == nullptr) {
    VERR("no IPv4 interface%s%s", ifname.empty() ? "" : " named ", ifname.c_str());
    res = vcclSystemError;
  } else {
    out->family = kFamV4;
    memcpy(out->addr, &pick->sin_addr, 4);
  }
  freeifaddrs(list);
  return res;
}

vcclResult_t tcpListen(uint16_t port, int* fd, uint16_t* boundPort) {
  int s = socket(AF_INET, SOCK_STREAM | SOCK_CLOEXEC, 0);
  if (s < 0) return vcclSystemError;
  int on = 1;
  setsockopt(s, SOL_SOCKET, SO_REUSEADDR, &on, sizeof(on));
  sockaddr_in a{};
  a.sin_family = AF_INET;
  a.sin_addr.s_addr = htonl(INADDR_ANY);
  a.sin_port = htons(port);
  if (bind(s, reinterpret_cast<sockaddr*>(&a), sizeof(a)) != 0 || listen(s, 256) != 0) {
    VERR("tcp listen on port %u failed: %s", port, strerror(errno));
    close(s);
    return vcclSystemError;
  }
  socklen_t len = sizeof(a);
  getsockname(s, reinterpret_cast<sockaddr*>(&a), &len);
  if (boundPort) *boundPort = ntohs(a.sin_port);
  *fd = s;
  return vcclSuccess;
}

vcclResult_t tcpConnect(const WireEndpoint& ep, int windowMs, int* fd) {
  sockaddr_storage ss;
  socklen_t len = toSockaddr(ep, &ss);
  auto end = std::chrono::steady_clock::now() + std::chrono::milliseconds(windowMs);
  int backoffMs = 10;
  for (;;) {
    int s = socket(ss.ss_family, SOCK_STREAM | SOCK_CLOEXEC, 0);
    if (s < 0) return vcclSystemError;
    if (connect(s, reinterpret_cast<sockaddr*>(&ss), len) == 0) {
      tuneTcp(s);
      *fd = s;
      return vcclSuccess;
    }
    int err = errno;
    close(s);
    if (std::chrono::steady_clock::now() >= end) {
      VERR("connect to %s failed: %s", endpointString(ep).c_str(), strerror(err));
      return vcclSystemError;
    }
    std::this_thread::sleep_for(std::chrono::milliseconds(backoffMs));
    backoffMs = std::min(backoffMs * 2, 400);
  }
}

vcclResult_t tcpAccept(int listenFd, const std::atomic<bool>* abortFlag, int* fd) {
  Deadline dl;
  for (;;) {
    VTRY(waitReady(listenFd, POLLIN, dl, abortFlag, "accept"));
    int s = accept4(listenFd, nullptr, nullptr, SOCK_CLOEXEC);
    if (s >= 0) {
      tuneTcp(s);
      *fd = s;
      return vcclSuccess;
    }
    if (errno == EINTR || errno == EAGAIN || errno == ECONNABORTED) continue;
    VERR("accept failed: %s", strerror(errno));
    return vcclSystemError;
  }
}

vcclResult_t sendFull(int fd, const void* buf, size_t n, const std::atomic<bool>* abortFlag) {
  const char* p = static_cast<const char*>(buf);
  Deadline dl;
  while (n > 0) {
    ssize_t k = send(fd, p, n, kNoSig | MSG_DONTWAIT);
    if (k > 0) {
      p += k;
      n -= static_cast<size_t>(k);
      continue;
    }
    if (k < 0 && errno == EINTR) continue;
    if (k < 0 && (errno == EAGAIN || errno == EWOULDBLOCK)) {
      VTRY(waitReady(fd, POLLOUT, dl, abortFlag, "send"));
      continue;
    }
    VERR("send failed: %s", k == 0 ? "connection closed" : strerror(errno));
    return vcclSystemError;
  }
  return vcclSuccess;
}

vcclResult_t recvFull(int fd, void* buf, size_t n, const std::atomic<bool>* abortFlag) {
  char* p = static_cast<char*>(buf);
  Deadline dl;
  while (n > 0) {
    ssize_t k = recv(fd, p, n, MSG_DONTWAIT);
    if (k > 0) {
      p += k;
      n -= static_cast<size_t>(k);
      continue;
    }
    if (k == 0) {
      VERR("recv failed: peer closed the connection");
      return vcclSystemError;
    }
    if (errno == EINTR) continue;
    if (errno == EAGAIN || errno == EWOULDBLOCK) {
      VTRY(waitReady(fd, POLLIN, dl, abortFlag, "recv"));
      continue;
    }
    VERR("recv failed: %s", strerror(errno));
    return vcclSystemError;
  }
  return vcclSuccess;
}

vcclResult_t unixListen(const std::string& name, int* fd) {
  int s = socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
  if (s < 0) return vcclSystemError;
  socklen_t len;
  sockaddr_un a = abstractAddr(name, &len);
  if (bind(s, reinterpret_cast<sockaddr*>(&a), len) != 0 || listen(s, 256) != 0) {
    VERR("unix listen '%s' failed: %s", name.c_str(), strerror(errno));
    close(s);
    return vcclSystemError;
  }
  *fd = s;
  return vcclSuccess;
}

vcclResult_t unixConnect(const std::string& name, int windowMs, int* fd) {
  socklen_t len;
  sockaddr_un a = abstractAddr(name, &len);
  auto end = std::chrono::steady_clock::now() + std::chrono::milliseconds(windowMs);
  for (;;) {
    int s = socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
    if (s < 0) return vcclSystemError;
    if (connect(s, reinterpret_cast<sockaddr*>(&a), len) == 0) {
      *fd = s;
      return vcclSuccess;
    }
    int err = errno;
    close(s);
    if (std::chrono::steady_clock::now() >= end) {
      VERR("unix connect '%s' failed: %s", name.c_str(), strerror(err));
      return vcclSystemError;
    }
    std::this_thread::sleep_for(std::chrono::milliseconds(5));
  }
}

vcclResult_t sendWithFds(int sock, const void* payload, size_t n, const std::vector<int>& fds) {
  if (n == 0) return vcclInvalidArgument;  // SCM_RIGHTS needs at least one data byte
  std::vector<char> ctrl(CMSG_SPACE(sizeof(int) * (fds.empty() ? 1 : fds.size())), 0);
  iovec iov{const_cast<void*>(payload), n};
  msghdr msg{};
  msg.msg_iov = &iov;
  msg.msg_iovlen = 1;
  if (!fds.empty()) {
    msg.msg_control = ctrl.data();
    msg.msg_controllen = CMSG_SPACE(sizeof(int) * fds.size());
    cmsghdr* c = CMSG_FIRSTHDR(&msg);
    c->cmsg_level = SOL_SOCKET;
    c->cmsg_type = SCM_RIGHTS;
    c->cmsg_len = CMSG_LEN(sizeof(int) * fds.size());
    memcpy(CMSG_DATA(c), fds.data(), sizeof(int) * fds.size());
  }
  for (;;) {
    ssize_t k = sendmsg(sock, &msg, kNoSig);
    if (k == static_cast<ssize_t>(n)) return vcclSuccess;
    if (k < 0 && errno == EINTR) continue;
    if (k >= 0) {
      // Descriptors went with the first byte; push the rest as plain data.
      return sendFull(sock, static_cast<const char*>(payload) + k, n - static_cast<size_t>(k));
    }
    VERR("sendmsg(SCM_RIGHTS) failed: %s", strerror(errno));
    return vcclSystemError;
  }
}

vcclResult_t recvWithFds(int sock, void* payload, size_t n, size_t maxFds, std::vector<int>* fds) {
  std::vector<char> ctrl(CMSG_SPACE(sizeof(int) * (maxFds ? maxFds : 1)), 0);
  iovec iov{payload, n};
  msghdr msg{};
  msg.msg_iov = &iov;
  msg.msg_iovlen = 1;
  msg.msg_control = ctrl.data();
  msg.msg_controllen = ctrl.size();
  Deadline dl;
  ssize_t k;
  for (;;) {
    k = recvmsg(sock, &msg, MSG_CMSG_CLOEXEC | MSG_DONTWAIT);
    if (k >= 0) break;
    if (errno == EINTR) continue;
    if (errno == EAGAIN || errno == EWOULDBLOCK) {
      VTRY(waitReady(sock, POLLIN, dl, nullptr, "recvmsg"));
      continue;
    }
    VERR("recvmsg failed: %s", strerror(errno));
    return vcclSystemError;
  }
  if (k == 0) {
    VERR("recvmsg: peer closed the connection");
    return vcclSystemError;
  }
  fds->clear();
  for (cmsghdr* c = CMSG_FIRSTHDR(&msg); c != nullptr; c = CMSG_NXTHDR(&msg, c)) {
    if (c->cmsg_level == SOL_SOCKET && c->cmsg_type == SCM_RIGHTS) {
      size_t cnt = (c->cmsg_len - CMSG_LEN(0)) / sizeof(int);
      const int* p = reinterpret_cast<const int*>(CMSG_DATA(c));
      fds->insert(fds->end(), p, p + cnt);
    }
  }
  if (static_cast<size_t>(k) < n)
    return recvFull(sock, static_cast<char*>(payload) + k, n - static_cast<size_t>(k));
  return vcclSuccess;
}

void closeFd(int fd) {
  if (fd >= 0) close(fd);
}

void shutdownFd(int fd) {
  if (fd >= 0) shutdown(fd, SHUT_RDWR);
}

}  // namespace vccl
