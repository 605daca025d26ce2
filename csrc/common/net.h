// SPDX-License-Identifier: Apache-2.0
// Socket helpers for the out-of-band control plane.
//
// TCP carries the rendezvous and small allgathers (the reference's bootstrap
// role, reference: src/util/socket.h:25-81).  Unix-domain sockets carry
// file descriptors (SCM_RIGHTS) between the ranks of one host: that is how
// CUDA VMM and multicast POSIX-fd handles reach the peers, which a TCP
// stream cannot do.
#pragma once

#include <sys/socket.h>

#include <atomic>
#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

#include "vccl.h"

namespace vccl {

// Portable 20-byte wire address: fixed family codes (1 = IPv4, 2 = IPv6),
// port in network byte order, address bytes (IPv4 in the first four).
struct WireEndpoint {
  uint16_t family;
  uint16_t portBE;
  uint8_t addr[16];
};
static_assert(sizeof(WireEndpoint) == 20, "wire endpoint must be packed");

std::string endpointString(const WireEndpoint& ep);
uint16_t endpointPort(const WireEndpoint& ep);

// Address this host advertises: VCCL_SOCKET_ADDR, else the IPv4 address of
// VCCL_SOCKET_IFNAME, else the first non-loopback IPv4, else loopback.
vcclResult_t localEndpoint(WireEndpoint* out);
vcclResult_t parseEndpoint(const char* hostPort, WireEndpoint* out);

vcclResult_t tcpListen(uint16_t port, int* fd, uint16_t* boundPort);
vcclResult_t tcpConnect(const WireEndpoint& ep, int windowMs, int* fd);
// Waits for one connection; `abortFlag` (may be null) ends the wait early.
vcclResult_t tcpAccept(int listenFd, const std::atomic<bool>* abortFlag, int* fd);

vcclResult_t sendFull(int fd, const void* buf, size_t n,
                      const std::atomic<bool>* abortFlag = nullptr);
vcclResult_t recvFull(int fd, void* buf, size_t n,
                      const std::atomic<bool>* abortFlag = nullptr);

// Abstract-namespace Unix stream sockets (no filesystem entry to clean up).
vcclResult_t unixListen(const std::string& name, int* fd);
vcclResult_t unixConnect(const std::string& name, int windowMs, int* fd);
// Send `payload` plus the descriptors in `fds` in one message.
vcclResult_t sendWithFds(int sock, const void* payload, size_t n,
                         const std::vector<int>& fds);
// Receive exactly `n` payload bytes and up to `maxFds` descriptors.
vcclResult_t recvWithFds(int sock, void* payload, size_t n, size_t maxFds,
                         std::vector<int>* fds);

void closeFd(int fd);
void shutdownFd(int fd);

}  // namespace vccl
