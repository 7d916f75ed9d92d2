// libaether_rt: TCP transport for the host control plane and cross-host
// CPU collectives (POSIX sockets).
//
// Reference ABI (runtime/src/lib.rs:1585-1780): aether_tcp_{listen,
// listen_addr, listener_port, accept_one, connect, connect_host, send, recv,
// close, stream_close}. Handles are indices into listener / stream tables;
// streams get 30 s send / receive timeouts so a stuck peer surfaces as an
// error instead of a hang. Send and receive move at most n bytes and return
// the count (0 = peer closed, -1 = error); aether_tcp_send_all /
// aether_tcp_recv_all loop until all n bytes moved.
#include <arpa/inet.h>
#include <netdb.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <sys/socket.h>
#include <sys/time.h>
#include <unistd.h>

#include <cstdint>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

namespace {
std::mutex g_mu;
std::vector<int> g_listeners, g_streams;  // -1 = free slot

int64_t put(std::vector<int>& v, int fd) {
  std::lock_guard<std::mutex> g(g_mu);
  for (size_t i = 0; i < v.size(); ++i)
    if (v[i] < 0) {
      v[i] = fd;
      return (int64_t)i;
    }
  v.push_back(fd);
  return (int64_t)v.size() - 1;
}
int get(std::vector<int>& v, int64_t h) {
  std::lock_guard<std::mutex> g(g_mu);
  return (h < 0 || (size_t)h >= v.size()) ? -1 : v[(size_t)h];
}
int drop(std::vector<int>& v, int64_t h) {
  std::lock_guard<std::mutex> g(g_mu);
  if (h < 0 || (size_t)h >= v.size() || v[(size_t)h] < 0) return -1;
  ::close(v[(size_t)h]);
  v[(size_t)h] = -1;
  return 0;
}
void stream_opts(int fd) {
  timeval tv{30, 0};
  setsockopt(fd, SOL_SOCKET, SO_RCVTIMEO, &tv, sizeof(tv));
  setsockopt(fd, SOL_SOCKET, SO_SNDTIMEO, &tv, sizeof(tv));
  const int one = 1;
  setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));
}
int64_t listen_on(const char* host, int64_t port) {
  if (port < 0 || port > 65535) return -1;
  addrinfo hints{}, *res = nullptr;
  hints.ai_family = AF_UNSPEC;
  hints.ai_socktype = SOCK_STREAM;
  hints.ai_flags = AI_PASSIVE;
  if (getaddrinfo(host, std::to_string(port).c_str(), &hints, &res) != 0) return -1;
  int fd = -1;
  for (addrinfo* a = res; a; a = a->ai_next) {
    fd = socket(a->ai_family, a->ai_socktype, a->ai_protocol);
    if (fd < 0) continue;
    const int one = 1;
    setsockopt(fd, SOL_SOCKET, SO_REUSEADDR, &one, sizeof(one));
    if (bind(fd, a->ai_addr, a->ai_addrlen) == 0 && listen(fd, 64) == 0) break;
    ::close(fd);
    fd = -1;
  }
  freeaddrinfo(res);
  return fd < 0 ? -1 : put(g_listeners, fd);
}
int64_t connect_to(const char* host, int64_t port) {
  if (port < 0 || port > 65535) return -1;
  addrinfo hints{}, *res = nullptr;
  hints.ai_family = AF_UNSPEC;
  hints.ai_socktype = SOCK_STREAM;
  if (getaddrinfo(host, std::to_string(port).c_str(), &hints, &res) != 0) return -1;
  int fd = -1;
  for (addrinfo* a = res; a; a = a->ai_next) {
    fd = socket(a->ai_family, a->ai_socktype, a->ai_protocol);
    if (fd < 0) continue;
    if (connect(fd, a->ai_addr, a->ai_addrlen) == 0) break;
    ::close(fd);
    fd = -1;
  }
  freeaddrinfo(res);
  if (fd < 0) return -1;
  stream_opts(fd);
  return put(g_streams, fd);
}
}  // namespace

extern "C" {

int64_t aether_tcp_listen(int64_t port) { return listen_on("127.0.0.1", port); }

int64_t aether_tcp_listen_addr(int64_t addr, int addr_len, int64_t port) {
  if (addr == 0 || addr_len <= 0) return -1;
  const std::string host(reinterpret_cast<const char*>(addr), (size_t)addr_len);
  return listen_on(host.c_str(), port);
}

int64_t aether_tcp_listener_port(int64_t handle) {
  const int fd = get(g_listeners, handle);
  if (fd < 0) return -1;
  sockaddr_storage ss{};
  socklen_t len = sizeof(ss);
  if (getsockname(fd, reinterpret_cast<sockaddr*>(&ss), &len) != 0) return -1;
  if (ss.ss_family == AF_INET) return ntohs(reinterpret_cast<sockaddr_in*>(&ss)->sin_port);
  if (ss.ss_family == AF_INET6) return ntohs(reinterpret_cast<sockaddr_in6*>(&ss)->sin6_port);
  return -1;
}

int aether_tcp_close(int64_t handle) { return drop(g_listeners, handle); }

int64_t aether_tcp_accept_one(int64_t listener) {
  const int lfd = get(g_listeners, listener);
  if (lfd < 0) return -1;
  const int fd = accept(lfd, nullptr, nullptr);
  if (fd < 0) return -1;
  stream_opts(fd);
  return put(g_streams, fd);
}

int aether_tcp_stream_close(int64_t handle) { return drop(g_streams, handle); }

int64_t aether_tcp_connect(int64_t port) { return connect_to("127.0.0.1", port); }

int64_t aether_tcp_connect_host(int64_t host, int host_len, int64_t port) {
  if (host == 0 || host_len <= 0) return -1;
  const std::string h(reinterpret_cast<const char*>(host), (size_t)host_len);
  return connect_to(h.c_str(), port);
}

int64_t aether_tcp_send(int64_t stream, int64_t buf, int64_t n) {
  const int fd = get(g_streams, stream);
  if (fd < 0 || buf == 0 || n < 0) return -1;
  const ssize_t w = ::send(fd, reinterpret_cast<const void*>(buf), (size_t)n, MSG_NOSIGNAL);
  return w < 0 ? -1 : (int64_t)w;
}

int64_t aether_tcp_recv(int64_t stream, int64_t buf, int64_t n) {
  const int fd = get(g_streams, stream);
  if (fd < 0 || buf == 0 || n < 0) return -1;
  const ssize_t r = ::recv(fd, reinterpret_cast<void*>(buf), (size_t)n, 0);
  return r < 0 ? -1 : (int64_t)r;
}

int64_t aether_tcp_send_all(int64_t stream, int64_t buf, int64_t n) {
  int64_t done = 0;
  while (done < n) {
    const int64_t w = aether_tcp_send(stream, buf + done, n - done);
    if (w <= 0) return -1;
    done += w;
  }
  return done;
}

int64_t aether_tcp_recv_all(int64_t stream, int64_t buf, int64_t n) {
  int64_t done = 0;
  while (done < n) {
    const int64_t r = aether_tcp_recv(stream, buf + done, n - done);
    if (r <= 0) return -1;
    done += r;
  }
  return done;
}

}  // extern "C"
