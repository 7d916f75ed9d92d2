// aether-allreduce: all-reduce of n f32 values across hosts over TCP.
//
// Rank 0 is the rendezvous: it accepts world_size - 1 connections, receives
// every peer's buffer (each prefixed with its rank), sums them with its own,
// and sends the sum back; every other rank connects, sends its buffer and
// receives the sum. Reference behaviour: trainer/src/bin/allreduce.rs (a star
// all-reduce used as the cross-host CPU fallback). The GPU collectives of
// this package run inside one NVLink domain through torch.distributed and its
// own kernels; this tool covers the host-to-host case.
//
//   aether-allreduce --role server --port 28080 --world-size 3 --rank 0 --n 16 --value 1
//   aether-allreduce --role client --host 10.0.0.1 --port 28080 --world-size 3 --rank 1 --n 16 --value 2
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include <algorithm>
#include <ctime>

extern "C" {
int64_t aether_tcp_listen_addr(int64_t, int, int64_t);
int64_t aether_tcp_accept_one(int64_t);
int64_t aether_tcp_connect_host(int64_t, int, int64_t);
int64_t aether_tcp_send_all(int64_t, int64_t, int64_t);
int64_t aether_tcp_recv_all(int64_t, int64_t, int64_t);
int aether_tcp_close(int64_t);
int aether_tcp_stream_close(int64_t);
}

int main(int argc, char** argv) {
  std::string role = "server", host = "127.0.0.1";
  int64_t port = 28080;
  int world = 2, rank = 0, n = 16;
  float value = 1.f;
  for (int i = 1; i < argc; ++i) {
    const std::string a = argv[i];
    auto next = [&]() { return i + 1 < argc ? std::string(argv[++i]) : std::string(); };
    if (a == "--role") role = next();
    else if (a == "--host") host = next();
    else if (a == "--port") port = std::atoll(next().c_str());
    else if (a == "--world-size") world = std::atoi(next().c_str());
    else if (a == "--rank") rank = std::atoi(next().c_str());
    else if (a == "--n") n = std::atoi(next().c_str());
    else if (a == "--value") value = (float)std::atof(next().c_str());
    else {
      std::fprintf(stderr, "unknown flag %s\n", a.c_str());
      return 2;
    }
  }
  if (world < 1 || n < 0 || rank < 0 || rank >= world) {
    std::fprintf(stderr, "bad --world-size / --rank / --n\n");
    return 2;
  }
  std::vector<float> buf((size_t)n, value), tmp((size_t)n);
  const int64_t bytes = (int64_t)n * 4;
  if (role == "server") {
    const int64_t l = aether_tcp_listen_addr((int64_t)(intptr_t)host.data(), (int)host.size(), port);
    if (l < 0) {
      std::fprintf(stderr, "[aether-allreduce] cannot listen on %s:%lld\n", host.c_str(), (long long)port);
      return 1;
    }
    std::vector<int64_t> peers;
    for (int p = 1; p < world; ++p) {
      const int64_t s = aether_tcp_accept_one(l);
      int32_t peer_rank = -1;
      if (s < 0 || aether_tcp_recv_all(s, (int64_t)(intptr_t)&peer_rank, 4) != 4 ||
          aether_tcp_recv_all(s, (int64_t)(intptr_t)tmp.data(), bytes) != bytes) {
        std::fprintf(stderr, "[aether-allreduce] peer %d failed\n", p);
        return 1;
      }
      for (int i = 0; i < n; ++i) buf[(size_t)i] += tmp[(size_t)i];
      peers.push_back(s);
    }
    for (int64_t s : peers) {
      if (aether_tcp_send_all(s, (int64_t)(intptr_t)buf.data(), bytes) != bytes) return 1;
      aether_tcp_stream_close(s);
    }
    aether_tcp_close(l);
  } else {
    int64_t s = -1;
    for (int tries = 0; tries < 100 && s < 0; ++tries) {  // the server may not be up yet
      s = aether_tcp_connect_host((int64_t)(intptr_t)host.data(), (int)host.size(), port);
      if (s < 0) {
        struct timespec ts = {0, 100000000};
        nanosleep(&ts, nullptr);
      }
    }
    const int32_t r = rank;
    if (s < 0 || aether_tcp_send_all(s, (int64_t)(intptr_t)&r, 4) != 4 ||
        aether_tcp_send_all(s, (int64_t)(intptr_t)buf.data(), bytes) != bytes ||
        aether_tcp_recv_all(s, (int64_t)(intptr_t)buf.data(), bytes) != bytes) {
      std::fprintf(stderr, "[aether-allreduce] rank %d: exchange with %s:%lld failed\n", rank, host.c_str(),
                   (long long)port);
      return 1;
    }
    aether_tcp_stream_close(s);
  }
  std::printf("rank=%d n=%d sum[0..%d]=", rank, n, std::min(n, 4));
  for (int i = 0; i < std::min(n, 4); ++i) std::printf("%s%g", i ? "," : "", buf[(size_t)i]);
  std::printf("\n");
  return 0;
}
