// libaether_rt: the generic collective ABI, real across processes.
//
// Reference surface (runtime/src/lib.rs:3277-3330, :670, :700; ABI.md
// "Distributed"): aether_op_{broadcast,all_gather,reduce_scatter,send,recv,
// all_to_all}_f32, aether_op_all_reduce_sum_f32 and aether_dist_all_reduce.
// The reference ships them as single-rank pass-throughs. Here they run over a
// process-wide default communicator:
//
//   * world 1 (no WORLD_SIZE / AETHER_WORLD_SIZE above 1): the single-rank
//     semantics of the reference (copies into the caller's buffer);
//   * world > 1: every process sets its rank and world size (AETHER_RANK /
//     AETHER_WORLD_SIZE, else RANK / WORLD_SIZE) and the same rendezvous in
//     AETHER_COMM_ADDR ("host:port"). On first use rank 0 listens there, every
//     other rank connects and reports the address of its own listener
//     (AETHER_COMM_HOST, default 127.0.0.1, on an ephemeral port); rank 0
//     sends the table back and ranks i < j connect pairwise, giving a full mesh
//     of TCP streams (tcp.cpp), so point-to-point calls go straight between
//     the two ranks.
//
// Shapes (n is per block): all_gather src [n] -> dst [world * n];
// reduce_scatter src [world * n] -> dst [n] = sum over ranks of block `rank`;
// all_to_all src [world * n] -> dst [world * n], block p of rank q's src
// lands in block q of rank p's dst; broadcast buf [n] from root; send / recv
// [n] to / from one rank. Exchanges post the outgoing side on a helper thread
// while the calling thread receives, so large messages cannot deadlock on full
// socket buffers. Return 0 on success, -1 for bad arguments or a world size
// that does not match the communicator, -2 when the rendezvous or a transfer
// fails.
#include <unistd.h>

#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#define AE_API extern "C" __attribute__((visibility("default")))

extern "C" {
int64_t aether_tcp_listen_addr(int64_t addr, int addr_len, int64_t port);
int64_t aether_tcp_listener_port(int64_t handle);
int aether_tcp_close(int64_t handle);
int64_t aether_tcp_accept_one(int64_t listener);
int aether_tcp_stream_close(int64_t handle);
int64_t aether_tcp_connect_host(int64_t host, int host_len, int64_t port);
int64_t aether_tcp_send_all(int64_t stream, int64_t buf, int64_t n);
int64_t aether_tcp_recv_all(int64_t stream, int64_t buf, int64_t n);
}

namespace {

struct Mesh {
  int world = 1, rank = 0;
  bool ready = false, failed = false;
  std::vector<int64_t> peer;  // stream to rank p (-1 for self)
};
std::mutex g_mesh_mu;
Mesh g_mesh;

int env_int(const char* a, const char* b, int dflt) {
  const char* e = std::getenv(a);
  if (!e) e = std::getenv(b);
  return e ? std::atoi(e) : dflt;
}

bool send_all(int64_t s, const void* p, int64_t n) {
  return aether_tcp_send_all(s, (int64_t)(intptr_t)p, n) == n;
}
bool recv_all(int64_t s, void* p, int64_t n) { return aether_tcp_recv_all(s, (int64_t)(intptr_t)p, n) == n; }

int64_t connect_retry(const std::string& host, int64_t port) {
  int64_t s = -1;
  for (int tries = 0; tries < 300 && s < 0; ++tries) {  // the listener may not be up yet: up to ~30 s
    s = aether_tcp_connect_host((int64_t)(intptr_t)host.data(), (int)host.size(), port);
    if (s < 0) usleep(100000);
  }
  return s;
}

// Builds the full mesh (called with g_mesh_mu held). Listener table entries
// are fixed-size records {port, host[64]}.
bool build_mesh(Mesh& m) {
  const char* addr = std::getenv("AETHER_COMM_ADDR");
  if (!addr) return false;
  const std::string a(addr);
  const size_t c = a.rfind(':');
  if (c == std::string::npos) return false;
  const std::string host0 = a.substr(0, c);
  const int64_t port0 = std::atoll(a.c_str() + c + 1);
  const char* me = std::getenv("AETHER_COMM_HOST");
  const std::string my_host = me ? me : "127.0.0.1";
  struct Rec {
    int64_t port;
    char host[64];
  };
  std::vector<Rec> table((size_t)m.world);
  m.peer.assign((size_t)m.world, -1);
  // every rank > 0 listens for the ranks above it
  int64_t lis = -1;
  if (m.rank > 0 && m.rank < m.world - 1) {
    lis = aether_tcp_listen_addr((int64_t)(intptr_t)my_host.data(), (int)my_host.size(), 0);
    if (lis < 0) return false;
  }
  if (m.rank == 0) {
    const int64_t l0 = aether_tcp_listen_addr((int64_t)(intptr_t)host0.data(), (int)host0.size(), port0);
    if (l0 < 0) return false;
    for (int i = 1; i < m.world; ++i) {
      const int64_t s = aether_tcp_accept_one(l0);
      int32_t r = -1;
      Rec rec{};
      if (s < 0 || !recv_all(s, &r, 4) || r < 1 || r >= m.world || m.peer[(size_t)r] >= 0 ||
          !recv_all(s, &rec, sizeof(Rec))) {
        aether_tcp_close(l0);
        return false;
      }
      rec.host[63] = 0;
      m.peer[(size_t)r] = s;
      table[(size_t)r] = rec;
    }
    aether_tcp_close(l0);
    for (int i = 1; i < m.world; ++i)
      if (!send_all(m.peer[(size_t)i], table.data(), (int64_t)(sizeof(Rec) * table.size()))) return false;
  } else {
    const int64_t s = connect_retry(host0, port0);
    const int32_t r = m.rank;
    Rec rec{};
    rec.port = lis >= 0 ? aether_tcp_listener_port(lis) : 0;
    std::strncpy(rec.host, my_host.c_str(), 63);
    if (s < 0 || !send_all(s, &r, 4) || !send_all(s, &rec, sizeof(Rec)) ||
        !recv_all(s, table.data(), (int64_t)(sizeof(Rec) * table.size())))
      return false;
    m.peer[0] = s;
    // connect down to ranks 1 .. rank-1, accept from rank+1 .. world-1
    for (int i = 1; i < m.rank; ++i) {
      const int64_t t = connect_retry(std::string(table[(size_t)i].host), table[(size_t)i].port);
      if (t < 0 || !send_all(t, &r, 4)) return false;
      m.peer[(size_t)i] = t;
    }
    for (int i = m.rank + 1; i < m.world; ++i) {
      const int64_t t = aether_tcp_accept_one(lis);
      int32_t from = -1;
      if (t < 0 || !recv_all(t, &from, 4) || from <= m.rank || from >= m.world || m.peer[(size_t)from] >= 0)
        return false;
      m.peer[(size_t)from] = t;
    }
    if (lis >= 0) aether_tcp_close(lis);
  }
  return true;
}

// The default communicator; nullptr when it cannot be set up.
Mesh* mesh() {
  std::lock_guard<std::mutex> g(g_mesh_mu);
  if (g_mesh.ready) return &g_mesh;
  if (g_mesh.failed) return nullptr;
  g_mesh.world = env_int("AETHER_WORLD_SIZE", "WORLD_SIZE", 1);
  g_mesh.rank = env_int("AETHER_RANK", "RANK", 0);
  if (g_mesh.world < 1 || g_mesh.rank < 0 || g_mesh.rank >= g_mesh.world) {
    g_mesh.failed = true;
    return nullptr;
  }
  if (g_mesh.world > 1 && !build_mesh(g_mesh)) {
    g_mesh.failed = true;
    return nullptr;
  }
  g_mesh.ready = true;
  return &g_mesh;
}

// Posts `sends` on a helper thread while the caller runs `recvs`: (rank,
// pointer, bytes) triples. Returns false if any transfer failed.
struct Xfer {
  int peer;
  void* p;
  int64_t bytes;
};
bool exchange(Mesh& m, const std::vector<Xfer>& sends, const std::vector<Xfer>& recvs) {
  bool send_ok = true;
  std::thread t([&]() {
    for (const Xfer& x : sends)
      if (x.bytes > 0 && !send_all(m.peer[(size_t)x.peer], x.p, x.bytes)) send_ok = false;
  });
  bool recv_ok = true;
  for (const Xfer& x : recvs)
    if (x.bytes > 0 && !recv_all(m.peer[(size_t)x.peer], x.p, x.bytes)) recv_ok = false;
  t.join();
  return send_ok && recv_ok;
}

Mesh* checked(int world) {
  Mesh* m = mesh();
  if (!m) return nullptr;
  return (world <= 0 || world == m->world) ? m : nullptr;
}

}  // namespace

extern "C" {

// Number of ranks / this rank of the default communicator (1 / 0 without one).
AE_API int aether_comm_world_size() {
  Mesh* m = mesh();
  return m ? m->world : 1;
}
AE_API int aether_comm_rank() {
  Mesh* m = mesh();
  return m ? m->rank : 0;
}

AE_API int aether_op_broadcast_f32(void* buf, int n, int root) {
  if (!buf || n < 0) return -1;
  Mesh* m = mesh();
  if (!m) return -2;
  if (root < 0 || root >= m->world) return -1;
  if (m->world == 1 || n == 0) return 0;
  const int64_t bytes = (int64_t)n * 4;
  std::vector<Xfer> sends, recvs;
  if (m->rank == root) {
    for (int p = 0; p < m->world; ++p)
      if (p != root) sends.push_back({p, buf, bytes});
  } else {
    recvs.push_back({root, buf, bytes});
  }
  return exchange(*m, sends, recvs) ? 0 : -2;
}

AE_API int aether_op_all_gather_f32(const void* src, void* dst, int n, int world) {
  if (!src || !dst || n < 0 || world < 1) return -1;
  Mesh* m = checked(world);
  if (!m) return mesh() ? -1 : -2;
  float* out = static_cast<float*>(dst);
  const int64_t bytes = (int64_t)n * 4;
  std::memmove(out + (size_t)m->rank * n, src, (size_t)bytes);
  if (m->world == 1) return 0;
  std::vector<Xfer> sends, recvs;
  for (int p = 0; p < m->world; ++p) {
    if (p == m->rank) continue;
    sends.push_back({p, out + (size_t)m->rank * n, bytes});
    recvs.push_back({p, out + (size_t)p * n, bytes});
  }
  return exchange(*m, sends, recvs) ? 0 : -2;
}

AE_API int aether_op_reduce_scatter_f32(const void* src, void* dst, int n, int world) {
  if (!src || !dst || n < 0 || world < 1) return -1;
  Mesh* m = checked(world);
  if (!m) return mesh() ? -1 : -2;
  const float* in = static_cast<const float*>(src);
  float* out = static_cast<float*>(dst);
  if (m->world == 1) {
    std::memmove(out, in, (size_t)n * 4);
    return 0;
  }
  const int64_t bytes = (int64_t)n * 4;
  std::vector<float> got((size_t)(m->world - 1) * n);
  std::vector<Xfer> sends, recvs;
  int k = 0;
  for (int p = 0; p < m->world; ++p) {
    if (p == m->rank) continue;
    sends.push_back({p, const_cast<float*>(in) + (size_t)p * n, bytes});
    recvs.push_back({p, got.data() + (size_t)k * n, bytes});
    ++k;
  }
  if (!exchange(*m, sends, recvs)) return -2;
  // own block first, then the other ranks in rank order: the same summation
  // order on every rank for a given block position
  std::vector<float> acc(in + (size_t)m->rank * n, in + (size_t)(m->rank + 1) * n);
  for (int j = 0; j < k; ++j)
    for (int i = 0; i < n; ++i) acc[(size_t)i] += got[(size_t)j * n + i];
  std::memcpy(out, acc.data(), (size_t)bytes);
  return 0;
}

AE_API int aether_op_all_to_all_f32(const void* src, void* dst, int n, int world) {
  if (!src || !dst || n < 0 || world < 1) return -1;
  Mesh* m = checked(world);
  if (!m) return mesh() ? -1 : -2;
  const float* in = static_cast<const float*>(src);
  float* out = static_cast<float*>(dst);
  const int64_t bytes = (int64_t)n * 4;
  if (m->world == 1) {
    std::memmove(out, in, (size_t)bytes);
    return 0;
  }
  std::vector<float> mine(in + (size_t)m->rank * n, in + (size_t)(m->rank + 1) * n);
  std::vector<float> stage;
  const float* s = in;
  if (src == dst) {  // in place: keep the outgoing blocks
    stage.assign(in, in + (size_t)m->world * n);
    s = stage.data();
  }
  std::vector<Xfer> sends, recvs;
  for (int p = 0; p < m->world; ++p) {
    if (p == m->rank) continue;
    sends.push_back({p, const_cast<float*>(s) + (size_t)p * n, bytes});
    recvs.push_back({p, out + (size_t)p * n, bytes});
  }
  if (!exchange(*m, sends, recvs)) return -2;
  std::memcpy(out + (size_t)m->rank * n, mine.data(), (size_t)bytes);
  return 0;
}

AE_API int aether_op_send_f32(const void* buf, int n, int dst_rank) {
  if (!buf || n < 0) return -1;
  Mesh* m = mesh();
  if (!m) return -2;
  if (dst_rank < 0 || dst_rank >= m->world) return -1;
  if (dst_rank == m->rank || n == 0) return 0;
  return send_all(m->peer[(size_t)dst_rank], buf, (int64_t)n * 4) ? 0 : -2;
}

AE_API int aether_op_recv_f32(void* buf, int n, int src_rank) {
  if (!buf || n < 0) return -1;
  Mesh* m = mesh();
  if (!m) return -2;
  if (src_rank < 0 || src_rank >= m->world) return -1;
  if (src_rank == m->rank || n == 0) return 0;
  return recv_all(m->peer[(size_t)src_rank], buf, (int64_t)n * 4) ? 0 : -2;
}

// In-place sum over the ranks of the default communicator: each rank gathers
// every rank's buffer and adds them in rank order, so all ranks hold
// bit-identical results.
AE_API int aether_op_all_reduce_sum_f32(void* buf, int world_size, int n) {
  if ((!buf && n > 0) || n < 0 || world_size < 1) return -1;
  Mesh* m = checked(world_size);
  if (!m) return mesh() ? -1 : -2;
  if (m->world == 1 || n == 0) return 0;
  std::vector<float> all((size_t)m->world * n);
  if (aether_op_all_gather_f32(buf, all.data(), n, m->world) != 0) return -2;
  float* out = static_cast<float*>(buf);
  for (int i = 0; i < n; ++i) {
    float s = 0.f;
    for (int p = 0; p < m->world; ++p) s += all[(size_t)p * n + i];
    out[i] = s;
  }
  return 0;
}

// Inserted by the compiler for `#[distributed(...)]` functions with a null
// buffer and no element count: a rendezvous of all ranks of the default
// communicator (backends 0 NCCL / 1 MPI / 2 Gloo map to it; 99 = no-op). A
// non-null buffer is left untouched, since the call carries no size.
AE_API void aether_dist_all_reduce(void* /*buf*/, int world_size, int backend) {
  if (backend == 99 || world_size <= 1) return;
  Mesh* m = checked(world_size);
  if (!m || m->world == 1) return;
  float token = 0.f;
  aether_op_all_reduce_sum_f32(&token, m->world, 1);
}

}  // extern "C"
