// libaether_rt: developer-tooling hooks, the NCCL-shaped host communicator,
// the CPU matmul tile autotuner and the image / audio preprocessing primitives.
//
// Reference ABI (runtime/src/lib.rs): aether_hot_reload_{arm,check} (:2152),
// aether_sbom_{reset,add,count,emit} (:2217), aether_autotune_matmul_tile_f32
// + unpack helpers (:2295), aether_cov_{record,hits,reset,dump} (:2352),
// aether_prefetch_{t0,t1,nta} (:2425), aether_nccl_* (:3336),
// aether_pgo_* (:3879), aether_img_{normalize,patchify}_f32 (:6302),
// aether_audio_{hann_window,dft_magnitude_f32} (:6352).
//
// The NCCL-shaped communicator is real across processes here: world_size 1
// is the identity; for world_size > 1 every rank passes the same rendezvous
// in AETHER_COMM_ADDR ("host:port"), rank 0 listens and the others connect
// over the TCP transport (tcp.cpp), and all_reduce is a star reduction (rank
// 0 combines sum / max / min / prod and sends the result back). GPU
// collectives of the package run through torch.distributed / NCCL; this is
// the host-side path the C ABI's callers get.
#include <sys/stat.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <unistd.h>
#include <utility>
#include <vector>

#define AE_API extern "C" __attribute__((visibility("default")))

extern "C" {
int64_t aether_tcp_listen_addr(int64_t, int, int64_t);
int64_t aether_tcp_accept_one(int64_t);
int64_t aether_tcp_connect_host(int64_t, int, int64_t);
int64_t aether_tcp_send_all(int64_t, int64_t, int64_t);
int64_t aether_tcp_recv_all(int64_t, int64_t, int64_t);
int aether_tcp_close(int64_t);
int aether_tcp_stream_close(int64_t);
}

namespace {

std::mutex g_mu;

std::string str_arg(const void* p, int64_t n) {
  return (p && n > 0) ? std::string(static_cast<const char*>(p), (size_t)n) : std::string();
}

// ------------------------------------------------------------------ hot reload
bool g_reload_armed = false;
timespec g_reload_mtime{};

bool mtime_of(const std::string& path, timespec& t) {
  struct stat st {};
  if (stat(path.c_str(), &st) != 0) return false;
  t = st.st_mtim;
  return true;
}
bool later(const timespec& a, const timespec& b) {
  return a.tv_sec > b.tv_sec || (a.tv_sec == b.tv_sec && a.tv_nsec > b.tv_nsec);
}

// ------------------------------------------------------------------ SBOM, coverage, PGO
std::vector<std::pair<std::string, std::string>> g_sbom;
std::map<std::pair<int64_t, int64_t>, int64_t> g_cov;         // (file, line) -> hits
std::map<int64_t, std::pair<int64_t, int64_t>> g_branches;     // site -> (taken, total)
std::map<int64_t, int64_t> g_calls;                             // callsite -> count

void json_str(const std::string& s, std::string& out) {
  out += '"';
  for (unsigned char c : s) {
    if (c == '"' || c == '\\') {
      out += '\\';
      out += (char)c;
    } else if (c < 0x20) {
      char b[8];
      std::snprintf(b, sizeof(b), "\\u%04x", c);
      out += b;
    } else {
      out += (char)c;
    }
  }
  out += '"';
}

// ------------------------------------------------------------------ communicator
struct Comm {
  int world = 1, rank = 0;
  int64_t listener = -1;
  std::vector<int64_t> peers;  // rank 0: streams to ranks 1..world-1; others: one stream to rank 0
};
std::atomic<int> g_nccl_inits{0};
std::map<int64_t, Comm> g_comms;
int64_t g_next_comm = 1;

bool parse_addr(std::string& host, int64_t& port) {
  const char* e = std::getenv("AETHER_COMM_ADDR");
  if (!e) return false;
  const std::string a(e);
  const size_t c = a.rfind(':');
  if (c == std::string::npos) return false;
  host = a.substr(0, c);
  port = std::atoll(a.c_str() + c + 1);
  return !host.empty() && port > 0 && port < 65536;
}

void combine(float* acc, const float* x, int n, int op) {
  for (int i = 0; i < n; ++i) {
    switch (op) {
      case 0: acc[i] += x[i]; break;
      case 1: acc[i] = std::max(acc[i], x[i]); break;
      case 2: acc[i] = std::min(acc[i], x[i]); break;
      default: acc[i] *= x[i]; break;
    }
  }
}

}  // namespace

extern "C" {

// ------------------------------------------------------------------ hot reload
// arm: remember the sentinel's modification time; check: 1 (and re-arm) when the
// file is newer than that, or when nothing was armed yet and the file exists.
AE_API int aether_hot_reload_arm(const void* path, int64_t len) {
  if (!path || len <= 0) return -1;
  std::lock_guard<std::mutex> g(g_mu);
  g_reload_armed = mtime_of(str_arg(path, len), g_reload_mtime);
  return 0;
}
AE_API int aether_hot_reload_check(const void* path, int64_t len) {
  if (!path || len <= 0) return 0;
  timespec t{};
  if (!mtime_of(str_arg(path, len), t)) return 0;
  std::lock_guard<std::mutex> g(g_mu);
  const bool fire = !g_reload_armed || later(t, g_reload_mtime);
  if (fire) {
    g_reload_armed = true;
    g_reload_mtime = t;
  }
  return fire ? 1 : 0;
}

// ------------------------------------------------------------------ SBOM (CycloneDX 1.5 JSON)
AE_API int aether_sbom_reset() {
  std::lock_guard<std::mutex> g(g_mu);
  g_sbom.clear();
  return 0;
}
AE_API int aether_sbom_add(const void* name, int64_t name_len, const void* version, int64_t version_len) {
  if (!name || name_len <= 0 || !version || version_len < 0) return -1;
  std::lock_guard<std::mutex> g(g_mu);
  g_sbom.emplace_back(str_arg(name, name_len), str_arg(version, version_len));
  return 0;
}
AE_API int64_t aether_sbom_count() {
  std::lock_guard<std::mutex> g(g_mu);
  return (int64_t)g_sbom.size();
}
AE_API int aether_sbom_emit(const void* out_path, int64_t out_len) {
  if (!out_path || out_len <= 0) return -1;
  // indented two spaces per level, one component per line
  std::string j = "{\n  \"bomFormat\": \"CycloneDX\",\n  \"specVersion\": \"1.5\",\n  \"version\": 1,\n  \"components\": [";
  {
    std::lock_guard<std::mutex> g(g_mu);
    for (size_t i = 0; i < g_sbom.size(); ++i) {
      j += i ? ",\n    " : "\n    ";
      j += "{\"type\": \"library\", \"name\": ";
      json_str(g_sbom[i].first, j);
      j += ", \"version\": ";
      json_str(g_sbom[i].second, j);
      j += '}';
    }
    if (!g_sbom.empty()) j += "\n  ";
  }
  j += "]\n}\n";
  const std::string path = str_arg(out_path, out_len), tmp = path + ".tmp";
  FILE* f = std::fopen(tmp.c_str(), "wb");
  if (!f) return -2;
  const bool ok = std::fwrite(j.data(), 1, j.size(), f) == j.size();
  std::fclose(f);
  if (!ok || std::rename(tmp.c_str(), path.c_str()) != 0) return -3;
  return 0;
}

// ------------------------------------------------------------------ matmul tile autotune
// Tile (tm, tn, tk) for the blocked CPU matmul: the largest of a few shapes
// whose A, B and C tiles (fp32) fit in half of this CPU's L1 data cache, no
// larger than the problem; unroll 8 for wide tiles. Packed as 16-bit fields
// tm | tn << 16 | tk << 32 | unroll << 48.
AE_API int64_t aether_autotune_matmul_tile_f32(int64_t m, int64_t n, int64_t k) {
  if (m <= 0 || n <= 0 || k <= 0) return 0;
  long l1 = sysconf(_SC_LEVEL1_DCACHE_SIZE);
  if (l1 <= 0) l1 = 32 * 1024;
  const int64_t budget = l1 / 2 / 4;  // fp32 elements
  static const int64_t cands[][3] = {{128, 128, 64}, {128, 64, 64}, {64, 64, 64}, {64, 64, 32},
                                     {32, 64, 32}, {32, 32, 32}, {16, 32, 16}, {16, 16, 16}};
  int64_t tm = 8, tn = 8, tk = 8;
  for (const auto& c : cands) {
    const int64_t a = std::min(c[0], m), b = std::min(c[1], n), d = std::min(c[2], k);
    if (a * d + d * b + a * b <= budget) {
      tm = a;
      tn = b;
      tk = d;
      break;
    }
  }
  const int64_t unroll = tn >= 64 ? 8 : 4;
  return (int64_t)((uint64_t)tm | ((uint64_t)tn << 16) | ((uint64_t)tk << 32) | ((uint64_t)unroll << 48));
}
AE_API int64_t aether_autotune_unpack_tile_m(int64_t h) { return (int64_t)((uint64_t)h & 0xFFFF); }
AE_API int64_t aether_autotune_unpack_tile_n(int64_t h) { return (int64_t)(((uint64_t)h >> 16) & 0xFFFF); }
AE_API int64_t aether_autotune_unpack_tile_k(int64_t h) { return (int64_t)(((uint64_t)h >> 32) & 0xFFFF); }
AE_API int64_t aether_autotune_unpack_unroll(int64_t h) { return (int64_t)(((uint64_t)h >> 48) & 0xFFFF); }

// ------------------------------------------------------------------ coverage counters
AE_API int aether_cov_record(int64_t file_id, int64_t line) {
  std::lock_guard<std::mutex> g(g_mu);
  ++g_cov[{file_id, line}];
  return 0;
}
AE_API int64_t aether_cov_hits(int64_t file_id, int64_t line) {
  std::lock_guard<std::mutex> g(g_mu);
  auto it = g_cov.find({file_id, line});
  return it == g_cov.end() ? 0 : it->second;
}
AE_API int aether_cov_reset() {
  std::lock_guard<std::mutex> g(g_mu);
  g_cov.clear();
  return 0;
}
AE_API int aether_cov_dump() {
  std::lock_guard<std::mutex> g(g_mu);
  for (const auto& e : g_cov)
    std::printf("cov file=%lld line=%lld hits=%lld\n", (long long)e.first.first, (long long)e.first.second,
                (long long)e.second);
  std::fflush(stdout);
  return 0;
}

// ------------------------------------------------------------------ PGO records
AE_API int aether_pgo_record_branch(int64_t site, int64_t taken) {
  std::lock_guard<std::mutex> g(g_mu);
  auto& e = g_branches[site];
  e.first += taken != 0;
  e.second += 1;
  return 0;
}
AE_API int aether_pgo_record_call(int64_t site) {
  std::lock_guard<std::mutex> g(g_mu);
  ++g_calls[site];
  return 0;
}
AE_API float aether_pgo_branch_freq(int64_t site) {
  std::lock_guard<std::mutex> g(g_mu);
  auto it = g_branches.find(site);
  return (it == g_branches.end() || it->second.second == 0) ? 0.f
                                                            : (float)it->second.first / (float)it->second.second;
}
AE_API int64_t aether_pgo_call_count(int64_t site) {
  std::lock_guard<std::mutex> g(g_mu);
  auto it = g_calls.find(site);
  return it == g_calls.end() ? 0 : it->second;
}
AE_API int aether_pgo_reset() {
  std::lock_guard<std::mutex> g(g_mu);
  g_branches.clear();
  g_calls.clear();
  return 0;
}
AE_API int aether_pgo_dump() {
  std::lock_guard<std::mutex> g(g_mu);
  for (const auto& e : g_branches)
    std::printf("site=%lld taken=%lld total=%lld\n", (long long)e.first, (long long)e.second.first,
                (long long)e.second.second);
  for (const auto& e : g_calls) std::printf("call=%lld count=%lld\n", (long long)e.first, (long long)e.second);
  std::fflush(stdout);
  return 0;
}

// ------------------------------------------------------------------ prefetch hints
AE_API int aether_prefetch_t0(int64_t p) {
  if (p) __builtin_prefetch(reinterpret_cast<const void*>(p), 0, 3);
  return 0;
}
AE_API int aether_prefetch_t1(int64_t p) {
  if (p) __builtin_prefetch(reinterpret_cast<const void*>(p), 0, 2);
  return 0;
}
AE_API int aether_prefetch_nta(int64_t p) {
  if (p) __builtin_prefetch(reinterpret_cast<const void*>(p), 0, 0);
  return 0;
}

// ------------------------------------------------------------------ NCCL-shaped communicator
AE_API int aether_nccl_init() {
  g_nccl_inits.fetch_add(1);
  return 0;
}
AE_API int aether_nccl_init_count() { return g_nccl_inits.load(); }
AE_API int aether_nccl_finalize() {
  std::lock_guard<std::mutex> g(g_mu);
  for (auto& kv : g_comms) {
    for (int64_t s : kv.second.peers) aether_tcp_stream_close(s);
    if (kv.second.listener >= 0) aether_tcp_close(kv.second.listener);
  }
  g_comms.clear();
  g_nccl_inits.store(0);
  return 0;
}

// Returns a handle >= 1, 0 for bad arguments, -1 when world_size > 1 has no
// rendezvous (AETHER_COMM_ADDR unset) or a peer could not be reached.
AE_API int64_t aether_nccl_comm_create(int world_size, int rank) {
  if (world_size <= 0 || rank < 0 || rank >= world_size) return 0;
  Comm c;
  c.world = world_size;
  c.rank = rank;
  if (world_size > 1) {
    std::string host;
    int64_t port = 0;
    if (!parse_addr(host, port)) return -1;
    if (rank == 0) {
      c.listener = aether_tcp_listen_addr((int64_t)(intptr_t)host.data(), (int)host.size(), port);
      if (c.listener < 0) return -1;
      c.peers.assign((size_t)world_size - 1, -1);
      for (int i = 1; i < world_size; ++i) {
        const int64_t s = aether_tcp_accept_one(c.listener);
        int32_t r = -1;
        if (s < 0 || aether_tcp_recv_all(s, (int64_t)(intptr_t)&r, 4) != 4 || r < 1 || r >= world_size ||
            c.peers[(size_t)r - 1] >= 0)
          return -1;
        c.peers[(size_t)r - 1] = s;
      }
    } else {
      int64_t s = -1;
      for (int tries = 0; tries < 200 && s < 0; ++tries) {  // rank 0 may not listen yet: up to ~20 s
        s = aether_tcp_connect_host((int64_t)(intptr_t)host.data(), (int)host.size(), port);
        if (s < 0) usleep(100000);
      }
      const int32_t r = rank;
      if (s < 0 || aether_tcp_send_all(s, (int64_t)(intptr_t)&r, 4) != 4) return -1;
      c.peers.push_back(s);
    }
  }
  std::lock_guard<std::mutex> g(g_mu);
  const int64_t h = g_next_comm++;
  g_comms[h] = std::move(c);
  return h;
}
AE_API int aether_nccl_comm_destroy(int64_t comm) {
  std::lock_guard<std::mutex> g(g_mu);
  auto it = g_comms.find(comm);
  if (it == g_comms.end()) return -1;
  for (int64_t s : it->second.peers) aether_tcp_stream_close(s);
  if (it->second.listener >= 0) aether_tcp_close(it->second.listener);
  g_comms.erase(it);
  return 0;
}
AE_API int aether_nccl_comm_world_size(int64_t comm) {
  std::lock_guard<std::mutex> g(g_mu);
  auto it = g_comms.find(comm);
  return it == g_comms.end() ? 1 : it->second.world;
}
AE_API int aether_nccl_comm_rank(int64_t comm) {
  std::lock_guard<std::mutex> g(g_mu);
  auto it = g_comms.find(comm);
  return it == g_comms.end() ? 0 : it->second.rank;
}

// recv = op over ranks of send (op: 0 sum, 1 max, 2 min, 3 prod); 0 on success.
AE_API int aether_nccl_all_reduce_f32(const void* send, void* recv, int n, int op, int64_t comm) {
  if (!send || !recv || n <= 0) return 1;
  if (op < 0 || op > 3) return 2;
  Comm c;
  {
    std::lock_guard<std::mutex> g(g_mu);
    auto it = g_comms.find(comm);
    if (it != g_comms.end()) c = it->second;  // copies the stream handles
  }
  float* out = static_cast<float*>(recv);
  if (out != send) std::memmove(out, send, sizeof(float) * (size_t)n);
  if (c.world <= 1) return 0;
  const int64_t bytes = (int64_t)n * 4;
  if (c.rank == 0) {
    std::vector<float> tmp((size_t)n);
    for (int64_t s : c.peers) {
      if (aether_tcp_recv_all(s, (int64_t)(intptr_t)tmp.data(), bytes) != bytes) return 3;
      combine(out, tmp.data(), n, op);
    }
    for (int64_t s : c.peers)
      if (aether_tcp_send_all(s, (int64_t)(intptr_t)out, bytes) != bytes) return 3;
  } else {
    const int64_t s = c.peers[0];
    if (aether_tcp_send_all(s, (int64_t)(intptr_t)out, bytes) != bytes) return 3;
    if (aether_tcp_recv_all(s, (int64_t)(intptr_t)out, bytes) != bytes) return 3;
  }
  return 0;
}

// ------------------------------------------------------------------ LLM inference bench entry points
// Forward passes per second of a pre-LayerNorm decoder (LN -> Q/K/V -> causal
// attention -> O + residual -> LN -> up -> SiLU -> down + residual) over a
// seq_len-token block, fp32 on this CPU through the C ABI's own ops; weights
// are drawn once from a fixed-seed SplitMix64 stream, scaled to +-0.01. The
// GPU variants (_cuda, _cuda_resident) live in the device library.
int aether_op_matmul_f32(const void*, const void*, void*, int, int, int);
int aether_op_layer_norm_f32(const void*, const void*, const void*, float, void*, void*, void*, int, int);
int aether_op_sdpa_causal_f32(const void*, const void*, const void*, void*, void*, int, int, int);
int aether_op_silu_f32(void*, int);

AE_API float aether_llm_inference_bench_tps(int n_iters, int d_model, int n_layers, int ff, int seq_len) {
  if (n_iters <= 0 || d_model <= 0 || n_layers <= 0 || ff <= 0 || seq_len <= 0) return 0.f;
  const size_t d = (size_t)d_model, f = (size_t)ff, s = (size_t)seq_len;
  uint64_t st = 0x2545F4914F6CDD1DULL;
  auto rnd = [&]() {
    st += 0x9E3779B97F4A7C15ULL;
    uint64_t z = st;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    z ^= z >> 31;
    return ((float)(z >> 40) / (float)(1 << 24) - 0.5f) * 0.02f;
  };
  struct Layer {
    std::vector<float> wq, wk, wv, wo, up, down;
  };
  std::vector<Layer> L((size_t)n_layers);
  for (auto& l : L) {
    for (auto* w : {&l.wq, &l.wk, &l.wv, &l.wo}) {
      w->resize(d * d);
      for (auto& e : *w) e = rnd();
    }
    l.up.resize(d * f);
    for (auto& e : l.up) e = rnd();
    l.down.resize(f * d);
    for (auto& e : l.down) e = rnd();
  }
  std::vector<float> ones(d, 1.f), zeros(d, 0.f), x(s * d), h(s * d), q(s * d), k(s * d), v(s * d), o(s * d),
      proj(s * d), att(s * s), up(s * f), mean(s), rstd(s);
  for (auto& e : x) e = rnd();
  const auto t0 = std::chrono::steady_clock::now();
  for (int it = 0; it < n_iters; ++it)
    for (auto& l : L) {
      aether_op_layer_norm_f32(x.data(), ones.data(), zeros.data(), 1e-5f, h.data(), mean.data(), rstd.data(),
                               (int)s, (int)d);
      aether_op_matmul_f32(h.data(), l.wq.data(), q.data(), (int)s, (int)d, (int)d);
      aether_op_matmul_f32(h.data(), l.wk.data(), k.data(), (int)s, (int)d, (int)d);
      aether_op_matmul_f32(h.data(), l.wv.data(), v.data(), (int)s, (int)d, (int)d);
      aether_op_sdpa_causal_f32(q.data(), k.data(), v.data(), o.data(), att.data(), 1, (int)s, (int)d);
      aether_op_matmul_f32(o.data(), l.wo.data(), proj.data(), (int)s, (int)d, (int)d);
      for (size_t i = 0; i < s * d; ++i) x[i] += proj[i];
      aether_op_layer_norm_f32(x.data(), ones.data(), zeros.data(), 1e-5f, h.data(), mean.data(), rstd.data(),
                               (int)s, (int)d);
      aether_op_matmul_f32(h.data(), l.up.data(), up.data(), (int)s, (int)d, (int)f);
      aether_op_silu_f32(up.data(), (int)(s * f));
      aether_op_matmul_f32(up.data(), l.down.data(), proj.data(), (int)s, (int)f, (int)d);
      for (size_t i = 0; i < s * d; ++i) x[i] += proj[i];
    }
  const double sec = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  return sec > 0 ? (float)(n_iters / sec) : 0.f;
}

// One bench line: "cpu|gpu  M= N= K= iters= us=".
AE_API int aether_print_bench(int64_t which, int m, int n, int k, int iters, int64_t us) {
  std::printf("%-3s  M=%4d  N=%4d  K=%4d  iters=%4d  us=%10lld\n", which == 0 ? "cpu" : "gpu", m, n, k, iters,
              (long long)us);
  std::fflush(stdout);
  return 0;
}

// ------------------------------------------------------------------ vision preprocessing
// out = (px / 255 - mean) / std for n 8-bit pixel values of one channel.
AE_API int aether_img_normalize_f32(const void* px_u8, void* out_f32, int n_pixels, float mean, float stdv) {
  if (!px_u8 || !out_f32 || n_pixels <= 0 || stdv == 0.f) return -1;
  const uint8_t* p = static_cast<const uint8_t*>(px_u8);
  float* o = static_cast<float*>(out_f32);
  const float inv = 1.f / stdv;
  for (int i = 0; i < n_pixels; ++i) o[i] = ((float)p[i] * (1.f / 255.f) - mean) * inv;
  return 0;
}

// (h, w) single-channel image -> (h / patch * w / patch) row-major patches of
// patch * patch values, patches in raster order; returns the patch count.
AE_API int aether_img_patchify_f32(const void* img, void* out, int h, int w, int patch) {
  if (!img || !out) return -1;
  if (h <= 0 || w <= 0 || patch <= 0) return -2;
  if (h % patch || w % patch) return -3;
  const float* x = static_cast<const float*>(img);
  float* o = static_cast<float*>(out);
  const int pr = h / patch, pc = w / patch;
  for (int py = 0; py < pr; ++py)
    for (int px = 0; px < pc; ++px) {
      float* dst = o + (size_t)(py * pc + px) * patch * patch;
      for (int iy = 0; iy < patch; ++iy)
        std::memcpy(dst + (size_t)iy * patch, x + (size_t)(py * patch + iy) * w + (size_t)px * patch,
                    sizeof(float) * (size_t)patch);
    }
  return pr * pc;
}

// ------------------------------------------------------------------ audio preprocessing
// Symmetric Hann window w[i] = 0.5 (1 - cos(2 pi i / (n - 1))).
AE_API int aether_audio_hann_window(void* out, int n) {
  if (!out || n <= 0) return -1;
  float* o = static_cast<float*>(out);
  if (n == 1) {
    o[0] = 1.f;
    return 0;
  }
  const double step = 2.0 * M_PI / (double)(n - 1);
  for (int i = 0; i < n; ++i) o[i] = (float)(0.5 * (1.0 - std::cos(step * i)));
  return 0;
}

// |X_k| of the real input for the first k_bins bins (direct DFT, double accumulators).
AE_API int aether_audio_dft_magnitude_f32(const void* input, int n, void* out_mag, int k_bins) {
  if (!input || !out_mag) return -1;
  if (n <= 0 || k_bins <= 0) return -2;
  const float* x = static_cast<const float*>(input);
  float* m = static_cast<float*>(out_mag);
  for (int k = 0; k < k_bins; ++k) {
    double re = 0.0, im = 0.0;
    const double w = -2.0 * M_PI * (double)k / (double)n;
    for (int t = 0; t < n; ++t) {
      const double ang = w * (double)t;
      re += x[t] * std::cos(ang);
      im += x[t] * std::sin(ang);
    }
    m[k] = (float)std::sqrt(re * re + im * im);
  }
  return 0;
}

}  // extern "C"
