// libaether_dev: the device-handle C ABI (aether_dev_* / aether_op_*_cuda).
//
// Programs written against the reference runtime (and the code its language
// compiler emits for Tensor method calls) drive the GPU through i64 handles:
// allocate a buffer, copy host data in, call ops by handle, copy results out.
// This library keeps those names, argument orders and return conventions
// (0 = ok, negative = error; handles are slot + 1, 0 = allocation failed) but
// none of the reference's machinery:
//   * one handle table for every element kind (f32 / i32 / u8), each entry
//     holding a stream-ordered allocation (cudaMallocAsync) and its device;
//   * a context per device (stream, GEMM scratch, captured graph) instead of
//     one global device-0 context, so several GPUs can be driven from one
//     process (aether_dev_set_device);
//   * every op checks each handle's kind and that the extents it is about to
//     touch fit the allocation, and returns -1 instead of launching;
//   * ahead-of-time sm_100a kernels (no runtime compilation, no cuBLAS). The
//     f32 GEMM family runs on the tcgen05 tensor cores (kind::tf32 with a
//     three-term hi / lo split for fp32-class accuracy) above ~96^3 and on a
//     tiled SIMT kernel below; everything else is a kernel in
//     this file: one CTA per row with shuffle reductions for norms / softmax /
//     cross-entropy, column-tiled deterministic reductions for parameter
//     gradients, and quantised mat-vecs that dequantise GGUF blocks in
//     registers (one warp per output row, 32-value chunks per lane).
//
// Reference: runtime/src/cuda.rs:7230-7410 (registry), 7419-8420 (GEMM family,
// training ops, graphs, sync), 8442-8480 (RoPE), 10185-10380 (GQA, embedding,
// SiLU, transpose, in-place ops), 10388-11120 (dequant and fused quantised
// mat-vecs), 11553 (d2d), 11609-11680 (KV append and one-token attention).
#include <cuda_fp16.h>
#include <cuda.h>
#include <cuda_runtime.h>
#include <nccl.h>

#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <algorithm>
#include <vector>

#include "../common.cuh"  // tcgen05 / TMA / mbarrier shims (header-only)

#define AE_API extern "C" __attribute__((visibility("default")))

namespace {

enum Kind { KF32 = 0, KI32 = 1, KU8 = 2 };

struct Buf {
  void* p = nullptr;
  size_t bytes = 0;
  int dev = -1;
  int kind = 0;
};

struct Ctx {
  bool ready = false;
  cudaStream_t s = nullptr;
  float* ws = nullptr;  // split-operand scratch of the f32 GEMM
  size_t ws_floats = 0;
  int* status = nullptr;  // bounded-wait status word of this device's kernels
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
};

// IQ3 codebooks (format data, shared with the host dequantisers), copied to
// every device when its context is created: global memory rather than
// __constant__, since the lanes of a warp index different entries and
// constant-cache reads of different addresses serialise.
namespace iq3 {
#include "iq3_grids.inc"
}
__device__ uint32_t g_iq3xxs_grid[256];
__device__ uint32_t g_iq3s_grid[512];

constexpr int kMaxDev = 64;
std::mutex g_mu;
std::vector<Buf> g_bufs;
std::vector<int64_t> g_free;
Ctx g_ctx[kMaxDev];
thread_local char g_err[256] = "";

void set_err(const char* what, cudaError_t e) {
  snprintf(g_err, sizeof(g_err), "%s: %s", what, cudaGetErrorString(e));
}

int cur_dev() {
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess) return -1;
  return d;
}

// Restores the calling thread's current device on scope exit.
struct DeviceScope {
  int prev = -1;
  explicit DeviceScope(int d) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != d) cudaSetDevice(d);
  }
  ~DeviceScope() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

Ctx* ctx_for(int d) {
  if (d < 0 || d >= kMaxDev) return nullptr;
  Ctx& c = g_ctx[d];
  if (c.ready) return &c;
  std::lock_guard<std::mutex> l(g_mu);
  if (c.ready) return &c;
  // the stream and the codebook copies belong to device d, whichever device
  // the caller has current (the NCCL clique creates every device's context)
  DeviceScope on(d);
  cudaError_t e = cudaStreamCreateWithFlags(&c.s, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    set_err("stream", e);
    return nullptr;
  }
  if ((e = cudaMemcpyToSymbol(g_iq3xxs_grid, iq3::IQ3XXS_GRID, sizeof(iq3::IQ3XXS_GRID))) != cudaSuccess ||
      (e = cudaMemcpyToSymbol(g_iq3s_grid, iq3::IQ3S_GRID, sizeof(iq3::IQ3S_GRID))) != cudaSuccess) {
    set_err("IQ3 codebooks", e);
    return nullptr;
  }
  c.ready = true;
  return &c;
}

Ctx* ctx() { return ctx_for(cur_dev()); }

// The buffer behind handle h if it has the given kind and holds at least
// `need` elements of size `esz`; nullptr otherwise.
void* lookup(int64_t h, int kind, size_t need, size_t esz) {
  std::lock_guard<std::mutex> l(g_mu);
  if (h <= 0 || (size_t)h > g_bufs.size()) return nullptr;
  const Buf& b = g_bufs[h - 1];
  if (!b.p || b.kind != kind || need * esz > b.bytes) return nullptr;
  return b.p;
}

size_t capacity(int64_t h, size_t esz) {
  std::lock_guard<std::mutex> l(g_mu);
  if (h <= 0 || (size_t)h > g_bufs.size() || !g_bufs[h - 1].p) return 0;
  return g_bufs[h - 1].bytes / esz;
}

float* F(int64_t h, size_t need) { return (float*)lookup(h, KF32, need, 4); }
int* I(int64_t h, size_t need) { return (int*)lookup(h, KI32, need, 4); }
uint8_t* U(int64_t h, size_t need) { return (uint8_t*)lookup(h, KU8, need, 1); }

int64_t alloc(size_t n, size_t esz, int kind) {
  Ctx* c = ctx();
  if (!c || n == 0) return 0;
  void* p = nullptr;
  cudaError_t e = cudaMallocAsync(&p, n * esz, c->s);
  if (e != cudaSuccess) {
    set_err("alloc", e);
    return 0;
  }
  cudaMemsetAsync(p, 0, n * esz, c->s);  // handles start zeroed, like the reference's alloc_zeros
  std::lock_guard<std::mutex> l(g_mu);
  Buf b{p, n * esz, cur_dev(), kind};
  if (!g_free.empty()) {
    int64_t h = g_free.back();
    g_free.pop_back();
    g_bufs[h - 1] = b;
    return h;
  }
  g_bufs.push_back(b);
  return (int64_t)g_bufs.size();
}

int release(int64_t h, int kind) {
  Buf b;
  {
    std::lock_guard<std::mutex> l(g_mu);
    if (h <= 0 || (size_t)h > g_bufs.size() || !g_bufs[h - 1].p || g_bufs[h - 1].kind != kind) return 0;
    b = g_bufs[h - 1];
    g_bufs[h - 1] = Buf{};
    g_free.push_back(h);
  }
  Ctx* c = ctx_for(b.dev);
  if (c) cudaFreeAsync(b.p, c->s);
  return 0;
}

int copy(void* dst, const void* src, size_t bytes, cudaMemcpyKind k) {
  Ctx* c = ctx();
  if (!c) return -1;
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, k, c->s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->s);  // the host buffer is the caller's again on return
  if (e != cudaSuccess) {
    set_err("copy", e);
    return -2;
  }
  return 0;
}

int launched(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_err(what, e);
    return -2;
  }
  return 0;
}

unsigned blocks(size_t n, unsigned t = 256) { return (unsigned)((n + t - 1) / t); }

// ---------------------------------------------------------------------------------------------- reductions
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Sum over the CTA (blockDim.x a multiple of 32, at most 1024); every thread gets the result.
__device__ float block_sum(float v) {
  __shared__ float sh[32];
  __shared__ float total;
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  if (w == 0) {
    float t = l < (int)(blockDim.x >> 5) ? sh[l] : 0.f;
    t = warp_sum(t);
    if (l == 0) total = t;
  }
  __syncthreads();
  return total;
}

__device__ float block_max(float v) {
  __shared__ float sh[32];
  __shared__ float total;
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  if (w == 0) {
    float t = l < (int)(blockDim.x >> 5) ? sh[l] : -INFINITY;
    t = warp_max(t);
    if (l == 0) total = t;
  }
  __syncthreads();
  return total;
}

constexpr int kRowThreads = 256;

// ---------------------------------------------------------------------------------------------- elementwise
__device__ __forceinline__ float gelu_tanh(float x) {
  // 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))  (Hendrycks & Gimpel's approximation)
  const float u = 0.7978845608028654f * (x + 0.044715f * x * x * x);
  return 0.5f * x * (1.f + tanhf(u));
}

__device__ __forceinline__ float gelu_tanh_grad(float x) {
  const float u = 0.7978845608028654f * (x + 0.044715f * x * x * x);
  const float t = tanhf(u);
  const float du = 0.7978845608028654f * (1.f + 3.f * 0.044715f * x * x);
  return 0.5f * (1.f + t) + 0.5f * x * (1.f - t * t) * du;
}

__global__ void k_add(const float* a, const float* b, float* o, size_t n) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i < n) o[i] = a[i] + b[i];
}
__global__ void k_add_inplace(float* x, const float* y, size_t n) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i < n) x[i] += y[i];
}
__global__ void k_mul_inplace(float* x, const float* y, size_t n) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i < n) x[i] *= y[i];
}
__global__ void k_scale(float* x, float s, size_t n) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i < n) x[i] *= s;
}
__global__ void k_gelu(const float* x, float* y, size_t n) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i < n) y[i] = gelu_tanh(x[i]);
}
__global__ void k_gelu_bwd(const float* x, const float* dy, float* dx, size_t n) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i < n) dx[i] = dy[i] * gelu_tanh_grad(x[i]);
}
__global__ void k_gelu_erf(const float* x, float* y, size_t n) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i < n) y[i] = 0.5f * x[i] * (1.f + erff(x[i] * 0.7071067811865476f));
}
__global__ void k_silu(float* x, size_t n) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i < n) x[i] = x[i] / (1.f + expf(-x[i]));
}
__global__ void k_silu_bwd(const float* x, const float* dy, float* dx, size_t n) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i < n) {
    const float s = 1.f / (1.f + expf(-x[i]));
    dx[i] = dy[i] * s * (1.f + x[i] * (1.f - s));
  }
}
__global__ void k_bias_add(float* x, const float* b, size_t rows, int cols) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i < rows * cols) x[i] += b[i % cols];
}
__global__ void k_transpose_021(const float* in, float* out, int d0, int d1, int d2) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;  // index into out [d1, d0, d2]
  size_t n = (size_t)d0 * d1 * d2;
  if (i >= n) return;
  const int k = (int)(i % d2);
  const size_t r = i / d2;
  const int a = (int)(r % d0), b = (int)(r / d0);
  out[i] = in[((size_t)a * d1 + b) * d2 + k];
}
__global__ void k_embed(const float* table, const int* ids, float* out, int t, int d, int vocab) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= (size_t)t * d) return;
  const int r = (int)(i / d), j = (int)(i % d);
  const int id = ids[r];
  out[i] = (id >= 0 && id < vocab) ? table[(size_t)id * d + j] : 0.f;
}
__global__ void k_embed_scatter(const float* dout, const int* ids, float* dtable, int t, int d, int vocab) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= (size_t)t * d) return;
  const int r = (int)(i / d), j = (int)(i % d);
  const int id = ids[r];
  if (id >= 0 && id < vocab) atomicAdd(&dtable[(size_t)id * d + j], dout[i]);
}
__global__ void k_gqa_repeat(const float* in, float* out, int seq, int hkv, int hd, int hq) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= (size_t)seq * hq * hd) return;
  const int k = (int)(i % hd);
  const size_t r = i / hd;
  const int h = (int)(r % hq), s = (int)(r / hq);
  out[i] = in[((size_t)s * hkv + h / (hq / hkv)) * hd + k];
}
__global__ void k_gqa_reduce(const float* dout, float* din, int seq, int hkv, int hd, int hq) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= (size_t)seq * hkv * hd) return;
  const int k = (int)(i % hd);
  const size_t r = i / hd;
  const int h = (int)(r % hkv), s = (int)(r / hkv);
  const int g = hq / hkv;
  float acc = 0.f;
  for (int j = 0; j < g; ++j) acc += dout[((size_t)s * hq + h * g + j) * hd + k];
  din[i] = acc;
}
__global__ void k_append_kv(const float* kn, const float* vn, float* kc, float* vc, int pos, int dkv) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < dkv) {
    kc[(size_t)pos * dkv + i] = kn[i];
    vc[(size_t)pos * dkv + i] = vn[i];
  }
}
__global__ void k_adamw(float* p, const float* g, float* m, float* v, float lr, float b1, float b2, float eps, float wd,
                        float bc1, float bc2, size_t n) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float gi = g[i];
  const float mi = b1 * m[i] + (1.f - b1) * gi;
  const float vi = b2 * v[i] + (1.f - b2) * gi * gi;
  m[i] = mi;
  v[i] = vi;
  p[i] -= lr * ((mi * bc1) / (sqrtf(vi * bc2) + eps) + wd * p[i]);
}

// RoPE on x [seq, heads, hd], pairs (i, i + hd/2), angle (pos_start + t) * base^(-2i/hd);
// dir = -1 rotates back (the backward pass).
__global__ void k_rope(float* x, int seq, int heads, int hd, float base, int pos0, float dir) {
  const int half = hd / 2;
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= (size_t)seq * heads * half) return;
  const int j = (int)(i % half);
  const size_t r = i / half;
  const int t = (int)(r / heads);
  const float ang = (float)(t + pos0) * powf(base, -2.f * (float)j / (float)hd);
  float sn, cs;
  sincosf(ang, &sn, &cs);
  sn *= dir;
  float* row = x + r * hd;
  const float a = row[j], b = row[j + half];
  row[j] = a * cs - b * sn;
  row[j + half] = a * sn + b * cs;
}

// ---------------------------------------------------------------------------------------------- row kernels
__global__ void k_softmax(const float* x, float* y, int d) {
  const float* xr = x + (size_t)blockIdx.x * d;
  float* yr = y + (size_t)blockIdx.x * d;
  float m = -INFINITY;
  for (int j = threadIdx.x; j < d; j += blockDim.x) m = fmaxf(m, xr[j]);
  m = block_max(m);
  float s = 0.f;
  for (int j = threadIdx.x; j < d; j += blockDim.x) s += expf(xr[j] - m);
  s = block_sum(s);
  const float inv = 1.f / s;
  for (int j = threadIdx.x; j < d; j += blockDim.x) yr[j] = expf(xr[j] - m) * inv;
}

// dx = scale * y * (dy - sum(dy * y))
__global__ void k_softmax_bwd(const float* y, const float* dy, float* dx, int d, float scale) {
  const size_t o = (size_t)blockIdx.x * d;
  float dot = 0.f;
  for (int j = threadIdx.x; j < d; j += blockDim.x) dot += y[o + j] * dy[o + j];
  dot = block_sum(dot);
  for (int j = threadIdx.x; j < d; j += blockDim.x) dx[o + j] = scale * y[o + j] * (dy[o + j] - dot);
}

// Causal softmax of pre-scaled scores, row i of each [s, s] matrix keeps columns <= i.
__global__ void k_causal_softmax(float* a, int s) {
  const int i = blockIdx.x % s;
  float* r = a + (size_t)blockIdx.x * s;
  float m = -INFINITY;
  for (int j = threadIdx.x; j <= i; j += blockDim.x) m = fmaxf(m, r[j]);
  m = block_max(m);
  float sum = 0.f;
  for (int j = threadIdx.x; j <= i; j += blockDim.x) sum += expf(r[j] - m);
  sum = block_sum(sum);
  const float inv = 1.f / sum;
  for (int j = threadIdx.x; j < s; j += blockDim.x) r[j] = j <= i ? expf(r[j] - m) * inv : 0.f;
}

// x (+ res, written back into x when res != null) -> layer norm; mean / rstd cached per row
__global__ void k_layernorm(const float* a, const float* b, const float* g, const float* beta, float* y, float* mean,
                            float* rstd, float eps, int d) {
  const size_t o = (size_t)blockIdx.x * d;
  float s = 0.f;
  for (int j = threadIdx.x; j < d; j += blockDim.x) s += a[o + j] + (b ? b[o + j] : 0.f);
  const float mu = block_sum(s) / d;
  float v = 0.f;
  for (int j = threadIdx.x; j < d; j += blockDim.x) {
    const float t = a[o + j] + (b ? b[o + j] : 0.f) - mu;
    v += t * t;
  }
  const float rs = rsqrtf(block_sum(v) / d + eps);
  for (int j = threadIdx.x; j < d; j += blockDim.x) {
    const float t = a[o + j] + (b ? b[o + j] : 0.f) - mu;
    y[o + j] = t * rs * g[j] + (beta ? beta[j] : 0.f);
  }
  if (threadIdx.x == 0) {
    if (mean) mean[blockIdx.x] = mu;
    if (rstd) rstd[blockIdx.x] = rs;
  }
}

__global__ void k_layernorm_bwd_dx(const float* x, const float* g, const float* mean, const float* rstd, const float* dy,
                                   float* dx, int d) {
  const size_t o = (size_t)blockIdx.x * d;
  const float mu = mean[blockIdx.x], rs = rstd[blockIdx.x];
  float s1 = 0.f, s2 = 0.f;
  for (int j = threadIdx.x; j < d; j += blockDim.x) {
    const float gy = dy[o + j] * g[j];
    s1 += gy;
    s2 += gy * (x[o + j] - mu) * rs;
  }
  s1 = block_sum(s1) / d;
  s2 = block_sum(s2) / d;
  for (int j = threadIdx.x; j < d; j += blockDim.x) {
    const float xh = (x[o + j] - mu) * rs;
    dx[o + j] = rs * (dy[o + j] * g[j] - s1 - xh * s2);
  }
}

__global__ void k_rmsnorm(float* x, const float* res, const float* g, float* y, float eps, int d) {
  const size_t o = (size_t)blockIdx.x * d;
  float s = 0.f;
  for (int j = threadIdx.x; j < d; j += blockDim.x) {
    float v = x[o + j];
    if (res) {
      v += res[o + j];
      x[o + j] = v;  // fused residual add writes the sum back
    }
    s += v * v;
  }
  const float inv = rsqrtf(block_sum(s) / d + eps);
  for (int j = threadIdx.x; j < d; j += blockDim.x) y[o + j] = x[o + j] * inv * g[j];
}

__global__ void k_rmsnorm_bwd_dx(const float* x, const float* g, const float* dy, float* dx, float* inv_rms, float eps,
                                 int d) {
  const size_t o = (size_t)blockIdx.x * d;
  float ss = 0.f, dot = 0.f;
  for (int j = threadIdx.x; j < d; j += blockDim.x) {
    ss += x[o + j] * x[o + j];
    dot += dy[o + j] * g[j] * x[o + j];
  }
  const float inv = rsqrtf(block_sum(ss) / d + eps);
  dot = block_sum(dot) / d;
  for (int j = threadIdx.x; j < d; j += blockDim.x)
    dx[o + j] = inv * (dy[o + j] * g[j] - x[o + j] * inv * inv * dot);
  if (threadIdx.x == 0) inv_rms[blockIdx.x] = inv;
}

// Parameter gradients: sum over rows of a per-element product, per column.
// 32 columns x 8 row stripes per CTA, fixed summation order (deterministic).
// mode 0: dgamma = sum dy * (x - mean) * rstd and dbeta = sum dy (layer norm);
// mode 1: dgamma = sum dy * x * inv_rms (RMSNorm).
__global__ void k_colsum(const float* x, const float* dy, const float* mean, const float* rstd, float* dg, float* db,
                         int rows, int d, int mode) {
  __shared__ float sg[8][33], sb[8][33];
  const int j = blockIdx.x * 32 + threadIdx.x;
  float ag = 0.f, ab = 0.f;
  if (j < d) {
    for (int r = threadIdx.y; r < rows; r += 8) {
      const size_t o = (size_t)r * d + j;
      const float xh = mode == 0 ? (x[o] - mean[r]) * rstd[r] : x[o] * rstd[r];
      ag += dy[o] * xh;
      ab += dy[o];
    }
  }
  sg[threadIdx.y][threadIdx.x] = ag;
  sb[threadIdx.y][threadIdx.x] = ab;
  __syncthreads();
  if (threadIdx.y == 0 && j < d) {
    float tg = 0.f, tb = 0.f;
    for (int k = 0; k < 8; ++k) {
      tg += sg[k][threadIdx.x];
      tb += sb[k][threadIdx.x];
    }
    dg[j] = tg;
    if (db) db[j] = tb;
  }
}

// Cross-entropy: per-row softmax probabilities and -log p[label] (0 for labels outside [0, v)).
__global__ void k_ce_fwd(const float* logits, const int* labels, float* probs, float* loss, int v) {
  const size_t o = (size_t)blockIdx.x * v;
  float m = -INFINITY;
  for (int j = threadIdx.x; j < v; j += blockDim.x) m = fmaxf(m, logits[o + j]);
  m = block_max(m);
  float s = 0.f;
  for (int j = threadIdx.x; j < v; j += blockDim.x) s += expf(logits[o + j] - m);
  s = block_sum(s);
  const float inv = 1.f / s;
  for (int j = threadIdx.x; j < v; j += blockDim.x) probs[o + j] = expf(logits[o + j] - m) * inv;
  if (threadIdx.x == 0) {
    const int lab = labels[blockIdx.x];
    loss[blockIdx.x] = (lab >= 0 && lab < v) ? -(logits[o + lab] - m - logf(s)) : 0.f;
  }
}

__global__ void k_ce_bwd(const float* probs, const int* labels, float* dl, int b, int v) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= (size_t)b * v) return;
  const int r = (int)(i / v), c = (int)(i % v);
  const float inv_b = 1.f / (float)b;
  dl[i] = probs[i] * inv_b - (c == labels[r] ? inv_b : 0.f);
}

// One query token against a [cur_seq, n_kv * hd] KV cache: one CTA per query
// head, scores in shared memory.
__global__ void k_attn_seq1(const float* q, const float* kc, const float* vc, float* out, int cur, int hq, int hkv, int hd,
                            float scale) {
  extern __shared__ float sc[];
  const int h = blockIdx.x, kvh = h / (hq / hkv), dkv = hkv * hd;
  const float* qh = q + (size_t)h * hd;
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int t = w; t < cur; t += nw) {  // one warp per key
    const float* kr = kc + (size_t)t * dkv + (size_t)kvh * hd;
    float acc = 0.f;
    for (int k = l; k < hd; k += 32) acc += qh[k] * kr[k];
    acc = warp_sum(acc);
    if (l == 0) sc[t] = acc * scale;
  }
  __syncthreads();
  float m = -INFINITY;
  for (int t = threadIdx.x; t < cur; t += blockDim.x) m = fmaxf(m, sc[t]);
  m = block_max(m);
  float s = 0.f;
  for (int t = threadIdx.x; t < cur; t += blockDim.x) {
    const float e = expf(sc[t] - m);
    sc[t] = e;
    s += e;
  }
  s = block_sum(s);
  const float inv = 1.f / s;
  for (int k = threadIdx.x; k < hd; k += blockDim.x) {
    float acc = 0.f;
    for (int t = 0; t < cur; ++t) acc += sc[t] * vc[(size_t)t * dkv + (size_t)kvh * hd + k];
    out[(size_t)h * hd + k] = acc * inv;
  }
}

// ---------------------------------------------------------------------------------------------- GGUF blocks
// Element types by their GGML numbers; block = (elements, bytes).
enum Q { TF32 = 0, TF16 = 1, TQ4_0 = 2, TQ5_0 = 6, TQ8_0 = 8, TQ3_K = 11, TQ4_K = 12, TQ5_K = 13, TQ6_K = 14,
         TIQ3_XXS = 18, TIQ4_NL = 20, TIQ3_S = 21, TIQ4_XS = 23 };

bool block_of(int t, int* ne, int* nb) {
  switch (t) {
    case TF32: *ne = 1; *nb = 4; return true;
    case TF16: *ne = 1; *nb = 2; return true;
    case TQ4_0: *ne = 32; *nb = 18; return true;
    case TQ5_0: *ne = 32; *nb = 22; return true;
    case TQ8_0: *ne = 32; *nb = 34; return true;
    case TIQ4_NL: *ne = 32; *nb = 18; return true;
    case TQ3_K: *ne = 256; *nb = 110; return true;
    case TQ4_K: *ne = 256; *nb = 144; return true;
    case TQ5_K: *ne = 256; *nb = 176; return true;
    case TQ6_K: *ne = 256; *nb = 210; return true;
    case TIQ4_XS: *ne = 256; *nb = 136; return true;
    case TIQ3_XXS: *ne = 256; *nb = 98; return true;
    case TIQ3_S: *ne = 256; *nb = 110; return true;
    default: return false;
  }
}

__constant__ float c_iq4[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};


__device__ __forceinline__ float h2f(const uint8_t* p) {
  __half_raw r;
  r.x = (unsigned short)(p[0] | (p[1] << 8));
  return __half2float(__half(r));
}

// Six-bit (scale, min) pair j of the 12 packed bytes of a Q4_K / Q5_K super-block.
__device__ __forceinline__ void k4_scale(const uint8_t* s, int j, float* sc, float* mn) {
  if (j < 4) {
    *sc = (float)(s[j] & 63);
    *mn = (float)(s[j + 4] & 63);
  } else {
    *sc = (float)((s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4));
    *mn = (float)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
  }
}

// The 32 values of chunk c (elements 32c .. 32c+31) of a row of type t.
template <int T>
__device__ __forceinline__ void chunk32(const uint8_t* row, int c, float* v) {
  if constexpr (T == TF32) {
    const float* p = (const float*)row + c * 32;
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = p[i];
  } else if constexpr (T == TF16) {
    const uint8_t* p = row + c * 64;
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = h2f(p + 2 * i);
  } else if constexpr (T == TQ8_0) {
    const uint8_t* b = row + c * 34;
    const float d = h2f(b);
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = d * (float)(int8_t)b[2 + i];
  } else if constexpr (T == TQ4_0 || T == TIQ4_NL) {
    const uint8_t* b = row + c * 18;
    const float d = h2f(b);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int lo = b[2 + i] & 0x0F, hi = b[2 + i] >> 4;
      if constexpr (T == TQ4_0) {
        v[i] = d * (float)(lo - 8);
        v[i + 16] = d * (float)(hi - 8);
      } else {
        v[i] = d * c_iq4[lo];
        v[i + 16] = d * c_iq4[hi];
      }
    }
  } else if constexpr (T == TQ5_0) {
    const uint8_t* b = row + c * 22;
    const float d = h2f(b);
    const uint32_t qh = b[2] | (b[3] << 8) | (b[4] << 16) | ((uint32_t)b[5] << 24);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int lo = (b[6 + i] & 0x0F) | (((qh >> i) & 1) << 4);
      const int hi = (b[6 + i] >> 4) | (((qh >> (i + 16)) & 1) << 4);
      v[i] = d * (float)(lo - 16);
      v[i + 16] = d * (float)(hi - 16);
    }
  } else if constexpr (T == TQ4_K || T == TQ5_K) {
    const int j = c & 7;
    const uint8_t* b = row + (size_t)(c >> 3) * (T == TQ4_K ? 144 : 176);
    const float d = h2f(b), dmin = h2f(b + 2);
    float sc, mn;
    k4_scale(b + 4, j, &sc, &mn);
    const float a = d * sc, o = dmin * mn;
    const uint8_t* qs = b + (T == TQ4_K ? 16 : 48) + (j >> 1) * 32;
    const int sh = (j & 1) * 4;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      int q = (qs[i] >> sh) & 0x0F;
      if constexpr (T == TQ5_K) q += ((b[16 + i] >> j) & 1) << 4;
      v[i] = a * (float)q - o;
    }
  } else if constexpr (T == TQ6_K) {
    const int j = c & 7, half = j >> 2, part = j & 3;
    const uint8_t* b = row + (size_t)(c >> 3) * 210;
    const uint8_t* ql = b + half * 64 + (part & 1) * 32;
    const uint8_t* qh = b + 128 + half * 32;
    const int8_t* scl = (const int8_t*)(b + 192);
    const float d = h2f(b + 208);
    const int lsh = (part >> 1) * 4, hsh = part * 2;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int q = (((ql[i] >> lsh) & 0x0F) | (((qh[i] >> hsh) & 3) << 4)) - 32;
      v[i] = d * (float)scl[half * 8 + part * 2 + (i >> 4)] * (float)q;
    }
  } else if constexpr (T == TQ3_K) {
    const int j = c & 7, half = j >> 2, sh = j & 3;
    const uint8_t* b = row + (size_t)(c >> 3) * 110;
    const uint8_t* hm = b;
    const uint8_t* qs = b + 32 + half * 32;
    const uint8_t* s = b + 96;
    const float d = h2f(b + 108);
    float scl[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {  // sixteen 6-bit scales: low nibbles in bytes 0-7, high pairs in 8-11
      const int si = half * 8 + sh * 2 + u;
      const int lo = si < 8 ? (s[si] & 0x0F) : (s[si - 8] >> 4);
      const int hi = (s[8 + (si & 3)] >> (2 * (si >> 2))) & 3;
      scl[u] = (float)((lo | (hi << 4)) - 32);
    }
    const int m = 1 << (half * 4 + sh);
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int q = ((qs[i] >> (2 * sh)) & 3) - ((hm[i] & m) ? 0 : 4);
      v[i] = d * scl[i >> 4] * (float)q;
    }
  } else if constexpr (T == TIQ3_XXS) {
    // 32 values: 8 codebook indices (4 magnitudes each), one u32 with a 4-bit
    // scale and four 7-bit sign-pattern indices (index + parity bit = 8 signs)
    const int j = c & 7;
    const uint8_t* b = row + (size_t)(c >> 3) * 98;
    const float d = h2f(b);
    const uint8_t* qs = b + 2 + 8 * j;
    const uint32_t aux = b[66 + 4 * j] | (b[67 + 4 * j] << 8) | (b[68 + 4 * j] << 16) | ((uint32_t)b[69 + 4 * j] << 24);
    const float db = d * (0.5f + (float)(aux >> 28)) * 0.5f;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const uint32_t i7 = (aux >> (7 * g)) & 127;
      const uint32_t sg = i7 | ((__popc(i7) & 1) << 7);
      const uint32_t e0 = __ldg(&g_iq3xxs_grid[qs[2 * g]]), e1 = __ldg(&g_iq3xxs_grid[qs[2 * g + 1]]);
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const float mag = (float)(((t < 4 ? e0 : e1) >> (8 * (t & 3))) & 0xff);
        v[8 * g + t] = db * mag * ((sg >> t) & 1 ? -1.f : 1.f);
      }
    }
  } else if constexpr (T == TIQ3_S) {
    // 32 values: 8 nine-bit codebook indices (low bytes + one high-bit byte),
    // 4 explicit sign bytes, one 4-bit scale d * (1 + 2 s)
    const int j = c & 7;
    const uint8_t* b = row + (size_t)(c >> 3) * 110;
    const float d = h2f(b);
    const uint8_t *qs = b + 2 + 8 * j, qh = b[66 + j], *sg = b + 74 + 4 * j;
    const float db = d * (float)(1 + 2 * ((b[106 + j / 2] >> (4 * (j & 1))) & 15));
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const uint32_t e0 = __ldg(&g_iq3s_grid[qs[2 * g] | (((qh >> (2 * g)) & 1) << 8)]);
      const uint32_t e1 = __ldg(&g_iq3s_grid[qs[2 * g + 1] | (((qh >> (2 * g + 1)) & 1) << 8)]);
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const float mag = (float)(((t < 4 ? e0 : e1) >> (8 * (t & 3))) & 0xff);
        v[8 * g + t] = db * mag * ((sg[g] >> t) & 1 ? -1.f : 1.f);
      }
    }
  } else if constexpr (T == TIQ4_XS) {
    const int j = c & 7;
    const uint8_t* b = row + (size_t)(c >> 3) * 136;
    const float d = h2f(b);
    const int sh = b[2] | (b[3] << 8);
    const int ls = ((b[4 + j / 2] >> (4 * (j & 1))) & 0x0F) | (((sh >> (2 * j)) & 3) << 4);
    const float dl = d * (float)(ls - 32);
    const uint8_t* qs = b + 8 + j * 16;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      v[i] = dl * c_iq4[qs[i] & 0x0F];
      v[i + 16] = dl * c_iq4[qs[i] >> 4];
    }
  }
}

// Row-major dequantisation: thread per 32-value chunk (rows are whole blocks,
// so chunk c of the flat tensor is chunk c of the flat block stream).
template <int T>
__global__ void k_dequant_flat(const uint8_t* w, float* out, size_t chunks) {
  size_t c = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (c >= chunks) return;
  float v[32];
  if constexpr (T == TQ4_K || T == TQ5_K || T == TQ6_K || T == TQ3_K || T == TIQ4_XS || T == TIQ3_XXS ||
                T == TIQ3_S) {
    chunk32<T>(w, (int)c, v);  // super-block c / 8, sub-block c % 8
  } else {
    const int nb = T == TQ8_0 ? 34 : T == TQ5_0 ? 22 : 18;  // one 32-value block per chunk
    chunk32<T>(w + c * nb, 0, v);
  }
  float4* o = (float4*)(out + c * 32);
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}

// y[r] = sum_k x[k] * W[r, k] (* silu gate variant): one warp per output row,
// lane l takes 32-value chunks l, l+32, ... Rows come in groups of `rpg`
// (per-head weights): group g reads x + g * xg and writes y[g * yg + r % rpg];
// grid.y walks a batch of inputs (x + b * xb, y + b * yb).
struct MV {
  const float* x;
  const uint8_t* w;
  float* y;
  const uint8_t* w2;
  int rows, chunks;
  size_t row_bytes;
  int rpg;
  long long xg, yg, xb, yb;
  const int8_t* xq;  // when set: x is q8_1 (int8 values xq, one scale xd per 32)
  const float* xd;
};

template <int T>
__global__ void k_matvec(MV p) {
  const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int l = threadIdx.x & 31;
  if (r >= p.rows) return;
  const int g = r / p.rpg;
  const float* x = p.x + blockIdx.y * p.xb + g * p.xg;
  const uint8_t* wr = p.w + (size_t)r * p.row_bytes;
  const uint8_t* wr2 = p.w2 ? p.w2 + (size_t)r * p.row_bytes : nullptr;
  float acc = 0.f, acc2 = 0.f;
  float v[32];
  for (int c = l; c < p.chunks; c += 32) {
    float xs[32];
    if (p.xq) {
      const int8_t* q = p.xq + (size_t)c * 32;
      const float d = p.xd[c];
#pragma unroll
      for (int i = 0; i < 32; ++i) xs[i] = d * (float)q[i];
    } else {
      const float4* xv = (const float4*)(x + (size_t)c * 32);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 t = __ldg(xv + i);
        xs[4 * i] = t.x;
        xs[4 * i + 1] = t.y;
        xs[4 * i + 2] = t.z;
        xs[4 * i + 3] = t.w;
      }
    }
    chunk32<T>(wr, c, v);
#pragma unroll
    for (int i = 0; i < 32; ++i) acc += xs[i] * v[i];
    if (wr2) {
      chunk32<T>(wr2, c, v);
#pragma unroll
      for (int i = 0; i < 32; ++i) acc2 += xs[i] * v[i];
    }
  }
  acc = warp_sum(acc);
  if (wr2) acc2 = warp_sum(acc2);
  if (l == 0) p.y[blockIdx.y * p.yb + g * p.yg + r % p.rpg] = wr2 ? acc / (1.f + expf(-acc)) * acc2 : acc;  // silu(gate) * up
}

// ---------------------------------------------------------------------------------------------- GEMM
// Row-major C[M,N] = alpha op(A)[M,K] op(B)[K,N] + beta C, strided-batched, in
// fp32 -- the contract of the reference's cuBLAS sgemm family
// (runtime/src/cuda.rs:7419-7760). Two kernels of this library, no cuBLAS:
//   * large problems: a tcgen05 kernel of kind::tf32 with the three-term
//     split x = hi + lo (hi = tf32(x), lo = tf32(x - hi)) and
//     C = A_hi B_hi + A_lo B_hi + A_hi B_lo accumulated in TMEM, which keeps
//     fp32-class accuracy (the dropped A_lo B_lo term is ~2^-22 relative).
//     A pre-pass writes the hi / lo parts K-major and zero-padded to whole
//     128 x 32 tiles, so every TMA box is in bounds and transposed operands
//     need no second kernel; 128 x 128 output tile per CTA, 3-stage TMA ring,
//     one thread issues the MMAs, four warps read TMEM back;
//   * small problems: a 32 x 32-tiled SIMT kernel with fp32 FMAs.
namespace tfg {
constexpr int BM = 128, BN = 128, BK = 32;  // BK fp32 = 128 bytes: one 128B-swizzle row
constexpr int STAGES = 3;
constexpr int TILE = BM * BK * 4;           // 16 KB
constexpr int STAGE_BYTES = 4 * TILE;       // A hi, A lo, B hi, B lo
constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
constexpr uint32_t kIdesc = (1u << 4)                // D: F32
                            | (2u << 7) | (2u << 10)  // A, B: TF32 (both K-major)
                            | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

struct Args {
  float* C;
  long long ldc, sC;
  int M, N, K, kb;  // kb: K blocks of BK
  int Mp, Np;       // padded rows of the split operands
  float alpha, beta;
  int* status;
};

__device__ __forceinline__ void umma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ float to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// dst[(b * 2 + part) * rows_p * Kp + r * Kp + k] = part 0: tf32(x), part 1:
// tf32(x - tf32(x)), x = op(src)[r][k] of batch b (0 outside the real shape).
// op(src)[r][k] = src[r * ld + k] or, transposed, src[k * ld + r].
__global__ void k_split(const float* __restrict__ src, long long ld, long long bstride, bool trans, int rows, int K,
                        int rows_p, int Kp, float* __restrict__ dst) {
  const long long n = (long long)rows_p * Kp;
  const int b = blockIdx.y;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(i / Kp), k = (int)(i % Kp);
    float x = 0.f;
    if (r < rows && k < K) x = src[b * bstride + (trans ? (long long)k * ld + r : (long long)r * ld + k)];
    const float hi = to_tf32(x);
    dst[((long long)b * 2) * n + i] = hi;
    dst[((long long)b * 2 + 1) * n + i] = to_tf32(x - hi);
  }
}

__global__ void __launch_bounds__(128, 1) k_gemm(const __grid_constant__ CUtensorMap tA,
                                                 const __grid_constant__ CUtensorMap tB, Args p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* done = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_word = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tn = blockIdx.x, tm = blockIdx.y, b = blockIdx.z;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      aether::mbar_init(&full[s], 1);
      aether::mbar_init(&empty[s], 1);
    }
    aether::mbar_init(done, 1);
    *abort_word = 0;
    aether::fence_mbar_init();
    aether::tma_prefetch_desc(&tA);
    aether::tma_prefetch_desc(&tB);
  }
  if (warp == 1) {
    aether::tmem_alloc(tmem_slot, BN);
    aether::tmem_relinquish();
  }
  aether::tc_fence_before();
  __syncthreads();
  aether::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;
  if (warp == 0 && lane == 0) {
    // producer: the hi / lo tiles of A and B for each K block
    const int a_hi = (2 * b) * p.Mp + tm * BM, a_lo = a_hi + p.Mp;
    const int b_hi = (2 * b) * p.Np + tn * BN, b_lo = b_hi + p.Np;
    uint32_t issued = 0;
    for (int kb = 0; kb < p.kb; ++kb) {
      const int s = kb % STAGES;
      const uint32_t ph = (uint32_t)(kb / STAGES) & 1u;
      if (!aether::mbar_wait(&empty[s], ph ^ 1u, abort_word)) {
        ok = false;
        break;
      }
      uint8_t* st = smem + s * STAGE_BYTES;
      aether::mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
      aether::tma_load_2d(st, &tA, &full[s], kb * BK, a_hi);
      aether::tma_load_2d(st + TILE, &tA, &full[s], kb * BK, a_lo);
      aether::tma_load_2d(st + 2 * TILE, &tB, &full[s], kb * BK, b_hi);
      aether::tma_load_2d(st + 3 * TILE, &tB, &full[s], kb * BK, b_lo);
      ++issued;
    }
    if (!ok) {
      *abort_word = 1;
      atomicExch(p.status, aether::kStatusTimeoutProducer);
      volatile int never = 0;  // copies in flight land before the CTA exits
      for (uint32_t j = 1; j <= (issued < (uint32_t)STAGES ? issued : (uint32_t)STAGES); ++j) {
        const uint32_t i = issued - j;
        aether::mbar_wait(&full[i % STAGES], (i / STAGES) & 1u, &never);
      }
    }
  } else if (warp == 1 && lane == 0) {
    // MMA issuer: per 8-wide K step, hi*hi + lo*hi + hi*lo into one accumulator
    for (int kb = 0; kb < p.kb && ok; ++kb) {
      const int s = kb % STAGES;
      if (!aether::mbar_wait(&full[s], (uint32_t)(kb / STAGES) & 1u, abort_word)) {
        ok = false;
        break;
      }
      aether::tc_fence_after();
      const uint32_t base = aether::smem_u32(smem + s * STAGE_BYTES);
#pragma unroll
      for (int kk = 0; kk < BK / 8; ++kk) {
        const uint64_t ah = aether::sdesc_sw128(base + kk * 32, 16, 1024);
        const uint64_t al = aether::sdesc_sw128(base + TILE + kk * 32, 16, 1024);
        const uint64_t bh = aether::sdesc_sw128(base + 2 * TILE + kk * 32, 16, 1024);
        const uint64_t bl = aether::sdesc_sw128(base + 3 * TILE + kk * 32, 16, 1024);
        umma_tf32(tmem, ah, bh, (kb | kk) != 0 ? 1u : 0u);
        umma_tf32(tmem, al, bh, 1u);
        umma_tf32(tmem, ah, bl, 1u);
      }
      aether::umma_commit(&empty[s]);
    }
    if (!ok) {
      *abort_word = 1;
      atomicExch(p.status, aether::kStatusTimeoutMma);
    }
    aether::umma_commit(done);  // also the drain: fires once every MMA issued above has completed
  }
  __syncwarp();
  // epilogue: warp w owns TMEM lanes (rows) 32w .. 32w + 31
  {
    // `done` fires once every MMA the issuer started has completed (it commits
    // even after an abort), so TMEM is quiet whether or not the tile finished
    volatile int never = 0;
    const bool got = aether::mbar_wait(done, 0, &never);
    aether::tc_fence_after();
    const int m = tm * BM + warp * 32 + lane;
    float* crow = p.C + b * p.sC + (long long)m * p.ldc;
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t r[32];
      aether::tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + c * 32, r);
      aether::tmem_ld_wait();
      if (!got || *abort_word || m >= p.M) continue;
      const int n0 = tn * BN + c * 32;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int n = n0 + j;
        if (n < p.N) {
          const float v = p.alpha * __uint_as_float(r[j]);
          crow[n] = p.beta != 0.f ? v + p.beta * crow[n] : v;
        }
      }
    }
  }
  aether::tc_fence_before();
  __syncthreads();
  if (warp == 1) aether::tmem_dealloc(tmem, BN);
}

// C = alpha op(A) op(B) + beta C, one thread per output, 32 x 32 shared tiles.
__global__ void k_gemm_simt(bool ta, bool tb, int M, int N, int K, float alpha, const float* __restrict__ A,
                            long long lda, const float* __restrict__ B, long long ldb, float beta, float* C,
                            long long ldc, long long sA, long long sB, long long sC) {
  __shared__ float As[32][33], Bs[32][33];
  const int b = blockIdx.z;
  A += b * sA;
  B += b * sB;
  C += b * sC;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8 threads, 4 rows each
  const int row0 = blockIdx.y * 32, col = blockIdx.x * 32 + tx;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int k0 = 0; k0 < K; k0 += 32) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = ty + 8 * i;
      const int m = row0 + r, k = k0 + tx;  // As[r][kk] = op(A)[m][k]
      As[r][tx] = (m < M && k < K) ? (ta ? A[(long long)k * lda + m] : A[(long long)m * lda + k]) : 0.f;
      const int kr = k0 + r, n = col;      // Bs[kk][c] = op(B)[k][n]
      Bs[r][tx] = (kr < K && n < N) ? (tb ? B[(long long)n * ldb + kr] : B[(long long)kr * ldb + n]) : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < 32; ++kk) {
      const float bv = Bs[kk][tx];
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i] += As[ty + 8 * i][kk] * bv;
    }
    __syncthreads();
  }
  if (col >= N) return;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = row0 + ty + 8 * i;
    if (m < M) {
      float* c = C + (long long)m * ldc + col;
      *c = beta != 0.f ? alpha * acc[i] + beta * *c : alpha * acc[i];
    }
  }
}
}  // namespace tfg

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiled encode_tiled() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(f);
  });
  return fn;
}

// [rows, Kp] fp32 K-major operand, 128-row x 32-column boxes, 128B swizzle.
bool tmap_f32(CUtensorMap* m, const float* base, int Kp, long long rows) {
  EncodeTiled fn = encode_tiled();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)Kp, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)Kp * 4};
  cuuint32_t box[2] = {tfg::BK, 128};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Grow-only scratch for the split operands, one per device context (stream-ordered).
float* gemm_scratch(Ctx* c, size_t floats) {
  if (c->ws_floats < floats) {
    if (c->ws) cudaFreeAsync(c->ws, c->s);
    c->ws = nullptr;
    c->ws_floats = 0;
    if (cudaMallocAsync(reinterpret_cast<void**>(&c->ws), floats * 4, c->s) != cudaSuccess) return nullptr;
    c->ws_floats = floats;
  }
  return c->ws;
}

int* dev_status() {
  Ctx* c = ctx();
  if (!c) return nullptr;
  if (!c->status) {
    if (cudaMalloc(reinterpret_cast<void**>(&c->status), sizeof(int)) != cudaSuccess) return nullptr;
    cudaMemset(c->status, 0, sizeof(int));
  }
  return c->status;
}

int gemm_rm(bool ta, bool tb, int M, int N, int K, float alpha, const float* A, int lda, const float* B, int ldb,
            float beta, float* C, int ldc, int batch = 1, long long sA = 0, long long sB = 0, long long sC = 0) {
  Ctx* c = ctx();
  if (!c) return -1;
  if (M <= 0 || N <= 0 || K <= 0 || batch <= 0) return -1;
  // the tensor-core path pays a split pre-pass and 128 x 128 tiles: worth it above ~96^3
  const bool tc = (long long)M * N * K >= (1ll << 20) * 3 / 4 && M >= 64 && N >= 64 && K >= 32 &&
                  getenv("AETHER_DEV_SIMT_GEMM") == nullptr;
  if (!tc) {
    dim3 grid((N + 31) / 32, (M + 31) / 32, batch);
    tfg::k_gemm_simt<<<grid, 256, 0, c->s>>>(ta, tb, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, sA, sB, sC);
    return launched("gemm");
  }
  const int Mp = (M + 127) / 128 * 128, Np = (N + 127) / 128 * 128, Kp = (K + 31) / 32 * 32;
  const size_t a_f = (size_t)batch * 2 * Mp * Kp, b_f = (size_t)batch * 2 * Np * Kp;
  float* ws = gemm_scratch(c, a_f + b_f);
  int* status = dev_status();
  if (!ws || !status) {
    snprintf(g_err, sizeof(g_err), "gemm: scratch allocation failed");
    return -2;
  }
  float *as = ws, *bs = ws + a_f;
  const unsigned ga = (unsigned)std::min<long long>(((long long)Mp * Kp + 255) / 256, 4096);
  const unsigned gb = (unsigned)std::min<long long>(((long long)Np * Kp + 255) / 256, 4096);
  tfg::k_split<<<dim3(ga, batch), 256, 0, c->s>>>(A, lda, sA, ta, M, K, Mp, Kp, as);
  tfg::k_split<<<dim3(gb, batch), 256, 0, c->s>>>(B, ldb, sB, !tb, N, K, Np, Kp, bs);  // B^T rows are op(B) columns
  CUtensorMap ta_map, tb_map;
  if (!tmap_f32(&ta_map, as, Kp, (long long)batch * 2 * Mp) || !tmap_f32(&tb_map, bs, Kp, (long long)batch * 2 * Np)) {
    snprintf(g_err, sizeof(g_err), "gemm: tensor map encoding failed");
    return -2;
  }
  static bool attr_set[kMaxDev] = {};
  const int d = cur_dev();
  if (!attr_set[d]) {
    cudaFuncSetAttribute(tfg::k_gemm, cudaFuncAttributeMaxDynamicSharedMemorySize, tfg::SMEM);
    attr_set[d] = true;
  }
  tfg::Args args{C, ldc, sC, M, N, K, Kp / tfg::BK, Mp, Np, alpha, beta, status};
  tfg::k_gemm<<<dim3(Np / tfg::BN, Mp / tfg::BM, batch), 128, tfg::SMEM, c->s>>>(ta_map, tb_map, args);
  return launched("gemm");
}

template <int T>
int matvec_launch(MV p, int batch) {
  Ctx* c = ctx();
  if (!c) return -1;
  k_matvec<T><<<dim3(blocks(p.rows, 8), batch), 256, 0, c->s>>>(p);
  return launched("matvec");
}

int matvec_typed(int t, MV p, int batch = 1) {
  switch (t) {
    case TF32: return matvec_launch<TF32>(p, batch);
    case TF16: return matvec_launch<TF16>(p, batch);
    case TQ4_0: return matvec_launch<TQ4_0>(p, batch);
    case TQ5_0: return matvec_launch<TQ5_0>(p, batch);
    case TQ8_0: return matvec_launch<TQ8_0>(p, batch);
    case TIQ4_NL: return matvec_launch<TIQ4_NL>(p, batch);
    case TQ3_K: return matvec_launch<TQ3_K>(p, batch);
    case TQ4_K: return matvec_launch<TQ4_K>(p, batch);
    case TQ5_K: return matvec_launch<TQ5_K>(p, batch);
    case TQ6_K: return matvec_launch<TQ6_K>(p, batch);
    case TIQ4_XS: return matvec_launch<TIQ4_XS>(p, batch);
    case TIQ3_XXS: return matvec_launch<TIQ3_XXS>(p, batch);
    case TIQ3_S: return matvec_launch<TIQ3_S>(p, batch);
    default: return -2;
  }
}

// Quantised mat-vec by handle: `rows` output rows of `nblk` blocks each, the
// weight starting `expert` whole matrices into the buffer; `batch` inputs of
// k values back to back give `batch` outputs of `rows` values.
int qmatvec(int t, int64_t xh, int64_t wh, int64_t yh, int rows, int nblk, int expert = 0, int64_t w2h = 0,
            int batch = 1) {
  int ne, nb;
  if (!block_of(t, &ne, &nb) || rows <= 0 || nblk <= 0 || expert < 0 || batch <= 0) return -1;
  const size_t k = (size_t)nblk * ne;
  if (k % 32) return -1;
  const size_t row_bytes = (size_t)nblk * nb, mat = row_bytes * rows;
  const float* x = F(xh, k * batch);
  const uint8_t* w = U(wh, mat * (expert + 1));
  float* y = F(yh, (size_t)rows * batch);
  const uint8_t* w2 = w2h ? U(w2h, mat) : nullptr;
  if (!x || !w || !y || (w2h && !w2)) return -1;
  MV p{x, w + mat * expert, y, w2, rows, (int)(k / 32), row_bytes, rows, 0, 0, (long long)k, rows, nullptr, nullptr};
  return matvec_typed(t, p, batch);
}

template <int T>
int dequant_launch(const uint8_t* w, float* out, size_t chunks) {
  Ctx* c = ctx();
  if (!c) return -1;
  k_dequant_flat<T><<<blocks(chunks), 256, 0, c->s>>>(w, out, chunks);
  return launched("dequant");
}

int dequant_typed(int t, const uint8_t* w, float* out, size_t chunks) {
  switch (t) {
    case TQ4_K: return dequant_launch<TQ4_K>(w, out, chunks);
    case TQ6_K: return dequant_launch<TQ6_K>(w, out, chunks);
    case TQ8_0: return dequant_launch<TQ8_0>(w, out, chunks);
    case TQ4_0: return dequant_launch<TQ4_0>(w, out, chunks);
    case TQ5_0: return dequant_launch<TQ5_0>(w, out, chunks);
    case TQ5_K: return dequant_launch<TQ5_K>(w, out, chunks);
    case TQ3_K: return dequant_launch<TQ3_K>(w, out, chunks);
    case TIQ4_NL: return dequant_launch<TIQ4_NL>(w, out, chunks);
    case TIQ4_XS: return dequant_launch<TIQ4_XS>(w, out, chunks);
    case TIQ3_XXS: return dequant_launch<TIQ3_XXS>(w, out, chunks);
    case TIQ3_S: return dequant_launch<TIQ3_S>(w, out, chunks);
    default: return -2;
  }
}

int dequant_handle(int t, int64_t wh, int64_t oh, int nblk) {
  int ne, nb;
  if (!block_of(t, &ne, &nb) || nblk <= 0 || ne < 32) return -1;
  const uint8_t* w = U(wh, (size_t)nblk * nb);
  float* o = F(oh, (size_t)nblk * ne);
  if (!w || !o) return -1;
  return dequant_typed(t, w, o, (size_t)nblk * ne / 32);
}

}  // namespace

// ================================================================================================ registry
AE_API int aether_dev_init() {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) return -1;
  return ctx() ? 0 : -1;
}

// Select the device later calls (allocations, ops, graphs) run on.
AE_API int aether_dev_set_device(int d) {
  if (cudaSetDevice(d) != cudaSuccess) return -1;
  return ctx() ? 0 : -1;
}

AE_API int aether_dev_count() {
  int n = 0;
  return cudaGetDeviceCount(&n) == cudaSuccess ? n : 0;
}

AE_API const char* aether_dev_last_error() { return g_err; }

AE_API int64_t aether_dev_mem_free_bytes() {
  size_t f = 0, t = 0;
  if (!ctx() || cudaMemGetInfo(&f, &t) != cudaSuccess) return -1;
  return (int64_t)f;
}

AE_API int64_t aether_dev_alloc_f32(int n) { return n > 0 ? alloc((size_t)n, 4, KF32) : 0; }
AE_API int64_t aether_dev_alloc_i32(int n) { return n > 0 ? alloc((size_t)n, 4, KI32) : 0; }
AE_API int64_t aether_dev_alloc_u8(int n) { return n > 0 ? alloc((size_t)n, 1, KU8) : 0; }
AE_API int aether_dev_free_f32(int64_t h) { return release(h, KF32); }
AE_API int aether_dev_free_i32(int64_t h) { return release(h, KI32); }
AE_API int aether_dev_free_u8(int64_t h) { return release(h, KU8); }

AE_API int aether_dev_h2d_f32(int64_t host, int64_t dev, int n) {
  float* d = n > 0 ? F(dev, n) : nullptr;
  return (!d || !host) ? -1 : copy(d, (const void*)host, (size_t)n * 4, cudaMemcpyHostToDevice);
}
AE_API int aether_dev_d2h_f32(int64_t dev, int64_t host, int n) {
  float* d = n > 0 ? F(dev, n) : nullptr;
  return (!d || !host) ? -1 : copy((void*)host, d, (size_t)n * 4, cudaMemcpyDeviceToHost);
}
AE_API int aether_dev_h2d_i32(int64_t host, int64_t dev, int n) {
  int* d = n > 0 ? I(dev, n) : nullptr;
  return (!d || !host) ? -1 : copy(d, (const void*)host, (size_t)n * 4, cudaMemcpyHostToDevice);
}
AE_API int aether_dev_d2h_i32(int64_t dev, int64_t host, int n) {
  int* d = n > 0 ? I(dev, n) : nullptr;
  return (!d || !host) ? -1 : copy((void*)host, d, (size_t)n * 4, cudaMemcpyDeviceToHost);
}
AE_API int aether_dev_h2d_u8(int64_t host, int64_t dev, int n) {
  uint8_t* d = n > 0 ? U(dev, n) : nullptr;
  return (!d || !host) ? -1 : copy(d, (const void*)host, (size_t)n, cudaMemcpyHostToDevice);
}
AE_API int aether_dev_d2h_u8(int64_t dev, int64_t host, int n) {
  uint8_t* d = n > 0 ? U(dev, n) : nullptr;
  return (!d || !host) ? -1 : copy((void*)host, d, (size_t)n, cudaMemcpyDeviceToHost);
}
// The first n elements of a possibly larger buffer (the plain forms already allow that here).
AE_API int aether_dev_h2d_f32_n(int64_t host, int64_t dev, int n) { return aether_dev_h2d_f32(host, dev, n); }
AE_API int aether_dev_d2h_f32_n(int64_t dev, int64_t host, int n) { return aether_dev_d2h_f32(dev, host, n); }
AE_API int aether_dev_h2d_i32_n(int64_t host, int64_t dev, int n) { return aether_dev_h2d_i32(host, dev, n); }

AE_API int aether_dev_d2d_f32_offset(int64_t src, int src_off, int64_t dst, int dst_off, int n) {
  if (n <= 0 || src_off < 0 || dst_off < 0) return -1;
  float* s = F(src, (size_t)src_off + n);
  float* d = F(dst, (size_t)dst_off + n);
  Ctx* c = ctx();
  if (!s || !d || !c) return -1;
  cudaError_t e = cudaMemcpyAsync(d + dst_off, s + src_off, (size_t)n * 4, cudaMemcpyDeviceToDevice, c->s);
  if (e != cudaSuccess) {
    set_err("d2d", e);
    return -2;
  }
  return 0;
}

AE_API int64_t aether_wall_us() {
  using namespace std::chrono;
  return duration_cast<microseconds>(steady_clock::now().time_since_epoch()).count();
}

AE_API int aether_dev_sync() {
  Ctx* c = ctx();
  if (!c) return -1;
  cudaError_t e = cudaStreamSynchronize(c->s);
  if (e != cudaSuccess) {
    set_err("sync", e);
    return -2;
  }
  return 0;
}

// ================================================================================================ graphs
// One captured graph per device: begin/end capture the device stream (thread-
// local mode), launch replays it, destroy frees it.
AE_API int aether_dev_graph_begin() {
  Ctx* c = ctx();
  if (!c) return -1;
  return cudaStreamBeginCapture(c->s, cudaStreamCaptureModeThreadLocal) == cudaSuccess ? 0 : -2;
}

AE_API int aether_dev_graph_end() {
  Ctx* c = ctx();
  if (!c) return -1;
  cudaGraph_t g = nullptr;
  if (cudaStreamEndCapture(c->s, &g) != cudaSuccess || !g) return -2;
  if (c->exec) cudaGraphExecDestroy(c->exec);
  if (c->graph) cudaGraphDestroy(c->graph);
  c->graph = g;
  c->exec = nullptr;
  return cudaGraphInstantiate(&c->exec, g, 0) == cudaSuccess ? 0 : -2;
}

AE_API int aether_dev_graph_launch() {
  Ctx* c = ctx();
  if (!c || !c->exec) return -1;
  return cudaGraphLaunch(c->exec, c->s) == cudaSuccess ? 0 : -2;
}

AE_API int aether_dev_graph_destroy() {
  Ctx* c = ctx();
  if (!c) return -1;
  if (c->exec) cudaGraphExecDestroy(c->exec);
  if (c->graph) cudaGraphDestroy(c->graph);
  c->exec = nullptr;
  c->graph = nullptr;
  return 0;
}

// ================================================================================================ GEMMs
#define NEED3(pa, na, pb, nb, pc, nc)                     \
  const float* pa##_ = F(pa, (size_t)(na));               \
  const float* pb##_ = F(pb, (size_t)(nb));               \
  float* pc##_ = F(pc, (size_t)(nc));                     \
  if (!pa##_ || !pb##_ || !pc##_ || m <= 0 || k <= 0 || n <= 0) return -1;

// out[m,n] = a[m,k] b[k,n]
AE_API int aether_op_matmul_f32_cuda(int64_t a, int64_t b, int64_t out, int m, int k, int n) {
  NEED3(a, (size_t)m * k, b, (size_t)k * n, out, (size_t)m * n);
  return gemm_rm(false, false, m, n, k, 1.f, a_, k, b_, n, 0.f, out_, n);
}
// out[m,n] = a[k,m]^T b[k,n]
AE_API int aether_op_matmul_tn_f32_cuda(int64_t a, int64_t b, int64_t out, int m, int k, int n) {
  NEED3(a, (size_t)k * m, b, (size_t)k * n, out, (size_t)m * n);
  return gemm_rm(true, false, m, n, k, 1.f, a_, m, b_, n, 0.f, out_, n);
}
// out[m,n] = a[m,k] b[n,k]^T
AE_API int aether_op_matmul_nt_f32_cuda(int64_t a, int64_t b, int64_t out, int m, int k, int n) {
  NEED3(a, (size_t)m * k, b, (size_t)n * k, out, (size_t)m * n);
  return gemm_rm(false, true, m, n, k, 1.f, a_, k, b_, k, 0.f, out_, n);
}
// out = gelu(a b), the GELU launched right behind the GEMM on the same stream
AE_API int aether_op_matmul_gelu_f32_cuda(int64_t a, int64_t b, int64_t out, int m, int k, int n) {
  int r = aether_op_matmul_f32_cuda(a, b, out, m, k, n);
  if (r) return r;
  float* o = F(out, (size_t)m * n);
  size_t cnt = (size_t)m * n;
  k_gelu<<<blocks(cnt), 256, 0, ctx()->s>>>(o, o, cnt);
  return launched("gelu");
}
// matmul timed with events on the device stream; prints the time and rate to stderr
AE_API int aether_op_matmul_f32_cuda_profile(int64_t a, int64_t b, int64_t out, int m, int k, int n) {
  Ctx* c = ctx();
  if (!c) return -1;
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  cudaEventRecord(e0, c->s);
  int r = aether_op_matmul_f32_cuda(a, b, out, m, k, n);
  cudaEventRecord(e1, c->s);
  cudaEventSynchronize(e1);
  float ms = 0.f;
  cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (!r)
    fprintf(stderr, "[aether_dev] matmul %dx%dx%d: %.3f ms, %.2f TFLOP/s\n", m, k, n, ms,
            2.0 * m * k * n / (ms * 1e-3) / 1e12);
  return r;
}
// db[k,n] = a[m,k]^T dy[m,n]
AE_API int aether_op_matmul_backward_rhs_f32_cuda(int64_t a, int64_t dy, int64_t db, int m, int k, int n) {
  NEED3(a, (size_t)m * k, dy, (size_t)m * n, db, (size_t)k * n);
  return gemm_rm(true, false, k, n, m, 1.f, a_, k, dy_, n, 0.f, db_, n);
}
// da[m,k] = dy[m,n] b[k,n]^T
AE_API int aether_op_matmul_backward_lhs_f32_cuda(int64_t dy, int64_t b, int64_t da, int m, int k, int n) {
  NEED3(dy, (size_t)m * n, b, (size_t)k * n, da, (size_t)m * k);
  return gemm_rm(false, true, m, k, n, 1.f, dy_, n, b_, n, 0.f, da_, k);
}
// Enqueue `iters` matmuls with no sync between them; prints enqueue and drain time.
AE_API int aether_bench_matmul_batch(int64_t a, int64_t b, int64_t out, int m, int k, int n, int iters) {
  if (iters <= 0) return -1;
  const int64_t t0 = aether_wall_us();
  for (int i = 0; i < iters; ++i) {
    int r = aether_op_matmul_f32_cuda(a, b, out, m, k, n);
    if (r) return r;
  }
  const int64_t t1 = aether_wall_us();
  int r = aether_dev_sync();
  const int64_t t2 = aether_wall_us();
  fprintf(stderr, "[aether_dev] %d x matmul %dx%dx%d: enqueue %lld us, drain %lld us, %.1f us/call\n", iters, m, k, n,
          (long long)(t1 - t0), (long long)(t2 - t1), (double)(t2 - t0) / iters);
  return r;
}
// dx[n_in] = W^T dy for a frozen quantised W [n_out, n_in] (Q4_K = 12, Q6_K = 14):
// W is dequantised into a transient buffer and multiplied.
AE_API int aether_op_quant_matmul_backward_lhs_f32_cuda(int64_t w, int dt, int64_t dy, int64_t dx, int n_out,
                                                        int n_in) {
  if (dt != TQ4_K && dt != TQ6_K) return -2;
  if (n_out <= 0 || n_in <= 0 || n_in % 256) return -1;
  int ne, nb;
  block_of(dt, &ne, &nb);
  const size_t nblk = (size_t)n_out * (n_in / 256);
  const uint8_t* wq = U(w, nblk * nb);
  const float* g = F(dy, n_out);
  float* o = F(dx, n_in);
  Ctx* c = ctx();
  if (!wq || !g || !o || !c) return -1;
  float* wf = nullptr;
  if (cudaMallocAsync(&wf, nblk * 256 * 4, c->s) != cudaSuccess) return -2;
  int r = dequant_typed(dt, wq, wf, nblk * 8);
  if (!r) r = gemm_rm(false, false, 1, n_in, n_out, 1.f, g, n_out, wf, n_in, 0.f, o, n_in);
  cudaFreeAsync(wf, c->s);
  return r;
}

// ================================================================================================ elementwise ops
#define EW_LAUNCH(kern, n, ...)                                   \
  do {                                                            \
    Ctx* c_ = ctx();                                              \
    if (!c_) return -1;                                           \
    kern<<<blocks(n), 256, 0, c_->s>>>(__VA_ARGS__);              \
    return launched(#kern);                                       \
  } while (0)

AE_API int aether_op_add_f32_cuda(int64_t a, int64_t b, int64_t out, int n) {
  const float *pa = F(a, n), *pb = F(b, n);
  float* po = F(out, n);
  if (n <= 0 || !pa || !pb || !po) return -1;
  EW_LAUNCH(k_add, n, pa, pb, po, (size_t)n);
}
AE_API int aether_op_add_inplace_f32_cuda(int64_t x, int64_t y, int n) {
  float* px = F(x, n);
  const float* py = F(y, n);
  if (n <= 0 || !px || !py) return -1;
  EW_LAUNCH(k_add_inplace, n, px, py, (size_t)n);
}
AE_API int aether_op_mul_inplace_f32_cuda(int64_t x, int64_t y, int n) {
  float* px = F(x, n);
  const float* py = F(y, n);
  if (n <= 0 || !px || !py) return -1;
  EW_LAUNCH(k_mul_inplace, n, px, py, (size_t)n);
}
AE_API int aether_op_scale_f32_cuda(int64_t x, float s, int n) {
  float* px = F(x, n);
  if (n <= 0 || !px) return -1;
  EW_LAUNCH(k_scale, n, px, s, (size_t)n);
}
AE_API int aether_op_gelu_f32_cuda(int64_t x, int64_t y, int n) {
  const float* px = F(x, n);
  float* py = F(y, n);
  if (n <= 0 || !px || !py) return -1;
  EW_LAUNCH(k_gelu, n, px, py, (size_t)n);
}
AE_API int aether_op_gelu_backward_f32_cuda(int64_t x, int64_t dy, int64_t dx, int n) {
  const float *px = F(x, n), *pg = F(dy, n);
  float* po = F(dx, n);
  if (n <= 0 || !px || !pg || !po) return -1;
  EW_LAUNCH(k_gelu_bwd, n, px, pg, po, (size_t)n);
}
AE_API int aether_op_gelu_erf_f32_cuda(int64_t x, int64_t y, int n) {
  const float* px = F(x, n);
  float* py = F(y, n);
  if (n <= 0 || !px || !py) return -1;
  EW_LAUNCH(k_gelu_erf, n, px, py, (size_t)n);
}
AE_API int aether_op_silu_f32_cuda(int64_t x, int n) {
  float* px = F(x, n);
  if (n <= 0 || !px) return -1;
  EW_LAUNCH(k_silu, n, px, (size_t)n);
}
AE_API int aether_op_silu_backward_f32_cuda(int64_t x, int64_t dy, int64_t dx, int n) {
  const float *px = F(x, n), *pg = F(dy, n);
  float* po = F(dx, n);
  if (n <= 0 || !px || !pg || !po) return -1;
  EW_LAUNCH(k_silu_bwd, n, px, pg, po, (size_t)n);
}
AE_API int aether_op_bias_add_f32_cuda(int64_t x, int64_t bias, int rows, int cols) {
  const size_t n = (size_t)rows * cols;
  float* px = F(x, n);
  const float* pb = F(bias, cols);
  if (rows <= 0 || cols <= 0 || !px || !pb) return -1;
  EW_LAUNCH(k_bias_add, n, px, pb, (size_t)rows, cols);
}
AE_API int aether_op_transpose_021_f32_cuda(int64_t in, int64_t out, int d0, int d1, int d2) {
  const size_t n = (size_t)d0 * d1 * d2;
  const float* pi = F(in, n);
  float* po = F(out, n);
  if (d0 <= 0 || d1 <= 0 || d2 <= 0 || !pi || !po || pi == po) return -1;
  EW_LAUNCH(k_transpose_021, n, pi, po, d0, d1, d2);
}
AE_API int aether_op_embed_lookup_f32_cuda(int64_t table, int64_t ids, int64_t out, int t, int d) {
  if (t <= 0 || d <= 0) return -1;
  const int vocab = (int)(capacity(table, 4) / d);
  const float* pt = F(table, (size_t)vocab * d);
  const int* pi = I(ids, t);
  float* po = F(out, (size_t)t * d);
  if (vocab <= 0 || !pt || !pi || !po) return -1;
  EW_LAUNCH(k_embed, (size_t)t * d, pt, pi, po, t, d, vocab);
}
AE_API int aether_op_embed_scatter_add_f32_cuda(int64_t dout, int64_t ids, int64_t dtable, int t, int d) {
  if (t <= 0 || d <= 0) return -1;
  const int vocab = (int)(capacity(dtable, 4) / d);
  const float* pg = F(dout, (size_t)t * d);
  const int* pi = I(ids, t);
  float* pt = F(dtable, (size_t)vocab * d);
  if (vocab <= 0 || !pg || !pi || !pt) return -1;
  EW_LAUNCH(k_embed_scatter, (size_t)t * d, pg, pi, pt, t, d, vocab);
}
AE_API int aether_op_gqa_repeat_kv_f32_cuda(int64_t kv_in, int64_t kv_out, int seq, int hkv, int hd, int hq) {
  if (seq <= 0 || hkv <= 0 || hd <= 0 || hq <= 0 || hq % hkv) return -1;
  const float* pi = F(kv_in, (size_t)seq * hkv * hd);
  float* po = F(kv_out, (size_t)seq * hq * hd);
  if (!pi || !po) return -1;
  EW_LAUNCH(k_gqa_repeat, (size_t)seq * hq * hd, pi, po, seq, hkv, hd, hq);
}
AE_API int aether_op_gqa_reduce_kv_grad_f32_cuda(int64_t dkv_out, int64_t dkv_in, int seq, int hkv, int hd, int hq) {
  if (seq <= 0 || hkv <= 0 || hd <= 0 || hq <= 0 || hq % hkv) return -1;
  const float* pg = F(dkv_out, (size_t)seq * hq * hd);
  float* po = F(dkv_in, (size_t)seq * hkv * hd);
  if (!pg || !po) return -1;
  EW_LAUNCH(k_gqa_reduce, (size_t)seq * hkv * hd, pg, po, seq, hkv, hd, hq);
}
AE_API int aether_op_append_kv_f32_cuda(int64_t kn, int64_t vn, int64_t kc, int64_t vc, int pos, int dkv) {
  if (pos < 0 || dkv <= 0) return -1;
  const float *pk = F(kn, dkv), *pv = F(vn, dkv);
  float *ck = F(kc, (size_t)(pos + 1) * dkv), *cv = F(vc, (size_t)(pos + 1) * dkv);
  if (!pk || !pv || !ck || !cv) return -1;
  EW_LAUNCH(k_append_kv, dkv, pk, pv, ck, cv, pos, dkv);
}
// AdamW with decoupled weight decay inside the step (p -= lr (m^ / (sqrt(v^) + eps) + wd p)),
// bias corrections 1 / (1 - beta^step).
AE_API int aether_op_adamw_step_f32_cuda(int64_t param, int64_t grad, int64_t m, int64_t v, float lr, float b1, float b2,
                                         float eps, float wd, int64_t step, int n) {
  float* pp = F(param, n);
  const float* pg = F(grad, n);
  float *pm = F(m, n), *pv = F(v, n);
  if (n <= 0 || step <= 0 || !pp || !pg || !pm || !pv) return -1;
  const float bc1 = (float)(1.0 / (1.0 - std::pow((double)b1, (double)step)));
  const float bc2 = (float)(1.0 / (1.0 - std::pow((double)b2, (double)step)));
  EW_LAUNCH(k_adamw, n, pp, pg, pm, pv, lr, b1, b2, eps, wd, bc1, bc2, (size_t)n);
}
AE_API int aether_op_rope_apply_f32_cuda(int64_t x, int seq, int heads, int hd, float base, int pos0) {
  if (seq <= 0 || heads <= 0 || hd <= 0 || hd % 2) return -1;
  float* px = F(x, (size_t)seq * heads * hd);
  if (!px) return -1;
  EW_LAUNCH(k_rope, (size_t)seq * heads * (hd / 2), px, seq, heads, hd, base, pos0, 1.f);
}
AE_API int aether_op_rope_apply_backward_f32_cuda(int64_t g, int seq, int heads, int hd, float base, int pos0) {
  if (seq <= 0 || heads <= 0 || hd <= 0 || hd % 2) return -1;
  float* px = F(g, (size_t)seq * heads * hd);
  if (!px) return -1;
  EW_LAUNCH(k_rope, (size_t)seq * heads * (hd / 2), px, seq, heads, hd, base, pos0, -1.f);
}

// ================================================================================================ row ops
#define ROW_LAUNCH(kern, rows, ...)                                     \
  do {                                                                  \
    Ctx* c_ = ctx();                                                    \
    if (!c_) return -1;                                                 \
    kern<<<(unsigned)(rows), kRowThreads, 0, c_->s>>>(__VA_ARGS__);     \
    return launched(#kern);                                             \
  } while (0)

AE_API int aether_op_softmax_f32_cuda(int64_t x, int64_t y, int b, int d) {
  const size_t n = (size_t)b * d;
  const float* px = F(x, n);
  float* py = F(y, n);
  if (b <= 0 || d <= 0 || !px || !py) return -1;
  ROW_LAUNCH(k_softmax, b, px, py, d);
}
AE_API int aether_op_softmax_backward_scaled_f32_cuda(int64_t y, int64_t dy, int64_t dx, float s, int b, int d) {
  const size_t n = (size_t)b * d;
  const float *py = F(y, n), *pg = F(dy, n);
  float* po = F(dx, n);
  if (b <= 0 || d <= 0 || !py || !pg || !po) return -1;
  ROW_LAUNCH(k_softmax_bwd, b, py, pg, po, d, s);
}
AE_API int aether_op_softmax_backward_f32_cuda(int64_t y, int64_t dy, int64_t dx, int b, int d) {
  return aether_op_softmax_backward_scaled_f32_cuda(y, dy, dx, 1.f, b, d);
}
AE_API int aether_op_layer_norm_f32_cuda(int64_t x, int64_t gamma, int64_t beta, int64_t y, int64_t mean, int64_t rstd,
                                         float eps, int b, int d) {
  const size_t n = (size_t)b * d;
  const float *px = F(x, n), *pg = F(gamma, d), *pb = F(beta, d);
  float *py = F(y, n), *pm = F(mean, b), *pr = F(rstd, b);
  if (b <= 0 || d <= 0 || !px || !pg || !pb || !py || !pm || !pr) return -1;
  ROW_LAUNCH(k_layernorm, b, px, nullptr, pg, pb, py, pm, pr, eps, d);
}
AE_API int aether_op_add_layer_norm_f32_cuda(int64_t a, int64_t bb, int64_t gamma, int64_t beta, int64_t y, int64_t mean,
                                             int64_t rstd, float eps, int b, int d) {
  const size_t n = (size_t)b * d;
  const float *pa = F(a, n), *p2 = F(bb, n), *pg = F(gamma, d), *pb = F(beta, d);
  float *py = F(y, n), *pm = F(mean, b), *pr = F(rstd, b);
  if (b <= 0 || d <= 0 || !pa || !p2 || !pg || !pb || !py || !pm || !pr) return -1;
  ROW_LAUNCH(k_layernorm, b, pa, p2, pg, pb, py, pm, pr, eps, d);
}
AE_API int aether_op_layer_norm_backward_dx_f32_cuda(int64_t x, int64_t gamma, int64_t mean, int64_t rstd, int64_t dy,
                                                     int64_t dx, int b, int d) {
  const size_t n = (size_t)b * d;
  const float *px = F(x, n), *pg = F(gamma, d), *pm = F(mean, b), *pr = F(rstd, b), *pd = F(dy, n);
  float* po = F(dx, n);
  if (b <= 0 || d <= 0 || !px || !pg || !pm || !pr || !pd || !po) return -1;
  ROW_LAUNCH(k_layernorm_bwd_dx, b, px, pg, pm, pr, pd, po, d);
}
AE_API int aether_op_layer_norm_backward_params_f32_cuda(int64_t x, int64_t mean, int64_t rstd, int64_t dy,
                                                         int64_t dgamma, int64_t dbeta, int b, int d) {
  const size_t n = (size_t)b * d;
  const float *px = F(x, n), *pm = F(mean, b), *pr = F(rstd, b), *pd = F(dy, n);
  float *pg = F(dgamma, d), *pb = F(dbeta, d);
  Ctx* c = ctx();
  if (b <= 0 || d <= 0 || !px || !pm || !pr || !pd || !pg || !pb || !c) return -1;
  k_colsum<<<blocks(d, 32), dim3(32, 8), 0, c->s>>>(px, pd, pm, pr, pg, pb, b, d, 0);
  return launched("layer_norm_backward_params");
}
AE_API int aether_op_rms_norm_f32_cuda(int64_t x, int64_t gamma, int64_t out, float eps, int rows, int d) {
  const size_t n = (size_t)rows * d;
  float* px = F(x, n);
  const float* pg = F(gamma, d);
  float* po = F(out, n);
  if (rows <= 0 || d <= 0 || !px || !pg || !po) return -1;
  ROW_LAUNCH(k_rmsnorm, rows, px, nullptr, pg, po, eps, d);
}
// x += residual (in place); out = rmsnorm(x) * gamma
AE_API int aether_op_fused_add_rmsnorm_f32_cuda(int64_t x, int64_t residual, int64_t gamma, int64_t out, float eps,
                                                int rows, int d) {
  const size_t n = (size_t)rows * d;
  float* px = F(x, n);
  const float *pr = F(residual, n), *pg = F(gamma, d);
  float* po = F(out, n);
  if (rows <= 0 || d <= 0 || !px || !pr || !pg || !po) return -1;
  ROW_LAUNCH(k_rmsnorm, rows, px, pr, pg, po, eps, d);
}
AE_API int aether_op_rms_norm_backward_dx_f32_cuda(int64_t x, int64_t gamma, int64_t dy, int64_t dx, int64_t inv_rms,
                                                   float eps, int rows, int d) {
  const size_t n = (size_t)rows * d;
  const float *px = F(x, n), *pg = F(gamma, d), *pd = F(dy, n);
  float *po = F(dx, n), *pi = F(inv_rms, rows);
  if (rows <= 0 || d <= 0 || !px || !pg || !pd || !po || !pi) return -1;
  ROW_LAUNCH(k_rmsnorm_bwd_dx, rows, px, pg, pd, po, pi, eps, d);
}
AE_API int aether_op_rms_norm_backward_gamma_f32_cuda(int64_t x, int64_t dy, int64_t inv_rms, int64_t dgamma, int rows,
                                                      int d) {
  const size_t n = (size_t)rows * d;
  const float *px = F(x, n), *pd = F(dy, n), *pi = F(inv_rms, rows);
  float* pg = F(dgamma, d);
  Ctx* c = ctx();
  if (rows <= 0 || d <= 0 || !px || !pd || !pi || !pg || !c) return -1;
  k_colsum<<<blocks(d, 32), dim3(32, 8), 0, c->s>>>(px, pd, nullptr, pi, pg, nullptr, rows, d, 1);
  return launched("rms_norm_backward_gamma");
}
// Mean cross-entropy over b rows (per-row losses summed on the host in double);
// probs_out gets the softmax. Returns NaN on a bad handle.
AE_API float aether_op_cross_entropy_f32_cuda(int64_t logits, int64_t labels, int64_t probs, int b, int v) {
  const size_t n = (size_t)b * v;
  const float* pl = F(logits, n);
  const int* pt = I(labels, b);
  float* pp = F(probs, n);
  Ctx* c = ctx();
  if (b <= 0 || v <= 0 || !pl || !pt || !pp || !c) return NAN;
  float* loss = nullptr;
  if (cudaMallocAsync(&loss, (size_t)b * 4, c->s) != cudaSuccess) return NAN;
  k_ce_fwd<<<(unsigned)b, kRowThreads, 0, c->s>>>(pl, pt, pp, loss, v);
  std::vector<float> h(b);
  cudaMemcpyAsync(h.data(), loss, (size_t)b * 4, cudaMemcpyDeviceToHost, c->s);
  cudaFreeAsync(loss, c->s);
  if (cudaStreamSynchronize(c->s) != cudaSuccess) return NAN;
  double s = 0.0;
  for (float x : h) s += x;
  return (float)(s / b);
}
// dlogits = (probs - onehot(label)) / b
AE_API int aether_op_cross_entropy_backward_f32_cuda(int64_t probs, int64_t labels, int64_t dlogits, int b, int v) {
  const size_t n = (size_t)b * v;
  const float* pp = F(probs, n);
  const int* pt = I(labels, b);
  float* pd = F(dlogits, n);
  if (b <= 0 || v <= 0 || !pp || !pt || !pd) return -1;
  EW_LAUNCH(k_ce_bwd, n, pp, pt, pd, b, v);
}

// ================================================================================================ attention
// Causal SDPA over [bh, s, d] with the [bh, s, s] probabilities kept for the
// backward: two strided-batched GEMMs around a causal row softmax, scale 1/sqrt(d).
AE_API int aether_op_sdpa_causal_forward_f32_cuda(int64_t q, int64_t k, int64_t v, int64_t out, int64_t attn, int bh,
                                                  int s, int d) {
  if (bh <= 0 || s <= 0 || d <= 0) return -1;
  const size_t nq = (size_t)bh * s * d, na = (size_t)bh * s * s;
  const float *pq = F(q, nq), *pk = F(k, nq), *pv = F(v, nq);
  float *po = F(out, nq), *pa = F(attn, na);
  Ctx* c = ctx();
  if (!pq || !pk || !pv || !po || !pa || !c) return -1;
  const float scale = 1.f / std::sqrt((float)d);
  const long long sq = (long long)s * d, ss = (long long)s * s;
  int r = gemm_rm(false, true, s, s, d, scale, pq, d, pk, d, 0.f, pa, s, bh, sq, sq, ss);
  if (r) return r;
  k_causal_softmax<<<(unsigned)(bh * s), kRowThreads, 0, c->s>>>(pa, s);
  if ((r = launched("causal_softmax"))) return r;
  return gemm_rm(false, false, s, d, s, 1.f, pa, s, pv, d, 0.f, po, d, bh, ss, sq, sq);
}

AE_API int aether_op_sdpa_causal_backward_f32_cuda(int64_t q, int64_t k, int64_t v, int64_t attn, int64_t dout,
                                                   int64_t dq, int64_t dk, int64_t dv, int64_t dscores, int bh, int s,
                                                   int d) {
  if (bh <= 0 || s <= 0 || d <= 0) return -1;
  const size_t nq = (size_t)bh * s * d, na = (size_t)bh * s * s;
  const float *pq = F(q, nq), *pk = F(k, nq), *pv = F(v, nq), *pa = F(attn, na), *pg = F(dout, nq);
  float *gq = F(dq, nq), *gk = F(dk, nq), *gv = F(dv, nq), *ps = F(dscores, na);
  Ctx* c = ctx();
  if (!pq || !pk || !pv || !pa || !pg || !gq || !gk || !gv || !ps || !c) return -1;
  const float scale = 1.f / std::sqrt((float)d);
  const long long sq = (long long)s * d, ss = (long long)s * s;
  int r;
  // dV = P^T dO ; dP = dO V^T
  if ((r = gemm_rm(true, false, s, d, s, 1.f, pa, s, pg, d, 0.f, gv, d, bh, ss, sq, sq))) return r;
  if ((r = gemm_rm(false, true, s, s, d, 1.f, pg, d, pv, d, 0.f, ps, s, bh, sq, sq, ss))) return r;
  // dS = scale * P * (dP - rowsum(dP * P))  (zero above the diagonal since P is)
  k_softmax_bwd<<<(unsigned)(bh * s), kRowThreads, 0, c->s>>>(pa, ps, ps, s, scale);
  if ((r = launched("sdpa_softmax_bwd"))) return r;
  // dQ = dS K ; dK = dS^T Q
  if ((r = gemm_rm(false, false, s, d, s, 1.f, ps, s, pk, d, 0.f, gq, d, bh, ss, sq, sq))) return r;
  return gemm_rm(true, false, s, d, s, 1.f, ps, s, pq, d, 0.f, gk, d, bh, ss, sq, sq);
}

// One decode token: q [hq * hd] against the first cur_seq rows of the KV cache.
AE_API int aether_op_attention_seq1_f32_cuda(int64_t q, int64_t kc, int64_t vc, int64_t out, int cur, int hq, int hkv,
                                             int hd, float scale) {
  if (cur <= 0 || hq <= 0 || hkv <= 0 || hd <= 0 || hq % hkv) return -1;
  const size_t smem = (size_t)cur * 4;
  if (smem > 200 * 1024) return -1;  // scores live in shared memory
  const float* pq = F(q, (size_t)hq * hd);
  const float *pk = F(kc, (size_t)cur * hkv * hd), *pv = F(vc, (size_t)cur * hkv * hd);
  float* po = F(out, (size_t)hq * hd);
  Ctx* c = ctx();
  if (!pq || !pk || !pv || !po || !c) return -1;
  if (smem > 48 * 1024) cudaFuncSetAttribute(k_attn_seq1, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  k_attn_seq1<<<(unsigned)hq, 256, smem, c->s>>>(pq, pk, pv, po, cur, hq, hkv, hd, scale);
  return launched("attention_seq1");
}

// ================================================================================================ quantised weights
// Dequantise n_blocks GGUF blocks (u8 handle) into f32 (256 values per K-quant super-block).
AE_API int aether_op_dequant_q4_k_m_f32_cuda(int64_t blk, int64_t out, int n) { return dequant_handle(TQ4_K, blk, out, n); }
AE_API int aether_op_dequant_q6_k_f32_cuda(int64_t blk, int64_t out, int n) { return dequant_handle(TQ6_K, blk, out, n); }
// Any supported GGML type number (Q4_0, Q5_0, Q8_0, Q3_K..Q6_K, IQ4_NL, IQ4_XS).
AE_API int aether_op_dequant_f32_cuda(int dt, int64_t blk, int64_t out, int n) { return dequant_handle(dt, blk, out, n); }

// out[n] = W[n, k] a[k] with W in GGUF blocks (k = n_blocks * block elements)
AE_API int aether_op_fused_q4k_matmul_seq1_cuda(int64_t a, int64_t w, int64_t o, int n, int nb) {
  return qmatvec(TQ4_K, a, w, o, n, nb);
}
AE_API int aether_op_fused_q4_0_matmul_seq1_cuda(int64_t a, int64_t w, int64_t o, int n, int nb) {
  return qmatvec(TQ4_0, a, w, o, n, nb);
}
AE_API int aether_op_fused_q5_0_matmul_seq1_cuda(int64_t a, int64_t w, int64_t o, int n, int nb) {
  return qmatvec(TQ5_0, a, w, o, n, nb);
}
AE_API int aether_op_fused_q8_0_matmul_seq1_cuda(int64_t a, int64_t w, int64_t o, int n, int nb) {
  return qmatvec(TQ8_0, a, w, o, n, nb);
}
AE_API int aether_op_fused_q5_k_matmul_seq1_cuda(int64_t a, int64_t w, int64_t o, int n, int nb) {
  return qmatvec(TQ5_K, a, w, o, n, nb);
}
AE_API int aether_op_fused_q3_k_matmul_seq1_cuda(int64_t a, int64_t w, int64_t o, int n, int nb) {
  return qmatvec(TQ3_K, a, w, o, n, nb);
}
AE_API int aether_op_fused_iq4_nl_matmul_seq1_cuda(int64_t a, int64_t w, int64_t o, int n, int nb) {
  return qmatvec(TIQ4_NL, a, w, o, n, nb);
}
AE_API int aether_op_fused_iq4_xs_matmul_seq1_cuda(int64_t a, int64_t w, int64_t o, int n, int nb) {
  return qmatvec(TIQ4_XS, a, w, o, n, nb);
}
AE_API int aether_op_fused_q6k_matmul_seq1_v2_cuda(int64_t a, int64_t w, int64_t o, int n, int nb) {
  return qmatvec(TQ6_K, a, w, o, n, nb);
}
// The reference's successive Q4_K kernel versions share one interface; all run the kernel above.
AE_API int aether_op_fused_q4k_matmul_seq1_v2_cuda(int64_t a, int64_t w, int64_t o, int n, int nb) {
  return qmatvec(TQ4_K, a, w, o, n, nb);
}
AE_API int aether_op_fused_q4k_matmul_seq1_v3_cuda(int64_t a, int64_t w, int64_t o, int n, int nb) {
  return qmatvec(TQ4_K, a, w, o, n, nb);
}
AE_API int aether_op_fused_q4k_matmul_seq1_v4_cuda(int64_t a, int64_t w, int64_t o, int n, int nb) {
  return qmatvec(TQ4_K, a, w, o, n, nb);
}
AE_API int aether_op_fused_q4k_matmul_seq1_v5_cuda(int64_t a, int64_t w, int64_t o, int n, int nb) {
  return qmatvec(TQ4_K, a, w, o, n, nb);
}
AE_API int aether_op_fused_q4k_matmul_seq1_v6_cuda(int64_t a, int64_t w, int64_t o, int n, int nb) {
  return qmatvec(TQ4_K, a, w, o, n, nb);
}
// out[n] = silu(W_gate a) * (W_up a), both Q4_K, in one pass over a
AE_API int aether_op_fused_q4k_ffn_gate_up_silu_mul_cuda(int64_t a, int64_t wg, int64_t wu, int64_t o, int n, int nb) {
  return qmatvec(TQ4_K, a, wg, o, n, nb, 0, wu);
}
AE_API int aether_op_fused_q4k_ffn_gate_up_silu_mul_v2_cuda(int64_t a, int64_t wg, int64_t wu, int64_t o, int n,
                                                           int nb) {
  return qmatvec(TQ4_K, a, wg, o, n, nb, 0, wu);
}
// y[o] = sum_i x[i] W[o, i] for F16 / F32 weights held in u8 buffers
AE_API int aether_op_fused_f16_matmul_seq1_cuda(int64_t x, int64_t w, int64_t y, int n_in, int n_out) {
  return qmatvec(TF16, x, w, y, n_out, n_in);
}
AE_API int aether_op_fused_f32_matmul_seq1_cuda(int64_t x, int64_t w, int64_t y, int n_in, int n_out) {
  return qmatvec(TF32, x, w, y, n_out, n_in);
}
// Expert e of a stacked [E, n_out, k] quantised expert tensor
AE_API int aether_op_fused_q4k_expert_matmul_seq1_cuda(int64_t x, int64_t w, int64_t y, int n_out, int bpr, int e) {
  return qmatvec(TQ4_K, x, w, y, n_out, bpr, e);
}
AE_API int aether_op_fused_q8_0_expert_matmul_seq1_cuda(int64_t x, int64_t w, int64_t y, int n_out, int bpr, int e) {
  return qmatvec(TQ8_0, x, w, y, n_out, bpr, e);
}
AE_API int aether_op_fused_q5_0_expert_matmul_seq1_cuda(int64_t x, int64_t w, int64_t y, int n_out, int bpr, int e) {
  return qmatvec(TQ5_0, x, w, y, n_out, bpr, e);
}
AE_API int aether_op_fused_q3_k_expert_matmul_seq1_cuda(int64_t x, int64_t w, int64_t y, int n_out, int bpr, int e) {
  return qmatvec(TQ3_K, x, w, y, n_out, bpr, e);
}
AE_API int aether_op_fused_q6_k_expert_matmul_seq1_cuda(int64_t x, int64_t w, int64_t y, int n_out, int bpr, int e) {
  return qmatvec(TQ6_K, x, w, y, n_out, bpr, e);
}
AE_API int aether_op_fused_q5_k_expert_matmul_seq1_cuda(int64_t x, int64_t w, int64_t y, int n_out, int bpr, int e) {
  return qmatvec(TQ5_K, x, w, y, n_out, bpr, e);
}
AE_API int aether_op_fused_iq4_xs_expert_matmul_seq1_cuda(int64_t x, int64_t w, int64_t y, int n_out, int bpr, int e) {
  return qmatvec(TIQ4_XS, x, w, y, n_out, bpr, e);
}
// IQ3_XXS / IQ3_S (GLM-4.7-flash's quantisation): dense and expert mat-vecs, dequantiser
AE_API int aether_op_fused_iq3_xxs_matmul_seq1_cuda(int64_t a, int64_t w, int64_t o, int n, int nb) {
  return qmatvec(TIQ3_XXS, a, w, o, n, nb);
}
AE_API int aether_op_fused_iq3_s_matmul_seq1_cuda(int64_t a, int64_t w, int64_t o, int n, int nb) {
  return qmatvec(TIQ3_S, a, w, o, n, nb);
}
AE_API int aether_op_fused_iq3_xxs_expert_matmul_seq1_cuda(int64_t x, int64_t w, int64_t y, int n_out, int bpr,
                                                           int e) {
  return qmatvec(TIQ3_XXS, x, w, y, n_out, bpr, e);
}
AE_API int aether_op_fused_iq3_s_expert_matmul_seq1_cuda(int64_t x, int64_t w, int64_t y, int n_out, int bpr, int e) {
  return qmatvec(TIQ3_S, x, w, y, n_out, bpr, e);
}
AE_API int aether_op_dequant_iq3_xxs_f32_cuda(int64_t blk, int64_t out, int n) {
  return dequant_handle(TIQ3_XXS, blk, out, n);
}

// ================================================================================================ NCCL clique
// One process driving n local GPUs (ncclCommInitAll): comm handle i + 1 is
// rank i on device i. A single thread drives every rank, so the per-rank
// all-reduce calls are queued and issued together in one NCCL group once every
// rank of the clique has called (in any order); a 1-GPU clique runs at once.
// Buffers are device handles allocated on the rank's device
// (aether_dev_set_device(i) first). Op codes: 0 sum, 1 max, 2 min, 3 prod.
namespace {
struct NComm {
  ncclComm_t c;
  int dev;
};
struct NPending {
  const float* s;
  float* r;
  size_t n;
  ncclRedOp_t op;
  int rank;
};
std::vector<NComm> g_comms;
std::vector<NPending> g_npend;
std::mutex g_nmu;

int nccl_flush_locked() {
  int prev = cur_dev();
  int rc = 0;
  if (ncclGroupStart() != ncclSuccess) return -2;
  for (const NPending& p : g_npend) {
    Ctx* c = ctx_for(g_comms[p.rank].dev);
    cudaSetDevice(g_comms[p.rank].dev);
    if (!c || ncclAllReduce(p.s, p.r, p.n, ncclFloat, p.op, g_comms[p.rank].c, c->s) != ncclSuccess) rc = -2;
  }
  if (ncclGroupEnd() != ncclSuccess) rc = -2;
  g_npend.clear();
  if (prev >= 0) cudaSetDevice(prev);
  return rc;
}
}  // namespace

AE_API int aether_nccl_real_finalize() {
  std::lock_guard<std::mutex> l(g_nmu);
  for (NComm& c : g_comms) ncclCommDestroy(c.c);
  g_comms.clear();
  g_npend.clear();
  return 0;
}

AE_API int aether_nccl_real_init_multi_gpu(int n) {
  int have = 0;
  if (n <= 0 || cudaGetDeviceCount(&have) != cudaSuccess || have < n) return -1;
  aether_nccl_real_finalize();
  std::vector<ncclComm_t> cs(n);
  std::vector<int> devs(n);
  for (int i = 0; i < n; ++i) {
    devs[i] = i;
    if (!ctx_for(i)) return -2;
  }
  if (ncclCommInitAll(cs.data(), n, devs.data()) != ncclSuccess) return -3;
  std::lock_guard<std::mutex> l(g_nmu);
  for (int i = 0; i < n; ++i) g_comms.push_back({cs[i], i});
  return n;
}

AE_API int64_t aether_nccl_real_get_handle(int i) {
  std::lock_guard<std::mutex> l(g_nmu);
  return (i >= 0 && (size_t)i < g_comms.size()) ? (int64_t)i + 1 : 0;
}

AE_API int aether_nccl_real_comm_world_size(int64_t comm) {
  std::lock_guard<std::mutex> l(g_nmu);
  return (comm >= 1 && (size_t)comm <= g_comms.size()) ? (int)g_comms.size() : -1;
}

AE_API int aether_nccl_real_comm_rank(int64_t comm) {
  std::lock_guard<std::mutex> l(g_nmu);
  return (comm >= 1 && (size_t)comm <= g_comms.size()) ? (int)comm - 1 : -1;
}

AE_API int aether_nccl_real_all_reduce_f32(int64_t send, int64_t recv, int n, int op, int64_t comm) {
  static const ncclRedOp_t ops[4] = {ncclSum, ncclMax, ncclMin, ncclProd};
  if (n <= 0 || op < 0 || op > 3) return -1;
  const float* s = F(send, n);
  float* r = F(recv, n);
  int sdev, rdev;
  {
    std::lock_guard<std::mutex> l(g_mu);
    sdev = s ? g_bufs[send - 1].dev : -1;
    rdev = r ? g_bufs[recv - 1].dev : -1;
  }
  std::lock_guard<std::mutex> l(g_nmu);
  if (!s || !r || comm < 1 || (size_t)comm > g_comms.size()) return -1;
  const int rank = (int)comm - 1;
  if (sdev != g_comms[rank].dev || rdev != g_comms[rank].dev) return -1;  // buffers live on the rank's GPU
  for (const NPending& p : g_npend)
    if (p.rank == rank || p.n != (size_t)n || p.op != ops[op]) return -1;  // one call per rank, same shape
  g_npend.push_back({s, r, (size_t)n, ops[op], rank});
  return g_npend.size() == g_comms.size() ? nccl_flush_locked() : 0;
}

// ================================================================================================ decode-step ops
// Variants of the decode ops that read the step's position / length from a
// device i32 buffer (step_args[0] = position, step_args[1] = current length;
// batched forms take one value per sequence), so a captured decode graph is
// replayed with only that buffer rewritten. KV caches are contiguous
// ([rows, d_row]) or paged pools ([physical blocks * block_size, d_row]) read
// through a page table (row = table[t / block_size] * block_size + t % block_size).
// Every device-side index is checked against the table length and the pool's
// rows: an out-of-range entry is skipped (its key is masked, its write dropped).
namespace {

struct RopeArgs {
  float* x;
  int rows, heads, hs, off, rd;  // rows x heads slices of stride hs; RoPE on dims [off, off + rd)
  float base;
  const int* pos;  // per_row ? pos[r] : pos[0] + r
  int per_row;
  float ys, yctx, yfast, yslow;  // YaRN (ys > 1)
};

// YaRN per-pair frequency factor: 1 for fast-rotating pairs, 1 / s for slow
// ones, linear in between over the pairs whose wavelength lies between
// beta_fast and beta_slow rotations of the original context.
__device__ float yarn_factor(int i, int rd, float base, float s, float ctx, float bfast, float bslow) {
  if (s <= 1.f) return 1.f;
  const float two_pi = 6.283185307179586f;
  const float lo = fmaxf(floorf(rd * logf(ctx / (bfast * two_pi)) / (2.f * logf(base))), 0.f);
  float hi = fminf(ceilf(rd * logf(ctx / (bslow * two_pi)) / (2.f * logf(base))), (float)(rd - 1));
  if (lo == hi) hi += 0.001f;
  const float ramp = fminf(fmaxf(((float)i - lo) / (hi - lo), 0.f), 1.f);
  return ramp / s + (1.f - ramp);
}

__global__ void k_rope_dev(RopeArgs a) {
  const int half = a.rd / 2;
  const size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= (size_t)a.rows * a.heads * half) return;
  const int j = (int)(i % half);
  const size_t rh = i / half;
  const int h = (int)(rh % a.heads), r = (int)(rh / a.heads);
  const int pos = a.per_row ? a.pos[r] : a.pos[0] + r;
  const float ang = (float)pos * yarn_factor(j, a.rd, a.base, a.ys, a.yctx, a.yfast, a.yslow) *
                    powf(a.base, -2.f * (float)j / (float)a.rd);
  float sn, cs;
  sincosf(ang, &sn, &cs);
  float* v = a.x + ((size_t)r * a.heads + h) * a.hs + a.off;
  const float x0 = v[j], x1 = v[j + half];
  v[j] = x0 * cs - x1 * sn;
  v[j + half] = x0 * sn + x1 * cs;
}

// q, k, v += biases, then RoPE on q and k at step_args[0], in one launch.
__global__ void k_qkv_bias_rope(float* q, float* k, float* v, const float* bq, const float* bk, const float* bv, int hq,
                                int hkv, int hd, float base, const int* step) {
  const int half = hd / 2;
  const int nq = hq * half, nk = hkv * half, nv = hkv * hd;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nq + nk + nv) return;
  if (i >= nq + nk) {
    const int e = i - nq - nk;
    v[e] += bv[e];
    return;
  }
  float* x = i < nq ? q : k;
  const float* b = i < nq ? bq : bk;
  const int pi = i < nq ? i : i - nq;
  const int h = pi / half, j = pi % half;
  const int o0 = h * hd + j, o1 = o0 + half;
  const float x0 = x[o0] + b[o0], x1 = x[o1] + b[o1];
  float sn, cs;
  sincosf((float)step[0] * powf(base, -2.f * (float)j / (float)hd), &sn, &cs);
  x[o0] = x0 * cs - x1 * sn;
  x[o1] = x0 * sn + x1 * cs;
}

struct AppendArgs {
  const float* kn;
  const float* vn;
  float* kp;
  float* vp;
  const int* pt;  // null: contiguous cache
  int pt_stride, bs, dk, dv;
  const int* pos;  // per_batch ? pos[b] : pos[0]
  int per_batch;
  long long rows_k, rows_v;
};

__device__ __forceinline__ long long kv_row(const int* pt, int pt_stride, int b, int bs, int t) {
  if (!pt) return t;
  const int blk = t / bs;
  if (blk >= pt_stride) return -1;
  const int phys = pt[(size_t)b * pt_stride + blk];
  return phys < 0 ? -1 : (long long)phys * bs + t % bs;
}

__global__ void k_append_dev(AppendArgs a) {
  const int b = blockIdx.y;
  const int pos = a.per_batch ? a.pos[b] : a.pos[0];
  if (pos < 0) return;
  const long long row = kv_row(a.pt, a.pt_stride, b, a.bs, pos);
  if (row < 0) return;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < a.dk && row < a.rows_k) a.kp[row * a.dk + i] = a.kn[(size_t)b * a.dk + i];
  if (i < a.dv && row < a.rows_v) a.vp[row * a.dv + i] = a.vn[(size_t)b * a.dv + i];
}

struct AttnArgs {
  const float* q;
  const float* kp;
  const float* vp;
  const int* pt;
  int pt_stride;
  float* out;
  int hq, hkv, dk, dv, bs;
  float scale;
  int window;        // > 0: only the last `window` positions
  const int* cur;    // null: cur_const; else per_batch ? cur[b] : cur[1]
  int cur_per_batch, cur_const, max_seq;
  long long rows_k, rows_v;
  long long q_bstride, o_bstride;
  int n_split;       // > 1: partials to sm / sl / sv, merged by k_attn_combine
  float* sm;
  float* sl;
  float* sv;
};

// One query token per (head, batch row[, split]): scores in shared memory (a
// warp per key), softmax, then a thread per output dim sums over the keys.
__global__ void k_attn_dev(AttnArgs a) {
  extern __shared__ float sc[];
  const int h = blockIdx.x, b = blockIdx.y, sp = blockIdx.z;
  int cur = a.cur ? (a.cur_per_batch ? a.cur[b] : a.cur[1]) : a.cur_const;
  cur = min(max(cur, 0), a.max_seq);
  const int lo = a.window > 0 ? max(0, cur - a.window) : 0;
  const int per = (cur - lo + a.n_split - 1) / a.n_split;
  const int t0 = lo + sp * per, t1 = min(cur, t0 + per);
  const int n = max(t1 - t0, 0);
  const int kvh = h / (a.hq / a.hkv);
  const float* q = a.q + b * a.q_bstride + (size_t)h * a.dk;
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int t = w; t < n; t += nw) {
    const long long row = kv_row(a.pt, a.pt_stride, b, a.bs, t0 + t);
    float acc = 0.f;
    const bool ok = row >= 0 && row < a.rows_k;
    if (ok) {
      const float* kr = a.kp + row * (long long)(a.hkv * a.dk) + (size_t)kvh * a.dk;
      for (int d = l; d < a.dk; d += 32) acc += q[d] * kr[d];
      acc = warp_sum(acc);
    }
    if (l == 0) sc[t] = ok ? acc * a.scale : -INFINITY;
  }
  __syncthreads();
  float m = -INFINITY;
  for (int t = threadIdx.x; t < n; t += blockDim.x) m = fmaxf(m, sc[t]);
  m = block_max(m);
  float sum = 0.f;
  for (int t = threadIdx.x; t < n; t += blockDim.x) {
    const float e = m == -INFINITY ? 0.f : expf(sc[t] - m);
    sc[t] = e;
    sum += e;
  }
  sum = block_sum(sum);
  for (int d = threadIdx.x; d < a.dv; d += blockDim.x) {
    float acc = 0.f;
    for (int t = 0; t < n; ++t) {
      const long long row = kv_row(a.pt, a.pt_stride, b, a.bs, t0 + t);
      if (row >= 0 && row < a.rows_v && sc[t] != 0.f)
        acc += sc[t] * a.vp[row * (long long)(a.hkv * a.dv) + (size_t)kvh * a.dv + d];
    }
    if (a.n_split > 1) {
      a.sv[((size_t)h * a.n_split + sp) * a.dv + d] = acc;
    } else {
      a.out[b * a.o_bstride + (size_t)h * a.dv + d] = sum > 0.f ? acc / sum : 0.f;
    }
  }
  if (a.n_split > 1 && threadIdx.x == 0) {
    a.sm[(size_t)h * a.n_split + sp] = m;
    a.sl[(size_t)h * a.n_split + sp] = sum;
  }
}

// Merge the splits of each head: out = sum_s v_s e^(m_s - M) / sum_s l_s e^(m_s - M).
__global__ void k_attn_combine(const float* sm, const float* sl, const float* sv, float* out, int n_split, int dv) {
  const int h = blockIdx.x;
  float M = -INFINITY;
  for (int s = 0; s < n_split; ++s) M = fmaxf(M, sm[(size_t)h * n_split + s]);
  float L = 0.f;
  for (int s = 0; s < n_split; ++s) {
    const float ms = sm[(size_t)h * n_split + s];
    L += ms == -INFINITY ? 0.f : sl[(size_t)h * n_split + s] * expf(ms - M);
  }
  for (int d = threadIdx.x; d < dv; d += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < n_split; ++s) {
      const float ms = sm[(size_t)h * n_split + s];
      if (ms != -INFINITY) acc += sv[((size_t)h * n_split + s) * dv + d] * expf(ms - M);
    }
    out[(size_t)h * dv + d] = L > 0.f ? acc / L : 0.f;
  }
}

int attn_launch(AttnArgs a, int batch) {
  Ctx* c = ctx();
  if (!c) return -1;
  const size_t smem = (size_t)a.max_seq * 4;
  if (a.max_seq <= 0 || smem > 200 * 1024 || a.hq % a.hkv) return -1;
  if (smem > 48 * 1024) cudaFuncSetAttribute(k_attn_dev, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  k_attn_dev<<<dim3(a.hq, batch, a.n_split), 256, smem, c->s>>>(a);
  int r = launched("attention_devarg");
  if (r || a.n_split <= 1) return r;
  k_attn_combine<<<a.hq, 128, 0, c->s>>>(a.sm, a.sl, a.sv, a.out, a.n_split, a.dv);
  return launched("attention_combine");
}

int append_launch(AppendArgs a, int batch) {
  Ctx* c = ctx();
  if (!c) return -1;
  k_append_dev<<<dim3(blocks(max(a.dk, a.dv)), batch), 256, 0, c->s>>>(a);
  return launched("append_kv_devarg");
}

int rope_launch(RopeArgs a) {
  Ctx* c = ctx();
  if (!c) return -1;
  k_rope_dev<<<blocks((size_t)a.rows * a.heads * (a.rd / 2)), 256, 0, c->s>>>(a);
  return launched("rope_devarg");
}

// Paged single-sequence attention behind the reference's several entry points.
int paged_attn(int64_t q, int64_t kp, int64_t vp, int64_t pt, int64_t out, int hq, int hkv, int dk, int dv, int bs,
               float scale, int max_seq, int64_t step, int window = 0, int n_split = 1, int64_t hm = 0,
               int64_t hl = 0, int64_t hv = 0) {
  if (hq <= 0 || hkv <= 0 || dk <= 0 || dv <= 0 || bs <= 0 || max_seq <= 0 || n_split <= 0) return -1;
  AttnArgs a{};
  a.q = F(q, (size_t)hq * dk);
  a.kp = F(kp, (size_t)hkv * dk);
  a.vp = F(vp, (size_t)hkv * dv);
  a.pt = I(pt, 1);
  a.pt_stride = (int)capacity(pt, 4);
  a.out = F(out, (size_t)hq * dv);
  a.hq = hq; a.hkv = hkv; a.dk = dk; a.dv = dv; a.bs = bs; a.scale = scale; a.window = window;
  a.cur = I(step, 2);
  a.max_seq = max_seq;
  a.rows_k = capacity(kp, 4) / ((size_t)hkv * dk);
  a.rows_v = capacity(vp, 4) / ((size_t)hkv * dv);
  a.n_split = n_split;
  if (n_split > 1) {
    a.sm = F(hm, (size_t)hq * n_split);
    a.sl = F(hl, (size_t)hq * n_split);
    a.sv = F(hv, (size_t)hq * n_split * dv);
    if (!a.sm || !a.sl || !a.sv) return -1;
  }
  if (!a.q || !a.kp || !a.vp || !a.pt || !a.out || !a.cur) return -1;
  return attn_launch(a, 1);
}

int paged_append(int64_t kn, int64_t vn, int64_t kp, int64_t vp, int64_t pt, int dk, int dv, int bs, int64_t step,
                 int batch = 1, int pt_stride = 0, int per_batch = 0) {
  if (dk <= 0 || dv <= 0 || bs <= 0 || batch <= 0) return -1;
  AppendArgs a{};
  a.kn = F(kn, (size_t)batch * dk);
  a.vn = F(vn, (size_t)batch * dv);
  a.kp = F(kp, dk);
  a.vp = F(vp, dv);
  a.pt = pt ? I(pt, 1) : nullptr;
  a.pt_stride = pt ? (pt_stride ? pt_stride : (int)capacity(pt, 4)) : 0;
  if (pt && (size_t)a.pt_stride * batch > capacity(pt, 4)) return -1;
  a.bs = bs; a.dk = dk; a.dv = dv;
  a.pos = I(step, per_batch ? batch : 1);
  a.per_batch = per_batch;
  a.rows_k = capacity(kp, 4) / dk;
  a.rows_v = capacity(vp, 4) / dv;
  if (!a.kn || !a.vn || !a.kp || !a.vp || (pt && !a.pt) || !a.pos) return -1;
  return append_launch(a, batch);
}

int batched_attn(int64_t q, int64_t kp, int64_t vp, int64_t pt, int64_t out, int batch, int hq, int hkv, int hd, int bs,
                 int pt_stride, float scale, int max_seq, int64_t cur, int per_batch) {
  if (batch <= 0 || hq <= 0 || hkv <= 0 || hd <= 0 || bs <= 0 || pt_stride <= 0) return -1;
  AttnArgs a{};
  a.q = F(q, (size_t)batch * hq * hd);
  a.kp = F(kp, (size_t)hkv * hd);
  a.vp = F(vp, (size_t)hkv * hd);
  a.pt = I(pt, (size_t)batch * pt_stride);
  a.pt_stride = pt_stride;
  a.out = F(out, (size_t)batch * hq * hd);
  a.hq = hq; a.hkv = hkv; a.dk = hd; a.dv = hd; a.bs = bs; a.scale = scale;
  a.cur = I(cur, per_batch ? batch : 2);
  a.cur_per_batch = per_batch;
  a.max_seq = max_seq;
  a.rows_k = a.rows_v = capacity(kp, 4) / ((size_t)hkv * hd);
  a.q_bstride = a.o_bstride = (long long)hq * hd;
  a.n_split = 1;
  if (!a.q || !a.kp || !a.vp || !a.pt || !a.out || !a.cur || capacity(vp, 4) < capacity(kp, 4)) return -1;
  return attn_launch(a, batch);
}

// Gather / scatter helpers of the MLA step: out[i] = in[map(i)] over n elements.
__global__ void k_mla_copy(const float* a, const float* b, float* out, int n_heads, int da, int db, int mode,
                           int extra) {
  // mode 0: split kv_a [da + db] -> a-part (out) and b-part (via `extra` as offset into out2 -- unused)
  // mode 1: assemble K: out[h, :da] = a[h, :da] (row stride da + extra), out[h, da:] = b[:db]
  // mode 2: extract V:  out[h, :db] = a[h, da : da + db] (row stride da + db)
  // mode 3: broadcast:  out[h, :da] = a[:da], out[h, da:] = b[:db]
  const int per = (mode == 2) ? db : da + db;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_heads * per) return;
  const int h = i / per, j = i % per;
  float v;
  if (mode == 1) v = j < da ? a[(size_t)h * (da + extra) + j] : b[j - da];
  else if (mode == 2) v = a[(size_t)h * (da + db) + da + j];
  else v = j < da ? a[j] : b[j - da];
  out[i] = v;
}

__global__ void k_copy_rows(const float* in, float* out, int rows, int n, long long in_stride, long long in_off,
                            long long out_stride, long long out_off) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * n) return;
  const int r = i / n, j = i % n;
  out[r * out_stride + out_off + j] = in[r * in_stride + in_off + j];
}

// q8_1 activations: per 32 values, d = max|x| / 127, q = round(x / d), s = d * sum(q).
__global__ void k_quant_q8_1(const float* x, int8_t* q, float* d, float* s, int nblk) {
  const int b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int l = threadIdx.x & 31;
  if (b >= nblk) return;
  const float v = x[(size_t)b * 32 + l];
  const float amax = warp_max(fabsf(v));
  const float dd = amax / 127.f;
  const int qi = dd > 0.f ? __float2int_rn(v / dd) : 0;
  q[(size_t)b * 32 + l] = (int8_t)qi;
  const float sum = warp_sum((float)qi);
  if (l == 0) {
    d[b] = dd;
    s[b] = dd * sum;
  }
}

__global__ void k_bert_embed(const int* ids, const int* tt, const float* word, const float* pos, const float* type,
                             float* out, int seq, int d, int vocab, int n_pos, int n_type) {
  const size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= (size_t)seq * d) return;
  const int t = (int)(i / d), j = (int)(i % d);
  const int id = ids[t], ty = tt ? tt[t] : 0;
  float v = (id >= 0 && id < vocab) ? word[(size_t)id * d + j] : 0.f;
  v += t < n_pos ? pos[(size_t)t * d + j] : 0.f;
  v += (ty >= 0 && ty < n_type) ? type[(size_t)ty * d + j] : 0.f;
  out[i] = v;
}

// Rotate-half 2-D RoPE of the patch tokens (after n_prefix tokens) with
// per-patch cos / sin tables [n_patches, head_dim].
__global__ void k_rope2d_tables(float* buf, const float* cs, const float* sn, int n_prefix, int heads, int hd,
                                int n_patches) {
  const int half = hd / 2;
  const size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= (size_t)n_patches * heads * half) return;
  const int j = (int)(i % half);
  const size_t ph = i / half;
  const int h = (int)(ph % heads), p = (int)(ph / heads);
  float* v = buf + ((size_t)(n_prefix + p) * heads + h) * hd;
  const float* c = cs + (size_t)p * hd;
  const float* s = sn + (size_t)p * hd;
  const float x0 = v[j], x1 = v[j + half];
  v[j] = x0 * c[j] - x1 * s[j];
  v[j + half] = x1 * c[j + half] + x0 * s[j + half];
}

// Per-head absorbed-MLA mat-vecs: `heads` groups of `rows` weight rows of `k`
// values; group h reads x + h * xg and writes y + h * yg.
int absorb(int t, int64_t xh, int64_t wh, int64_t yh, int heads, int rows, int k, long long xg, long long yg,
           size_t x_need, size_t y_need) {
  int ne, nb;
  if (!block_of(t, &ne, &nb) || heads <= 0 || rows <= 0 || k <= 0 || k % 32 || k % ne || xg % 4) return -1;
  const size_t row_bytes = (size_t)(k / ne) * nb;
  const float* x = F(xh, x_need);
  const uint8_t* w = U(wh, row_bytes * rows * heads);
  float* y = F(yh, y_need);
  if (!x || !w || !y) return -1;
  MV p{x, w, y, nullptr, heads * rows, k / 32, row_bytes, rows, xg, yg, 0, 0, nullptr, nullptr};
  return matvec_typed(t, p, 1);
}

int absorb_q(int t, int64_t q, int64_t w, int64_t out, int heads, int key_mla, int qk_rope, int lora, int k_nope) {
  const int q_nope = key_mla - qk_rope;
  if (heads <= 0 || qk_rope < 0 || lora <= 0 || q_nope <= 0 || k_nope != q_nope) return -1;
  const int per = lora + qk_rope;
  int r = absorb(t, q, w, out, heads, lora, q_nope, key_mla, per, (size_t)heads * key_mla, (size_t)heads * per);
  if (r || qk_rope == 0) return r;
  // q_pe rides along: out[h, lora:] = q[h, q_nope:]
  Ctx* c = ctx();
  k_copy_rows<<<blocks((size_t)heads * qk_rope), 256, 0, c->s>>>(F(q, (size_t)heads * key_mla), F(out, (size_t)heads * per),
                                                                  heads, qk_rope, key_mla, q_nope, per, lora);
  return launched("mla_absorb_q");
}

int absorb_v(int t, int64_t av, int64_t w, int64_t out, int heads, int lora, int vdim, int k) {
  if (heads <= 0 || lora <= 0 || vdim <= 0 || k != lora) return -1;
  return absorb(t, av, w, out, heads, vdim, lora, lora, vdim, (size_t)heads * lora, (size_t)heads * vdim);
}

int elements_per_row(int t, int blocks_per_row) {
  int ne, nb;
  return block_of(t, &ne, &nb) ? blocks_per_row * ne : -1;
}

}  // namespace

AE_API int aether_op_rope_apply_devarg_f32_cuda(int64_t x, int seq, int heads, int hd, float base, int64_t step) {
  if (seq <= 0 || heads <= 0 || hd <= 0 || hd % 2) return -1;
  RopeArgs a{F(x, (size_t)seq * heads * hd), seq, heads, hd, 0, hd, base, I(step, 1), 0, 1.f, 1.f, 1.f, 1.f};
  return (!a.x || !a.pos) ? -1 : rope_launch(a);
}
// x [batch, heads, hd], row b at pos_batch[b]
AE_API int aether_op_batched_rope_apply_devarg_f32_cuda(int64_t x, int batch, int heads, int hd, float base,
                                                        int64_t pos_batch) {
  if (batch <= 0 || heads <= 0 || hd <= 0 || hd % 2) return -1;
  RopeArgs a{F(x, (size_t)batch * heads * hd), batch, heads, hd, 0, hd, base, I(pos_batch, batch), 1, 1.f, 1.f, 1.f,
             1.f};
  return (!a.x || !a.pos) ? -1 : rope_launch(a);
}
AE_API int aether_op_qkv_bias_rope_devarg_f32_cuda(int64_t q, int64_t k, int64_t v, int64_t bq, int64_t bk, int64_t bv,
                                                   int hq, int hkv, int hd, float base, int64_t step) {
  if (hq <= 0 || hkv <= 0 || hd <= 0 || hd % 2) return -1;
  float *pq = F(q, (size_t)hq * hd), *pk = F(k, (size_t)hkv * hd), *pv = F(v, (size_t)hkv * hd);
  const float *bq_ = F(bq, (size_t)hq * hd), *bk_ = F(bk, (size_t)hkv * hd), *bv_ = F(bv, (size_t)hkv * hd);
  const int* st = I(step, 1);
  if (!pq || !pk || !pv || !bq_ || !bk_ || !bv_ || !st) return -1;
  const int n = hq * (hd / 2) + hkv * (hd / 2) + hkv * hd;
  EW_LAUNCH(k_qkv_bias_rope, n, pq, pk, pv, bq_, bk_, bv_, hq, hkv, hd, base, st);
}
AE_API int aether_op_append_kv_devarg_f32_cuda(int64_t kn, int64_t vn, int64_t kc, int64_t vc, int dkv, int64_t step) {
  return paged_append(kn, vn, kc, vc, 0, dkv, dkv, 1, step);
}
AE_API int aether_op_attention_seq1_devarg_f32_cuda(int64_t q, int64_t kc, int64_t vc, int64_t out, int hq, int hkv,
                                                    int hd, float scale, int max_seq, int64_t step) {
  if (hq <= 0 || hkv <= 0 || hd <= 0) return -1;
  AttnArgs a{};
  a.q = F(q, (size_t)hq * hd);
  a.kp = F(kc, (size_t)hkv * hd);
  a.vp = F(vc, (size_t)hkv * hd);
  a.out = F(out, (size_t)hq * hd);
  a.hq = hq; a.hkv = hkv; a.dk = hd; a.dv = hd; a.bs = 1; a.scale = scale;
  a.cur = I(step, 2);
  a.max_seq = max_seq;
  a.rows_k = capacity(kc, 4) / ((size_t)hkv * hd);
  a.rows_v = capacity(vc, 4) / ((size_t)hkv * hd);
  a.n_split = 1;
  if (!a.q || !a.kp || !a.vp || !a.out || !a.cur) return -1;
  return attn_launch(a, 1);
}
AE_API int aether_op_paged_append_kv_devarg_f32_cuda(int64_t kn, int64_t vn, int64_t kp, int64_t vp, int64_t pt, int dkv,
                                                     int bs, int64_t step) {
  return pt ? paged_append(kn, vn, kp, vp, pt, dkv, dkv, bs, step) : -1;
}
AE_API int aether_op_paged_append_kv_mla_devarg_f32_cuda(int64_t kn, int64_t vn, int64_t kp, int64_t vp, int64_t pt,
                                                         int dk, int dv, int bs, int64_t step) {
  return pt ? paged_append(kn, vn, kp, vp, pt, dk, dv, bs, step) : -1;
}
AE_API int aether_op_paged_attention_seq1_devarg_f32_cuda(int64_t q, int64_t kp, int64_t vp, int64_t pt, int64_t out,
                                                          int hq, int hkv, int hd, int bs, float scale, int max_seq,
                                                          int64_t step) {
  return paged_attn(q, kp, vp, pt, out, hq, hkv, hd, hd, bs, scale, max_seq, step);
}
// The reference's successive versions of the paged kernel share one interface and one kernel here.
AE_API int aether_op_paged_attention_seq1_v2_devarg_f32_cuda(int64_t q, int64_t kp, int64_t vp, int64_t pt, int64_t out,
                                                             int hq, int hkv, int hd, int bs, float scale, int max_seq,
                                                             int64_t step) {
  return paged_attn(q, kp, vp, pt, out, hq, hkv, hd, hd, bs, scale, max_seq, step);
}
AE_API int aether_op_paged_attention_seq1_v3_devarg_f32_cuda(int64_t q, int64_t kp, int64_t vp, int64_t pt, int64_t out,
                                                             int hq, int hkv, int hd, int bs, float scale, int max_seq,
                                                             int64_t step) {
  return paged_attn(q, kp, vp, pt, out, hq, hkv, hd, hd, bs, scale, max_seq, step);
}
// Split-K over the keys: partials (m, l, v) in caller scratch of hq * n_split * (2 + hd) floats.
AE_API int aether_op_paged_attention_seq1_v4_devarg_f32_cuda(int64_t q, int64_t kp, int64_t vp, int64_t pt, int64_t out,
                                                             int64_t sm, int64_t sl, int64_t sv, int hq, int hkv, int hd,
                                                             int bs, float scale, int max_seq, int n_split,
                                                             int64_t step) {
  if (n_split <= 0 || n_split > 256) return -1;
  return paged_attn(q, kp, vp, pt, out, hq, hkv, hd, hd, bs, scale, max_seq, step, 0, n_split, sm, sl, sv);
}
// Any head_dim; sliding_window > 0 keeps only the last sliding_window positions.
AE_API int aether_op_paged_attention_flex_devarg_f32_cuda(int64_t q, int64_t kp, int64_t vp, int64_t pt, int64_t out,
                                                          int hq, int hkv, int hd, int bs, int window, float scale,
                                                          int max_seq, int64_t step) {
  return paged_attn(q, kp, vp, pt, out, hq, hkv, hd, hd, bs, scale, max_seq, step, window);
}
// Per-head K of qk_head_dim and V of v_head_dim (non-absorbed MLA).
AE_API int aether_op_paged_attention_mla_devarg_f32_cuda(int64_t q, int64_t kp, int64_t vp, int64_t pt, int64_t out,
                                                         int heads, int qk_hd, int v_hd, int bs, float scale,
                                                         int max_seq, int64_t step) {
  return paged_attn(q, kp, vp, pt, out, heads, heads, qk_hd, v_hd, bs, scale, max_seq, step);
}
// B sequences at one shared position step_args[0] (seqB) or their own pos_batch[b] (hetero).
AE_API int aether_op_batched_paged_append_kv_seqB_devarg_f32_cuda(int64_t kn, int64_t vn, int64_t kp, int64_t vp,
                                                                  int64_t pt, int batch, int dkv, int bs, int pt_stride,
                                                                  int64_t step) {
  return (pt && pt_stride > 0) ? paged_append(kn, vn, kp, vp, pt, dkv, dkv, bs, step, batch, pt_stride, 0) : -1;
}
AE_API int aether_op_batched_paged_append_kv_hetero_devarg_f32_cuda(int64_t kn, int64_t vn, int64_t kp, int64_t vp,
                                                                    int64_t pt, int batch, int dkv, int bs,
                                                                    int pt_stride, int64_t pos_batch) {
  return (pt && pt_stride > 0) ? paged_append(kn, vn, kp, vp, pt, dkv, dkv, bs, pos_batch, batch, pt_stride, 1) : -1;
}
AE_API int aether_op_batched_paged_attention_seqB_devarg_f32_cuda(int64_t q, int64_t kp, int64_t vp, int64_t pt,
                                                                  int64_t out, int batch, int hq, int hkv, int hd, int bs,
                                                                  int pt_stride, float scale, int max_seq,
                                                                  int64_t step) {
  return batched_attn(q, kp, vp, pt, out, batch, hq, hkv, hd, bs, pt_stride, scale, max_seq, step, 0);
}
AE_API int aether_op_batched_paged_attention_hetero_devarg_f32_cuda(int64_t q, int64_t kp, int64_t vp, int64_t pt,
                                                                    int64_t out, int batch, int hq, int hkv, int hd,
                                                                    int bs, int pt_stride, float scale, int max_seq,
                                                                    int64_t cur_batch) {
  return batched_attn(q, kp, vp, pt, out, batch, hq, hkv, hd, bs, pt_stride, scale, max_seq, cur_batch, 1);
}

// ------------------------------------------------------------------------------------------------ encoders
// Bidirectional attention over [seq, heads, hd] (every query sees every key).
AE_API int aether_op_bert_self_attention_fwd_f32_cuda(int64_t q, int64_t k, int64_t v, int64_t out, int seq, int heads,
                                                      int hd, float scale) {
  if (seq <= 0 || heads <= 0 || hd <= 0) return -1;
  const size_t n = (size_t)seq * heads * hd;
  AttnArgs a{};
  a.q = F(q, n);
  a.kp = F(k, n);
  a.vp = F(v, n);
  a.out = F(out, n);
  a.hq = a.hkv = heads; a.dk = a.dv = hd; a.bs = 1; a.scale = scale;
  a.cur_const = seq;
  a.max_seq = seq;
  a.rows_k = a.rows_v = seq;
  a.q_bstride = a.o_bstride = (long long)heads * hd;
  a.n_split = 1;
  if (!a.q || !a.kp || !a.vp || !a.out) return -1;
  return attn_launch(a, seq);
}
// out[t] = word[ids[t]] + pos[t] + type[token_type[t]] (type handle 0: type 0)
AE_API int aether_op_bert_embed_sum_f32_cuda(int64_t ids, int64_t tt, int64_t word, int64_t pos, int64_t type,
                                             int64_t out, int seq, int d) {
  if (seq <= 0 || d <= 0) return -1;
  const int* pi = I(ids, seq);
  const int* pt = tt ? I(tt, seq) : nullptr;
  const int vocab = (int)(capacity(word, 4) / d), n_pos = (int)(capacity(pos, 4) / d),
            n_type = (int)(capacity(type, 4) / d);
  const float *pw = F(word, (size_t)vocab * d), *pp = F(pos, (size_t)n_pos * d), *py = F(type, (size_t)n_type * d);
  float* po = F(out, (size_t)seq * d);
  if (!pi || (tt && !pt) || !pw || !pp || !py || !po || vocab <= 0 || n_type <= 0) return -1;
  EW_LAUNCH(k_bert_embed, (size_t)seq * d, pi, pt, pw, pp, py, po, seq, d, vocab, n_pos, n_type);
}
// DINOv3 axial RoPE on the patch tokens of buf [seq, heads, hd] with tables [n_patches, hd].
AE_API int aether_op_dinov3_rope2d_f32_cuda(int64_t buf, int64_t cosb, int64_t sinb, int seq, int n_prefix, int heads,
                                            int hd, int n_patches) {
  if (seq <= 0 || n_prefix < 0 || heads <= 0 || hd <= 0 || hd % 2 || n_patches < 0 || n_prefix + n_patches > seq)
    return -1;
  float* pb = F(buf, (size_t)seq * heads * hd);
  const float *pc = F(cosb, (size_t)n_patches * hd), *ps = F(sinb, (size_t)n_patches * hd);
  if (!pb || (n_patches && (!pc || !ps))) return -1;
  if (!n_patches) return 0;
  EW_LAUNCH(k_rope2d_tables, (size_t)n_patches * heads * (hd / 2), pb, pc, ps, n_prefix, heads, hd, n_patches);
}

// ------------------------------------------------------------------------------------------------ MLA
// kv_a [lora + rope] -> c_kv [lora], k_rope [rope]
AE_API int aether_op_mla_split_kv_a_f32_cuda(int64_t kv_a, int64_t c_kv, int64_t k_rope, int lora, int rope) {
  if (lora <= 0 || rope < 0) return -1;
  const float* pa = F(kv_a, (size_t)lora + rope);
  float *pc = F(c_kv, lora), *pr = rope ? F(k_rope, rope) : nullptr;
  Ctx* c = ctx();
  if (!pa || !pc || (rope && !pr) || !c) return -1;
  k_copy_rows<<<blocks(lora), 256, 0, c->s>>>(pa, pc, 1, lora, 0, 0, 0, 0);
  if (rope) k_copy_rows<<<blocks(rope), 256, 0, c->s>>>(pa, pr, 1, rope, 0, lora, 0, 0);
  return launched("mla_split_kv_a");
}
// k_row[h] = [kv_b_out[h, :nope] | k_rope]  (kv_b_out rows of nope + v_hd)
AE_API int aether_op_mla_assemble_k_f32_cuda(int64_t kv_b, int64_t k_rope, int64_t k_row, int heads, int nope, int rope,
                                             int v_hd) {
  if (heads <= 0 || nope <= 0 || rope < 0 || v_hd < 0) return -1;
  const float *pb = F(kv_b, (size_t)heads * (nope + v_hd)), *pr = F(k_rope, rope ? rope : 1);
  float* po = F(k_row, (size_t)heads * (nope + rope));
  if (!pb || !pr || !po) return -1;
  EW_LAUNCH(k_mla_copy, (size_t)heads * (nope + rope), pb, pr, po, heads, nope, rope, 1, v_hd);
}
// v_row[h] = kv_b_out[h, nope : nope + v_hd]
AE_API int aether_op_mla_extract_v_f32_cuda(int64_t kv_b, int64_t v_row, int heads, int nope, int v_hd) {
  if (heads <= 0 || nope < 0 || v_hd <= 0) return -1;
  const float* pb = F(kv_b, (size_t)heads * (nope + v_hd));
  float* po = F(v_row, (size_t)heads * v_hd);
  if (!pb || !po) return -1;
  EW_LAUNCH(k_mla_copy, (size_t)heads * v_hd, pb, nullptr, po, heads, nope, v_hd, 2, 0);
}
// k_row[h] = [c_kv | k_pe], v_row[h] = c_kv for every head (MQA view of the latent)
AE_API int aether_op_mla_broadcast_kv_for_mqa_f32_cuda(int64_t c_kv, int64_t k_pe, int64_t k_row, int64_t v_row,
                                                       int heads, int lora, int rope) {
  if (heads <= 0 || lora <= 0 || rope < 0) return -1;
  const float *pc = F(c_kv, lora), *pp = F(k_pe, rope ? rope : 1);
  float *pk = F(k_row, (size_t)heads * (lora + rope)), *pv = F(v_row, (size_t)heads * lora);
  Ctx* c = ctx();
  if (!pc || !pp || !pk || !pv || !c) return -1;
  k_mla_copy<<<blocks((size_t)heads * (lora + rope)), 256, 0, c->s>>>(pc, pp, pk, heads, lora, rope, 3, 0);
  k_mla_copy<<<blocks((size_t)heads * lora), 256, 0, c->s>>>(pc, pp, pv, heads, lora, 0, 3, 0);
  return launched("mla_broadcast_kv");
}
// RoPE on the last (qk_hd - nope) dims of each head of q, at step_args[0].
AE_API int aether_op_mla_rope_q_partial_f32_cuda(int64_t q, int heads, int qk_hd, int nope, float base, int64_t step) {
  const int rd = qk_hd - nope;
  if (heads <= 0 || nope < 0 || rd <= 0 || rd % 2) return -1;
  RopeArgs a{F(q, (size_t)heads * qk_hd), 1, heads, qk_hd, nope, rd, base, I(step, 1), 0, 1.f, 1.f, 1.f, 1.f};
  return (!a.x || !a.pos) ? -1 : rope_launch(a);
}
AE_API int aether_op_mla_rope_k_shared_f32_cuda(int64_t k_rope, int rd, float base, int64_t step) {
  if (rd <= 0 || rd % 2) return -1;
  RopeArgs a{F(k_rope, rd), 1, 1, rd, 0, rd, base, I(step, 1), 0, 1.f, 1.f, 1.f, 1.f};
  return (!a.x || !a.pos) ? -1 : rope_launch(a);
}
AE_API int aether_op_mla_rope_q_partial_yarn_f32_cuda(int64_t q, int heads, int qk_hd, int nope, float base, float ys,
                                                      float yctx, float yfast, float yslow, int64_t step) {
  const int rd = qk_hd - nope;
  if (heads <= 0 || nope < 0 || rd <= 0 || rd % 2) return -1;
  RopeArgs a{F(q, (size_t)heads * qk_hd), 1, heads, qk_hd, nope, rd, base, I(step, 1), 0, ys, yctx, yfast, yslow};
  return (!a.x || !a.pos) ? -1 : rope_launch(a);
}
AE_API int aether_op_mla_rope_k_shared_yarn_f32_cuda(int64_t k_rope, int rd, float base, float ys, float yctx,
                                                     float yfast, float yslow, int64_t step) {
  if (rd <= 0 || rd % 2) return -1;
  RopeArgs a{F(k_rope, rd), 1, 1, rd, 0, rd, base, I(step, 1), 0, ys, yctx, yfast, yslow};
  return (!a.x || !a.pos) ? -1 : rope_launch(a);
}
// Absorbed MLA: q_out[h] = [W_kb[h] q_nope[h] | q_pe[h]] and attn_out[h] = W_vb[h] attn_v[h],
// per-head weights in GGUF blocks (rows of q_nope resp. kv_lora values).
#define MLA_ABSORB(name, T)                                                                                        \
  AE_API int aether_op_mla_absorb_q_##name##_cuda(int64_t q, int64_t w, int64_t out, int heads, int key_mla,         \
                                                  int qk_rope, int lora, int bpr) {                                 \
    return absorb_q(T, q, w, out, heads, key_mla, qk_rope, lora, elements_per_row(T, bpr));                         \
  }                                                                                                                 \
  AE_API int aether_op_mla_absorb_v_##name##_cuda(int64_t av, int64_t w, int64_t out, int heads, int lora, int vdim, \
                                                  int bpr) {                                                        \
    return absorb_v(T, av, w, out, heads, lora, vdim, elements_per_row(T, bpr));                                     \
  }
MLA_ABSORB(q8_0, TQ8_0)
MLA_ABSORB(q4_k, TQ4_K)
MLA_ABSORB(q5_k, TQ5_K)
MLA_ABSORB(q6_k, TQ6_K)
MLA_ABSORB(iq4_nl, TIQ4_NL)
MLA_ABSORB(f16, TF16)  // F16: the last argument counts elements per row (block of one)

// ------------------------------------------------------------------------------------------------ q8_1 activations
// x [n_in] -> int8 values, per-32 scales d and d * sum(q) (n_in a multiple of 32).
AE_API int aether_op_quantize_q8_1_llama_cuda(int64_t x, int64_t aq, int64_t ad, int64_t as, int n_in) {
  if (n_in <= 0 || n_in % 32) return -1;
  const int nblk = n_in / 32;
  const float* px = F(x, n_in);
  int8_t* pq = (int8_t*)U(aq, n_in);
  float *pd = F(ad, nblk), *ps = F(as, nblk);
  Ctx* c = ctx();
  if (!px || !pq || !pd || !ps || !c) return -1;
  k_quant_q8_1<<<blocks(nblk, 8), 256, 0, c->s>>>(px, pq, pd, ps, nblk);
  return launched("quantize_q8_1");
}
namespace {
int mmvq(int t, int64_t w, int64_t w2, int64_t aq, int64_t ad, int64_t out, int n_out, int bpr) {
  int ne, nb;
  if (!block_of(t, &ne, &nb) || n_out <= 0 || bpr <= 0) return -1;
  const size_t k = (size_t)bpr * ne, row_bytes = (size_t)bpr * nb;
  const uint8_t* pw = U(w, row_bytes * n_out);
  const uint8_t* pw2 = w2 ? U(w2, row_bytes * n_out) : nullptr;
  const int8_t* pq = (const int8_t*)U(aq, k);
  const float* pd = F(ad, k / 32);
  float* po = F(out, n_out);
  if (!pw || (w2 && !pw2) || !pq || !pd || !po) return -1;
  MV p{nullptr, pw, po, pw2, n_out, (int)(k / 32), row_bytes, n_out, 0, 0, 0, 0, pq, pd};
  return matvec_typed(t, p, 1);
}
}  // namespace
// out = W x for x given as q8_1 (quantize_q8_1_llama output); swiglu: silu(W_gate x) * (W_up x)
AE_API int aether_op_mmvq_q4k_q8_1_single_cuda(int64_t w, int64_t aq, int64_t ad, int64_t out, int n_out, int bpr) {
  return mmvq(TQ4_K, w, 0, aq, ad, out, n_out, bpr);
}
AE_API int aether_op_mmvq_q6k_q8_1_single_cuda(int64_t w, int64_t aq, int64_t ad, int64_t out, int n_out, int bpr) {
  return mmvq(TQ6_K, w, 0, aq, ad, out, n_out, bpr);
}
AE_API int aether_op_mmvq_q4k_q8_1_swiglu_cuda(int64_t wg, int64_t wu, int64_t aq, int64_t ad, int64_t out, int n_out,
                                               int bpr) {
  return mmvq(TQ4_K, wg, wu, aq, ad, out, n_out, bpr);
}
// `batch` activation rows against one quantised weight: out [batch, n]
AE_API int aether_op_fused_q4k_matmul_seqB_v3_cuda(int64_t a, int64_t w, int64_t o, int n, int nb, int batch) {
  return qmatvec(TQ4_K, a, w, o, n, nb, 0, 0, batch);
}
AE_API int aether_op_fused_q4k_matmul_seqB_fp16_cuda(int64_t a, int64_t w, int64_t o, int n, int nb, int batch) {
  return qmatvec(TQ4_K, a, w, o, n, nb, 0, 0, batch);
}
AE_API int aether_op_fused_q6k_matmul_seqB_v3_cuda(int64_t a, int64_t w, int64_t o, int n, int nb, int batch) {
  return qmatvec(TQ6_K, a, w, o, n, nb, 0, 0, batch);
}
AE_API int aether_op_fused_q6k_matmul_seqB_fp16_cuda(int64_t a, int64_t w, int64_t o, int n, int nb, int batch) {
  return qmatvec(TQ6_K, a, w, o, n, nb, 0, 0, batch);
}
// A Q4_K mat-vec kept under the reference's bandwidth-probe name.
AE_API int aether_op_fused_q4k_membw_probe_cuda(int64_t a, int64_t w, int64_t o, int n, int nb) {
  return qmatvec(TQ4_K, a, w, o, n, nb);
}

// ================================================================================================ tiny-LM benches
// Iterations per second of a pre-LayerNorm decoder block stack (LN -> Q/K/V ->
// causal attention -> O + residual -> LN -> up -> SiLU -> down + residual) over
// seq_len tokens in fp32, the weights drawn from the same fixed-seed SplitMix64
// stream as the host library's CPU bench. -1 when no GPU is present.
//   _cuda: every matmul is one round trip through the device (weights and
//          activations uploaded, result downloaded, buffers allocated and
//          freed per call); the other ops run on the host.
//   _cuda_resident: weights uploaded once and every op on the device; one
//          iteration is captured in a CUDA graph and replayed (eager launches
//          when capture is not possible).
namespace {
struct TinyLM {
  int d, f, s, layers;
  std::vector<float> w, x;  // per layer: wq, wk, wv, wo (d x d), up (d x f), down (f x d)
  TinyLM(int d_, int l_, int f_, int s_) : d(d_), f(f_), s(s_), layers(l_) {
    uint64_t st = 0x2545F4914F6CDD1DULL;
    auto rnd = [&]() {
      st += 0x9E3779B97F4A7C15ULL;
      uint64_t z = st;
      z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
      z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
      z ^= z >> 31;
      return ((float)(z >> 40) / (float)(1 << 24) - 0.5f) * 0.02f;
    };
    w.resize(per_layer() * layers);
    for (auto& e : w) e = rnd();
    x.resize((size_t)s * d);
    for (auto& e : x) e = rnd();
  }
  size_t per_layer() const { return 4 * (size_t)d * d + 2 * (size_t)d * f; }
  const float* W(int l, int i) const {  // i: 0..3 = q,k,v,o; 4 = up; 5 = down
    const float* b = w.data() + per_layer() * l;
    return i < 4 ? b + (size_t)i * d * d : b + 4 * (size_t)d * d + (size_t)(i - 4) * d * f;
  }
};

void host_ln(const float* x, float* y, int s, int d) {
  for (int r = 0; r < s; ++r) {
    double m = 0, v = 0;
    for (int j = 0; j < d; ++j) m += x[(size_t)r * d + j];
    m /= d;
    for (int j = 0; j < d; ++j) v += (x[(size_t)r * d + j] - m) * (x[(size_t)r * d + j] - m);
    const float rs = (float)(1.0 / std::sqrt(v / d + 1e-5));
    for (int j = 0; j < d; ++j) y[(size_t)r * d + j] = (float)(x[(size_t)r * d + j] - m) * rs;
  }
}
void host_attn(const float* q, const float* k, const float* v, float* o, int s, int d) {
  std::vector<float> p(s);
  const float sc = 1.f / std::sqrt((float)d);
  for (int i = 0; i < s; ++i) {
    float m = -INFINITY, sum = 0.f;
    for (int j = 0; j <= i; ++j) {
      float a = 0.f;
      for (int t = 0; t < d; ++t) a += q[(size_t)i * d + t] * k[(size_t)j * d + t];
      p[j] = a * sc;
      m = std::max(m, p[j]);
    }
    for (int j = 0; j <= i; ++j) sum += (p[j] = std::exp(p[j] - m));
    for (int t = 0; t < d; ++t) {
      float a = 0.f;
      for (int j = 0; j <= i; ++j) a += p[j] * v[(size_t)j * d + t];
      o[(size_t)i * d + t] = a / sum;
    }
  }
}
// One matmul as a self-contained device round trip.
bool routed_matmul(Ctx* c, const float* a, const float* b, float* out, int m, int k, int n) {
  float *da = nullptr, *db = nullptr, *dc = nullptr;
  if (cudaMallocAsync(&da, (size_t)m * k * 4, c->s) || cudaMallocAsync(&db, (size_t)k * n * 4, c->s) ||
      cudaMallocAsync(&dc, (size_t)m * n * 4, c->s))
    return false;
  cudaMemcpyAsync(da, a, (size_t)m * k * 4, cudaMemcpyHostToDevice, c->s);
  cudaMemcpyAsync(db, b, (size_t)k * n * 4, cudaMemcpyHostToDevice, c->s);
  const int r = gemm_rm(false, false, m, n, k, 1.f, da, k, db, n, 0.f, dc, n);
  cudaMemcpyAsync(out, dc, (size_t)m * n * 4, cudaMemcpyDeviceToHost, c->s);
  cudaFreeAsync(da, c->s);
  cudaFreeAsync(db, c->s);
  cudaFreeAsync(dc, c->s);
  return r == 0 && cudaStreamSynchronize(c->s) == cudaSuccess;
}
}  // namespace

AE_API float aether_llm_inference_bench_tps_cuda(int iters, int d_model, int n_layers, int ff, int seq_len) {
  if (iters <= 0 || d_model <= 0 || n_layers <= 0 || ff <= 0 || seq_len <= 0) return 0.f;
  Ctx* c = ctx();
  if (!c) return -1.f;
  TinyLM m(d_model, n_layers, ff, seq_len);
  const int s = seq_len, d = d_model, f = ff;
  std::vector<float> x = m.x, h((size_t)s * d), q(h), k(h), v(h), o(h), proj(h), up((size_t)s * f);
  const auto t0 = std::chrono::steady_clock::now();
  for (int it = 0; it < iters; ++it)
    for (int l = 0; l < n_layers; ++l) {
      host_ln(x.data(), h.data(), s, d);
      if (!routed_matmul(c, h.data(), m.W(l, 0), q.data(), s, d, d) ||
          !routed_matmul(c, h.data(), m.W(l, 1), k.data(), s, d, d) ||
          !routed_matmul(c, h.data(), m.W(l, 2), v.data(), s, d, d))
        return 0.f;
      host_attn(q.data(), k.data(), v.data(), o.data(), s, d);
      if (!routed_matmul(c, o.data(), m.W(l, 3), proj.data(), s, d, d)) return 0.f;
      for (size_t i = 0; i < x.size(); ++i) x[i] += proj[i];
      host_ln(x.data(), h.data(), s, d);
      if (!routed_matmul(c, h.data(), m.W(l, 4), up.data(), s, d, f)) return 0.f;
      for (auto& e : up) e = e / (1.f + std::exp(-e));
      if (!routed_matmul(c, up.data(), m.W(l, 5), proj.data(), s, f, d)) return 0.f;
      for (size_t i = 0; i < x.size(); ++i) x[i] += proj[i];
    }
  const double sec = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  return sec > 0 ? (float)(iters / sec) : 0.f;
}

AE_API float aether_llm_inference_bench_tps_cuda_resident(int iters, int d_model, int n_layers, int ff,
                                                          int seq_len) {
  if (iters <= 0 || d_model <= 0 || n_layers <= 0 || ff <= 0 || seq_len <= 0) return 0.f;
  Ctx* c = ctx();
  if (!c) return -1.f;
  TinyLM m(d_model, n_layers, ff, seq_len);
  const int s = seq_len, d = d_model, f = ff;
  const size_t sd = (size_t)s * d;
  float* buf = nullptr;  // weights | x | h | q | k | v | o | proj | up | att | mean | rstd | ones | zeros
  const size_t n_w = m.w.size(), total = n_w + 7 * sd + (size_t)s * f + (size_t)s * s + 2 * (size_t)s + 2 * (size_t)d;
  if (cudaMallocAsync(&buf, total * 4, c->s) != cudaSuccess) return 0.f;
  float* W = buf;
  float *x = W + n_w, *h = x + sd, *q = h + sd, *k = q + sd, *v = k + sd, *o = v + sd, *proj = o + sd;
  float *up = proj + sd, *att = up + (size_t)s * f, *mean = att + (size_t)s * s, *rstd = mean + s, *ones = rstd + s;
  float* zeros = ones + d;
  cudaMemcpyAsync(W, m.w.data(), n_w * 4, cudaMemcpyHostToDevice, c->s);
  cudaMemcpyAsync(x, m.x.data(), sd * 4, cudaMemcpyHostToDevice, c->s);
  std::vector<float> one(d, 1.f);
  cudaMemcpyAsync(ones, one.data(), (size_t)d * 4, cudaMemcpyHostToDevice, c->s);
  cudaMemsetAsync(zeros, 0, (size_t)d * 4, c->s);
  cudaStreamSynchronize(c->s);
  const float scale = 1.f / std::sqrt((float)d);
  auto layer_w = [&](int l, int i) { return W + (m.W(l, i) - m.w.data()); };
  auto iteration = [&]() {
    for (int l = 0; l < n_layers; ++l) {
      k_layernorm<<<s, kRowThreads, 0, c->s>>>(x, nullptr, ones, zeros, h, mean, rstd, 1e-5f, d);
      gemm_rm(false, false, s, d, d, 1.f, h, d, layer_w(l, 0), d, 0.f, q, d);
      gemm_rm(false, false, s, d, d, 1.f, h, d, layer_w(l, 1), d, 0.f, k, d);
      gemm_rm(false, false, s, d, d, 1.f, h, d, layer_w(l, 2), d, 0.f, v, d);
      gemm_rm(false, true, s, s, d, scale, q, d, k, d, 0.f, att, s);
      k_causal_softmax<<<s, kRowThreads, 0, c->s>>>(att, s);
      gemm_rm(false, false, s, d, s, 1.f, att, s, v, d, 0.f, o, d);
      gemm_rm(false, false, s, d, d, 1.f, o, d, layer_w(l, 3), d, 1.f, x, d);  // residual in the GEMM (beta 1)
      k_layernorm<<<s, kRowThreads, 0, c->s>>>(x, nullptr, ones, zeros, h, mean, rstd, 1e-5f, d);
      gemm_rm(false, false, s, f, d, 1.f, h, d, layer_w(l, 4), f, 0.f, up, f);
      k_silu<<<blocks((size_t)s * f), 256, 0, c->s>>>(up, (size_t)s * f);
      gemm_rm(false, false, s, d, f, 1.f, up, f, layer_w(l, 5), d, 1.f, x, d);
    }
  };
  iteration();  // one eager pass first: cuBLAS sets up its workspace outside the capture
  cudaStreamSynchronize(c->s);
  // capture one iteration; replay it
  cudaGraph_t g = nullptr;
  cudaGraphExec_t ge = nullptr;
  if (cudaStreamBeginCapture(c->s, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
    iteration();
    if (cudaStreamEndCapture(c->s, &g) != cudaSuccess || !g || cudaGraphInstantiate(&ge, g, 0) != cudaSuccess)
      ge = nullptr;
  }
  cudaGetLastError();  // a failed capture falls back to eager launches
  auto run = [&]() {
    if (ge) cudaGraphLaunch(ge, c->s);
    else iteration();
  };
  for (int i = 0; i < 3; ++i) run();  // warm-up
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  cudaEventRecord(e0, c->s);
  for (int i = 0; i < iters; ++i) run();
  cudaEventRecord(e1, c->s);
  const bool ok = cudaEventSynchronize(e1) == cudaSuccess;
  float ms = 0.f;
  cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (ge) cudaGraphExecDestroy(ge);
  if (g) cudaGraphDestroy(g);
  cudaFreeAsync(buf, c->s);
  cudaStreamSynchronize(c->s);
  return (ok && ms > 0.f) ? (float)(iters / (ms * 1e-3)) : 0.f;
}
