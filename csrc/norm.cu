// Row-wise normalisation kernels: RMSNorm (optionally fused with the residual
// add), LayerNorm and softmax, forward and backward, bf16 in/out with fp32
// statistics.
//
// Reference semantics: rms_norm_fwd / fused_add_rmsnorm / rms_norm_bwd_dx /
// rms_norm_bwd_gamma (runtime/src/cuda.rs:2900-2990, 6944-6985),
// layer_norm_fwd / add_layer_norm_fwd / layer_norm_bwd_dx / _params
// (cuda.rs:2781-2900, 6874-6923) and softmax_f32 / softmax_bwd
// (cuda.rs:2678, 6693-6735). The reference runs one thread per row for the
// parameter gradients and a 3-pass softmax; here one warp owns a row, every
// row is held in registers as packed bf16 (16-byte vector loads), and the
// parameter gradients are reduced in two stages (per-CTA partials accumulated
// in shared memory, then one column reduction) so no global atomics are used.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "host_utils.h"

namespace aether {
namespace {

constexpr int kWarps = 8;  // rows in flight per CTA

// A row is held as packed bf16 (VPT x 16 bytes per lane, lane-strided chunks
// of 8 elements), so even a 4096-wide row costs only 64 registers.
template <int VPT>
__device__ __forceinline__ void load_raw(const __nv_bfloat16* src, int d, int lane, uint4 (&r)[VPT]) {
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (i * 32 + lane) * 8;
    r[i] = (c < d) ? *reinterpret_cast<const uint4*>(src + c) : make_uint4(0, 0, 0, 0);
  }
}

__device__ __forceinline__ void unpack8(const uint4& u, float (&v)[8]) {
  v[0] = bf16lo(u.x); v[1] = bf16hi(u.x); v[2] = bf16lo(u.y); v[3] = bf16hi(u.y);
  v[4] = bf16lo(u.z); v[5] = bf16hi(u.z); v[6] = bf16lo(u.w); v[7] = bf16hi(u.w);
}
__device__ __forceinline__ uint4 pack8(const float (&v)[8]) {
  uint4 u;
  u.x = pack_bf16(v[0], v[1]); u.y = pack_bf16(v[2], v[3]);
  u.z = pack_bf16(v[4], v[5]); u.w = pack_bf16(v[6], v[7]);
  return u;
}
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&v)[8]) {
  unpack8(__ldg(reinterpret_cast<const uint4*>(p)), v);
}

// ----------------------------------------------------------------- RMSNorm fwd
// h = x (+ res) rounded to bf16; y = h * rsqrt(mean(h^2) + eps) * w.
// Writes y, rstd, and h (the residual stream after the add) if h_out != null.
template <int VPT>
__global__ void __launch_bounds__(kWarps * 32) rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x,
                                                                  const __nv_bfloat16* __restrict__ res,
                                                                  const __nv_bfloat16* __restrict__ w,
                                                                  __nv_bfloat16* __restrict__ y,
                                                                  __nv_bfloat16* __restrict__ h_out,
                                                                  float* __restrict__ rstd_out, int rows, int d,
                                                                  float eps) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  uint4 r[VPT];
  load_raw<VPT>(x + (int64_t)row * d, d, lane, r);
  if (res != nullptr) {
    uint4 q[VPT];
    load_raw<VPT>(res + (int64_t)row * d, d, lane, q);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      float a[8], b[8];
      unpack8(r[i], a);
      unpack8(q[i], b);
#pragma unroll
      for (int j = 0; j < 8; ++j) a[j] += b[j];
      r[i] = pack8(a);
      const int c = (i * 32 + lane) * 8;
      if (h_out != nullptr && c < d) *reinterpret_cast<uint4*>(h_out + (int64_t)row * d + c) = r[i];
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    float a[8];
    unpack8(r[i], a);
#pragma unroll
    for (int j = 0; j < 8; ++j) ss += a[j] * a[j];
  }
  ss = warp_sum(ss);
  const float rstd = rsqrtf(ss / d + eps);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < d) {
      float a[8], wv[8];
      unpack8(r[i], a);
      load8(w + c, wv);
#pragma unroll
      for (int j = 0; j < 8; ++j) a[j] = a[j] * rstd * wv[j];
      *reinterpret_cast<uint4*>(y + (int64_t)row * d + c) = pack8(a);
    }
  }
  if (rstd_out != nullptr && lane == 0) rstd_out[row] = rstd;
}

// ----------------------------------------------------------------- RMSNorm bwd
// dx = rstd * (g - xhat * mean(g * xhat)) (+ dres), g = dy * w, xhat = x * rstd.
// dw partial per CTA (shared-memory accumulation) -> part[blockIdx.x, d].
template <int VPT>
__global__ void __launch_bounds__(kWarps * 32) rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy,
                                                                  const __nv_bfloat16* __restrict__ x,
                                                                  const __nv_bfloat16* __restrict__ w,
                                                                  const float* __restrict__ rstd,
                                                                  const __nv_bfloat16* __restrict__ dres,
                                                                  __nv_bfloat16* __restrict__ dx,
                                                                  float* __restrict__ part, int rows, int d) {
  extern __shared__ float sdw[];  // [d]
  for (int c = threadIdx.x; c < d; c += blockDim.x) sdw[c] = 0.f;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  // dw: a lane owns the same columns in every row, so up to 2048 wide the
  // partial sums stay in registers and meet in shared memory once per CTA
  constexpr bool kRegDw = VPT <= 8;
  float dwr[kRegDw ? VPT : 1][8];
#pragma unroll
  for (int i = 0; i < (kRegDw ? VPT : 1); ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) dwr[i][j] = 0.f;
  for (int row = blockIdx.x * kWarps + warp; row < rows; row += gridDim.x * kWarps) {
    uint4 rx[VPT], rg[VPT];
    load_raw<VPT>(x + (int64_t)row * d, d, lane, rx);
    load_raw<VPT>(dy + (int64_t)row * d, d, lane, rg);
    const float rs = rstd[row];
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = (i * 32 + lane) * 8;
      if (c < d) {
        float a[8], g[8], wv[8];
        unpack8(rx[i], a);
        unpack8(rg[i], g);
        load8(w + c, wv);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float xh = a[j] * rs;
          if constexpr (kRegDw) {
            dwr[i][j] += g[j] * xh;
          } else {
            atomicAdd(&sdw[c + j], g[j] * xh);
          }
          dot += g[j] * wv[j] * xh;
        }
      }
    }
    dot = warp_sum(dot) / d;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = (i * 32 + lane) * 8;
      if (c < d) {
        float a[8], g[8], wv[8];
        unpack8(rx[i], a);
        unpack8(rg[i], g);
        load8(w + c, wv);
#pragma unroll
        for (int j = 0; j < 8; ++j) g[j] = rs * (g[j] * wv[j] - a[j] * rs * dot);
        if (dres != nullptr) {
          float q[8];
          load8(dres + (int64_t)row * d + c, q);
#pragma unroll
          for (int j = 0; j < 8; ++j) g[j] += q[j];
        }
        *reinterpret_cast<uint4*>(dx + (int64_t)row * d + c) = pack8(g);
      }
    }
  }
  if constexpr (kRegDw) {
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = (i * 32 + lane) * 8;
      if (c < d) {
#pragma unroll
        for (int j = 0; j < 8; ++j) atomicAdd(&sdw[c + j], dwr[i][j]);
      }
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < d; c += blockDim.x) part[(int64_t)blockIdx.x * d + c] = sdw[c];
}

// Column reduction of per-CTA partials: out[c] (+)= sum_b part[b, c].
__global__ void column_reduce_kernel(const float* __restrict__ part, int nparts, int64_t ldp, int d,
                                     float* __restrict__ out, bool accumulate) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= d) return;
  float s = 0.f;
  for (int b = 0; b < nparts; ++b) s += part[(int64_t)b * ldp + c];
  out[c] = accumulate ? out[c] + s : s;
}

// ----------------------------------------------------------------- LayerNorm
template <int VPT>
__global__ void __launch_bounds__(kWarps * 32) layernorm_fwd_kernel(const __nv_bfloat16* __restrict__ x,
                                                                    const __nv_bfloat16* __restrict__ res,
                                                                    const __nv_bfloat16* __restrict__ w,
                                                                    const __nv_bfloat16* __restrict__ b,
                                                                    __nv_bfloat16* __restrict__ y,
                                                                    __nv_bfloat16* __restrict__ h_out,
                                                                    float* __restrict__ mean_out,
                                                                    float* __restrict__ rstd_out, int rows, int d,
                                                                    float eps) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  uint4 r[VPT];
  load_raw<VPT>(x + (int64_t)row * d, d, lane, r);
  if (res != nullptr) {
    uint4 q[VPT];
    load_raw<VPT>(res + (int64_t)row * d, d, lane, q);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      float a[8], bb[8];
      unpack8(r[i], a);
      unpack8(q[i], bb);
#pragma unroll
      for (int j = 0; j < 8; ++j) a[j] += bb[j];
      r[i] = pack8(a);
      const int c = (i * 32 + lane) * 8;
      if (h_out != nullptr && c < d) *reinterpret_cast<uint4*>(h_out + (int64_t)row * d + c) = r[i];
    }
  }
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    float a[8];
    unpack8(r[i], a);
#pragma unroll
    for (int j = 0; j < 8; ++j) s += a[j];
  }
  const float mean = warp_sum(s) / d;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < d) {
      float a[8];
      unpack8(r[i], a);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += (a[j] - mean) * (a[j] - mean);
    }
  }
  const float rstd = rsqrtf(warp_sum(ss) / d + eps);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < d) {
      float a[8], wv[8], bv[8];
      unpack8(r[i], a);
      load8(w + c, wv);
      if (b != nullptr) load8(b + c, bv);
#pragma unroll
      for (int j = 0; j < 8; ++j) a[j] = (a[j] - mean) * rstd * wv[j] + (b != nullptr ? bv[j] : 0.f);
      *reinterpret_cast<uint4*>(y + (int64_t)row * d + c) = pack8(a);
    }
  }
  if (lane == 0) {
    if (mean_out) mean_out[row] = mean;
    if (rstd_out) rstd_out[row] = rstd;
  }
}

// dx = rstd * (g - mean(g) - xhat * mean(g * xhat)) (+ dres), g = dy * w.
// Partials: part[blk, 0:d] = sum dy*xhat (dw), part[blk, d:2d] = sum dy (db).
template <int VPT>
__global__ void __launch_bounds__(kWarps * 32) layernorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy,
                                                                    const __nv_bfloat16* __restrict__ x,
                                                                    const __nv_bfloat16* __restrict__ w,
                                                                    const float* __restrict__ mean,
                                                                    const float* __restrict__ rstd,
                                                                    const __nv_bfloat16* __restrict__ dres,
                                                                    __nv_bfloat16* __restrict__ dx,
                                                                    float* __restrict__ part, int rows, int d) {
  extern __shared__ float sdw[];  // [2d]
  for (int c = threadIdx.x; c < 2 * d; c += blockDim.x) sdw[c] = 0.f;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  // dw / db partials in registers across the warp's rows up to 1024 wide
  // (BERT / ViT widths); wider rows add into shared memory per element
  constexpr bool kRegDw = VPT <= 4;
  float dwr[kRegDw ? VPT : 1][8], dbr[kRegDw ? VPT : 1][8];
#pragma unroll
  for (int i = 0; i < (kRegDw ? VPT : 1); ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) dwr[i][j] = dbr[i][j] = 0.f;
  for (int row = blockIdx.x * kWarps + warp; row < rows; row += gridDim.x * kWarps) {
    uint4 rx[VPT], rg[VPT];
    load_raw<VPT>(x + (int64_t)row * d, d, lane, rx);
    load_raw<VPT>(dy + (int64_t)row * d, d, lane, rg);
    const float mu = mean[row], rs = rstd[row];
    float sg = 0.f, sgx = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = (i * 32 + lane) * 8;
      if (c < d) {
        float a[8], g[8], wv[8];
        unpack8(rx[i], a);
        unpack8(rg[i], g);
        load8(w + c, wv);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float xh = (a[j] - mu) * rs;
          if constexpr (kRegDw) {
            dwr[i][j] += g[j] * xh;
            dbr[i][j] += g[j];
          } else {
            atomicAdd(&sdw[c + j], g[j] * xh);
            atomicAdd(&sdw[d + c + j], g[j]);
          }
          const float gw = g[j] * wv[j];
          sg += gw;
          sgx += gw * xh;
        }
      }
    }
    sg = warp_sum(sg) / d;
    sgx = warp_sum(sgx) / d;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = (i * 32 + lane) * 8;
      if (c < d) {
        float a[8], g[8], wv[8];
        unpack8(rx[i], a);
        unpack8(rg[i], g);
        load8(w + c, wv);
#pragma unroll
        for (int j = 0; j < 8; ++j) g[j] = rs * (g[j] * wv[j] - sg - (a[j] - mu) * rs * sgx);
        if (dres != nullptr) {
          float q[8];
          load8(dres + (int64_t)row * d + c, q);
#pragma unroll
          for (int j = 0; j < 8; ++j) g[j] += q[j];
        }
        *reinterpret_cast<uint4*>(dx + (int64_t)row * d + c) = pack8(g);
      }
    }
  }
  if constexpr (kRegDw) {
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = (i * 32 + lane) * 8;
      if (c < d) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          atomicAdd(&sdw[c + j], dwr[i][j]);
          atomicAdd(&sdw[d + c + j], dbr[i][j]);
        }
      }
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < 2 * d; c += blockDim.x) part[(int64_t)blockIdx.x * 2 * d + c] = sdw[c];
}

// ----------------------------------------------------------------- softmax
// y = softmax(scale * x) over the row, held packed in registers.
template <int VPT>
__global__ void __launch_bounds__(kWarps * 32) softmax_fwd_kernel(const __nv_bfloat16* __restrict__ x,
                                                                  __nv_bfloat16* __restrict__ y, int rows, int d,
                                                                  float scale) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  uint4 r[VPT];
  load_raw<VPT>(x + (int64_t)row * d, d, lane, r);
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < d) {
      float a[8];
      unpack8(r[i], a);
#pragma unroll
      for (int j = 0; j < 8; ++j) mx = fmaxf(mx, a[j] * scale);
    }
  }
  mx = warp_max(mx);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < d) {
      float a[8];
      unpack8(r[i], a);
#pragma unroll
      for (int j = 0; j < 8; ++j) s += __expf(a[j] * scale - mx);
    }
  }
  const float inv = 1.f / warp_sum(s);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < d) {
      float a[8];
      unpack8(r[i], a);
#pragma unroll
      for (int j = 0; j < 8; ++j) a[j] = __expf(a[j] * scale - mx) * inv;
      *reinterpret_cast<uint4*>(y + (int64_t)row * d + c) = pack8(a);
    }
  }
}

// dx = scale * y * (dy - <y, dy>)
template <int VPT>
__global__ void __launch_bounds__(kWarps * 32) softmax_bwd_kernel(const __nv_bfloat16* __restrict__ y,
                                                                  const __nv_bfloat16* __restrict__ dy,
                                                                  __nv_bfloat16* __restrict__ dx, int rows, int d,
                                                                  float scale) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  uint4 ry[VPT], rg[VPT];
  load_raw<VPT>(y + (int64_t)row * d, d, lane, ry);
  load_raw<VPT>(dy + (int64_t)row * d, d, lane, rg);
  float dot = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    float a[8], g[8];
    unpack8(ry[i], a);
    unpack8(rg[i], g);
#pragma unroll
    for (int j = 0; j < 8; ++j) dot += a[j] * g[j];
  }
  dot = warp_sum(dot);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (i * 32 + lane) * 8;
    if (c < d) {
      float a[8], g[8];
      unpack8(ry[i], a);
      unpack8(rg[i], g);
#pragma unroll
      for (int j = 0; j < 8; ++j) g[j] = scale * a[j] * (g[j] - dot);
      *reinterpret_cast<uint4*>(dx + (int64_t)row * d + c) = pack8(g);
    }
  }
}

#define AETHER_VPT_DISPATCH(d, ...)                                              \
  do {                                                                           \
    const int _vpt = ((d) + 255) / 256;                                          \
    switch (_vpt) {                                                              \
      case 1: { constexpr int VPT = 1; __VA_ARGS__; } break;                     \
      case 2: { constexpr int VPT = 2; __VA_ARGS__; } break;                     \
      case 3: { constexpr int VPT = 3; __VA_ARGS__; } break;                     \
      case 4: { constexpr int VPT = 4; __VA_ARGS__; } break;                     \
      case 5: case 6: { constexpr int VPT = 6; __VA_ARGS__; } break;             \
      case 7: case 8: { constexpr int VPT = 8; __VA_ARGS__; } break;             \
      case 9: case 10: case 11: case 12: { constexpr int VPT = 12; __VA_ARGS__; } break; \
      case 13: case 14: case 15: case 16: { constexpr int VPT = 16; __VA_ARGS__; } break; \
      default: TORCH_CHECK(false, "row width ", d, " exceeds 4096");             \
    }                                                                            \
  } while (0)

const __nv_bfloat16* bf(const at::Tensor& t) { return reinterpret_cast<const __nv_bfloat16*>(t.data_ptr()); }
__nv_bfloat16* bfm(const at::Tensor& t) { return reinterpret_cast<__nv_bfloat16*>(t.data_ptr()); }
const __nv_bfloat16* bf_opt(const std::optional<at::Tensor>& t) {
  return (t && t->defined()) ? bf(*t) : nullptr;
}

void check_rows(const at::Tensor& t, int64_t d, const char* what) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.is_contiguous(), what, ": contiguous bf16 CUDA tensor required");
  TORCH_CHECK(t.size(-1) == d, what, ": last dim mismatch");
}

int bwd_grid(int64_t rows) {
  const int n = num_sms(current_device()) * 2;
  return (int)std::max<int64_t>(1, std::min<int64_t>(n, (rows + kWarps - 1) / kWarps));
}

}  // namespace

// Returns rstd [rows] fp32. When `res` is given, `h_out` receives x + res.
void rmsnorm_fwd(at::Tensor x, std::optional<at::Tensor> res, at::Tensor w, at::Tensor y,
                 std::optional<at::Tensor> h_out, std::optional<at::Tensor> rstd, double eps) {
  const int64_t d = x.size(-1);
  const int64_t rows = x.numel() / d;
  check_rows(x, d, "rmsnorm x");
  check_rows(y, d, "rmsnorm y");
  TORCH_CHECK(d % 8 == 0, "rmsnorm: width must be a multiple of 8");
  c10::cuda::CUDAGuard g(x.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const int grid = (int)((rows + kWarps - 1) / kWarps);
  float* rs = (rstd && rstd->defined()) ? rstd->data_ptr<float>() : nullptr;
  __nv_bfloat16* h = (h_out && h_out->defined()) ? bfm(*h_out) : nullptr;
  AETHER_VPT_DISPATCH(d, rmsnorm_fwd_kernel<VPT><<<grid, kWarps * 32, 0, stream>>>(
                             bf(x), bf_opt(res), bf(w), bfm(y), h, rs, (int)rows, (int)d, (float)eps));
  AETHER_CUDA_CHECK(cudaGetLastError());
}

// dx (bf16), dw accumulated into dw_f32 (fp32 [d]) when accumulate, else written.
void rmsnorm_bwd(at::Tensor dy, at::Tensor x, at::Tensor w, at::Tensor rstd, std::optional<at::Tensor> dres,
                 at::Tensor dx, at::Tensor dw_f32, bool accumulate) {
  const int64_t d = x.size(-1);
  const int64_t rows = x.numel() / d;
  check_rows(dy, d, "rmsnorm_bwd dy");
  check_rows(x, d, "rmsnorm_bwd x");
  check_rows(dx, d, "rmsnorm_bwd dx");
  c10::cuda::CUDAGuard g(x.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const int grid = bwd_grid(rows);
  auto part = at::empty({grid, d}, x.options().dtype(at::kFloat));
  const size_t smem = (size_t)d * sizeof(float);
  AETHER_VPT_DISPATCH(d, {
    auto k = rmsnorm_bwd_kernel<VPT>;
    if (smem > 48 * 1024) AETHER_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    k<<<grid, kWarps * 32, smem, stream>>>(bf(dy), bf(x), bf(w), rstd.data_ptr<float>(), bf_opt(dres), bfm(dx),
                                           part.data_ptr<float>(), (int)rows, (int)d);
  });
  AETHER_CUDA_CHECK(cudaGetLastError());
  column_reduce_kernel<<<(int)((d + 255) / 256), 256, 0, stream>>>(part.data_ptr<float>(), grid, d, (int)d,
                                                                   dw_f32.data_ptr<float>(), accumulate);
  AETHER_CUDA_CHECK(cudaGetLastError());
}

void layernorm_fwd(at::Tensor x, std::optional<at::Tensor> res, at::Tensor w, std::optional<at::Tensor> b,
                   at::Tensor y, std::optional<at::Tensor> h_out, at::Tensor mean, at::Tensor rstd, double eps) {
  const int64_t d = x.size(-1);
  const int64_t rows = x.numel() / d;
  check_rows(x, d, "layernorm x");
  check_rows(y, d, "layernorm y");
  TORCH_CHECK(d % 8 == 0, "layernorm: width must be a multiple of 8");
  c10::cuda::CUDAGuard g(x.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const int grid = (int)((rows + kWarps - 1) / kWarps);
  __nv_bfloat16* h = (h_out && h_out->defined()) ? bfm(*h_out) : nullptr;
  AETHER_VPT_DISPATCH(d, layernorm_fwd_kernel<VPT><<<grid, kWarps * 32, 0, stream>>>(
                             bf(x), bf_opt(res), bf(w), bf_opt(b), bfm(y), h, mean.data_ptr<float>(),
                             rstd.data_ptr<float>(), (int)rows, (int)d, (float)eps));
  AETHER_CUDA_CHECK(cudaGetLastError());
}

void layernorm_bwd(at::Tensor dy, at::Tensor x, at::Tensor w, at::Tensor mean, at::Tensor rstd,
                   std::optional<at::Tensor> dres, at::Tensor dx, at::Tensor dw_f32, at::Tensor db_f32,
                   bool accumulate) {
  const int64_t d = x.size(-1);
  const int64_t rows = x.numel() / d;
  check_rows(dy, d, "layernorm_bwd dy");
  check_rows(x, d, "layernorm_bwd x");
  c10::cuda::CUDAGuard g(x.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const int grid = bwd_grid(rows);
  auto part = at::empty({grid, 2 * d}, x.options().dtype(at::kFloat));
  const size_t smem = (size_t)2 * d * sizeof(float);
  AETHER_VPT_DISPATCH(d, {
    auto k = layernorm_bwd_kernel<VPT>;
    if (smem > 48 * 1024) AETHER_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    k<<<grid, kWarps * 32, smem, stream>>>(bf(dy), bf(x), bf(w), mean.data_ptr<float>(), rstd.data_ptr<float>(),
                                           bf_opt(dres), bfm(dx), part.data_ptr<float>(), (int)rows, (int)d);
  });
  AETHER_CUDA_CHECK(cudaGetLastError());
  // dw = column sums of part[:, :d], db = column sums of part[:, d:].
  column_reduce_kernel<<<(int)((d + 255) / 256), 256, 0, stream>>>(part.data_ptr<float>(), grid, 2 * d, (int)d,
                                                                   dw_f32.data_ptr<float>(), accumulate);
  column_reduce_kernel<<<(int)((d + 255) / 256), 256, 0, stream>>>(part.data_ptr<float>() + d, grid, 2 * d, (int)d,
                                                                   db_f32.data_ptr<float>(), accumulate);
  AETHER_CUDA_CHECK(cudaGetLastError());
}

void softmax_fwd(at::Tensor x, at::Tensor y, double scale) {
  const int64_t d = x.size(-1);
  const int64_t rows = x.numel() / d;
  check_rows(x, d, "softmax x");
  check_rows(y, d, "softmax y");
  TORCH_CHECK(d % 8 == 0, "softmax: width must be a multiple of 8");
  c10::cuda::CUDAGuard g(x.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const int grid = (int)((rows + kWarps - 1) / kWarps);
  AETHER_VPT_DISPATCH(d, softmax_fwd_kernel<VPT><<<grid, kWarps * 32, 0, stream>>>(bf(x), bfm(y), (int)rows, (int)d,
                                                                                    (float)scale));
  AETHER_CUDA_CHECK(cudaGetLastError());
}

void softmax_bwd(at::Tensor y, at::Tensor dy, at::Tensor dx, double scale) {
  const int64_t d = y.size(-1);
  const int64_t rows = y.numel() / d;
  check_rows(y, d, "softmax_bwd y");
  check_rows(dy, d, "softmax_bwd dy");
  c10::cuda::CUDAGuard g(y.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const int grid = (int)((rows + kWarps - 1) / kWarps);
  AETHER_VPT_DISPATCH(d, softmax_bwd_kernel<VPT><<<grid, kWarps * 32, 0, stream>>>(bf(y), bf(dy), bfm(dx), (int)rows,
                                                                                    (int)d, (float)scale));
  AETHER_CUDA_CHECK(cudaGetLastError());
}


namespace {
// In-place RMSNorm of heads [h0, h0 + nh) of every row of x [T, ld] (head h at
// h * D), with a weight [D] shared by all heads (Qwen3 q/k norm). One warp per
// (row, head); D a multiple of 64 up to 256.
__global__ void head_rmsnorm_kernel(__nv_bfloat16* __restrict__ x, int64_t ld, int T, int h0, int nh, int D,
                                    const __nv_bfloat16* __restrict__ w, float eps) {
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= (int64_t)T * nh) return;
  const int t = (int)(wid / nh), h = h0 + (int)(wid % nh);
  __nv_bfloat16* row = x + (int64_t)t * ld + (int64_t)h * D;
  const int per = D / 32;  // 2, 4 or 8 elements per lane
  float v[8];
  float ss = 0.f;
  for (int j = 0; j < per; ++j) {
    v[j] = __bfloat162float(row[lane * per + j]);
    ss += v[j] * v[j];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float r = rsqrtf(ss / D + eps);
  for (int j = 0; j < per; ++j)
    row[lane * per + j] = __float2bfloat16(v[j] * r * __bfloat162float(w[lane * per + j]));
}
}  // namespace

void head_rmsnorm(at::Tensor x, int64_t h0, int64_t nh, int64_t D, at::Tensor w, double eps) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1,
              "head_rmsnorm: bf16 [T, row]");
  TORCH_CHECK(D % 64 == 0 && D <= 256 && w.numel() == D && w.is_contiguous() && (h0 + nh) * D <= x.size(1),
              "head_rmsnorm: D in {64, 128, 192, 256}, weight [D]");
  c10::cuda::CUDAGuard g(x.device());
  const int64_t warps = x.size(0) * nh;
  if (warps == 0) return;
  head_rmsnorm_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(x.data_ptr()), x.stride(0), (int)x.size(0), (int)h0, (int)nh, (int)D,
      reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), (float)eps);
  AETHER_CUDA_CHECK(cudaGetLastError());
}

}  // namespace aether
