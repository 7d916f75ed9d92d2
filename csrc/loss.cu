// Fused cross-entropy (loss + logits gradient in one pass pair) and argmax.
//
// Reference: cross_entropy_fwd / cross_entropy_bwd (runtime/src/cuda.rs:6615-6657)
// use one thread per row walking all V logits serially and materialise an fp32
// `probs` tensor. Here one CTA owns a row: pass 1 computes an online
// max / sum-of-exp with 16-byte loads, pass 2 (which hits L2) writes
// (softmax - onehot) * scale straight over the bf16 logits (or into a separate
// buffer), so no [T, V] fp32 tensor ever exists. The probability floor of the
// reference (-log(max(p, 1e-12))) is kept.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "host_utils.h"

namespace aether {
namespace {

constexpr int kCeThreads = 512;

__device__ __forceinline__ void online_update(float& m, float& s, float x) {
  if (x > m) {
    s = s * __expf(m - x) + 1.f;
    m = x;
  } else {
    s += __expf(x - m);
  }
}

__device__ __forceinline__ void merge_ms(float& m, float& s, float m2, float s2) {
  const float mx = fmaxf(m, m2);
  if (mx == -INFINITY) return;
  s = s * __expf(m - mx) + s2 * __expf(m2 - mx);
  m = mx;
}

// logits [T, ld] bf16 (first V columns used); targets int64 [T] (-100 = ignore).
// loss[t] = lse - x[target] (floored), lse_out[t] = lse.
// If dlogits != null: dlogits[t, :] = (softmax - onehot) * scale (bf16), may alias logits.
__global__ void __launch_bounds__(kCeThreads) cross_entropy_kernel(const __nv_bfloat16* logits, int64_t ld, int V,
                                                                    const int64_t* __restrict__ targets,
                                                                    float* __restrict__ loss,
                                                                    float* __restrict__ lse_out,
                                                                    __nv_bfloat16* dlogits, int64_t ldd,
                                                                    const float* __restrict__ scale_ptr,
                                                                    float scale, int ignore_index) {
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* x = logits + row * ld;
  // 16-byte vector path only when every row (and the gradient row) starts aligned.
  const bool vec = ((ld & 7) == 0) && (dlogits == nullptr || (ldd & 7) == 0);
  const int nchunk = vec ? V / 8 : 0;
  const int64_t tgt = targets[row];
  const bool valid = tgt != ignore_index && tgt >= 0 && tgt < V;
  // Read the target logit before any thread can overwrite the row in pass 2.
  const float xt = (threadIdx.x == 0 && valid) ? __bfloat162float(x[tgt]) : 0.f;
  float m = -INFINITY, s = 0.f;
  for (int c = threadIdx.x; c < nchunk; c += kCeThreads) {
    const uint4 u = reinterpret_cast<const uint4*>(x)[c];
    const float v[8] = {bf16lo(u.x), bf16hi(u.x), bf16lo(u.y), bf16hi(u.y),
                        bf16lo(u.z), bf16hi(u.z), bf16lo(u.w), bf16hi(u.w)};
    float cm = v[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) cm = fmaxf(cm, v[j]);
    float cs = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) cs += __expf(v[j] - cm);
    merge_ms(m, s, cm, cs);
  }
  for (int c = nchunk * 8 + threadIdx.x; c < V; c += kCeThreads) online_update(m, s, __bfloat162float(x[c]));
  // block reduce (m, s)
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    merge_ms(m, s, m2, s2);
  }
  __shared__ float sm[kCeThreads / 32], ss[kCeThreads / 32];
  __shared__ float s_lse;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sm[warp] = m;
    ss[warp] = s;
  }
  __syncthreads();
  if (warp == 0) {
    m = lane < kCeThreads / 32 ? sm[lane] : -INFINITY;
    s = lane < kCeThreads / 32 ? ss[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      merge_ms(m, s, m2, s2);
    }
    if (lane == 0) s_lse = m + __logf(s);
  }
  __syncthreads();
  const float lse = s_lse;
  if (threadIdx.x == 0) {
    float l = 0.f;
    if (valid) {
      const float p = fmaxf(__expf(xt - lse), 1e-12f);
      l = -__logf(p);
    }
    loss[row] = l;
    if (lse_out) lse_out[row] = lse;
  }
  if (dlogits == nullptr) return;
  const float sc = valid ? (scale_ptr ? *scale_ptr * scale : scale) : 0.f;
  __nv_bfloat16* dx = dlogits + row * ldd;
  // pass 2 (the row is re-read from L2); the target column is corrected below.
  for (int c = threadIdx.x; c < nchunk; c += kCeThreads) {
    const uint4 u = reinterpret_cast<const uint4*>(x)[c];
    float v[8] = {bf16lo(u.x), bf16hi(u.x), bf16lo(u.y), bf16hi(u.y),
                  bf16lo(u.z), bf16hi(u.z), bf16lo(u.w), bf16hi(u.w)};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float g = __expf(v[j] - lse);
      if (c * 8 + j == tgt) g -= 1.f;
      v[j] = g * sc;
    }
    uint4 o;
    o.x = pack_bf16(v[0], v[1]); o.y = pack_bf16(v[2], v[3]);
    o.z = pack_bf16(v[4], v[5]); o.w = pack_bf16(v[6], v[7]);
    reinterpret_cast<uint4*>(dx)[c] = o;
  }
  for (int c = nchunk * 8 + threadIdx.x; c < V; c += kCeThreads) {
    float g = __expf(__bfloat162float(x[c]) - lse);
    if (c == tgt) g -= 1.f;
    dx[c] = __float2bfloat16(g * sc);
  }
}

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }

// Row argmax over the first V columns of a bf16 or fp32 matrix. One CTA per
// row; each thread keeps 4 independent 16-byte loads in flight (64 bytes per
// trip) so a single row of a 152K vocabulary is read at many bytes per clock
// instead of one dependent load chain per thread. Ties go to the lowest index.
__device__ __forceinline__ void argmax_take(float v, int c, float& best, int& idx) {
  if (v > best || (v == best && c < idx)) {
    best = v;
    idx = c;
  }
}
__device__ __forceinline__ void argmax_vec(const uint4& u, int c0, const float*, float& best, int& idx) {
  const float f[4] = {__uint_as_float(u.x), __uint_as_float(u.y), __uint_as_float(u.z), __uint_as_float(u.w)};
#pragma unroll
  for (int j = 0; j < 4; ++j) argmax_take(f[j], c0 + j, best, idx);
}
__device__ __forceinline__ void argmax_vec(const uint4& u, int c0, const __nv_bfloat16*, float& best, int& idx) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    argmax_take(__uint_as_float(w[j] << 16), c0 + 2 * j, best, idx);
    argmax_take(__uint_as_float(w[j] & 0xffff0000u), c0 + 2 * j + 1, best, idx);
  }
}

template <typename T>
__global__ void __launch_bounds__(1024) argmax_kernel(const T* __restrict__ x, int64_t ld, int V,
                                                      int64_t* __restrict__ out, bool vec) {
  const T* row = x + (int64_t)blockIdx.x * ld;
  float best = -INFINITY;
  int idx = 0x7fffffff;
  constexpr int E = 16 / sizeof(T);  // elements per 16-byte load
  constexpr int U = 4;               // loads in flight per thread
  int done = 0;
  if (vec) {
    const int per_trip = 1024 * E * U;
    const int full = V / per_trip * per_trip;
    for (int base = 0; base < full; base += per_trip) {
      uint4 u[U];
#pragma unroll
      for (int k = 0; k < U; ++k)
        u[k] = __ldg(reinterpret_cast<const uint4*>(row + base + (k * 1024 + threadIdx.x) * E));
#pragma unroll
      for (int k = 0; k < U; ++k) argmax_vec(u[k], base + (k * 1024 + threadIdx.x) * E, row, best, idx);
    }
    done = full;
  }
  for (int c = done + threadIdx.x; c < V; c += blockDim.x) argmax_take(to_f(row[c]), c, best, idx);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float b2 = __shfl_xor_sync(0xffffffffu, best, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
    argmax_take(b2, i2, best, idx);
  }
  __shared__ float sb[32];
  __shared__ int si[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sb[warp] = best;
    si[warp] = idx;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x / 32;
    best = lane < nw ? sb[lane] : -INFINITY;
    idx = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float b2 = __shfl_xor_sync(0xffffffffu, best, o);
      const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
      argmax_take(b2, i2, best, idx);
    }
    if (lane == 0) out[blockIdx.x] = idx == 0x7fffffff ? 0 : idx;
  }
}

}  // namespace

// Fused CE. Returns nothing; writes loss [T] fp32, lse [T] fp32 (optional) and,
// when dlogits is given, the scaled gradient (may alias logits).
void cross_entropy_fused(at::Tensor logits, at::Tensor targets, at::Tensor loss, std::optional<at::Tensor> lse,
                         std::optional<at::Tensor> dlogits, std::optional<at::Tensor> scale_t, double scale,
                         int64_t ignore_index) {
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1 && logits.scalar_type() == at::kBFloat16, "ce: logits [T, V] bf16");
  TORCH_CHECK(targets.scalar_type() == at::kLong && targets.is_contiguous(), "ce: targets int64");
  const int64_t T = logits.size(0);
  const int V = (int)logits.size(1);
  c10::cuda::CUDAGuard g(logits.device());
  __nv_bfloat16* dptr = nullptr;
  int64_t ldd = 0;
  if (dlogits && dlogits->defined()) {
    TORCH_CHECK(dlogits->stride(1) == 1 && dlogits->size(0) == T, "ce: dlogits layout");
    dptr = reinterpret_cast<__nv_bfloat16*>(dlogits->data_ptr());
    ldd = dlogits->stride(0);
  }
  if (T == 0) return;
  cross_entropy_kernel<<<(unsigned)T, kCeThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), logits.stride(0), V, targets.data_ptr<int64_t>(),
      loss.data_ptr<float>(), (lse && lse->defined()) ? lse->data_ptr<float>() : nullptr, dptr, ldd,
      (scale_t && scale_t->defined()) ? scale_t->data_ptr<float>() : nullptr, (float)scale, (int)ignore_index);
  AETHER_CUDA_CHECK(cudaGetLastError());
}

void argmax_rows(at::Tensor x, at::Tensor out) {
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "argmax: 2-D rows");
  TORCH_CHECK(out.scalar_type() == at::kLong && out.numel() == x.size(0), "argmax: out int64 [rows]");
  c10::cuda::CUDAGuard g(x.device());
  const unsigned rows = (unsigned)x.size(0);
  if (rows == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  const bool vec = reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 && (x.stride(0) * x.element_size()) % 16 == 0;
  if (x.scalar_type() == at::kBFloat16)
    argmax_kernel<__nv_bfloat16><<<rows, 1024, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
                                                            x.stride(0), (int)x.size(1), out.data_ptr<int64_t>(), vec);
  else if (x.scalar_type() == at::kFloat)
    argmax_kernel<float><<<rows, 1024, 0, stream>>>(x.data_ptr<float>(), x.stride(0), (int)x.size(1),
                                                    out.data_ptr<int64_t>(), vec);
  else
    TORCH_CHECK(false, "argmax: bf16 or fp32");
  AETHER_CUDA_CHECK(cudaGetLastError());
}

}  // namespace aether
