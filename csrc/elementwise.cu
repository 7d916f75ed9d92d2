// Elementwise / gather kernels: SwiGLU, tanh-GELU, half-split RoPE, embedding
// gather and scatter-add, plus small helpers (scale, add).
//
// Reference semantics: silu_inplace / mul_inplace / silu_bwd
// (runtime/src/cuda.rs:3111-3147, 7011), gelu_fwd / gelu_bwd (cuda.rs:2756,
// 6855), rope_apply / rope_apply_devarg / rope_apply_backward (cuda.rs:2994,
// 3034, 6986; theta_i = base^(-2i/hd), pairs (i, i + hd/2)), embed_lookup /
// embed_scatter_add (cuda.rs:6659-6692). Every kernel here moves 16 bytes per
// thread per access; RoPE reads positions from device memory so a captured
// CUDA graph replays it for any step.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "host_utils.h"

namespace aether {
namespace {

__device__ __forceinline__ float silu_f(float g) { return g / (1.f + __expf(-g)); }

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

// h: [T, 2F] = [gate | up]; act: [T, F] = silu(gate) * up
__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ h, __nv_bfloat16* __restrict__ act, int64_t T,
                                  int F, int64_t ldh) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // one 8-wide chunk
  const int64_t chunks_per_row = F / 8;
  if (i >= T * chunks_per_row) return;
  const int64_t t = i / chunks_per_row;
  const int c = (int)(i - t * chunks_per_row) * 8;
  float g[8], u[8], o[8];
  unpack8(*reinterpret_cast<const uint4*>(h + t * ldh + c), g);
  unpack8(*reinterpret_cast<const uint4*>(h + t * ldh + F + c), u);
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j] = silu_f(g[j]) * u[j];
  *reinterpret_cast<uint4*>(act + t * F + c) = pack8(o);
}

// dh[:, :F] = dact * up * silu'(gate); dh[:, F:] = dact * silu(gate)
__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ h, const __nv_bfloat16* __restrict__ dact,
                                  __nv_bfloat16* __restrict__ dh, int64_t T, int F, int64_t ldh) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t chunks_per_row = F / 8;
  if (i >= T * chunks_per_row) return;
  const int64_t t = i / chunks_per_row;
  const int c = (int)(i - t * chunks_per_row) * 8;
  float g[8], u[8], da[8], dg[8], du[8];
  unpack8(*reinterpret_cast<const uint4*>(h + t * ldh + c), g);
  unpack8(*reinterpret_cast<const uint4*>(h + t * ldh + F + c), u);
  unpack8(*reinterpret_cast<const uint4*>(dact + t * F + c), da);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float s = 1.f / (1.f + __expf(-g[j]));
    const float sl = g[j] * s;
    du[j] = da[j] * sl;
    dg[j] = da[j] * u[j] * s * (1.f + g[j] * (1.f - s));
  }
  *reinterpret_cast<uint4*>(dh + t * 2 * F + c) = pack8(dg);
  *reinterpret_cast<uint4*>(dh + t * 2 * F + F + c) = pack8(du);
}

__device__ __forceinline__ float gelu_tanh(float x) {
  const float k = 0.7978845608028654f;  // sqrt(2/pi)
  return 0.5f * x * (1.f + tanhf(k * (x + 0.044715f * x * x * x)));
}
__device__ __forceinline__ float gelu_tanh_grad(float x) {
  const float k = 0.7978845608028654f;
  const float u = k * (x + 0.044715f * x * x * x);
  const float th = tanhf(u);
  return 0.5f * (1.f + th) + 0.5f * x * (1.f - th * th) * k * (1.f + 3.f * 0.044715f * x * x);
}

__global__ void gelu_fwd_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y, int64_t n8) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  float v[8];
  unpack8(reinterpret_cast<const uint4*>(x)[i], v);
#pragma unroll
  for (int j = 0; j < 8; ++j) v[j] = gelu_tanh(v[j]);
  reinterpret_cast<uint4*>(y)[i] = pack8(v);
}

__global__ void gelu_bwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ dy,
                                __nv_bfloat16* __restrict__ dx, int64_t n8) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  float v[8], g[8];
  unpack8(reinterpret_cast<const uint4*>(x)[i], v);
  unpack8(reinterpret_cast<const uint4*>(dy)[i], g);
#pragma unroll
  for (int j = 0; j < 8; ++j) g[j] *= gelu_tanh_grad(v[j]);
  reinterpret_cast<uint4*>(dx)[i] = pack8(g);
}

// In-place half-split RoPE over the first `n_heads` heads of each token row.
// x: [T, row_stride] bf16, head h occupies [h*D, (h+1)*D). pos: int32 [T]
// (position of each token), cos/sin: fp32 [max_pos, D/2]. `sign` = -1 applies
// the inverse rotation (backward).
__global__ void rope_kernel(__nv_bfloat16* __restrict__ x, const int* __restrict__ pos,
                            const float* __restrict__ cos_t, const float* __restrict__ sin_t, int64_t T,
                            int n_heads, int D, int64_t row_stride, float sign) {
  const int half = D / 2;
  const int chunks = half / 8;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= T * n_heads * chunks) return;
  const int c = (int)(i % chunks) * 8;
  const int64_t th = i / chunks;
  const int h = (int)(th % n_heads);
  const int64_t t = th / n_heads;
  const int p = pos[t];
  __nv_bfloat16* base = x + t * row_stride + (int64_t)h * D;
  float a[8], b[8];
  unpack8(*reinterpret_cast<const uint4*>(base + c), a);
  unpack8(*reinterpret_cast<const uint4*>(base + half + c), b);
  const float4* cp = reinterpret_cast<const float4*>(cos_t + (int64_t)p * half + c);
  const float4* sp = reinterpret_cast<const float4*>(sin_t + (int64_t)p * half + c);
  const float4 c0 = cp[0], c1 = cp[1], s0 = sp[0], s1 = sp[1];
  const float cs[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
  const float sn[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
  float oa[8], ob[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float s = sign * sn[j];
    oa[j] = a[j] * cs[j] - b[j] * s;
    ob[j] = b[j] * cs[j] + a[j] * s;
  }
  *reinterpret_cast<uint4*>(base + c) = pack8(oa);
  *reinterpret_cast<uint4*>(base + half + c) = pack8(ob);
}

// out[t] = table[ids[t]]  (bf16 rows)
__global__ void embedding_fwd_kernel(const __nv_bfloat16* __restrict__ table, const int64_t* __restrict__ ids,
                                     __nv_bfloat16* __restrict__ out, int64_t T, int D, int64_t vocab) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int chunks = D / 8;
  if (i >= T * chunks) return;
  const int64_t t = i / chunks;
  const int c = (int)(i - t * chunks) * 8;
  int64_t id = ids[t];
  id = id < 0 ? 0 : (id >= vocab ? vocab - 1 : id);
  *reinterpret_cast<uint4*>(out + t * D + c) = *reinterpret_cast<const uint4*>(table + id * D + c);
}

// dtable[ids[t]] += dy[t]  (fp32 accumulation, 4-wide vector atomics)
__global__ void embedding_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const int64_t* __restrict__ ids,
                                     float* __restrict__ dtable, int64_t T, int D, int64_t vocab) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int chunks = D / 8;
  if (i >= T * chunks) return;
  const int64_t t = i / chunks;
  const int c = (int)(i - t * chunks) * 8;
  int64_t id = ids[t];
  if (id < 0 || id >= vocab) return;
  float v[8];
  unpack8(*reinterpret_cast<const uint4*>(dy + t * D + c), v);
  float4* dst = reinterpret_cast<float4*>(dtable + id * D + c);
  atomicAdd(dst, make_float4(v[0], v[1], v[2], v[3]));
  atomicAdd(dst + 1, make_float4(v[4], v[5], v[6], v[7]));
}

inline int blocks_for(int64_t n, int threads = 256) { return (int)((n + threads - 1) / threads); }
const __nv_bfloat16* bf(const at::Tensor& t) { return reinterpret_cast<const __nv_bfloat16*>(t.data_ptr()); }
__nv_bfloat16* bfm(const at::Tensor& t) { return reinterpret_cast<__nv_bfloat16*>(t.data_ptr()); }

}  // namespace

void swiglu_fwd(at::Tensor h, at::Tensor act) {
  TORCH_CHECK(h.scalar_type() == at::kBFloat16 && act.scalar_type() == at::kBFloat16, "swiglu: bf16");
  TORCH_CHECK(h.stride(-1) == 1 && act.is_contiguous(), "swiglu: contiguous last dim");
  const int64_t F = act.size(-1);
  const int64_t T = act.numel() / F;
  TORCH_CHECK(h.size(-1) == 2 * F && F % 8 == 0, "swiglu: h must be [T, 2F], F % 8 == 0");
  const int64_t ldh = h.stride(-2);
  c10::cuda::CUDAGuard g(h.device());
  const int64_t n = T * (F / 8);
  swiglu_fwd_kernel<<<blocks_for(n), 256, 0, at::cuda::getCurrentCUDAStream()>>>(bf(h), bfm(act), T, (int)F, ldh);
  AETHER_CUDA_CHECK(cudaGetLastError());
}

void swiglu_bwd(at::Tensor h, at::Tensor dact, at::Tensor dh) {
  const int64_t F = dact.size(-1);
  const int64_t T = dact.numel() / F;
  TORCH_CHECK(h.size(-1) == 2 * F && dh.size(-1) == 2 * F && dh.is_contiguous() && dact.is_contiguous(), "swiglu_bwd: shapes");
  c10::cuda::CUDAGuard g(h.device());
  const int64_t n = T * (F / 8);
  swiglu_bwd_kernel<<<blocks_for(n), 256, 0, at::cuda::getCurrentCUDAStream()>>>(bf(h), bf(dact), bfm(dh), T, (int)F,
                                                                                   h.stride(-2));
  AETHER_CUDA_CHECK(cudaGetLastError());
}

void gelu_fwd(at::Tensor x, at::Tensor y) {
  TORCH_CHECK(x.is_contiguous() && y.is_contiguous() && x.numel() % 8 == 0, "gelu: contiguous, numel % 8");
  c10::cuda::CUDAGuard g(x.device());
  const int64_t n8 = x.numel() / 8;
  gelu_fwd_kernel<<<blocks_for(n8), 256, 0, at::cuda::getCurrentCUDAStream()>>>(bf(x), bfm(y), n8);
  AETHER_CUDA_CHECK(cudaGetLastError());
}

void gelu_bwd(at::Tensor x, at::Tensor dy, at::Tensor dx) {
  TORCH_CHECK(x.is_contiguous() && dy.is_contiguous() && dx.is_contiguous() && x.numel() % 8 == 0, "gelu_bwd");
  c10::cuda::CUDAGuard g(x.device());
  const int64_t n8 = x.numel() / 8;
  gelu_bwd_kernel<<<blocks_for(n8), 256, 0, at::cuda::getCurrentCUDAStream()>>>(bf(x), bf(dy), bfm(dx), n8);
  AETHER_CUDA_CHECK(cudaGetLastError());
}

// x: [T, row_stride] (2-D view), rotates heads [0, n_heads) in place.
void rope_apply(at::Tensor x, at::Tensor pos, at::Tensor cos_t, at::Tensor sin_t, int64_t n_heads, int64_t head_dim,
                bool inverse) {
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && x.scalar_type() == at::kBFloat16, "rope: x must be 2-D bf16 rows");
  TORCH_CHECK(pos.scalar_type() == at::kInt && pos.numel() == x.size(0), "rope: pos must be int32 [T]");
  TORCH_CHECK(head_dim % 16 == 0 && n_heads * head_dim <= x.size(1), "rope: head layout");
  TORCH_CHECK(cos_t.size(1) == head_dim / 2 && cos_t.is_contiguous() && sin_t.is_contiguous(), "rope: tables");
  TORCH_CHECK(x.stride(0) % 8 == 0, "rope: row stride must be a multiple of 8");
  c10::cuda::CUDAGuard g(x.device());
  const int64_t T = x.size(0);
  const int64_t n = T * n_heads * (head_dim / 16);
  rope_kernel<<<blocks_for(n), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      bfm(x), pos.data_ptr<int>(), cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), T, (int)n_heads, (int)head_dim,
      x.stride(0), inverse ? -1.f : 1.f);
  AETHER_CUDA_CHECK(cudaGetLastError());
}

void embedding_fwd(at::Tensor table, at::Tensor ids, at::Tensor out) {
  TORCH_CHECK(table.is_contiguous() && out.is_contiguous() && ids.scalar_type() == at::kLong, "embedding_fwd");
  const int64_t D = table.size(1);
  TORCH_CHECK(D % 8 == 0, "embedding: D % 8");
  auto idc = ids.contiguous();
  const int64_t T = idc.numel();
  c10::cuda::CUDAGuard g(table.device());
  embedding_fwd_kernel<<<blocks_for(T * (D / 8)), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      bf(table), idc.data_ptr<int64_t>(), bfm(out), T, (int)D, table.size(0));
  AETHER_CUDA_CHECK(cudaGetLastError());
}

void embedding_bwd(at::Tensor dy, at::Tensor ids, at::Tensor dtable_f32) {
  TORCH_CHECK(dy.is_contiguous() && dtable_f32.is_contiguous() && dtable_f32.scalar_type() == at::kFloat, "embedding_bwd");
  const int64_t D = dtable_f32.size(1);
  auto idc = ids.contiguous();
  const int64_t T = idc.numel();
  c10::cuda::CUDAGuard g(dy.device());
  embedding_bwd_kernel<<<blocks_for(T * (D / 8)), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      bf(dy), idc.data_ptr<int64_t>(), dtable_f32.data_ptr<float>(), T, (int)D, dtable_f32.size(0));
  AETHER_CUDA_CHECK(cudaGetLastError());
}

}  // namespace aether
