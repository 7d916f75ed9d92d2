// Optimiser kernels over flat fp32 master buffers: AdamW (writing the bf16
// compute copy in the same pass), SGD, global grad-norm and clipping.
//
// Reference: adamw_step (runtime/src/cuda.rs:6924-6942), the CPU optimisers in
// runtime/src/lib.rs (aether_op_adamw_step_f32 / sgd) and clip_grads
// (trainer/src/model.rs:671-689). The update rule is the reference's decoupled
// form p -= lr * (m_hat / (sqrt(v_hat) + eps) + wd * p). Parameters live in one
// flat arena, so a whole model's update is one launch that streams
// p/g/m/v (+ the bf16 copy) at HBM rate; the gradient scale (1/world, clip
// coefficient) is read from device memory so no host sync is needed.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "host_utils.h"

namespace aether {
namespace {

struct AdamArgs {
  float lr, beta1, beta2, eps, wd, bc1_inv, bc2_inv, gscale;
};

__device__ __forceinline__ float adam_one(float& p, float g, float& m, float& v, const AdamArgs& a) {
  m = a.beta1 * m + (1.f - a.beta1) * g;
  v = a.beta2 * v + (1.f - a.beta2) * g * g;
  const float mh = m * a.bc1_inv;
  const float vh = v * a.bc2_inv;
  p -= a.lr * (mh / (sqrtf(vh) + a.eps) + a.wd * p);
  return p;
}

__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, __nv_bfloat16* __restrict__ p_bf16, int64_t n, AdamArgs a,
                             const float* __restrict__ gscale_ptr) {
  const float gs = a.gscale * (gscale_ptr ? *gscale_ptr : 1.f);
  const int64_t n4 = n / 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 pp = reinterpret_cast<float4*>(p)[i];
    const float4 gg = reinterpret_cast<const float4*>(g)[i];
    float4 mm = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    adam_one(pp.x, gg.x * gs, mm.x, vv.x, a);
    adam_one(pp.y, gg.y * gs, mm.y, vv.y, a);
    adam_one(pp.z, gg.z * gs, mm.z, vv.z, a);
    adam_one(pp.w, gg.w * gs, mm.w, vv.w, a);
    reinterpret_cast<float4*>(p)[i] = pp;
    reinterpret_cast<float4*>(m)[i] = mm;
    reinterpret_cast<float4*>(v)[i] = vv;
    if (p_bf16) {
      uint2 o;
      o.x = pack_bf16(pp.x, pp.y);
      o.y = pack_bf16(pp.z, pp.w);
      reinterpret_cast<uint2*>(p_bf16)[i] = o;
    }
  }
  // tail
  for (int64_t i = n4 * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    float pp = p[i], mm = m[i], vv = v[i];
    adam_one(pp, g[i] * gs, mm, vv, a);
    p[i] = pp;
    m[i] = mm;
    v[i] = vv;
    if (p_bf16) p_bf16[i] = __float2bfloat16(pp);
  }
}

__global__ void sgd_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ buf,
                           __nv_bfloat16* __restrict__ p_bf16, int64_t n, float lr, float momentum, float wd,
                           float gscale, const float* __restrict__ gscale_ptr) {
  const float gs = gscale * (gscale_ptr ? *gscale_ptr : 1.f);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    float gg = g[i] * gs + wd * p[i];
    if (buf) {
      const float b = momentum * buf[i] + gg;
      buf[i] = b;
      gg = b;
    }
    const float pp = p[i] - lr * gg;
    p[i] = pp;
    if (p_bf16) p_bf16[i] = __float2bfloat16(pp);
  }
}

// partial sums of squares, one per block
__global__ void sumsq_kernel(const float* __restrict__ g, int64_t n, float* __restrict__ part) {
  float s = 0.f;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t n4 = n / 4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    const float4 v = reinterpret_cast<const float4*>(g)[i];
    s += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  for (int64_t i = n4 * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) s += g[i] * g[i];
  s = warp_sum(s);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    s = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
    s = warp_sum(s);
    if (threadIdx.x == 0) part[blockIdx.x] = s;
  }
}

// norm_out[0] = sqrt(sum(part) * pre_scale^2); clip_out[0] = min(1, max_norm / (norm + 1e-6))
__global__ void finish_norm_kernel(const float* __restrict__ part, int nparts, float pre_scale, float max_norm,
                                   float* __restrict__ norm_out, float* __restrict__ clip_out) {
  float s = 0.f;
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) s += part[i];
  s = warp_sum(s);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    s = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
    s = warp_sum(s);
    if (threadIdx.x == 0) {
      const float nrm = sqrtf(s) * pre_scale;
      norm_out[0] = nrm;
      if (clip_out) clip_out[0] = max_norm > 0.f ? fminf(1.f, max_norm / (nrm + 1e-6f)) : 1.f;
    }
  }
}

int stream_grid(int64_t n) {
  const int sms = num_sms(current_device());
  const int64_t want = (n / 4 + 255) / 256;
  return (int)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)sms * 8));
}

}  // namespace

void adamw_step(at::Tensor p, at::Tensor g, at::Tensor m, at::Tensor v, std::optional<at::Tensor> p_bf16, double lr,
                double beta1, double beta2, double eps, double wd, int64_t step, double gscale,
                std::optional<at::Tensor> gscale_t) {
  TORCH_CHECK(p.is_contiguous() && g.is_contiguous() && m.is_contiguous() && v.is_contiguous(), "adamw: contiguous");
  TORCH_CHECK(p.scalar_type() == at::kFloat && g.scalar_type() == at::kFloat && m.scalar_type() == at::kFloat &&
                  v.scalar_type() == at::kFloat,
              "adamw: fp32 state");
  const int64_t n = p.numel();
  TORCH_CHECK(g.numel() == n && m.numel() == n && v.numel() == n, "adamw: sizes");
  TORCH_CHECK(step >= 1, "adamw: step counts from 1");
  c10::cuda::CUDAGuard guard(p.device());
  AdamArgs a;
  a.lr = (float)lr;
  a.beta1 = (float)beta1;
  a.beta2 = (float)beta2;
  a.eps = (float)eps;
  a.wd = (float)wd;
  a.bc1_inv = (float)(1.0 / (1.0 - std::pow(beta1, (double)step)));
  a.bc2_inv = (float)(1.0 / (1.0 - std::pow(beta2, (double)step)));
  a.gscale = (float)gscale;
  __nv_bfloat16* pb = nullptr;
  if (p_bf16 && p_bf16->defined()) {
    TORCH_CHECK(p_bf16->numel() == n && p_bf16->is_contiguous() && p_bf16->scalar_type() == at::kBFloat16, "adamw: bf16 copy");
    pb = reinterpret_cast<__nv_bfloat16*>(p_bf16->data_ptr());
  }
  if (n == 0) return;
  adamw_kernel<<<stream_grid(n), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), pb, n, a,
      (gscale_t && gscale_t->defined()) ? gscale_t->data_ptr<float>() : nullptr);
  AETHER_CUDA_CHECK(cudaGetLastError());
}

void sgd_step(at::Tensor p, at::Tensor g, std::optional<at::Tensor> buf, std::optional<at::Tensor> p_bf16, double lr,
              double momentum, double wd, double gscale, std::optional<at::Tensor> gscale_t) {
  TORCH_CHECK(p.is_contiguous() && g.is_contiguous() && p.scalar_type() == at::kFloat, "sgd: fp32 contiguous");
  const int64_t n = p.numel();
  c10::cuda::CUDAGuard guard(p.device());
  if (n == 0) return;
  sgd_kernel<<<stream_grid(n), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      p.data_ptr<float>(), g.data_ptr<float>(), (buf && buf->defined()) ? buf->data_ptr<float>() : nullptr,
      (p_bf16 && p_bf16->defined()) ? reinterpret_cast<__nv_bfloat16*>(p_bf16->data_ptr()) : nullptr, n, (float)lr,
      (float)momentum, (float)wd, (float)gscale, (gscale_t && gscale_t->defined()) ? gscale_t->data_ptr<float>() : nullptr);
  AETHER_CUDA_CHECK(cudaGetLastError());
}

// Writes ||g|| * pre_scale into norm_out[0] and the clip coefficient into clip_out[0].
void grad_norm(at::Tensor g, at::Tensor norm_out, std::optional<at::Tensor> clip_out, double pre_scale,
               double max_norm) {
  TORCH_CHECK(g.is_contiguous() && g.scalar_type() == at::kFloat, "grad_norm: fp32 contiguous");
  c10::cuda::CUDAGuard guard(g.device());
  const int64_t n = g.numel();
  const int grid = stream_grid(std::max<int64_t>(n, 1));
  auto part = at::empty({grid}, g.options());
  auto stream = at::cuda::getCurrentCUDAStream();
  sumsq_kernel<<<grid, 256, 0, stream>>>(g.data_ptr<float>(), n, part.data_ptr<float>());
  finish_norm_kernel<<<1, 1024, 0, stream>>>(part.data_ptr<float>(), grid, (float)pre_scale, (float)max_norm,
                                             norm_out.data_ptr<float>(),
                                             (clip_out && clip_out->defined()) ? clip_out->data_ptr<float>() : nullptr);
  AETHER_CUDA_CHECK(cudaGetLastError());
}

}  // namespace aether
