// Mixture-of-experts routing kernels around the grouped tcgen05 GEMM.
//
//   moe_route    router logits [T, E] -> top-k experts and weights per token
//                (softmax over all experts, then top-k, optionally renormalised
//                -- Qwen-MoE / DeepSeek-V2 style -- or softmax over the top-k
//                logits only -- Mixtral style -- or per-expert sigmoid scores,
//                optionally renormalised -- DeepSeek-V3 / GLM-4.7-flash
//                style); weights times a routed scaling factor; one warp per
//                token.
//   moe_permute  counting sort of the T*k (token, expert) pairs by expert into
//                expert segments that start on 128-row boundaries, so every
//                128-row GEMM tile belongs to one expert: writes the row of
//                each pair, the source token of each permuted row (-1 for
//                padding) and the expert of each 128-row tile (-1: unused).
//                With an expert range [e0, e0 + E) (expert parallelism: this
//                GPU holds E of the experts) pairs routed elsewhere get row -1.
//                One CTA; everything stays on the device (CUDA-graph safe).
//   moe_gather   permuted activations X[r] = x[src_row[r]] (zero rows for padding)
//   moe_combine  out[t] = sum_j w[t, j] * Y[row_of[t, j]] (+ residual); rows -1 skipped
//
// Reference: the MoE fields of the serving ModelConfig and the host-side top-k
// routing (runtime/src/serving.rs:2335, 459-900) with one expert GEMV per
// (token, expert) (`fused_*_expert_matmul_seq1`, runtime/src/cuda.rs:5666-6135).
// Here the experts' work is two grouped GEMMs over tokens sorted by expert.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "host_utils.h"

namespace aether {
namespace moe {

constexpr int kMaxExperts = 256;
constexpr int kMaxTopK = 16;
constexpr int kTile = 128;

__global__ void route_kernel(const float* __restrict__ logits, int64_t ld, int T, int E, int k, bool softmax_all,
                             bool renorm, bool sigmoid, float scale, int* __restrict__ idx, float* __restrict__ wt) {
  const int t = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  constexpr int PER = kMaxExperts / 32;
  float v[PER];
  const float* row = logits + (int64_t)t * ld;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = i * 32 + lane;
    v[i] = e < E ? row[e] : -INFINITY;
  }
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < PER; ++i) mx = fmaxf(mx, v[i]);
  mx = warp_max(mx);
  float denom = 1.f;
  if (sigmoid) {
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (v[i] != -INFINITY) v[i] = 1.f / (1.f + __expf(-v[i]));
  } else if (softmax_all) {
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      v[i] = v[i] == -INFINITY ? 0.f : __expf(v[i] - mx);
      sum += v[i];
    }
    denom = warp_sum(sum);
#pragma unroll
    for (int i = 0; i < PER; ++i) v[i] /= denom;
  }
  // k rounds of warp argmax; the winner is removed (ties -> lowest expert id)
  float sel_v[kMaxTopK];
  int sel_e[kMaxTopK];
  for (int j = 0; j < k; ++j) {
    float best = -INFINITY;
    int be = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = i * 32 + lane;
      if (e < E && (v[i] > best || (v[i] == best && e < be))) {
        best = v[i];
        be = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float b2 = __shfl_xor_sync(0xffffffffu, best, o);
      const int e2 = __shfl_xor_sync(0xffffffffu, be, o);
      if (b2 > best || (b2 == best && e2 < be)) {
        best = b2;
        be = e2;
      }
    }
    sel_v[j] = best;
    sel_e[j] = be;
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (i * 32 + lane == be) v[i] = -INFINITY;
  }
  if (lane == 0) {
    float w[kMaxTopK];
    float tot = 0.f;
    if (softmax_all || sigmoid) {
      for (int j = 0; j < k; ++j) {
        w[j] = sel_v[j];
        tot += w[j];
      }
      const float s = renorm && tot > 0.f ? 1.f / tot : 1.f;
      for (int j = 0; j < k; ++j) w[j] *= s;
    } else {  // softmax over the selected logits
      for (int j = 0; j < k; ++j) {
        w[j] = __expf(sel_v[j] - sel_v[0]);
        tot += w[j];
      }
      for (int j = 0; j < k; ++j) w[j] /= tot;
    }
    for (int j = 0; j < k; ++j) {
      idx[(int64_t)t * k + j] = sel_e[j];
      wt[(int64_t)t * k + j] = w[j] * scale;
    }
  }
}

// One CTA of 1024 threads.
__global__ void __launch_bounds__(1024) permute_kernel(const int* __restrict__ idx, int TK, int E, int e0, int Mpad,
                                                       int* __restrict__ row_of, int* __restrict__ src_row,
                                                       int* __restrict__ tile_group, int k) {
  __shared__ int cnt[kMaxExperts];
  __shared__ int off[kMaxExperts + 1];
  __shared__ int cur[kMaxExperts];
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    cnt[e] = 0;
    cur[e] = 0;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < TK; i += blockDim.x) {
    const int e = idx[i] - e0;
    if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int o = 0;
    for (int e = 0; e < E; ++e) {
      off[e] = o;
      o += (cnt[e] + kTile - 1) / kTile * kTile;
    }
    off[E] = o;
  }
  __syncthreads();
  const int used = off[E];
  for (int r = threadIdx.x; r < Mpad; r += blockDim.x) src_row[r] = -1;
  for (int tt = threadIdx.x; tt < Mpad / kTile; tt += blockDim.x) {
    const int r0 = tt * kTile;
    int g = -1;
    if (r0 < used) {
      // expert whose segment holds row r0 (segments are contiguous, E small)
      int lo = 0, hi = E - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (off[mid] <= r0) lo = mid;
        else hi = mid - 1;
      }
      g = lo;
    }
    tile_group[tt] = g;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < TK; i += blockDim.x) {
    const int e = idx[i] - e0;
    if (e < 0 || e >= E) {  // routed to an expert on another GPU
      row_of[i] = -1;
      continue;
    }
    const int r = off[e] + atomicAdd(&cur[e], 1);
    row_of[i] = r;
    src_row[r] = i / k;
  }
}

// 8 bf16 per thread; d % 8 == 0
__global__ void gather_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, const int* __restrict__ src_row,
                              __nv_bfloat16* __restrict__ X, int Mpad, int d) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int per_row = d / 8;
  if (i >= (int64_t)Mpad * per_row) return;
  const int r = (int)(i / per_row), c = (int)(i % per_row) * 8;
  const int s = src_row[r];
  uint4 v = make_uint4(0, 0, 0, 0);
  if (s >= 0) v = *reinterpret_cast<const uint4*>(x + (int64_t)s * ldx + c);
  *reinterpret_cast<uint4*>(X + (int64_t)r * d + c) = v;
}

__global__ void combine_kernel(const __nv_bfloat16* __restrict__ Y, int64_t ldy, const int* __restrict__ row_of,
                               const float* __restrict__ wt, int k, const __nv_bfloat16* __restrict__ res,
                               const __nv_bfloat16* __restrict__ extra, __nv_bfloat16* __restrict__ out, int T,
                               int d) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int per_row = d / 8;
  if (i >= (int64_t)T * per_row) return;
  const int t = (int)(i / per_row), c = (int)(i % per_row) * 8;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int j = 0; j < k; ++j) {
    const int r = row_of[(int64_t)t * k + j];
    if (r < 0) continue;
    const float w = wt[(int64_t)t * k + j];
    const uint4 u = *reinterpret_cast<const uint4*>(Y + (int64_t)r * ldy + c);
    acc[0] += w * bf16lo(u.x); acc[1] += w * bf16hi(u.x); acc[2] += w * bf16lo(u.y); acc[3] += w * bf16hi(u.y);
    acc[4] += w * bf16lo(u.z); acc[5] += w * bf16hi(u.z); acc[6] += w * bf16lo(u.w); acc[7] += w * bf16hi(u.w);
  }
  const __nv_bfloat16* adds[2] = {res, extra};
#pragma unroll
  for (int a = 0; a < 2; ++a) {
    if (adds[a] == nullptr) continue;
    const uint4 u = *reinterpret_cast<const uint4*>(adds[a] + (int64_t)t * d + c);
    acc[0] += bf16lo(u.x); acc[1] += bf16hi(u.x); acc[2] += bf16lo(u.y); acc[3] += bf16hi(u.y);
    acc[4] += bf16lo(u.z); acc[5] += bf16hi(u.z); acc[6] += bf16lo(u.w); acc[7] += bf16hi(u.w);
  }
  uint4 o;
  o.x = pack_bf16(acc[0], acc[1]);
  o.y = pack_bf16(acc[2], acc[3]);
  o.z = pack_bf16(acc[4], acc[5]);
  o.w = pack_bf16(acc[6], acc[7]);
  *reinterpret_cast<uint4*>(out + (int64_t)t * d + c) = o;
}

}  // namespace moe

void moe_route(at::Tensor logits, at::Tensor idx, at::Tensor wt, int64_t k, bool softmax_all, bool renorm,
               bool sigmoid, double scale) {
  TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == at::kFloat && logits.dim() == 2 && logits.stride(1) == 1,
              "moe_route: fp32 [T, E] logits (rows may be strided)");
  const int T = (int)logits.size(0), E = (int)logits.size(1);
  TORCH_CHECK(E <= moe::kMaxExperts && k >= 1 && k <= moe::kMaxTopK && k <= E, "moe_route: E <= 256, 1 <= k <= 16");
  TORCH_CHECK(idx.scalar_type() == at::kInt && wt.scalar_type() == at::kFloat && idx.numel() == (int64_t)T * k &&
                  wt.numel() == (int64_t)T * k,
              "moe_route: outputs [T, k]");
  c10::cuda::CUDAGuard g(logits.device());
  if (T == 0) return;
  moe::route_kernel<<<(T + 3) / 4, 128, 0, at::cuda::getCurrentCUDAStream()>>>(
      logits.data_ptr<float>(), logits.stride(0), T, E, (int)k, softmax_all, renorm, sigmoid, (float)scale,
      idx.data_ptr<int>(),
      wt.data_ptr<float>());
  AETHER_CUDA_CHECK(cudaGetLastError());
}

void moe_permute(at::Tensor idx, int64_t E, at::Tensor row_of, at::Tensor src_row, at::Tensor tile_group,
                 int64_t e0) {
  TORCH_CHECK(idx.is_cuda() && idx.scalar_type() == at::kInt && idx.dim() == 2, "moe_permute: int32 [T, k] experts");
  const int TK = (int)idx.numel(), k = (int)idx.size(1);
  const int Mpad = (int)src_row.numel();
  TORCH_CHECK(E <= moe::kMaxExperts && Mpad % moe::kTile == 0 && Mpad >= TK + E * (moe::kTile - 1),
              "moe_permute: src_row must hold T*k + E*127 rows rounded up to 128");
  TORCH_CHECK(row_of.numel() == TK && tile_group.numel() >= Mpad / moe::kTile, "moe_permute: output sizes");
  c10::cuda::CUDAGuard g(idx.device());
  moe::permute_kernel<<<1, 1024, 0, at::cuda::getCurrentCUDAStream()>>>(
      idx.data_ptr<int>(), TK, (int)E, (int)e0, Mpad, row_of.data_ptr<int>(), src_row.data_ptr<int>(),
      tile_group.data_ptr<int>(), k);
  AETHER_CUDA_CHECK(cudaGetLastError());
}

void moe_gather(at::Tensor x, at::Tensor src_row, at::Tensor X) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && X.scalar_type() == at::kBFloat16 && x.stride(1) == 1 &&
                  X.is_contiguous() && x.size(1) % 8 == 0 && x.stride(0) % 8 == 0,
              "moe_gather: bf16 rows, d % 8 == 0");
  const int Mpad = (int)X.size(0), d = (int)X.size(1);
  c10::cuda::CUDAGuard g(x.device());
  const int64_t n = (int64_t)Mpad * (d / 8);
  if (n == 0) return;
  moe::gather_kernel<<<(unsigned)((n + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0), src_row.data_ptr<int>(),
      reinterpret_cast<__nv_bfloat16*>(X.data_ptr()), Mpad, d);
  AETHER_CUDA_CHECK(cudaGetLastError());
}

void moe_combine(at::Tensor Y, at::Tensor row_of, at::Tensor wt, int64_t k, std::optional<at::Tensor> res,
                 std::optional<at::Tensor> extra, at::Tensor out) {
  TORCH_CHECK(Y.scalar_type() == at::kBFloat16 && Y.stride(1) == 1 && Y.stride(0) % 8 == 0 && out.is_contiguous(),
              "moe_combine: layouts");
  const int T = (int)out.size(0), d = (int)out.size(1);
  TORCH_CHECK(d % 8 == 0 && row_of.numel() == (int64_t)T * k && wt.numel() == (int64_t)T * k, "moe_combine: sizes");
  for (auto* t : {&res, &extra})
    if (*t && (*t)->defined())
      TORCH_CHECK((*t)->is_contiguous() && (*t)->size(0) == T && (*t)->size(1) == d, "moe_combine: addend [T, d]");
  c10::cuda::CUDAGuard g(Y.device());
  const int64_t n = (int64_t)T * (d / 8);
  if (n == 0) return;
  moe::combine_kernel<<<(unsigned)((n + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(Y.data_ptr()), Y.stride(0), row_of.data_ptr<int>(), wt.data_ptr<float>(),
      (int)k, (res && res->defined()) ? reinterpret_cast<const __nv_bfloat16*>(res->data_ptr()) : nullptr,
      (extra && extra->defined()) ? reinterpret_cast<const __nv_bfloat16*>(extra->data_ptr()) : nullptr,
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), T, d);
  AETHER_CUDA_CHECK(cudaGetLastError());
}

}  // namespace aether
