// KV-cache kernels for serving: RoPE + KV append, and split-K flash-decoding.
//
// Reference: rope_apply_devarg + append_kv_devarg / paged_append_kv_devarg
// (runtime/src/cuda.rs:3034, 5339-5360, 1126) and the split-K decode attention
// paged_attention_seq1_v4_split_devarg + _v4_combine (cuda.rs:1546-1717): each
// split keeps (max, sum, V-accumulator) and a log-sum-exp merge combines them.
// Here:
//   * one kernel rotates q/k in place for every new token, and writes the
//     rotated k and the v rows straight into the cache at (slot, position) --
//     positions and slots are read from device memory so a captured CUDA
//     graph replays the same kernels for any step;
//   * a decode CTA owns one (sequence, KV head, split) and serves all query
//     heads of that KV head's GQA group, so each K/V row is read once per
//     group instead of once per query head;
//   * the per-sequence lengths come from device memory, the split count is a
//     launch constant, and empty splits emit lse = -inf.
// Cache layout per layer: K and V as [slots, max_seq, Hkv, D] bf16.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "host_utils.h"

namespace aether {
namespace dec {

constexpr float kLog2e = 1.4426950408889634f;
constexpr int kMaxGroup = 8;

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

// qkv: [T, row] with q heads [0,Hq), k heads [Hq, Hq+Hkv), v heads after.
// One thread per (token, head, 8-wide chunk of the half head).
__global__ void rope_kv_append_kernel(__nv_bfloat16* __restrict__ qkv, int64_t row, const int* __restrict__ pos,
                                      const int* __restrict__ slot, const float* __restrict__ cos_t,
                                      const float* __restrict__ sin_t, __nv_bfloat16* __restrict__ kc,
                                      __nv_bfloat16* __restrict__ vc, int64_t T, int Hq, int Hkv, int D,
                                      int64_t slot_stride, int64_t pos_stride) {
  const int half = D / 2, chunks = half / 8;
  const int H = Hq + 2 * Hkv;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= T * H * chunks) return;
  const int c = (int)(i % chunks) * 8;
  const int h = (int)((i / chunks) % H);
  const int64_t t = i / ((int64_t)chunks * H);
  const int p = pos[t];
  __nv_bfloat16* base = qkv + t * row + (int64_t)h * D;
  float a[8], b[8];
  unpack8(*reinterpret_cast<const uint4*>(base + c), a);
  unpack8(*reinterpret_cast<const uint4*>(base + half + c), b);
  if (h < Hq + Hkv) {
    const float4* cp = reinterpret_cast<const float4*>(cos_t + (int64_t)p * half + c);
    const float4* sp = reinterpret_cast<const float4*>(sin_t + (int64_t)p * half + c);
    const float4 c0 = cp[0], c1 = cp[1], s0 = sp[0], s1 = sp[1];
    const float cs[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    const float sn[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float x1 = a[j], x2 = b[j];
      a[j] = x1 * cs[j] - x2 * sn[j];
      b[j] = x2 * cs[j] + x1 * sn[j];
    }
  }
  const uint4 ua = pack8(a), ub = pack8(b);
  if (h < Hq) {
    *reinterpret_cast<uint4*>(base + c) = ua;
    *reinterpret_cast<uint4*>(base + half + c) = ub;
    return;
  }
  const int s = slot[t];
  const bool is_k = h < Hq + Hkv;
  const int hk = is_k ? h - Hq : h - Hq - Hkv;
  __nv_bfloat16* dst = (is_k ? kc : vc) + (int64_t)s * slot_stride + (int64_t)p * pos_stride + (int64_t)hk * D;
  *reinterpret_cast<uint4*>(dst + c) = ua;
  *reinterpret_cast<uint4*>(dst + half + c) = ub;
  if (is_k) {  // keep the rotated k in qkv too (prefill attention reads it there)
    *reinterpret_cast<uint4*>(base + c) = ua;
    *reinterpret_cast<uint4*>(base + half + c) = ub;
  }
}

struct DecParams {
  const __nv_bfloat16* q;  // [B, q_rs] with head h at h*D
  int64_t q_rs;
  const __nv_bfloat16* kc;
  const __nv_bfloat16* vc;
  int64_t slot_stride, pos_stride;  // elements
  const int* slot;                  // [B]
  const int* seqlen;                // [B] number of valid keys
  float* part_o;                    // [B, Hq, splits, D]
  float* part_lse;                  // [B, Hq, splits]
  int Hq, Hkv, splits;
  float scale_log2;
};

// grid (splits, B * Hkv), 128 threads. D == 128.
__global__ void __launch_bounds__(128) decode_attn_kernel(DecParams p) {
  constexpr int D = 128;
  const int split = blockIdx.x;
  const int b = blockIdx.y / p.Hkv, hk = blockIdx.y % p.Hkv;
  const int G = p.Hq / p.Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ float sq[kMaxGroup][D];
  __shared__ float sp[4][kMaxGroup][32];
  __shared__ float sm_m[4][kMaxGroup], sm_l[4][kMaxGroup];
  __shared__ float so[4][kMaxGroup][D];

  const int len = p.seqlen[b];
  const int per = ((len + p.splits - 1) / p.splits + 127) / 128 * 128;
  const int k_begin = split * per;
  const int k_end = min(len, k_begin + per);

  for (int i = threadIdx.x; i < G * D; i += 128) {
    const int g = i / D, d = i % D;
    sq[g][d] = __bfloat162float(p.q[(int64_t)b * p.q_rs + (int64_t)(hk * G + g) * D + d]) * p.scale_log2;
  }
  __syncthreads();

  const int s = p.slot[b];
  const __nv_bfloat16* kbase = p.kc + (int64_t)s * p.slot_stride + (int64_t)hk * D;
  const __nv_bfloat16* vbase = p.vc + (int64_t)s * p.slot_stride + (int64_t)hk * D;
  float m[kMaxGroup], l[kMaxGroup], o[kMaxGroup][4];
#pragma unroll
  for (int g = 0; g < kMaxGroup; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
    o[g][0] = o[g][1] = o[g][2] = o[g][3] = 0.f;
  }
  for (int kb = k_begin + warp * 32; kb < k_end; kb += 128) {
    const int key = kb + lane;
    float sc[kMaxGroup];
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g) sc[g] = 0.f;
    if (key < k_end) {
      const uint4* kr = reinterpret_cast<const uint4*>(kbase + (int64_t)key * p.pos_stride);
#pragma unroll 4
      for (int c = 0; c < D / 8; ++c) {
        float kv[8];
        unpack8(kr[c], kv);
#pragma unroll
        for (int g = 0; g < kMaxGroup; ++g) {
          if (g < G) {
#pragma unroll
            for (int j = 0; j < 8; ++j) sc[g] += sq[g][c * 8 + j] * kv[j];
          }
        }
      }
    } else {
#pragma unroll
      for (int g = 0; g < kMaxGroup; ++g) sc[g] = -INFINITY;
    }
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g) {
      if (g < G) {
        const float bm = warp_max(sc[g]);
        const float mn = fmaxf(m[g], bm);
        const float alpha = exp2f(m[g] - mn);  // m = -inf on the first block -> 0
        const float pe = key < k_end ? exp2f(sc[g] - mn) : 0.f;
        l[g] = l[g] * alpha + warp_sum(pe);
        m[g] = mn;
        o[g][0] *= alpha; o[g][1] *= alpha; o[g][2] *= alpha; o[g][3] *= alpha;
        sp[warp][g][lane] = pe;
      }
    }
    __syncwarp();
    const int nkeys = min(32, k_end - kb);
    for (int j = 0; j < nkeys; ++j) {
      const uint2 vv = *reinterpret_cast<const uint2*>(vbase + (int64_t)(kb + j) * p.pos_stride + lane * 4);
      const float v0 = bf16lo(vv.x), v1 = bf16hi(vv.x), v2 = bf16lo(vv.y), v3 = bf16hi(vv.y);
#pragma unroll
      for (int g = 0; g < kMaxGroup; ++g) {
        if (g < G) {
          const float pj = sp[warp][g][j];
          o[g][0] += pj * v0; o[g][1] += pj * v1; o[g][2] += pj * v2; o[g][3] += pj * v3;
        }
      }
    }
    __syncwarp();
  }
  // merge the 4 warps
#pragma unroll
  for (int g = 0; g < kMaxGroup; ++g) {
    if (g < G) {
      if (lane == 0) {
        sm_m[warp][g] = m[g];
        sm_l[warp][g] = l[g];
      }
      so[warp][g][lane * 4 + 0] = o[g][0];
      so[warp][g][lane * 4 + 1] = o[g][1];
      so[warp][g][lane * 4 + 2] = o[g][2];
      so[warp][g][lane * 4 + 3] = o[g][3];
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * D; i += 128) {
    const int g = i / D, d = i % D;
    float mm = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) mm = fmaxf(mm, sm_m[w][g]);
    float ll = 0.f, acc = 0.f;
    if (mm != -INFINITY) {
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float f = exp2f(sm_m[w][g] - mm);
        ll += sm_l[w][g] * f;
        acc += so[w][g][d] * f;
      }
    }
    const int hq = hk * G + g;
    const int64_t idx = ((int64_t)b * p.Hq + hq) * p.splits + split;
    p.part_o[idx * D + d] = ll > 0.f ? acc / ll : 0.f;
    if (d == 0) p.part_lse[idx] = ll > 0.f ? mm + __log2f(ll) : -INFINITY;  // log2 domain
  }
}

// out[b, h*D + d] = sum_s w_s * part_o[b,h,s,d], w_s = 2^(lse_s - lse)
__global__ void decode_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_lse,
                                      __nv_bfloat16* __restrict__ out, int64_t out_rs, int Hq, int splits, int D) {
  const int bh = blockIdx.x;
  const int b = bh / Hq, h = bh % Hq;
  const float* lse = part_lse + (int64_t)bh * splits;
  float mx = -INFINITY;
  for (int s = 0; s < splits; ++s) mx = fmaxf(mx, lse[s]);
  float tot = 0.f;
  for (int s = 0; s < splits; ++s) tot += (lse[s] == -INFINITY) ? 0.f : exp2f(lse[s] - mx);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < splits; ++s) {
      if (lse[s] != -INFINITY) acc += exp2f(lse[s] - mx) * part_o[((int64_t)bh * splits + s) * D + d];
    }
    out[(int64_t)b * out_rs + (int64_t)h * D + d] = __float2bfloat16(tot > 0.f ? acc / tot : 0.f);
  }
}

}  // namespace dec

// qkv [T, row] bf16 (rotated in place), pos/slot int32 [T], cos/sin [max_pos, D/2],
// k_cache/v_cache [slots, max_seq, Hkv, D].
void rope_kv_append(at::Tensor qkv, at::Tensor pos, at::Tensor slot, at::Tensor cos_t, at::Tensor sin_t,
                    at::Tensor k_cache, at::Tensor v_cache, int64_t Hq, int64_t Hkv, int64_t D) {
  TORCH_CHECK(qkv.dim() == 2 && qkv.stride(1) == 1 && qkv.scalar_type() == at::kBFloat16, "rope_kv_append: qkv");
  TORCH_CHECK(qkv.size(1) >= (Hq + 2 * Hkv) * D && qkv.stride(0) % 8 == 0, "rope_kv_append: qkv row");
  TORCH_CHECK(pos.scalar_type() == at::kInt && slot.scalar_type() == at::kInt, "rope_kv_append: int32 pos/slot");
  TORCH_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous() && k_cache.dim() == 4 && k_cache.size(2) == Hkv &&
                  k_cache.size(3) == D,
              "rope_kv_append: cache [slots, max_seq, Hkv, D]");
  TORCH_CHECK(D % 16 == 0, "rope_kv_append: head_dim % 16");
  c10::cuda::CUDAGuard g(qkv.device());
  const int64_t T = qkv.size(0);
  if (T == 0) return;
  const int64_t n = T * (Hq + 2 * Hkv) * (D / 16);
  dec::rope_kv_append_kernel<<<(unsigned)((n + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(qkv.data_ptr()), qkv.stride(0), pos.data_ptr<int>(), slot.data_ptr<int>(),
      cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(k_cache.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(v_cache.data_ptr()), T, (int)Hq, (int)Hkv, (int)D, k_cache.stride(0),
      k_cache.stride(1));
  AETHER_CUDA_CHECK(cudaGetLastError());
}

// q: [B, q_rs] (head h at h*D); out: [B, out_rs]; part buffers sized [B*Hq*splits*(D+1)].
void decode_attention(at::Tensor q, at::Tensor k_cache, at::Tensor v_cache, at::Tensor slot, at::Tensor seqlen,
                      at::Tensor out, at::Tensor part_o, at::Tensor part_lse, int64_t Hq, int64_t splits,
                      double scale) {
  const int64_t B = q.size(0);
  const int64_t Hkv = k_cache.size(2), D = k_cache.size(3);
  TORCH_CHECK(D == 128, "decode_attention: head_dim 128");
  TORCH_CHECK(Hq % Hkv == 0 && Hq / Hkv <= dec::kMaxGroup, "decode_attention: GQA group must be <= 8");
  TORCH_CHECK(q.stride(1) == 1 && out.stride(1) == 1, "decode_attention: rows");
  TORCH_CHECK(part_o.numel() >= B * Hq * splits * D && part_lse.numel() >= B * Hq * splits, "decode_attention: scratch");
  c10::cuda::CUDAGuard g(q.device());
  if (B == 0) return;
  dec::DecParams p{};
  p.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  p.q_rs = q.stride(0);
  p.kc = reinterpret_cast<const __nv_bfloat16*>(k_cache.data_ptr());
  p.vc = reinterpret_cast<const __nv_bfloat16*>(v_cache.data_ptr());
  p.slot_stride = k_cache.stride(0);
  p.pos_stride = k_cache.stride(1);
  p.slot = slot.data_ptr<int>();
  p.seqlen = seqlen.data_ptr<int>();
  p.part_o = part_o.data_ptr<float>();
  p.part_lse = part_lse.data_ptr<float>();
  p.Hq = (int)Hq;
  p.Hkv = (int)Hkv;
  p.splits = (int)splits;
  p.scale_log2 = (float)scale * dec::kLog2e;
  auto stream = at::cuda::getCurrentCUDAStream();
  dec::decode_attn_kernel<<<dim3((unsigned)splits, (unsigned)(B * Hkv)), 128, 0, stream>>>(p);
  AETHER_CUDA_CHECK(cudaGetLastError());
  dec::decode_combine_kernel<<<(unsigned)(B * Hq), 128, 0, stream>>>(
      p.part_o, p.part_lse, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0), (int)Hq, (int)splits,
      (int)D);
  AETHER_CUDA_CHECK(cudaGetLastError());
}

}  // namespace aether
