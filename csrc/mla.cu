// Multi-head latent attention (DeepSeek-V2 / GLM-4.7-flash) for serving, in
// the weight-absorbed form.
//
// Every token's cache row is its latent: c_kv (kv_lora_rank = 512, RMS-
// normalised) followed by the RoPE'd shared key k_pe (64) -- 576 bf16 per
// token for all heads together. Per head h the query is absorbed into the
// latent space, q_abs[h] = [q_nope[h] W_uk[h] (512), rope(q_pe[h]) (64)], so
//     S[h, t] = q_abs[h] . cache[t]          (D_qk = 576)
//     O[h]    = softmax(S[h]) cache[t, :512] (D_v = 512, the same rows)
// and the caller maps O[h] back through W_uv[h] and W_o.
//
//   mla_attention   split-K flash decoding over the latent cache: a CTA owns
//                   (query, group of 16 heads, split); the 16 heads are the M
//                   rows of warp-level m16n8k16 MMAs, so every cache row is
//                   read once per query for all heads (MQA with 16-row tiles).
//                   64-key blocks stream through a 2-stage cp.async ring; the
//                   four warps each score 16 keys, the block max goes through
//                   shared memory, P (bf16) is staged in shared memory and each
//                   warp accumulates O for 128 of the 512 latent dims. Every
//                   query carries its own length, so prefill runs the same
//                   kernel with length = position + 1 (causal).
//   mla_combine     log-sum-exp merge of the splits -> bf16 O.
//   mla_prep        per token: c_kv <- RMSNorm(kv_a[:512]) * w, k_pe <-
//                   rope(kv_a[512:]), both appended to the cache at (slot,
//                   pos), and q_abs[:, h, 512:] <- rope(q[:, h, 128:192]).
//
// Reference: paged_attention_mla_devarg, mla_split_kv_a, mla_rope_q_partial,
// mla_rope_k_shared and the mla_absorb_* kernels (runtime/src/cuda.rs:
// 1718-2670), one thread block per head on fp32 data.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "host_utils.h"

namespace aether {
namespace mla {

constexpr int kLat = 512;                 // kv_lora_rank (latent / value dims)
constexpr int kRope = 64;                 // shared RoPE key dims
constexpr int kRow = kLat + kRope;        // 576 cached dims per token
constexpr int kRowBytes = kRow * 2;       // 1152
constexpr int kChunks = kRowBytes / 16;   // 72 16-byte chunks per row
constexpr int kKeys = 64;                 // keys per block
constexpr int kHeads = 16;                // heads per CTA (MMA M)
constexpr int kStageBytes = kKeys * kRowBytes;           // 73,728
constexpr int kQBytes = kHeads * kRowBytes;              // 18,432
constexpr int kPBytes = kHeads * kKeys * 2;              // 2,048
constexpr int kSmem = 2 * kStageBytes + kQBytes + kPBytes + 1024;
constexpr float kLog2e = 1.4426950408889634f;

struct Params {
  const __nv_bfloat16* q;  // q_abs, head h of query n at n * q_rs + h * q_hs
  int64_t q_rs, q_hs;
  const __nv_bfloat16* cache;  // [slots, max_seq, 576]
  int64_t slot_stride, pos_stride;
  const int* slot;    // [N]
  const int* seqlen;  // [N] keys visible to query n
  float* part_o;      // [N, H, splits, 512]
  float* part_lse;    // [N, H, splits] (log2 domain)
  int N, H, splits, hgroups;
  float scale_log2;
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(pred ? 16 : 0) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// byte offset of 16-byte chunk c of row r in a [rows][72 chunks] tile (XOR swizzle inside groups of 8)
__device__ __forceinline__ uint32_t row_off(int r, int c) {
  return (uint32_t)(r * kRowBytes + ((c ^ (r & 7)) << 4));
}
__device__ __forceinline__ uint32_t p_off(int r, int c) {  // P tile: [16][8 chunks]
  return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4));
}

// grid (splits, N * hgroups), 128 threads.
__global__ void __launch_bounds__(128) mla_attn_kernel(Params p) {
  const int split = blockIdx.x;
  const int n = blockIdx.y / p.hgroups, hg = blockIdx.y % p.hgroups;
  const int h0 = hg * kHeads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, quad = lane & 3;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const uint32_t sKV = smem_u32(smem);
  const uint32_t sQ = sKV + 2 * kStageBytes;
  const uint32_t sP = sQ + kQBytes;
  __shared__ float red_m[4][kHeads];
  __shared__ float red_l[4][kHeads];

  const int len = p.seqlen[n];
  const int per = ((len + p.splits - 1) / p.splits + kKeys - 1) / kKeys * kKeys;
  const int k_begin = split * per;
  const int k_end = min(len, k_begin + per);
  const int nb = k_end > k_begin ? (k_end - k_begin + kKeys - 1) / kKeys : 0;
  const __nv_bfloat16* base = p.cache + (int64_t)p.slot[n] * p.slot_stride;

  auto stage_load = [&](int blk_i, int st) {
    const int blk = k_begin + blk_i * kKeys;
    const int nblk = min(kKeys, k_end - blk);
    const uint32_t dst = sKV + st * kStageBytes;
    for (int i = threadIdx.x; i < kKeys * kChunks; i += 128) {
      const int r = i / kChunks, c = i % kChunks;
      const bool ok = r < nblk;
      const __nv_bfloat16* src = base + (int64_t)(ok ? blk + r : blk) * p.pos_stride + c * 8;
      cp_async16(dst + row_off(r, c), src, ok);
    }
  };
  // Q tile (rows >= H are zero) with the first K/V block in the same group
  for (int i = threadIdx.x; i < kHeads * kChunks; i += 128) {
    const int r = i / kChunks, c = i % kChunks;
    const bool ok = h0 + r < p.H;
    const __nv_bfloat16* src = p.q + (int64_t)n * p.q_rs + (int64_t)(ok ? h0 + r : 0) * p.q_hs + c * 8;
    cp_async16(sQ + row_off(r, c), src, ok);
  }
  if (nb > 0) stage_load(0, 0);
  asm volatile("cp.async.commit_group;" ::: "memory");

  float o[16][4];
#pragma unroll
  for (int t = 0; t < 16; ++t) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};  // rows g, g + 8
  const int kw = warp * 16;
  const int mi = lane >> 3, r8 = lane & 7;

  for (int it = 0; it < nb; ++it) {
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    // block `it` (and Q) landed everywhere, and every warp is done with block
    // it - 1: its stage, P and the max exchange may be overwritten
    __syncthreads();
    if (it + 1 < nb) stage_load(it + 1, (it + 1) & 1);  // overlaps this block's math
    asm volatile("cp.async.commit_group;" ::: "memory");
    const uint32_t sK = sKV + (it & 1) * kStageBytes;
    const int blk = k_begin + it * kKeys;

    // S = Q K^T for this warp's 16 keys (two n-tiles of 8)
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll 4
    for (int kk = 0; kk < kRow / 16; ++kk) {
      uint32_t a[4], b[4];
      ldsm_x4(sQ + row_off((mi & 1) * 8 + r8, 2 * kk + (mi >> 1)), a);
      const int krow = kw + (mi >> 1) * 8 + r8;
      ldsm_x4(sK + row_off(krow, 2 * kk + (mi & 1)), b);
      mma16816(sc[0], a, b[0], b[1]);
      mma16816(sc[1], a, b[2], b[3]);
    }
    // block-wide row max
    float x[2][4];
    float wm[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = blk + kw + 8 * j + 2 * quad + (e & 1);
        const float v = key < k_end ? sc[j][e] * p.scale_log2 : -INFINITY;
        x[j][e] = v;
        wm[e >> 1] = fmaxf(wm[e >> 1], v);
      }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      wm[r] = fmaxf(wm[r], __shfl_xor_sync(0xffffffffu, wm[r], 1));
      wm[r] = fmaxf(wm[r], __shfl_xor_sync(0xffffffffu, wm[r], 2));
    }
    if (quad == 0) {
      red_m[warp][g] = wm[0];
      red_m[warp][g + 8] = wm[1];
    }
    __syncthreads();
    float alpha[2], base2[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int row = g + 8 * r;
      const float bm = fmaxf(fmaxf(red_m[0][row], red_m[1][row]), fmaxf(red_m[2][row], red_m[3][row]));
      const float mn = fmaxf(m_run[r], bm);
      base2[r] = mn == -INFINITY ? 0.f : mn;
      alpha[r] = exp2f(m_run[r] - base2[r]);
      m_run[r] = mn;
    }
    float ps[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float p0 = exp2f(x[j][0] - base2[0]), p1 = exp2f(x[j][1] - base2[0]);
      const float p2 = exp2f(x[j][2] - base2[1]), p3 = exp2f(x[j][3] - base2[1]);
      ps[0] += p0 + p1;
      ps[1] += p2 + p3;
      const int chunk = 2 * warp + j, inb = quad * 4;  // byte within the chunk
      *reinterpret_cast<uint32_t*>(smem + (sP - sKV) + p_off(g, chunk) + inb) = pack_bf16(p0, p1);
      *reinterpret_cast<uint32_t*>(smem + (sP - sKV) + p_off(g + 8, chunk) + inb) = pack_bf16(p2, p3);
    }
    l_run[0] = l_run[0] * alpha[0] + ps[0];
    l_run[1] = l_run[1] * alpha[1] + ps[1];
#pragma unroll
    for (int t = 0; t < 16; ++t) {
      o[t][0] *= alpha[0];
      o[t][1] *= alpha[0];
      o[t][2] *= alpha[1];
      o[t][3] *= alpha[1];
    }
    __syncthreads();  // P complete
    // O[:, warp's 128 dims] += P V over the block's 64 keys
#pragma unroll
    for (int kc = 0; kc < kKeys / 16; ++kc) {
      uint32_t a[4];
      ldsm_x4(sP + p_off((mi & 1) * 8 + r8, 2 * kc + (mi >> 1)), a);
      const int vrow = kc * 16 + (mi & 1) * 8 + r8;
#pragma unroll
      for (int nn = 0; nn < 8; ++nn) {
        uint32_t b[4];
        ldsm_x4_t(sK + row_off(vrow, warp * 16 + 2 * nn + (mi >> 1)), b);
        mma16816(o[2 * nn], a, b[0], b[1]);
        mma16816(o[2 * nn + 1], a, b[2], b[3]);
      }
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  // l: this thread's keys -> quad -> warps
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 1);
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 2);
  }
  __syncthreads();
  if (quad == 0) {
    red_l[warp][g] = l_run[0];
    red_l[warp][g + 8] = l_run[1];
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = g + 8 * r;
    const int h = h0 + row;
    if (h >= p.H) continue;
    const float l = red_l[0][row] + red_l[1][row] + red_l[2][row] + red_l[3][row];
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const int64_t idx = ((int64_t)n * p.H + h) * p.splits + split;
    float* po = p.part_o + idx * kLat + warp * 128;
#pragma unroll
    for (int t = 0; t < 16; ++t) {
      float2 v = make_float2(o[t][2 * r] * inv, o[t][2 * r + 1] * inv);
      *reinterpret_cast<float2*>(po + 8 * t + 2 * quad) = v;
    }
    if (warp == 0 && quad == 0) p.part_lse[idx] = l > 0.f ? m_run[r] + __log2f(l) : -INFINITY;
  }
}

// one CTA per (query, head): out[n, h, :] = sum_s w_s part_o[n, h, s, :]
__global__ void mla_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_lse,
                                   __nv_bfloat16* __restrict__ out, int64_t out_rs, int64_t out_hs, int H,
                                   int splits) {
  const int nh = blockIdx.x;
  const int n = nh / H, h = nh % H;
  const float* lse = part_lse + (int64_t)nh * splits;
  float mx = -INFINITY;
  for (int s = 0; s < splits; ++s) mx = fmaxf(mx, lse[s]);
  float tot = 0.f;
  for (int s = 0; s < splits; ++s) tot += lse[s] == -INFINITY ? 0.f : exp2f(lse[s] - mx);
  const float inv = tot > 0.f ? 1.f / tot : 0.f;
  for (int d = threadIdx.x * 4; d < kLat; d += blockDim.x * 4) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int s = 0; s < splits; ++s) {
      if (lse[s] == -INFINITY) continue;
      const float w = exp2f(lse[s] - mx) * inv;
      const float4 v = *reinterpret_cast<const float4*>(part_o + ((int64_t)nh * splits + s) * kLat + d);
      acc[0] += w * v.x;
      acc[1] += w * v.y;
      acc[2] += w * v.z;
      acc[3] += w * v.w;
    }
    uint2 u;
    u.x = pack_bf16(acc[0], acc[1]);
    u.y = pack_bf16(acc[2], acc[3]);
    *reinterpret_cast<uint2*>(out + (int64_t)n * out_rs + (int64_t)h * out_hs + d) = u;
  }
}

// one CTA (128 threads) per token
__global__ void mla_prep_kernel(const __nv_bfloat16* __restrict__ kv_a, int64_t kv_rs, const float* __restrict__ nw,
                                float eps, const __nv_bfloat16* __restrict__ q, int64_t q_rs, int H, int q_hd,
                                int nope, const int* __restrict__ pos, const int* __restrict__ slot,
                                const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                __nv_bfloat16* __restrict__ cache, int64_t slot_stride, int64_t pos_stride,
                                __nv_bfloat16* __restrict__ q_abs, int64_t qa_rs, int64_t qa_hs) {
  const int t = blockIdx.x;
  const __nv_bfloat16* a = kv_a + (int64_t)t * kv_rs;
  __nv_bfloat16* dst = cache + (int64_t)slot[t] * slot_stride + (int64_t)pos[t] * pos_stride;
  // RMSNorm of the 512-dim latent (4 per thread)
  float v[4], ss = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[i] = __bfloat162float(a[threadIdx.x * 4 + i]);
    ss += v[i] * v[i];
  }
  ss = warp_sum(ss);
  __shared__ float red[4];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  const float rs = rsqrtf((red[0] + red[1] + red[2] + red[3]) / kLat + eps);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int d = threadIdx.x * 4 + i;
    dst[d] = __float2bfloat16(v[i] * rs * nw[d]);
  }
  // RoPE (half-split pairs) of k_pe and of every head's q_pe
  const float* cs = cos_t + (int64_t)pos[t] * (kRope / 2);
  const float* sn = sin_t + (int64_t)pos[t] * (kRope / 2);
  for (int i = threadIdx.x; i < (H + 1) * (kRope / 2); i += blockDim.x) {
    const int hh = i / (kRope / 2), j = i % (kRope / 2);
    const __nv_bfloat16* src = hh == H ? a + kLat : q + (int64_t)t * q_rs + (int64_t)hh * q_hd + nope;
    const float x0 = __bfloat162float(src[j]), x1 = __bfloat162float(src[j + kRope / 2]);
    const float y0 = x0 * cs[j] - x1 * sn[j], y1 = x1 * cs[j] + x0 * sn[j];
    __nv_bfloat16* o = hh == H ? dst + kLat : q_abs + (int64_t)t * qa_rs + (int64_t)hh * qa_hs + kLat;
    o[j] = __float2bfloat16(y0);
    o[j + kRope / 2] = __float2bfloat16(y1);
  }
}

}  // namespace mla

// q_abs [N, H, 576] bf16 (rows 16-byte aligned, head stride multiple of 8);
// cache [slots, max_seq, 576]; out [N, H, 512] bf16.
void mla_attention(at::Tensor q_abs, at::Tensor cache, at::Tensor slot, at::Tensor seqlen, at::Tensor out,
                   at::Tensor part_o, at::Tensor part_lse, int64_t splits, double scale) {
  TORCH_CHECK(q_abs.scalar_type() == at::kBFloat16 && cache.scalar_type() == at::kBFloat16 &&
                  out.scalar_type() == at::kBFloat16, "mla_attention: bf16");
  TORCH_CHECK(q_abs.dim() == 3 && q_abs.size(2) == mla::kRow && q_abs.stride(2) == 1, "mla_attention: q [N, H, 576]");
  TORCH_CHECK(q_abs.stride(0) % 8 == 0 && q_abs.stride(1) % 8 == 0, "mla_attention: q strides");
  TORCH_CHECK(cache.dim() == 3 && cache.size(2) == mla::kRow && cache.stride(2) == 1 && cache.stride(1) % 8 == 0 &&
                  cache.stride(0) % 8 == 0, "mla_attention: cache [slots, max_seq, 576]");
  TORCH_CHECK(out.dim() == 3 && out.size(2) == mla::kLat && out.stride(2) == 1 && out.stride(1) % 4 == 0 &&
                  out.stride(0) % 4 == 0, "mla_attention: out [N, H, 512]");
  for (const at::Tensor* t : {&q_abs, &cache, &out})
    TORCH_CHECK((reinterpret_cast<uintptr_t>(t->data_ptr()) & 15) == 0, "mla_attention: 16-byte aligned");
  const int64_t N = q_abs.size(0), H = q_abs.size(1);
  TORCH_CHECK(slot.numel() >= N && seqlen.numel() >= N && splits >= 1, "mla_attention: sizes");
  TORCH_CHECK(part_o.numel() >= N * H * splits * mla::kLat && part_lse.numel() >= N * H * splits,
              "mla_attention: scratch");
  c10::cuda::CUDAGuard g(q_abs.device());
  if (N == 0) return;
  mla::Params p{};
  p.q = reinterpret_cast<const __nv_bfloat16*>(q_abs.data_ptr());
  p.q_rs = q_abs.stride(0);
  p.q_hs = q_abs.stride(1);
  p.cache = reinterpret_cast<const __nv_bfloat16*>(cache.data_ptr());
  p.slot_stride = cache.stride(0);
  p.pos_stride = cache.stride(1);
  p.slot = slot.data_ptr<int>();
  p.seqlen = seqlen.data_ptr<int>();
  p.part_o = part_o.data_ptr<float>();
  p.part_lse = part_lse.data_ptr<float>();
  p.N = (int)N;
  p.H = (int)H;
  p.splits = (int)splits;
  p.hgroups = (int)((H + mla::kHeads - 1) / mla::kHeads);
  p.scale_log2 = (float)scale * mla::kLog2e;
  auto stream = at::cuda::getCurrentCUDAStream();
  static bool attr_set[64] = {false};
  const int dev = current_device();
  if (!attr_set[dev]) {
    AETHER_CUDA_CHECK(cudaFuncSetAttribute(mla::mla_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, mla::kSmem));
    attr_set[dev] = true;
  }
  mla::mla_attn_kernel<<<dim3((unsigned)splits, (unsigned)(N * p.hgroups)), 128, mla::kSmem, stream>>>(p);
  AETHER_CUDA_CHECK(cudaGetLastError());
  mla::mla_combine_kernel<<<(unsigned)(N * H), 128, 0, stream>>>(p.part_o, p.part_lse,
                                                                 reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
                                                                 out.stride(0), out.stride(1), (int)H, (int)splits);
  AETHER_CUDA_CHECK(cudaGetLastError());
}

// kv_a [T, >=576] bf16; q [T, H * q_hd] bf16 with q_pe at [nope, nope + 64) of each head;
// writes cache rows and q_abs[:, :, 512:576].
void mla_prep(at::Tensor kv_a, at::Tensor norm_w, double eps, at::Tensor q, int64_t H, int64_t q_hd, int64_t nope,
              at::Tensor pos, at::Tensor slot, at::Tensor cos_t, at::Tensor sin_t, at::Tensor cache,
              at::Tensor q_abs) {
  TORCH_CHECK(kv_a.scalar_type() == at::kBFloat16 && q.scalar_type() == at::kBFloat16 &&
                  cache.scalar_type() == at::kBFloat16 && q_abs.scalar_type() == at::kBFloat16,
              "mla_prep: bf16 tensors");
  TORCH_CHECK(norm_w.scalar_type() == at::kFloat && norm_w.numel() == mla::kLat, "mla_prep: fp32 norm weight [512]");
  TORCH_CHECK(cos_t.scalar_type() == at::kFloat && cos_t.size(1) == mla::kRope / 2, "mla_prep: rope tables [S, 32]");
  TORCH_CHECK(kv_a.stride(1) == 1 && q.stride(1) == 1 && cache.stride(2) == 1 && q_abs.stride(2) == 1,
              "mla_prep: unit inner strides");
  const int64_t T = kv_a.size(0);
  c10::cuda::CUDAGuard g(kv_a.device());
  if (T == 0) return;
  mla::mla_prep_kernel<<<(unsigned)T, 128, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(kv_a.data_ptr()), kv_a.stride(0), norm_w.data_ptr<float>(), (float)eps,
      reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), q.stride(0), (int)H, (int)q_hd, (int)nope,
      pos.data_ptr<int>(), slot.data_ptr<int>(), cos_t.data_ptr<float>(), sin_t.data_ptr<float>(),
      reinterpret_cast<__nv_bfloat16*>(cache.data_ptr()), cache.stride(0), cache.stride(1),
      reinterpret_cast<__nv_bfloat16*>(q_abs.data_ptr()), q_abs.stride(0), q_abs.stride(1));
  AETHER_CUDA_CHECK(cudaGetLastError());
}

}  // namespace aether
