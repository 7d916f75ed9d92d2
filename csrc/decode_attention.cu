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
#include "decode_common.cuh"
#include "host_utils.h"

namespace aether {
PeerWait make_peer_wait(const std::optional<at::Tensor>& my_sig, const std::optional<at::Tensor>& epoch, int64_t rank,
                        int64_t world, double timeout_s);
namespace dec {

constexpr float kLog2e = 1.4426950408889634f;
constexpr int kMaxGroup = 8;
constexpr int kMaxSplits = 64;
constexpr int kKeysPerBlock = 64;                      // keys per pipeline stage
constexpr int kStages = 3;
constexpr int kStageBytes = 2 * kKeysPerBlock * 256;   // K and V rows of one block
constexpr int kKvSmem = kStages * kStageBytes;         // 96 KB

// qkv: [T, row] with q heads [0,Hq), k heads [Hq, Hq+Hkv), v heads after.
// One thread per (token, head, 8-wide chunk of the half head).
__global__ void rope_kv_append_kernel(__nv_bfloat16* __restrict__ qkv, int64_t row, const int* __restrict__ pos,
                                      const int* __restrict__ slot, const float* __restrict__ cos_t,
                                      const float* __restrict__ sin_t, __nv_bfloat16* __restrict__ kc,
                                      __nv_bfloat16* __restrict__ vc, int64_t T, int Hq, int Hkv, int D,
                                      int64_t slot_stride, int64_t pos_stride, PageMap pm) {
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
  __nv_bfloat16* dst = (is_k ? kc : vc) + kv_offset(pm, s, p, slot_stride, pos_stride) + (int64_t)hk * D;
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
  int* counters;                    // [B * Hkv] zero-initialised; the last split CTA merges
  __nv_bfloat16* out;               // [B, out_rs]
  int64_t out_rs;
  int Hq, Hkv, splits;
  float scale_log2;
  PageMap pm;  // table == nullptr: contiguous per-slot caches
  // flex attention: window > 0 keeps the last `window` keys; cap_in > 0 soft-caps
  // the logits, s' = cap * tanh(s * scale / cap) (cap_in = scale / cap, cap_out = cap * log2 e)
  int window;
  float cap_in, cap_out;
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
// c += a(16x16, rows 8..15 zero) * b(16x8)
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}

// grid (splits, B * Hkv), 128 threads, D == 128.
// A CTA owns one (sequence, KV head, split). The G <= 8 query heads of the KV
// head's GQA group are the M rows of warp-level tensor-core MMAs (m16n8k16,
// rows G..15 zero), so every K/V row is read once for the whole group:
//   S = Q K^T over 64-key blocks (each warp takes 16 keys of the block),
//   online softmax in registers, O += P V with P re-packed from the S
//   accumulators straight into the A operand.
// K/V blocks stream through a 3-stage cp.async ring (16-byte chunks
// XOR-swizzled by row for conflict-free ldmatrix); the four warps' partial
// (max, sum, O) are merged through shared memory at the end.
__global__ void __launch_bounds__(128) decode_attn_kernel(DecParams p) {
  constexpr int D = 128;
  asm volatile("griddepcontrol.launch_dependents;");
  const int split = blockIdx.x;
  const int b = blockIdx.y / p.Hkv, hk = blockIdx.y % p.Hkv;
  const int G = p.Hq / p.Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = lane >> 2;        // query head of this thread's accumulator rows
  const int quad = lane & 3;
  extern __shared__ __align__(128) uint8_t kv_smem[];  // kStages x (K block, V block), 64 rows x 256 B each
  const uint32_t sbase = smem_u32(kv_smem);

  const int len = p.seqlen[b];
  const int lo = p.window > 0 ? max(0, len - p.window) : 0;  // sliding window: keys [lo, len)
  const int span = len - lo;
  const int per = ((span + p.splits - 1) / p.splits + kKeysPerBlock - 1) / kKeysPerBlock * kKeysPerBlock;
  const int k_begin = lo + split * per;
  const int k_end = min(len, k_begin + per);
  const int nb = k_end > k_begin ? (k_end - k_begin + kKeysPerBlock - 1) / kKeysPerBlock : 0;
  const int s = p.slot[b];
  const __nv_bfloat16* kbase = p.kc + (int64_t)hk * D;
  const __nv_bfloat16* vbase = p.vc + (int64_t)hk * D;

  auto stage_load = [&](int blk_i, int st) {
    const int blk = k_begin + blk_i * kKeysPerBlock;
    const int nblk = min(kKeysPerBlock, k_end - blk);
    const uint32_t sK = sbase + st * kStageBytes, sV = sK + kKeysPerBlock * 256;
    for (int i = threadIdx.x; i < kKeysPerBlock * 16; i += 128) {
      const int r = i >> 4, c = i & 15;
      const bool ok = r < nblk;
      const int64_t ro = kv_offset(p.pm, s, ok ? blk + r : blk, p.slot_stride, p.pos_stride);
      const uint32_t off = (uint32_t)(r * 256 + ((c ^ (r & 7)) << 4));
      cp_async16(sK + off, kbase + ro + c * 8, ok);
      cp_async16(sV + off, vbase + ro + c * 8, ok);
    }
  };
#pragma unroll
  for (int st = 0; st < kStages - 1; ++st) {
    if (st < nb) stage_load(st, st);
    asm volatile("cp.async.commit_group;" ::: "memory");
  }

  // Q as A fragments (rows = heads of the group, pre-scaled into the log2 domain)
  uint32_t qa[8][2];
  {
    const bool ok = row < G;
    const __nv_bfloat16* qr = p.q + (int64_t)b * p.q_rs + (int64_t)(hk * G + (ok ? row : 0)) * D;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int d0 = kk * 16 + quad * 2;
      const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(qr + d0));
      const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(qr + d0 + 8));
      qa[kk][0] = ok ? pack_bf16(lo.x, lo.y) : 0u;
      qa[kk][1] = ok ? pack_bf16(hi.x, hi.y) : 0u;
    }
  }
  float o[16][4];
#pragma unroll
  for (int t = 0; t < 16; ++t) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;
  const int kw = warp * 16;  // this warp's keys within a block

  for (int it = 0; it < nb; ++it) {
    asm volatile("cp.async.wait_group %0;" ::"n"(kStages - 2) : "memory");
    __syncthreads();  // block `it` landed everywhere; stage (it-1) % kStages is free again
    if (it + kStages - 1 < nb) stage_load(it + kStages - 1, (it + kStages - 1) % kStages);
    asm volatile("cp.async.commit_group;" ::: "memory");
    const uint32_t sK = sbase + (it % kStages) * kStageBytes, sV = sK + kKeysPerBlock * 256;
    const int blk = k_begin + it * kKeysPerBlock;

    // S (16 x 16 keys) = Q K^T
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    {
      const int mi = lane >> 3, r8 = lane & 7;
      const int krow = kw + (mi >> 1) * 8 + r8;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int c = 2 * kk + (mi & 1);
        uint32_t bq[4];
        ldsm_x4(sK + (uint32_t)(krow * 256 + ((c ^ (krow & 7)) << 4)), bq);
        mma16816(sc[0], qa[kk][0], qa[kk][1], bq[0], bq[1]);
        mma16816(sc[1], qa[kk][0], qa[kk][1], bq[2], bq[3]);
      }
    }
    // online softmax on this thread's row (keys kw + 8j + 2*quad + e)
    float x[4];
    float bm = -INFINITY;
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = blk + kw + 8 * j + 2 * quad + e;
        const float sv = p.cap_in > 0.f ? p.cap_out * tanh_sfu(sc[j][e] * p.cap_in) : sc[j][e] * p.scale_log2;
        const float v = key < k_end ? sv : -INFINITY;
        x[j * 2 + e] = v;
        bm = fmaxf(bm, v);
      }
    bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 1));
    bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 2));
    const float mn = fmaxf(m_run, bm);
    const float base = mn == -INFINITY ? 0.f : mn;
    const float alpha = exp2f(m_run - base);
    float pe[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) pe[i] = exp2f(x[i] - base);
    l_run = l_run * alpha + (pe[0] + pe[1] + pe[2] + pe[3]);
    m_run = mn;
#pragma unroll
    for (int t = 0; t < 16; ++t) {
      o[t][0] *= alpha;
      o[t][1] *= alpha;
    }
    // O += P V (k = this warp's 16 keys)
    const uint32_t pa0 = pack_bf16(pe[0], pe[1]), pa2 = pack_bf16(pe[2], pe[3]);
    {
      const int mi = lane >> 3, r8 = lane & 7;
      const int vrow = kw + (mi & 1) * 8 + r8;
#pragma unroll
      for (int nn = 0; nn < 8; ++nn) {
        const int c = 2 * nn + (mi >> 1);
        uint32_t bv[4];
        ldsm_x4_t(sV + (uint32_t)(vrow * 256 + ((c ^ (vrow & 7)) << 4)), bv);
        mma16816(o[2 * nn], pa0, pa2, bv[0], bv[1]);
        mma16816(o[2 * nn + 1], pa0, pa2, bv[2], bv[3]);
      }
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
  __syncthreads();  // every warp is done with the ring; reuse it for the merge
  // merge the 4 warps (rows >= G are padding)
  float* sm_m = reinterpret_cast<float*>(kv_smem);        // [4][8]
  float* sm_l = sm_m + 32;                                // [4][8]
  float* so = sm_m + 64;                                  // [4][8][D]
  if (quad == 0) {
    sm_m[warp * 8 + row] = m_run;
    sm_l[warp * 8 + row] = l_run;
  }
#pragma unroll
  for (int t = 0; t < 16; ++t) {
    so[(warp * 8 + row) * D + 8 * t + 2 * quad] = o[t][0];
    so[(warp * 8 + row) * D + 8 * t + 2 * quad + 1] = o[t][1];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * D; i += 128) {
    const int g = i / D, d = i % D;
    float mm = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) mm = fmaxf(mm, sm_m[w * 8 + g]);
    float ll = 0.f, acc = 0.f;
    if (mm != -INFINITY) {
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float f = exp2f(sm_m[w * 8 + g] - mm);
        ll += sm_l[w * 8 + g] * f;
        acc += so[(w * 8 + g) * D + d] * f;
      }
    }
    const int hq = hk * G + g;
    const int64_t idx = ((int64_t)b * p.Hq + hq) * p.splits + split;
    p.part_o[idx * D + d] = ll > 0.f ? acc / ll : 0.f;
    if (d == 0) p.part_lse[idx] = ll > 0.f ? mm + __log2f(ll) : -INFINITY;  // log2 domain
  }
  if (p.counters == nullptr) return;
  // The last split CTA of this (sequence, KV head) merges all splits.
  __threadfence();
  __syncthreads();
  __shared__ int s_last;
  if (threadIdx.x == 0) s_last = atomicAdd(p.counters + blockIdx.y, 1) == p.splits - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // Only the splits that own keys take part: split s covers [s * per, ...),
  // so the first ceil(len / per) are non-empty.
  const int n_act = per > 0 ? min(p.splits, (span + per - 1) / per) : 0;
  // Per-split merge weights for every head of the group, computed once.
  __shared__ float s_w[kMaxGroup][kMaxSplits];
  for (int i = threadIdx.x; i < G * n_act; i += 128) {
    const int g = i / n_act, s2 = i % n_act;
    s_w[g][s2] = __ldcg(p.part_lse + ((int64_t)b * p.Hq + hk * G + g) * p.splits + s2);
  }
  __syncthreads();
  if (threadIdx.x < G) {
    const int g = threadIdx.x;
    float mx = -INFINITY;
    for (int s2 = 0; s2 < n_act; ++s2) mx = fmaxf(mx, s_w[g][s2]);
    float tot = 0.f;
    for (int s2 = 0; s2 < n_act; ++s2) {
      const float w = s_w[g][s2] == -INFINITY ? 0.f : exp2f(s_w[g][s2] - mx);
      s_w[g][s2] = w;
      tot += w;
    }
    const float inv = tot > 0.f ? 1.f / tot : 0.f;
    for (int s2 = 0; s2 < n_act; ++s2) s_w[g][s2] *= inv;
  }
  __syncthreads();
  // out = sum_s w_s * part_o[s]: float4 loads, four splits in flight per step
  constexpr int D4 = D / 4;
  for (int i = threadIdx.x; i < G * D4; i += 128) {
    const int g = i / D4, d4 = i % D4;
    const int hq = hk * G + g;
    const float4* po = reinterpret_cast<const float4*>(p.part_o + (((int64_t)b * p.Hq + hq) * p.splits) * D) + d4;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    int s2 = 0;
    for (; s2 + 4 <= n_act; s2 += 4) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = __ldcg(po + (int64_t)(s2 + u) * D4);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float w = s_w[g][s2 + u];
        a0 += w * v[u].x; a1 += w * v[u].y; a2 += w * v[u].z; a3 += w * v[u].w;
      }
    }
    for (; s2 < n_act; ++s2) {
      const float4 v = __ldcg(po + (int64_t)s2 * D4);
      const float w = s_w[g][s2];
      a0 += w * v.x; a1 += w * v.y; a2 += w * v.z; a3 += w * v.w;
    }
    uint2 packed;
    packed.x = pack_bf16(a0, a1);
    packed.y = pack_bf16(a2, a3);
    *reinterpret_cast<uint2*>(p.out + (int64_t)b * p.out_rs + (int64_t)hq * D + d4 * 4) = packed;
  }
  if (threadIdx.x == 0) p.counters[blockIdx.y] = 0;  // ready for the next step (graph replay)
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

// Decode QKV finalisation: qkv = acc + bias, RoPE on q/k at pos, q (and k)
// written to the bf16 qkv rows, k/v appended to the cache; acc re-zeroed.
// One thread per (row, head, 8-wide chunk of the half head).
__global__ void qkv_finalize_rope_kernel(float* __restrict__ acc, int64_t ldacc, const __nv_bfloat16* __restrict__ bias,
                                         __nv_bfloat16* __restrict__ qkv, int64_t row, const int* __restrict__ pos,
                                         const int* __restrict__ slot, const float* __restrict__ cos_t,
                                         const float* __restrict__ sin_t, __nv_bfloat16* __restrict__ kc,
                                         __nv_bfloat16* __restrict__ vc, int B, int Hq, int Hkv, int D,
                                         int64_t slot_stride, int64_t pos_stride, PageMap pm) {
  asm volatile("griddepcontrol.launch_dependents;");
  const int half = D / 2, chunks = half / 8;
  const int H = Hq + 2 * Hkv;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)B * H * chunks) return;
  const int c = (int)(i % chunks) * 8;
  const int h = (int)((i / chunks) % H);
  const int b = (int)(i / ((int64_t)chunks * H));
  float* ar = acc + (int64_t)b * ldacc + (int64_t)h * D;
  float a[8], bb[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    a[j] = ar[c + j];
    bb[j] = ar[half + c + j];
    ar[c + j] = 0.f;
    ar[half + c + j] = 0.f;
  }
  if (bias) {
    const __nv_bfloat16* br = bias + (int64_t)h * D;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      a[j] += __bfloat162float(br[c + j]);
      bb[j] += __bfloat162float(br[half + c + j]);
    }
  }
  // round to bf16 first (the values the prefill path stores), then rotate
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    a[j] = __bfloat162float(__float2bfloat16(a[j]));
    bb[j] = __bfloat162float(__float2bfloat16(bb[j]));
  }
  const int p_ = pos[b];
  if (h < Hq + Hkv) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float cs = cos_t[(int64_t)p_ * half + c + j], sn = sin_t[(int64_t)p_ * half + c + j];
      const float x1 = a[j], x2 = bb[j];
      a[j] = x1 * cs - x2 * sn;
      bb[j] = x2 * cs + x1 * sn;
    }
  }
  const uint4 ua = pack8(a), ub = pack8(bb);
  __nv_bfloat16* qr = qkv + (int64_t)b * row + (int64_t)h * D;
  *reinterpret_cast<uint4*>(qr + c) = ua;
  *reinterpret_cast<uint4*>(qr + half + c) = ub;
  if (h >= Hq) {
    const bool is_k = h < Hq + Hkv;
    const int hk = is_k ? h - Hq : h - Hq - Hkv;
    __nv_bfloat16* dst = (is_k ? kc : vc) + kv_offset(pm, slot[b], p_, slot_stride, pos_stride) + (int64_t)hk * D;
    *reinterpret_cast<uint4*>(dst + c) = ua;
    *reinterpret_cast<uint4*>(dst + half + c) = ub;
  }
}

// y = bf16(acc + bias + res) (the residual stream), h = rmsnorm(y) * w; acc
// re-zeroed. One CTA per row.
__global__ void __launch_bounds__(1024) finalize_residual_norm_kernel(float* __restrict__ acc, int64_t ldacc, int N,
                                                                     const __nv_bfloat16* __restrict__ bias,
                                                                     const __nv_bfloat16* __restrict__ res,
                                                                     __nv_bfloat16* __restrict__ y,
                                                                     const __nv_bfloat16* __restrict__ w,
                                                                     __nv_bfloat16* __restrict__ h, float eps,
                                                                     PeerWait wait) {
  asm volatile("griddepcontrol.launch_dependents;");
  peer_wait(wait);  // tensor parallel: every rank's reductions into acc have landed
  constexpr int kMaxPer = 8;  // N <= 1024 * 8 = 8192
  const int r = blockIdx.x;
  float* ar = acc + (int64_t)r * ldacc;
  float v[kMaxPer];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kMaxPer; ++k) {
    const int c = threadIdx.x + k * 1024;
    v[k] = 0.f;
    if (c < N) {
      float x = ar[c];
      ar[c] = 0.f;
      if (bias) x += __bfloat162float(bias[c]);
      if (res) x += __bfloat162float(res[(int64_t)r * N + c]);
      const __nv_bfloat16 xb = __float2bfloat16(x);
      y[(int64_t)r * N + c] = xb;
      v[k] = __bfloat162float(xb);
      ss += v[k] * v[k];
    }
  }
  ss = warp_sum(ss);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int k = 0; k < 32; ++k) tot += red[k];
  const float rstd = rsqrtf(tot / N + eps);
#pragma unroll
  for (int k = 0; k < kMaxPer; ++k) {
    const int c = threadIdx.x + k * 1024;
    if (c < N) h[(int64_t)r * N + c] = __float2bfloat16(v[k] * rstd * __bfloat162float(w[c]));
  }
}

}  // namespace dec

dec::PageMap page_map(const std::optional<at::Tensor>& page_table, const at::Tensor& cache) {
  dec::PageMap pm;
  if (!page_table || !page_table->defined()) return pm;
  TORCH_CHECK(page_table->is_cuda() && page_table->scalar_type() == at::kInt && page_table->dim() == 2 &&
                  page_table->stride(1) == 1,
              "page_table: CUDA int32 [rows, max_pages] with unit inner stride");
  const int64_t P = cache.size(1);
  TORCH_CHECK(P > 0 && (P & (P - 1)) == 0, "paged cache: page size must be a power of two");
  pm.table = page_table->data_ptr<int>();
  pm.stride = (int)page_table->stride(0);
  int shift = 0;
  while ((int64_t(1) << shift) < P) ++shift;
  pm.shift = shift;
  return pm;
}

// qkv [T, row] bf16 (rotated in place), pos/slot int32 [T], cos/sin [max_pos, D/2],
// k_cache/v_cache [slots, max_seq, Hkv, D] (or page pools with page_table).
void rope_kv_append(at::Tensor qkv, at::Tensor pos, at::Tensor slot, at::Tensor cos_t, at::Tensor sin_t,
                    at::Tensor k_cache, at::Tensor v_cache, int64_t Hq, int64_t Hkv, int64_t D,
                    std::optional<at::Tensor> page_table) {
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
      k_cache.stride(1), page_map(page_table, k_cache));
  AETHER_CUDA_CHECK(cudaGetLastError());
}

// q: [B, q_rs] (head h at h*D); out: [B, out_rs]; part buffers sized [B*Hq*splits*(D+1)].
void decode_attention(at::Tensor q, at::Tensor k_cache, at::Tensor v_cache, at::Tensor slot, at::Tensor seqlen,
                      at::Tensor out, at::Tensor part_o, at::Tensor part_lse, int64_t Hq, int64_t splits,
                      double scale, std::optional<at::Tensor> counters, std::optional<at::Tensor> page_table,
                      int64_t window, double softcap) {
  const int64_t B = q.size(0);
  const int64_t Hkv = k_cache.size(2), D = k_cache.size(3);
  TORCH_CHECK(D == 128, "decode_attention: head_dim 128");
  TORCH_CHECK(Hq % Hkv == 0 && Hq / Hkv <= dec::kMaxGroup, "decode_attention: GQA group must be <= 8");
  TORCH_CHECK(q.stride(1) == 1 && out.stride(1) == 1, "decode_attention: rows");
  TORCH_CHECK(out.stride(0) % 4 == 0 && reinterpret_cast<uintptr_t>(out.data_ptr()) % 8 == 0,
              "decode_attention: out rows must start on 8-byte boundaries");
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
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.out_rs = out.stride(0);
  p.pm = page_map(page_table, k_cache);
  p.window = (int)window;
  if (softcap > 0.0) {
    p.cap_in = (float)(scale / softcap);
    p.cap_out = (float)softcap * dec::kLog2e;
  }
  auto stream = at::cuda::getCurrentCUDAStream();
  static bool attr_set[64] = {false};
  const int dev = current_device();
  if (!attr_set[dev]) {
    AETHER_CUDA_CHECK(cudaFuncSetAttribute(dec::decode_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dec::kKvSmem));
    attr_set[dev] = true;
  }
  if (counters && counters->defined()) {
    TORCH_CHECK(counters->scalar_type() == at::kInt && counters->numel() >= B * Hkv, "decode_attention: counters");
    TORCH_CHECK(splits <= dec::kMaxSplits, "decode_attention: at most 64 splits with the fused combine");
    p.counters = counters->data_ptr<int>();
    dec::decode_attn_kernel<<<dim3((unsigned)splits, (unsigned)(B * Hkv)), 128, dec::kKvSmem, stream>>>(p);
    AETHER_CUDA_CHECK(cudaGetLastError());
    return;
  }
  dec::decode_attn_kernel<<<dim3((unsigned)splits, (unsigned)(B * Hkv)), 128, dec::kKvSmem, stream>>>(p);
  AETHER_CUDA_CHECK(cudaGetLastError());
  dec::decode_combine_kernel<<<(unsigned)(B * Hq), 128, 0, stream>>>(
      p.part_o, p.part_lse, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0), (int)Hq, (int)splits,
      (int)D);
  AETHER_CUDA_CHECK(cudaGetLastError());
}

}  // namespace aether

namespace aether {

// Decode QKV epilogue: qkv rows = rope(acc + bias); k/v appended to the caches; acc zeroed.
void qkv_finalize_rope(at::Tensor acc, std::optional<at::Tensor> bias, at::Tensor qkv, at::Tensor pos, at::Tensor slot,
                       at::Tensor cos_t, at::Tensor sin_t, at::Tensor k_cache, at::Tensor v_cache, int64_t Hq,
                       int64_t Hkv, int64_t D, std::optional<at::Tensor> page_table) {
  const int64_t B = qkv.size(0);
  TORCH_CHECK(acc.scalar_type() == at::kFloat && acc.size(1) >= (Hq + 2 * Hkv) * D, "qkv_finalize_rope: acc");
  TORCH_CHECK(qkv.stride(1) == 1 && qkv.stride(0) % 8 == 0 && D % 16 == 0, "qkv_finalize_rope: qkv layout");
  TORCH_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous(), "qkv_finalize_rope: caches");
  c10::cuda::CUDAGuard g(acc.device());
  const int64_t n = B * (Hq + 2 * Hkv) * (D / 16);
  if (n == 0) return;
  dec::qkv_finalize_rope_kernel<<<(unsigned)((n + 127) / 128), 128, 0, at::cuda::getCurrentCUDAStream()>>>(
      acc.data_ptr<float>(), acc.stride(0),
      (bias && bias->defined()) ? reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr()) : nullptr,
      reinterpret_cast<__nv_bfloat16*>(qkv.data_ptr()), qkv.stride(0), pos.data_ptr<int>(), slot.data_ptr<int>(),
      cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(k_cache.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(v_cache.data_ptr()), (int)B, (int)Hq, (int)Hkv, (int)D, k_cache.stride(0),
      k_cache.stride(1), page_map(page_table, k_cache));
  AETHER_CUDA_CHECK(cudaGetLastError());
}

// y = bf16(acc + bias + res); h = rmsnorm(y) * w; acc zeroed. y/h/res: [B, N] contiguous.
void finalize_residual_norm(at::Tensor acc, std::optional<at::Tensor> bias, std::optional<at::Tensor> res,
                            at::Tensor y, at::Tensor w, at::Tensor h, double eps,
                            std::optional<at::Tensor> wait_sig, std::optional<at::Tensor> wait_epoch,
                            int64_t wait_rank, int64_t wait_world, double wait_timeout_s) {
  const int64_t B = y.size(0), N = y.size(1);
  TORCH_CHECK(N <= 8192 && y.is_contiguous() && h.is_contiguous(), "finalize_residual_norm: rows up to 8192, contiguous");
  TORCH_CHECK(acc.scalar_type() == at::kFloat && acc.size(1) >= N, "finalize_residual_norm: acc");
  c10::cuda::CUDAGuard g(acc.device());
  if (B == 0) return;
  dec::finalize_residual_norm_kernel<<<(unsigned)B, 1024, 0, at::cuda::getCurrentCUDAStream()>>>(
      acc.data_ptr<float>(), acc.stride(0), (int)N,
      (bias && bias->defined()) ? reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr()) : nullptr,
      (res && res->defined()) ? reinterpret_cast<const __nv_bfloat16*>(res->data_ptr()) : nullptr,
      reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(h.data_ptr()), (float)eps,
      make_peer_wait(wait_sig, wait_epoch, wait_rank, wait_world, wait_timeout_s));
  AETHER_CUDA_CHECK(cudaGetLastError());
}

}  // namespace aether

// ---------------------------------------------------------------------------
// Allocation-free variant of decode_attention (fused combine). Declared, with
// its rules and limits, in aether_noalloc.h. It has no counterpart in the
// reference. Same kernel as above; only where the scratch comes from differs.
#include <atomic>
#include <mutex>

#include "aether_noalloc.h"

namespace aether {
namespace noalloc {

constexpr int kMaxRows = AETHER_NOALLOC_MAX_PARTIAL_ROWS;
constexpr int kMaxCounters = AETHER_NOALLOC_MAX_COUNTERS;
constexpr int kMaxDevices = 64;

// One scratch block per device: split partial outputs [rows, 128] fp32, their
// log-sum-exps [rows] fp32, and the last-CTA counters [kMaxCounters] int32
// (must be zero before a launch; every launch leaves them zero again).
static __device__ __align__(256) float g_part_o[kMaxRows * 128];
static __device__ __align__(256) float g_part_lse[kMaxRows];
static __device__ __align__(256) int g_counters[kMaxCounters];

struct DeviceScratch {
  float* part_o = nullptr;
  float* part_lse = nullptr;
  int* counters = nullptr;
};
static DeviceScratch g_dev[kMaxDevices];
static std::atomic<bool> g_ready[kMaxDevices];  // set (release) after g_dev[dev] is filled in
static std::mutex g_setup_mu;

// Set-up of one device, run with that device current. A device is marked
// ready only when every step succeeded, so a failed set-up (for example a
// memset refused during another stream's global-mode capture) is retried by
// the next call instead of failing every later call.
static int setup(int dev) {
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (g_ready[dev].load(std::memory_order_acquire)) return AETHER_NOALLOC_OK;
  DeviceScratch s;
  if (cudaGetSymbolAddress(reinterpret_cast<void**>(&s.part_o), g_part_o) != cudaSuccess ||
      cudaGetSymbolAddress(reinterpret_cast<void**>(&s.part_lse), g_part_lse) != cudaSuccess ||
      cudaGetSymbolAddress(reinterpret_cast<void**>(&s.counters), g_counters) != cudaSuccess ||
      cudaFuncSetAttribute(dec::decode_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dec::kKvSmem) !=
          cudaSuccess ||
      cudaMemset(s.counters, 0, sizeof(int) * kMaxCounters) != cudaSuccess ||
      cudaDeviceSynchronize() != cudaSuccess) {
    cudaGetLastError();  // clear the failed call's error so the caller's next CUDA call does not see it
    return AETHER_NOALLOC_ECUDA;
  }
  g_dev[dev] = s;
  g_ready[dev].store(true, std::memory_order_release);
  return AETHER_NOALLOC_OK;
}

}  // namespace noalloc
}  // namespace aether

extern "C" __attribute__((visibility("default"))) int aether_decode_attention_noalloc(
    const void* q, int64_t q_rs, const void* k_cache, const void* v_cache, int64_t slot_stride, int64_t pos_stride,
    const int* slot, const int* seqlen, void* out, int64_t out_rs, int B, int Hq, int Hkv, int D, int splits,
    float scale, void* stream) {
  using namespace aether;
  if (!q || !k_cache || !v_cache || !slot || !seqlen || !out) return AETHER_NOALLOC_EINVAL;
  // The kernel reads K/V rows with 16-byte copies and q with 4-byte loads, and
  // writes out with 8-byte stores: a misaligned base or stride would be a GPU
  // fault (which ends the context), so it is an argument error here.
  if (out_rs % 4 != 0 || reinterpret_cast<uintptr_t>(out) % 8 != 0) return AETHER_NOALLOC_EINVAL;
  if (reinterpret_cast<uintptr_t>(k_cache) % 16 != 0 || reinterpret_cast<uintptr_t>(v_cache) % 16 != 0 ||
      slot_stride % 8 != 0 || pos_stride % 8 != 0 || slot_stride < 0 || pos_stride < 0)
    return AETHER_NOALLOC_EINVAL;
  if (reinterpret_cast<uintptr_t>(q) % 4 != 0 || q_rs % 2 != 0 || q_rs < 0) return AETHER_NOALLOC_EINVAL;
  if (B < 0 || D != 128 || Hkv <= 0 || Hq <= 0 || Hq % Hkv != 0 || Hq / Hkv > dec::kMaxGroup || splits < 1 ||
      splits > dec::kMaxSplits)
    return AETHER_NOALLOC_EINVAL;
  if ((int64_t)B * Hq * splits > noalloc::kMaxRows || (int64_t)B * Hkv > noalloc::kMaxCounters)
    return AETHER_NOALLOC_ETOOBIG;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= noalloc::kMaxDevices) return AETHER_NOALLOC_ECUDA;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (st != nullptr && st != cudaStreamLegacy && st != cudaStreamPerThread) {
    int sdev = -1;  // the scratch address belongs to the current device: the stream must be on it too
    if (cudaStreamGetDevice(st, &sdev) != cudaSuccess) {
      cudaGetLastError();
      return AETHER_NOALLOC_EINVAL;
    }
    if (sdev != dev) return AETHER_NOALLOC_EINVAL;
  }
  if (!noalloc::g_ready[dev].load(std::memory_order_acquire)) {
    const int rc = noalloc::setup(dev);
    if (rc != AETHER_NOALLOC_OK) return rc;
  }
  const noalloc::DeviceScratch& s = noalloc::g_dev[dev];
  if (B == 0) return AETHER_NOALLOC_OK;
  dec::DecParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.q_rs = q_rs;
  p.kc = static_cast<const __nv_bfloat16*>(k_cache);
  p.vc = static_cast<const __nv_bfloat16*>(v_cache);
  p.slot_stride = slot_stride;
  p.pos_stride = pos_stride;
  p.slot = slot;
  p.seqlen = seqlen;
  p.part_o = s.part_o;
  p.part_lse = s.part_lse;
  p.counters = s.counters;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_rs = out_rs;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.splits = splits;
  p.scale_log2 = scale * dec::kLog2e;
  // cudaLaunchKernelEx reports this launch's own error (cudaGetLastError
  // would also return, and clear, an unrelated earlier error of the thread).
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)splits, (unsigned)(B * Hkv));
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = dec::kKvSmem;
  cfg.stream = st;
  return cudaLaunchKernelEx(&cfg, dec::decode_attn_kernel, p) == cudaSuccess ? AETHER_NOALLOC_OK
                                                                               : AETHER_NOALLOC_ECUDA;
}
