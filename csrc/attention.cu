// Flash-style scaled-dot-product attention, forward and backward, bf16 in /
// fp32 accumulate, O(S) memory (only the per-row log-sum-exp is saved).
//
// Reference: sdpa_causal_fwd / sdpa_causal_bwd_dq / sdpa_causal_bwd_dkv
// (runtime/src/cuda.rs:6736-6854) materialise the [B*H, S, S] probability and
// d_scores tensors with one thread per query row, and gqa_repeat_kv /
// gqa_reduce_kv_grad (cuda.rs:3062-3110) copy K/V per query head. Here:
//   * forward: a CTA owns 128 query rows of one head, streams 64-key K/V tiles
//     through a double-buffered cp.async ring, keeps S/P in registers and the
//     running (max, sum) online-softmax state per row;
//   * backward: a CTA owns 64 keys of one KV head, loops over every query head
//     of its GQA group and every query tile, accumulates dK/dV in registers and
//     adds dQ with fp32 atomics (converted to bf16 by a small epilogue kernel);
//   * GQA is native (kv_head = q_head / group) -- no K/V copies;
//   * `causal_offset` lets query i see keys <= i + offset (prefill on top of a
//     KV cache);
//   * flex attention (forward and backward): `window` > 0 also hides keys < i + offset -
//     window + 1 (sliding window), `softcap` > 0 maps the scaled logits
//     through cap * tanh(s / cap).
// Tiles live in shared memory with a 16-byte-chunk XOR swizzle so every
// ldmatrix is conflict-free. Matrix products use mma.sync m16n8k16 bf16.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "host_utils.h"

namespace aether {
namespace attn {

constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(pred ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Byte offset of 16-byte chunk `c` of row `r` in a swizzled tile whose rows are
// ROWB bytes (ROWB >= 128).
template <int ROWB>
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return (uint32_t)(r * ROWB + ((c ^ (r & 7)) << 4));
}

// Copies rows [row0, row0 + R) x D columns of a strided bf16 matrix into a
// swizzled tile; rows >= nvalid are zero-filled.
template <int R, int D, int NT>
__device__ __forceinline__ void load_tile(uint32_t sbase, const __nv_bfloat16* g, int64_t ld, int row0, int nvalid) {
  constexpr int CH = D / 8;
#pragma unroll
  for (int i = threadIdx.x; i < R * CH; i += NT) {
    const int r = i / CH, c = i % CH;
    const bool ok = row0 + r < nvalid;
    const __nv_bfloat16* src = g + (int64_t)(ok ? row0 + r : 0) * ld + c * 8;
    cp_async16(sbase + swz<D * 2>(r, c), src, ok);
  }
}

struct FwdParams {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  __nv_bfloat16* o;
  float* lse;  // [B, Hq, Sq] natural-log LSE (may be null)
  int64_t q_bs, q_rs, k_bs, k_rs, v_bs, v_rs, o_bs, o_rs;
  int B, Hq, Hkv, Sq, Sk;
  float scale_log2;  // softmax scale * log2(e)
  int causal;
  int causal_offset;
  int window;            // > 0: sliding window (forward only)
  float cap_in, cap_out;  // softcap > 0: scale / cap and cap * log2(e) (forward only)
};

// ============================================================== forward
template <int D>
__global__ void __launch_bounds__(256, 1) attn_fwd_kernel(FwdParams p) {
  constexpr int BR = 128, BC = 64, NT = 256;
  constexpr int ROWB = D * 2;
  constexpr int KC = D / 16;  // k-chunks over head dim
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK0 = sQ + BR * ROWB;
  const uint32_t sV0 = sK0 + 2 * BC * ROWB;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int qb = gridDim.x - 1 - blockIdx.x;  // longest causal rows first
  const int bh = blockIdx.y;
  const int b = bh / p.Hq, h = bh % p.Hq;
  const int hk = h / (p.Hq / p.Hkv);
  const __nv_bfloat16* qg = p.q + b * p.q_bs + (int64_t)h * D;
  const __nv_bfloat16* kg = p.k + b * p.k_bs + (int64_t)hk * D;
  const __nv_bfloat16* vg = p.v + b * p.v_bs + (int64_t)hk * D;
  const int q0 = qb * BR;

  int kv_end = p.Sk;
  if (p.causal) kv_end = min(p.Sk, q0 + BR + p.causal_offset);
  const int n_kv = kv_end > 0 ? (kv_end + BC - 1) / BC : 0;

  load_tile<BR, D, NT>(sQ, qg, p.q_rs, q0, p.Sq);
  if (n_kv > 0) {
    load_tile<BC, D, NT>(sK0, kg, p.k_rs, 0, p.Sk);
    load_tile<BC, D, NT>(sV0, vg, p.v_rs, 0, p.Sk);
  }
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();

  // Q fragments for this warp's 16 rows stay in registers.
  uint32_t qf[KC][4];
  {
    const int mi = lane >> 3;
    const int r = warp * 16 + (mi & 1) * 8 + (lane & 7);
#pragma unroll
    for (int kc = 0; kc < KC; ++kc)
      ldsm_x4(sQ + swz<ROWB>(r, 2 * kc + (mi >> 1)), qf[kc][0], qf[kc][1], qf[kc][2], qf[kc][3]);
  }

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const int row0 = q0 + warp * 16 + g;  // this thread's rows: row0, row0 + 8

  for (int j = 0; j < n_kv; ++j) {
    const int st = j & 1;
    if (j + 1 < n_kv) {
      load_tile<BC, D, NT>(sK0 + (st ^ 1) * BC * ROWB, kg, p.k_rs, (j + 1) * BC, p.Sk);
      load_tile<BC, D, NT>(sV0 + (st ^ 1) * BC * ROWB, vg, p.v_rs, (j + 1) * BC, p.Sk);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint32_t sK = sK0 + st * BC * ROWB;
    const uint32_t sV = sV0 + st * BC * ROWB;

    float s[BC / 8][4];
#pragma unroll
    for (int i = 0; i < BC / 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
    {
      const int mi = lane >> 3;
#pragma unroll
      for (int kc = 0; kc < KC; ++kc) {
#pragma unroll
        for (int np = 0; np < BC / 16; ++np) {
          uint32_t b0, b1, b2, b3;
          const int key = np * 16 + (mi >> 1) * 8 + (lane & 7);
          ldsm_x4(sK + swz<ROWB>(key, 2 * kc + (mi & 1)), b0, b1, b2, b3);
          mma16816(s[2 * np], qf[kc], b0, b1);
          mma16816(s[2 * np + 1], qf[kc], b2, b3);
        }
      }
    }
    // scale + mask
    const int key0 = j * BC;
    const bool need_mask = (key0 + BC > p.Sk) || (p.causal && key0 + BC - 1 > q0 + warp * 16 + p.causal_offset) ||
                           (p.window > 0 && key0 < q0 + warp * 16 + 15 + p.causal_offset - p.window + 1);
#pragma unroll
    for (int nt = 0; nt < BC / 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float x = p.cap_in > 0.f ? p.cap_out * tanh_sfu(s[nt][e] * p.cap_in) : s[nt][e] * p.scale_log2;
        if (need_mask) {
          const int col = key0 + nt * 8 + 2 * t + (e & 1);
          const int row = row0 + (e >> 1) * 8;
          if (col >= p.Sk || (p.causal && col > row + p.causal_offset) ||
              (p.window > 0 && col < row + p.causal_offset - p.window + 1))
            x = -INFINITY;
        }
        s[nt][e] = x;
      }
    }
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < BC / 8; ++nt) {
      mx0 = fmaxf(mx0, fmaxf(s[nt][0], s[nt][1]));
      mx1 = fmaxf(mx1, fmaxf(s[nt][2], s[nt][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float base0 = mn0 == -INFINITY ? 0.f : mn0;
    const float base1 = mn1 == -INFINITY ? 0.f : mn1;
    const float al0 = exp2f(m0 - base0), al1 = exp2f(m1 - base1);
    m0 = mn0;
    m1 = mn1;
    float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
    for (int nt = 0; nt < BC / 8; ++nt) {
      s[nt][0] = exp2f(s[nt][0] - base0);
      s[nt][1] = exp2f(s[nt][1] - base0);
      s[nt][2] = exp2f(s[nt][2] - base1);
      s[nt][3] = exp2f(s[nt][3] - base1);
      rs0 += s[nt][0] + s[nt][1];
      rs1 += s[nt][2] + s[nt][3];
    }
    l0 = l0 * al0 + rs0;
    l1 = l1 * al1 + rs1;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      o[i][0] *= al0;
      o[i][1] *= al0;
      o[i][2] *= al1;
      o[i][3] *= al1;
    }
    // O += P V
    {
      const int mi = lane >> 3;
#pragma unroll
      for (int kc2 = 0; kc2 < BC / 16; ++kc2) {
        uint32_t pa[4];
        pa[0] = pack_bf16(s[2 * kc2][0], s[2 * kc2][1]);
        pa[1] = pack_bf16(s[2 * kc2][2], s[2 * kc2][3]);
        pa[2] = pack_bf16(s[2 * kc2 + 1][0], s[2 * kc2 + 1][1]);
        pa[3] = pack_bf16(s[2 * kc2 + 1][2], s[2 * kc2 + 1][3]);
        const int key = kc2 * 16 + (mi & 1) * 8 + (lane & 7);
#pragma unroll
        for (int dp = 0; dp < D / 16; ++dp) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(sV + swz<ROWB>(key, 2 * dp + (mi >> 1)), b0, b1, b2, b3);
          mma16816(o[2 * dp], pa, b0, b1);
          mma16816(o[2 * dp + 1], pa, b2, b3);
        }
      }
    }
    __syncthreads();
  }

  // finalise
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f;
  const float inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
  // stage the warp's 16 output rows through its slice of the Q tile
  uint8_t* sQp = smem;
#pragma unroll
  for (int nt = 0; nt < D / 8; ++nt) {
    const int c = nt * 8 + 2 * t;
    const int r_a = warp * 16 + g, r_b = r_a + 8;
    *reinterpret_cast<uint32_t*>(sQp + swz<ROWB>(r_a, c >> 3) + (c & 7) * 2) = pack_bf16(o[nt][0] * inv0, o[nt][1] * inv0);
    *reinterpret_cast<uint32_t*>(sQp + swz<ROWB>(r_b, c >> 3) + (c & 7) * 2) = pack_bf16(o[nt][2] * inv1, o[nt][3] * inv1);
  }
  __syncwarp();
  __nv_bfloat16* og = p.o + b * p.o_bs + (int64_t)h * D;
  constexpr int CH = D / 8;
#pragma unroll
  for (int i = lane; i < 16 * CH; i += 32) {
    const int r = warp * 16 + i / CH, c = i % CH;
    const int row = q0 + r;
    if (row < p.Sq)
      *reinterpret_cast<uint4*>(og + (int64_t)row * p.o_rs + c * 8) = *reinterpret_cast<const uint4*>(sQp + swz<ROWB>(r, c));
  }
  if (p.lse != nullptr && t == 0) {
    float* lg = p.lse + ((int64_t)b * p.Hq + h) * p.Sq;
    if (row0 < p.Sq) lg[row0] = l0 > 0.f ? (m0 + __log2f(l0)) / kLog2e : INFINITY;
    if (row0 + 8 < p.Sq) lg[row0 + 8] = l1 > 0.f ? (m1 + __log2f(l1)) / kLog2e : INFINITY;
  }
}

// ============================================================== backward
struct BwdParams {
  const __nv_bfloat16 *q, *k, *v, *o, *dout;
  const float* lse;   // [B, Hq, Sq]
  const float* dsum;  // [B, Hq, Sq]  rowsum(dO * O)
  float* dq_acc;      // [B, Sq, Hq, D] fp32, pre-zeroed
  __nv_bfloat16 *dk, *dv;
  int64_t q_bs, q_rs, k_bs, k_rs, v_bs, v_rs, do_bs, do_rs, dk_bs, dk_rs, dv_bs, dv_rs;
  int B, Hq, Hkv, Sq, Sk;
  float scale;  // softmax scale
  int causal;
  int causal_offset;
  int window;             // > 0: sliding window, as in the forward
  float cap_in, cap_out;  // softcap > 0: scale / cap and cap * log2(e), as in the forward
};

// D[b,h,i] = sum_d dO[b,i,h,d] * O[b,i,h,d]; one warp per row. The same warp
// zeroes the row's fp32 dQ accumulator dq_acc[b,i,h,:] (no separate memset).
template <int D>
__global__ void attn_bwd_dsum_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dout,
                                     float* __restrict__ dsum, float* __restrict__ dq_acc, int64_t o_bs,
                                     int64_t o_rs, int64_t do_bs, int64_t do_rs, int B, int Hq, int Sq) {
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= (int64_t)B * Hq * Sq) return;
  const int i = (int)(wid % Sq);
  const int64_t bh = wid / Sq;
  const int h = (int)(bh % Hq), b = (int)(bh / Hq);
  const __nv_bfloat16* op = o + b * o_bs + (int64_t)i * o_rs + (int64_t)h * D;
  const __nv_bfloat16* dp = dout + b * do_bs + (int64_t)i * do_rs + (int64_t)h * D;
  float s = 0.f;
  for (int c = lane * 4; c < D; c += 128) {
    const uint2 a = *reinterpret_cast<const uint2*>(op + c);
    const uint2 d = *reinterpret_cast<const uint2*>(dp + c);
    s += bf16lo(a.x) * bf16lo(d.x) + bf16hi(a.x) * bf16hi(d.x) + bf16lo(a.y) * bf16lo(d.y) + bf16hi(a.y) * bf16hi(d.y);
  }
  s = warp_sum(s);
  if (lane == 0) dsum[wid] = s;
  float* q_acc = dq_acc + (((int64_t)b * Sq + i) * Hq + h) * D;
  for (int c = lane * 4; c < D; c += 128) *reinterpret_cast<float4*>(q_acc + c) = make_float4(0.f, 0.f, 0.f, 0.f);
}

template <int D>
__global__ void attn_bwd_dq_convert_kernel(const float* __restrict__ acc, __nv_bfloat16* __restrict__ dq,
                                           int64_t dq_bs, int64_t dq_rs, int B, int Sq, int Hq, float scale) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // one 4-wide chunk
  const int64_t total = (int64_t)B * Sq * Hq * D / 4;
  if (i >= total) return;
  const int64_t e = i * 4;
  const int d = (int)(e % D);
  const int64_t r = e / D;  // (b, s, h)
  const int h = (int)(r % Hq);
  const int64_t bs = r / Hq;
  const int s = (int)(bs % Sq), b = (int)(bs / Sq);
  const float4 v = reinterpret_cast<const float4*>(acc)[i];
  uint2 out;
  out.x = pack_bf16(v.x * scale, v.y * scale);
  out.y = pack_bf16(v.z * scale, v.w * scale);
  *reinterpret_cast<uint2*>(dq + b * dq_bs + (int64_t)s * dq_rs + (int64_t)h * D + d) = out;
}

template <int D>
__global__ void __launch_bounds__(256, 1) attn_bwd_kernel(BwdParams p) {
  constexpr int BR = 64, BC = 64, NT = 256;
  constexpr int ROWB = D * 2;
  constexpr int KC = D / 16;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sK = smem_u32(smem);
  const uint32_t sV = sK + BC * ROWB;
  const uint32_t sQ0 = sV + BC * ROWB;            // 2 stages
  const uint32_t sdO0 = sQ0 + 2 * BR * ROWB;      // 2 stages
  const uint32_t sP = sdO0 + 2 * BR * ROWB;       // [BR][BC] bf16, 128-byte rows
  const uint32_t sdS = sP + BR * BC * 2;
  float* sL = reinterpret_cast<float*>(smem + (sdS - sK) + BR * BC * 2);  // [2][BR] lse*log2e
  float* sDs = sL + 2 * BR;                                               // [2][BR]
  uint8_t* sPp = smem + (sP - sK);
  uint8_t* sdSp = smem + (sdS - sK);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int wr = warp & 3, wc = warp >> 2;
  const int mi = lane >> 3;
  const int kb = blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / p.Hkv, hk = bh % p.Hkv;
  const int group = p.Hq / p.Hkv;
  const int k0 = kb * BC;
  const float scale_log2 = p.scale * kLog2e;

  const __nv_bfloat16* kg = p.k + b * p.k_bs + (int64_t)hk * D;
  const __nv_bfloat16* vg = p.v + b * p.v_bs + (int64_t)hk * D;
  load_tile<BC, D, NT>(sK, kg, p.k_rs, k0, p.Sk);
  load_tile<BC, D, NT>(sV, vg, p.v_rs, k0, p.Sk);
  cp_async_commit();

  // dK / dV accumulators: warp owns keys wr*16.., head-dim columns wc*(D/2)..
  constexpr int DN = D / 16;  // n-tiles of 8 per warp half
  float dk[DN][4], dv[DN][4];
#pragma unroll
  for (int i = 0; i < DN; ++i) {
    dk[i][0] = dk[i][1] = dk[i][2] = dk[i][3] = 0.f;
    dv[i][0] = dv[i][1] = dv[i][2] = dv[i][3] = 0.f;
  }

  int i_start = 0;
  if (p.causal) i_start = max(0, k0 - p.causal_offset) / BR;
  const int n_q = (p.Sq + BR - 1) / BR;
  const int iters_per_head = n_q - i_start;
  const int total = iters_per_head > 0 ? iters_per_head * group : 0;

  auto issue = [&](int it, int stage) {
    const int hq = hk * group + it / iters_per_head;
    const int qi = i_start + it % iters_per_head;
    const __nv_bfloat16* qg = p.q + b * p.q_bs + (int64_t)hq * D;
    const __nv_bfloat16* dg = p.dout + b * p.do_bs + (int64_t)hq * D;
    load_tile<BR, D, NT>(sQ0 + stage * BR * ROWB, qg, p.q_rs, qi * BR, p.Sq);
    load_tile<BR, D, NT>(sdO0 + stage * BR * ROWB, dg, p.do_rs, qi * BR, p.Sq);
    if (threadIdx.x < BR) {
      const int row = qi * BR + threadIdx.x;
      const int64_t base = ((int64_t)b * p.Hq + hq) * p.Sq;
      sL[stage * BR + threadIdx.x] = row < p.Sq ? p.lse[base + row] * kLog2e : INFINITY;
      sDs[stage * BR + threadIdx.x] = row < p.Sq ? p.dsum[base + row] : 0.f;
    }
  };

  if (total > 0) issue(0, 0);
  cp_async_commit();

  for (int it = 0; it < total; ++it) {
    const int st = it & 1;
    const int hq = hk * group + it / iters_per_head;
    const int qi = i_start + it % iters_per_head;
    const int q0 = qi * BR;
    if (it + 1 < total) {
      issue(it + 1, st ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint32_t sQ = sQ0 + st * BR * ROWB;
    const uint32_t sdO = sdO0 + st * BR * ROWB;

    // S = Q K^T and dP = dO V^T for rows wr*16.., keys wc*32..
    float s[4][4], dp[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
      dp[i][0] = dp[i][1] = dp[i][2] = dp[i][3] = 0.f;
    }
#pragma unroll
    for (int kc = 0; kc < KC; ++kc) {
      uint32_t a[4], ad[4];
      const int r = wr * 16 + (mi & 1) * 8 + (lane & 7);
      ldsm_x4(sQ + swz<ROWB>(r, 2 * kc + (mi >> 1)), a[0], a[1], a[2], a[3]);
      ldsm_x4(sdO + swz<ROWB>(r, 2 * kc + (mi >> 1)), ad[0], ad[1], ad[2], ad[3]);
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        const int key = wc * 32 + np * 16 + (mi >> 1) * 8 + (lane & 7);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(sK + swz<ROWB>(key, 2 * kc + (mi & 1)), b0, b1, b2, b3);
        mma16816(s[2 * np], a, b0, b1);
        mma16816(s[2 * np + 1], a, b2, b3);
        ldsm_x4(sV + swz<ROWB>(key, 2 * kc + (mi & 1)), b0, b1, b2, b3);
        mma16816(dp[2 * np], ad, b0, b1);
        mma16816(dp[2 * np + 1], ad, b2, b3);
      }
    }
    // P = exp2(S * scale_log2 - lse2), dS = P * (dP - Dsum)
    const float* L = sL + st * BR;
    const float* Dv = sDs + st * BR;
    const int ra = wr * 16 + g, rb = ra + 8;
    const float la = L[ra], lb = L[rb], da = Dv[ra], db = Dv[rb];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      const int colb = wc * 32 + nt * 8 + 2 * t;
      float pv[4], ds[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = k0 + colb + (e & 1);
        const int row = q0 + ((e >> 1) ? rb : ra);
        const float lrow = (e >> 1) ? lb : la;
        bool ok = col < p.Sk && row < p.Sq;
        if (p.causal && col > row + p.causal_offset) ok = false;
        if (p.window > 0 && col < row + p.causal_offset - p.window + 1) ok = false;
        // soft-capped logits: z = cap tanh(s scale / cap), dz / d(s scale) = 1 - tanh^2
        float logit2 = s[nt][e] * scale_log2, dcap = 1.f;
        if (p.cap_in > 0.f) {
          const float th = tanh_sfu(s[nt][e] * p.cap_in);
          logit2 = p.cap_out * th;
          dcap = 1.f - th * th;
        }
        const float pe = ok ? exp2f(logit2 - lrow) : 0.f;
        pv[e] = pe;
        ds[e] = pe * (dp[nt][e] - ((e >> 1) ? db : da)) * dcap;
      }
      const int ch = colb >> 3, off = (colb & 7) * 2;
      *reinterpret_cast<uint32_t*>(sPp + swz<128>(ra, ch) + off) = pack_bf16(pv[0], pv[1]);
      *reinterpret_cast<uint32_t*>(sPp + swz<128>(rb, ch) + off) = pack_bf16(pv[2], pv[3]);
      *reinterpret_cast<uint32_t*>(sdSp + swz<128>(ra, ch) + off) = pack_bf16(ds[0], ds[1]);
      *reinterpret_cast<uint32_t*>(sdSp + swz<128>(rb, ch) + off) = pack_bf16(ds[2], ds[3]);
    }
    __syncthreads();

    // dV += P^T dO, dK += dS^T Q  (keys wr*16.., d columns wc*D/2..)
#pragma unroll
    for (int kc = 0; kc < BR / 16; ++kc) {
      uint32_t ap[4], as[4];
      // A = P^T: stored [q][key]; matrices (q lo, key lo), (q lo, key hi), (q hi, key lo), (q hi, key hi)
      const int qr = kc * 16 + (mi >> 1) * 8 + (lane & 7);
      const int kch = (wr * 16) / 8 + (mi & 1);
      ldsm_x4_t(sP + swz<128>(qr, kch), ap[0], ap[1], ap[2], ap[3]);
      ldsm_x4_t(sdS + swz<128>(qr, kch), as[0], as[1], as[2], as[3]);
      const int qrow = kc * 16 + (mi & 1) * 8 + (lane & 7);
#pragma unroll
      for (int dp2 = 0; dp2 < DN / 2; ++dp2) {
        const int dch = (wc * (D / 2)) / 8 + 2 * dp2 + (mi >> 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(sdO + swz<ROWB>(qrow, dch), b0, b1, b2, b3);
        mma16816(dv[2 * dp2], ap, b0, b1);
        mma16816(dv[2 * dp2 + 1], ap, b2, b3);
        ldsm_x4_t(sQ + swz<ROWB>(qrow, dch), b0, b1, b2, b3);
        mma16816(dk[2 * dp2], as, b0, b1);
        mma16816(dk[2 * dp2 + 1], as, b2, b3);
      }
    }
    // dQ += dS K  (rows wr*16.., d columns wc*D/2..) -> fp32 atomics
    {
      float dq[DN][4];
#pragma unroll
      for (int i = 0; i < DN; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;
#pragma unroll
      for (int kc = 0; kc < BC / 16; ++kc) {
        uint32_t a[4];
        const int r = wr * 16 + (mi & 1) * 8 + (lane & 7);
        ldsm_x4(sdS + swz<128>(r, 2 * kc + (mi >> 1)), a[0], a[1], a[2], a[3]);
        const int key = kc * 16 + (mi & 1) * 8 + (lane & 7);
#pragma unroll
        for (int dp2 = 0; dp2 < DN / 2; ++dp2) {
          const int dch = (wc * (D / 2)) / 8 + 2 * dp2 + (mi >> 1);
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(sK + swz<ROWB>(key, dch), b0, b1, b2, b3);
          mma16816(dq[2 * dp2], a, b0, b1);
          mma16816(dq[2 * dp2 + 1], a, b2, b3);
        }
      }
      const int row_a = q0 + wr * 16 + g, row_b = row_a + 8;
      float* base = p.dq_acc + (((int64_t)b * p.Sq) * p.Hq + hq) * D;
#pragma unroll
      for (int nt = 0; nt < DN; ++nt) {
        const int col = wc * (D / 2) + nt * 8 + 2 * t;
        if (row_a < p.Sq) {
          float* d0 = base + ((int64_t)row_a * p.Hq) * D + col;
          atomicAdd(reinterpret_cast<float2*>(d0), make_float2(dq[nt][0], dq[nt][1]));
        }
        if (row_b < p.Sq) {
          float* d1 = base + ((int64_t)row_b * p.Hq) * D + col;
          atomicAdd(reinterpret_cast<float2*>(d1), make_float2(dq[nt][2], dq[nt][3]));
        }
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();

  // write dK (scaled) and dV
  const int key_a = k0 + wr * 16 + g, key_b = key_a + 8;
  __nv_bfloat16* dkg = p.dk + b * p.dk_bs + (int64_t)hk * D;
  __nv_bfloat16* dvg = p.dv + b * p.dv_bs + (int64_t)hk * D;
#pragma unroll
  for (int nt = 0; nt < DN; ++nt) {
    const int col = wc * (D / 2) + nt * 8 + 2 * t;
    if (key_a < p.Sk) {
      *reinterpret_cast<uint32_t*>(dkg + (int64_t)key_a * p.dk_rs + col) = pack_bf16(dk[nt][0] * p.scale, dk[nt][1] * p.scale);
      *reinterpret_cast<uint32_t*>(dvg + (int64_t)key_a * p.dv_rs + col) = pack_bf16(dv[nt][0], dv[nt][1]);
    }
    if (key_b < p.Sk) {
      *reinterpret_cast<uint32_t*>(dkg + (int64_t)key_b * p.dk_rs + col) = pack_bf16(dk[nt][2] * p.scale, dk[nt][3] * p.scale);
      *reinterpret_cast<uint32_t*>(dvg + (int64_t)key_b * p.dv_rs + col) = pack_bf16(dv[nt][2], dv[nt][3]);
    }
  }
}

template <int D>
constexpr int fwd_smem() { return (128 + 4 * 64) * D * 2; }
template <int D>
constexpr int bwd_smem() { return (2 * 64 + 4 * 64) * D * 2 + 2 * 64 * 64 * 2 + 4 * 64 * 4; }

// [B, S, H, D] view with strides checked: last dim contiguous, head stride D.
void check_bshd(const at::Tensor& x, int64_t H, int64_t D, const char* what) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16, what, ": bf16 CUDA tensor required");
  TORCH_CHECK(x.dim() == 4 && x.size(2) == H && x.size(3) == D, what, ": expected [B, S, H, D]");
  TORCH_CHECK(x.stride(3) == 1 && x.stride(2) == D, what, ": head dim must be contiguous with head stride D");
  TORCH_CHECK(x.stride(1) % 8 == 0 && x.stride(0) % 8 == 0, what, ": strides must be multiples of 8");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(x.data_ptr()) & 15) == 0, what, ": 16-byte aligned base required");
}

}  // namespace attn

// q: [B, Sq, Hq, D], k/v: [B, Sk, Hkv, D] (strided views allowed), out: [B, Sq, Hq, D].
// lse: optional fp32 [B, Hq, Sq].
void attention_fwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor out, std::optional<at::Tensor> lse,
                   double scale, bool causal, int64_t causal_offset, int64_t window, double softcap) {
  const int64_t B = q.size(0), Sq = q.size(1), Hq = q.size(2), D = q.size(3);
  const int64_t Sk = k.size(1), Hkv = k.size(2);
  attn::check_bshd(q, Hq, D, "attention q");
  attn::check_bshd(k, Hkv, D, "attention k");
  attn::check_bshd(v, Hkv, D, "attention v");
  attn::check_bshd(out, Hq, D, "attention out");
  TORCH_CHECK(Hq % Hkv == 0, "attention: Hq must be a multiple of Hkv");
  TORCH_CHECK(D == 64 || D == 128, "attention: head_dim 64 or 128");
  c10::cuda::CUDAGuard guard(q.device());
  attn::FwdParams p{};
  p.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  p.k = reinterpret_cast<const __nv_bfloat16*>(k.data_ptr());
  p.v = reinterpret_cast<const __nv_bfloat16*>(v.data_ptr());
  p.o = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.lse = (lse && lse->defined()) ? lse->data_ptr<float>() : nullptr;
  p.q_bs = q.stride(0); p.q_rs = q.stride(1);
  p.k_bs = k.stride(0); p.k_rs = k.stride(1);
  p.v_bs = v.stride(0); p.v_rs = v.stride(1);
  p.o_bs = out.stride(0); p.o_rs = out.stride(1);
  p.B = (int)B; p.Hq = (int)Hq; p.Hkv = (int)Hkv; p.Sq = (int)Sq; p.Sk = (int)Sk;
  p.scale_log2 = (float)scale * attn::kLog2e;
  p.causal = causal ? 1 : 0;
  p.causal_offset = (int)causal_offset;
  p.window = (int)window;
  if (softcap > 0.0) {
    p.cap_in = (float)(scale / softcap);
    p.cap_out = (float)softcap * attn::kLog2e;
  }
  if (B == 0 || Sq == 0) return;
  dim3 grid((unsigned)((Sq + 127) / 128), (unsigned)(B * Hq));
  auto stream = at::cuda::getCurrentCUDAStream();
  if (D == 128) {
    constexpr int sm = attn::fwd_smem<128>();
    AETHER_CUDA_CHECK(cudaFuncSetAttribute(attn::attn_fwd_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
    attn::attn_fwd_kernel<128><<<grid, 256, sm, stream>>>(p);
  } else {
    constexpr int sm = attn::fwd_smem<64>();
    AETHER_CUDA_CHECK(cudaFuncSetAttribute(attn::attn_fwd_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
    attn::attn_fwd_kernel<64><<<grid, 256, sm, stream>>>(p);
  }
  AETHER_CUDA_CHECK(cudaGetLastError());
}

void attention_bwd_tc(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor dout, at::Tensor lse, at::Tensor dsum,
                      at::Tensor dq_acc, at::Tensor dk, at::Tensor dv, double scale, bool causal,
                      int64_t causal_offset);

// Gradients of attention_fwd. dq/dk/dv are written (not accumulated). With
// use_tc (head_dim 128) the main pass runs on the tcgen05 kernel of
// attention_bwd_sm100.cu; the rowsum(dO*O) pre-pass and the dQ conversion are shared.
void attention_bwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor out, at::Tensor dout, at::Tensor lse,
                   at::Tensor dq, at::Tensor dk, at::Tensor dv, double scale, bool causal, int64_t causal_offset,
                   bool use_tc, int64_t window, double softcap) {
  const int64_t B = q.size(0), Sq = q.size(1), Hq = q.size(2), D = q.size(3);
  const int64_t Sk = k.size(1), Hkv = k.size(2);
  attn::check_bshd(q, Hq, D, "attention_bwd q");
  attn::check_bshd(k, Hkv, D, "attention_bwd k");
  attn::check_bshd(v, Hkv, D, "attention_bwd v");
  attn::check_bshd(out, Hq, D, "attention_bwd out");
  attn::check_bshd(dout, Hq, D, "attention_bwd dout");
  attn::check_bshd(dq, Hq, D, "attention_bwd dq");
  attn::check_bshd(dk, Hkv, D, "attention_bwd dk");
  attn::check_bshd(dv, Hkv, D, "attention_bwd dv");
  TORCH_CHECK(D == 64 || D == 128, "attention_bwd: head_dim 64 or 128");
  TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.is_contiguous() && lse.numel() == B * Hq * Sq, "attention_bwd: lse");
  c10::cuda::CUDAGuard guard(q.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  if (B == 0 || Sq == 0) return;
  auto dsum = at::empty({B, Hq, Sq}, q.options().dtype(at::kFloat));
  auto dq_acc = at::empty({B, Sq, Hq, D}, q.options().dtype(at::kFloat));  // zeroed by the dsum pre-pass
  const int64_t rows = B * Hq * Sq;
  const unsigned dgrid = (unsigned)((rows * 32 + 255) / 256);
  if (D == 128)
    attn::attn_bwd_dsum_kernel<128><<<dgrid, 256, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(out.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()),
        dsum.data_ptr<float>(), dq_acc.data_ptr<float>(), out.stride(0), out.stride(1), dout.stride(0), dout.stride(1),
        (int)B, (int)Hq, (int)Sq);
  else
    attn::attn_bwd_dsum_kernel<64><<<dgrid, 256, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(out.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()),
        dsum.data_ptr<float>(), dq_acc.data_ptr<float>(), out.stride(0), out.stride(1), dout.stride(0), dout.stride(1),
        (int)B, (int)Hq, (int)Sq);
  AETHER_CUDA_CHECK(cudaGetLastError());

  TORCH_CHECK(window >= 0 && softcap >= 0.0, "attention_bwd: window and softcap must be >= 0");
  if (window > 0 || softcap > 0.0) use_tc = false;  // the flex forms run on the mma.sync kernel
  if (use_tc) {
    TORCH_CHECK(D == 128, "attention_bwd: the tcgen05 path needs head_dim 128");
    attention_bwd_tc(q, k, v, dout, lse, dsum, dq_acc, dk, dv, scale, causal, causal_offset);
  } else {
  attn::BwdParams p{};
  p.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  p.k = reinterpret_cast<const __nv_bfloat16*>(k.data_ptr());
  p.v = reinterpret_cast<const __nv_bfloat16*>(v.data_ptr());
  p.o = reinterpret_cast<const __nv_bfloat16*>(out.data_ptr());
  p.dout = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr());
  p.lse = lse.data_ptr<float>();
  p.dsum = dsum.data_ptr<float>();
  p.dq_acc = dq_acc.data_ptr<float>();
  p.dk = reinterpret_cast<__nv_bfloat16*>(dk.data_ptr());
  p.dv = reinterpret_cast<__nv_bfloat16*>(dv.data_ptr());
  p.q_bs = q.stride(0); p.q_rs = q.stride(1);
  p.k_bs = k.stride(0); p.k_rs = k.stride(1);
  p.v_bs = v.stride(0); p.v_rs = v.stride(1);
  p.do_bs = dout.stride(0); p.do_rs = dout.stride(1);
  p.dk_bs = dk.stride(0); p.dk_rs = dk.stride(1);
  p.dv_bs = dv.stride(0); p.dv_rs = dv.stride(1);
  p.B = (int)B; p.Hq = (int)Hq; p.Hkv = (int)Hkv; p.Sq = (int)Sq; p.Sk = (int)Sk;
  p.scale = (float)scale;
  p.causal = causal ? 1 : 0;
  p.causal_offset = (int)causal_offset;
  p.window = (int)window;
  if (softcap > 0.0) {
    p.cap_in = (float)(scale / softcap);
    p.cap_out = (float)softcap * attn::kLog2e;
  }
  dim3 grid((unsigned)((Sk + 63) / 64), (unsigned)(B * Hkv));
  if (D == 128) {
    constexpr int sm = attn::bwd_smem<128>();
    AETHER_CUDA_CHECK(cudaFuncSetAttribute(attn::attn_bwd_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
    attn::attn_bwd_kernel<128><<<grid, 256, sm, stream>>>(p);
  } else {
    constexpr int sm = attn::bwd_smem<64>();
    AETHER_CUDA_CHECK(cudaFuncSetAttribute(attn::attn_bwd_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
    attn::attn_bwd_kernel<64><<<grid, 256, sm, stream>>>(p);
  }
  AETHER_CUDA_CHECK(cudaGetLastError());
  }
  const int64_t n4 = B * Sq * Hq * D / 4;
  const unsigned cgrid = (unsigned)((n4 + 255) / 256);
  if (D == 128)
    attn::attn_bwd_dq_convert_kernel<128><<<cgrid, 256, 0, stream>>>(dq_acc.data_ptr<float>(),
                                                                     reinterpret_cast<__nv_bfloat16*>(dq.data_ptr()),
                                                                     dq.stride(0), dq.stride(1), (int)B, (int)Sq, (int)Hq, (float)scale);
  else
    attn::attn_bwd_dq_convert_kernel<64><<<cgrid, 256, 0, stream>>>(dq_acc.data_ptr<float>(),
                                                                    reinterpret_cast<__nv_bfloat16*>(dq.data_ptr()),
                                                                    dq.stride(0), dq.stride(1), (int)B, (int)Sq, (int)Hq, (float)scale);
  AETHER_CUDA_CHECK(cudaGetLastError());
}

}  // namespace aether
