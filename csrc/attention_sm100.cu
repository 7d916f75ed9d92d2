// Flash-attention forward on the sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// One CTA computes 256 query rows (two 128-row sub-tiles) of one head (head_dim 128):
//   warp 0      : TMA producer -- the Q tile once, then K and V tiles of 128
//                 keys through a 2-stage ring (128B-swizzled, no multicast)
//   warp 1      : TMEM allocator + single-thread MMA issuer:
//                   S_j = Q K_j^T        (SS MMA, M128 N128, into TMEM S[j%2])
//                   O  += P_{j-1} V_{j-1} (TS MMA: P read from TMEM, V from smem)
//                 QK_j is issued before PV_{j-1}, so the tensor core computes
//                 the next scores while the softmax warps work on this tile
//   warps 2..9  : two softmax warpgroups, one per sub-tile, one thread per query
//                 row: tcgen05.ld of its S row, masking,
//                 online softmax (max / exp2 / sum in registers), P written back
//                 as bf16 over the S columns (tcgen05.st), and O rescaled in
//                 TMEM only when the row maximum outgrows the exponent base
//                 by more than 2^8 (lazy rescaling)
// TMEM: per sub-tile an S/P region (128 columns) and an O accumulator (128).
// The MMA issuer interleaves the sub-tiles (PV of one, QK of the other) so the
// tensor core stays busy while each warpgroup runs its softmax.
//
// Reference counterpart: sdpa_causal_fwd (runtime/src/cuda.rs:6736-6786), one
// thread per query row materialising the [bh, s, s] probability matrix.
// Same semantics as attention.cu's attention_fwd (GQA, causal offset, LSE out,
// sliding window and logit softcap).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cstdlib>
#include <string>

#include "common.cuh"
#include "host_utils.h"

namespace aether {
namespace fa {

constexpr int BM = 256;   // query rows per CTA (two 128-row sub-tiles)
constexpr int BN = 128;   // keys per tile
constexpr int D = 128;    // head dim
constexpr int KV_STAGES = 2;
constexpr int kThreads = 320;  // producer, MMA, two softmax warpgroups
constexpr int TILE_BYTES = 128 * D * 2;  // 32 KB: [128 rows][128 d] as two 128B-swizzled halves
constexpr int kSmem = TILE_BYTES * (2 + 2 * KV_STAGES) + 1024 + 256;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleLog2 = 8.f;  // base moves when the row max grows by > 2^8

struct Params {
  __nv_bfloat16* out;
  int64_t o_bs, o_rs;
  float* lse;  // [B, Hq, Sq] or null
  int B, Hq, Hkv, Sq, Sk;
  float scale_log2;
  int causal, causal_offset;
  int window;             // > 0: keys < row + offset - window + 1 are hidden
  float cap_in, cap_out;  // softcap > 0: s' = cap tanh(s scale / cap), in the log2 domain
  int* status;
};

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// Loads one [128 rows][128 d] tile as two 64-column boxes (128B swizzle).
__device__ __forceinline__ void load_tile(uint8_t* dst, const CUtensorMap* map, uint64_t* bar, int x0, int y0) {
  tma_load_2d(dst, map, bar, x0, y0);
  tma_load_2d(dst + TILE_BYTES / 2, map, bar, x0 + 64, y0);
}

// 2^x on the SFU (ex2.approx.ftz.f32); probabilities are rounded to bf16 next.
__device__ __forceinline__ float ex2_sfu(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x for x <= 0 on the FMA / integer pipes, so the softmax is not bound by
// the SFU's 16 results per clock: x = n + f with n = round(x) taken from the
// low mantissa bits of x + 1.5 * 2^23, 2^f for f in [-0.5, 0.5] from a cubic
// fitted here (least squares reweighted to the minimax relative error,
// max 1.0e-4 -- bf16 keeps 2^-9), and n added to the exponent field.
__device__ __forceinline__ float ex2_poly(float x) {
  x = fmaxf(x, -126.f);
  const float t = x + 12582912.f;
  const float f = x - (t - 12582912.f);
  const float p = fmaf(fmaf(fmaf(0.055008791f, f, 0.24221075f), f, 0.69328290f), f, 1.f);
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

// Blackwell's three-input max and packed two-lane fp32 FMA / add: half the
// issue slots of the scalar forms in the softmax's per-score work.
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ uint64_t pack_f32x2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void unpack_f32x2(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t fma_f32x2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

template <bool kPoly>
__global__ void __launch_bounds__(kThreads, 1)
    fa_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                       // [2 sub-tiles]
  uint8_t* sK = sQ + 2 * TILE_BYTES;        // [KV_STAGES]
  uint8_t* sV = sK + KV_STAGES * TILE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + KV_STAGES * TILE_BYTES);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;                // [KV_STAGES]
  uint64_t* v_full = k_full + KV_STAGES;      // [KV_STAGES]
  uint64_t* kv_empty = v_full + KV_STAGES;    // [KV_STAGES]
  uint64_t* s_full = kv_empty + KV_STAGES;    // [2 groups]
  uint64_t* p_full = s_full + 2;              // [2 groups]
  uint64_t* o_done = p_full + 2;              // [2 groups]
  uint64_t* drain = o_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_word = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qb = gridDim.x - 1 - blockIdx.x;  // longest causal rows first
  const int bh = blockIdx.y;
  const int b = bh / p.Hq, h = bh % p.Hq;
  const int hk = h / (p.Hq / p.Hkv);
  const int q0 = qb * BM;
  // KV tiles each 128-row sub-tile needs (causal rows see keys <= row + offset)
  int nkv[2];
#pragma unroll
  for (int g = 0; g < 2; ++g) {
    int kv_end = p.Sk;
    if (p.causal) kv_end = min(p.Sk, q0 + 128 * (g + 1) + p.causal_offset);
    nkv[g] = kv_end > 0 ? (kv_end + BN - 1) / BN : 0;
  }
  const int n_kv = max(nkv[0], nkv[1]);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < KV_STAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(&s_full[g], 1);
      mbar_init(&p_full[g], 128);
      mbar_init(&o_done[g], 1);
    }
    mbar_init(drain, 1);
    *abort_word = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;  // group g: S at 256g, O at 256g + 128

  if (warp == 0) {
    if (lane == 0 && n_kv > 0) {
      // ------------------------------------------------------------ producer
      mbar_arrive_expect_tx(q_full, 2 * TILE_BYTES);
      load_tile(sQ, &tmQ, q_full, h * D, b * p.Sq + q0);
      load_tile(sQ + TILE_BYTES, &tmQ, q_full, h * D, b * p.Sq + q0 + 128);
      bool ok = true;
      for (int j = 0; j < n_kv && ok; ++j) {
        const int st = j % KV_STAGES;
        const uint32_t ph = (j / KV_STAGES) & 1u;
        if (!mbar_wait(&kv_empty[st], ph ^ 1u, abort_word)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&k_full[st], TILE_BYTES);
        load_tile(sK + st * TILE_BYTES, &tmK, &k_full[st], hk * D, b * p.Sk + j * BN);
        mbar_arrive_expect_tx(&v_full[st], TILE_BYTES);
        load_tile(sV + st * TILE_BYTES, &tmV, &v_full[st], hk * D, b * p.Sk + j * BN);
      }
      if (!ok) {
        *abort_word = 1;
        atomicExch(p.status, kStatusTimeoutProducer);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && n_kv > 0) {
      // ------------------------------------------------------------ MMA issuer
      // Order: QK(0,0) QK(1,0) | PV(0,j) QK(0,j+1) PV(1,j) QK(1,j+1) | ...
      // so the tensor core works on one sub-tile while the other's softmax runs.
      constexpr uint32_t idesc_qk = idesc_bf16_f32(128, BN, false, false);
      constexpr uint32_t idesc_pv = idesc_bf16_f32(128, D, false, true);
      bool ok = mbar_wait(q_full, 0, abort_word);
      tc_fence_after();
      auto issue_qk = [&](int g, int j) -> bool {
        const int st = j % KV_STAGES;
        if (!mbar_wait(&k_full[st], (j / KV_STAGES) & 1u, abort_word)) return false;
        tc_fence_after();
        const uint32_t q_addr = smem_u32(sQ + g * TILE_BYTES);
        const uint32_t k_addr = smem_u32(sK + st * TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (TILE_BYTES / 2) + (kk & 3) * 32;
          umma_f16(tmem + 256 * g, sdesc_sw128(q_addr + off, 16, 1024), sdesc_sw128(k_addr + off, 16, 1024), idesc_qk,
                   kk != 0 ? 1u : 0u);
        }
        umma_commit(&s_full[g]);
        return true;
      };
      auto issue_pv = [&](int g, int j) -> bool {
        const int st = j % KV_STAGES;
        if (!mbar_wait(&p_full[g], j & 1u, abort_word)) return false;
        if (!mbar_wait(&v_full[st], (j / KV_STAGES) & 1u, abort_word)) return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sV + st * TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)
          umma_f16_ts(tmem + 256 * g + 128, tmem + 256 * g + kk * 8,
                      sdesc_sw128(v_addr + kk * 2048, TILE_BYTES / 2, 1024), idesc_pv, (j != 0 || kk != 0) ? 1u : 0u);
        umma_commit(&o_done[g]);
        return true;
      };
      for (int g = 0; g < 2 && ok; ++g)
        if (nkv[g] > 0) ok = issue_qk(g, 0);
      for (int j = 0; j < n_kv && ok; ++j) {
        if (j < nkv[0]) ok = issue_pv(0, j);
        if (ok && j + 1 < nkv[0]) ok = issue_qk(0, j + 1);
        if (ok && j < nkv[1]) ok = issue_pv(1, j);
        if (ok && j + 1 < nkv[1]) ok = issue_qk(1, j + 1);
        if (ok) umma_commit(&kv_empty[j % KV_STAGES]);  // K_j and V_j consumed by every MMA issued so far
      }
      if (!ok) {
        *abort_word = 1;
        atomicExch(p.status, kStatusTimeoutMma);
      }
      volatile int never = 0;
      umma_commit(drain);
      mbar_wait(drain, 0, &never);
    }
  } else {
    // -------------------------------------------------------------- softmax groups
    const int grp = (warp - 2) >> 2;
    const int quad = warp & 3;
    const int row = quad * 32 + lane;  // row within the sub-tile = TMEM lane
    const int qpos = q0 + 128 * grp + row;
    const int qsub0 = q0 + 128 * grp;  // first row of this sub-tile
    const int my_kv = nkv[grp];
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t tS = tmem + 256 * grp, tO = tS + 128;
    float m = -INFINITY, l = 0.f;
    uint32_t o_phase = 0;
    bool ok = true;
    for (int j = 0; j < my_kv; ++j) {
      if (!mbar_wait(&s_full[grp], j & 1u, abort_word)) {
        ok = false;
        break;
      }
      __syncwarp();
      tc_fence_after();
      // Scores stay in raw units (the softmax scale is folded into the
      // exponent's FMA below); with a softcap they are capped logits in log2 units.
      float s[BN];
      {
        uint32_t r[BN];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) tmem_ld32(tS + lane_off + c * 32, *reinterpret_cast<uint32_t(*)[32]>(r + c * 32));
        tmem_ld_wait();
        if (p.cap_in > 0.f) {
#pragma unroll
          for (int t = 0; t < BN; ++t) s[t] = p.cap_out * tanh_sfu(__uint_as_float(r[t]) * p.cap_in);
        } else {
#pragma unroll
          for (int t = 0; t < BN; ++t) s[t] = __uint_as_float(r[t]);
        }
      }
      const float sc = p.cap_in > 0.f ? 1.f : p.scale_log2;
      const int key0 = j * BN;
      const bool need_mask = (key0 + BN > p.Sk) || (p.causal && key0 + BN - 1 > qsub0 + p.causal_offset);
      if (need_mask) {
        const int lim = p.causal ? min(p.Sk, qpos + p.causal_offset + 1) : p.Sk;
#pragma unroll
        for (int t = 0; t < BN; ++t)
          if (key0 + t >= lim) s[t] = -INFINITY;
      }
      if (p.window > 0) {
        const int lo = qpos + p.causal_offset - p.window + 1;  // first visible key of this row
        if (key0 < lo) {
#pragma unroll
          for (int t = 0; t < BN; ++t)
            if (key0 + t < lo) s[t] = -INFINITY;
        }
      }
      // row max over eight independent accumulators (a single chain would
      // serialise 128 dependent max operations per tile)
      // (three-input max: two new scores per instruction)
      float m8[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) m8[u] = -INFINITY;
#pragma unroll
      for (int t = 0; t < BN; t += 2) m8[(t >> 1) & 7] = max3f(m8[(t >> 1) & 7], s[t], s[t + 1]);
      const float mx = sc * max3f(max3f(m8[0], m8[1], m8[2]), max3f(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
      // Lazy rescaling: the exponent base only moves when the row maximum
      // grows by more than 2^8 over it. Until then probabilities may reach
      // 2^8 (exact in fp32 / bf16 range), and O and l share the stale base,
      // so O / l is unchanged; the TMEM rescale of O (128 loads, multiplies
      // and stores per row) drops out of nearly every tile.
      const bool grow = mx > m + kRescaleLog2;
      const float mn = grow ? mx : m;
      const float alpha = grow ? ex2_sfu(m - mn) : 1.f;
      const float base = mn == -INFINITY ? 0.f : mn;
      // exponent arguments and row sums two at a time (packed f32x2 FMA / add)
      const uint64_t sc2 = pack_f32x2(sc, sc), nb2 = pack_f32x2(-base, -base);
      uint64_t r4[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) r4[u] = 0ull;
      // P_j goes over the S_j columns as each half is ready (S_j landing means
      // PV_{j-1}, which read P_{j-1} there, has completed), which also frees
      // the half's score registers early.
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        uint32_t pk[32];
#pragma unroll
        for (int t = 64 * hf; t < 64 * hf + 64; t += 2) {
          float x0, x1;
          unpack_f32x2(fma_f32x2(pack_f32x2(s[t], s[t + 1]), sc2, nb2), x0, x1);
          float a0, a1;
          if (kPoly && ((t >> 1) & 3) == 3) {  // a quarter of the exponentials on the FMA pipe
            a0 = ex2_poly(x0);
            a1 = ex2_poly(x1);
          } else {
            a0 = ex2_sfu(x0);
            a1 = ex2_sfu(x1);
          }
          r4[(t >> 1) & 3] = add_f32x2(r4[(t >> 1) & 3], pack_f32x2(a0, a1));
          pk[(t - 64 * hf) / 2] = pack_bf16(a0, a1);
        }
        tmem_st32(tS + lane_off + 32 * hf, pk);
      }
      const uint64_t r2 = add_f32x2(add_f32x2(r4[0], r4[1]), add_f32x2(r4[2], r4[3]));
      float rs0, rs1;
      unpack_f32x2(r2, rs0, rs1);
      const float rs = rs0 + rs1;
      l = l * alpha + rs;
      m = mn;
      // PV_{j-1} must have landed before O may be touched; every PV completion
      // is awaited in order so the o_done barrier never runs two phases ahead.
      if (j > 0) {
        if (!mbar_wait(&o_done[grp], o_phase, abort_word)) {
          ok = false;
          break;
        }
        o_phase ^= 1u;
      }
      // Rescale O only if some row of this warp moved its base.
      const bool need = (j > 0) && grow;
      if (__any_sync(0xffffffffu, need)) {
        __syncwarp();
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tO + lane_off + c * 32, r);
          tmem_ld_wait();
#pragma unroll
          for (int t = 0; t < 32; ++t) r[t] = __float_as_uint(__uint_as_float(r[t]) * alpha);
          tmem_st32(tO + lane_off + c * 32, r);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[grp]);
    }
    if (ok && my_kv > 0) {
      if (!mbar_wait(&o_done[grp], o_phase, abort_word)) ok = false;
    }
    if (!ok) {
      *abort_word = 1;
      if (lane == 0) atomicExch(p.status, kStatusTimeoutEpilogue);
    } else {
      __syncwarp();
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* orow = p.out + (int64_t)b * p.o_bs + (int64_t)qpos * p.o_rs + (int64_t)h * D;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t r[32];
        if (my_kv > 0) {
          tmem_ld32(tO + lane_off + c * 32, r);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int t = 0; t < 32; ++t) r[t] = 0u;
        }
        if (qpos < p.Sq) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 o;
            o.x = pack_bf16(__uint_as_float(r[q * 8 + 0]) * inv, __uint_as_float(r[q * 8 + 1]) * inv);
            o.y = pack_bf16(__uint_as_float(r[q * 8 + 2]) * inv, __uint_as_float(r[q * 8 + 3]) * inv);
            o.z = pack_bf16(__uint_as_float(r[q * 8 + 4]) * inv, __uint_as_float(r[q * 8 + 5]) * inv);
            o.w = pack_bf16(__uint_as_float(r[q * 8 + 6]) * inv, __uint_as_float(r[q * 8 + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + c * 32 + q * 8) = o;
          }
        }
      }
      if (p.lse != nullptr && qpos < p.Sq)
        p.lse[((int64_t)b * p.Hq + h) * p.Sq + qpos] = l > 0.f ? (m + __log2f(l)) / kLog2e : INFINITY;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace fa

// Same contract as attention_fwd (head_dim 128 only): q [B,Sq,Hq,128], k/v
// [B,Sk,Hkv,128] with unit head-dim stride, head stride 128 and any token-row
// stride that is a multiple of 8 elements; lse optional fp32 [B,Hq,Sq].
void attention_fwd_tc(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor out, std::optional<at::Tensor> lse,
                      double scale, bool causal, int64_t causal_offset, int64_t window, double softcap) {
  const int64_t B = q.size(0), Sq = q.size(1), Hq = q.size(2), D = q.size(3);
  const int64_t Sk = k.size(1), Hkv = k.size(2);
  TORCH_CHECK(D == 128 && k.size(3) == 128, "attention_fwd_tc: head_dim 128");
  for (const at::Tensor* t : {&q, &k, &v, &out}) {
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->dim() == 4, "attention_fwd_tc: bf16 [B,S,H,D]");
    TORCH_CHECK(t->stride(3) == 1 && t->stride(2) == 128 && t->stride(1) % 8 == 0, "attention_fwd_tc: layout");
  }
  // the 2-D tensor maps flatten (batch, token): each batch's rows must follow the previous batch's
  TORCH_CHECK(q.stride(0) == Sq * q.stride(1) && k.stride(0) == Sk * k.stride(1) && v.stride(0) == Sk * v.stride(1),
              "attention_fwd_tc: batch stride must equal S * row stride");
  TORCH_CHECK(Hq % Hkv == 0, "attention_fwd_tc: GQA group");
  c10::cuda::CUDAGuard guard(q.device());
  if (B == 0 || Sq == 0) return;
  const CUtensorMap tq = make_tmap_2d_bf16(q.data_ptr(), q.stride(1), B * Sq, q.stride(1) * 2, 64, 128);
  const CUtensorMap tk = make_tmap_2d_bf16(k.data_ptr(), k.stride(1), B * Sk, k.stride(1) * 2, 64, 128);
  const CUtensorMap tv = make_tmap_2d_bf16(v.data_ptr(), v.stride(1), B * Sk, v.stride(1) * 2, 64, 128);
  fa::Params p{};
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.o_bs = out.stride(0);
  p.o_rs = out.stride(1);
  p.lse = (lse && lse->defined()) ? lse->data_ptr<float>() : nullptr;
  p.B = (int)B;
  p.Hq = (int)Hq;
  p.Hkv = (int)Hkv;
  p.Sq = (int)Sq;
  p.Sk = (int)Sk;
  p.scale_log2 = (float)scale * fa::kLog2e;
  p.causal = causal ? 1 : 0;
  p.causal_offset = (int)causal_offset;
  p.window = (int)window;
  if (softcap > 0.0) {
    p.cap_in = (float)(scale / softcap);
    p.cap_out = (float)softcap * fa::kLog2e;
  }
  p.status = device_status_word();
  static bool attr_set[64] = {false};
  const int dev = current_device();
  if (!attr_set[dev]) {
    AETHER_CUDA_CHECK(
        cudaFuncSetAttribute(fa::fa_fwd_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, fa::kSmem));
    AETHER_CUDA_CHECK(
        cudaFuncSetAttribute(fa::fa_fwd_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, fa::kSmem));
    attr_set[dev] = true;
  }
  dim3 grid((unsigned)((Sq + fa::BM - 1) / fa::BM), (unsigned)(B * Hq));
  // AETHER_FA_FWD_POLY=1 moves a quarter of the exponentials to the FMA pipe
  // (measured slower here: the SFU is not the limiter; kept for A/B runs)
  static const bool poly = [] {
    const char* e = std::getenv("AETHER_FA_FWD_POLY");
    return e != nullptr && std::string(e) == "1";
  }();
  if (poly)
    fa::fa_fwd_kernel<true><<<grid, fa::kThreads, fa::kSmem, at::cuda::getCurrentCUDAStream()>>>(tq, tk, tv, p);
  else
    fa::fa_fwd_kernel<false><<<grid, fa::kThreads, fa::kSmem, at::cuda::getCurrentCUDAStream()>>>(tq, tk, tv, p);
  AETHER_CUDA_CHECK(cudaGetLastError());
}

}  // namespace aether
