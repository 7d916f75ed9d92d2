// Flash-attention backward on the sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// One CTA owns 128 keys of one KV head and walks every (query head of its GQA
// group, 128-query tile) pair:
//   S^T  = K Q^T          SS MMA -> TMEM (lanes = keys)
//   dP^T = V dO^T         SS MMA -> TMEM
//   P^T  = exp2(S^T*c - lse), dS^T = P^T (dP^T - rowsum(dO*O))   [one thread per key]
//          both written back to TMEM as bf16; dS^T also to shared memory
//   dV  += P^T dO         TS MMA (A = P^T from TMEM)
//   dK  += dS^T Q         TS MMA (A = dS^T from TMEM)
//   dQ   = dS K           SS MMA (A = dS from shared memory, MN-major)
//          -> fp32 partial, reduced into the global dQ accumulator with TMA
//             reduce-add (the L2 adds; no atomics from the SM)
// TMEM columns: S^T / P^T / dQ [0,128), dP^T / dS^T [128,256), dV [256,384),
// dK [384,512). Warp 0 loads (K, V once; Q, dO double-buffered), warp 1 issues
// the MMAs, warps 2..9 (two groups over query-column halves) do the
// elementwise work and the dQ / dK / dV epilogues.
//
// Reference counterpart: sdpa_causal_bwd_dq / sdpa_causal_bwd_dkv
// (runtime/src/cuda.rs:6787-6854), which read a materialised [bh, s, s]
// probability matrix and a d_scores scratch.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cstdlib>
#include <string>

#include "common.cuh"
#include "host_utils.h"

namespace aether {
namespace fab {

constexpr int BK = 128;  // keys per CTA
constexpr int BQ = 128;  // queries per tile
constexpr int D = 128;
constexpr int kThreads = 320;  // producer, MMA, 8 compute warps (two column halves)
constexpr int kCompute = 256;
constexpr int TILE = 128 * D * 2;  // 32 KB, two 128B-swizzled 64-column halves
constexpr int kSmem = TILE * 7 + 1024 + 512 + 1024;  // K, V, Q x2, dO x2, dS, barriers, lse/dsum
constexpr float kLog2e = 1.4426950408889634f;

struct Params {
  const float* lse;   // [B, Hq, Sq] natural log
  const float* dsum;  // [B, Hq, Sq]
  __nv_bfloat16 *dk, *dv;
  int64_t dk_bs, dk_rs, dv_bs, dv_rs;
  int B, Hq, Hkv, Sq, Sk;
  float scale_log2, scale;
  int causal, causal_offset;
  int* status;
};

__device__ __forceinline__ void tmem_st16b(uint32_t taddr, const uint32_t (&r)[16]) { tmem_st16(taddr, r); }

__device__ __forceinline__ void load_tile(uint8_t* dst, const CUtensorMap* map, uint64_t* bar, int x0, int y0) {
  tma_load_2d(dst, map, bar, x0, y0);
  tma_load_2d(dst + TILE / 2, map, bar, x0 + 64, y0);
}

__device__ __forceinline__ void named_barrier_compute() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// 2^x on the SFU (ex2.approx.ftz.f32, relative error about 2^-22): probabilities
// are rounded to bf16 right after.
__device__ __forceinline__ float ex2_sfu(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__global__ void __launch_bounds__(kThreads, 1)
    fa_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                  const __grid_constant__ CUtensorMap tmDQ, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = sK + TILE;
  uint8_t* sQ = sV + TILE;       // [2]
  uint8_t* sDO = sQ + 2 * TILE;  // [2]
  uint8_t* sDS = sDO + 2 * TILE; // dS (MN-major A of the dQ MMA), then dQ staging
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDS + TILE);
  uint64_t* kv_full = bars;
  uint64_t* q_full = bars + 1;     // [2]
  uint64_t* do_full = q_full + 2;  // [2]
  uint64_t* qdo_empty = do_full + 2;  // [2]
  uint64_t* s_full = qdo_empty + 2;
  uint64_t* dp_full = s_full + 1;
  uint64_t* ds_ready = dp_full + 1;
  uint64_t* dq_full = ds_ready + 1;
  uint64_t* dq_read = dq_full + 1;
  uint64_t* kv_done = dq_read + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(kv_done + 1);
  volatile int* abort_word = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* s_lse = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + 512);  // [128] lse * log2(e)
  float* s_dsum = s_lse + BQ;                                                       // [128]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kb = blockIdx.x;
  const int b = blockIdx.y / p.Hkv, hk = blockIdx.y % p.Hkv;
  const int group = p.Hq / p.Hkv;
  const int k0 = kb * BK;
  int i_start = 0;
  if (p.causal) i_start = max(0, k0 - p.causal_offset) / BQ;
  const int n_q = (p.Sq + BQ - 1) / BQ;
  const int per_head = max(0, n_q - i_start);
  const int n_it = per_head * group;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&do_full[i], 1);
      mbar_init(&qdo_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(dp_full, 1);
    mbar_init(ds_ready, kCompute);
    mbar_init(dq_full, 1);
    mbar_init(dq_read, kCompute);
    mbar_init(kv_done, 1);
    *abort_word = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmDO);
    tma_prefetch_desc(&tmDQ);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tDP = tmem + 128, tDV = tmem + 256, tDK = tmem + 384;

  if (warp == 0) {
    if (lane == 0 && n_it > 0) {
      // ------------------------------------------------------------ producer
      mbar_arrive_expect_tx(kv_full, 2 * TILE);
      load_tile(sK, &tmK, kv_full, hk * D, b * p.Sk + k0);
      load_tile(sV, &tmV, kv_full, hk * D, b * p.Sk + k0);
      bool ok = true;
      for (int it = 0; it < n_it && ok; ++it) {
        const int st = it & 1;
        const int hq = hk * group + it / per_head;
        const int q0 = (i_start + it % per_head) * BQ;
        if (!mbar_wait(&qdo_empty[st], ((it >> 1) & 1u) ^ 1u, abort_word)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&q_full[st], TILE);
        load_tile(sQ + st * TILE, &tmQ, &q_full[st], hq * D, b * p.Sq + q0);
        mbar_arrive_expect_tx(&do_full[st], TILE);
        load_tile(sDO + st * TILE, &tmDO, &do_full[st], hq * D, b * p.Sq + q0);
      }
      if (!ok) {
        *abort_word = 1;
        atomicExch(p.status, kStatusTimeoutProducer);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && n_it > 0) {
      // ------------------------------------------------------------ MMA issuer
      constexpr uint32_t id_ss = idesc_bf16_f32(128, 128, false, false);  // K-major A and B
      constexpr uint32_t id_ts = idesc_bf16_f32(128, 128, false, true);   // TMEM A, MN-major B
      constexpr uint32_t id_dq = idesc_bf16_f32(128, 128, true, true);    // MN-major A and B
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV), ds_addr = smem_u32(sDS);
      bool ok = mbar_wait(kv_full, 0, abort_word);
      for (int it = 0; it < n_it && ok; ++it) {
        const int st = it & 1;
        const uint32_t ph = it & 1;
        if (!mbar_wait(&q_full[st], (it >> 1) & 1u, abort_word)) { ok = false; break; }
        if (it > 0 && !mbar_wait(dq_read, ph ^ 1u, abort_word)) { ok = false; break; }
        tc_fence_after();
        const uint32_t q_addr = smem_u32(sQ + st * TILE), do_addr = smem_u32(sDO + st * TILE);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (TILE / 2) + (kk & 3) * 32;
          umma_f16(tS, sdesc_sw128(k_addr + off, 16, 1024), sdesc_sw128(q_addr + off, 16, 1024), id_ss, kk != 0);
        }
        umma_commit(s_full);
        if (!mbar_wait(&do_full[st], (it >> 1) & 1u, abort_word)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (TILE / 2) + (kk & 3) * 32;
          umma_f16(tDP, sdesc_sw128(v_addr + off, 16, 1024), sdesc_sw128(do_addr + off, 16, 1024), id_ss, kk != 0);
        }
        umma_commit(dp_full);
        if (!mbar_wait(ds_ready, ph, abort_word)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk)
          umma_f16_ts(tDV, tS + (kk >> 1) * 32 + (kk & 1) * 8, sdesc_sw128(do_addr + kk * 2048, TILE / 2, 1024), id_ts,
                      (it | kk) != 0);
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk)
          umma_f16_ts(tDK, tDP + (kk >> 1) * 32 + (kk & 1) * 8, sdesc_sw128(q_addr + kk * 2048, TILE / 2, 1024), id_ts,
                      (it | kk) != 0);
        umma_commit(&qdo_empty[st]);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)
          umma_f16(tS, sdesc_sw128(ds_addr + kk * 2048, TILE / 2, 1024), sdesc_sw128(k_addr + kk * 2048, TILE / 2, 1024),
                   id_dq, kk != 0);
        umma_commit(dq_full);
      }
      if (!ok) {
        *abort_word = 1;
        atomicExch(p.status, kStatusTimeoutMma);
      }
      umma_commit(kv_done);  // also drains every MMA issued above
      volatile int never = 0;
      mbar_wait(kv_done, 0, &never);
    }
  } else {
    // -------------------------------------------------------------- compute warps
    // Warps 2..9: TMEM lane quadrant = warp % 4, column half = (warp - 2) / 4.
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int ctid = threadIdx.x - 64;  // 0..255
    const int r = quad * 32 + lane;  // key row (S^T / dP^T lanes) or query row (dQ lanes)
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const int key = k0 + r;
    bool ok = true;
    for (int it = 0; it < n_it; ++it) {
      const uint32_t ph = it & 1;
      const int hq = hk * group + it / per_head;
      const int q0 = (i_start + it % per_head) * BQ;
      const int64_t row_base = ((int64_t)b * p.Hq + hq) * p.Sq;
      if (ctid < BQ) {
        const int q = q0 + ctid;
        s_lse[ctid] = q < p.Sq ? p.lse[row_base + q] * kLog2e : 0.f;
        s_dsum[ctid] = q < p.Sq ? p.dsum[row_base + q] : 0.f;
      }
      named_barrier_compute();
      if (!mbar_wait(s_full, ph, abort_word) || !mbar_wait(dp_full, ph, abort_word)) {
        ok = false;
        break;
      }
      __syncwarp();
      tc_fence_after();
#pragma unroll 1
      for (int cc = 0; cc < 2; ++cc) {
        const int c = half * 2 + cc;  // 32-query chunk
        uint32_t rs[32], rd[32];
        tmem_ld32(tS + lane_off + c * 32, rs);
        tmem_ld32(tDP + lane_off + c * 32, rd);
        tmem_ld_wait();
        uint32_t pp[16], pd[16];
#pragma unroll
        for (int t = 0; t < 32; t += 2) {
          float pv[2], dv[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int ql = c * 32 + t + u;
            const int q = q0 + ql;
            bool valid = q < p.Sq && key < p.Sk;
            if (p.causal && key > q + p.causal_offset) valid = false;
            const float pe = valid ? exp2f(__uint_as_float(rs[t + u]) * p.scale_log2 - s_lse[ql]) : 0.f;
            pv[u] = pe;
            dv[u] = pe * (__uint_as_float(rd[t + u]) - s_dsum[ql]);
          }
          pp[t / 2] = pack_bf16(pv[0], pv[1]);
          pd[t / 2] = pack_bf16(dv[0], dv[1]);
        }
        // packed bf16 of query chunk c goes to the first 16 columns of that
        // chunk's own S^T / dP^T columns, so the two column halves never write
        // TMEM the other half still has to read
        tmem_st16b(tS + lane_off + c * 32, pp);
        tmem_st16b(tDP + lane_off + c * 32, pd);
        // dS^T row (this key) into the MN-major A tile of the dQ MMA:
        // queries [64h, 64h+64) of key row r live at h*16KB + r*128, 16 B granules XOR (r & 7)
        uint8_t* dst = sDS + (c >> 1) * (TILE / 2) + r * 128;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const int gran = (c & 1) * 4 + g;
          *reinterpret_cast<uint4*>(dst + ((gran ^ (r & 7)) << 4)) =
              make_uint4(pd[g * 4 + 0], pd[g * 4 + 1], pd[g * 4 + 2], pd[g * 4 + 3]);
        }
      }
      fence_async_smem();
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(ds_ready);
      // dQ tile (lanes = queries) -> 32 x 32 fp32 slabs -> TMA reduce-add into the global accumulator
      if (!mbar_wait(dq_full, ph, abort_word)) {
        ok = false;
        break;
      }
      __syncwarp();
      tc_fence_after();
      uint8_t* slab = sDS + (warp - 2) * 4096;
#pragma unroll 1
      for (int cc = 0; cc < 2; ++cc) {
        const int c = half * 2 + cc;
        uint32_t rq[32];
        tmem_ld32(tS + lane_off + c * 32, rq);
        tmem_ld_wait();
        if (lane == 0) bulk_wait_read<0>();
        __syncwarp();
#pragma unroll
        for (int g = 0; g < 8; ++g)
          *reinterpret_cast<uint4*>(slab + lane * 128 + ((g ^ (lane & 7)) << 4)) =
              make_uint4(rq[g * 4 + 0], rq[g * 4 + 1], rq[g * 4 + 2], rq[g * 4 + 3]);
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_reduce_add_2d(&tmDQ, slab, hq * D + c * 32, b * p.Sq + q0 + quad * 32);
          bulk_commit();
        }
      }
      tc_fence_before();
      mbar_arrive(dq_read);
      if (lane == 0) bulk_wait_read<0>();  // staging is reused for the next tile's dS
      named_barrier_compute();
    }
    if (!ok) {
      *abort_word = 1;
      if (lane == 0) atomicExch(p.status, kStatusTimeoutEpilogue);
    } else {
      // dK (scaled) and dV: this warp writes head-dim columns [64*half, 64*half + 64) of its key rows
      if (n_it > 0) {
        mbar_wait(kv_done, 0, abort_word);
        __syncwarp();
        tc_fence_after();
      }
      __nv_bfloat16* dkr = p.dk + (int64_t)b * p.dk_bs + (int64_t)key * p.dk_rs + (int64_t)hk * D;
      __nv_bfloat16* dvr = p.dv + (int64_t)b * p.dv_bs + (int64_t)key * p.dv_rs + (int64_t)hk * D;
#pragma unroll 1
      for (int cc = 0; cc < 2; ++cc) {
        const int c = half * 2 + cc;
        uint32_t a[32], v[32];
        if (n_it > 0) {
          tmem_ld32(tDK + lane_off + c * 32, a);
          tmem_ld32(tDV + lane_off + c * 32, v);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int t = 0; t < 32; ++t) a[t] = v[t] = 0u;
        }
        if (key < p.Sk) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 o, w;
            o.x = pack_bf16(__uint_as_float(a[q * 8 + 0]) * p.scale, __uint_as_float(a[q * 8 + 1]) * p.scale);
            o.y = pack_bf16(__uint_as_float(a[q * 8 + 2]) * p.scale, __uint_as_float(a[q * 8 + 3]) * p.scale);
            o.z = pack_bf16(__uint_as_float(a[q * 8 + 4]) * p.scale, __uint_as_float(a[q * 8 + 5]) * p.scale);
            o.w = pack_bf16(__uint_as_float(a[q * 8 + 6]) * p.scale, __uint_as_float(a[q * 8 + 7]) * p.scale);
            w.x = pack_bf16(__uint_as_float(v[q * 8 + 0]), __uint_as_float(v[q * 8 + 1]));
            w.y = pack_bf16(__uint_as_float(v[q * 8 + 2]), __uint_as_float(v[q * 8 + 3]));
            w.z = pack_bf16(__uint_as_float(v[q * 8 + 4]), __uint_as_float(v[q * 8 + 5]));
            w.w = pack_bf16(__uint_as_float(v[q * 8 + 6]), __uint_as_float(v[q * 8 + 7]));
            *reinterpret_cast<uint4*>(dkr + c * 32 + q * 8) = o;
            *reinterpret_cast<uint4*>(dvr + c * 32 + q * 8) = w;
          }
        }
      }
    }
    if (lane == 0) bulk_wait<0>();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}


// ---------------------------------------------------------------------------
// Pipelined variant: 64-query tiles and two TMEM stages, so the tensor core
// computes tile j+1's S^T / dP^T and tile j's dV / dK / dQ while the compute
// warps turn tile j's scores into P^T / dS^T and write tile j-1's dQ out.
//   TMEM stage s in {0,1}: S^T / P^T at [128s, 128s+64), dP^T / dS^T / dQ^T at
//   [128s+64, 128s+128); dV at [256,384), dK at [384,512).
//   dQ^T = K^T dS^T (M = head dim, N = 64 queries) lands over the consumed
//   dS^T, so the next tile's S^T needs no wait and only its dP^T waits for the
//   dQ read-out.
//   MMA order: S/dP(0), S/dP(1), then per tile j: dV(j), dK(j), dQ^T(j)
//   [after ds_ready(j)], S(j+2), dP(j+2) [after dq_read(j)].
//   Compute order: P/dS(j) (P from S^T before waiting on dP^T), then the dQ
//   read-out of tile j-1.
// Q / dO stream through three shared-memory stages; dS^T has two.
constexpr int PQ = 64;                  // queries per tile
constexpr int QTILE = PQ * D * 2;       // 16 KB: two 8 KB 64-column halves
constexpr int DSTILE = BK * PQ * 2;     // 16 KB: [128 keys][64 queries]
constexpr int kQStages = 3;
constexpr int kPipeSmem = 2 * TILE + 2 * kQStages * QTILE + 2 * DSTILE + 8 * 4096 + 1024 + 1024 + 1024;

__global__ void __launch_bounds__(kThreads, 1)
    fa_bwd_pipe_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                       const __grid_constant__ CUtensorMap tmDQ, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = sK + TILE;
  uint8_t* sQ = sV + TILE;                   // [kQStages]
  uint8_t* sDO = sQ + kQStages * QTILE;      // [kQStages]
  uint8_t* sDS = sDO + kQStages * QTILE;     // [2] dS^T (MN-major B of the dQ^T MMA)
  uint8_t* sSlab = sDS + 2 * DSTILE;         // 8 x 4 KB dQ staging (one per compute warp)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sSlab + 8 * 4096);
  uint64_t* kv_full = bars;
  uint64_t* q_full = bars + 1;                  // [3]
  uint64_t* do_full = q_full + kQStages;        // [3]
  uint64_t* qdo_empty = do_full + kQStages;     // [3]
  uint64_t* s_full = qdo_empty + kQStages;      // [2]
  uint64_t* dp_full = s_full + 2;               // [2]
  uint64_t* ds_ready = dp_full + 2;             // [2]
  uint64_t* dq_full = ds_ready + 2;             // [2]
  uint64_t* dq_read = dq_full + 2;              // [2]
  uint64_t* kv_done = dq_read + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(kv_done + 1);
  volatile int* abort_word = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* s_lse = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + 1024);  // [2][64] lse * log2(e)
  float* s_dsum = s_lse + 2 * PQ;                                                     // [2][64]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kb = blockIdx.y;  // grid (B * Hkv, key blocks): the heaviest (first) key blocks launch first
  const int b = blockIdx.x / p.Hkv, hk = blockIdx.x % p.Hkv;
  const int group = p.Hq / p.Hkv;
  const int k0 = kb * BK;
  int i_start = 0;
  if (p.causal) i_start = max(0, k0 - p.causal_offset) / PQ;
  const int n_q = (p.Sq + PQ - 1) / PQ;
  const int per_head = max(0, n_q - i_start);
  const int n_it = per_head * group;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < kQStages; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&do_full[i], 1);
      mbar_init(&qdo_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&dp_full[i], 1);
      mbar_init(&ds_ready[i], kCompute);
      mbar_init(&dq_full[i], 1);
      mbar_init(&dq_read[i], kCompute);
    }
    mbar_init(kv_done, 1);
    *abort_word = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmDO);
    tma_prefetch_desc(&tmDQ);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tDV = tmem + 256, tDK = tmem + 384;

  if (warp == 0) {
    if (lane == 0 && n_it > 0) {
      // ------------------------------------------------------------ producer
      mbar_arrive_expect_tx(kv_full, 2 * TILE);
      load_tile(sK, &tmK, kv_full, hk * D, b * p.Sk + k0);
      load_tile(sV, &tmV, kv_full, hk * D, b * p.Sk + k0);
      bool ok = true;
      for (int it = 0; it < n_it && ok; ++it) {
        const int st = it % kQStages;
        const int hq = hk * group + it / per_head;
        const int q0 = (i_start + it % per_head) * PQ;
        if (!mbar_wait(&qdo_empty[st], ((it / kQStages) & 1u) ^ 1u, abort_word)) {
          ok = false;
          break;
        }
        uint8_t* q = sQ + st * QTILE;
        uint8_t* o = sDO + st * QTILE;
        mbar_arrive_expect_tx(&q_full[st], QTILE);
        tma_load_2d(q, &tmQ, &q_full[st], hq * D, b * p.Sq + q0);
        tma_load_2d(q + QTILE / 2, &tmQ, &q_full[st], hq * D + 64, b * p.Sq + q0);
        mbar_arrive_expect_tx(&do_full[st], QTILE);
        tma_load_2d(o, &tmDO, &do_full[st], hq * D, b * p.Sq + q0);
        tma_load_2d(o + QTILE / 2, &tmDO, &do_full[st], hq * D + 64, b * p.Sq + q0);
      }
      if (!ok) {
        *abort_word = 1;
        atomicExch(p.status, kStatusTimeoutProducer);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && n_it > 0) {
      // ------------------------------------------------------------ MMA issuer
      constexpr uint32_t id_s = idesc_bf16_f32(128, PQ, false, false);  // S^T, dP^T: K-major A and B
      constexpr uint32_t id_ts = idesc_bf16_f32(128, 128, false, true); // dV, dK: TMEM A, MN-major B
      constexpr uint32_t id_dq = idesc_bf16_f32(128, PQ, true, true);   // dQ^T = K^T dS^T: MN-major A and B
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV);
      auto issue_s = [&](int j) -> bool {  // S^T(j) into stage j & 1
        const int st = j % kQStages;
        if (!mbar_wait(&q_full[st], (j / kQStages) & 1u, abort_word)) return false;
        tc_fence_after();
        const uint32_t q_addr = smem_u32(sQ + st * QTILE), tS = tmem + (j & 1) * 128;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_f16(tS, sdesc_sw128(k_addr + (kk >> 2) * (TILE / 2) + (kk & 3) * 32, 16, 1024),
                   sdesc_sw128(q_addr + (kk >> 2) * (QTILE / 2) + (kk & 3) * 32, 16, 1024), id_s, kk != 0);
        umma_commit(&s_full[j & 1]);
        return true;
      };
      auto issue_dp = [&](int j) -> bool {  // dP^T(j) into stage j & 1
        const int st = j % kQStages;
        if (!mbar_wait(&do_full[st], (j / kQStages) & 1u, abort_word)) return false;
        tc_fence_after();
        const uint32_t do_addr = smem_u32(sDO + st * QTILE), tDP = tmem + (j & 1) * 128 + 64;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_f16(tDP, sdesc_sw128(v_addr + (kk >> 2) * (TILE / 2) + (kk & 3) * 32, 16, 1024),
                   sdesc_sw128(do_addr + (kk >> 2) * (QTILE / 2) + (kk & 3) * 32, 16, 1024), id_s, kk != 0);
        umma_commit(&dp_full[j & 1]);
        return true;
      };
      bool ok = mbar_wait(kv_full, 0, abort_word);
      ok = ok && issue_s(0) && issue_dp(0);
      if (ok && n_it > 1) ok = issue_s(1) && issue_dp(1);
      for (int j = 0; j < n_it && ok; ++j) {
        const int s = j & 1, st = j % kQStages;
        const uint32_t tS = tmem + s * 128, tDP = tS + 64;
        if (!mbar_wait(&ds_ready[s], (j >> 1) & 1u, abort_word)) { ok = false; break; }
        tc_fence_after();
        const uint32_t q_addr = smem_u32(sQ + st * QTILE), do_addr = smem_u32(sDO + st * QTILE);
        const uint32_t ds_addr = smem_u32(sDS + s * DSTILE);
#pragma unroll
        for (int kk = 0; kk < PQ / 16; ++kk)
          umma_f16_ts(tDV, tS + (kk >> 1) * 32 + (kk & 1) * 8, sdesc_sw128(do_addr + kk * 2048, QTILE / 2, 1024),
                      id_ts, (j | kk) != 0);
#pragma unroll
        for (int kk = 0; kk < PQ / 16; ++kk)
          umma_f16_ts(tDK, tDP + (kk >> 1) * 32 + (kk & 1) * 8, sdesc_sw128(q_addr + kk * 2048, QTILE / 2, 1024),
                      id_ts, (j | kk) != 0);
        umma_commit(&qdo_empty[st]);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)
          umma_f16(tDP, sdesc_sw128(k_addr + kk * 2048, TILE / 2, 1024), sdesc_sw128(ds_addr + kk * 2048, DSTILE, 1024),
                   id_dq, kk != 0);
        umma_commit(&dq_full[s]);
        if (j + 2 < n_it) {
          if (!issue_s(j + 2)) { ok = false; break; }
          if (!mbar_wait(&dq_read[s], (j >> 1) & 1u, abort_word)) { ok = false; break; }
          if (!issue_dp(j + 2)) { ok = false; break; }
        }
      }
      if (!ok) {
        *abort_word = 1;
        atomicExch(p.status, kStatusTimeoutMma);
      }
      umma_commit(kv_done);  // also drains every MMA issued above
      volatile int never = 0;
      mbar_wait(kv_done, 0, &never);
    }
  } else {
    // -------------------------------------------------------------- compute warps
    // Warps 2..9: TMEM lane quadrant = warp % 4, query half (32 of the 64) = (warp - 2) / 4.
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int ctid = threadIdx.x - 64;  // 0..255
    const int r = quad * 32 + lane;     // key row (S^T / dP^T lanes) or head-dim row (dQ^T lanes)
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const int key = k0 + r;
    uint8_t* slab = sSlab + (warp - 2) * 4096;
    bool ok = true;
    // dQ^T of tile jj (lanes = head dims, 32 query columns of this half) -> TMA reduce-add
    auto dq_out = [&](int jj) -> bool {
      const int s = jj & 1;
      const int hq = hk * group + jj / per_head;
      const int q0 = (i_start + jj % per_head) * PQ;
      if (!mbar_wait(&dq_full[s], (jj >> 1) & 1u, abort_word)) return false;
      __syncwarp();
      tc_fence_after();
      uint32_t rq[32];
      tmem_ld32(tmem + s * 128 + 64 + lane_off + half * 32, rq);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&dq_read[s]);  // the TMEM columns may now take the next dP^T
      if (lane == 0) bulk_wait_read<0>();  // the previous reduce has read this slab
      __syncwarp();
      // slab: 32 query rows x 32 head dims (128 B), 16 B granules XOR (row & 7);
      // the eight per-lane granule offsets are computed once
      uint32_t* gofs[8];
#pragma unroll
      for (int g8 = 0; g8 < 8; ++g8)
        gofs[g8] = reinterpret_cast<uint32_t*>(slab + ((((lane >> 2) ^ g8)) << 4) + (lane & 3) * 4);
#pragma unroll
      for (int t = 0; t < 32; ++t) gofs[t & 7][t * 32] = rq[t];
      fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_reduce_add_2d(&tmDQ, slab, hq * D + quad * 32, b * p.Sq + q0 + half * 32);
        bulk_commit();
      }
      return true;
    };
    // lse / dsum of tile jj (threads 0..63 of the compute group), fetched one
    // tile ahead into registers so no barrier waits on their global latency
    auto fetch = [&](int jj, float& l, float& d) {
      const int hq = hk * group + jj / per_head;
      const int q = (i_start + jj % per_head) * PQ + ctid;
      const int64_t idx = ((int64_t)b * p.Hq + hq) * p.Sq + q;
      l = q < p.Sq ? __ldg(p.lse + idx) * kLog2e : 0.f;
      d = q < p.Sq ? __ldg(p.dsum + idx) : 0.f;
    };
    float nl = 0.f, nd = 0.f;
    if (ctid < PQ && n_it > 0) {
      fetch(0, nl, nd);
      s_lse[ctid] = nl;
      s_dsum[ctid] = nd;
      if (n_it > 1) fetch(1, nl, nd);
    }
    for (int it = 0; it < n_it; ++it) {
      const int s = it & 1;
      const uint32_t ph = (it >> 1) & 1u;
      const int q0 = (i_start + it % per_head) * PQ;
      float* lse_s = s_lse + s * PQ;
      float* dsum_s = s_dsum + s * PQ;
      named_barrier_compute();  // stage s holds tile it's lse / dsum
      if (ctid < PQ && it + 1 < n_it) {  // stage s ^ 1 (tile it - 1) is no longer read
        s_lse[(s ^ 1) * PQ + ctid] = nl;
        s_dsum[(s ^ 1) * PQ + ctid] = nd;
        if (it + 2 < n_it) fetch(it + 2, nl, nd);
      }
      const uint32_t tS = tmem + s * 128, tDP = tS + 64;
      if (!mbar_wait(&s_full[s], ph, abort_word)) {
        ok = false;
        break;
      }
      __syncwarp();
      tc_fence_after();
      uint32_t rs[32], pp[16];
      tmem_ld32(tS + lane_off + half * 32, rs);
      tmem_ld_wait();
      float pv[32];
      // this thread's 32 queries are q0 + half*32 + [0, 32); visible ones form [lo, hi)
      const int qb = q0 + half * 32;
      const int lo = p.causal ? key - p.causal_offset - qb : 0;  // first visible (causal)
      const int hi = key < p.Sk ? p.Sq - qb : 0;                    // past the last query
      const float4* l4 = reinterpret_cast<const float4*>(lse_s + half * 32);
      if (lo <= 0 && hi >= 32) {  // the whole row chunk is visible: no per-element masks
#pragma unroll
        for (int t4 = 0; t4 < 8; ++t4) {
          const float4 l = l4[t4];
          pv[4 * t4 + 0] = ex2_sfu(__uint_as_float(rs[4 * t4 + 0]) * p.scale_log2 - l.x);
          pv[4 * t4 + 1] = ex2_sfu(__uint_as_float(rs[4 * t4 + 1]) * p.scale_log2 - l.y);
          pv[4 * t4 + 2] = ex2_sfu(__uint_as_float(rs[4 * t4 + 2]) * p.scale_log2 - l.z);
          pv[4 * t4 + 3] = ex2_sfu(__uint_as_float(rs[4 * t4 + 3]) * p.scale_log2 - l.w);
        }
      } else {
#pragma unroll
        for (int t4 = 0; t4 < 8; ++t4) {
          const float4 l = l4[t4];
          const float lv[4] = {l.x, l.y, l.z, l.w};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int t = 4 * t4 + u;
            pv[t] = (t >= lo && t < hi) ? ex2_sfu(__uint_as_float(rs[t]) * p.scale_log2 - lv[u]) : 0.f;
          }
        }
      }
#pragma unroll
      for (int t = 0; t < 32; t += 2) pp[t / 2] = pack_bf16(pv[t], pv[t + 1]);
      tmem_st16b(tS + lane_off + half * 32, pp);  // P^T over the first 16 columns of this half's own 32
      if (!mbar_wait(&dp_full[s], ph, abort_word)) {
        ok = false;
        break;
      }
      __syncwarp();
      tc_fence_after();
      uint32_t rd[32], pd[16];
      tmem_ld32(tDP + lane_off + half * 32, rd);
      tmem_ld_wait();
      const float4* d4 = reinterpret_cast<const float4*>(dsum_s + half * 32);
#pragma unroll
      for (int t4 = 0; t4 < 8; ++t4) {
        const float4 d = d4[t4];
        const int t = 4 * t4;
        pd[t / 2] = pack_bf16(pv[t] * (__uint_as_float(rd[t]) - d.x), pv[t + 1] * (__uint_as_float(rd[t + 1]) - d.y));
        pd[t / 2 + 1] =
            pack_bf16(pv[t + 2] * (__uint_as_float(rd[t + 2]) - d.z), pv[t + 3] * (__uint_as_float(rd[t + 3]) - d.w));
      }
      tmem_st16b(tDP + lane_off + half * 32, pd);
      // dS^T row (this key) into the [128 keys][64 queries] tile: 16 B granules XOR (r & 7)
      uint8_t* dst = sDS + s * DSTILE + r * 128;
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        const int gran = half * 4 + g;
        *reinterpret_cast<uint4*>(dst + ((gran ^ (r & 7)) << 4)) =
            make_uint4(pd[g * 4 + 0], pd[g * 4 + 1], pd[g * 4 + 2], pd[g * 4 + 3]);
      }
      fence_async_smem();
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&ds_ready[s]);
      if (it > 0 && !dq_out(it - 1)) {
        ok = false;
        break;
      }
    }
    if (ok && n_it > 0 && !dq_out(n_it - 1)) ok = false;
    if (!ok) {
      *abort_word = 1;
      if (lane == 0) atomicExch(p.status, kStatusTimeoutEpilogue);
    } else {
      // dK (scaled) and dV: this warp writes head-dim columns [64*half, 64*half + 64) of its key rows
      if (n_it > 0) {
        mbar_wait(kv_done, 0, abort_word);
        __syncwarp();
        tc_fence_after();
      }
      __nv_bfloat16* dkr = p.dk + (int64_t)b * p.dk_bs + (int64_t)key * p.dk_rs + (int64_t)hk * D;
      __nv_bfloat16* dvr = p.dv + (int64_t)b * p.dv_bs + (int64_t)key * p.dv_rs + (int64_t)hk * D;
#pragma unroll 1
      for (int cc = 0; cc < 2; ++cc) {
        const int c = half * 2 + cc;
        uint32_t a[32], v[32];
        if (n_it > 0) {
          tmem_ld32(tDK + lane_off + c * 32, a);
          tmem_ld32(tDV + lane_off + c * 32, v);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int t = 0; t < 32; ++t) a[t] = v[t] = 0u;
        }
        if (key < p.Sk) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 o, w;
            o.x = pack_bf16(__uint_as_float(a[q * 8 + 0]) * p.scale, __uint_as_float(a[q * 8 + 1]) * p.scale);
            o.y = pack_bf16(__uint_as_float(a[q * 8 + 2]) * p.scale, __uint_as_float(a[q * 8 + 3]) * p.scale);
            o.z = pack_bf16(__uint_as_float(a[q * 8 + 4]) * p.scale, __uint_as_float(a[q * 8 + 5]) * p.scale);
            o.w = pack_bf16(__uint_as_float(a[q * 8 + 6]) * p.scale, __uint_as_float(a[q * 8 + 7]) * p.scale);
            w.x = pack_bf16(__uint_as_float(v[q * 8 + 0]), __uint_as_float(v[q * 8 + 1]));
            w.y = pack_bf16(__uint_as_float(v[q * 8 + 2]), __uint_as_float(v[q * 8 + 3]));
            w.z = pack_bf16(__uint_as_float(v[q * 8 + 4]), __uint_as_float(v[q * 8 + 5]));
            w.w = pack_bf16(__uint_as_float(v[q * 8 + 6]), __uint_as_float(v[q * 8 + 7]));
            *reinterpret_cast<uint4*>(dkr + c * 32 + q * 8) = o;
            *reinterpret_cast<uint4*>(dvr + c * 32 + q * 8) = w;
          }
        }
      }
    }
    if (lane == 0) bulk_wait<0>();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace fab

// Main backward pass on tcgen05 (head_dim 128). lse / dsum fp32 [B, Hq, Sq];
// dq_acc fp32 [B, Sq, Hq, 128] zero-initialised (dS K accumulates into it);
// dk / dv written. Layout contract as attention_fwd_tc.
void attention_bwd_tc(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor dout, at::Tensor lse, at::Tensor dsum,
                      at::Tensor dq_acc, at::Tensor dk, at::Tensor dv, double scale, bool causal,
                      int64_t causal_offset) {
  const int64_t B = q.size(0), Sq = q.size(1), Hq = q.size(2), D = q.size(3);
  const int64_t Sk = k.size(1), Hkv = k.size(2);
  TORCH_CHECK(D == 128, "attention_bwd_tc: head_dim 128");
  for (const at::Tensor* t : {&q, &k, &v, &dout, &dk, &dv}) {
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->dim() == 4, "attention_bwd_tc: bf16 [B,S,H,D]");
    TORCH_CHECK(t->stride(3) == 1 && t->stride(2) == 128 && t->stride(1) % 8 == 0, "attention_bwd_tc: layout");
  }
  TORCH_CHECK(q.stride(0) == Sq * q.stride(1) && k.stride(0) == Sk * k.stride(1) && v.stride(0) == Sk * v.stride(1) &&
                  dout.stride(0) == Sq * dout.stride(1),
              "attention_bwd_tc: batch stride must equal S * row stride");
  TORCH_CHECK(dq_acc.scalar_type() == at::kFloat && dq_acc.is_contiguous() && dq_acc.numel() == B * Sq * Hq * D,
              "attention_bwd_tc: dq_acc fp32 [B, Sq, Hq, D]");
  c10::cuda::CUDAGuard guard(q.device());
  if (B == 0 || Sq == 0 || Sk == 0) return;
  const CUtensorMap tq = make_tmap_2d_bf16(q.data_ptr(), q.stride(1), B * Sq, q.stride(1) * 2, 64, 128);
  const CUtensorMap tk = make_tmap_2d_bf16(k.data_ptr(), k.stride(1), B * Sk, k.stride(1) * 2, 64, 128);
  const CUtensorMap tv = make_tmap_2d_bf16(v.data_ptr(), v.stride(1), B * Sk, v.stride(1) * 2, 64, 128);
  const CUtensorMap tdo = make_tmap_2d_bf16(dout.data_ptr(), dout.stride(1), B * Sq, dout.stride(1) * 2, 64, 128);
  const CUtensorMap tdq = make_tmap_2d(dq_acc.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, Hq * D, B * Sq,
                                       Hq * D * 4, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B);
  fab::Params p{};
  p.lse = lse.data_ptr<float>();
  p.dsum = dsum.data_ptr<float>();
  p.dk = reinterpret_cast<__nv_bfloat16*>(dk.data_ptr());
  p.dv = reinterpret_cast<__nv_bfloat16*>(dv.data_ptr());
  p.dk_bs = dk.stride(0);
  p.dk_rs = dk.stride(1);
  p.dv_bs = dv.stride(0);
  p.dv_rs = dv.stride(1);
  p.B = (int)B;
  p.Hq = (int)Hq;
  p.Hkv = (int)Hkv;
  p.Sq = (int)Sq;
  p.Sk = (int)Sk;
  p.scale_log2 = (float)scale * fab::kLog2e;
  p.scale = (float)scale;
  p.causal = causal ? 1 : 0;
  p.causal_offset = (int)causal_offset;
  p.status = device_status_word();
  static bool attr_set[64] = {false};
  const int dev = current_device();
  if (!attr_set[dev]) {
    AETHER_CUDA_CHECK(cudaFuncSetAttribute(fab::fa_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, fab::kSmem));
    AETHER_CUDA_CHECK(
        cudaFuncSetAttribute(fab::fa_bwd_pipe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, fab::kPipeSmem));
    attr_set[dev] = true;
  }
  dim3 grid((unsigned)((Sk + 127) / 128), (unsigned)(B * Hkv));
  // AETHER_FA_BWD=serial selects the one-stage kernel (A/B comparisons)
  static const bool serial = [] {
    const char* e = std::getenv("AETHER_FA_BWD");
    return e != nullptr && std::string(e) == "serial";
  }();
  if (serial) {
    fab::fa_bwd_kernel<<<grid, fab::kThreads, fab::kSmem, at::cuda::getCurrentCUDAStream()>>>(tq, tk, tv, tdo, tdq, p);
  } else {
    // 64-row boxes for the 64-query Q / dO tiles
    const CUtensorMap tq64 = make_tmap_2d_bf16(q.data_ptr(), q.stride(1), B * Sq, q.stride(1) * 2, 64, fab::PQ);
    const CUtensorMap tdo64 =
        make_tmap_2d_bf16(dout.data_ptr(), dout.stride(1), B * Sq, dout.stride(1) * 2, 64, fab::PQ);
    const dim3 pgrid((unsigned)(B * Hkv), (unsigned)((Sk + 127) / 128));
    fab::fa_bwd_pipe_kernel<<<pgrid, fab::kThreads, fab::kPipeSmem, at::cuda::getCurrentCUDAStream()>>>(
        tq64, tk, tv, tdo64, tdq, p);
  }
  AETHER_CUDA_CHECK(cudaGetLastError());
}

}  // namespace aether
