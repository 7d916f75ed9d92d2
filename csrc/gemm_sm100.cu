// Persistent, warp-specialised bf16 GEMM on the sm_100a tensor cores.
//
//   C[M,N] = alpha * opA(A)[M,K] . opB(B)[N,K]^T  (+ bias[N]) (+ residual[M,N])
//
// Replaces the reference's cuBLAS sgemm family (runtime/src/cuda.rs:7419-7760,
// aether_op_matmul_f32_cuda / _tn_ / _nt_ / backward_lhs / backward_rhs): the
// three training layouts (forward x.W^T, dgrad dy.W, wgrad dy^T.x) are one
// kernel whose A/B operands are either K-major or MN-major in shared memory,
// so no transpose kernel ever runs.
//
// Structure (one CTA per SM, persistent over output tiles):
//   warp 0      : TMA producer -- 128B-swizzled tiles into a 4-stage ring
//   warp 1      : TMEM allocator + MMA issuer (one thread, tcgen05.mma M128 N256 K16)
//   warps 2..5  : epilogue -- tcgen05.ld of the fp32 accumulator, fused bias /
//                 residual / scale, staged through 128B-swizzled shared memory
//                 and written by TMA bulk-tensor stores; fp32 gradient
//                 accumulation uses the TMA reduce-add (the L2 adds, the SM
//                 never reads the old value)
// Two 128x256 fp32 accumulators (all 512 TMEM columns) let the epilogue of tile
// i overlap the main loop of tile i+1.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <ATen/ATen.h>

#include <cstdlib>

#include "common.cuh"
#include "host_utils.h"

namespace aether {
namespace gemm {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int STAGES = 4;
constexpr int kThreads = 192;
constexpr int A_BYTES = BM * BK * 2;  // 16 KB
constexpr int B_BYTES = BN * BK * 2;  // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int kTmemCols = 2 * BN;  // double-buffered accumulator
constexpr int kStageBytes = 32 * 128;          // one epilogue warp's 32-row x 128-byte output slab
constexpr int kStageTotal = 4 * 2 * kStageBytes;  // 4 epilogue warps, double-buffered
constexpr int kSmemBytes = STAGES * STAGE_BYTES + kStageTotal + 1024 /*align slack*/ + 256 /*barriers*/;
constexpr int kGroupM = 16;  // tile raster: groups of 16 M-tiles sweep N together (L2 reuse)

enum OutMode : int { OUT_BF16 = 0, OUT_F32 = 1, OUT_F32_ACCUM = 2 };

struct Params {
  void* out;
  int64_t ldo;
  const __nv_bfloat16* bias;      // [N] or null
  const __nv_bfloat16* residual;  // [M, N] (row stride ldr) or null
  int64_t ldr;
  int M, N, K;
  float alpha;
  const float* alpha_ptr;  // optional device scalar multiplied into alpha
  int* status;
  // Grouped (mixture-of-experts) mode: M-tile tm multiplies A's rows by group
  // tile_group[tm]'s B rows [g * N, (g + 1) * N) of a [groups * N, K] B; a
  // negative entry marks an unused tile, which every role skips.
  const int* tile_group;
};

// B row of the tile's first output column (-1: tile skipped).
__device__ __forceinline__ int b_row(const Params& p, int tm, int tn) {
  if (p.tile_group == nullptr) return tn * BN;
  const int g = p.tile_group[tm];
  return g < 0 ? -1 : g * p.N + tn * BN;
}

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& tm, int& tn) {
  const int per_group = kGroupM * num_n;
  const int g = t / per_group;
  const int first_m = g * kGroupM;
  const int gsize = min(num_m - first_m, kGroupM);
  const int r = t - g * per_group;
  tm = first_m + r % gsize;
  tn = r / gsize;
}

// One accumulator tile of 128 rows x BN columns from TMEM to global memory:
// tcgen05.ld, alpha, bias, residual, bf16 / fp32 conversion, then 32-row x
// 128-byte slabs staged through 128B-swizzled shared memory and written (or
// reduce-added) by TMA. Run by the four epilogue warps; `quad` is the TMEM lane
// quadrant of this warp, `tmem_acc` the accumulator's first column, m_base /
// n_base the tile's first output row / column.
template <int OUT>
__device__ __forceinline__ void epilogue_tile(const Params& p, const CUtensorMap* tmC, uint8_t* sStage,
                                              uint32_t tmem_acc, int m_base, int n_base, int quad, int lane,
                                              float alpha, uint32_t& stage_ctr) {
  const int row = quad * 32 + lane;
  const int m = m_base + row;
  const bool row_ok = m < p.M;
  const int m_warp = m_base + quad * 32;  // first output row of this warp's slab
  // Output chunks are 128 bytes wide per row: 32 fp32 or 64 bf16 columns.
  constexpr int CW = (OUT == OUT_BF16) ? 64 : 32;
#pragma unroll 1
  for (int c = 0; c < BN / CW; ++c) {
    const int n0 = n_base + c * CW;
    float v[CW];
#pragma unroll
    for (int h = 0; h < CW / 32; ++h) {
      uint32_t r[32];
      tmem_ld32(tmem_acc + (static_cast<uint32_t>(quad * 32) << 16) + c * CW + h * 32, r);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 32; ++j) v[h * 32 + j] = __uint_as_float(r[j]) * alpha;
    }
    if (n0 >= p.N) continue;  // whole chunk beyond N (warp-uniform)
    if (p.bias != nullptr) {
      const uint4* bp = reinterpret_cast<const uint4*>(p.bias + n0);
#pragma unroll
      for (int q = 0; q < CW / 8; ++q) {
        if (n0 + q * 8 < p.N) {
          const uint4 b = bp[q];
          v[q * 8 + 0] += bf16lo(b.x); v[q * 8 + 1] += bf16hi(b.x);
          v[q * 8 + 2] += bf16lo(b.y); v[q * 8 + 3] += bf16hi(b.y);
          v[q * 8 + 4] += bf16lo(b.z); v[q * 8 + 5] += bf16hi(b.z);
          v[q * 8 + 6] += bf16lo(b.w); v[q * 8 + 7] += bf16hi(b.w);
        }
      }
    }
    if (p.residual != nullptr && row_ok) {
      const uint4* rp = reinterpret_cast<const uint4*>(p.residual + (int64_t)m * p.ldr + n0);
#pragma unroll
      for (int q = 0; q < CW / 8; ++q) {
        if (n0 + q * 8 < p.N) {
          const uint4 b = rp[q];
          v[q * 8 + 0] += bf16lo(b.x); v[q * 8 + 1] += bf16hi(b.x);
          v[q * 8 + 2] += bf16lo(b.y); v[q * 8 + 3] += bf16hi(b.y);
          v[q * 8 + 4] += bf16lo(b.z); v[q * 8 + 5] += bf16hi(b.z);
          v[q * 8 + 6] += bf16lo(b.w); v[q * 8 + 7] += bf16hi(b.w);
        }
      }
    }
    // Stage this warp's 32 x 128-byte slab (128B-swizzled) and hand it to TMA.
    uint8_t* stage_buf = sStage + (quad * 2 + (stage_ctr & 1)) * kStageBytes;
    if (lane == 0) bulk_wait_read<1>();  // the store that last used this buffer has read it
    __syncwarp();
    uint8_t* my_row = stage_buf + lane * 128;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      uint4 o;
      if constexpr (OUT == OUT_BF16) {
        o.x = pack_bf16(v[q * 8 + 0], v[q * 8 + 1]);
        o.y = pack_bf16(v[q * 8 + 2], v[q * 8 + 3]);
        o.z = pack_bf16(v[q * 8 + 4], v[q * 8 + 5]);
        o.w = pack_bf16(v[q * 8 + 6], v[q * 8 + 7]);
      } else {
        o.x = __float_as_uint(v[q * 4 + 0]);
        o.y = __float_as_uint(v[q * 4 + 1]);
        o.z = __float_as_uint(v[q * 4 + 2]);
        o.w = __float_as_uint(v[q * 4 + 3]);
      }
      *reinterpret_cast<uint4*>(my_row + ((q ^ (lane & 7)) << 4)) = o;
    }
    fence_async_smem();
    __syncwarp();
    if (lane == 0) {
      if constexpr (OUT == OUT_F32_ACCUM) tma_reduce_add_2d(tmC, stage_buf, n0, m_warp);
      else tma_store_2d(tmC, stage_buf, n0, m_warp);
      bulk_commit();
    }
    ++stage_ctr;
  }
}

template <bool A_MN, bool B_MN, int OUT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* sStage = sB + STAGES * B_BYTES;  // 4 warps x 2 buffers x 32 rows x 128 B
  uint64_t* full = reinterpret_cast<uint64_t*>(sStage + kStageTotal);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_word = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (p.M + BM - 1) / BM;
  const int num_n = (p.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_k = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
    mbar_init(drain, 1);
    *abort_word = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int tm, tn;
        tile_coords(t, num_m, num_n, tm, tn);
        const int brow = b_row(p, tm, tn);
        if (brow < 0) continue;
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_word)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          uint8_t* a_dst = sA + stage * A_BYTES;
          uint8_t* b_dst = sB + stage * B_BYTES;
          if constexpr (!A_MN) {
            tma_load_2d(a_dst, &tmA, &full[stage], kb * BK, tm * BM);
          } else {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j) tma_load_2d(a_dst + j * 8192, &tmA, &full[stage], tm * BM + j * 64, kb * BK);
          }
          if constexpr (!B_MN) {
            tma_load_2d(b_dst, &tmB, &full[stage], kb * BK, brow);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_2d(b_dst + j * 8192, &tmB, &full[stage], tn * BN + j * 64, kb * BK);
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        *abort_word = 1;
        atomicExch(p.status, kStatusTimeoutProducer);
        // Let the copies already in flight land before the CTA exits.
        volatile int never = 0;
        const uint32_t n_back = issued < (uint32_t)STAGES ? issued : (uint32_t)STAGES;
        for (uint32_t j = 1; j <= n_back; ++j) {
          const uint32_t i = issued - j;
          mbar_wait(&full[i % STAGES], (i / STAGES) & 1u, &never);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        if (p.tile_group != nullptr) {
          int tm, tn;
          tile_coords(t, num_m, num_n, tm, tn);
          if (b_row(p, tm, tn) < 0) continue;
        }
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_word)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_word)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * A_BYTES);
          const uint32_t b_base = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t adesc = A_MN ? sdesc_sw128(a_base + kk * 2048, 8192, 1024) : sdesc_sw128(a_base + kk * 32, 16, 1024);
            const uint64_t bdesc = B_MN ? sdesc_sw128(b_base + kk * 2048, 8192, 1024) : sdesc_sw128(b_base + kk * 32, 16, 1024);
            umma_f16(d_tmem, adesc, bdesc, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      if (!ok) {
        *abort_word = 1;
        atomicExch(p.status, kStatusTimeoutMma);
      }
      // Drain: every MMA this thread issued has completed before TMEM is freed.
      volatile int never = 0;
      umma_commit(drain);
      mbar_wait(drain, 0, &never);
    }
  } else {
    // -------------------------------------------------------------- epilogue
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const float alpha = p.alpha * (p.alpha_ptr != nullptr ? *p.alpha_ptr : 1.f);
    uint32_t stage_ctr = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      int tm, tn;
      tile_coords(t, num_m, num_n, tm, tn);
      if (b_row(p, tm, tn) < 0) continue;
      if (!mbar_wait(&tfull[acc], acc_phase, abort_word)) {
        *abort_word = 1;
        if (lane == 0) atomicExch(p.status, kStatusTimeoutEpilogue);
        break;
      }
      __syncwarp();
      tc_fence_after();
      epilogue_tile<OUT>(p, &tmC, sStage, tmem_base + acc * BN, tm * BM, tn * BN, quad, lane, alpha, stage_ctr);
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
    if (lane == 0) bulk_wait<0>();  // every output store of this warp has landed
  }

  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// CTA-pair variant: a cluster of two CTAs computes a 256 x 256 output tile with
// tcgen05.mma.cta_group::2 (M = 256, N = 256). Each CTA loads its own 128 rows
// of A and its own 128 rows of B (half of the tile's N) per 64-deep K block, so
// a stage is 32 KB instead of 48 KB and six stages fit; the tensor core reads
// half as many B bytes per FLOP from each SM's shared memory as the one-CTA
// M128 x N256 form. The even CTA's MMA thread issues every MMA; TMA copies of
// both CTAs count their bytes on the even CTA's `full` barriers; MMA
// completion (stage free, accumulator ready) is committed to the barriers of
// both CTAs; each CTA's epilogue drains its own 128 accumulator rows and
// releases the accumulator on the even CTA's barrier. All loads are local (no
// cluster multicast), so the kernel is usable inside multi-GPU training.
constexpr int P_BM = 256;  // rows per pair tile (128 per CTA)
constexpr int P_BN = 256;  // columns per pair tile (B rows: 128 per CTA)
constexpr int P_STAGES = 6;
constexpr int P_HALF_BYTES = 128 * BK * 2;  // 16 KB: one CTA's A or B rows of a K block
constexpr int P_STAGE_BYTES = 2 * P_HALF_BYTES;
constexpr int kPairSmemBytes = P_STAGES * P_STAGE_BYTES + kStageTotal + 1024 + 256;
constexpr int kPairEpiArrivals = 8;  // 4 epilogue warps x 2 CTAs release an accumulator
static_assert(kPairSmemBytes <= 232448, "pair GEMM shared memory");
static_assert(P_BN == BN, "the pair epilogue drains BN accumulator columns per CTA");

template <bool A_MN, bool B_MN, int OUT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + P_STAGES * P_HALF_BYTES;
  uint8_t* sStage = sB + P_STAGES * P_HALF_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sStage + kStageTotal);
  uint64_t* empty = full + P_STAGES;
  uint64_t* tfull = empty + P_STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_word = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0: issues the MMAs
  const int pair = (int)cluster_id_x();
  const int npairs = (int)cluster_count_x();
  const int num_m = (p.M + P_BM - 1) / P_BM;
  const int num_n = (p.N + P_BN - 1) / P_BN;
  const int num_tiles = num_m * num_n;
  const int num_k = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(&full[s], 1);   // the even CTA's producer (expect_tx for both CTAs' bytes)
      mbar_init(&empty[s], 1);  // one MMA commit
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kPairEpiArrivals);
    }
    mbar_init(drain, 1);
    *abort_word = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  // Both CTAs' barriers are initialised before either CTA signals the other's.
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer (both CTAs)
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = pair; t < num_tiles && ok; t += npairs) {
        int tm, tn;
        tile_coords(t, num_m, num_n, tm, tn);
        const int m0 = tm * P_BM + (int)rank * 128;
        const int n0 = tn * P_BN + (int)rank * 128;
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_word)) {
            ok = false;
            break;
          }
          const uint32_t bar = mapa_shared(smem_u32(&full[stage]), 0);
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * P_STAGE_BYTES);
          uint8_t* a_dst = sA + stage * P_HALF_BYTES;
          uint8_t* b_dst = sB + stage * P_HALF_BYTES;
          if constexpr (!A_MN) {
            tma_load_2d_pair(a_dst, &tmA, bar, kb * BK, m0);
          } else {
            tma_load_2d_pair(a_dst, &tmA, bar, m0, kb * BK);
            tma_load_2d_pair(a_dst + 8192, &tmA, bar, m0 + 64, kb * BK);
          }
          if constexpr (!B_MN) {
            tma_load_2d_pair(b_dst, &tmB, bar, kb * BK, n0);
          } else {
            tma_load_2d_pair(b_dst, &tmB, bar, n0, kb * BK);
            tma_load_2d_pair(b_dst + 8192, &tmB, bar, n0 + 64, kb * BK);
          }
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        *abort_word = 1;
        atomicExch(p.status, kStatusTimeoutProducer);
        // Copies in flight complete on the even CTA's barriers, which this CTA
        // cannot observe: give them a fixed time to land before leaving.
        const uint64_t t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 2000000ull) {
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ------------------------------------------------------------ MMA issuer (even CTA)
      constexpr uint32_t idesc = idesc_bf16_f32(P_BM, P_BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = pair; t < num_tiles && ok; t += npairs) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_word)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * P_BN;
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_word)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * P_HALF_BYTES);
          const uint32_t b_base = smem_u32(sB + stage * P_HALF_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t adesc = A_MN ? sdesc_sw128(a_base + kk * 2048, 8192, 1024) : sdesc_sw128(a_base + kk * 32, 16, 1024);
            const uint64_t bdesc = B_MN ? sdesc_sw128(b_base + kk * 2048, 8192, 1024) : sdesc_sw128(b_base + kk * 32, 16, 1024);
            umma_f16_pair(d_tmem, adesc, bdesc, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          umma_commit_pair(&empty[stage], 0x3);  // the stage is free in both CTAs
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair(&tfull[acc], 0x3);  // both CTAs' accumulator rows are final
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      if (!ok) {
        *abort_word = 1;
        atomicExch(p.status, kStatusTimeoutMma);
      }
      // Drain: every MMA issued has completed before either CTA frees TMEM.
      volatile int never = 0;
      umma_commit_pair(drain, 0x1);
      mbar_wait(drain, 0, &never);
    }
  } else {
    // -------------------------------------------------------------- epilogue (both CTAs)
    const int quad = warp & 3;
    const float alpha = p.alpha * (p.alpha_ptr != nullptr ? *p.alpha_ptr : 1.f);
    uint32_t stage_ctr = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = pair; t < num_tiles; t += npairs) {
      int tm, tn;
      tile_coords(t, num_m, num_n, tm, tn);
      if (!mbar_wait(&tfull[acc], acc_phase, abort_word)) {
        *abort_word = 1;
        if (lane == 0) atomicExch(p.status, kStatusTimeoutEpilogue);
        break;
      }
      __syncwarp();
      tc_fence_after();
      epilogue_tile<OUT>(p, &tmC, sStage, tmem_base + acc * P_BN, tm * P_BM + (int)rank * 128, tn * P_BN, quad,
                         lane, alpha, stage_ctr);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[acc]), 0));
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
    if (lane == 0) bulk_wait<0>();
  }

  // Neither CTA frees TMEM or leaves while the pair's MMAs, copies or
  // barrier signals may still reach it.
  __syncwarp();
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

template <bool A_MN, bool B_MN, int OUT>
static void launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const Params& p,
                   cudaStream_t stream) {
  auto kern = gemm_bf16_kernel<A_MN, B_MN, OUT>;
  static bool attr_set[64] = {false};
  const int dev = current_device();
  if (!attr_set[dev]) {
    AETHER_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
    attr_set[dev] = true;
  }
  const int num_tiles = ((p.M + BM - 1) / BM) * ((p.N + BN - 1) / BN);
  const int grid = std::min(num_tiles, num_sms(dev));
  kern<<<grid, kThreads, kSmemBytes, stream>>>(ta, tb, tc, p);
  AETHER_CUDA_CHECK(cudaGetLastError());
}

template <bool A_MN, bool B_MN, int OUT>
static void launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const Params& p,
                        cudaStream_t stream) {
  auto kern = gemm_pair_kernel<A_MN, B_MN, OUT>;
  static bool attr_set[64] = {false};
  const int dev = current_device();
  if (!attr_set[dev]) {
    AETHER_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kPairSmemBytes));
    attr_set[dev] = true;
  }
  const int num_tiles = ((p.M + P_BM - 1) / P_BM) * ((p.N + P_BN - 1) / P_BN);
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kPairSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // Persistent: no more pairs than can be resident at once (an SM pair must
  // share a GPC, so this can be below half the SM count), or the pairs that
  // start late would each add a whole share of tiles to the tail.
  static int resident[64] = {0};
  if (resident[dev] == 0) {
    cfg.gridDim = dim3(2 * (num_sms(dev) / 2));
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, (void*)kern, &cfg) != cudaSuccess || n <= 0) {
      (void)cudaGetLastError();
      n = num_sms(dev) / 2;
    }
    resident[dev] = std::min(n, num_sms(dev) / 2);
  }
  const int pairs = std::min(num_tiles, resident[dev]);
  cfg.gridDim = dim3(2 * pairs);
  AETHER_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, ta, tb, tc, p));
}

// Which kernel a GEMM runs on: 0 the one-CTA kernel, 1 the CTA-pair kernel
// for every problem with M, N >= 256, -1 (default) the pair kernel whenever its
// 256 x 256 tiles keep at least as many SMs busy as the one-CTA kernel's
// 128 x 256 tiles would (measured on a B200: 4-18 % faster than the one-CTA
// kernel from 4096^3 to the GPT-24L training shapes, every layout).
// Initialised from AETHER_GEMM_PAIR; gemm_pair_mode() changes it at run time.
static int g_pair_mode = [] {
  const char* e = std::getenv("AETHER_GEMM_PAIR");
  return e == nullptr ? -1 : std::atoi(e);
}();

static bool use_pair(int64_t M, int64_t N) {
  if (g_pair_mode == 0 || M < P_BM || N < P_BN) return false;
  if (g_pair_mode == 1) return true;
  const int64_t pair_tiles = ((M + P_BM - 1) / P_BM) * ((N + P_BN - 1) / P_BN);
  const int64_t one_tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int64_t sms = num_sms(current_device());
  return 2 * std::min<int64_t>(pair_tiles, sms / 2) >= std::min<int64_t>(one_tiles, sms);
}

}  // namespace gemm

// Sets the GEMM kernel choice (see use_pair) and returns the previous one.
int64_t gemm_pair_mode(int64_t mode) {
  const int old = gemm::g_pair_mode;
  gemm::g_pair_mode = (int)mode;
  return old;
}

// Python-facing entry: out (+)= alpha * opA(a) . opB(b)^T (+ bias) (+ residual).
//   a_mn == false: a is [M, K] (row stride a.stride(0));  true: a is [K, M].
//   b_mn == false: b is [N, K];                          true: b is [K, N].
// out is bf16 [M, N] or fp32 [M, N]; `accumulate` (fp32 only) adds into out.
// alpha_t (optional CUDA fp32 scalar) multiplies alpha on the device (no host sync).
void gemm_bf16(at::Tensor a, at::Tensor b, at::Tensor out, bool a_mn, bool b_mn,
               std::optional<at::Tensor> bias, std::optional<at::Tensor> residual, double alpha,
               bool accumulate, std::optional<at::Tensor> alpha_t) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && out.is_cuda(), "gemm_bf16: CUDA tensors required");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16, "gemm_bf16: bf16 operands");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && out.dim() == 2, "gemm_bf16: 2-D operands");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1 && out.stride(1) == 1, "gemm_bf16: inner dim must be contiguous");
  const int64_t M = a_mn ? a.size(1) : a.size(0);
  const int64_t K = a_mn ? a.size(0) : a.size(1);
  const int64_t N = b_mn ? b.size(1) : b.size(0);
  const int64_t Kb = b_mn ? b.size(0) : b.size(1);
  TORCH_CHECK(K == Kb, "gemm_bf16: K mismatch ", K, " vs ", Kb);
  TORCH_CHECK(out.size(0) == M && out.size(1) == N, "gemm_bf16: out shape mismatch");
  TORCH_CHECK(N % 8 == 0 && K % 8 == 0 && (!a_mn || M % 8 == 0), "gemm_bf16: dims must be multiples of 8");
  TORCH_CHECK((a.stride(0) * 2) % 16 == 0 && (b.stride(0) * 2) % 16 == 0, "gemm_bf16: row strides must be 16B multiples");
  TORCH_CHECK(out.stride(0) % 8 == 0, "gemm_bf16: out row stride must be a multiple of 8 elements");
  TORCH_CHECK(M > 0 && N > 0 && K > 0, "gemm_bf16: empty problem");
  const bool out_f32 = out.scalar_type() == at::kFloat;
  TORCH_CHECK(out_f32 || out.scalar_type() == at::kBFloat16, "gemm_bf16: out must be bf16 or fp32");
  TORCH_CHECK(!accumulate || out_f32, "gemm_bf16: accumulate requires an fp32 output");
  c10::cuda::CUDAGuard guard(a.device());

  gemm::Params p{};
  p.out = out.data_ptr();
  p.ldo = out.stride(0);
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.alpha = (float)alpha;
  p.status = device_status_word();
  if (alpha_t && alpha_t->defined()) {
    TORCH_CHECK(alpha_t->is_cuda() && alpha_t->scalar_type() == at::kFloat && alpha_t->numel() >= 1, "gemm_bf16: alpha_t must be a CUDA fp32 scalar");
    p.alpha_ptr = alpha_t->data_ptr<float>();
  }
  if (bias && bias->defined()) {
    TORCH_CHECK(bias->scalar_type() == at::kBFloat16 && bias->numel() == N && bias->is_contiguous(), "gemm_bf16: bias must be bf16 [N]");
    p.bias = reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr());
  }
  if (residual && residual->defined()) {
    TORCH_CHECK(residual->scalar_type() == at::kBFloat16 && residual->size(0) == M && residual->size(1) == N &&
                    residual->stride(1) == 1 && residual->stride(0) % 8 == 0,
                "gemm_bf16: residual must be bf16 [M, N]");
    p.residual = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
    p.ldr = residual->stride(0);
  }

  const bool pair = gemm::use_pair(M, N);
  CUtensorMap ta, tb;
  if (!a_mn) ta = make_tmap_2d_bf16(a.data_ptr(), K, M, a.stride(0) * 2, gemm::BK, gemm::BM);
  else ta = make_tmap_2d_bf16(a.data_ptr(), M, K, a.stride(0) * 2, 64, gemm::BK);
  // K-major B: a pair kernel's CTA loads 128 of the tile's 256 B rows
  if (!b_mn) tb = make_tmap_2d_bf16(b.data_ptr(), K, N, b.stride(0) * 2, gemm::BK, pair ? 128 : gemm::BN);
  else tb = make_tmap_2d_bf16(b.data_ptr(), N, K, b.stride(0) * 2, 64, gemm::BK);

  // Output map: 128-byte wide boxes (32 fp32 or 64 bf16 columns) x 32 rows, 128B swizzle.
  CUtensorMap tc;
  if (out_f32)
    tc = make_tmap_2d(out.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, N, M, out.stride(0) * 4, 32, 32,
                      CU_TENSOR_MAP_SWIZZLE_128B);
  else
    tc = make_tmap_2d(out.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, M, out.stride(0) * 2, 64, 32,
                      CU_TENSOR_MAP_SWIZZLE_128B);

  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int mode = accumulate ? gemm::OUT_F32_ACCUM : (out_f32 ? gemm::OUT_F32 : gemm::OUT_BF16);
#define AETHER_GEMM_CASE(AM, BMN, OM)                                         \
  if (a_mn == AM && b_mn == BMN && mode == OM) {                              \
    if (pair) gemm::launch_pair<AM, BMN, OM>(ta, tb, tc, p, stream);          \
    else gemm::launch<AM, BMN, OM>(ta, tb, tc, p, stream);                    \
    return;                                                                   \
  }
  AETHER_GEMM_CASE(false, false, gemm::OUT_BF16)
  AETHER_GEMM_CASE(false, false, gemm::OUT_F32)
  AETHER_GEMM_CASE(false, false, gemm::OUT_F32_ACCUM)
  AETHER_GEMM_CASE(false, true, gemm::OUT_BF16)
  AETHER_GEMM_CASE(false, true, gemm::OUT_F32)
  AETHER_GEMM_CASE(false, true, gemm::OUT_F32_ACCUM)
  AETHER_GEMM_CASE(true, true, gemm::OUT_BF16)
  AETHER_GEMM_CASE(true, true, gemm::OUT_F32)
  AETHER_GEMM_CASE(true, true, gemm::OUT_F32_ACCUM)
  AETHER_GEMM_CASE(true, false, gemm::OUT_BF16)
  AETHER_GEMM_CASE(true, false, gemm::OUT_F32)
  AETHER_GEMM_CASE(true, false, gemm::OUT_F32_ACCUM)
#undef AETHER_GEMM_CASE
  TORCH_CHECK(false, "gemm_bf16: unsupported configuration");
}

// Grouped GEMM for mixture-of-experts layers: out[Mpad, N] = a[Mpad, K] .
// w[g]^T with g = tile_group[m / 128] for every 128-row tile of a (rows of
// one expert are contiguous and start on a 128-row boundary; -1 skips the
// tile). w: [groups, N, K] (or [groups * N, K]) bf16, K-major.
void gemm_grouped(at::Tensor a, at::Tensor w, at::Tensor out, at::Tensor tile_group) {
  TORCH_CHECK(a.is_cuda() && w.is_cuda() && out.is_cuda() && tile_group.is_cuda(), "gemm_grouped: CUDA tensors");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 &&
                  out.scalar_type() == at::kBFloat16,
              "gemm_grouped: bf16 operands and output");
  TORCH_CHECK(tile_group.scalar_type() == at::kInt && tile_group.is_contiguous(), "gemm_grouped: int32 tile_group");
  TORCH_CHECK(a.dim() == 2 && a.stride(1) == 1 && w.is_contiguous() && out.dim() == 2 && out.stride(1) == 1,
              "gemm_grouped: layouts");
  const int64_t M = a.size(0), K = a.size(1);
  const int64_t N = out.size(1);
  const int64_t rows_w = w.numel() / K;
  TORCH_CHECK(w.size(-1) == K && rows_w % N == 0, "gemm_grouped: w must be [groups, N, K]");
  TORCH_CHECK(out.size(0) == M && M % gemm::BM == 0 && tile_group.numel() >= M / gemm::BM,
              "gemm_grouped: M must be a multiple of 128 with one tile_group entry per 128 rows");
  TORCH_CHECK(N % 8 == 0 && K % 8 == 0 && (a.stride(0) * 2) % 16 == 0 && out.stride(0) % 8 == 0,
              "gemm_grouped: dims / strides must be multiples of 8 elements");
  c10::cuda::CUDAGuard guard(a.device());
  gemm::Params p{};
  p.out = out.data_ptr();
  p.ldo = out.stride(0);
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.alpha = 1.f;
  p.status = device_status_word();
  p.tile_group = tile_group.data_ptr<int>();
  CUtensorMap ta = make_tmap_2d_bf16(a.data_ptr(), K, M, a.stride(0) * 2, gemm::BK, gemm::BM);
  CUtensorMap tb = make_tmap_2d_bf16(w.data_ptr(), K, rows_w, K * 2, gemm::BK, gemm::BN);
  CUtensorMap tc = make_tmap_2d(out.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, M, out.stride(0) * 2, 64, 32,
                                CU_TENSOR_MAP_SWIZZLE_128B);
  gemm::launch<false, false, gemm::OUT_BF16>(ta, tb, tc, p, at::cuda::getCurrentCUDAStream());
}

}  // namespace aether
