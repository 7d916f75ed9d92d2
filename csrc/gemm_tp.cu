// Tensor-parallel training GEMMs with their collective fused in: one
// persistent tcgen05 kernel per call, the NVLink transfer running inside it
// tile by tile.
//
// With sequence parallelism every TP rank holds Ml = M / tp token rows of the
// residual stream. The Megatron pair of projections then needs an all-gather
// of the rows before each column-parallel GEMM (qkv, gate_up) and a
// reduce-scatter of the partial sums after each row-parallel one (o_proj,
// down_proj); backward needs the mirror images. Here each of them is ONE
// kernel that does the math and the transfer together:
//
//   ag_mode 1  all-gather -> GEMM. Two pusher warps of every CTA copy this
//              rank's rows (128-row chunks) into every peer's gather buffer
//              with P2P stores and release a per-chunk flag in each peer. (A
//              multicast address may be passed instead -- one multimem.st per
//              16 bytes -- but such a store reaches this GPU's own copy through
//              the switch under another virtual alias, unordered with the local
//              flag store, so no caller that reads its own rows back uses it.) The tile schedule starts with this rank's own
//              rows (read straight from the local tensor); a tile of a peer's
//              rows waits (bounded) for that chunk's flag and then TMA-loads it
//              from local memory, so every remote byte crosses NVLink once and
//              the transfer hides behind the local tiles' MMAs.
//   rs         GEMM -> reduce-scatter. Tiles of rows owned by a peer are
//              converted to bf16 in the epilogue and stored straight into the
//              owner's receive slot (P2P, coalesced 128-byte rows out of the
//              staging shared memory), then a per-(tile, 32-row slab) counter
//              in the owner is released. The schedule visits the next rank's
//              rows first and this rank's own rows LAST; an own tile's
//              epilogue waits for the tp - 1 contributions of its slab and
//              writes acc + sum(peer partials) + residual (fp32, fixed rank
//              order) -- the reduction happens in the epilogue, no extra pass.
//   ag_mode 2  gather alongside: the pushers distribute an unrelated [Ml, Kp]
//              tensor while the GEMM runs (backward of a column-parallel
//              projection: the dgrad GEMM reduce-scatters while the saved
//              input rows travel for the weight-gradient GEMM that follows);
//              each CTA then waits for its share of incoming chunks, so when
//              the kernel ends the gather buffer is complete.
//
// Each buffer kind (gather, receive) is a two-slot ring; a call passes, per
// ring, the number of times its slot has been used (this one included). Flags only grow, so
// nothing is ever reset. Reuse is safe without a separate barrier: a rank
// finishing call e + 1 proves every peer started call e + 1 (it consumed their
// rows or contributions), hence finished call e on the same stream, so call
// e + 2 never overwrites a slot that a peer is still reading.
//
// Every wait is bounded (kWaitTimeoutNs); on expiry the kernel records a
// status code and returns. No TMA load here uses cluster multicast, and no
// library kernel ever sees a peer's memory: peer memory is touched only by
// this kernel's own stores and multimem stores.
//
// Reference: the reference runs its Megatron plan (runtime/src/
// tensor_parallel.rs:8-29) on one GPU with two all-reduces per block and has
// no sequence parallelism; its only real collective is an NCCL all-reduce.
//
// Ranks on one GPU (tests): gridDim.y > 1 runs that many ranks' kernels as one
// cooperative launch, rank y's buffers standing in for peer memory.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <ATen/ATen.h>

#include <memory>
#include <string>
#include <vector>

#include "common.cuh"
#include "host_utils.h"

namespace aether {
namespace tpg {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int STAGES = 4;
constexpr int kThreads = 256;  // producer, MMA, 4 epilogue warps, 2 pusher warps
constexpr int kPushThreads = 64;
constexpr int kPushUnroll = 16;  // 16-byte loads in flight per pusher thread
constexpr int A_BYTES = BM * BK * 2;
constexpr int B_BYTES = BN * BK * 2;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int kTmemCols = 2 * BN;
constexpr int kSlab = 32 * 128;                 // one epilogue warp's 32 rows x 128 bytes
constexpr int kStageTotal = 4 * 2 * kSlab;
constexpr int kSmemBytes = STAGES * STAGE_BYTES + kStageTotal + 1024 + 256;
constexpr int kMaxRanks = 8;
constexpr int kMaxEmu = 4;

struct RankArgs {
  int rank;
  const __nv_bfloat16* push_src;  // [Ml, Kp] rows this rank contributes to the gather
  int64_t ld_push;
  const __nv_bfloat16* residual;  // rs: [Ml, N] added by the owner (or null)
  int64_t ldr;
  uint32_t* pg_ctr;  // pg: this rank's [chunk ticket, finished CTAs] pair (0 between calls)
};

struct Params {
  int M, N, K;     // out[M, N] = A[M, K] . B^T over all ranks' rows (M = tp * Ml)
  int Ml, tp;
  int ag_mode, rs, local_copy;
  int Kp;          // gathered row width (elements)
  int gm;          // tile raster group (divides Ml / BM)
  uint32_t ag_epoch;  // uses of the gather ring slot, this call included
  uint32_t rs_epoch;  // uses of the receive ring slot, this call included
  uint64_t ag_buf[kMaxRanks];   // each rank's gather buffer [M, Kp] bf16, as mapped here
  uint64_t ag_flag[kMaxRanks];  // each rank's gather flags u32 [tp][Ml / BM]
  uint64_t ag_mc;               // multicast address of the gather buffer (0: P2P)
  uint64_t rs_buf[kMaxRanks];   // each rank's receive buffer [tp][Ml][N] bf16
  uint64_t rs_flag[kMaxRanks];  // each rank's receive counters u32 [Ml / BM][ceil(N / BN)][4]
  RankArgs r[kMaxEmu];
  int* status;
  uint64_t timeout_ns;
  // pg: parameter all-gather into the consuming GEMM. Every rank's unit buffer
  // (ag_buf) holds one flat parameter unit of tp * pg_shard bf16 elements,
  // rank q's shard at [q * pg_shard, (q + 1) * pg_shard), moved in pg_chunk
  // element chunks with one flag each (ag_flag, [tp][pg_cpr]); B is the view
  // at element pg_boff of the unit.
  int pg;
  int pg_chunk, pg_cpr;
  int64_t pg_shard, pg_boff;
  uint64_t pg_ready[kMaxRanks];  // each rank's readiness array u32 [tp], as mapped here
};

struct Maps {
  CUtensorMap a_local[kMaxEmu];  // ag_mode 1: this rank's rows [Ml, K]; else A [M, K]
  CUtensorMap a_ag[kMaxEmu];     // ag_mode 1: the gather buffer [M, K]
  CUtensorMap b[kMaxEmu];
  CUtensorMap c[kMaxEmu];        // rs: [Ml, N]; else [M, N]
};

__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
__device__ __forceinline__ void red_release_sys_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void pusher_bar() { asm volatile("bar.sync 1, 64;" ::: "memory"); }
__device__ __forceinline__ void mm_st_b128(void* mc, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(mc), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint4 ld_cg_b128(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

// Bounded acquire-spin until *f >= target (wrap-safe). False on timeout or abort.
__device__ __forceinline__ bool flag_wait_ge(const uint32_t* f, uint32_t target, volatile int* abort_word,
                                             uint64_t timeout_ns) {
  if ((int32_t)(ld_acquire_sys_u32(f) - target) >= 0) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if ((int32_t)(ld_acquire_sys_u32(f) - target) >= 0) return true;
    if ((it & 63u) == 0u) {
      if (abort_word != nullptr && *abort_word) return false;
      if (globaltimer_ns() - t0 > timeout_ns) return false;
    }
  }
}

// Virtual tile t -> (tm, tn). The raster walks groups of gm M-tiles across N
// (the last group possibly shorter); the M index is rotated so ag_mode 1
// starts at this rank's rows and rs starts at the next rank's rows (its own
// rows come last). In those modes gm divides Ml / BM, so a group never mixes
// two ranks' rows and an rs CTA meets every foreign tile of its sequence
// before any own tile.
__device__ __forceinline__ void tile_coords(const Params& p, int rank, int t, int num_m, int num_n, int& tm,
                                            int& tn) {
  const int per_group = p.gm * num_n;
  const int g = t / per_group;
  const int first = g * p.gm;
  const int gsize = min(num_m - first, p.gm);  // the last group may be short (pg mode)
  const int r = t - g * per_group;
  const int tv = first + r % gsize;
  tn = r / gsize;
  const int mt = p.Ml / BM;
  int start = 0;
  if (p.ag_mode == 1) start = rank * mt;
  else if (p.rs) start = ((rank + 1) % p.tp) * mt;
  tm = tv + start;
  if (tm >= num_m) tm -= num_m;
}

// EMU: ranks emulated on one GPU (rank = blockIdx.y, descriptors picked at run
// time); otherwise one rank per GPU and every descriptor at a fixed parameter
// address, as in the plain GEMM.
template <bool B_MN, bool EMU>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tp_kernel(const __grid_constant__ Maps maps, const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* sStage = sB + STAGES * B_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sStage + kStageTotal);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_word = reinterpret_cast<volatile int*>(tmem_slot + 1);
  __shared__ int s_ticket;

  const int y = EMU ? (int)blockIdx.y : 0;
  const RankArgs& ra = p.r[y];
  const int rank = ra.rank;
  const CUtensorMap* tmA = &maps.a_local[y];
  const CUtensorMap* tmG = &maps.a_ag[y];
  const CUtensorMap* tmB = &maps.b[y];
  const CUtensorMap* tmC = &maps.c[y];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = p.M / BM;
  const int num_n = (p.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_k = (p.K + BK - 1) / BK;
  const int mt = p.Ml / BM;

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
    tma_prefetch_desc(tmA);
    if (p.ag_mode == 1) tma_prefetch_desc(tmG);
    tma_prefetch_desc(tmB);
    tma_prefetch_desc(tmC);
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
      int64_t pg_lo = 0, pg_hi = 0;  // B range already confirmed present (pg)
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int tm, tn;
        tile_coords(p, rank, t, num_m, num_n, tm, tn);
        const CUtensorMap* amap = tmA;
        int arow = tm * BM;
        if (p.ag_mode == 1) {
          const int owner = tm / mt;
          if (owner == rank) {
            arow = (tm - owner * mt) * BM;
          } else {
            const uint32_t* f = reinterpret_cast<const uint32_t*>(p.ag_flag[rank]) + owner * mt + (tm - owner * mt);
            if (!flag_wait_ge(f, p.ag_epoch, abort_word, p.timeout_ns)) {
              ok = false;
              atomicExch(p.status, kStatusTimeoutPeer);
              break;
            }
            fence_proxy_async_global();  // peer-written rows, read next by the async proxy
            amap = tmG;
          }
        }
        if (p.pg) {
          // the chunks holding this tile's B rows ([N, K]) -- or all of B ([K, N])
          const int64_t lo = B_MN ? p.pg_boff : p.pg_boff + (int64_t)tn * BN * p.K;
          const int64_t hi = B_MN ? p.pg_boff + (int64_t)p.K * p.N
                                  : p.pg_boff + (int64_t)min(p.N, (tn + 1) * BN) * p.K;
          if (lo < pg_lo || hi > pg_hi) {
            const uint32_t* flags = reinterpret_cast<const uint32_t*>(p.ag_flag[rank]);
            for (int64_t c = lo / p.pg_chunk; c <= (hi - 1) / p.pg_chunk && ok; ++c) {
              const int64_t q = c / p.pg_cpr;  // owner of the chunk
              if (!flag_wait_ge(flags + q * p.pg_cpr + (c - q * p.pg_cpr), p.ag_epoch, abort_word, p.timeout_ns)) {
                ok = false;
                atomicExch(p.status, kStatusTimeoutPeer);
              }
            }
            if (!ok) break;
            fence_proxy_async_global();
            pg_lo = lo;
            pg_hi = hi;
          }
        }
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_word)) {
            ok = false;
            atomicExch(p.status, kStatusTimeoutProducer);
            break;
          }
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          uint8_t* a_dst = sA + stage * A_BYTES;
          uint8_t* b_dst = sB + stage * B_BYTES;
          tma_load_2d(a_dst, amap, &full[stage], kb * BK, arow);
          if constexpr (!B_MN) {
            tma_load_2d(b_dst, tmB, &full[stage], kb * BK, tn * BN);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_2d(b_dst + j * 8192, tmB, &full[stage], tn * BN + j * 64, kb * BK);
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
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN, false, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
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
            const uint64_t adesc = sdesc_sw128(a_base + kk * 32, 16, 1024);
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
      volatile int never = 0;
      umma_commit(drain);
      mbar_wait(drain, 0, &never);
    }
  } else if (warp < 6) {
    // -------------------------------------------------------------- epilogue
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    uint32_t stage_ctr = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      int tm, tn;
      tile_coords(p, rank, t, num_m, num_n, tm, tn);
      if (!mbar_wait(&tfull[acc], acc_phase, abort_word)) {
        *abort_word = 1;
        if (lane == 0) atomicExch(p.status, kStatusTimeoutEpilogue);
        break;
      }
      __syncwarp();
      tc_fence_after();
      const int owner = p.rs ? tm / mt : rank;
      const bool foreign = p.rs && owner != rank;
      const bool own_rs = p.rs && owner == rank;
      // first output row of this warp's slab: local rows of the owner under rs
      const int m_warp = p.rs ? (tm - owner * mt) * BM + quad * 32 : tm * BM + quad * 32;
      uint32_t* slab_flag =
          p.rs ? reinterpret_cast<uint32_t*>(p.rs_flag[owner]) + ((tm - owner * mt) * num_n + tn) * 4 + quad : nullptr;
      if (own_rs) {
        bool ok = true;
        if (lane == 0) ok = flag_wait_ge(slab_flag, (uint32_t)(p.tp - 1) * p.rs_epoch, abort_word, p.timeout_ns);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) {
          *abort_word = 1;
          if (lane == 0) atomicExch(p.status, kStatusTimeoutPeer);
          break;
        }
      }
#pragma unroll 1
      for (int c = 0; c < BN / 64; ++c) {
        const int n0 = tn * BN + c * 64;
        float v[64];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t r[32];
          tmem_ld32(tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * BN + c * 64 + h * 32, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) v[h * 32 + j] = __uint_as_float(r[j]);
        }
        if (n0 >= p.N) continue;  // warp-uniform
        if (own_rs) {
          // peers' bf16 partials of this row (fixed rank order), then the residual
          const int64_t lrow = m_warp + lane;
          for (int s = 0; s < p.tp; ++s) {
            if (s == rank) continue;
            const __nv_bfloat16* src =
                reinterpret_cast<const __nv_bfloat16*>(p.rs_buf[rank]) + ((int64_t)s * p.Ml + lrow) * p.N + n0;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              if (n0 + q * 8 < p.N) {
                const uint4 b = ld_cg_b128(src + q * 8);
                v[q * 8 + 0] += bf16lo(b.x); v[q * 8 + 1] += bf16hi(b.x);
                v[q * 8 + 2] += bf16lo(b.y); v[q * 8 + 3] += bf16hi(b.y);
                v[q * 8 + 4] += bf16lo(b.z); v[q * 8 + 5] += bf16hi(b.z);
                v[q * 8 + 6] += bf16lo(b.w); v[q * 8 + 7] += bf16hi(b.w);
              }
            }
          }
          if (ra.residual != nullptr) {
            const uint4* rp = reinterpret_cast<const uint4*>(ra.residual + lrow * ra.ldr + n0);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              if (n0 + q * 8 < p.N) {
                const uint4 b = rp[q];
                v[q * 8 + 0] += bf16lo(b.x); v[q * 8 + 1] += bf16hi(b.x);
                v[q * 8 + 2] += bf16lo(b.y); v[q * 8 + 3] += bf16hi(b.y);
                v[q * 8 + 4] += bf16lo(b.z); v[q * 8 + 5] += bf16hi(b.z);
                v[q * 8 + 6] += bf16lo(b.w); v[q * 8 + 7] += bf16hi(b.w);
              }
            }
          }
        }
        uint8_t* stage_buf = sStage + (quad * 2 + (stage_ctr & 1)) * kSlab;
        if (lane == 0) bulk_wait_read<1>();
        __syncwarp();
        uint8_t* my_row = stage_buf + lane * 128;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          uint4 o;
          o.x = pack_bf16(v[q * 8 + 0], v[q * 8 + 1]);
          o.y = pack_bf16(v[q * 8 + 2], v[q * 8 + 3]);
          o.z = pack_bf16(v[q * 8 + 4], v[q * 8 + 5]);
          o.w = pack_bf16(v[q * 8 + 6], v[q * 8 + 7]);
          *reinterpret_cast<uint4*>(my_row + ((q ^ (lane & 7)) << 4)) = o;
        }
        if (foreign) {
          // 32 rows x 128 bytes into the owner's slot for this rank: lanes 8j..8j+7
          // write one row's eight 16-byte pieces, four rows per step
          __syncwarp();
          __nv_bfloat16* dst =
              reinterpret_cast<__nv_bfloat16*>(p.rs_buf[owner]) + ((int64_t)rank * p.Ml + m_warp) * p.N + n0;
          const int seg = lane & 7;
#pragma unroll
          for (int it = 0; it < 8; ++it) {
            const int rr = it * 4 + (lane >> 3);
            const uint4 val = *reinterpret_cast<const uint4*>(stage_buf + rr * 128 + ((seg ^ (rr & 7)) << 4));
            if (n0 + seg * 8 < p.N) *reinterpret_cast<uint4*>(dst + (int64_t)rr * p.N + seg * 8) = val;
          }
          __syncwarp();
        } else {
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(tmC, stage_buf, n0, m_warp);
            bulk_commit();
          }
        }
        ++stage_ctr;
      }
      if (foreign) {
        // the warp's stores of this slab, ordered before lane 0's release of the count
        __syncwarp();
        if (lane == 0) red_release_sys_add(slab_flag, 1u);
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
    if (lane == 0) bulk_wait<0>();
  } else {
    // -------------------------------------------------------------- pushers
    const int pt = threadIdx.x - 6 * 32;
    if (p.pg) {
      // this rank's shard, chunk by chunk, into every rank's unit buffer (this
      // one's included: B is read from there), then a flag per chunk everywhere.
      // Chunks are claimed from a ticket counter, so whichever CTAs are resident
      // move all of them (another stream's kernels may hold some SMs).
      const int vecs = p.pg_chunk / 8;
      // The buffer may still hold a unit a slower rank is computing with: every
      // rank announces, as this kernel starts (its earlier work on the stream is
      // done), that its buffer may be overwritten, and nothing is pushed into a
      // rank's buffer before its announcement for this use has arrived.
      // (every CTA announces -- the same value -- so no CTA's residency matters)
      if (pt < p.tp) st_release_sys_u32(reinterpret_cast<uint32_t*>(p.pg_ready[pt]) + rank, p.ag_epoch);
      bool ready = true;
      if (pt < p.tp)
        ready = flag_wait_ge(reinterpret_cast<const uint32_t*>(p.pg_ready[rank]) + pt, p.ag_epoch, nullptr, p.timeout_ns);
      if (!ready) atomicExch(p.status, kStatusTimeoutPeer);
      pusher_bar();
      while (true) {
        if (pt == 0) s_ticket = (int)atomicAdd(ra.pg_ctr, 1u);
        pusher_bar();
        const int c = s_ticket;
        pusher_bar();
        if (c >= p.pg_cpr) break;
        const uint4* src = reinterpret_cast<const uint4*>(ra.push_src + (int64_t)c * p.pg_chunk);
        const int64_t off0 = ((int64_t)rank * p.pg_shard + (int64_t)c * p.pg_chunk) * 2;  // bytes
        for (int base = pt; base < vecs; base += kPushThreads * kPushUnroll) {
          uint4 v[kPushUnroll];
#pragma unroll
          for (int u = 0; u < kPushUnroll; ++u)
            if (base + u * kPushThreads < vecs) v[u] = __ldg(src + base + u * kPushThreads);
#pragma unroll
          for (int u = 0; u < kPushUnroll; ++u) {
            const int i = base + u * kPushThreads;
            if (i >= vecs) continue;
            const int64_t off = off0 + (int64_t)i * 16;
            if (p.ag_mc != 0) {
              mm_st_b128(reinterpret_cast<void*>(p.ag_mc + off), v[u]);
            } else {
              for (int q = 0; q < p.tp; ++q) *reinterpret_cast<uint4*>(p.ag_buf[q] + off) = v[u];
            }
          }
        }
        fence_acq_rel_sys();
        pusher_bar();
        if (pt == 0)
          for (int q = 0; q < p.tp; ++q)
            st_release_sys_u32(reinterpret_cast<uint32_t*>(p.ag_flag[q]) + rank * p.pg_cpr + c, p.ag_epoch);
      }
      // the whole unit is present before the kernel ends (later consumers read it freely)
      const uint32_t* flags = reinterpret_cast<const uint32_t*>(p.ag_flag[rank]);
      const int total = p.tp * p.pg_cpr;
      for (int j = blockIdx.x * kPushThreads + pt; j < total; j += gridDim.x * kPushThreads) {
        if (!flag_wait_ge(flags + j, p.ag_epoch, nullptr, p.timeout_ns)) {
          atomicExch(p.status, kStatusTimeoutPeer);
          break;
        }
      }
    } else if (p.ag_mode != 0) {
      const int segs = p.Kp / 8;  // 16-byte pieces per row
      const int total = BM * segs;
      for (int c = blockIdx.x; c < mt; c += gridDim.x) {
        const __nv_bfloat16* src = ra.push_src + (int64_t)c * BM * ra.ld_push;
        const int64_t row0 = (int64_t)rank * p.Ml + (int64_t)c * BM;
        for (int base = pt; base < total; base += kPushThreads * kPushUnroll) {
          uint4 v[kPushUnroll];
#pragma unroll
          for (int u = 0; u < kPushUnroll; ++u) {
            const int i = base + u * kPushThreads;
            if (i < total) v[u] = __ldg(reinterpret_cast<const uint4*>(src + (int64_t)(i / segs) * ra.ld_push) + i % segs);
          }
#pragma unroll
          for (int u = 0; u < kPushUnroll; ++u) {
            const int i = base + u * kPushThreads;
            if (i >= total) continue;
            const int64_t off = ((row0 + i / segs) * p.Kp + (int64_t)(i % segs) * 8) * 2;  // bytes
            if (p.ag_mc != 0) {
              mm_st_b128(reinterpret_cast<void*>(p.ag_mc + off), v[u]);
            } else {
              for (int q = 0; q < p.tp; ++q)
                if (q != rank || p.local_copy) *reinterpret_cast<uint4*>(p.ag_buf[q] + off) = v[u];
            }
          }
        }
        fence_acq_rel_sys();
        pusher_bar();
        if (pt == 0)
          for (int q = 0; q < p.tp; ++q)
            if (q != rank) st_release_sys_u32(reinterpret_cast<uint32_t*>(p.ag_flag[q]) + rank * mt + c, p.ag_epoch);
      }
      if (p.ag_mode == 2 && pt < p.tp && pt != rank) {
        // this CTA's share of incoming chunks has landed before the kernel ends
        for (int c = blockIdx.x; c < mt; c += gridDim.x) {
          const uint32_t* f = reinterpret_cast<const uint32_t*>(p.ag_flag[rank]) + pt * mt + c;
          if (!flag_wait_ge(f, p.ag_epoch, nullptr, p.timeout_ns)) {
            atomicExch(p.status, kStatusTimeoutPeer);
            break;
          }
        }
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  if (p.pg && threadIdx.x == 0) {
    // the last CTA of this rank returns the ticket counter to zero for the next call
    __threadfence();
    if (atomicAdd(ra.pg_ctr + 1, 1u) == gridDim.x - 1) {
      ra.pg_ctr[0] = 0;
      ra.pg_ctr[1] = 0;
    }
  }
}

}  // namespace tpg

// Argument checks return their message instead of throwing: the Python
// wrapper raises it (no C++ exception leaves these entry points).
#define TPG_REQUIRE(cond, ...)                                     \
  do {                                                             \
    if (!(cond)) return c10::str(__VA_ARGS__);                     \
  } while (0)

// out = A . B^T with the TP collective fused in (see the file comment). Every
// per-rank list has one entry per rank run by this launch (1 on a real TP
// group; tp when all ranks are emulated on one GPU); `ranks` names them.
//   a_local  ag_mode 1: this rank's rows [Ml, K]; otherwise A [M, K]
//   a_ag     ag_mode 1: this rank's gather buffer as a [M, K] tensor
//   b        [N, K] (b_mn false) or [K, N] (b_mn true)
//   out      rs: [Ml, N] (this rank's rows of the sum); otherwise [M, N]
//   residual rs: optional [Ml, N]
//   push_src ag_mode 1 / 2: the [Ml, Kp] rows this rank contributes
// ag_buf / ag_flag / rs_buf / rs_flag: every rank's buffer as mapped on this
// GPU (tp entries); ag_mc: multicast address of the gather buffer or 0.
std::string gemm_tp(std::vector<at::Tensor> a_local, std::vector<at::Tensor> a_ag, std::vector<at::Tensor> b,
             std::vector<at::Tensor> out, std::vector<at::Tensor> residual, std::vector<at::Tensor> push_src,
             std::vector<int64_t> ranks, int64_t tp, int64_t Ml, bool b_mn, int64_t ag_mode, bool rs,
             bool local_copy, std::vector<int64_t> ag_buf, std::vector<int64_t> ag_flag, int64_t ag_mc,
             std::vector<int64_t> rs_buf, std::vector<int64_t> rs_flag, int64_t ag_epoch, int64_t rs_epoch,
             double timeout_s) {
  using namespace tpg;
  const int ne = (int)ranks.size();
  TPG_REQUIRE(ne >= 1 && ne <= kMaxEmu, "gemm_tp: 1..", kMaxEmu, " ranks per launch");
  TPG_REQUIRE(tp >= 2 && tp <= kMaxRanks && (ne == 1 || ne == tp), "gemm_tp: tp in [2, 8]; one rank or all of them");
  TPG_REQUIRE(ag_mode >= 0 && ag_mode <= 2, "gemm_tp: ag_mode 0, 1 or 2");
  TPG_REQUIRE(ag_mode != 0 || rs, "gemm_tp: nothing to fuse");
  TPG_REQUIRE(!(ag_mode == 1 && rs), "gemm_tp: gathered A and reduce-scattered output are separate calls");
  TPG_REQUIRE(Ml > 0 && Ml % BM == 0, "gemm_tp: rows per rank must be a positive multiple of 128");
  TPG_REQUIRE((ag_mode == 0 || ag_epoch >= 1) && (!rs || rs_epoch >= 1), "gemm_tp: epochs count uses of a ring slot from 1");
  TPG_REQUIRE((int64_t)a_local.size() == ne && (int64_t)b.size() == ne && (int64_t)out.size() == ne,
              "gemm_tp: one a_local / b / out per rank");
  TPG_REQUIRE(residual.empty() || (int64_t)residual.size() == ne, "gemm_tp: residual per rank or none");
  const int64_t M = tp * Ml;
  const at::Tensor& b0 = b[0];
  const int64_t N = b_mn ? b0.size(1) : b0.size(0);
  const int64_t K = b_mn ? b0.size(0) : b0.size(1);
  TPG_REQUIRE(N % 8 == 0 && K % 8 == 0 && N > 0 && K > 0, "gemm_tp: N and K must be positive multiples of 8");
  // Every argument is checked before any guard, tensor map or launch state
  // exists: a refused call leaves nothing behind.
  const int dev = a_local[0].is_cuda() ? (int)a_local[0].get_device() : -1;
  TPG_REQUIRE(dev >= 0, "gemm_tp: CUDA tensors required");
  const int64_t Kp = ag_mode != 0 && !push_src.empty() ? push_src[0].size(1) : 0;
  if (ag_mode != 0) {
    TPG_REQUIRE((int64_t)ag_buf.size() == tp && (int64_t)ag_flag.size() == tp && (int64_t)push_src.size() == ne,
                "gemm_tp: gather needs tp buffers / flags and one push_src per rank");
    TPG_REQUIRE(Kp % 8 == 0 && Kp > 0, "gemm_tp: gathered rows must be a positive multiple of 8 elements");
    for (int q = 0; q < tp; ++q)
      TPG_REQUIRE(ag_buf[q] % 16 == 0 && ag_flag[q] % 4 == 0 && ag_buf[q] != 0 && ag_flag[q] != 0,
                  "gemm_tp: gather buffers 16-byte and flags 4-byte aligned");
    TPG_REQUIRE(ag_mc % 16 == 0, "gemm_tp: multicast address 16-byte aligned");
    TPG_REQUIRE(ag_mc == 0 || ne == 1, "gemm_tp: multicast only on a real TP group");
    TPG_REQUIRE(ag_mode != 1 || ((int64_t)a_ag.size() == ne && Kp == K),
                "gemm_tp: ag_mode 1 needs each rank's gather buffer tensor, rows as wide as A's");
  }
  if (rs) {
    TPG_REQUIRE((int64_t)rs_buf.size() == tp && (int64_t)rs_flag.size() == tp, "gemm_tp: rs needs tp buffers / flags");
    for (int q = 0; q < tp; ++q)
      TPG_REQUIRE(rs_buf[q] % 16 == 0 && rs_flag[q] % 4 == 0 && rs_buf[q] != 0 && rs_flag[q] != 0,
                  "gemm_tp: receive buffers 16-byte and counters 4-byte aligned");
  }
  const int64_t a_rows = ag_mode == 1 ? Ml : M;
  const int64_t o_rows = rs ? Ml : M;
  for (int y = 0; y < ne; ++y) {
    const at::Tensor& a = a_local[y];
    const at::Tensor& w = b[y];
    const at::Tensor& o = out[y];
    TPG_REQUIRE(ranks[y] >= 0 && ranks[y] < tp, "gemm_tp: rank out of range");
    TPG_REQUIRE(a.is_cuda() && w.is_cuda() && o.is_cuda() && a.get_device() == dev && w.get_device() == dev &&
                    o.get_device() == dev,
                "gemm_tp: tensors on one device");
    TPG_REQUIRE(a.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 &&
                    o.scalar_type() == at::kBFloat16,
                "gemm_tp: bf16 operands and output");
    TPG_REQUIRE(a.dim() == 2 && w.dim() == 2 && o.dim() == 2 && a.stride(1) == 1 && w.stride(1) == 1 &&
                    o.stride(1) == 1,
                "gemm_tp: 2-D tensors with contiguous rows");
    TPG_REQUIRE((a.stride(0) * 2) % 16 == 0 && (w.stride(0) * 2) % 16 == 0 && o.stride(0) % 8 == 0,
                "gemm_tp: row strides must be 16-byte multiples");
    TPG_REQUIRE(w.size(0) == b0.size(0) && w.size(1) == b0.size(1), "gemm_tp: every rank's B has the same shape");
    TPG_REQUIRE(a.size(0) == a_rows && a.size(1) == K, "gemm_tp: a_local must be [", a_rows, ", ", K, "]");
    TPG_REQUIRE(o.size(0) == o_rows && o.size(1) == N, "gemm_tp: out must be [", o_rows, ", ", N, "]");
    if (ag_mode == 1) {
      const at::Tensor& g = a_ag[y];
      TPG_REQUIRE(g.is_cuda() && g.get_device() == dev && g.scalar_type() == at::kBFloat16 && g.dim() == 2 &&
                      g.size(0) == M && g.size(1) == K && g.is_contiguous() &&
                      (uint64_t)g.data_ptr() == (uint64_t)ag_buf[ranks[y]],
                  "gemm_tp: a_ag must be this rank's gather buffer as a contiguous [M, K] tensor");
    }
    if (ag_mode != 0) {
      const at::Tensor& ps = push_src[y];
      TPG_REQUIRE(ps.is_cuda() && ps.get_device() == dev && ps.scalar_type() == at::kBFloat16 && ps.dim() == 2 &&
                      ps.size(0) == Ml && ps.size(1) == Kp && ps.stride(1) == 1 && (ps.stride(0) * 2) % 16 == 0 &&
                      ((uint64_t)ps.data_ptr() % 16) == 0,
                  "gemm_tp: push_src must be bf16 [Ml, Kp] with 16-byte aligned rows");
    }
    if (rs && !residual.empty() && residual[y].defined()) {
      const at::Tensor& rr = residual[y];
      TPG_REQUIRE(rr.is_cuda() && rr.get_device() == dev && rr.scalar_type() == at::kBFloat16 && rr.dim() == 2 &&
                      rr.size(0) == Ml && rr.size(1) == N && rr.stride(1) == 1 && rr.stride(0) % 8 == 0 &&
                      ((uint64_t)rr.data_ptr() % 16) == 0,
                  "gemm_tp: residual must be bf16 [Ml, N] with 16-byte aligned rows");
    }
  }

  // ---------------------------------------------------------------- launch state
  c10::cuda::CUDAGuard guard(a_local[0].device());
  struct Launch {
    Maps maps;
    Params p;
  };
  std::unique_ptr<Launch> L(new Launch());  // 64-byte aligned tensor maps, kept off the stack
  memset(&L->maps, 0, sizeof(Maps));
  Params& p = L->p;
  Maps& maps = L->maps;
  p = Params{};
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.Ml = (int)Ml;
  p.tp = (int)tp;
  p.ag_mode = (int)ag_mode;
  p.rs = rs ? 1 : 0;
  p.local_copy = local_copy ? 1 : 0;
  p.ag_epoch = (uint32_t)ag_epoch;
  p.rs_epoch = (uint32_t)rs_epoch;
  p.status = device_status_word();
  p.timeout_ns = (uint64_t)(timeout_s * 1e9);
  p.Kp = (int)Kp;
  const int64_t mt = Ml / BM;
  p.gm = 1;
  while (p.gm < 16 && mt % (p.gm * 2) == 0) p.gm *= 2;
  if (ag_mode != 0) {
    for (int q = 0; q < tp; ++q) {
      p.ag_buf[q] = (uint64_t)ag_buf[q];
      p.ag_flag[q] = (uint64_t)ag_flag[q];
    }
    p.ag_mc = (uint64_t)ag_mc;
  }
  if (rs) {
    for (int q = 0; q < tp; ++q) {
      p.rs_buf[q] = (uint64_t)rs_buf[q];
      p.rs_flag[q] = (uint64_t)rs_flag[q];
    }
  }
  for (int y = 0; y < ne; ++y) {
    const at::Tensor& a = a_local[y];
    const at::Tensor& w = b[y];
    const at::Tensor& o = out[y];
    RankArgs& r = p.r[y];
    r.rank = (int)ranks[y];
    maps.a_local[y] = make_tmap_2d_bf16(a.data_ptr(), K, a_rows, a.stride(0) * 2, BK, BM);
    if (ag_mode == 1) maps.a_ag[y] = make_tmap_2d_bf16(a_ag[y].data_ptr(), K, M, K * 2, BK, BM);
    if (!b_mn) maps.b[y] = make_tmap_2d_bf16(w.data_ptr(), K, N, w.stride(0) * 2, BK, BN);
    else maps.b[y] = make_tmap_2d_bf16(w.data_ptr(), N, K, w.stride(0) * 2, 64, BK);
    maps.c[y] = make_tmap_2d(o.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, o_rows, o.stride(0) * 2, 64, 32,
                             CU_TENSOR_MAP_SWIZZLE_128B);
    if (ag_mode != 0) {
      r.push_src = reinterpret_cast<const __nv_bfloat16*>(push_src[y].data_ptr());
      r.ld_push = push_src[y].stride(0);
    }
    if (rs && !residual.empty() && residual[y].defined()) {
      r.residual = reinterpret_cast<const __nv_bfloat16*>(residual[y].data_ptr());
      r.ldr = residual[y].stride(0);
    }
  }

  auto kern = ne > 1 ? (b_mn ? gemm_tp_kernel<true, true> : gemm_tp_kernel<false, true>)
                     : (b_mn ? gemm_tp_kernel<true, false> : gemm_tp_kernel<false, false>);
  static bool attr_set[4][64] = {};
  const int variant = (b_mn ? 1 : 0) + (ne > 1 ? 2 : 0);
  if (!attr_set[variant][dev]) {
    AETHER_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
    attr_set[variant][dev] = true;
  }
  const int64_t tiles = (M / BM) * ((N + BN - 1) / BN);
  const int per_rank = std::max(1, num_sms(dev) / ne);
  dim3 grid((unsigned)std::min<int64_t>(tiles, per_rank), (unsigned)ne);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  if (ne == 1) {
    kern<<<grid, kThreads, kSmemBytes, stream>>>(maps, p);
    AETHER_CUDA_CHECK(cudaGetLastError());
  } else {
    // the emulated ranks wait on one another: all their CTAs must be resident
    void* args[] = {(void*)&maps, (void*)&p};
    AETHER_CUDA_CHECK(cudaLaunchCooperativeKernel((const void*)kern, grid, dim3(kThreads), args, kSmemBytes, stream));
  }
  return std::string();
}


// out = A . B^T where B is a weight inside a ZeRO-3 parameter unit that is
// all-gathered by this same kernel (pg mode; see Params). Per rank run by
// this launch (1 on a real group, all of them when emulated on one GPU):
//   a        [M, K] activations
//   b        the weight as a view of this rank's unit buffer: [N, K] (b_mn
//            false) or [K, N] (b_mn true), contiguous rows
//   out      [M, N]
//   shard    this rank's flat shard of the unit (world * shard = unit length)
//   ctr      uint32 [2], zero before the first call (the kernel leaves it zero)
// unit_buf / flags / ready: every rank's unit buffer, flag array ([world][shard
// / chunk] uint32) and readiness array ([world] uint32) as mapped here; mc:
// multicast address of the unit buffer or 0; epoch: uses of this unit buffer,
// this call included.
std::string gemm_param_gather(std::vector<at::Tensor> a, std::vector<at::Tensor> b, std::vector<at::Tensor> out,
                       std::vector<at::Tensor> shard, std::vector<at::Tensor> ctr, std::vector<int64_t> ranks,
                       int64_t world, int64_t chunk, bool b_mn, std::vector<int64_t> unit_buf,
                       std::vector<int64_t> flags, std::vector<int64_t> ready, int64_t mc, int64_t epoch,
                       double timeout_s) {
  using namespace tpg;
  const int ne = (int)ranks.size();
  TPG_REQUIRE(ne >= 1 && ne <= kMaxEmu, "gemm_param_gather: 1..", kMaxEmu, " ranks per launch");
  TPG_REQUIRE(world >= 2 && world <= kMaxRanks && (ne == 1 || ne == world), "gemm_param_gather: world in [2, 8]");
  TPG_REQUIRE((int64_t)a.size() == ne && (int64_t)b.size() == ne && (int64_t)out.size() == ne &&
                  (int64_t)shard.size() == ne && (int64_t)ctr.size() == ne,
              "gemm_param_gather: one a / b / out / shard / ctr per rank");
  TPG_REQUIRE((int64_t)unit_buf.size() == world && (int64_t)flags.size() == world && (int64_t)ready.size() == world,
              "gemm_param_gather: world unit buffers, flag arrays and readiness arrays");
  for (int q = 0; q < world; ++q)
    TPG_REQUIRE(ready[q] != 0 && ready[q] % 4 == 0, "gemm_param_gather: readiness arrays 4-byte aligned");
  TPG_REQUIRE(chunk > 0 && chunk % 8 == 0, "gemm_param_gather: chunk must be a positive multiple of 8 elements");
  TPG_REQUIRE(epoch >= 1, "gemm_param_gather: epochs count uses of the unit buffer from 1");
  TPG_REQUIRE(mc % 16 == 0 && (mc == 0 || ne == 1), "gemm_param_gather: multicast only on a real group");
  const int dev = a[0].is_cuda() ? (int)a[0].get_device() : -1;
  TPG_REQUIRE(dev >= 0, "gemm_param_gather: CUDA tensors required");
  const int64_t S = shard[0].numel();
  TPG_REQUIRE(S > 0 && S % chunk == 0, "gemm_param_gather: the shard must be a whole number of chunks");
  const int64_t unit_bytes = world * S * 2;
  const at::Tensor& b0 = b[0];
  TPG_REQUIRE(b0.dim() == 2, "gemm_param_gather: 2-D weight view");
  const int64_t N = b_mn ? b0.size(1) : b0.size(0);
  const int64_t K = b_mn ? b0.size(0) : b0.size(1);
  const int64_t M = a[0].size(0);
  TPG_REQUIRE(N % 8 == 0 && K % 8 == 0 && N > 0 && K > 0 && M > 0, "gemm_param_gather: dims must be positive multiples of 8");
  for (int q = 0; q < world; ++q)
    TPG_REQUIRE(unit_buf[q] != 0 && unit_buf[q] % 16 == 0 && flags[q] != 0 && flags[q] % 4 == 0,
                "gemm_param_gather: unit buffers 16-byte and flags 4-byte aligned");
  int64_t boff = -1;
  for (int y = 0; y < ne; ++y) {
    const at::Tensor& x = a[y];
    const at::Tensor& w = b[y];
    const at::Tensor& o = out[y];
    const at::Tensor& sh = shard[y];
    TPG_REQUIRE(ranks[y] >= 0 && ranks[y] < world, "gemm_param_gather: rank out of range");
    const at::Tensor* all[] = {&x, &w, &o, &sh, &ctr[y]};
    for (const at::Tensor* t : all)
      TPG_REQUIRE(t->is_cuda() && t->get_device() == dev, "gemm_param_gather: tensors on one device");
    TPG_REQUIRE(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 &&
                    o.scalar_type() == at::kBFloat16 && sh.scalar_type() == at::kBFloat16,
                "gemm_param_gather: bf16 operands, output and shard");
    TPG_REQUIRE(ctr[y].scalar_type() == at::kInt && ctr[y].numel() >= 2 && ctr[y].is_contiguous(),
                "gemm_param_gather: ctr must be int32 [2]");
    TPG_REQUIRE(x.dim() == 2 && x.size(0) == M && x.size(1) == K && x.stride(1) == 1 && (x.stride(0) * 2) % 16 == 0,
                "gemm_param_gather: a must be [M, K] with 16-byte aligned rows");
    TPG_REQUIRE(w.dim() == 2 && w.sizes() == b0.sizes() && w.is_contiguous(), "gemm_param_gather: contiguous weight views");
    TPG_REQUIRE(o.dim() == 2 && o.size(0) == M && o.size(1) == N && o.stride(1) == 1 && o.stride(0) % 8 == 0,
                "gemm_param_gather: out must be [M, N]");
    TPG_REQUIRE(sh.is_contiguous() && sh.numel() == S && ((uint64_t)sh.data_ptr() % 16) == 0,
                "gemm_param_gather: every rank's shard has the same length, 16-byte aligned");
    const int64_t wb = (int64_t)(uint64_t)w.data_ptr() - unit_buf[ranks[y]];
    TPG_REQUIRE(wb >= 0 && wb % 16 == 0 && wb + w.numel() * 2 <= unit_bytes,
                "gemm_param_gather: the weight must be a 16-byte aligned view inside this rank's unit buffer");
    TPG_REQUIRE(boff < 0 || boff == wb / 2, "gemm_param_gather: every rank's weight at the same unit offset");
    boff = wb / 2;
  }

  c10::cuda::CUDAGuard guard(a[0].device());
  struct Launch {
    Maps maps;
    Params p;
  };
  std::unique_ptr<Launch> L(new Launch());
  memset(&L->maps, 0, sizeof(Maps));
  Params& p = L->p;
  Maps& maps = L->maps;
  p = Params{};
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.Ml = (int)M;
  p.tp = (int)world;
  p.gm = 16;
  p.ag_epoch = (uint32_t)epoch;
  p.status = device_status_word();
  p.timeout_ns = (uint64_t)(timeout_s * 1e9);
  p.pg = 1;
  p.pg_chunk = (int)chunk;
  p.pg_cpr = (int)(S / chunk);
  p.pg_shard = S;
  p.pg_boff = boff;
  p.ag_mc = (uint64_t)mc;
  for (int q = 0; q < world; ++q) {
    p.ag_buf[q] = (uint64_t)unit_buf[q];
    p.ag_flag[q] = (uint64_t)flags[q];
    p.pg_ready[q] = (uint64_t)ready[q];
  }
  for (int y = 0; y < ne; ++y) {
    RankArgs& r = p.r[y];
    r.rank = (int)ranks[y];
    r.push_src = reinterpret_cast<const __nv_bfloat16*>(shard[y].data_ptr());
    r.pg_ctr = reinterpret_cast<uint32_t*>(ctr[y].data_ptr());
    maps.a_local[y] = make_tmap_2d_bf16(a[y].data_ptr(), K, M, a[y].stride(0) * 2, BK, BM);
    if (!b_mn) maps.b[y] = make_tmap_2d_bf16(b[y].data_ptr(), K, N, K * 2, BK, BN);
    else maps.b[y] = make_tmap_2d_bf16(b[y].data_ptr(), N, K, N * 2, 64, BK);
    maps.c[y] = make_tmap_2d(out[y].data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, M, out[y].stride(0) * 2, 64, 32,
                             CU_TENSOR_MAP_SWIZZLE_128B);
  }
  auto kern = ne > 1 ? (b_mn ? gemm_tp_kernel<true, true> : gemm_tp_kernel<false, true>)
                     : (b_mn ? gemm_tp_kernel<true, false> : gemm_tp_kernel<false, false>);
  static bool attr_set[4][64] = {};
  const int variant = (b_mn ? 1 : 0) + (ne > 1 ? 2 : 0);
  if (!attr_set[variant][dev]) {
    AETHER_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
    attr_set[variant][dev] = true;
  }
  const int64_t tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int per_rank = std::max(1, num_sms(dev) / ne);
  dim3 grid((unsigned)std::min<int64_t>(tiles, per_rank), (unsigned)ne);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  if (ne == 1) {
    kern<<<grid, kThreads, kSmemBytes, stream>>>(maps, p);
    AETHER_CUDA_CHECK(cudaGetLastError());
  } else {
    void* args[] = {(void*)&maps, (void*)&p};
    AETHER_CUDA_CHECK(cudaLaunchCooperativeKernel((const void*)kern, grid, dim3(kThreads), args, kSmemBytes, stream));
  }
  return std::string();
}

}  // namespace aether
