// Small-M ("skinny") GEMM for decode: y[M, N] = x[M, K] . W[N, K]^T with M <= 64.
//
// Decode multiplies a handful of token rows by every weight matrix, so the
// work is a pure weight stream (memory-bound) and a 128-row M tile would both
// waste the tensor core and leave most SMs idle. This kernel swaps the
// operands -- the weight rows are the MMA's M dimension (128 per CTA) and the
// batch rows are its N dimension (16/32/64) -- and splits K so that every SM
// streams a slice of W:
//
//   grid = one wave of CTAs; stream-K over (weight-row tile, K block) units
//   warp 0      : TMA producer, 8-deep ring of (128 x 64 W) + (BN x 64 x) tiles
//   warp 1      : TMEM allocator + single-thread tcgen05.mma issuer (M128, N=BN)
//   warps 2..5  : epilogue -- tcgen05.ld, then fp32 atomics into acc[M, N]
//                 (transposed: lane = output feature, so each warp's atomics
//                 cover 32 consecutive features = 128 contiguous bytes)
//
// `skinny_finalize` then turns the fp32 accumulator into bf16 with the fused
// bias / residual / SwiGLU epilogue and writes zeros back, so the scratch is
// ready for the next GEMM without a memset (CUDA-graph friendly).
//
// Two decode projections finish inside the GEMM instead (one kernel fewer per
// layer each): every stream-K segment adds its K-block count to a per-tile
// counter after its atomics, and the CTA that completes a tile finalises it
// while the others move on --
//   * SwiGLU (gate/up): a 128-row tile holds 64 gate rows and the matching 64
//     up rows (two 64-row TMA boxes), so its finisher writes silu(g) * u for
//     64 outputs of every batch row;
//   * QKV: a 128-row tile is one head, so its finisher adds the bias, rotates
//     q / k (RoPE at the row's position), writes the bf16 q / k / v row and
//     appends k / v to the (optionally paged) KV cache.
//
// Reference counterpart: the decode GEMVs fused_*_matmul_seq1 and the batched
// seqB variants (runtime/src/cuda.rs:3347-4010, 903-1001), which run one
// thread block per output row on CUDA cores.
#include <cstdlib>

#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "decode_common.cuh"
#include "host_utils.h"

namespace aether {
namespace skinny {

enum Fin : int { FIN_NONE = 0, FIN_SWIGLU = 1, FIN_QKV = 2 };

// Fused tile finalisation (see the header comment).
struct TileFin {
  int* tile_cnt;          // per tile: K blocks accumulated so far (the finisher resets it to 0)
  __nv_bfloat16* y;       // SwiGLU: act [M, F]; QKV: bf16 qkv rows
  int64_t ldy;
  int F;                  // SwiGLU: outputs of each half (gate rows [0, F), up rows [F, 2F))
  const __nv_bfloat16* bias;  // QKV bias [(Hq + 2 Hkv) * 128] or null
  const int* pos;
  const int* slot;
  const float* cos_t;
  const float* sin_t;
  __nv_bfloat16* kc;
  __nv_bfloat16* vc;
  int Hq, Hkv;
  int64_t slot_stride, pos_stride;
  dec::PageMap pm;
};

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int STAGES = 8;
constexpr int kThreads = 192;

struct Params {
  float* acc;  // [M, ldacc] fp32, pre-zeroed (or an NVLS multicast address)
  int64_t ldacc;
  int M, N, K;
  int num_kb;      // K blocks of 64
  int64_t units;   // (weight-row tile, K block) pairs: n_tiles * num_kb
  int* status;
  PeerSignal sig;  // tensor parallel: announce that this rank's reductions have landed
  TileFin fin;
};

// Bounded barrier of the four epilogue warps (an mbarrier of 128 arrivals):
// false when the wait gave up (another role aborted or the time ran out).
__device__ __forceinline__ bool epi_sync(uint64_t* bar, uint32_t& phase, volatile int* abort_word) {
  mbar_arrive(bar);
  const bool ok = mbar_wait(bar, phase, abort_word);
  phase ^= 1u;
  return ok;
}

// SwiGLU finisher of logical tile t: act[m, 64t + j] = silu(g) * u, acc zeroed.
__device__ __forceinline__ void fin_swiglu(const Params& p, int t, int tid) {
  const int F = p.fin.F;
  for (int i = tid; i < p.M * 64; i += 128) {
    const int m = i >> 6, c = t * 64 + (i & 63);
    float* a = p.acc + (int64_t)m * p.ldacc;
    const float g = __ldcg(a + c), u = __ldcg(a + F + c);
    a[c] = 0.f;
    a[F + c] = 0.f;
    p.fin.y[(int64_t)m * p.fin.ldy + c] = __float2bfloat16(g / (1.f + __expf(-g)) * u);
  }
}

// QKV finisher of head tile h (head_dim 128): bias, bf16 rounding, RoPE on
// q / k at pos[m], the bf16 row written, k / v appended to the cache, acc zeroed.
__device__ __forceinline__ void fin_qkv(const Params& p, int h, int tid) {
  constexpr int D = 128, half = 64;
  const TileFin& f = p.fin;
  for (int i = tid; i < p.M * 8; i += 128) {
    const int b = i >> 3, c = (i & 7) * 8;
    float* ar = p.acc + (int64_t)b * p.ldacc + (int64_t)h * D;
    float a[8], bb[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      a[j] = __ldcg(ar + c + j);
      bb[j] = __ldcg(ar + half + c + j);
      ar[c + j] = 0.f;
      ar[half + c + j] = 0.f;
    }
    if (f.bias) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        a[j] += __bfloat162float(f.bias[(int64_t)h * D + c + j]);
        bb[j] += __bfloat162float(f.bias[(int64_t)h * D + half + c + j]);
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {  // the values a prefill would store, then rotated
      a[j] = __bfloat162float(__float2bfloat16(a[j]));
      bb[j] = __bfloat162float(__float2bfloat16(bb[j]));
    }
    const int p_ = f.pos[b];
    if (h < f.Hq + f.Hkv) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float cs = f.cos_t[(int64_t)p_ * half + c + j], sn = f.sin_t[(int64_t)p_ * half + c + j];
        const float x1 = a[j], x2 = bb[j];
        a[j] = x1 * cs - x2 * sn;
        bb[j] = x2 * cs + x1 * sn;
      }
    }
    const uint4 ua = dec::pack8(a), ub = dec::pack8(bb);
    __nv_bfloat16* qr = f.y + (int64_t)b * f.ldy + (int64_t)h * D;
    *reinterpret_cast<uint4*>(qr + c) = ua;
    *reinterpret_cast<uint4*>(qr + half + c) = ub;
    if (h >= f.Hq) {
      const bool is_k = h < f.Hq + f.Hkv;
      const int hk = is_k ? h - f.Hq : h - f.Hq - f.Hkv;
      __nv_bfloat16* dst =
          (is_k ? f.kc : f.vc) + dec::kv_offset(f.pm, f.slot[b], p_, f.slot_stride, f.pos_stride) + (int64_t)hk * D;
      *reinterpret_cast<uint4*>(dst + c) = ua;
      *reinterpret_cast<uint4*>(dst + half + c) = ub;
    }
  }
}

// Stream-K partition: CTA c owns units [c*U/G, (c+1)*U/G) in tile-major order
// (u = tile * num_kb + kb) and walks them as per-tile segments; every segment
// ends in an accumulator hand-off to the epilogue, which adds the partial sums
// into the fp32 output with atomics. One wave of CTAs, equal weight bytes each.
//
// With MC, `acc` is an NVLS multicast address and the epilogue's reductions go
// through the switch into every rank's accumulator (tensor-parallel
// row-parallel layers: GEMM and all-reduce in one kernel).
template <int BN, bool MC, int FIN>
__global__ void __launch_bounds__(kThreads, 1)
    skinny_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, Params p) {
  constexpr int A_BYTES = BM * BK * 2;
  constexpr int B_BYTES = BN * BK * 2;
  constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr int ACC_COLS = BN < 32 ? 32 : BN;
  constexpr int TMEM_COLS = 2 * ACC_COLS;  // double-buffered accumulator
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* epi_bar = drain + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(epi_bar + 1);
  volatile int* abort_word = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = abort_word + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t u0 = (int64_t)blockIdx.x * p.units / gridDim.x;
  const int64_t u1 = (int64_t)(blockIdx.x + 1) * p.units / gridDim.x;
  const int nkb = p.num_kb;

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
    mbar_init(epi_bar, 128);
    *abort_word = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    // The weights do not depend on the previous kernel: with programmatic
    // dependent launch this CTA may start while that kernel still runs, so
    // the first ring of weight tiles is requested before waiting for it; only
    // the activation tiles (x) are loaded after griddepcontrol.wait.
    // W rows of unit u: a 128-row tile, or (SwiGLU) 64 gate rows and the matching 64 up rows
    auto load_w = [&](uint8_t* dst, uint64_t* bar, int64_t u) {
      if constexpr (FIN == FIN_SWIGLU) {
        const int t = (int)(u / nkb);
        tma_load_2d(dst, &tmW, bar, (int)(u % nkb) * BK, t * 64);
        tma_load_2d(dst + A_BYTES / 2, &tmW, bar, (int)(u % nkb) * BK, p.fin.F + t * 64);
      } else {
        tma_load_2d(dst, &tmW, bar, (int)(u % nkb) * BK, (int)(u / nkb) * BM);
      }
    };
    const int pre = (int)((u1 - u0) < (int64_t)STAGES ? (u1 - u0) : (int64_t)STAGES);
    for (int i = 0; i < pre; ++i) {
      const int64_t u = u0 + i;
      asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(&full[i])),
                   "r"((uint32_t)STAGE_BYTES)
                   : "memory");
      load_w(sA + i * A_BYTES, &full[i], u);
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    for (int i = 0; i < pre; ++i) {
      tma_load_2d(sB + i * B_BYTES, &tmX, &full[i], (int)((u0 + i) % nkb) * BK, 0);
      mbar_arrive(&full[i]);
    }
    int stage = pre % STAGES;
    uint32_t phase = pre == STAGES ? 1u : 0u;
    uint32_t issued = pre;
    bool ok = true;
    for (int64_t u = u0 + pre; u < u1; ++u) {
      if (!mbar_wait(&empty[stage], phase ^ 1u, abort_word)) {
        ok = false;
        break;
      }
      mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
      load_w(sA + stage * A_BYTES, &full[stage], u);
      tma_load_2d(sB + stage * B_BYTES, &tmX, &full[stage], (int)(u % nkb) * BK, 0);
      ++issued;
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1u;
      }
    }
    if (!ok) {
      *abort_word = 1;
      atomicExch(p.status, kStatusTimeoutProducer);
      volatile int never = 0;
      const uint32_t n_back = issued < (uint32_t)STAGES ? issued : (uint32_t)STAGES;
      for (uint32_t j = 1; j <= n_back; ++j) {
        const uint32_t i = issued - j;
        mbar_wait(&full[i % STAGES], (i / STAGES) & 1u, &never);
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = idesc_bf16_f32(BM, BN, false, false);
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int64_t u = u0; u < u1 && ok;) {
      const int64_t seg_end = min(u1, (u / nkb + 1) * nkb);
      if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_word)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * ACC_COLS;
      for (int64_t v = u; v < seg_end; ++v) {
        if (!mbar_wait(&full[stage], phase, abort_word)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a_base = smem_u32(sA + stage * A_BYTES);
        const uint32_t b_base = smem_u32(sB + stage * B_BYTES);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)
          umma_f16(d_tmem, sdesc_sw128(a_base + kk * 32, 16, 1024), sdesc_sw128(b_base + kk * 32, 16, 1024), idesc,
                   (v != u || kk != 0) ? 1u : 0u);
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
      u = seg_end;
    }
    if (!ok) {
      *abort_word = 1;
      atomicExch(p.status, kStatusTimeoutMma);
    }
    volatile int never = 0;
    umma_commit(drain);  // TMEM is not freed while an MMA may still write it
    mbar_wait(drain, 0, &never);
  } else if (warp >= 2) {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;
    const int etid = (warp - 2) * 32 + lane;  // 0..127 across the four epilogue warps
    uint32_t epi_phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int64_t u = u0; u < u1;) {
      const int64_t tile = u / nkb;
      const int64_t seg_end = min(u1, (tile + 1) * nkb);
      if (!mbar_wait(&tfull[acc], acc_phase, abort_word)) {
        *abort_word = 1;
        if (lane == 0) atomicExch(p.status, kStatusTimeoutEpilogue);
        break;
      }
      __syncwarp();
      tc_fence_after();
      const int r = quad * 32 + lane;  // accumulator row = output feature within the tile
      int n;
      if constexpr (FIN == FIN_SWIGLU) n = r < 64 ? (int)tile * 64 + r : p.fin.F + (int)tile * 64 + (r - 64);
      else n = (int)tile * BM + r;
#pragma unroll
      for (int c = 0; c < (BN + 15) / 16; ++c) {
        uint32_t rr[16];
        tmem_ld16(tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * ACC_COLS + c * 16, rr);
        tmem_ld_wait();
        if (n < p.N) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = c * 16 + j;
            if (m < p.M) {
              float* dst = p.acc + (int64_t)m * p.ldacc + n;
              if constexpr (MC)
                asm volatile("multimem.red.relaxed.sys.global.add.f32 [%0], %1;" ::"l"(dst), "f"(__uint_as_float(rr[j]))
                             : "memory");
              else
                atomicAdd(dst, __uint_as_float(rr[j]));
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
      if constexpr (FIN != FIN_NONE) {
        // the tile's K blocks are counted after this segment's atomics; the
        // segment that completes the count finalises the tile
        if (!epi_sync(epi_bar, epi_phase, abort_word)) {
          *abort_word = 1;
          if (lane == 0) atomicExch(p.status, kStatusTimeoutEpilogue);
          break;
        }
        if (etid == 0) {
          __threadfence();
          const int add = (int)(seg_end - u);
          const int old = atomicAdd(p.fin.tile_cnt + tile, add);
          const bool last = old + add == nkb;
          if (last) atomicExch(p.fin.tile_cnt + tile, 0);
          *last_flag = last ? 1 : 0;
        }
        if (!epi_sync(epi_bar, epi_phase, abort_word)) {
          *abort_word = 1;
          if (lane == 0) atomicExch(p.status, kStatusTimeoutEpilogue);
          break;
        }
        if (*last_flag) {
          __threadfence();
          if constexpr (FIN == FIN_SWIGLU) fin_swiglu(p, (int)tile, etid);
          else fin_qkv(p, (int)tile, etid);
        }
        if (!epi_sync(epi_bar, epi_phase, abort_word)) {  // last_flag is reused by the next segment
          *abort_word = 1;
          if (lane == 0) atomicExch(p.status, kStatusTimeoutEpilogue);
          break;
        }
      }
      u = seg_end;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
  if constexpr (MC) peer_signal_done(p.sig);
}

// y = bf16(acc + bias + residual) (or SwiGLU of the [gate | up] halves);
// writes zeros back into acc.
template <bool SWIGLU>
__global__ void finalize_kernel(float* __restrict__ acc, int64_t ldacc, int M, int Nout,
                                const __nv_bfloat16* __restrict__ bias, const __nv_bfloat16* __restrict__ res,
                                int64_t ldr, __nv_bfloat16* __restrict__ y, int64_t ldy, PeerWait wait) {
  asm volatile("griddepcontrol.launch_dependents;");
  peer_wait(wait);  // tensor parallel: every rank's reductions into acc have landed
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // 4-wide chunk of the output
  const int chunks = Nout / 4;
  if (i >= (int64_t)M * chunks) return;
  const int m = (int)(i / chunks);
  const int n = (int)(i % chunks) * 4;
  float* a = acc + (int64_t)m * ldacc;
  float v[4];
  if constexpr (SWIGLU) {
    float4 g = *reinterpret_cast<float4*>(a + n);
    float4 u = *reinterpret_cast<float4*>(a + Nout + n);
    if (bias) {
      g.x += __bfloat162float(bias[n]); g.y += __bfloat162float(bias[n + 1]);
      g.z += __bfloat162float(bias[n + 2]); g.w += __bfloat162float(bias[n + 3]);
      u.x += __bfloat162float(bias[Nout + n]); u.y += __bfloat162float(bias[Nout + n + 1]);
      u.z += __bfloat162float(bias[Nout + n + 2]); u.w += __bfloat162float(bias[Nout + n + 3]);
    }
    const float gg[4] = {g.x, g.y, g.z, g.w}, uu[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = gg[j] / (1.f + __expf(-gg[j])) * uu[j];
    *reinterpret_cast<float4*>(a + n) = make_float4(0.f, 0.f, 0.f, 0.f);
    *reinterpret_cast<float4*>(a + Nout + n) = make_float4(0.f, 0.f, 0.f, 0.f);
  } else {
    const float4 t = *reinterpret_cast<float4*>(a + n);
    v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
    if (bias) {
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] += __bfloat162float(bias[n + j]);
    }
    if (res) {
      const uint2 r = *reinterpret_cast<const uint2*>(res + (int64_t)m * ldr + n);
      v[0] += bf16lo(r.x); v[1] += bf16hi(r.x); v[2] += bf16lo(r.y); v[3] += bf16hi(r.y);
    }
    *reinterpret_cast<float4*>(a + n) = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  uint2 o;
  o.x = pack_bf16(v[0], v[1]);
  o.y = pack_bf16(v[2], v[3]);
  *reinterpret_cast<uint2*>(y + (int64_t)m * ldy + n) = o;
}

template <int BN, bool MC, int FIN = FIN_NONE>
void launch(const CUtensorMap& tw, const CUtensorMap& tx, const Params& p, int grid, cudaStream_t stream) {
  constexpr int smem = STAGES * (BM * BK * 2 + BN * BK * 2) + 1024 + 256;
  auto k = skinny_kernel<BN, MC, FIN>;
  static bool set[64] = {false};
  const int dev = current_device();
  if (!set[dev]) {
    AETHER_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    set[dev] = true;
  }
  // Programmatic dependent launch: the kernel may begin (TMEM, barriers,
  // weight prefetch) before the previous kernel in the stream has finished.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  static const bool pdl = std::getenv("AETHER_NO_PDL") == nullptr;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  AETHER_CUDA_CHECK(cudaLaunchKernelEx(&cfg, k, tw, tx, p));
}

}  // namespace skinny

// acc[M, N] += x[M, K] . w[N, K]^T (fp32, acc must start zeroed); M <= 64.
// acc_mc != 0: reduce into every rank's accumulator through that NVLS
// multicast address (acc is then this rank's local view of the same buffer).
PeerSignal make_peer_signal(const std::optional<at::Tensor>& peers, const std::optional<at::Tensor>& epoch,
                            const std::optional<at::Tensor>& done, int64_t rank, int64_t world) {
  PeerSignal s{};
  if (world <= 0) return s;
  TORCH_CHECK(world <= 8 && peers && peers->numel() == world && !peers->is_cuda() &&
                  peers->scalar_type() == at::kLong && epoch && done,
              "peer signal: CPU int64 [world] peer slot pointers, CUDA epoch and done counters");
  auto acc = peers->accessor<int64_t, 1>();
  for (int q = 0; q < world; ++q) s.peer_sig[q] = (uint64_t)acc[q];
  s.epoch = reinterpret_cast<uint32_t*>(epoch->data_ptr());
  s.done = done->data_ptr<int>();
  s.rank = (int)rank;
  s.world = (int)world;
  return s;
}

PeerWait make_peer_wait(const std::optional<at::Tensor>& my_sig, const std::optional<at::Tensor>& epoch, int64_t rank,
                        int64_t world, double timeout_s) {
  PeerWait w{};
  if (world <= 0) return w;
  TORCH_CHECK(my_sig && epoch && my_sig->is_cuda() && epoch->is_cuda(), "peer wait: CUDA signal array and epoch");
  w.my_sig = reinterpret_cast<const uint32_t*>(my_sig->data_ptr());
  w.epoch = reinterpret_cast<const uint32_t*>(epoch->data_ptr());
  w.rank = (int)rank;
  w.world = (int)world;
  w.timeout_ns = (uint64_t)(timeout_s * 1e9);
  w.status = device_status_word();
  return w;
}

void skinny_gemm(at::Tensor x, at::Tensor w, at::Tensor acc, int64_t splits, int64_t acc_mc,
                 std::optional<at::Tensor> sig_peers, std::optional<at::Tensor> sig_epoch,
                 std::optional<at::Tensor> sig_done, int64_t sig_rank, int64_t sig_world) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && acc.is_cuda(), "skinny_gemm: CUDA tensors");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 && acc.scalar_type() == at::kFloat,
              "skinny_gemm: bf16 x/w, fp32 acc");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.stride(1) == 1 && w.stride(1) == 1 && acc.stride(1) == 1,
              "skinny_gemm: row-major 2-D operands");
  const int64_t M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K && acc.size(0) >= M && acc.size(1) >= N, "skinny_gemm: shapes");
  TORCH_CHECK(M >= 1 && M <= 64, "skinny_gemm: M must be in [1, 64]");
  TORCH_CHECK(K % 8 == 0 && (x.stride(0) * 2) % 16 == 0 && (w.stride(0) * 2) % 16 == 0, "skinny_gemm: alignment");
  c10::cuda::CUDAGuard g(x.device());
  const int n_tiles = (int)((N + skinny::BM - 1) / skinny::BM);
  const int num_kb = (int)((K + skinny::BK - 1) / skinny::BK);
  const int64_t units = (int64_t)n_tiles * num_kb;
  // one wave; at least 4 K blocks per CTA so the fixed per-CTA cost is amortised
  int64_t grid = splits > 0 ? splits : std::min<int64_t>(num_sms(current_device()), (units + 3) / 4);
  grid = std::max<int64_t>(1, std::min<int64_t>(grid, units));
  skinny::Params p{};
  p.acc = acc_mc != 0 ? reinterpret_cast<float*>(acc_mc) : acc.data_ptr<float>();
  p.ldacc = acc.stride(0);
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.num_kb = num_kb;
  p.units = units;
  p.status = device_status_word();
  p.sig = make_peer_signal(sig_peers, sig_epoch, sig_done, sig_rank, sig_world);
  TORCH_CHECK(p.sig.world == 0 || acc_mc != 0, "skinny_gemm: the completion signal needs the multicast reduction");

  const int BN = M <= 16 ? 16 : (M <= 32 ? 32 : 64);
  CUtensorMap tw = make_tmap_2d_bf16(w.data_ptr(), K, N, w.stride(0) * 2, skinny::BK, skinny::BM);
  CUtensorMap tx = make_tmap_2d_bf16(x.data_ptr(), K, M, x.stride(0) * 2, skinny::BK, BN);
  auto stream = at::cuda::getCurrentCUDAStream();
  const bool mc = acc_mc != 0;
  const int ng = (int)grid;
  if (BN == 16) mc ? skinny::launch<16, true>(tw, tx, p, ng, stream) : skinny::launch<16, false>(tw, tx, p, ng, stream);
  else if (BN == 32) mc ? skinny::launch<32, true>(tw, tx, p, ng, stream) : skinny::launch<32, false>(tw, tx, p, ng, stream);
  else mc ? skinny::launch<64, true>(tw, tx, p, ng, stream) : skinny::launch<64, false>(tw, tx, p, ng, stream);
}

namespace {
// The launch shared by the fused-epilogue forms: `tiles` logical tiles of 128
// accumulator rows, W boxes of `box_rows` rows.
template <int FIN>
void skinny_fused(at::Tensor x, at::Tensor w, at::Tensor acc, at::Tensor tile_cnt, int64_t tiles, int box_rows,
                  const skinny::TileFin& fin, int64_t splits) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && acc.is_cuda() && tile_cnt.is_cuda(), "skinny_gemm: CUDA tensors");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 && acc.scalar_type() == at::kFloat,
              "skinny_gemm: bf16 x/w, fp32 acc");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.stride(1) == 1 && w.stride(1) == 1 && acc.stride(1) == 1,
              "skinny_gemm: row-major 2-D operands");
  const int64_t M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K && acc.size(0) >= M && acc.size(1) >= N, "skinny_gemm: shapes");
  TORCH_CHECK(M >= 1 && M <= 64, "skinny_gemm: M must be in [1, 64]");
  TORCH_CHECK(K % 8 == 0 && (x.stride(0) * 2) % 16 == 0 && (w.stride(0) * 2) % 16 == 0, "skinny_gemm: alignment");
  TORCH_CHECK(tile_cnt.scalar_type() == at::kInt && tile_cnt.numel() >= tiles, "skinny_gemm: tile counters");
  c10::cuda::CUDAGuard g(x.device());
  const int num_kb = (int)((K + skinny::BK - 1) / skinny::BK);
  const int64_t units = tiles * num_kb;
  int64_t grid = splits > 0 ? splits : std::min<int64_t>(num_sms(current_device()), (units + 3) / 4);
  grid = std::max<int64_t>(1, std::min<int64_t>(grid, units));
  skinny::Params p{};
  p.acc = acc.data_ptr<float>();
  p.ldacc = acc.stride(0);
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.num_kb = num_kb;
  p.units = units;
  p.status = device_status_word();
  p.fin = fin;
  p.fin.tile_cnt = tile_cnt.data_ptr<int>();
  const int BN = M <= 16 ? 16 : (M <= 32 ? 32 : 64);
  CUtensorMap tw = make_tmap_2d_bf16(w.data_ptr(), K, N, w.stride(0) * 2, skinny::BK, box_rows);
  CUtensorMap tx = make_tmap_2d_bf16(x.data_ptr(), K, M, x.stride(0) * 2, skinny::BK, BN);
  auto stream = at::cuda::getCurrentCUDAStream();
  const int ng = (int)grid;
  if (BN == 16) skinny::launch<16, false, FIN>(tw, tx, p, ng, stream);
  else if (BN == 32) skinny::launch<32, false, FIN>(tw, tx, p, ng, stream);
  else skinny::launch<64, false, FIN>(tw, tx, p, ng, stream);
}
}  // namespace

// act[M, F] = silu(x w_gate^T) * (x w_up^T) with w = [gate (F rows); up (F
// rows)], finished inside the GEMM (acc: zeroed scratch, left zeroed).
void skinny_gemm_swiglu(at::Tensor x, at::Tensor w, at::Tensor acc, at::Tensor act, at::Tensor tile_cnt,
                        int64_t splits) {
  const int64_t F = w.size(0) / 2;
  TORCH_CHECK(w.size(0) == 2 * F && F % 64 == 0, "skinny_gemm_swiglu: w must be [2F, K] with F % 64 == 0");
  TORCH_CHECK(act.scalar_type() == at::kBFloat16 && act.stride(1) == 1 && act.size(0) >= x.size(0) &&
                  act.size(1) >= F,
              "skinny_gemm_swiglu: act [M, F] bf16");
  skinny::TileFin fin{};
  fin.y = reinterpret_cast<__nv_bfloat16*>(act.data_ptr());
  fin.ldy = act.stride(0);
  fin.F = (int)F;
  skinny_fused<skinny::FIN_SWIGLU>(x, w, acc, tile_cnt, F / 64, 64, fin, splits);
}

// The decode QKV projection finished inside the GEMM: qkv (bf16 rows) =
// x wqkv^T + bias with RoPE on q / k at pos, and k / v appended to the cache
// at (slot, pos). Head dim 128 (one head per 128-row tile).
void skinny_gemm_qkv(at::Tensor x, at::Tensor w, at::Tensor acc, at::Tensor tile_cnt, std::optional<at::Tensor> bias,
                     at::Tensor qkv, at::Tensor pos, at::Tensor slot, at::Tensor cos_t, at::Tensor sin_t,
                     at::Tensor k_cache, at::Tensor v_cache, int64_t Hq, int64_t Hkv,
                     std::optional<at::Tensor> page_table, int64_t splits) {
  constexpr int64_t D = 128;
  TORCH_CHECK(w.size(0) == (Hq + 2 * Hkv) * D, "skinny_gemm_qkv: w rows must be (Hq + 2 Hkv) * 128");
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16 && qkv.stride(1) == 1 && qkv.stride(0) % 8 == 0 &&
                  qkv.size(1) >= w.size(0),
              "skinny_gemm_qkv: qkv layout");
  TORCH_CHECK(pos.scalar_type() == at::kInt && slot.scalar_type() == at::kInt, "skinny_gemm_qkv: int32 pos / slot");
  TORCH_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous() && k_cache.size(-1) == D, "skinny_gemm_qkv: caches");
  TORCH_CHECK(cos_t.scalar_type() == at::kFloat && sin_t.scalar_type() == at::kFloat, "skinny_gemm_qkv: tables");
  skinny::TileFin fin{};
  fin.y = reinterpret_cast<__nv_bfloat16*>(qkv.data_ptr());
  fin.ldy = qkv.stride(0);
  fin.bias = (bias && bias->defined()) ? reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr()) : nullptr;
  fin.pos = pos.data_ptr<int>();
  fin.slot = slot.data_ptr<int>();
  fin.cos_t = cos_t.data_ptr<float>();
  fin.sin_t = sin_t.data_ptr<float>();
  fin.kc = reinterpret_cast<__nv_bfloat16*>(k_cache.data_ptr());
  fin.vc = reinterpret_cast<__nv_bfloat16*>(v_cache.data_ptr());
  fin.Hq = (int)Hq;
  fin.Hkv = (int)Hkv;
  fin.slot_stride = k_cache.stride(0);
  fin.pos_stride = k_cache.stride(1);
  fin.pm = page_map(page_table, k_cache);
  skinny_fused<skinny::FIN_QKV>(x, w, acc, tile_cnt, Hq + 2 * Hkv, 128, fin, splits);
}

// y = bf16(acc (+bias) (+res)), or swiglu over acc's [gate | up] halves when swiglu;
// acc is re-zeroed. y: [M, Nout] (Nout = N or N/2 for swiglu).
void skinny_finalize(at::Tensor acc, at::Tensor y, std::optional<at::Tensor> bias, std::optional<at::Tensor> res,
                     bool swiglu, std::optional<at::Tensor> wait_sig, std::optional<at::Tensor> wait_epoch,
                     int64_t wait_rank, int64_t wait_world, double wait_timeout_s) {
  const int64_t M = y.size(0), Nout = y.size(1);
  TORCH_CHECK(acc.scalar_type() == at::kFloat && y.scalar_type() == at::kBFloat16 && y.stride(1) == 1, "skinny_finalize: dtypes");
  TORCH_CHECK(Nout % 4 == 0 && acc.size(0) >= M && acc.size(1) >= (swiglu ? 2 * Nout : Nout), "skinny_finalize: shapes");
  TORCH_CHECK(acc.stride(0) % 4 == 0 && y.stride(0) % 4 == 0, "skinny_finalize: strides");
  const __nv_bfloat16* b = (bias && bias->defined()) ? reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr()) : nullptr;
  const __nv_bfloat16* r = nullptr;
  int64_t ldr = 0;
  if (res && res->defined()) {
    TORCH_CHECK(!swiglu && res->stride(1) == 1 && res->stride(0) % 4 == 0, "skinny_finalize: residual layout");
    r = reinterpret_cast<const __nv_bfloat16*>(res->data_ptr());
    ldr = res->stride(0);
  }
  c10::cuda::CUDAGuard g(acc.device());
  const int64_t n = M * (Nout / 4);
  const unsigned grid = (unsigned)((n + 255) / 256);
  auto stream = at::cuda::getCurrentCUDAStream();
  const PeerWait pw = make_peer_wait(wait_sig, wait_epoch, wait_rank, wait_world, wait_timeout_s);
  if (swiglu)
    skinny::finalize_kernel<true><<<grid, 256, 0, stream>>>(acc.data_ptr<float>(), acc.stride(0), (int)M, (int)Nout, b,
                                                            nullptr, 0, reinterpret_cast<__nv_bfloat16*>(y.data_ptr()),
                                                            y.stride(0), pw);
  else
    skinny::finalize_kernel<false><<<grid, 256, 0, stream>>>(acc.data_ptr<float>(), acc.stride(0), (int)M, (int)Nout, b,
                                                             r, ldr, reinterpret_cast<__nv_bfloat16*>(y.data_ptr()),
                                                             y.stride(0), pw);
  AETHER_CUDA_CHECK(cudaGetLastError());
}

}  // namespace aether
