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
// Reference counterpart: the decode GEMVs fused_*_matmul_seq1 and the batched
// seqB variants (runtime/src/cuda.rs:3347-4010, 903-1001), which run one
// thread block per output row on CUDA cores.
#include <cstdlib>

#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "host_utils.h"

namespace aether {
namespace skinny {

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
};

// Stream-K partition: CTA c owns units [c*U/G, (c+1)*U/G) in tile-major order
// (u = tile * num_kb + kb) and walks them as per-tile segments; every segment
// ends in an accumulator hand-off to the epilogue, which adds the partial sums
// into the fp32 output with atomics. One wave of CTAs, equal weight bytes each.
//
// With MC, `acc` is an NVLS multicast address and the epilogue's reductions go
// through the switch into every rank's accumulator (tensor-parallel
// row-parallel layers: GEMM and all-reduce in one kernel).
template <int BN, bool MC>
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
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_word = reinterpret_cast<volatile int*>(tmem_slot + 1);

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
    const int pre = (int)((u1 - u0) < (int64_t)STAGES ? (u1 - u0) : (int64_t)STAGES);
    for (int i = 0; i < pre; ++i) {
      const int64_t u = u0 + i;
      asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(&full[i])),
                   "r"((uint32_t)STAGE_BYTES)
                   : "memory");
      tma_load_2d(sA + i * A_BYTES, &tmW, &full[i], (int)(u % nkb) * BK, (int)(u / nkb) * BM);
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
      tma_load_2d(sA + stage * A_BYTES, &tmW, &full[stage], (int)(u % nkb) * BK, (int)(u / nkb) * BM);
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
      const int n = (int)tile * BM + quad * 32 + lane;
#pragma unroll
      for (int c = 0; c < (BN + 15) / 16; ++c) {
        uint32_t r[16];
        tmem_ld16(tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * ACC_COLS + c * 16, r);
        tmem_ld_wait();
        if (n < p.N) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = c * 16 + j;
            if (m < p.M) {
              float* dst = p.acc + (int64_t)m * p.ldacc + n;
              if constexpr (MC)
                asm volatile("multimem.red.relaxed.sys.global.add.f32 [%0], %1;" ::"l"(dst), "f"(__uint_as_float(r[j]))
                             : "memory");
              else
                atomicAdd(dst, __uint_as_float(r[j]));
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
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

template <int BN, bool MC>
void launch(const CUtensorMap& tw, const CUtensorMap& tx, const Params& p, int grid, cudaStream_t stream) {
  constexpr int smem = STAGES * (BM * BK * 2 + BN * BK * 2) + 1024 + 256;
  auto k = skinny_kernel<BN, MC>;
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
