// Tensor-parallel decode exchanges over NVLink 5 / NVSwitch symmetric memory.
//
//   vocab_argmax   the LM head is split by vocabulary rows over the TP ranks:
//                  each rank takes the argmax of its own logit slice, pushes
//                  (value, index) into every rank's exchange slot with a
//                  release-stored epoch, and merges all ranks' candidates --
//                  one kernel, no collective launch, CUDA-graph safe (the
//                  epoch is a per-row device counter)
//   put_cols       copies this rank's logit slice into every rank's full-width
//                  logits buffer (P2P stores), for the sampling paths that need
//                  the whole distribution (followed by a team barrier)
//   push_reduce    the per-layer row-parallel reduction of decode as a
//                  one-shot push: each rank stores its fp32 partial row into
//                  every rank's inbox (NVLS multimem.st, or P2P stores), raises
//                  a per-(row, source) epoch flag, waits for every other rank's
//                  flag and sums -- fused with the bias / residual add and the
//                  RMSNorm of the next sub-layer, so a reduction is one small
//                  kernel after a GEMM that only does local atomics
//
// Reference: the reference's TP plan all-reduces [d_model] per token twice per
// block with NCCL (runtime/src/tensor_parallel.rs:8-29; hook at :490-494) and
// replicates the LM head; its decode copies the full [vocab] fp32 logits to
// the host every step (runtime/src/serving.rs:3389-3418).
//
// Every wait is bounded (timeout_ns); on expiry the kernel records
// kStatusTimeoutPeer in the status word and carries on with what it has, so a
// missing peer shows up as an error instead of a hung GPU.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "host_utils.h"

namespace aether {
namespace tpd {

constexpr int kMaxWorld = 8;
constexpr int kThreads = 1024;
constexpr int kMaxVec = 2;  // float4 per thread: rows up to 1024 * 4 * 2 = 8192

struct Team {
  uint64_t data[kMaxWorld];   // every rank's exchange data area, as mapped here
  uint64_t flags[kMaxWorld];  // every rank's flag area (uint32), as mapped here
  uint64_t data_mc;           // multicast address of the data area (0: P2P stores)
  int rank, world;
  uint64_t timeout_ns;
  int* status;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ld_relaxed_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void mm_st_f32x4(float* mc, float4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(mc), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}

// Bounded acquire-spin until *flag == e.
__device__ __forceinline__ void wait_epoch(const uint32_t* flag, uint32_t e, const Team& t) {
  const uint64_t t0 = globaltimer_ns();
  uint32_t it = 0;
  while (ld_acquire_sys(flag) != e) {
    if ((++it & 255u) == 0 && globaltimer_ns() - t0 > t.timeout_ns) {
      atomicExch(t.status, kStatusTimeoutPeer);
      return;
    }
  }
}

// ---------------------------------------------------------------- vocab argmax
// Exchange record per (parity, source rank, row): {value bits, global index,
// epoch, unused}, 16 bytes, in the `flags` area (uint32).
__global__ void __launch_bounds__(kThreads) vocab_argmax_kernel(const float* __restrict__ logits, int64_t ld, int n_loc,
                                                                int col0, int rows_cap, uint32_t* __restrict__ ctr,
                                                                int64_t* __restrict__ out, Team t) {
  const int r = blockIdx.x;
  const float* row = logits + (int64_t)r * ld;
  float best = -INFINITY;
  int idx = 0x7fffffff;
  // 16-byte loads when the row allows them, four in flight per thread
  const bool vec = (ld % 4 == 0) && ((reinterpret_cast<uintptr_t>(logits) & 15) == 0);
  int start = 0;
  if (vec) {
    const int n4 = n_loc / 4;
    const float4* r4 = reinterpret_cast<const float4*>(row);
    for (int i = threadIdx.x; i < n4; i += kThreads * 4) {
      float4 u[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int k = i + j * kThreads;
        u[j] = k < n4 ? __ldg(r4 + k) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = 4 * (i + j * kThreads);
        const float f[4] = {u[j].x, u[j].y, u[j].z, u[j].w};
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (f[q] > best || (f[q] == best && c + q < idx)) {
            best = f[q];
            idx = c + q;
          }
      }
    }
    start = n4 * 4;
  }
  for (int c = start + threadIdx.x; c < n_loc; c += kThreads) {
    const float f = row[c];
    if (f > best || (f == best && c < idx)) {
      best = f;
      idx = c;
    }
  }
  // CTA reduction: warp shuffles, then one warp over the warp winners
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float b2 = __shfl_xor_sync(0xffffffffu, best, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
    if (b2 > best || (b2 == best && i2 < idx)) {
      best = b2;
      idx = i2;
    }
  }
  __shared__ float s_best[32 + kMaxWorld];
  __shared__ int s_idx[32 + kMaxWorld];
  __shared__ uint32_t s_e;
  if ((threadIdx.x & 31) == 0) {
    s_best[threadIdx.x >> 5] = best;
    s_idx[threadIdx.x >> 5] = idx;
  }
  if (threadIdx.x == 0) s_e = ctr[r] + 1;
  __syncthreads();
  if (threadIdx.x < 32) {
    best = s_best[threadIdx.x];
    idx = s_idx[threadIdx.x];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float b2 = __shfl_xor_sync(0xffffffffu, best, o);
      const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
      if (b2 > best || (b2 == best && i2 < idx)) {
        best = b2;
        idx = i2;
      }
    }
  }
  const uint32_t e = s_e;
  const int par = (int)(e & 1u);
  const int gidx = (idx == 0x7fffffff) ? 0x7fffffff : col0 + idx;
  // thread p publishes this rank's candidate to rank p
  const int p = threadIdx.x;
  if (threadIdx.x < 32) best = __shfl_sync(0xffffffffu, best, 0);
  const int g0 = __shfl_sync(0xffffffffu, gidx, 0);
  if (p < t.world) {
    uint32_t* rec = reinterpret_cast<uint32_t*>(t.flags[p]) + (((int64_t)par * kMaxWorld + t.rank) * rows_cap + r) * 4;
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(rec), "r"(__float_as_uint(best)) : "memory");
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(rec + 1), "r"((uint32_t)g0) : "memory");
    st_release_sys(rec + 2, e);
    // thread p then collects rank p's candidate from this rank's own area
    const uint32_t* mine =
        reinterpret_cast<const uint32_t*>(t.flags[t.rank]) + (((int64_t)par * kMaxWorld + p) * rows_cap + r) * 4;
    wait_epoch(mine + 2, e, t);
    s_best[32 + p] = __uint_as_float(ld_relaxed_sys(mine));
    s_idx[32 + p] = (int)ld_relaxed_sys(mine + 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = -INFINITY;
    int i = 0x7fffffff;
    for (int q = 0; q < t.world; ++q) {
      const float v = s_best[32 + q];
      const int j = s_idx[32 + q];
      if (v > b || (v == b && j < i)) {
        b = v;
        i = j;
      }
    }
    out[r] = (i == 0x7fffffff) ? 0 : i;
    ctr[r] = e;
  }
}

// ---------------------------------------------------------------- logits gather
// dst_p[row, col0 + c] = src[row, c] for every rank p (P2P stores).
__global__ void put_cols_kernel(const float* __restrict__ src, int64_t lds, int n_loc, int col0, int64_t ldd,
                                Team t) {
  const int r = blockIdx.y;
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < n_loc; c += gridDim.x * blockDim.x) {
    const float v = src[(int64_t)r * lds + c];
    for (int p = 0; p < t.world; ++p) reinterpret_cast<float*>(t.data[p])[(int64_t)r * ldd + col0 + c] = v;
  }
}

// ---------------------------------------------------------------- push reduce
// One CTA per row. acc: this rank's fp32 partial [rows, ldacc] (zeroed here for
// the next GEMM). Inbox layout (data area, fp32): [2 parities][kMaxWorld
// sources][rows_cap][ld]; flags (uint32): [2][kMaxWorld][rows_cap].
// y = bf16(sum + bias + res); with w, h = rmsnorm(y) * w.
template <bool MC>
__global__ void __launch_bounds__(kThreads) push_reduce_kernel(float* __restrict__ acc, int64_t ldacc, int N,
                                                               int64_t ld, int rows_cap, uint32_t* __restrict__ ctr,
                                                               const __nv_bfloat16* __restrict__ bias,
                                                               const __nv_bfloat16* __restrict__ res,
                                                               __nv_bfloat16* __restrict__ y,
                                                               const __nv_bfloat16* __restrict__ w,
                                                               __nv_bfloat16* __restrict__ h, float eps, Team t) {
  const int r = blockIdx.x;
  __shared__ uint32_t s_e;
  __shared__ float red[32];
  if (threadIdx.x == 0) s_e = ctr[r] + 1;
  __syncthreads();
  const uint32_t e = s_e;
  const int par = (int)(e & 1u);
  const int n4 = N / 4;
  float4 v[kMaxVec];
  float4* a4 = reinterpret_cast<float4*>(acc + (int64_t)r * ldacc);
  const int64_t slot = (((int64_t)par * kMaxWorld + t.rank) * rows_cap + r) * ld;
#pragma unroll
  for (int k = 0; k < kMaxVec; ++k) {
    const int i = threadIdx.x + k * kThreads;
    v[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (i < n4) {
      v[k] = a4[i];
      a4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      if constexpr (MC) {
        mm_st_f32x4(reinterpret_cast<float*>(t.data_mc) + slot + 4 * i, v[k]);
      } else {
        for (int p = 0; p < t.world; ++p)
          if (p != t.rank) reinterpret_cast<float4*>(reinterpret_cast<float*>(t.data[p]) + slot)[i] = v[k];
      }
    }
  }
  __syncthreads();
  const int q = threadIdx.x;
  if (q < t.world && q != t.rank) {
    __threadfence_system();  // this CTA's stores to rank q are visible before the flag
    st_release_sys(reinterpret_cast<uint32_t*>(t.flags[q]) + ((int64_t)par * kMaxWorld + t.rank) * rows_cap + r, e);
    wait_epoch(reinterpret_cast<const uint32_t*>(t.flags[t.rank]) + ((int64_t)par * kMaxWorld + q) * rows_cap + r, e,
               t);
  }
  __syncthreads();
  const float* inbox = reinterpret_cast<const float*>(t.data[t.rank]);
  float ss = 0.f;
  float4 o[kMaxVec];
#pragma unroll
  for (int k = 0; k < kMaxVec; ++k) {
    const int i = threadIdx.x + k * kThreads;
    o[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (i < n4) {
      float4 s = v[k];
      for (int p = 0; p < t.world; ++p) {
        if (p == t.rank) continue;
        // __ldcv: fetch from L2 again, never from a line this SM cached on an earlier call
        const float4 u = __ldcv(reinterpret_cast<const float4*>(inbox + (((int64_t)par * kMaxWorld + p) * rows_cap + r) * ld) + i);
        s.x += u.x; s.y += u.y; s.z += u.z; s.w += u.w;
      }
      const int c = 4 * i;
      if (bias) {
        s.x += __bfloat162float(bias[c]); s.y += __bfloat162float(bias[c + 1]);
        s.z += __bfloat162float(bias[c + 2]); s.w += __bfloat162float(bias[c + 3]);
      }
      if (res) {
        const __nv_bfloat16* rr = res + (int64_t)r * N + c;
        s.x += __bfloat162float(rr[0]); s.y += __bfloat162float(rr[1]);
        s.z += __bfloat162float(rr[2]); s.w += __bfloat162float(rr[3]);
      }
      __nv_bfloat16* yr = y + (int64_t)r * N + c;
      const __nv_bfloat16 b0 = __float2bfloat16(s.x), b1 = __float2bfloat16(s.y), b2 = __float2bfloat16(s.z),
                          b3 = __float2bfloat16(s.w);
      yr[0] = b0; yr[1] = b1; yr[2] = b2; yr[3] = b3;
      o[k] = make_float4(__bfloat162float(b0), __bfloat162float(b1), __bfloat162float(b2), __bfloat162float(b3));
      ss += o[k].x * o[k].x + o[k].y * o[k].y + o[k].z * o[k].z + o[k].w * o[k].w;
    }
  }
  if (threadIdx.x == 0) ctr[r] = e;
  if (w == nullptr) return;
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int k = 0; k < 32; ++k) tot += red[k];
  const float rstd = rsqrtf(tot / N + eps);
#pragma unroll
  for (int k = 0; k < kMaxVec; ++k) {
    const int i = threadIdx.x + k * kThreads;
    if (i < n4) {
      const int c = 4 * i;
      __nv_bfloat16* hr = h + (int64_t)r * N + c;
      hr[0] = __float2bfloat16(o[k].x * rstd * __bfloat162float(w[c]));
      hr[1] = __float2bfloat16(o[k].y * rstd * __bfloat162float(w[c + 1]));
      hr[2] = __float2bfloat16(o[k].z * rstd * __bfloat162float(w[c + 2]));
      hr[3] = __float2bfloat16(o[k].w * rstd * __bfloat162float(w[c + 3]));
    }
  }
}

}  // namespace tpd

// --------------------------------------------------------------------- host API
namespace {
tpd::Team make_tp_team(const at::Tensor& data_peers, const at::Tensor& flag_peers, int64_t data_mc, int64_t rank,
                       int64_t world, double timeout_s) {
  TORCH_CHECK(world >= 1 && world <= tpd::kMaxWorld, "tp exchange: world size must be in [1, 8]");
  TORCH_CHECK(rank >= 0 && rank < world, "tp exchange: rank");
  TORCH_CHECK(!data_peers.is_cuda() && data_peers.scalar_type() == at::kLong && data_peers.numel() == world,
              "tp exchange: data_peers must be a CPU int64 tensor of world entries");
  TORCH_CHECK(!flag_peers.is_cuda() && flag_peers.scalar_type() == at::kLong && flag_peers.numel() == world,
              "tp exchange: flag_peers must be a CPU int64 tensor of world entries");
  tpd::Team t{};
  auto d = data_peers.accessor<int64_t, 1>();
  auto f = flag_peers.accessor<int64_t, 1>();
  for (int i = 0; i < world; ++i) {
    t.data[i] = (uint64_t)d[i];
    t.flags[i] = (uint64_t)f[i];
    TORCH_CHECK(t.data[i] % 16 == 0 && t.flags[i] % 16 == 0, "tp exchange: 16-byte aligned areas");
  }
  t.data_mc = (uint64_t)data_mc;
  t.rank = (int)rank;
  t.world = (int)world;
  t.timeout_ns = (uint64_t)(timeout_s * 1e9);
  t.status = device_status_word();
  return t;
}
}  // namespace

// out[r] = global argmax over all ranks' slices; logits [rows, ld] fp32 with
// this rank's n_loc columns starting at global column col0. flag area: uint32
// [2][8][rows_cap][4] per rank; ctr: int32 [rows_cap] (zero-initialised).
void tp_vocab_argmax(at::Tensor logits, int64_t n_loc, int64_t col0, at::Tensor flag_peers, at::Tensor ctr,
                     int64_t rows_cap, at::Tensor out, int64_t rank, int64_t world, double timeout_s) {
  c10::cuda::CUDAGuard g(logits.device());
  const int64_t rows = out.numel();
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.stride(1) == 1 && logits.size(0) >= rows &&
                  logits.size(1) >= n_loc,
              "tp_vocab_argmax: fp32 [rows, >= n_loc] logits");
  TORCH_CHECK(out.scalar_type() == at::kLong && out.is_contiguous(), "tp_vocab_argmax: int64 out");
  TORCH_CHECK(ctr.is_cuda() && ctr.scalar_type() == at::kInt && ctr.numel() >= rows && rows <= rows_cap,
              "tp_vocab_argmax: counters");
  if (rows == 0) return;
  tpd::Team t = make_tp_team(flag_peers, flag_peers, 0, rank, world, timeout_s);
  tpd::vocab_argmax_kernel<<<(unsigned)rows, tpd::kThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      logits.data_ptr<float>(), logits.stride(0), (int)n_loc, (int)col0, (int)rows_cap,
      reinterpret_cast<uint32_t*>(ctr.data_ptr()), out.data_ptr<int64_t>(), t);
  AETHER_CUDA_CHECK(cudaGetLastError());
}

// Every rank's full logits buffer (data_peers: [rows, ldd] fp32 each) receives
// this rank's src [rows, n_loc] at column col0. A team barrier must follow.
void tp_put_cols(at::Tensor src, int64_t n_loc, int64_t col0, at::Tensor data_peers, int64_t ldd, int64_t rank,
                 int64_t world) {
  c10::cuda::CUDAGuard g(src.device());
  TORCH_CHECK(src.scalar_type() == at::kFloat && src.stride(1) == 1 && src.size(1) >= n_loc, "tp_put_cols: src");
  TORCH_CHECK(col0 + n_loc <= ldd, "tp_put_cols: columns");
  const int64_t rows = src.size(0);
  if (rows == 0 || n_loc == 0) return;
  tpd::Team t = make_tp_team(data_peers, data_peers, 0, rank, world, 1.0);
  dim3 grid((unsigned)std::min<int64_t>((n_loc + 255) / 256, 64), (unsigned)rows);
  tpd::put_cols_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(src.data_ptr<float>(), src.stride(0),
                                                                          (int)n_loc, (int)col0, ldd, t);
  AETHER_CUDA_CHECK(cudaGetLastError());
}

// One-shot push reduction of acc [rows, N] over the TP ranks, fused with the
// bias / residual add (-> y) and optionally RMSNorm (-> h with weight w).
void tp_push_reduce(at::Tensor acc, at::Tensor y, std::optional<at::Tensor> bias, std::optional<at::Tensor> res,
                    std::optional<at::Tensor> w, std::optional<at::Tensor> h, double eps, at::Tensor data_peers,
                    int64_t data_mc, int64_t ld, at::Tensor flag_peers, at::Tensor ctr, int64_t rows_cap,
                    int64_t rank, int64_t world, double timeout_s) {
  c10::cuda::CUDAGuard g(acc.device());
  const int64_t rows = y.size(0), N = y.size(1);
  TORCH_CHECK(acc.scalar_type() == at::kFloat && acc.stride(1) == 1 && acc.stride(0) % 4 == 0 &&
                  acc.size(0) >= rows && acc.size(1) >= N,
              "tp_push_reduce: fp32 acc [rows, >= N], row stride % 4");
  TORCH_CHECK(y.scalar_type() == at::kBFloat16 && y.is_contiguous(), "tp_push_reduce: bf16 contiguous y");
  TORCH_CHECK(N % 4 == 0 && N <= tpd::kThreads * 4 * tpd::kMaxVec && N <= ld && ld % 4 == 0,
              "tp_push_reduce: N % 4 == 0, N <= 8192, N <= ld");
  TORCH_CHECK(rows <= rows_cap && ctr.is_cuda() && ctr.scalar_type() == at::kInt && ctr.numel() >= rows,
              "tp_push_reduce: rows / counters");
  const bool norm = w && w->defined();
  TORCH_CHECK(!norm || (h && h->defined() && h->is_contiguous() && h->sizes() == y.sizes()), "tp_push_reduce: h");
  if (res && res->defined()) TORCH_CHECK(res->is_contiguous() && res->sizes() == y.sizes(), "tp_push_reduce: res");
  if (rows == 0) return;
  tpd::Team t = make_tp_team(data_peers, flag_peers, data_mc, rank, world, timeout_s);
  TORCH_CHECK(data_mc % 16 == 0, "tp_push_reduce: multicast address alignment");
  auto* bp = (bias && bias->defined()) ? reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr()) : nullptr;
  auto* rp = (res && res->defined()) ? reinterpret_cast<const __nv_bfloat16*>(res->data_ptr()) : nullptr;
  auto* wp = norm ? reinterpret_cast<const __nv_bfloat16*>(w->data_ptr()) : nullptr;
  auto* hp = norm ? reinterpret_cast<__nv_bfloat16*>(h->data_ptr()) : nullptr;
  auto stream = at::cuda::getCurrentCUDAStream();
  auto* yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  auto* cp = reinterpret_cast<uint32_t*>(ctr.data_ptr());
  if (data_mc != 0)
    tpd::push_reduce_kernel<true><<<(unsigned)rows, tpd::kThreads, 0, stream>>>(
        acc.data_ptr<float>(), acc.stride(0), (int)N, ld, (int)rows_cap, cp, bp, rp, yp, wp, hp, (float)eps, t);
  else
    tpd::push_reduce_kernel<false><<<(unsigned)rows, tpd::kThreads, 0, stream>>>(
        acc.data_ptr<float>(), acc.stride(0), (int)N, ld, (int)rows_cap, cp, bp, rp, yp, wp, hp, (float)eps, t);
  AETHER_CUDA_CHECK(cudaGetLastError());
}

}  // namespace aether
