// In-kernel collectives over NVLink 5 / NVSwitch on symmetric memory.
//
// Every rank maps every peer's buffer (P2P pointers) and, where NVSwitch
// multicast (NVLS) is available, one multicast address that fans a store out
// to -- or reduces a load across -- all ranks inside the switch. The kernels:
//
//   team_barrier          release-store an epoch into each peer's signal slot,
//                         acquire-spin (bounded) on the own slots; graph-safe
//                         (the epoch is a device counter, not a launch arg)
//   allreduce_sum         one-shot over P2P loads, or two-shot NVLS
//                         (multimem.ld_reduce of an owned slice, multimem.st of
//                         the sum) -- bf16 or fp32
//   dp_reduce_adamw       the data-parallel optimiser step as ONE kernel:
//                         reduce this rank's gradient shard across all ranks
//                         (multimem.ld_reduce or P2P loads), scale, AdamW on the
//                         fp32 master/m/v shard, and write the new bf16
//                         parameters into every rank's compute copy
//                         (multimem.st or P2P stores) -- i.e. reduce-scatter +
//                         update + all-gather without a round trip through NCCL
//
// Reference: the only real collective of the reference is an NCCL all-reduce
// of the whole fp32 gradient followed by identical AdamW on every rank
// (trainer/src/dp.rs:99-105; runtime/src/nccl_real.rs:60-100).
//
// Waits are bounded (kCommTimeoutNs); on timeout the kernel records
// kStatusTimeoutPeer in the status word and returns, leaving the context usable.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "host_utils.h"

namespace aether {
namespace comm {

constexpr int kMaxWorld = 8;

struct Team {
  uint64_t peer_sig[kMaxWorld];  // each rank's signal slots (uint32 [kMaxWorld]) as seen from this rank
  uint32_t* my_sig;              // this rank's slots
  uint32_t* epoch;               // local device counter of barriers issued
  int* status;
  int rank, world;
  uint64_t timeout_ns;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One block; thread p signals peer p and waits for peer p's signal.
__global__ void team_barrier_kernel(Team t) {
  __shared__ uint32_t s_epoch;
  if (threadIdx.x == 0) s_epoch = *t.epoch + 1;
  asm volatile("fence.sc.sys;" ::: "memory");  // this rank's earlier writes (local and remote) first
  __syncthreads();
  const uint32_t e = s_epoch;
  const int p = threadIdx.x;
  if (p < t.world && p != t.rank) {
    st_release_sys(reinterpret_cast<uint32_t*>(t.peer_sig[p]) + t.rank, e);
    const uint64_t t0 = globaltimer_ns();
    uint32_t it = 0;
    while ((int32_t)(ld_acquire_sys(t.my_sig + p) - e) < 0) {
      if ((++it & 255u) == 0 && globaltimer_ns() - t0 > t.timeout_ns) {
        atomicExch(t.status, kStatusTimeoutPeer);
        break;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) *t.epoch = e;
}

// ---------------------------------------------------------------- multimem PTX
__device__ __forceinline__ float4 mm_ld_reduce_f32x4(const float* mc) {
  float4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(mc)
               : "memory");
  return v;
}
__device__ __forceinline__ void mm_st_f32x4(float* mc, float4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(mc), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}
// 8 bf16 (16 bytes) reduced across ranks with fp32 accumulation in the switch.
__device__ __forceinline__ uint4 mm_ld_reduce_bf16x8(const __nv_bfloat16* mc) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(mc)
               : "memory");
  return v;
}
__device__ __forceinline__ void mm_st_b128(void* mc, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(mc), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void mm_st_b64(void* mc, uint2 v) {
  asm volatile("multimem.st.relaxed.sys.global.v2.f32 [%0], {%1,%2};" ::"l"(mc), "r"(v.x), "r"(v.y) : "memory");
}

// ---------------------------------------------------------------- all-reduce
// One-shot: every rank sums all peers' copies of its whole buffer (P2P loads).
template <typename T>
__global__ void allreduce_oneshot_kernel(const uint64_t* __restrict__ peers, int world, T* __restrict__ out,
                                         int64_t n_vec);

template <>
__global__ void allreduce_oneshot_kernel<float>(const uint64_t* __restrict__ peers, int world, float* __restrict__ out,
                                                int64_t n_vec) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_vec; i += (int64_t)gridDim.x * blockDim.x) {
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int p = 0; p < world; ++p) {
      const float4 v = reinterpret_cast<const float4*>(peers[p])[i];
      s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
    }
    reinterpret_cast<float4*>(out)[i] = s;
  }
}

template <>
__global__ void allreduce_oneshot_kernel<__nv_bfloat16>(const uint64_t* __restrict__ peers, int world,
                                                        __nv_bfloat16* __restrict__ out, int64_t n_vec) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_vec; i += (int64_t)gridDim.x * blockDim.x) {
    float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int p = 0; p < world; ++p) {
      const uint4 v = reinterpret_cast<const uint4*>(peers[p])[i];
      s[0] += bf16lo(v.x); s[1] += bf16hi(v.x); s[2] += bf16lo(v.y); s[3] += bf16hi(v.y);
      s[4] += bf16lo(v.z); s[5] += bf16hi(v.z); s[6] += bf16lo(v.w); s[7] += bf16hi(v.w);
    }
    uint4 o;
    o.x = pack_bf16(s[0], s[1]); o.y = pack_bf16(s[2], s[3]);
    o.z = pack_bf16(s[4], s[5]); o.w = pack_bf16(s[6], s[7]);
    reinterpret_cast<uint4*>(out)[i] = o;
  }
}

// Two-shot NVLS: rank r reduces slice r through the switch and multicasts it.
__global__ void allreduce_nvls_f32_kernel(float* mc, int64_t n_vec, int rank, int world) {
  const int64_t per = (n_vec + world - 1) / world;
  const int64_t b = rank * per, e = min(n_vec, b + per);
  for (int64_t i = b + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < e; i += (int64_t)gridDim.x * blockDim.x)
    mm_st_f32x4(mc + 4 * i, mm_ld_reduce_f32x4(mc + 4 * i));
}

__global__ void allreduce_nvls_bf16_kernel(__nv_bfloat16* mc, int64_t n_vec, int rank, int world) {
  const int64_t per = (n_vec + world - 1) / world;
  const int64_t b = rank * per, e = min(n_vec, b + per);
  for (int64_t i = b + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < e; i += (int64_t)gridDim.x * blockDim.x)
    mm_st_b128(mc + 8 * i, mm_ld_reduce_bf16x8(mc + 8 * i));
}

// ---------------------------------------------------------------- DP optimiser
struct AdamArgs {
  float lr, beta1, beta2, eps, wd, bc1_inv, bc2_inv, gscale;
};

__device__ __forceinline__ float adam1(float& p, float g, float& m, float& v, const AdamArgs& a, float wd) {
  m = a.beta1 * m + (1.f - a.beta1) * g;
  v = a.beta2 * v + (1.f - a.beta2) * g * g;
  p -= a.lr * ((m * a.bc1_inv) / (sqrtf(v * a.bc2_inv) + a.eps) + wd * p);
  return p;
}

// Shard [begin, begin + n) of the flat arena (n % 4 == 0, begin % 4 == 0).
// grad: NVLS multicast pointer of the fp32 gradient arena (MC) or the peer
// pointer table (P2P); param: same for the bf16 compute copy.
// decay_blocks: one byte per 128-element block of the arena (1 = weight decay).
template <bool MC>
__global__ void dp_reduce_adamw_kernel(const uint64_t* __restrict__ grad_peers, float* grad_mc,
                                       const uint64_t* __restrict__ param_peers, __nv_bfloat16* param_mc,
                                       float* __restrict__ master, float* __restrict__ m, float* __restrict__ v,
                                       const uint8_t* __restrict__ decay_blocks, int64_t begin, int64_t n, int world,
                                       AdamArgs a, const float* __restrict__ gscale_ptr) {
  const float gs = a.gscale * (gscale_ptr ? *gscale_ptr : 1.f);
  const int64_t n4 = n / 4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t idx = begin + 4 * i;  // arena index
    float4 g;
    if constexpr (MC) {
      g = mm_ld_reduce_f32x4(grad_mc + idx);
    } else {
      g = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int p = 0; p < world; ++p) {
        const float4 t = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(grad_peers[p]) + idx);
        g.x += t.x; g.y += t.y; g.z += t.z; g.w += t.w;
      }
    }
    const float wd = decay_blocks[idx >> 7] ? a.wd : 0.f;
    float4 pp = reinterpret_cast<float4*>(master)[i];
    float4 mm = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    adam1(pp.x, g.x * gs, mm.x, vv.x, a, wd);
    adam1(pp.y, g.y * gs, mm.y, vv.y, a, wd);
    adam1(pp.z, g.z * gs, mm.z, vv.z, a, wd);
    adam1(pp.w, g.w * gs, mm.w, vv.w, a, wd);
    reinterpret_cast<float4*>(master)[i] = pp;
    reinterpret_cast<float4*>(m)[i] = mm;
    reinterpret_cast<float4*>(v)[i] = vv;
    uint2 o;
    o.x = pack_bf16(pp.x, pp.y);
    o.y = pack_bf16(pp.z, pp.w);
    if constexpr (MC) {
      mm_st_b64(param_mc + idx, o);
    } else {
      for (int p = 0; p < world; ++p)
        *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(param_peers[p]) + idx) = o;
    }
  }
}

}  // namespace comm

// --------------------------------------------------------------------- host API
namespace {
comm::Team make_team(at::Tensor peer_sig_ptrs, at::Tensor my_sig, at::Tensor epoch, int64_t rank, int64_t world,
                     double timeout_s) {
  TORCH_CHECK(world >= 1 && world <= comm::kMaxWorld, "team: world size must be in [1, 8]");
  TORCH_CHECK(peer_sig_ptrs.scalar_type() == at::kLong && peer_sig_ptrs.numel() == world && !peer_sig_ptrs.is_cuda(),
              "team: peer_sig_ptrs must be a CPU int64 tensor of world entries");
  comm::Team t{};
  auto acc = peer_sig_ptrs.accessor<int64_t, 1>();
  for (int i = 0; i < world; ++i) t.peer_sig[i] = (uint64_t)acc[i];
  t.my_sig = reinterpret_cast<uint32_t*>(my_sig.data_ptr());
  t.epoch = reinterpret_cast<uint32_t*>(epoch.data_ptr());
  t.status = device_status_word();
  t.rank = (int)rank;
  t.world = (int)world;
  t.timeout_ns = (uint64_t)(timeout_s * 1e9);
  return t;
}

int grid_for(int64_t n_vec) {
  const int sms = num_sms(current_device());
  return (int)std::max<int64_t>(1, std::min<int64_t>((n_vec + 255) / 256, (int64_t)sms * 4));
}
}  // namespace

void team_barrier(at::Tensor peer_sig_ptrs, at::Tensor my_sig, at::Tensor epoch, int64_t rank, int64_t world,
                  double timeout_s) {
  c10::cuda::CUDAGuard g(my_sig.device());
  comm::Team t = make_team(peer_sig_ptrs, my_sig, epoch, rank, world, timeout_s);
  comm::team_barrier_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(t);
  AETHER_CUDA_CHECK(cudaGetLastError());
}

// out = sum over ranks of the symmetric buffer (P2P one-shot). peers: CUDA int64 [world].
void allreduce_oneshot(at::Tensor peers, at::Tensor out, int64_t world) {
  c10::cuda::CUDAGuard g(out.device());
  TORCH_CHECK(peers.is_cuda() && peers.scalar_type() == at::kLong, "allreduce_oneshot: device pointer table");
  TORCH_CHECK(out.is_contiguous(), "allreduce_oneshot: contiguous out");
  auto stream = at::cuda::getCurrentCUDAStream();
  const uint64_t* pp = reinterpret_cast<const uint64_t*>(peers.data_ptr());
  if (out.scalar_type() == at::kFloat) {
    TORCH_CHECK(out.numel() % 4 == 0, "allreduce: fp32 numel % 4");
    const int64_t nv = out.numel() / 4;
    comm::allreduce_oneshot_kernel<float><<<grid_for(nv), 256, 0, stream>>>(pp, (int)world, out.data_ptr<float>(), nv);
  } else {
    TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.numel() % 8 == 0, "allreduce: bf16 numel % 8");
    const int64_t nv = out.numel() / 8;
    comm::allreduce_oneshot_kernel<__nv_bfloat16><<<grid_for(nv), 256, 0, stream>>>(
        pp, (int)world, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), nv);
  }
  AETHER_CUDA_CHECK(cudaGetLastError());
}

// In-place NVLS all-reduce of `numel` elements at multicast address mc_ptr.
void allreduce_nvls(int64_t mc_ptr, int64_t numel, bool is_bf16, int64_t rank, int64_t world) {
  auto stream = at::cuda::getCurrentCUDAStream();
  if (is_bf16) {
    TORCH_CHECK(numel % 8 == 0, "allreduce_nvls: bf16 numel % 8");
    const int64_t nv = numel / 8;
    comm::allreduce_nvls_bf16_kernel<<<grid_for(nv / world + 1), 256, 0, stream>>>(
        reinterpret_cast<__nv_bfloat16*>(mc_ptr), nv, (int)rank, (int)world);
  } else {
    TORCH_CHECK(numel % 4 == 0, "allreduce_nvls: fp32 numel % 4");
    const int64_t nv = numel / 4;
    comm::allreduce_nvls_f32_kernel<<<grid_for(nv / world + 1), 256, 0, stream>>>(reinterpret_cast<float*>(mc_ptr), nv,
                                                                                 (int)rank, (int)world);
  }
  AETHER_CUDA_CHECK(cudaGetLastError());
}

// Fused DP step over this rank's shard [begin, begin + n) of the flat arena.
// grad_mc / param_mc: multicast addresses (0 = use the P2P tables instead).
void dp_reduce_adamw(at::Tensor grad_peers, int64_t grad_mc, at::Tensor param_peers, int64_t param_mc,
                     at::Tensor master, at::Tensor m, at::Tensor v, at::Tensor decay_blocks, int64_t begin, int64_t n,
                     int64_t world, double lr, double beta1, double beta2, double eps, double wd, int64_t step,
                     double gscale, std::optional<at::Tensor> gscale_t) {
  c10::cuda::CUDAGuard g(master.device());
  TORCH_CHECK(n % 4 == 0 && begin % 4 == 0, "dp_reduce_adamw: shard must be 4-aligned");
  TORCH_CHECK(master.numel() >= n && m.numel() >= n && v.numel() >= n, "dp_reduce_adamw: state sizes");
  TORCH_CHECK(decay_blocks.is_cuda() && decay_blocks.scalar_type() == at::kByte, "dp_reduce_adamw: decay mask");
  comm::AdamArgs a;
  a.lr = (float)lr;
  a.beta1 = (float)beta1;
  a.beta2 = (float)beta2;
  a.eps = (float)eps;
  a.wd = (float)wd;
  a.bc1_inv = (float)(1.0 / (1.0 - std::pow(beta1, (double)step)));
  a.bc2_inv = (float)(1.0 / (1.0 - std::pow(beta2, (double)step)));
  a.gscale = (float)gscale;
  const float* gsp = (gscale_t && gscale_t->defined()) ? gscale_t->data_ptr<float>() : nullptr;
  auto stream = at::cuda::getCurrentCUDAStream();
  const int grid = grid_for(n / 4);
  if (grad_mc != 0 && param_mc != 0) {
    comm::dp_reduce_adamw_kernel<true><<<grid, 256, 0, stream>>>(
        nullptr, reinterpret_cast<float*>(grad_mc), nullptr, reinterpret_cast<__nv_bfloat16*>(param_mc),
        master.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), decay_blocks.data_ptr<uint8_t>(), begin, n,
        (int)world, a, gsp);
  } else {
    TORCH_CHECK(grad_peers.is_cuda() && param_peers.is_cuda(), "dp_reduce_adamw: device pointer tables");
    comm::dp_reduce_adamw_kernel<false><<<grid, 256, 0, stream>>>(
        reinterpret_cast<const uint64_t*>(grad_peers.data_ptr()), nullptr,
        reinterpret_cast<const uint64_t*>(param_peers.data_ptr()), nullptr, master.data_ptr<float>(),
        m.data_ptr<float>(), v.data_ptr<float>(), decay_blocks.data_ptr<uint8_t>(), begin, n, (int)world, a, gsp);
  }
  AETHER_CUDA_CHECK(cudaGetLastError());
}

}  // namespace aether
