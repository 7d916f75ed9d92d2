// Block quantisation for frozen base weights (QLoRA): GGUF Q8_0 and Q4_0
// blocks, quantised from and dequantised to bf16 on the GPU.
//
// Block layouts (the published GGUF formats, so files and device buffers are
// interchangeable):
//   Q8_0: 32 values -> f16 scale d, 32 x int8 q;           x = d * q
//   Q4_0: 32 values -> f16 scale d, 16 bytes of nibbles;  x = d * (q - 8), byte j
//         holds element j in its low nibble and element j + 16 in its high one
// Quantisation: Q8_0 d = absmax / 127, q = clamp(rint(x / d), -127, 127);
// Q4_0 d = x[argmax |x|] / -8, q = clamp(rint(x / d) + 8, 0, 15) -- the same
// rules as the CPU quantiser in aether_b200/formats/gguf.py, so both produce
// identical bytes.
//
// Reference: the GGUF quantised weights of the QLoRA stage stay quantised on
// the GPU and are expanded per use (trainer/src/qwen_qlora_stage.rs:78-110);
// the CPU dequantisers are runtime/src/lib.rs:217, 9218-9404.
//
// A warp owns 32 consecutive blocks and a lane one block: the warp's span of
// blocks (32 x 34 or 32 x 18 bytes, a multiple of 16) moves between global
// and shared memory as 16-byte vectors, the bf16 side as 16-byte vectors per
// lane, so global traffic is fully vectorised although blocks are not
// 16-byte aligned. Spans that do not fill a warp take the per-element path.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "host_utils.h"

namespace aether {
namespace quant {

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

template <int BB>  // block bytes: 34 (Q8_0) or 18 (Q4_0)
__device__ __forceinline__ void put_scale(uint8_t* b, __half d16) {
  const uint16_t bits = __half_as_ushort(d16);
  b[0] = (uint8_t)(bits & 0xff);
  b[1] = (uint8_t)(bits >> 8);
}

__device__ __forceinline__ float load_scale(const uint8_t* b) {
  return __half2float(__ushort_as_half((uint16_t)(b[0] | (b[1] << 8))));
}

// 32 bf16 values of one block into registers (four 16-byte loads).
__device__ __forceinline__ void load32(const __nv_bfloat16* x, float (&v)[32]) {
  const uint4* p = reinterpret_cast<const uint4*>(x);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint4 u = __ldg(p + i);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[8 * i + 2 * j] = __uint_as_float(w[j] << 16);
      v[8 * i + 2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
    }
  }
}

__device__ __forceinline__ void store32(__nv_bfloat16* y, const float (&v)[32]) {
  uint4* p = reinterpret_cast<uint4*>(y);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 u;
    u.x = pack2(v[8 * i], v[8 * i + 1]);
    u.y = pack2(v[8 * i + 2], v[8 * i + 3]);
    u.z = pack2(v[8 * i + 4], v[8 * i + 5]);
    u.w = pack2(v[8 * i + 6], v[8 * i + 7]);
    p[i] = u;
  }
}

// Quantise one block (Q8_0 or Q4_0) from 32 values into its BB bytes.
template <int BB>
__device__ __forceinline__ void quant_block(const float (&v)[32], uint8_t* ob) {
  if constexpr (BB == 34) {
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
    const __half d16 = __float2half_rn(amax / 127.f);
    const float d = __half2float(d16);
    const float inv = d > 0.f ? 1.f / d : 0.f;
    put_scale<BB>(ob, d16);
#pragma unroll
    for (int i = 0; i < 32; ++i) ob[2 + i] = (uint8_t)(int8_t)fminf(fmaxf(rintf(v[i] * inv), -127.f), 127.f);
  } else {
    float best = 0.f, val = 0.f;  // the first element of largest magnitude, with its sign
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (fabsf(v[i]) > best) {
        best = fabsf(v[i]);
        val = v[i];
      }
    const __half d16 = __float2half_rn(val / -8.f);
    const float d = __half2float(d16);
    const float inv = d != 0.f ? 1.f / d : 0.f;
    put_scale<BB>(ob, d16);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int lo = (int)fminf(fmaxf(rintf(v[i] * inv) + 8.f, 0.f), 15.f);
      const int hi = (int)fminf(fmaxf(rintf(v[i + 16] * inv) + 8.f, 0.f), 15.f);
      ob[2 + i] = (uint8_t)(lo | (hi << 4));
    }
  }
}

template <int BB>
__device__ __forceinline__ void dequant_block(const uint8_t* b, float (&v)[32]) {
  const float d = load_scale(b);
  if constexpr (BB == 34) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = d * (float)(int8_t)b[2 + i];
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      v[i] = d * (float)((b[2 + i] & 0x0f) - 8);
      v[i + 16] = d * (float)((b[2 + i] >> 4) - 8);
    }
  }
}

constexpr int kWarps = 8;

template <int BB>
__global__ void __launch_bounds__(kWarps * 32) quantize_kernel(const __nv_bfloat16* __restrict__ x,
                                                               uint8_t* __restrict__ out, int64_t nblocks) {
  __shared__ __align__(16) uint8_t span[kWarps][32 * BB];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t blk0 = ((int64_t)blockIdx.x * kWarps + warp) * 32;
  if (blk0 >= nblocks) return;
  const int nb = (int)(nblocks - blk0 < 32 ? nblocks - blk0 : 32);
  if (lane < nb) {
    float v[32];
    load32(x + (blk0 + lane) * 32, v);
    quant_block<BB>(v, span[warp] + lane * BB);
  }
  __syncwarp();
  uint8_t* dst = out + blk0 * BB;
  if (nb == 32) {  // a full span: 16-byte stores (32 * BB is a multiple of 16)
    const uint4* src = reinterpret_cast<const uint4*>(span[warp]);
    for (int i = lane; i < 2 * BB; i += 32) reinterpret_cast<uint4*>(dst)[i] = src[i];
  } else {
    for (int i = lane; i < nb * BB; i += 32) dst[i] = span[warp][i];
  }
}

template <int BB>
__global__ void __launch_bounds__(kWarps * 32) dequant_kernel(const uint8_t* __restrict__ in,
                                                              __nv_bfloat16* __restrict__ y, int64_t nblocks) {
  __shared__ __align__(16) uint8_t span[kWarps][32 * BB];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t blk0 = ((int64_t)blockIdx.x * kWarps + warp) * 32;
  if (blk0 >= nblocks) return;
  const int nb = (int)(nblocks - blk0 < 32 ? nblocks - blk0 : 32);
  const uint8_t* src = in + blk0 * BB;
  if (nb == 32 && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
    for (int i = lane; i < 2 * BB; i += 32)
      reinterpret_cast<uint4*>(span[warp])[i] = __ldg(reinterpret_cast<const uint4*>(src) + i);
  } else {
    for (int i = lane; i < nb * BB; i += 32) span[warp][i] = src[i];
  }
  __syncwarp();
  if (lane < nb) {
    float v[32];
    dequant_block<BB>(span[warp] + lane * BB, v);
    store32(y + (blk0 + lane) * 32, v);
  }
}

}  // namespace quant

namespace {
int block_bytes(int64_t fmt) {
  TORCH_CHECK(fmt == 8 || fmt == 2, "quant: format must be 8 (Q8_0) or 2 (Q4_0)");
  return fmt == 8 ? 34 : 18;
}
}  // namespace

// x: contiguous bf16 with numel % 32 == 0 -> out: uint8 [numel / 32 * block bytes]
void quantize_blocks(at::Tensor x, at::Tensor out, int64_t fmt) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.numel() % 32 == 0,
              "quantize_blocks: contiguous bf16, numel % 32 == 0");
  const int64_t nb = x.numel() / 32;
  TORCH_CHECK(out.scalar_type() == at::kByte && out.is_contiguous() && out.numel() == nb * block_bytes(fmt),
              "quantize_blocks: out size");
  c10::cuda::CUDAGuard g(x.device());
  if (nb == 0) return;
  TORCH_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0, "quantize_blocks: 16-byte aligned input");
  const unsigned grid = (unsigned)((nb + 32 * quant::kWarps - 1) / (32 * quant::kWarps));
  auto st = at::cuda::getCurrentCUDAStream();
  auto xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  if (fmt == 8)
    quant::quantize_kernel<34><<<grid, 32 * quant::kWarps, 0, st>>>(xp, out.data_ptr<uint8_t>(), nb);
  else
    quant::quantize_kernel<18><<<grid, 32 * quant::kWarps, 0, st>>>(xp, out.data_ptr<uint8_t>(), nb);
  AETHER_CUDA_CHECK(cudaGetLastError());
}

void dequantize_blocks(at::Tensor in, at::Tensor y, int64_t fmt) {
  TORCH_CHECK(y.is_cuda() && y.scalar_type() == at::kBFloat16 && y.is_contiguous() && y.numel() % 32 == 0,
              "dequantize_blocks: contiguous bf16 out, numel % 32 == 0");
  const int64_t nb = y.numel() / 32;
  TORCH_CHECK(in.scalar_type() == at::kByte && in.numel() >= nb * block_bytes(fmt), "dequantize_blocks: in size");
  c10::cuda::CUDAGuard g(y.device());
  if (nb == 0) return;
  TORCH_CHECK(reinterpret_cast<uintptr_t>(y.data_ptr()) % 16 == 0, "dequantize_blocks: 16-byte aligned output");
  const unsigned grid = (unsigned)((nb + 32 * quant::kWarps - 1) / (32 * quant::kWarps));
  auto st = at::cuda::getCurrentCUDAStream();
  auto yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  if (fmt == 8)
    quant::dequant_kernel<34><<<grid, 32 * quant::kWarps, 0, st>>>(in.data_ptr<uint8_t>(), yp, nb);
  else
    quant::dequant_kernel<18><<<grid, 32 * quant::kWarps, 0, st>>>(in.data_ptr<uint8_t>(), yp, nb);
  AETHER_CUDA_CHECK(cudaGetLastError());
}

}  // namespace aether
