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
// One warp per 32-value block; lane l owns element l.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "host_utils.h"

namespace aether {
namespace quant {

__global__ void quantize_q8_0_kernel(const __nv_bfloat16* __restrict__ x, uint8_t* __restrict__ out, int64_t nblocks) {
  const int64_t blk = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (blk >= nblocks) return;
  const float v = __bfloat162float(x[blk * 32 + lane]);
  float amax = fabsf(v);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const __half d16 = __float2half_rn(amax / 127.f);
  const float d = __half2float(d16);
  const float inv = d > 0.f ? 1.f / d : 0.f;
  const float q = fminf(fmaxf(rintf(v * inv), -127.f), 127.f);
  uint8_t* ob = out + blk * 34;
  ob[2 + lane] = (uint8_t)(int8_t)q;
  if (lane == 0) {
    const uint16_t bits = __half_as_ushort(d16);
    ob[0] = (uint8_t)(bits & 0xff);
    ob[1] = (uint8_t)(bits >> 8);
  }
}

__global__ void quantize_q4_0_kernel(const __nv_bfloat16* __restrict__ x, uint8_t* __restrict__ out, int64_t nblocks) {
  const int64_t blk = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (blk >= nblocks) return;
  const float v = __bfloat162float(x[blk * 32 + lane]);
  // value of the first element with the largest magnitude
  float best = fabsf(v), val = v;
  int idx = lane;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const float ov = __shfl_xor_sync(0xffffffffu, val, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ob > best || (ob == best && oi < idx)) {
      best = ob;
      val = ov;
      idx = oi;
    }
  }
  const __half d16 = __float2half_rn(val / -8.f);
  const float d = __half2float(d16);
  const float inv = d != 0.f ? 1.f / d : 0.f;
  const int q = (int)fminf(fmaxf(rintf(v * inv) + 8.f, 0.f), 15.f);
  const int hi = __shfl_down_sync(0xffffffffu, q, 16);
  uint8_t* ob = out + blk * 18;
  if (lane < 16) ob[2 + lane] = (uint8_t)(q | (hi << 4));
  if (lane == 0) {
    const uint16_t bits = __half_as_ushort(d16);
    ob[0] = (uint8_t)(bits & 0xff);
    ob[1] = (uint8_t)(bits >> 8);
  }
}

__device__ __forceinline__ float load_scale(const uint8_t* b) {
  return __half2float(__ushort_as_half((uint16_t)(b[0] | (b[1] << 8))));
}

__global__ void dequant_q8_0_kernel(const uint8_t* __restrict__ in, __nv_bfloat16* __restrict__ y, int64_t nblocks) {
  const int64_t blk = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (blk >= nblocks) return;
  const uint8_t* b = in + blk * 34;
  y[blk * 32 + lane] = __float2bfloat16(load_scale(b) * (float)(int8_t)b[2 + lane]);
}

__global__ void dequant_q4_0_kernel(const uint8_t* __restrict__ in, __nv_bfloat16* __restrict__ y, int64_t nblocks) {
  const int64_t blk = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (blk >= nblocks) return;
  const uint8_t* b = in + blk * 18;
  const uint8_t byte = b[2 + (lane & 15)];
  const int q = lane < 16 ? (byte & 0x0f) : (byte >> 4);
  y[blk * 32 + lane] = __float2bfloat16(load_scale(b) * (float)(q - 8));
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
  const unsigned grid = (unsigned)((nb * 32 + 255) / 256);
  auto st = at::cuda::getCurrentCUDAStream();
  auto xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  if (fmt == 8)
    quant::quantize_q8_0_kernel<<<grid, 256, 0, st>>>(xp, out.data_ptr<uint8_t>(), nb);
  else
    quant::quantize_q4_0_kernel<<<grid, 256, 0, st>>>(xp, out.data_ptr<uint8_t>(), nb);
  AETHER_CUDA_CHECK(cudaGetLastError());
}

void dequantize_blocks(at::Tensor in, at::Tensor y, int64_t fmt) {
  TORCH_CHECK(y.is_cuda() && y.scalar_type() == at::kBFloat16 && y.is_contiguous() && y.numel() % 32 == 0,
              "dequantize_blocks: contiguous bf16 out, numel % 32 == 0");
  const int64_t nb = y.numel() / 32;
  TORCH_CHECK(in.scalar_type() == at::kByte && in.numel() >= nb * block_bytes(fmt), "dequantize_blocks: in size");
  c10::cuda::CUDAGuard g(y.device());
  if (nb == 0) return;
  const unsigned grid = (unsigned)((nb * 32 + 255) / 256);
  auto st = at::cuda::getCurrentCUDAStream();
  auto yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  if (fmt == 8)
    quant::dequant_q8_0_kernel<<<grid, 256, 0, st>>>(in.data_ptr<uint8_t>(), yp, nb);
  else
    quant::dequant_q4_0_kernel<<<grid, 256, 0, st>>>(in.data_ptr<uint8_t>(), yp, nb);
  AETHER_CUDA_CHECK(cudaGetLastError());
}

}  // namespace aether
