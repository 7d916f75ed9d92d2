// GGUF weight blocks -> bf16 rows on the device, for frozen quantised bases
// that are expanded right before each use (QLoRA over a GGUF model).
//
// One thread decodes one 32-element run of a row (a whole Q4_0 / Q5_0 / Q8_0
// block, or an eighth of a Q4_K / Q5_K / Q6_K super-block) and writes it as
// four 16-byte bf16 stores. The block layouts are the published GGUF formats
// (the same arithmetic as the host dequantiser in formats/gguf.py):
//   Q8_0  fp16 d, 32 x int8                          x = d q
//   Q4_0  fp16 d, 16 B of nibbles (low: 0-15)        x = d (q - 8)
//   Q5_0  fp16 d, u32 high bits, 16 B of nibbles     x = d (q - 16)
//   Q4_K  fp16 d, dmin, 12 B of 6-bit (scale, min) pairs, 128 B nibbles
//         run j: x = d sc_j q - dmin m_j (runs 2g / 2g+1 = low / high nibbles of bytes 32g..)
//   Q5_K  as Q4_K plus 32 B of high bits (bit 2g / 2g+1 of byte i)
//   Q6_K  128 B low 4 bits, 64 B high 2 bits, 16 int8 scales, fp16 d
//   F32 / F16 / BF16 plain.
// Reference: the device dequantiser cuda.rs:6388 (dequant_iq3_xxs) and the
// per-format fused mat-vecs (cuda.rs:3347-3420); format tables from the GGUF
// specification.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "host_utils.h"

namespace aether {
namespace gq {

enum : int { F32 = 0, F16 = 1, Q4_0 = 2, Q5_0 = 6, Q8_0 = 8, Q4_K = 12, Q5_K = 13, Q6_K = 14, BF16 = 30 };

__device__ __forceinline__ float f16_at(const uint8_t* p) {
  return __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
}

// the j-th (scale, min) pair of the 12 packed bytes of Q4_K / Q5_K
__device__ __forceinline__ void k4_scale(const uint8_t* sc, int j, float& s, float& m) {
  if (j < 4) {
    s = (float)(sc[j] & 63);
    m = (float)(sc[j + 4] & 63);
  } else {
    s = (float)((sc[j + 4] & 0x0F) | ((sc[j - 4] >> 6) << 4));
    m = (float)((sc[j + 4] >> 4) | ((sc[j] >> 6) << 4));
  }
}

__global__ void dequant_kernel(const uint8_t* __restrict__ blocks, int type, int64_t rows, int K,
                               int64_t row_bytes, __nv_bfloat16* __restrict__ out, int64_t ld) {
  const int runs = K >> 5;
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows * runs) return;
  const int64_t row = r / runs;
  const int run = (int)(r - row * runs);
  const uint8_t* rb = blocks + row * row_bytes;
  float v[32];
  switch (type) {
    case F32: {
      const float* f = reinterpret_cast<const float*>(rb) + run * 32;
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = f[i];
      break;
    }
    case F16: {
      const uint8_t* b = rb + run * 64;
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = f16_at(b + 2 * i);
      break;
    }
    case BF16: {
      const uint8_t* b = rb + run * 64;
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = __uint_as_float((uint32_t)(b[2 * i] | (b[2 * i + 1] << 8)) << 16);
      break;
    }
    case Q8_0: {
      const uint8_t* b = rb + run * 34;
      const float d = f16_at(b);
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = d * (float)(int8_t)b[2 + i];
      break;
    }
    case Q4_0: {
      const uint8_t* b = rb + run * 18;
      const float d = f16_at(b);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        v[i] = d * ((float)(b[2 + i] & 0x0F) - 8.f);
        v[i + 16] = d * ((float)(b[2 + i] >> 4) - 8.f);
      }
      break;
    }
    case Q5_0: {
      const uint8_t* b = rb + run * 22;
      const float d = f16_at(b);
      const uint32_t qh = b[2] | (b[3] << 8) | (b[4] << 16) | ((uint32_t)b[5] << 24);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int lo = (b[6 + i] & 0x0F) | (((qh >> i) & 1) << 4);
        const int hi = (b[6 + i] >> 4) | (((qh >> (i + 16)) & 1) << 4);
        v[i] = d * (float)(lo - 16);
        v[i + 16] = d * (float)(hi - 16);
      }
      break;
    }
    case Q4_K:
    case Q5_K: {
      const int nb = type == Q4_K ? 144 : 176;
      const uint8_t* b = rb + (run >> 3) * nb;
      const int j = run & 7, g = j >> 1, hi = j & 1;
      const float d = f16_at(b), dmin = f16_at(b + 2);
      float sc, mn;
      k4_scale(b + 4, j, sc, mn);
      const float a = d * sc, c = dmin * mn;
      const uint8_t* qs = b + (type == Q4_K ? 16 : 48) + g * 32;
      const uint8_t* qh = b + 16;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        int q = hi ? (qs[i] >> 4) : (qs[i] & 0x0F);
        if (type == Q5_K) q |= ((qh[i] >> (2 * g + hi)) & 1) << 4;
        v[i] = a * (float)q - c;
      }
      break;
    }
    case Q6_K: {
      const uint8_t* b = rb + (run >> 3) * 210;
      const int j = run & 7, half = j >> 2, part = j & 3;
      const uint8_t* ql = b + half * 64 + ((part & 1) ? 32 : 0);
      const uint8_t* qh = b + 128 + half * 32;
      const int8_t* sc = reinterpret_cast<const int8_t*>(b + 192) + half * 8 + part * 2;
      const float d = f16_at(b + 208);
      const int lsh = (part >= 2) ? 4 : 0, hsh = 2 * part;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int q = ((ql[i] >> lsh) & 0x0F) | (((qh[i] >> hsh) & 3) << 4);
        v[i] = d * (float)sc[i >> 4] * (float)(q - 32);
      }
      break;
    }
    default:
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = 0.f;
  }
  uint4* o = reinterpret_cast<uint4*>(out + row * ld + run * 32);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 u;
    u.x = pack_bf16(v[8 * q + 0], v[8 * q + 1]);
    u.y = pack_bf16(v[8 * q + 2], v[8 * q + 3]);
    u.z = pack_bf16(v[8 * q + 4], v[8 * q + 5]);
    u.w = pack_bf16(v[8 * q + 6], v[8 * q + 7]);
    o[q] = u;
  }
}

int64_t row_bytes_of(int type, int K) {
  switch (type) {
    case F32: return (int64_t)K * 4;
    case F16:
    case BF16: return (int64_t)K * 2;
    case Q8_0: return (int64_t)K / 32 * 34;
    case Q4_0: return (int64_t)K / 32 * 18;
    case Q5_0: return (int64_t)K / 32 * 22;
    case Q4_K: return (int64_t)K / 256 * 144;
    case Q5_K: return (int64_t)K / 256 * 176;
    case Q6_K: return (int64_t)K / 256 * 210;
    default: return -1;
  }
}

}  // namespace gq

// True if the device decoder handles this GGUF tensor type.
bool gguf_device_type(int64_t type) { return gq::row_bytes_of((int)type, 256) > 0; }

// blocks: uint8 CUDA tensor holding `rows` rows of K elements of GGUF type
// `type` back to back; out: bf16 [rows, >= K] with unit inner stride and a
// row stride that is a multiple of 8.
void gguf_dequant(at::Tensor blocks, int64_t type, int64_t rows, int64_t K, at::Tensor out) {
  const int64_t rb = gq::row_bytes_of((int)type, (int)K);
  TORCH_CHECK(rb > 0, "gguf_dequant: tensor type ", type, " has no device decoder");
  const int64_t blk = (type == gq::Q4_K || type == gq::Q5_K || type == gq::Q6_K) ? 256 : 32;
  TORCH_CHECK(K % blk == 0, "gguf_dequant: K must be a multiple of the block size");
  TORCH_CHECK(blocks.is_cuda() && blocks.scalar_type() == at::kByte && blocks.is_contiguous() &&
                  blocks.numel() >= rows * rb,
              "gguf_dequant: blocks uint8 contiguous, rows x row bytes");
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kBFloat16 && out.dim() == 2 && out.size(0) >= rows &&
                  out.size(1) >= K && out.stride(1) == 1 && out.stride(0) % 8 == 0 &&
                  reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0,
              "gguf_dequant: out bf16 [rows, >= K], 16-byte aligned rows");
  if (type == gq::F32)
    TORCH_CHECK(reinterpret_cast<uintptr_t>(blocks.data_ptr()) % 4 == 0, "gguf_dequant: F32 rows 4-byte aligned");
  c10::cuda::CUDAGuard g(blocks.device());
  const int64_t n = rows * (K / 32);
  if (n == 0) return;
  gq::dequant_kernel<<<(unsigned)((n + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      blocks.data_ptr<uint8_t>(), (int)type, rows, (int)K, rb, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
      out.stride(0));
  AETHER_CUDA_CHECK(cudaGetLastError());
}

}  // namespace aether
