// Host dequantisers for the GGUF IQ3 block formats (256 values per block):
//   IQ3_XXS (98 bytes): f16 d; 64 codebook indices (4 values each); per 32
//     values one u32 whose top 4 bits give the scale d * (0.5 + s) / 2 and whose
//     four 7-bit fields select sign patterns for 8 values each;
//   IQ3_S (110 bytes): f16 d; 64 low index bytes; 8 bytes of ninth index bits;
//     32 sign bytes (one per 8 values); 4 bytes of 4-bit scales d * (1 + 2 s).
// A 7-bit sign index expands to 8 sign bits: the index plus its parity as bit 7.
// The reference exports aether_dequant_iq3_s (runtime/src/lib.rs:9404); the IQ3_XXS
// form is this library's addition.
#include <cstdint>
#include <cstring>

#include "iq3_grids.inc"

namespace {
float f16(const uint8_t* p) {
  const uint16_t h = (uint16_t)(p[0] | p[1] << 8);
  const uint32_t s = (uint32_t)(h & 0x8000) << 16, e = (h >> 10) & 0x1f, m = h & 0x3ff;
  uint32_t bits;
  if (e == 0) {
    if (m == 0) {
      bits = s;
    } else {  // subnormal: renormalise
      int k = -1;
      uint32_t mm = m;
      do {
        ++k;
        mm <<= 1;
      } while (!(mm & 0x400));
      bits = s | (uint32_t)(127 - 15 - k) << 23 | (mm & 0x3ff) << 13;
    }
  } else if (e == 31) {
    bits = s | 0x7f800000u | m << 13;
  } else {
    bits = s | (e + 112) << 23 | m << 13;
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}
uint8_t sign_pattern(uint32_t idx7) { return (uint8_t)(idx7 | (__builtin_popcount(idx7) & 1) << 7); }
uint8_t grid_val(uint32_t entry, int j) { return (uint8_t)(entry >> (8 * j)); }
}  // namespace

extern "C" {

int aether_dequant_iq3_xxs(const void* blocks, void* out, int n_blocks) {
  if (!blocks || !out || n_blocks < 0) return -1;
  const uint8_t* b = (const uint8_t*)blocks;
  float* o = (float*)out;
  for (int k = 0; k < n_blocks; ++k, b += 98, o += 256) {
    const float d = f16(b);
    const uint8_t* qs = b + 2;
    for (int ib = 0; ib < 8; ++ib) {
      uint32_t aux;
      memcpy(&aux, b + 66 + 4 * ib, 4);
      const float db = d * (0.5f + (float)(aux >> 28)) * 0.5f;
      for (int g = 0; g < 4; ++g) {
        const uint8_t signs = sign_pattern((aux >> (7 * g)) & 127);
        for (int j = 0; j < 8; ++j) {
          const uint32_t e = IQ3XXS_GRID[qs[8 * ib + 2 * g + j / 4]];
          o[32 * ib + 8 * g + j] = db * (float)grid_val(e, j % 4) * ((signs >> j) & 1 ? -1.f : 1.f);
        }
      }
    }
  }
  return 0;
}

int aether_dequant_iq3_s(const void* blocks, void* out, int n_blocks) {
  if (!blocks || !out || n_blocks < 0) return -1;
  const uint8_t* b = (const uint8_t*)blocks;
  float* o = (float*)out;
  for (int k = 0; k < n_blocks; ++k, b += 110, o += 256) {
    const float d = f16(b);
    const uint8_t *qs = b + 2, *qh = b + 66, *signs = b + 74, *sc = b + 106;
    for (int ib = 0; ib < 8; ++ib) {
      const float db = d * (float)(1 + 2 * ((sc[ib / 2] >> (4 * (ib % 2))) & 15));
      for (int g = 0; g < 4; ++g)
        for (int j = 0; j < 8; ++j) {
          const int q = 8 * ib + 2 * g + j / 4;
          const uint32_t e = IQ3S_GRID[qs[q] | ((qh[q / 8] >> (q % 8)) & 1) << 8];
          const float sgn = (signs[4 * ib + g] >> j) & 1 ? -1.f : 1.f;
          o[32 * ib + 8 * g + j] = db * (float)grid_val(e, j % 4) * sgn;
        }
    }
  }
  return 0;
}

}  // extern "C"
