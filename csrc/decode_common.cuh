// Device helpers shared by the decode kernels (decode_attention.cu) and the
// decode GEMM's fused QKV epilogue (gemm_skinny.cu): bf16 x8 packing and the
// paged-KV address map.
#pragma once

#include <ATen/ATen.h>

#include "common.cuh"

namespace aether {
namespace dec {

__device__ __forceinline__ void unpack8(const uint4& u, float (&v)[8]) {
  v[0] = bf16lo(u.x); v[1] = bf16hi(u.x); v[2] = bf16lo(u.y); v[3] = bf16hi(u.y);
  v[4] = bf16lo(u.z); v[5] = bf16hi(u.z); v[6] = bf16lo(u.w); v[7] = bf16hi(u.w);
}
__device__ __forceinline__ uint4 pack8(const float (&v)[8]) {
  uint4 u;
  u.x = pack_bf16(v[0], v[1]); u.y = pack_bf16(v[2], v[3]);
  u.z = pack_bf16(v[4], v[5]); u.w = pack_bf16(v[6], v[7]);
  return u;
}

// Paged KV: with a page table, a cache is a pool [pages, page_size, Hkv, D]
// and key t of the sequence in table row `seq` lives in physical page
// table[seq * stride + t / page_size] at row t % page_size (page_size a power of
// two). Without one, the cache is [slots, max_seq, Hkv, D] indexed by slot.
struct PageMap {
  const int* table = nullptr;
  int stride = 0;
  int shift = 0;
};

// element offset of (sequence row `seq`, position t) -- head 0, dim 0
__device__ __forceinline__ int64_t kv_offset(const PageMap& pm, int seq, int t, int64_t slot_stride,
                                             int64_t pos_stride) {
  if (pm.table == nullptr) return (int64_t)seq * slot_stride + (int64_t)t * pos_stride;
  const int64_t phys = pm.table[(int64_t)seq * pm.stride + (t >> pm.shift)];
  return ((phys << pm.shift) | (int64_t)(t & ((1 << pm.shift) - 1))) * pos_stride;
}

}  // namespace dec

// page_table: CUDA int32 [rows, max_pages] (rows indexed by `slot`), caches
// [pages, page_size, Hkv, D] with page_size a power of two; no table: a
// contiguous [slots, max_seq, Hkv, D] cache.
dec::PageMap page_map(const std::optional<at::Tensor>& page_table, const at::Tensor& cache);

}  // namespace aether
