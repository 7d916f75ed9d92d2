// Host-side helpers shared by the torch extension's .cu/.cpp files.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>

#define AETHER_CUDA_CHECK(expr)                                                                      \
  do {                                                                                               \
    cudaError_t _e = (expr);                                                                         \
    if (_e != cudaSuccess)                                                                           \
      throw std::runtime_error(std::string("CUDA error: ") + cudaGetErrorString(_e) + " at " + \
                               __FILE__ + ":" + std::to_string(__LINE__));                          \
  } while (0)

namespace aether {

int current_device();
int num_sms(int device);

// Per-device int32 status word written by kernels whose bounded waits gave up
// (0 = ok). Read and cleared with read_and_clear_status().
int* device_status_word();
int read_and_clear_status();

// 2-D bf16 tensor map with 128-byte swizzle. `inner`/`outer` are the global
// extents in elements, `row_stride_bytes` the byte distance between rows.
CUtensorMap make_tmap_2d_bf16(const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_bytes,
                              uint32_t box_inner, uint32_t box_outer);

// 2-D tensor map of any element type (CU_TENSOR_MAP_DATA_TYPE_*), given swizzle.
CUtensorMap make_tmap_2d(const void* base, CUtensorMapDataType dtype, uint32_t elem_bytes, uint64_t inner,
                         uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                         CUtensorMapSwizzle swizzle);

// 3-D bf16 tensor map, 128-byte swizzle: dims {inner, mid, outer}.
CUtensorMap make_tmap_3d_bf16(const void* base, uint64_t inner, uint64_t mid, uint64_t outer, uint64_t mid_stride_bytes,
                              uint64_t outer_stride_bytes, uint32_t box_inner, uint32_t box_mid, uint32_t box_outer);

}  // namespace aether
