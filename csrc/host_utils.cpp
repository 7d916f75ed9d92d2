// Device properties, the kernel status word and TMA descriptor encoding.
#include "host_utils.h"

#include <mutex>
#include <vector>

namespace aether {

namespace {
constexpr int kMaxDevices = 64;
int g_num_sms[kMaxDevices] = {0};
int* g_status[kMaxDevices] = {nullptr};
std::mutex g_mu;

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q);
    if (e == cudaSuccess && q == cudaDriverEntryPointSuccess) fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  if (fn == nullptr) throw std::runtime_error("cuTensorMapEncodeTiled is unavailable from the driver");
  return fn;
}
}  // namespace

int current_device() {
  int d = 0;
  AETHER_CUDA_CHECK(cudaGetDevice(&d));
  return d;
}

int num_sms(int device) {
  if (g_num_sms[device] == 0) {
    int n = 0;
    AETHER_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device));
    g_num_sms[device] = n;
  }
  return g_num_sms[device];
}

int* device_status_word() {
  const int d = current_device();
  if (g_status[d] == nullptr) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_status[d] == nullptr) {
      int* p = nullptr;
      AETHER_CUDA_CHECK(cudaMalloc(&p, sizeof(int)));
      AETHER_CUDA_CHECK(cudaMemset(p, 0, sizeof(int)));
      g_status[d] = p;
    }
  }
  return g_status[d];
}

int read_and_clear_status() {
  int* p = device_status_word();
  int v = 0;
  AETHER_CUDA_CHECK(cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost));
  if (v != 0) AETHER_CUDA_CHECK(cudaMemset(p, 0, sizeof(int)));
  return v;
}

// Driver calls (tensor-map encoding) need a context current on the calling
// thread. Threads that have not made a runtime call yet (autograd's device
// worker, for one) have none, so bind the runtime's primary context once per
// thread.
static void ensure_context_bound() {
  thread_local bool bound = false;
  if (!bound) {
    AETHER_CUDA_CHECK(cudaFree(nullptr));
    bound = true;
  }
}

CUtensorMap make_tmap_2d_bf16(const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_bytes,
                              uint32_t box_inner, uint32_t box_outer) {
  ensure_context_bound();
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) throw std::runtime_error("TMA base must be 16-byte aligned");
  if (row_stride_bytes % 16 != 0) throw std::runtime_error("TMA row stride must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled (2d) failed: " + std::to_string((int)r));
  return m;
}

CUtensorMap make_tmap_2d(const void* base, CUtensorMapDataType dtype, uint32_t elem_bytes, uint64_t inner,
                         uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                         CUtensorMapSwizzle swizzle) {
  ensure_context_bound();
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) throw std::runtime_error("TMA base must be 16-byte aligned");
  if (row_stride_bytes % 16 != 0) throw std::runtime_error("TMA row stride must be a multiple of 16 bytes");
  if ((box_inner * elem_bytes) % 16 != 0) throw std::runtime_error("TMA box inner extent must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled (2d) failed: " + std::to_string((int)r));
  return m;
}

CUtensorMap make_tmap_3d_bf16(const void* base, uint64_t inner, uint64_t mid, uint64_t outer, uint64_t mid_stride_bytes,
                              uint64_t outer_stride_bytes, uint32_t box_inner, uint32_t box_mid, uint32_t box_outer) {
  ensure_context_bound();
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) throw std::runtime_error("TMA base must be 16-byte aligned");
  if (mid_stride_bytes % 16 != 0 || outer_stride_bytes % 16 != 0)
    throw std::runtime_error("TMA strides must be multiples of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[3] = {inner, mid, outer};
  cuuint64_t strides[2] = {mid_stride_bytes, outer_stride_bytes};
  cuuint32_t box[3] = {box_inner, box_mid, box_outer};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled (3d) failed: " + std::to_string((int)r));
  return m;
}

}  // namespace aether
