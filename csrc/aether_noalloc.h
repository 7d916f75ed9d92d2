// Allocation-free entry point for split-K decode attention.
//
// This entry point has no counterpart in the reference: the reference's
// decode attention takes its scratch from buffers its session allocated.
//
// Who needs it: callers that must not allocate device memory on the call
// path. Examples are a server that has handed all free device memory to its
// KV-cache pool (an allocation could fail mid-request), and a host runtime
// that forbids allocation on its hot path because freeing device memory
// synchronises the device and allocators can block on a lock. The regular
// entry point (`decode_attention` in the Python extension) takes its scratch
// as tensors, which the caller must allocate; this one takes none.
//
// How: the split partials and the combine counters live in one fixed block of
// device memory per GPU (a file-scope `__device__` array in the library), so
// the call itself allocates nothing, through CUDA, torch or anything else.
//
// Limits and rules:
//   * B * Hq * splits <= AETHER_NOALLOC_MAX_PARTIAL_ROWS (8192) and
//     B * Hkv <= AETHER_NOALLOC_MAX_COUNTERS (1024); larger problems are
//     rejected with AETHER_NOALLOC_ETOOBIG before anything is launched.
//     The scratch costs 8192 * 129 * 4 bytes + 4 KB, about 4.2 MB per GPU.
//   * D must be 128, Hq a multiple of Hkv with Hq / Hkv <= 8, 1 <= splits <= 64.
//   * Alignment, because the kernel moves K/V rows in 16-byte copies, q in
//     4-byte loads and out in 8-byte stores: k_cache and v_cache 16-byte
//     aligned with slot_stride and pos_stride multiples of 8 elements; q
//     4-byte aligned with q_rs even; out 8-byte aligned with out_rs a multiple
//     of 4. Anything else returns AETHER_NOALLOC_EINVAL and launches nothing.
//   * `stream` must belong to the current device (the scratch address is the
//     current device's); a stream of another device returns
//     AETHER_NOALLOC_EINVAL.
//   * The first call on each device does one-time set-up for that device: it
//     looks up the scratch address, raises the kernel's shared-memory limit and
//     clears the counters (a memset followed by a device synchronise). Make
//     that first call before any stream capture, for example with a tiny
//     warm-up problem. If the set-up fails, the call returns
//     AETHER_NOALLOC_ECUDA and the next call on that device tries again.
//   * The scratch is shared by all calls on a device. Two calls whose
//     executions overlap (different streams, or different host threads without
//     ordering between them) race on it and give wrong results. Order the
//     calls, e.g. issue them on one stream.
//   * The call is asynchronous on `stream` (a cudaStream_t; null means the
//     legacy default stream). The return value only reports argument and
//     launch errors.
#pragma once

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AETHER_NOALLOC_MAX_PARTIAL_ROWS 8192
#define AETHER_NOALLOC_MAX_COUNTERS 1024

#define AETHER_NOALLOC_OK 0
#define AETHER_NOALLOC_EINVAL (-1)   // unsupported shape or null pointer
#define AETHER_NOALLOC_ETOOBIG (-2)  // problem exceeds the static scratch
#define AETHER_NOALLOC_ECUDA (-3)    // set-up or launch failed (cudaGetLastError)

// q:       [B, q_rs] bf16, head h of the new token at q + h * D
// k_cache, v_cache: bf16, element (slot s, position t, kv head h, d) at
//          s * slot_stride + t * pos_stride + h * D + d
// slot:    [B] int32 cache slot per row; seqlen: [B] int32 valid keys per row
// out:     [B, out_rs] bf16, head h at out + h * D
// scale:   softmax scale (usually 1 / sqrt(D))
int aether_decode_attention_noalloc(const void* q, int64_t q_rs, const void* k_cache, const void* v_cache,
                                    int64_t slot_stride, int64_t pos_stride, const int* slot, const int* seqlen,
                                    void* out, int64_t out_rs, int B, int Hq, int Hkv, int D, int splits,
                                    float scale, void* stream);

#ifdef __cplusplus
}
#endif
