// Whole-model decode step in ONE persistent kernel (batch 1..4, Qwen2 / Llama
// family, head_dim 128), for one GPU or one tensor-parallel rank.
//
// Why: at batch 1 a decode step streams every weight once (Qwen2.5-7B at TP=8:
// 58 MB per layer per rank, about 9 us of HBM time), but a kernel-per-op step
// pays a launch, a ramp and a tail for each of ~9 dependent kernels per layer.
// Here one CTA per SM lives for the whole step:
//   warp 14     : producer -- streams this CTA's share of every weight matrix
//                 (contiguous row ranges, 1-D cp.async.bulk) through a 3-stage
//                 shared-memory ring, in the exact order the consumers use
//                 them, running ahead ACROSS phase boundaries: weights do not
//                 depend on activations, so the next phase's rows are already
//                 in flight while the consumers wait at a barrier
//   warps 0..13 : consumers -- per layer
//       A  h = RMSNorm(x);  qkv rows (pairs d, d+64 of a head) + bias, RoPE;
//          q to scratch, k / v appended to the KV cache
//       B  split-K attention (one CTA per (row, KV head, key range); online
//          softmax over 64-key chunks; the last CTA of a (row, KV head)
//          merges the partials by log-sum-exp)
//       C  o_proj rows -> partial sums reduced over the TP ranks through the
//          NVSwitch (multimem.red into every rank's buffer)
//       D  x2 = x + attn; h = RMSNorm(x2); gate/up row pairs -> SwiGLU
//       E  down rows -> reduced like C
//     then the final norm, this rank's vocabulary rows of the LM head and a
//     greedy argmax merged over the CTAs (atomicMax on a packed key) and over
//     the ranks (one record per rank, exchanged with the last flag barrier).
// A GEMV step: every consumer thread owns 8-column groups of the K dimension,
// multiplies the ring's rows by the activation rows held in shared memory,
// and a 32-value butterfly reduces (row, batch) partial sums across lanes.
// Phases are separated by grid barriers (a counter / generation pair in global
// memory; the kernel is launched cooperatively so every CTA is resident);
// tensor-parallel phases C and E end with a flag barrier over the ranks. Every
// wait is bounded: on a timeout the kernel records a status, raises an abort
// word that every other wait polls, drains its own copies in flight and
// returns; the host must then reset the state block before the next launch.
//
// Reference counterpart: the per-token decode loop of QwenSession
// (runtime/src/serving.rs:3389-3418) with one host-launched kernel per op and
// the full logits copied to the host each step.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "decode_common.cuh"
#include "host_utils.h"

namespace aether {
namespace mk {

using bf16 = __nv_bfloat16;

constexpr int kConsumerWarps = 14;
constexpr int kConsumers = kConsumerWarps * 32;  // 448
constexpr int kThreads = kConsumers + 32;        // + producer warp
constexpr int kStages = 3;
constexpr int kSlot = 56 * 1024;   // one ring stage: whole weight rows
constexpr int kUnion = 40 * 1024;  // activation rows [B][K] bf16, or attention staging
constexpr int kKeys = 32;          // keys per attention chunk (one per lane in the softmax)
constexpr int kMaxG = 8;           // query heads per KV head
constexpr int kMaxB = 4;
constexpr int kPartStride = 2 + 128;  // attention partial: m, l, o[128]
constexpr int kSmem = kStages * kSlot + kUnion + 2 * kConsumerWarps * 32 * 4 + 1024;

enum Kind : int { ROWS = 0, HEADPAIR = 1, FFPAIR = 2 };

struct Layer {  // 11 pointers, the host passes an int64 [L, 11] table
  const bf16 *wqkv, *bqkv, *wo, *wgu, *wd, *attn_norm, *mlp_norm;
  bf16 *kc, *vc;
  const float *cos, *sin;
};

struct State {  // zeroed once; `count` only grows (every launch continues from gbase)
  unsigned count, gbase, xepoch, abort;
  unsigned pad[4];
  unsigned long long cand[kMaxB];
};

struct Params {
  const Layer* layers;
  int L;
  const bf16* embed;
  const bf16* final_norm;
  const bf16* head;
  int vocab_rows, vocab_col0;
  int d, hq, hkv, f;
  float eps, scale_log2;
  const int64_t* tok;
  const int* pos;
  const int* slot;
  const int* seqlen;
  int64_t* next;
  float* logits;
  int64_t ld_logits;
  int64_t slot_stride, pos_stride;
  dec::PageMap pm;
  bf16 *x, *x2, *q, *o, *act;  // scratch rows
  float* part;                 // attention partials
  int* pair_ctr;               // [B * hkv], return to zero
  float* red[2];               // this rank's reduction rows [kMaxB][d]
  float* red_mc[2];            // their multicast addresses (world > 1)
  uint32_t* flags;             // this rank's flag words [8]
  uint64_t peer_flags[8];
  unsigned long long* keys;  // this rank's argmax records [8][kMaxB]
  uint64_t peer_keys[8];
  int rank, world;
  State* st;
  int* status;
  uint64_t timeout_ns;
  unsigned long long* trace;  // optional: CTA 0's globaltimer at each phase boundary
  int debug;                  // bit 0: no L2 prefetch; bit 1: fence before the barrier arrival
};

struct Phase {
  const bf16* W;
  int K, U, kind, off;
};

// ---------------------------------------------------------------- small helpers
__device__ __forceinline__ void consumer_bar() { asm volatile("bar.sync 1, 448;" ::: "memory"); }

__device__ __forceinline__ uint4 ldcg16(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ float ldcg_f(const float* p) {
  float v;
  asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ float2 ldcg_f2(const float* p) {
  float2 v;
  asm volatile("ld.global.cg.v2.f32 {%0,%1}, [%2];" : "=f"(v.x), "=f"(v.y) : "l"(p));
  return v;
}
__device__ __forceinline__ unsigned long long ldcg_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.global.cg.u64 %0, [%1];" : "=l"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(unsigned* p, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void mc_red_add(float* mc, float v) {
  asm volatile("multimem.red.relaxed.sys.global.add.f32 [%0], %1;" ::"l"(mc), "f"(v) : "memory");
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void split_range(int U, int n, int c, int& u0, int& u1) {
  u0 = (int)((int64_t)U * c / n);
  u1 = (int)((int64_t)U * (c + 1) / n);
}
__device__ __forceinline__ int rows_per_unit(const Phase& ph) { return ph.kind == ROWS ? 1 : 2; }
// A CTA's share of a phase is cut into row groups of at most group_rows(B)
// rows (one accumulator per (row, batch row) in each thread) that fit one ring
// stage; each group is streamed whole (one contiguous bulk copy per row block)
// and reduced once.
// rows per group: 32 accumulators per thread at B = 2 / 4; 16 at B = 1 (32
// guarded rows there cost registers the GEMV loop needs)
__host__ __device__ constexpr int group_rows(int B) { return B == 1 ? 16 : 32 / B; }
__device__ __forceinline__ int stage_units(const Phase& ph);
__device__ __forceinline__ int group_units(const Phase& ph, int B) {
  return max(1, min(stage_units(ph), group_rows(B) / rows_per_unit(ph)));
}
__device__ __forceinline__ int group_len(const Phase& ph, int u, int u1, int upg) {
  int n = min(u1 - u, upg);
  if (ph.kind == HEADPAIR) n = min(n, 64 - (u & 63));
  return n;
}
// units of a group that one ring stage holds (whole rows: one contiguous bulk
// copy per row block)
__device__ __forceinline__ int stage_units(const Phase& ph) {
  return max(1, kSlot / (ph.K * 2 * rows_per_unit(ph)));
}
// first weight row of unit u's first (and, for pairs, second) row block
__device__ __forceinline__ int first_row(const Phase& ph, int u) {
  return ph.kind == HEADPAIR ? (u >> 6) * 128 + (u & 63) : u;
}
__device__ __forceinline__ int second_row_off(const Phase& ph) { return ph.kind == HEADPAIR ? 64 : ph.off; }
// weight row of row r of a group of n units starting at unit u
__device__ __forceinline__ int weight_row(const Phase& ph, int u, int n, int r) {
  return r < n ? first_row(ph, u) + r : first_row(ph, u) + second_row_off(ph) + (r - n);
}

__device__ __forceinline__ void unpack8f(const uint4& u, float (&v)[8]) { dec::unpack8(u, v); }

__device__ __forceinline__ void trace_at(const Params& p, int k) {
  if (p.trace != nullptr && blockIdx.x == 0 && threadIdx.x == 0) p.trace[k] = globaltimer_ns();
}
// event log of one layer (CTA 0, thread 0): trace[256 + 2n] = code, [257 + 2n] = time
__device__ __forceinline__ void ev(const Params& p, int* misc, int code) {
  if (p.trace != nullptr && blockIdx.x == 0 && threadIdx.x == 0 && misc[6] == 10 && misc[5] < 1000) {
    const int n = misc[5]++;
    p.trace[256 + 2 * n] = code | ((unsigned long long)clock64() << 8);
    p.trace[257 + 2 * n] = globaltimer_ns();
  }
}

// float -> key ordered like the float, with the lower index winning ties
__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
  unsigned u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned)idx);
}

// ---------------------------------------------------------------- shared state
struct Smem {
  uint8_t* ring;
  uint8_t* uni;
  float* red;  // [2][14][32]
  uint64_t* full;
  uint64_t* empty;
  float* wsum;  // [14][kMaxB]
  float* rstd;  // [kMaxB]
  int* misc;    // [0] grid barrier ok, [1] last-arriver flag, [2] issued chunks, [3] consumed chunks,
                // [4] flag barrier ok, [5] / [6] event log, [7] first chunk whose wait gave up,
                // [8] grid barrier target (thread 0)
  int* rows;    // tok / pos / slot / seqlen per batch row: [4][kMaxB]
  int* fail;    // a consumer's ring wait gave up (read by all after a barrier)
  uint64_t* empty_cur;  // the stage being consumed (per thread, set before the GEMV)
};

__device__ __forceinline__ void raise_abort(const Params& p, int code) {
  atomicExch(reinterpret_cast<unsigned*>(&p.st->abort), 1u);
  atomicExch(p.status, code);
}

// All consumer threads of all CTAs; false if the barrier gave up. The arrival
// counter only grows: each CTA adds 1 with a release reduction and waits
// (acquire, bounded) until it reaches this barrier's target -- no reset and no
// returned atomic on the critical path.
__device__ bool grid_sync(const Params& p, const Smem& s) {
  consumer_bar();
  if (threadIdx.x == 0) {
    int ok = 1;
    const unsigned target = (unsigned)s.misc[8] + gridDim.x;
    s.misc[8] = (int)target;
    if (p.debug & 2) __threadfence();
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(&p.st->count) : "memory");
    const uint64_t t0 = globaltimer_ns();
    for (unsigned it = 1;; ++it) {
      if ((int)(ld_acquire_gpu(&p.st->count) - target) >= 0) break;
      if ((it & 63u) == 0u) {
        if (*reinterpret_cast<volatile unsigned*>(&p.st->abort) || globaltimer_ns() - t0 > p.timeout_ns) {
          ok = 0;
          raise_abort(p, kStatusTimeoutEpilogue);
          break;
        }
      }
    }
    s.misc[0] = ok;
  }
  consumer_bar();
  return s.misc[0] != 0;
}

// Flag barrier over the ranks (no grid barrier): CTA 0 releases epoch ++xep
// to every rank's flag word of this rank after a system fence; then every
// calling CTA waits (bounded) until all ranks have reached it.
__device__ bool flag_exchange(const Params& p, const Smem& s, unsigned& xep) {
  ++xep;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    asm volatile("fence.sc.sys;" ::: "memory");
    for (int q = 0; q < p.world; ++q) st_release_sys_u32(reinterpret_cast<uint32_t*>(p.peer_flags[q]) + p.rank, xep);
  }
  int ok = 1;
  if (threadIdx.x < (unsigned)p.world) {
    const uint64_t t0 = globaltimer_ns();
    for (unsigned it = 1;; ++it) {
      if ((int)(ld_acquire_sys_u32(p.flags + threadIdx.x) - xep) >= 0) break;
      if ((it & 63u) == 0u) {
        if (*reinterpret_cast<volatile unsigned*>(&p.st->abort)) {
          ok = 0;
          break;
        }
        if (globaltimer_ns() - t0 > p.timeout_ns) {
          ok = 0;
          raise_abort(p, kStatusTimeoutPeer);
          break;
        }
      }
    }
  }
  if (threadIdx.x == 0) s.misc[4] = 1;  // a word of its own: misc[0] may still be read after grid_sync
  consumer_bar();
  if (!ok) s.misc[4] = 0;
  consumer_bar();
  return s.misc[4] != 0;
}

// Grid barrier, then (world > 1) the flag barrier over the ranks.
__device__ bool cross_sync(const Params& p, const Smem& s, unsigned& xep) {
  if (!grid_sync(p, s)) return false;
  if (p.world == 1) return true;
  return flag_exchange(p, s, xep);
}

// ---------------------------------------------------------------- producer
// The producer walks this CTA's groups of every phase of every layer, then the
// head, in consumption order (a cursor over layer / phase / unit). A second
// cursor runs kPrefetch bytes ahead and pulls those rows into L2
// (cp.async.bulk.prefetch), so the ring refills from L2 even right after a
// phase barrier, when the ring itself has been full for a while.
constexpr int kPrefetch = 256 * 1024;

struct Cursor {
  int layer, ph, u, u1;
};
struct Block {
  const bf16* src;
  int64_t off2;  // element offset of the second row block (pairs), else 0
  uint32_t bytes;
  int rpu;
};

__device__ __forceinline__ Phase phase_of(const Params& p, int layer, int ph) {
  if (ph == 4) return Phase{p.head, p.d, p.vocab_rows, ROWS, 0};
  const Layer& ly = p.layers[layer];
  if (ph == 0) return Phase{ly.wqkv, p.d, (p.hq + 2 * p.hkv) * 64, HEADPAIR, 0};
  if (ph == 1) return Phase{ly.wo, p.hq * 128, p.d, ROWS, 0};
  if (ph == 2) return Phase{ly.wgu, p.d, p.f, FFPAIR, p.f};
  return Phase{ly.wd, p.f, p.d, ROWS, 0};
}

template <int B>
__device__ bool cursor_next(const Params& p, Cursor& c, Block& out) {
  for (;;) {
    if (c.ph > 4) return false;
    if (c.layer >= p.L) c.ph = 4;  // no (more) layers: the head
    const Phase ph = phase_of(p, c.layer, c.ph);
    if (c.u < 0) split_range(ph.U, gridDim.x, blockIdx.x, c.u, c.u1);
    if (c.u < c.u1) {
      const int n = group_len(ph, c.u, c.u1, group_units(ph, B));
      out.src = ph.W + (int64_t)first_row(ph, c.u) * ph.K;
      out.rpu = rows_per_unit(ph);
      out.off2 = out.rpu == 2 ? (int64_t)second_row_off(ph) * ph.K : 0;
      out.bytes = (uint32_t)n * ph.K * 2;
      c.u += n;
      return true;
    }
    c.u = -1;
    if (c.ph == 4) {
      c.ph = 5;
    } else if (++c.ph == 4) {
      c.ph = 0;
      if (++c.layer >= p.L) c.ph = 4;
    }
  }
}

__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

template <int B>
__device__ void attn_prefetch(const Smem& s, const Params& p, int layer);

template <int B>
__device__ void producer(const Smem& s, const Params& p) {
  Cursor ld{0, 0, -1, 0}, pf{0, 0, -1, 0};
  int64_t ld_bytes = 0, pf_bytes = 0;
  bool pf_more = true;
  Block b{}, q{};
  int it = 0, layer_seen = -1;
  while (cursor_next<B>(p, ld, b)) {
    if (ld.layer < p.L && ld.layer != layer_seen) {  // a new layer: its attention K / V into L2
      layer_seen = ld.layer;
      attn_prefetch<B>(s, p, layer_seen);
    }
    while (pf_more && !(p.debug & 1) && pf_bytes < ld_bytes + kPrefetch) {
      pf_more = cursor_next<B>(p, pf, q);
      if (pf_more) {
        prefetch_l2(q.src, q.bytes);
        if (q.rpu == 2) prefetch_l2(q.src + q.off2, q.bytes);
        pf_bytes += (int64_t)q.bytes * q.rpu;
      }
    }
    const int st = it % kStages;
    const uint32_t par = (uint32_t)(it / kStages) & 1u;
    if (!mbar_wait(&s.empty[st], par ^ 1u, reinterpret_cast<volatile int*>(&p.st->abort))) {
      raise_abort(p, kStatusTimeoutProducer);
      return;
    }
    mbar_arrive_expect_tx(&s.full[st], b.bytes * b.rpu);
    uint8_t* dst = s.ring + st * kSlot;
    bulk_g2s(dst, b.src, b.bytes, &s.full[st]);
    if (b.rpu == 2) bulk_g2s(dst + b.bytes, b.src + b.off2, b.bytes, &s.full[st]);
    ld_bytes += (int64_t)b.bytes * b.rpu;
    ++it;
    *reinterpret_cast<volatile int*>(&s.misc[2]) = it;
  }
}

// ---------------------------------------------------------------- consumer GEMV
// One row group (n units: n rows, or n row pairs) of a phase: its rows arrive
// through the ring in whole-row stages; activations [B][K] bf16 are in
// s.uni. Thread t takes the 8-column groups t, t + 448, ... of every row and
// accumulates (row, batch) partial sums in registers across the stages.
// Returns, in lane L of warp 0, the sum for index L = row * B + b; false (in
// every thread) on abort.
template <int B, int RP>
__device__ __forceinline__ void stage_fma(const uint4* ws, const uint4* xs, int K8, int rows, float (&acc)[32]) {
  for (int g = threadIdx.x; g < K8; g += kConsumers) {
    float xf[B][8];
#pragma unroll
    for (int b = 0; b < B; ++b) unpack8f(xs[b * K8 + g], xf[b]);
#pragma unroll
    for (int r = 0; r < RP; ++r) {
      // rows past the group's last repeat it (straight-line code: the
      // padding sums are computed and never read)
      const int rr = r < rows ? r : rows - 1;
      float wf[8];
      unpack8f(ws[rr * K8 + g], wf);
#pragma unroll
      for (int b = 0; b < B; ++b) {
        float a = acc[r * B + b];
#pragma unroll
        for (int e = 0; e < 8; ++e) a = fmaf(wf[e], xf[b][e], a);
        acc[r * B + b] = a;
      }
    }
  }
}

// NV values per lane summed over the warp: after log2(NV) halving steps and
// plain steps for the remaining lane bits, lane L holds the total of value
// index L >> (5 - log2 NV).
template <int NV>
__device__ __forceinline__ float warp_reduce_n(float (&v)[32], int lane) {
  int cnt = NV;
#pragma unroll
  for (int sft = 16; sft >= 1; sft >>= 1) {
    if (cnt > 1) {
      const int h = cnt / 2;
      const bool up = (lane & sft) != 0;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        if (i < h) {
          const float send = up ? v[i] : v[i + h];
          const float keep = up ? v[i + h] : v[i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, sft);
        }
      }
      cnt = h;
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], sft);
    }
  }
  return v[0];
}

template <int NV>
__device__ __forceinline__ constexpr int log2c() {
  return NV <= 1 ? 0 : NV == 2 ? 1 : NV == 4 ? 2 : NV == 8 ? 3 : NV == 16 ? 4 : 5;
}

template <int B, int RP>
__device__ __forceinline__ void stage_reduce(const Smem& s, const uint4* ws, const uint4* xs, int K8, int rows,
                                             int rbuf, float& out) {
  constexpr int NV = RP * B;
  constexpr int SH = 5 - log2c<NV>();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float acc[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) acc[i] = 0.f;
  stage_fma<B, RP>(ws, xs, K8, rows, acc);
  __syncwarp();
  if (lane == 0) mbar_arrive(s.empty_cur);
  const float v = warp_reduce_n<NV>(acc, lane);
  float* red = s.red + rbuf * kConsumerWarps * 32;
  red[warp * 32 + lane] = v;
  consumer_bar();
  if (warp == 0) {
    float t = 0.f;
    if (lane < NV) {
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) t += red[w * 32 + (lane << SH)];
    }
    out = t;
  }
}

// One row group (n units: n rows, or n row pairs stored as [first rows |
// second rows]) of a phase, in one ring stage; activations [B][K] bf16 in
// s.uni. Thread t takes the 8-column groups t, t + 448, ... of every row; the
// row count is rounded up to a power of two so the loop is straight-line code.
// Returns, in lane L of warp 0, the sum for index L = row * B + b; false (in
// every thread) on abort.
template <int B>
__device__ bool gemv_group(Smem& s, int& it, const Phase& ph, int n, int& rbuf, float& out, const Params& p) {
  const int K8 = ph.K >> 3, rows = n * rows_per_unit(ph);
  const int st = it % kStages;
  const uint32_t par = (uint32_t)(it / kStages) & 1u;
  // A wait that gives up is recorded, not returned on: every consumer thread
  // must still reach the group's named barrier, after which all of them read
  // the flag and leave together (the slot's contents are then unused).
  ev(p, s.misc, 11);
  if (!mbar_wait(&s.full[st], par, reinterpret_cast<volatile int*>(&p.st->abort))) {
    *reinterpret_cast<volatile int*>(s.fail) = 1;
    atomicMin(&s.misc[7], it);
    raise_abort(p, kStatusTimeoutMma);
  }
  ev(p, s.misc, 2);
  const uint4* ws = reinterpret_cast<const uint4*>(s.ring + st * kSlot);
  const uint4* xs = reinterpret_cast<const uint4*>(s.uni);
  s.empty_cur = &s.empty[st];
  constexpr int RB = group_rows(B);
  if (rows <= 1) stage_reduce<B, 1>(s, ws, xs, K8, rows, rbuf, out);
  else if (rows <= 2) stage_reduce<B, 2>(s, ws, xs, K8, rows, rbuf, out);
  else if (rows <= 4) stage_reduce<B, 4>(s, ws, xs, K8, rows, rbuf, out);
  else if (RB >= 8 && rows <= 8) stage_reduce<B, (RB >= 8 ? 8 : 4)>(s, ws, xs, K8, rows, rbuf, out);
  else stage_reduce<B, RB>(s, ws, xs, K8, rows, rbuf, out);
  ++it;
  if (*reinterpret_cast<volatile int*>(s.fail)) return false;
  ev(p, s.misc, 3);
  rbuf ^= 1;
  return true;
}

// ---------------------------------------------------------------- prologues
// x = bf16(a + red) (red optional); store x (CTA 0, when xout); uni = bf16(rmsnorm(x) * w)
template <int B>
__device__ void norm_rows(const Smem& s, const Params& p, const bf16* const (&a)[kMaxB], const float* red,
                          const bf16* w, bf16* xout) {
  const int d = p.d, d8 = d >> 3, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  bf16* xs = reinterpret_cast<bf16*>(s.uni);
  float ss[B];
#pragma unroll
  for (int b = 0; b < B; ++b) ss[b] = 0.f;
  for (int g = tid; g < d8; g += kConsumers) {
#pragma unroll
    for (int b = 0; b < B; ++b) {
      float v[8];
      unpack8f(ldcg16(a[b] + 8 * g), v);
      if (red != nullptr) {
        const float* rr = red + (int64_t)b * d + 8 * g;
        const uint4 r0 = ldcg16(rr), r1 = ldcg16(rr + 4);
        v[0] += __uint_as_float(r0.x); v[1] += __uint_as_float(r0.y);
        v[2] += __uint_as_float(r0.z); v[3] += __uint_as_float(r0.w);
        v[4] += __uint_as_float(r1.x); v[5] += __uint_as_float(r1.y);
        v[6] += __uint_as_float(r1.z); v[7] += __uint_as_float(r1.w);
      }
      const uint4 xb = dec::pack8(v);
      float vr[8];
      unpack8f(xb, vr);  // statistics of the rounded residual, as stored
#pragma unroll
      for (int e = 0; e < 8; ++e) ss[b] += vr[e] * vr[e];
      reinterpret_cast<uint4*>(xs)[b * d8 + g] = xb;
      if (xout != nullptr && blockIdx.x == 0) reinterpret_cast<uint4*>(xout + (int64_t)b * d)[g] = xb;
    }
  }
#pragma unroll
  for (int b = 0; b < B; ++b) {
    const float t = warp_sum(ss[b]);
    if (lane == 0) s.wsum[warp * kMaxB + b] = t;
  }
  consumer_bar();
  if (tid < B) {
    float t = 0.f;
    for (int w2 = 0; w2 < kConsumerWarps; ++w2) t += s.wsum[w2 * kMaxB + tid];
    s.rstd[tid] = rsqrtf(t / d + p.eps);
  }
  consumer_bar();
  for (int g = tid; g < d8; g += kConsumers) {
    float wv[8];
    unpack8f(*reinterpret_cast<const uint4*>(w + 8 * g), wv);
#pragma unroll
    for (int b = 0; b < B; ++b) {
      float v[8];
      unpack8f(reinterpret_cast<uint4*>(xs)[b * d8 + g], v);
      const float r = s.rstd[b];
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = v[e] * r * wv[e];
      reinterpret_cast<uint4*>(xs)[b * d8 + g] = dec::pack8(v);
    }
  }
  consumer_bar();
}

template <int B>
__device__ void copy_rows(const Smem& s, const bf16* src, int K) {
  const int K8 = K >> 3;
  uint4* xs = reinterpret_cast<uint4*>(s.uni);
  for (int i = threadIdx.x; i < B * K8; i += kConsumers) {
    const int b = i / K8, g = i - b * K8;
    xs[i] = ldcg16(src + (int64_t)b * K + 8 * g);
  }
  consumer_bar();
}

// zero this CTA's column slice of a reduction buffer (world > 1)
template <int B>
__device__ void zero_slice(const Params& p, float* buf) {
  int c0, c1;
  split_range(p.d, gridDim.x, blockIdx.x, c0, c1);
  const int n = c1 - c0;
  for (int i = threadIdx.x; i < B * n; i += kConsumers) buf[(int64_t)(i / n) * p.d + c0 + i % n] = 0.f;
}

// ---------------------------------------------------------------- attention
// Split-K decode attention. Each (row, KV head) pair gets S = CTAs / pairs
// CTAs (or, with more pairs than CTAs, a CTA takes whole pairs), each a
// contiguous range of 32-key chunks; the next chunk's K / V are loaded into
// registers while the current one is scored, then stored to the other half of
// a double buffer. Every working CTA writes one partial (running max m, sum l
// and unnormalised o for each of its G query heads); the o_proj prologue
// merges them (merge_attention), so no CTA waits on another here.
struct AttnSplit {
  int S;     // CTAs per pair (1 when pairs >= CTAs)
  bool many;
};
template <int B>
__device__ __forceinline__ AttnSplit attn_split(const Params& p) {
  const int P = B * p.hkv, nb = gridDim.x;
  AttnSplit a;
  a.many = P >= nb;
  a.S = a.many ? 1 : nb / P;
  return a;
}
__device__ __forceinline__ int attn_used(int S, int n) {  // splits that get keys: >= 2 chunks each
  return max(1, min(S, (n + 2 * kKeys - 1) / (2 * kKeys)));
}

// Producer side: pull this CTA's K / V chunks of layer `layer`'s attention
// into L2 while the QKV phase runs (the row that phase appends is re-read
// from L2 anyway). Only where a KV head's keys are contiguous (one KV head
// per rank); runs split at page boundaries.
template <int B>
__device__ void attn_prefetch(const Smem& s, const Params& p, int layer) {
  if (p.hkv != 1) return;
  const Layer& ly = p.layers[layer];
  const AttnSplit as = attn_split<B>(p);
  const int P = B * p.hkv, nb = gridDim.x;
  int pi = as.many ? (int)blockIdx.x : (int)blockIdx.x / as.S;
  const int sidx = as.many ? 0 : (int)blockIdx.x % as.S;
  const int run = p.pm.table != nullptr ? (1 << p.pm.shift) : 1 << 30;
  for (; pi < P; pi += as.many ? nb : P) {
    const int b = pi / p.hkv;
    const int n = s.rows[3 * kMaxB + b], seq = s.rows[2 * kMaxB + b];
    const int nch = (n + kKeys - 1) / kKeys, Su = attn_used(as.S, n);
    if (sidx < Su) {
      const int t1 = min(n, (sidx + 1) * nch / Su * kKeys);
      for (int t = sidx * nch / Su * kKeys; t < t1;) {
        const int len = min(t1 - t, run - (t & (run - 1)));
        const int64_t off = dec::kv_offset(p.pm, seq, t, p.slot_stride, p.pos_stride);
        prefetch_l2(ly.kc + off, (uint32_t)len * 256);
        prefetch_l2(ly.vc + off, (uint32_t)len * 256);
        t += len;
      }
    }
    if (!as.many) break;
  }
}

template <int B>
__device__ bool attention_phase(const Smem& s, const Params& p, const Layer& ly) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = p.hq / p.hkv, P = B * p.hkv, nb = gridDim.x;
  bf16* kvbuf = reinterpret_cast<bf16*>(s.uni);  // [2 buffers][K | V][kKeys][128]
  float* sq = reinterpret_cast<float*>(kvbuf + 2 * 2 * kKeys * 128);  // [G][128]
  float* sp = sq + kMaxG * 128;                                      // [G][kKeys]
  float* sm = sp + kMaxG * kKeys;                                    // m [G], l [G], alpha [G]
  const AttnSplit as = attn_split<B>(p);
  int pi = as.many ? (int)blockIdx.x : (int)blockIdx.x / as.S;
  const int sidx = as.many ? 0 : (int)blockIdx.x % as.S;
  constexpr int kPieces = 2 * kKeys * 16, kPer = (kPieces + kConsumers - 1) / kConsumers;
  for (; pi < P; pi += as.many ? nb : P) {
    const int b = pi / p.hkv, kvh = pi % p.hkv;
    const int n = s.rows[3 * kMaxB + b], seq = s.rows[2 * kMaxB + b];
    const int nch = (n + kKeys - 1) / kKeys;
    const int Su = attn_used(as.S, n);
    if (sidx < Su) {
      const int c0 = sidx * nch / Su, c1 = (sidx + 1) * nch / Su;
      uint4 qreg = make_uint4(0u, 0u, 0u, 0u);
      if (tid < G * 16) qreg = ldcg16(p.q + (int64_t)b * p.hq * 128 + (kvh * G + (tid >> 4)) * 128 + 8 * (tid & 15));
      auto load_chunk = [&](int ch, uint4 (&vb)[kPer]) {
        const int t0 = ch * kKeys;
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
          const int i = tid + j * kConsumers;
          vb[j] = make_uint4(0u, 0u, 0u, 0u);
          if (i < kPieces) {
            const int kv = i / (kKeys * 16), rem = i % (kKeys * 16), key = rem >> 4, c = rem & 15;
            const int t = t0 + key;
            if (t < n)
              vb[j] = ldcg16((kv ? ly.vc : ly.kc) + dec::kv_offset(p.pm, seq, t, p.slot_stride, p.pos_stride) +
                             kvh * 128 + 8 * c);
          }
        }
      };
      auto store_chunk = [&](int buf, const uint4 (&vb)[kPer]) {
        uint4* dst = reinterpret_cast<uint4*>(kvbuf + buf * 2 * kKeys * 128);
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
          const int i = tid + j * kConsumers;
          if (i < kPieces) dst[i] = vb[j];  // K pieces then V pieces, [key][16] each
        }
      };
      uint4 vb[kPer];
      load_chunk(c0, vb);
      if (tid < G) {
        sm[tid] = -INFINITY;
        sm[kMaxG + tid] = 0.f;
      }
      if (tid < G * 16) {
        float v[8];
        unpack8f(qreg, v);
#pragma unroll
        for (int e = 0; e < 8; ++e) sq[(tid >> 4) * 128 + 8 * (tid & 15) + e] = v[e] * p.scale_log2;
      }
      store_chunk(0, vb);
      ev(p, s.misc, 5);
      float2 oacc[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      for (int ch = c0; ch < c1; ++ch) {
        const int buf = (ch - c0) & 1, t0 = ch * kKeys;
        if (ch + 1 < c1) load_chunk(ch + 1, vb);  // in flight while this chunk is scored
        consumer_bar();
        const bf16* sK = kvbuf + buf * 2 * kKeys * 128;
        const bf16* sV = sK + kKeys * 128;
        ev(p, s.misc, 6);
        // one thread per (query head, key): a 128-long dot product, 16-B pieces
        // in a key-rotated order (fewer bank conflicts between a warp's keys)
        for (int item = tid; item < G * kKeys; item += kConsumers) {
          const int g = item / kKeys, key = item % kKeys;
          const uint4* kr = reinterpret_cast<const uint4*>(sK + key * 128);
          const float4* qg = reinterpret_cast<const float4*>(sq + g * 128);
          float a0 = 0.f, a1 = 0.f;
#pragma unroll 4
          for (int c = 0; c < 16; ++c) {
            const int cc = (c + key) & 15;
            float kf[8];
            unpack8f(kr[cc], kf);
            const float4 q0 = qg[2 * cc], q1 = qg[2 * cc + 1];
            a0 = fmaf(kf[0], q0.x, a0); a1 = fmaf(kf[1], q0.y, a1);
            a0 = fmaf(kf[2], q0.z, a0); a1 = fmaf(kf[3], q0.w, a1);
            a0 = fmaf(kf[4], q1.x, a0); a1 = fmaf(kf[5], q1.y, a1);
            a0 = fmaf(kf[6], q1.z, a0); a1 = fmaf(kf[7], q1.w, a1);
          }
          sp[g * kKeys + key] = (t0 + key < n) ? a0 + a1 : -INFINITY;
        }
        consumer_bar();
        ev(p, s.misc, 7);
        if (warp < G) {  // kKeys == 32: one score per lane
          const int g = warp;
          const float sc = sp[g * kKeys + lane];
          const float cm = warp_max(sc);
          const float mo = sm[g], mn = fmaxf(mo, cm);
          const float pr = exp2f(sc - mn);
          sp[g * kKeys + lane] = pr;
          const float ls = warp_sum(pr);
          if (lane == 0) {
            const float al = exp2f(mo - mn);
            sm[2 * kMaxG + g] = al;
            sm[kMaxG + g] = sm[kMaxG + g] * al + ls;
            sm[g] = mn;
          }
        }
        consumer_bar();
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const int item = tid + k * kConsumers;
          if (item < G * 64) {
            const int g = item >> 6, d2 = item & 63;
            const float al = sm[2 * kMaxG + g];
            float ox = oacc[k].x * al, oy = oacc[k].y * al;
            const float* pg = sp + g * kKeys;
            const uint32_t* vcol = reinterpret_cast<const uint32_t*>(sV) + d2;
#pragma unroll 8
            for (int key = 0; key < kKeys; ++key) {
              const uint32_t vv = vcol[key * 64];
              const float pk = pg[key];
              ox = fmaf(pk, bf16lo(vv), ox);
              oy = fmaf(pk, bf16hi(vv), oy);
            }
            oacc[k] = make_float2(ox, oy);
          }
        }
        if (ch + 1 < c1) store_chunk(buf ^ 1, vb);  // the other buffer: last read two chunks ago
      }
      consumer_bar();
      ev(p, s.misc, 9);
      float* part = p.part + ((int64_t)pi * nb + sidx) * G * kPartStride;
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int item = tid + k * kConsumers;
        if (item < G * 64) reinterpret_cast<float2*>(part + (item >> 6) * kPartStride + 2)[item & 63] = oacc[k];
      }
      if (tid < G) {
        part[tid * kPartStride] = sm[tid];
        part[tid * kPartStride + 1] = sm[kMaxG + tid];
      }
      consumer_bar();  // the shared buffers of this pair are free for the next one
    }
    if (!as.many) break;
  }
  return true;
}

// o_proj prologue: the activation rows are the attention output, merged here
// from the partials by log-sum-exp (every CTA merges all of them -- a few
// hundred KB from L2 at most -- instead of one CTA merging while the others
// wait). T threads share each (pair, head, 4-dim chunk) item: each loads the
// m, l and o of every T-th split in one round of loads (up to 12 splits in
// flight), folds them relative to its own running max, and the T results are
// combined through shared memory. Writes bf16 o [B][hq * 128] into s.uni.
template <int B>
__device__ void merge_attention(const Smem& s, const Params& p) {
  const int tid = threadIdx.x;
  const int G = p.hq / p.hkv, P = B * p.hkv, nb = gridDim.x;
  const AttnSplit as = attn_split<B>(p);
  const int items = P * G * 32;
  const int T = max(1, kConsumers / items);
  bf16* xs = reinterpret_cast<bf16*>(s.uni);
  // [T][items] (acc, then M and L) right after the bf16 rows (B * hq * 768
  // bytes in all, checked by the host against the 40 KB area)
  float4* pacc = reinterpret_cast<float4*>(s.uni + B * p.hq * 256);
  float2* pml = reinterpret_cast<float2*>(pacc + T * items);
  for (int w0 = tid; w0 < items * T; w0 += kConsumers) {
    const int item = w0 % items, j0 = w0 / items;
    const int d4 = item & 31, pg = item >> 5, pi = pg / G, g = pg % G;
    const int Su = attn_used(as.S, s.rows[3 * kMaxB + pi / p.hkv]);
    const float* p0 = p.part + (int64_t)pi * nb * G * kPartStride + g * kPartStride;
    float M = -INFINITY, L = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int sb = j0; sb < Su; sb += 12 * T) {
      float2 ml[12];
      float4 v[12];
#pragma unroll
      for (int j = 0; j < 12; ++j) {
        const int sp2 = sb + j * T;
        ml[j] = make_float2(-INFINITY, 0.f);
        v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (sp2 < Su) {
          const float* pe = p0 + (int64_t)sp2 * G * kPartStride;
          ml[j] = ldcg_f2(pe);
          const float2 a = ldcg_f2(pe + 2 + 4 * d4), c = ldcg_f2(pe + 4 + 4 * d4);
          v[j] = make_float4(a.x, a.y, c.x, c.y);
        }
      }
      float bm = M;
#pragma unroll
      for (int j = 0; j < 12; ++j) bm = fmaxf(bm, ml[j].x);
      const float sc = exp2f(M - bm);  // 0 on the first batch (M = -inf)
      acc.x *= sc; acc.y *= sc; acc.z *= sc; acc.w *= sc;
      L *= sc;
      M = bm;
#pragma unroll
      for (int j = 0; j < 12; ++j) {
        const float w = exp2f(ml[j].x - M);  // 0 for missing splits
        L = fmaf(w, ml[j].y, L);
        acc.x = fmaf(w, v[j].x, acc.x);
        acc.y = fmaf(w, v[j].y, acc.y);
        acc.z = fmaf(w, v[j].z, acc.z);
        acc.w = fmaf(w, v[j].w, acc.w);
      }
    }
    pacc[j0 * items + item] = acc;
    pml[j0 * items + item] = make_float2(M, L);
  }
  consumer_bar();
  for (int item = tid; item < items; item += kConsumers) {
    float M = -INFINITY;
    for (int j = 0; j < T; ++j) M = fmaxf(M, pml[j * items + item].x);
    float L = 0.f;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < T; ++j) {
      const float2 ml = pml[j * items + item];
      const float w = ml.x == -INFINITY ? 0.f : exp2f(ml.x - M);
      const float4 c = pacc[j * items + item];
      L = fmaf(w, ml.y, L);
      a.x = fmaf(w, c.x, a.x); a.y = fmaf(w, c.y, a.y); a.z = fmaf(w, c.z, a.z); a.w = fmaf(w, c.w, a.w);
    }
    const int d4 = item & 31, pg = item >> 5, pi = pg / G, g = pg % G;
    const int b = pi / p.hkv, kvh = pi % p.hkv;
    const float iL = 1.f / L;
    uint2 o;
    o.x = pack_bf16(a.x * iL, a.y * iL);
    o.y = pack_bf16(a.z * iL, a.w * iL);
    reinterpret_cast<uint2*>(xs + (int64_t)b * p.hq * 128 + (kvh * G + g) * 128)[d4] = o;
  }
  consumer_bar();
}

// ---------------------------------------------------------------- the kernel
template <int B>
__global__ void __launch_bounds__(kThreads, 1) decode_mega_kernel(Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Smem s;
  s.empty_cur = nullptr;
  s.ring = smem_raw;
  s.uni = s.ring + kStages * kSlot;
  s.red = reinterpret_cast<float*>(s.uni + kUnion);
  uint8_t* tail = reinterpret_cast<uint8_t*>(s.red + 2 * kConsumerWarps * 32);
  s.full = reinterpret_cast<uint64_t*>(tail);
  s.empty = s.full + kStages;
  s.wsum = reinterpret_cast<float*>(s.empty + kStages);
  s.rstd = s.wsum + kConsumerWarps * kMaxB;
  s.misc = reinterpret_cast<int*>(s.rstd + kMaxB);
  s.rows = s.misc + 12;
  s.fail = s.rows + 4 * kMaxB;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], kConsumerWarps);
    }
    fence_mbar_init();
    s.misc[2] = 0;
    s.misc[3] = 0;
    s.misc[5] = 0;
    s.misc[6] = -1;
    s.misc[7] = 0x7fffffff;
    s.misc[8] = (int)p.st->gbase;
    *s.fail = 0;
  }
  if (tid < B) {
    s.rows[tid] = (int)p.tok[tid];
    s.rows[kMaxB + tid] = p.pos[tid];
    s.rows[2 * kMaxB + tid] = p.slot[tid];
    s.rows[3 * kMaxB + tid] = p.seqlen[tid];
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) producer<B>(s, p);
  } else {
    // ------------------------------------------------------------ consumers
    unsigned xep = p.st->xepoch;
    int it = 0, rbuf = 0;
    bool ok = true;
    const bf16* rows_a[kMaxB];
    // per-lane role in a chunk epilogue: value index lane = r * B + b
    const int eb = lane % B, er = lane / B;
    unsigned long long best = 0ull;
    trace_at(p, 0);
    for (int i = 0; i < p.L && ok; ++i) {
      const Layer& ly = p.layers[i];
      Phase ph[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) ph[k] = phase_of(p, i, k);
      if (tid == 0) s.misc[6] = i;
      ev(p, s.misc, 0);
      // ---- A: h = RMSNorm(x); qkv + bias + RoPE; q out, k / v into the cache
      for (int b = 0; b < B; ++b)
        rows_a[b] = i == 0 ? p.embed + (int64_t)s.rows[b] * p.d : p.x2 + (int64_t)b * p.d;
      norm_rows<B>(s, p, rows_a, i == 0 ? nullptr : p.red[1], ly.attn_norm, p.x);
      ev(p, s.misc, 1);
      {
        const Phase& P0 = ph[0];
        int u0, u1;
        split_range(P0.U, gridDim.x, blockIdx.x, u0, u1);
        const int upg = group_units(P0, B);
        for (int u = u0; u < u1 && ok;) {
          const int n = group_len(P0, u, u1, upg);
          float v = 0.f;
          if (!gemv_group<B>(s, it, P0, n, rbuf, v, p)) {
            ok = false;
            break;
          }
          if (warp == 0) {
            const float v2 = __shfl_sync(0xffffffffu, v, min(lane + n * B, 31));
            if (er < n) {
              const int hh = u >> 6, j = (u & 63) + er;
              float a = v, c = v2;
              if (ly.bqkv != nullptr) {
                a += __bfloat162float(ly.bqkv[hh * 128 + j]);
                c += __bfloat162float(ly.bqkv[hh * 128 + 64 + j]);
              }
              a = __bfloat162float(__float2bfloat16(a));
              c = __bfloat162float(__float2bfloat16(c));
              const int ps = s.rows[kMaxB + eb];
              if (hh < p.hq + p.hkv) {
                const float cs = ly.cos[(int64_t)ps * 64 + j], sn = ly.sin[(int64_t)ps * 64 + j];
                const float a2 = a * cs - c * sn, c2 = c * cs + a * sn;
                a = a2;
                c = c2;
              }
              if (hh < p.hq) {
                bf16* qr = p.q + (int64_t)eb * p.hq * 128 + hh * 128;
                qr[j] = __float2bfloat16(a);
                qr[j + 64] = __float2bfloat16(c);
              } else {
                const bool isk = hh < p.hq + p.hkv;
                const int kvh = isk ? hh - p.hq : hh - p.hq - p.hkv;
                bf16* cache = (isk ? ly.kc : ly.vc) +
                              dec::kv_offset(p.pm, s.rows[2 * kMaxB + eb], ps, p.slot_stride, p.pos_stride) +
                              kvh * 128;
                cache[j] = __float2bfloat16(a);
                cache[j + 64] = __float2bfloat16(c);
              }
            }
          }
          u += n;
        }
      }
      if (!ok || !grid_sync(p, s)) break;
      trace_at(p, 1 + 5 * i);
      ev(p, s.misc, 4);
      // ---- B: attention (and the reduction buffer read in A is re-zeroed)
      if (p.world > 1) zero_slice<B>(p, p.red[1]);
      attention_phase<B>(s, p, ly);
      if (!grid_sync(p, s)) break;
      trace_at(p, 2 + 5 * i);
      ev(p, s.misc, 4);
      // ---- C: o_proj, reduced over the ranks
      merge_attention<B>(s, p);
      ev(p, s.misc, 1);
      {
        const Phase& P1 = ph[1];
        int u0, u1;
        split_range(P1.U, gridDim.x, blockIdx.x, u0, u1);
        const int upg = group_units(P1, B);
        for (int u = u0; u < u1 && ok;) {
          const int n = group_len(P1, u, u1, upg);
          float v = 0.f;
          if (!gemv_group<B>(s, it, P1, n, rbuf, v, p)) {
            ok = false;
            break;
          }
          if (warp == 0 && er < n) {
            const int64_t idx = (int64_t)eb * p.d + u + er;
            if (p.world > 1) mc_red_add(p.red_mc[0] + idx, v);
            else p.red[0][idx] = v;
          }
          u += n;
        }
      }
      if (!ok || !cross_sync(p, s, xep)) break;
      trace_at(p, 3 + 5 * i);
      ev(p, s.misc, 4);
      // ---- D: x2 = x + attn; h = RMSNorm(x2); gate / up -> SwiGLU
      for (int b = 0; b < B; ++b) rows_a[b] = p.x + (int64_t)b * p.d;
      norm_rows<B>(s, p, rows_a, p.red[0], ly.mlp_norm, p.x2);
      ev(p, s.misc, 1);
      {
        const Phase& P2 = ph[2];
        int u0, u1;
        split_range(P2.U, gridDim.x, blockIdx.x, u0, u1);
        const int upg = group_units(P2, B);
        for (int u = u0; u < u1 && ok;) {
          const int n = group_len(P2, u, u1, upg);
          float v = 0.f;
          if (!gemv_group<B>(s, it, P2, n, rbuf, v, p)) {
            ok = false;
            break;
          }
          if (warp == 0) {
            const float up = __shfl_sync(0xffffffffu, v, min(lane + n * B, 31));
            if (er < n) p.act[(int64_t)eb * p.f + u + er] = __float2bfloat16(v / (1.f + __expf(-v)) * up);
          }
          u += n;
        }
      }
      if (!ok || !grid_sync(p, s)) break;
      trace_at(p, 4 + 5 * i);
      ev(p, s.misc, 4);
      // ---- E: down_proj, reduced over the ranks (the buffer read in D is re-zeroed)
      if (p.world > 1) zero_slice<B>(p, p.red[0]);
      copy_rows<B>(s, p.act, p.f);
      ev(p, s.misc, 1);
      {
        const Phase& P3 = ph[3];
        int u0, u1;
        split_range(P3.U, gridDim.x, blockIdx.x, u0, u1);
        const int upg = group_units(P3, B);
        for (int u = u0; u < u1 && ok;) {
          const int n = group_len(P3, u, u1, upg);
          float v = 0.f;
          if (!gemv_group<B>(s, it, P3, n, rbuf, v, p)) {
            ok = false;
            break;
          }
          if (warp == 0 && er < n) {
            const int64_t idx = (int64_t)eb * p.d + u + er;
            if (p.world > 1) mc_red_add(p.red_mc[1] + idx, v);
            else p.red[1][idx] = v;
          }
          u += n;
        }
      }
      if (!ok || !cross_sync(p, s, xep)) {
        ok = false;
        break;
      }
      trace_at(p, 5 + 5 * i);
      ev(p, s.misc, 4);
    }
    // ---- final norm, LM head rows of this rank, argmax
    if (ok) {
      for (int b = 0; b < B; ++b) rows_a[b] = p.x2 + (int64_t)b * p.d;
      norm_rows<B>(s, p, rows_a, p.red[1], p.final_norm, nullptr);
      const Phase hp = phase_of(p, 0, 4);
      int u0, u1;
      split_range(hp.U, gridDim.x, blockIdx.x, u0, u1);
      const int upg = group_units(hp, B);
      for (int u = u0; u < u1 && ok;) {
        const int n = group_len(hp, u, u1, upg);
        float v = 0.f;
        if (!gemv_group<B>(s, it, hp, n, rbuf, v, p)) {
          ok = false;
          break;
        }
        if (warp == 0 && er < n) {
          const int row = u + er;
          const unsigned long long key = argmax_key(v, p.vocab_col0 + row);
          best = key > best ? key : best;
          if (p.logits != nullptr) p.logits[(int64_t)eb * p.ld_logits + row] = v;
        }
        u += n;
      }
      if (ok && warp == 0) {
        // lanes with the same b (lane % B) hold candidates: max over them
#pragma unroll
        for (int sft = 16; sft >= B; sft >>= 1) {
          const unsigned long long o2 = __shfl_xor_sync(0xffffffffu, best, sft);
          best = o2 > best ? o2 : best;
        }
        if (lane < B) atomicMax(&p.st->cand[lane], best);
      }
    }
    if (ok) ok = grid_sync(p, s);
    trace_at(p, 1 + 5 * p.L);
    // every CTA has read the last reduction rows: re-zero this CTA's slice
    if (ok && p.world > 1) zero_slice<B>(p, p.red[1]);
    if (ok && blockIdx.x == 0) {
      if (p.world > 1) {
        if (tid < B) {
          const unsigned long long c = *reinterpret_cast<volatile unsigned long long*>(&p.st->cand[tid]);
          for (int q = 0; q < p.world; ++q)
            reinterpret_cast<unsigned long long*>(p.peer_keys[q])[p.rank * kMaxB + tid] = c;
        }
        ok = flag_exchange(p, s, xep);
        if (ok && tid < B) {
          unsigned long long c = 0ull;
          for (int q = 0; q < p.world; ++q) {
            const unsigned long long k = ldcg_u64(p.keys + q * kMaxB + tid);
            c = k > c ? k : c;
          }
          p.next[tid] = (int64_t)(0xFFFFFFFFu - (unsigned)(c & 0xFFFFFFFFull));
        }
      } else if (tid < B) {
        const unsigned long long c = *reinterpret_cast<volatile unsigned long long*>(&p.st->cand[tid]);
        p.next[tid] = (int64_t)(0xFFFFFFFFu - (unsigned)(c & 0xFFFFFFFFull));
      }
      if (tid < B) p.st->cand[tid] = 0ull;
      if (tid == 0) {
        p.st->xepoch = xep;
        p.st->gbase = (unsigned)s.misc[8];  // every CTA has passed the last grid barrier
      }
    }
    if (!ok && tid == 0) raise_abort(p, kStatusTimeoutEpilogue);
    // consumers record how far they got, for the drain below
    if (tid == 0) s.misc[3] = min(it, s.misc[7]);
  }
  __syncthreads();
  // Drain: every bulk copy this CTA issued must land before the CTA exits
  // (only chunks issued but never consumed remain after an abort).
  if (tid == 0) {
    const int issued = *reinterpret_cast<volatile int*>(&s.misc[2]);
    for (int c = s.misc[3]; c < issued; ++c) {
      volatile int never = 0;
      uint64_t* bar = &s.full[c % kStages];
      const uint32_t par = (uint32_t)(c / kStages) & 1u;
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(smem_u32(bar), par)) {
        if (globaltimer_ns() - t0 > p.timeout_ns) break;
      }
      (void)never;
    }
  }
}

}  // namespace mk

// ---------------------------------------------------------------- host
static int64_t ptr_of(const std::optional<at::Tensor>& t) {
  return (t && t->defined()) ? reinterpret_cast<int64_t>(t->data_ptr()) : 0;
}

// One decode step (see the file comment). `layers`: int64 [L, 11] device table
// of per-layer pointers (wqkv, bqkv or 0, wo, wgu, wd, attn_norm, mlp_norm,
// k cache, v cache, cos, sin); scratch tensors sized by the caller; for
// world > 1 the reduction rows, flags and argmax records are symmetric buffers
// (`*_peers`: every rank's address of the same buffer; `red_mc`: multicast).
void decode_mega(at::Tensor layers, at::Tensor embed, at::Tensor final_norm, at::Tensor head, int64_t vocab_rows,
                 int64_t vocab_col0, int64_t d, int64_t hq, int64_t hkv, int64_t f, double eps, double scale,
                 at::Tensor tok, at::Tensor pos, at::Tensor slot, at::Tensor seqlen, at::Tensor next,
                 std::optional<at::Tensor> logits, at::Tensor cache0, std::optional<at::Tensor> page_table,
                 at::Tensor x, at::Tensor x2, at::Tensor q, at::Tensor o, at::Tensor act, at::Tensor part,
                 at::Tensor pair_ctr, at::Tensor red0, at::Tensor red1, int64_t red0_mc, int64_t red1_mc,
                 at::Tensor flags, at::Tensor flag_peers, at::Tensor keys, at::Tensor key_peers, int64_t rank,
                 int64_t world, at::Tensor state, double timeout_s, std::optional<at::Tensor> trace,
                 int64_t debug) {
  c10::cuda::CUDAGuard g(embed.device());
  const int64_t B = tok.size(0);
  TORCH_CHECK(B == 1 || B == 2 || B == 4, "decode_mega: batch 1, 2 or 4");
  TORCH_CHECK(layers.is_cuda() && layers.scalar_type() == at::kLong && layers.dim() == 2 && layers.size(1) == 11,
              "decode_mega: layers int64 [L, 11]");
  TORCH_CHECK(d % 8 == 0 && f % 8 == 0 && hq % hkv == 0 && hq / hkv <= mk::kMaxG && B * hq * 1024 <= mk::kUnion,
              "decode_mega: shapes (query heads x batch rows too many for the attention merge)");
  TORCH_CHECK(B * std::max({d, hq * 128, f}) * 2 <= mk::kUnion, "decode_mega: activation rows exceed shared memory");
  TORCH_CHECK(world >= 1 && world <= 8 && (world == 1 || (red0_mc != 0 && red1_mc != 0)),
              "decode_mega: tensor parallel needs multicast reduction buffers");
  TORCH_CHECK(state.is_cuda() && state.numel() * state.element_size() >= (int64_t)sizeof(mk::State),
              "decode_mega: state block");
  const int dev = embed.get_device();
  int nsm = 0;
  AETHER_CUDA_CHECK(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));
  TORCH_CHECK(part.numel() >= B * hkv * nsm * (hq / hkv) * mk::kPartStride, "decode_mega: attention partials");
  TORCH_CHECK(pair_ctr.numel() >= B * hkv, "decode_mega: pair counters");

  mk::Params p{};
  p.layers = reinterpret_cast<const mk::Layer*>(layers.data_ptr());
  p.L = (int)layers.size(0);
  p.embed = reinterpret_cast<const mk::bf16*>(embed.data_ptr());
  p.final_norm = reinterpret_cast<const mk::bf16*>(final_norm.data_ptr());
  p.head = reinterpret_cast<const mk::bf16*>(head.data_ptr());
  p.vocab_rows = (int)vocab_rows;
  p.vocab_col0 = (int)vocab_col0;
  p.d = (int)d;
  p.hq = (int)hq;
  p.hkv = (int)hkv;
  p.f = (int)f;
  p.eps = (float)eps;
  p.scale_log2 = (float)(scale * 1.4426950408889634);
  p.tok = tok.data_ptr<int64_t>();
  p.pos = pos.data_ptr<int>();
  p.slot = slot.data_ptr<int>();
  p.seqlen = seqlen.data_ptr<int>();
  p.next = next.data_ptr<int64_t>();
  p.logits = logits && logits->defined() ? logits->data_ptr<float>() : nullptr;
  p.ld_logits = logits && logits->defined() ? logits->stride(0) : 0;
  p.slot_stride = cache0.stride(0);
  p.pos_stride = cache0.stride(1);
  p.pm = page_map(page_table, cache0);
  p.x = reinterpret_cast<mk::bf16*>(x.data_ptr());
  p.x2 = reinterpret_cast<mk::bf16*>(x2.data_ptr());
  p.q = reinterpret_cast<mk::bf16*>(q.data_ptr());
  p.o = reinterpret_cast<mk::bf16*>(o.data_ptr());
  p.act = reinterpret_cast<mk::bf16*>(act.data_ptr());
  p.part = part.data_ptr<float>();
  p.pair_ctr = pair_ctr.data_ptr<int>();
  p.red[0] = red0.data_ptr<float>();
  p.red[1] = red1.data_ptr<float>();
  p.red_mc[0] = reinterpret_cast<float*>(red0_mc);
  p.red_mc[1] = reinterpret_cast<float*>(red1_mc);
  p.flags = reinterpret_cast<uint32_t*>(flags.data_ptr());
  p.keys = reinterpret_cast<unsigned long long*>(keys.data_ptr());
  if (world > 1) {
    TORCH_CHECK(flag_peers.numel() >= world && key_peers.numel() >= world, "decode_mega: peer tables");
    auto fp = flag_peers.cpu(), kp = key_peers.cpu();
    for (int64_t r = 0; r < world; ++r) {
      p.peer_flags[r] = (uint64_t)fp.data_ptr<int64_t>()[r];
      p.peer_keys[r] = (uint64_t)kp.data_ptr<int64_t>()[r];
    }
  }
  p.rank = (int)rank;
  p.world = (int)world;
  p.st = reinterpret_cast<mk::State*>(state.data_ptr());
  p.status = device_status_word();
  p.timeout_ns = (uint64_t)(timeout_s * 1e9);
  p.trace = trace && trace->defined() ? reinterpret_cast<unsigned long long*>(trace->data_ptr()) : nullptr;
  p.debug = (int)debug;
  (void)ptr_of;

  static bool attr[3][64] = {};  // per batch instantiation and device
  const int bi = B == 1 ? 0 : (B == 2 ? 1 : 2);
  auto launch = [&](auto kernel) {
    if (!attr[bi][dev]) {
      AETHER_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, mk::kSmem));
      attr[bi][dev] = true;
    }
    int per_sm = 0;
    AETHER_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, mk::kThreads, mk::kSmem));
    if (per_sm < 1) {
      cudaFuncAttributes fa{};
      AETHER_CUDA_CHECK(cudaFuncGetAttributes(&fa, kernel));
      TORCH_CHECK(false, "decode_mega: kernel does not fit on an SM (registers ", fa.numRegs, ", max threads ",
                  fa.maxThreadsPerBlock, ", dynamic smem ", mk::kSmem, ")");
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)nsm);
    cfg.blockDim = dim3(mk::kThreads);
    cfg.dynamicSmemBytes = mk::kSmem;
    cfg.stream = at::cuda::getCurrentCUDAStream();
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;
    at[0].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    AETHER_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kernel, p));
  };
  if (B == 1) launch(mk::decode_mega_kernel<1>);
  else if (B == 2) launch(mk::decode_mega_kernel<2>);
  else launch(mk::decode_mega_kernel<4>);
}

}  // namespace aether
