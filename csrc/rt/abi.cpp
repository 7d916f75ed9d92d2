// The C ABI of libaether_rt: the `aether_*` symbols of the reference runtime
// (runtime/ABI.md; runtime/src/lib.rs:69-860) with the same names and the same
// positional argument order, so aetherc-emitted programs and the trainer link
// against this library unchanged. Buffers are caller-owned fp32/i32 host
// arrays; return codes follow the reference (0 = ok; losses return f32).
//
// The autodiff tape keeps the reference's stable partial op codes
// (ABI.md: ADD=1 SUB_PLUS=2 SUB_MINUS=3 MUL=4 MATMUL_LHS=5 MATMUL_RHS=6 RELU=7
// CROSS_ENTROPY=8 FORWARD_VJP=9 PARAM=10).
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "cpu_ops.h"

using namespace aether_rt;

namespace {
struct Partial {
  int dst, op, src;
};
struct Tape {
  std::vector<const void*> values;
  std::vector<Partial> partials;
  std::vector<const void*> grads;
  int reversed = 0;
};
std::mutex g_tape_mu;
Tape g_tape;  // the reference keeps one per-step tape, addressed by an opaque pointer

inline const float* F(const void* p) { return static_cast<const float*>(p); }
inline float* FM(void* p) { return static_cast<float*>(p); }
}  // namespace

extern "C" {

// ------------------------------------------------------------------ tape
void aether_autodiff_init(void* /*tape*/) {
  std::lock_guard<std::mutex> lk(g_tape_mu);
  g_tape = Tape();
}
void aether_autodiff_push(void* /*tape*/, const void* value) {
  std::lock_guard<std::mutex> lk(g_tape_mu);
  g_tape.values.push_back(value);
}
void aether_autodiff_accumulate(void* /*tape*/, const void* grad) {
  std::lock_guard<std::mutex> lk(g_tape_mu);
  g_tape.grads.push_back(grad);
}
void aether_autodiff_partial(void* /*tape*/, int dst_node, int op_code, int src_node) {
  std::lock_guard<std::mutex> lk(g_tape_mu);
  g_tape.partials.push_back({dst_node, op_code, src_node});
}
void aether_autodiff_reverse(void* /*tape*/) {
  std::lock_guard<std::mutex> lk(g_tape_mu);
  g_tape.reversed += 1;
}
int aether_rt_self_check() {
  std::lock_guard<std::mutex> lk(g_tape_mu);
  return (int)g_tape.values.size();
}
int aether_autodiff_partial_count() {
  std::lock_guard<std::mutex> lk(g_tape_mu);
  return (int)g_tape.partials.size();
}

// ------------------------------------------------------------------ host memory
// Every block carries a 16-byte header with its size, so the allocation
// probes (aether_prof_alloc_{total,live,peak}) can track frees too.
void aether_prof_note_alloc(int64_t bytes);  // ext.cpp
void aether_prof_note_free(int64_t bytes);
static int64_t rt_alloc(int64_t bytes) {
  bytes = std::max<int64_t>(bytes, 1);
  uint8_t* p = static_cast<uint8_t*>(std::calloc((size_t)bytes + 16, 1));
  if (!p) return 0;
  *reinterpret_cast<int64_t*>(p) = bytes;
  aether_prof_note_alloc(bytes);
  return (int64_t)(intptr_t)(p + 16);
}
int64_t aether_alloc_f32(int n) { return rt_alloc((int64_t)std::max(n, 1) * (int64_t)sizeof(float)); }
int64_t aether_alloc_i32(int n) { return rt_alloc((int64_t)std::max(n, 1) * (int64_t)sizeof(int32_t)); }
int64_t aether_alloc_bytes(int64_t n) { return rt_alloc(n); }
void aether_free(int64_t p) {
  if (p == 0) return;
  uint8_t* base = reinterpret_cast<uint8_t*>((intptr_t)p) - 16;
  aether_prof_note_free(*reinterpret_cast<int64_t*>(base));
  std::free(base);
}

// SplitMix64 + Box-Muller N(0, scale^2) fill (same generator as the trainer).
int aether_init_normal_f32(void* buf, int n, float scale, int64_t seed) {
  const float mean = 0.f, std = scale;
  uint64_t state = (uint64_t)seed + 0x9E3779B97F4A7C15ull;
  auto next = [&]() {
    state += 0x9E3779B97F4A7C15ull;
    uint64_t z = state;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
  };
  auto f32 = [&]() { return (float)(next() >> 40) / (float)(1ull << 24); };
  float* o = FM(buf);
  for (int i = 0; i < n; ++i) {
    float u;
    do {
      u = f32();
    } while (u <= 1e-10f);
    const float v = f32();
    o[i] = mean + std * std::sqrt(-2.f * std::log(u)) * std::cos(2.f * 3.14159265358979f * v);
  }
  return 0;
}

int aether_fill_labels_i32(void* buf, int n, int modulo, int64_t seed) {
  uint64_t s = (uint64_t)seed;
  int32_t* o = static_cast<int32_t*>(buf);
  for (int i = 0; i < n; ++i) {
    s = s * 6364136223846793005ull + 1442695040888963407ull;
    o[i] = (int32_t)((s >> 33) % (uint64_t)std::max(1, modulo));
  }
  return 0;
}

float aether_load_f32(const void* buf, int i) { return F(buf)[i]; }
void aether_store_f32(void* buf, int i, float v) { FM(buf)[i] = v; }

// ------------------------------------------------------------------ ops
int aether_op_matmul_f32(const void* a, const void* b, void* out, int m, int k, int n) {
  matmul(F(a), F(b), FM(out), m, k, n);
  return 0;
}
int aether_op_matmul_backward_lhs_f32(const void* dy, const void* b, void* da, int m, int k, int n) {
  matmul_bwd_lhs(F(dy), F(b), FM(da), m, k, n);
  return 0;
}
int aether_op_matmul_backward_rhs_f32(const void* a, const void* dy, void* db, int m, int k, int n) {
  matmul_bwd_rhs(F(a), F(dy), FM(db), m, k, n);
  return 0;
}
int aether_op_matmul_blocked_f32(const void* a, const void* b, void* out, int m, int k, int n) {
  return aether_op_matmul_f32(a, b, out, m, k, n);
}
int aether_op_matmul_f32_auto(const void* a, const void* b, void* out, int m, int k, int n) {
  return aether_op_matmul_f32(a, b, out, m, k, n);
}
int aether_op_conv2d_f32(const void* input, const void* kernel, void* output, int n, int c_in, int h, int w, int c_out,
                         int kh, int kw) {
  // valid convolution, stride 1, NCHW input, [c_out, c_in, kh, kw] kernel
  const int oh = h - kh + 1, ow = w - kw + 1;
  const float* x = F(input);
  const float* K = F(kernel);
  float* y = FM(output);
  for (int b = 0; b < n; ++b)
    for (int co = 0; co < c_out; ++co)
      for (int i = 0; i < oh; ++i)
        for (int j = 0; j < ow; ++j) {
          float s = 0.f;
          for (int ci = 0; ci < c_in; ++ci)
            for (int u = 0; u < kh; ++u)
              for (int v = 0; v < kw; ++v)
                s += x[(((size_t)b * c_in + ci) * h + i + u) * w + j + v] * K[(((size_t)co * c_in + ci) * kh + u) * kw + v];
          y[(((size_t)b * c_out + co) * oh + i) * ow + j] = s;
        }
  return 0;
}
int aether_op_add_f32(const void* a, const void* b, void* out, int n) {
  for (int i = 0; i < n; ++i) FM(out)[i] = F(a)[i] + F(b)[i];
  return 0;
}
int aether_op_add_inplace_f32(void* x, const void* y, int n) {
  for (int i = 0; i < n; ++i) FM(x)[i] += F(y)[i];
  return 0;
}
int aether_op_add_bias_f32(void* x, const void* b, int rows, int cols) {
  for (int r = 0; r < rows; ++r)
    for (int c = 0; c < cols; ++c) FM(x)[(size_t)r * cols + c] += F(b)[c];
  return 0;
}
int aether_op_scale_f32(void* x, float s, int n) {
  for (int i = 0; i < n; ++i) FM(x)[i] *= s;
  return 0;
}
int aether_op_axpy_f32(float alpha, const void* x, void* y, int n) {
  for (int i = 0; i < n; ++i) FM(y)[i] += alpha * F(x)[i];
  return 0;
}
int aether_op_gelu_f32(void* x, int n) {
  for (int i = 0; i < n; ++i) FM(x)[i] = gelu_tanh(FM(x)[i]);
  return 0;
}
int aether_op_gelu_backward_f32(const void* x, const void* dy, void* dx, int n) {
  for (int i = 0; i < n; ++i) FM(dx)[i] = F(dy)[i] * gelu_tanh_grad(F(x)[i]);
  return 0;
}
int aether_op_gelu_erf_f32(void* x, int n) {
  for (int i = 0; i < n; ++i) {
    const float v = FM(x)[i];
    FM(x)[i] = 0.5f * v * (1.f + std::erf(v * 0.70710678118654752f));
  }
  return 0;
}
int aether_op_silu_f32(void* x, int n) {
  for (int i = 0; i < n; ++i) {
    const float v = FM(x)[i];
    FM(x)[i] = v / (1.f + std::exp(-v));
  }
  return 0;
}
int aether_op_silu_backward_f32(const void* x, const void* dy, void* dx, int n) {
  for (int i = 0; i < n; ++i) {
    const float v = F(x)[i], s = 1.f / (1.f + std::exp(-v));
    FM(dx)[i] = F(dy)[i] * s * (1.f + v * (1.f - s));
  }
  return 0;
}
int aether_op_relu_f32(void* x, int n) {
  for (int i = 0; i < n; ++i) FM(x)[i] = std::max(0.f, FM(x)[i]);
  return 0;
}
int aether_op_relu_backward_f32(const void* x, const void* dy, void* dx, int n) {
  for (int i = 0; i < n; ++i) FM(dx)[i] = F(x)[i] > 0.f ? F(dy)[i] : 0.f;
  return 0;
}
int aether_op_tanh_f32(void* x, int n) {
  for (int i = 0; i < n; ++i) FM(x)[i] = std::tanh(FM(x)[i]);
  return 0;
}
int aether_op_sigmoid_f32(void* x, int n) {
  for (int i = 0; i < n; ++i) FM(x)[i] = 1.f / (1.f + std::exp(-FM(x)[i]));
  return 0;
}
int aether_op_softmax_f32(void* x, int rows, int cols, int /*axis*/) {
  softmax_rows(FM(x), rows, cols);
  return 0;
}
int aether_op_softmax_backward_f32(const void* y, const void* dy, void* dx, int rows, int cols) {
  softmax_bwd(F(y), F(dy), FM(dx), rows, cols);
  return 0;
}
int aether_op_layer_norm_f32(const void* x, const void* gamma, const void* beta, float eps, void* out, void* mean_out,
                             void* inv_std_out, int rows, int d) {
  layer_norm(F(x), F(gamma), F(beta), eps, FM(out), FM(mean_out), FM(inv_std_out), rows, d);
  return 0;
}
int aether_op_layer_norm_backward_f32(const void* x, const void* gamma, const void* dy, const void* mean,
                                      const void* inv_std, void* dx, void* dgamma, void* dbeta, int rows, int d) {
  std::memset(dgamma, 0, sizeof(float) * d);
  std::memset(dbeta, 0, sizeof(float) * d);
  layer_norm_bwd(F(x), F(gamma), F(dy), F(mean), F(inv_std), FM(dx), FM(dgamma), FM(dbeta), rows, d);
  return 0;
}
int aether_op_rms_norm_f32(const void* x, const void* gamma, float eps, void* out, int rows, int d) {
  rms_norm(F(x), F(gamma), eps, FM(out), rows, d);
  return 0;
}
int aether_op_rope_apply_f32(void* x, int seq, int n_heads, int head_dim, float base, int pos_start) {
  rope(FM(x), seq, n_heads, head_dim, base, pos_start);
  return 0;
}
int aether_op_gqa_repeat_kv_f32(const void* kv_in, void* kv_out, int seq, int n_kv_heads, int head_dim,
                                int n_q_heads) {
  const int g = n_q_heads / n_kv_heads;
  for (int t = 0; t < seq; ++t)
    for (int h = 0; h < n_q_heads; ++h)
      std::memcpy(FM(kv_out) + ((size_t)t * n_q_heads + h) * head_dim,
                  F(kv_in) + ((size_t)t * n_kv_heads + h / g) * head_dim, sizeof(float) * head_dim);
  return 0;
}
int aether_op_apply_lora_f32(void* w, const void* lora_a, const void* lora_b, float scale, int d_in, int d_out,
                             int rank) {
  // W[d_in, d_out] += scale * A[d_in? r] ... : the reference stores A [r, d_in], B [d_out, r]
  for (int i = 0; i < d_in; ++i)
    for (int o = 0; o < d_out; ++o) {
      float s = 0.f;
      for (int r = 0; r < rank; ++r) s += F(lora_b)[(size_t)o * rank + r] * F(lora_a)[(size_t)r * d_in + i];
      FM(w)[(size_t)i * d_out + o] += scale * s;
    }
  return 0;
}
int aether_op_sdpa_causal_f32(const void* q, const void* k, const void* v, void* out, void* attn_out, int bh,
                              int s_len, int d) {
  sdpa_causal(F(q), F(k), F(v), FM(out), FM(attn_out), bh, s_len, d);
  return 0;
}
int aether_op_sdpa_full_f32(const void* q, const void* k, const void* v, void* out, void* attn_out, int bh, int s_len,
                            int d) {
  sdpa_full(F(q), F(k), F(v), FM(out), FM(attn_out), bh, s_len, d);
  return 0;
}
int aether_op_sdpa_causal_backward_f32(const void* q, const void* k, const void* v, const void* attn,
                                       const void* dout, void* dq, void* dk, void* dv, int bh, int s_len, int d) {
  sdpa_causal_bwd(F(q), F(k), F(v), F(attn), F(dout), FM(dq), FM(dk), FM(dv), bh, s_len, d);
  return 0;
}
int aether_flash_attention_v2_f32(const void* q, const void* k, const void* v, void* out, int seq_len, int d_head) {
  flash_attention_v2(F(q), F(k), F(v), FM(out), seq_len, d_head);
  return 0;
}
float aether_op_cross_entropy_f32(const void* logits, const void* labels, void* probs_out, int b, int v) {
  return cross_entropy(F(logits), static_cast<const int32_t*>(labels), FM(probs_out), b, v);
}
int aether_op_cross_entropy_backward_f32(const void* probs, const void* labels, void* dlogits, int b, int v) {
  cross_entropy_bwd(F(probs), static_cast<const int32_t*>(labels), FM(dlogits), b, v);
  return 0;
}
float aether_op_mse_f32(const void* pred, const void* target, int n) {
  double s = 0.0;
  for (int i = 0; i < n; ++i) s += (double)(F(pred)[i] - F(target)[i]) * (F(pred)[i] - F(target)[i]);
  return (float)(s / std::max(1, n));
}
int aether_op_mse_backward_f32(const void* pred, const void* target, void* dpred, int n) {
  for (int i = 0; i < n; ++i) FM(dpred)[i] = 2.f * (F(pred)[i] - F(target)[i]) / std::max(1, n);
  return 0;
}
float aether_op_mae_f32(const void* pred, const void* target, int n) {
  double s = 0.0;
  for (int i = 0; i < n; ++i) s += std::fabs(F(pred)[i] - F(target)[i]);
  return (float)(s / std::max(1, n));
}
int aether_op_mae_backward_f32(const void* pred, const void* target, void* dpred, int n) {
  for (int i = 0; i < n; ++i) {
    const float d = F(pred)[i] - F(target)[i];
    FM(dpred)[i] = (d > 0.f ? 1.f : (d < 0.f ? -1.f : 0.f)) / std::max(1, n);
  }
  return 0;
}
float aether_op_bce_with_logits_f32(const void* pred, const void* target, int n) {
  double s = 0.0;
  for (int i = 0; i < n; ++i) {
    const float x = F(pred)[i], y = F(target)[i];
    s += std::max(x, 0.f) - x * y + std::log1p(std::exp(-std::fabs(x)));
  }
  return (float)(s / std::max(1, n));
}
int aether_op_bce_with_logits_backward_f32(const void* pred, const void* target, void* dpred, int n) {
  for (int i = 0; i < n; ++i) FM(dpred)[i] = (1.f / (1.f + std::exp(-F(pred)[i])) - F(target)[i]) / std::max(1, n);
  return 0;
}
float aether_op_huber_f32(const void* pred, const void* target, int n, float delta) {
  double s = 0.0;
  for (int i = 0; i < n; ++i) {
    const float d = std::fabs(F(pred)[i] - F(target)[i]);
    s += d <= delta ? 0.5 * d * d : delta * (d - 0.5 * delta);
  }
  return (float)(s / std::max(1, n));
}
int aether_op_huber_backward_f32(const void* pred, const void* target, void* dpred, int n, float delta) {
  for (int i = 0; i < n; ++i) {
    const float d = F(pred)[i] - F(target)[i];
    FM(dpred)[i] = (std::fabs(d) <= delta ? d : (d > 0 ? delta : -delta)) / std::max(1, n);
  }
  return 0;
}
int aether_op_embedding_lookup_f32(const void* w, const void* ids, void* out, int b, int s_len, int v_size, int d) {
  const int32_t* id = static_cast<const int32_t*>(ids);
  for (int t = 0; t < b * s_len; ++t) {
    const int r = std::min(std::max(id[t], 0), v_size - 1);
    std::memcpy(FM(out) + (size_t)t * d, F(w) + (size_t)r * d, sizeof(float) * d);
  }
  return 0;
}
int aether_op_embedding_backward_f32(const void* ids, const void* dy, void* dw, int b, int s_len, int v_size, int d) {
  const int32_t* id = static_cast<const int32_t*>(ids);
  for (int t = 0; t < b * s_len; ++t) {
    const int r = id[t];
    if (r < 0 || r >= v_size) continue;
    for (int i = 0; i < d; ++i) FM(dw)[(size_t)r * d + i] += F(dy)[(size_t)t * d + i];
  }
  return 0;
}
int aether_op_zero_grad_f32(void* g, int n) {
  std::memset(g, 0, sizeof(float) * (size_t)std::max(n, 0));
  return 0;
}
float aether_op_clip_grad_norm_f32(void* g, float max_norm, int n) { return clip_grad_norm(FM(g), max_norm, (size_t)n); }
int aether_op_adamw_step_f32(void* param, const void* grad, void* m, void* v, float lr, float beta1, float beta2,
                             float eps, float wd, int64_t step, int n) {
  adamw(FM(param), F(grad), FM(m), FM(v), lr, beta1, beta2, eps, wd, step, (size_t)n);
  return 0;
}
int aether_op_sgd_step_f32(void* param, const void* grad, float lr, float momentum, float wd, void* state, int n) {
  for (int i = 0; i < n; ++i) {
    float g = F(grad)[i] + wd * FM(param)[i];
    if (state && momentum != 0.f) {
      FM(state)[i] = momentum * FM(state)[i] + g;
      g = FM(state)[i];
    }
    FM(param)[i] -= lr * g;
  }
  return 0;
}
// Single-process fallbacks of the collective ABI (multi-rank programs use the
// torch.distributed engines; these keep world-size-1 programs linking).
// aether_op_all_reduce_sum_f32 and aether_dist_all_reduce: collectives.cpp

}  // extern "C"
