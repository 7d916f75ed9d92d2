// fp32 CPU operator bodies of libaether_rt (row-major, caller-owned buffers).
//
// These restate the reference runtime's CPU ops (runtime/src/ops.rs) -- the
// numerics oracle of the reference and the op set its trainer and
// aetherc-emitted programs call through the C ABI (runtime/ABI.md). Semantics
// kept alike on purpose so programs behave the same: tanh-GELU with 0.044715,
// half-split RoPE theta_i = base^(-2i/hd), cross-entropy floored at 1e-12,
// decoupled AdamW, global-norm clipping in double precision.
#pragma once

#include <cstddef>
#include <cstdint>

namespace aether_rt {

void matmul(const float* a, const float* b, float* out, int m, int k, int n);            // out = a[m,k] b[k,n]
void matmul_acc(const float* a, const float* b, float* out, int m, int k, int n);        // out += a b
void matmul_bwd_lhs(const float* dy, const float* b, float* da, int m, int k, int n);    // da = dy b^T
void matmul_bwd_lhs_acc(const float* dy, const float* b, float* da, int m, int k, int n);
void matmul_bwd_rhs(const float* a, const float* dy, float* db, int m, int k, int n);    // db = a^T dy
void matmul_bwd_rhs_acc(const float* a, const float* dy, float* db, int m, int k, int n);
void matmul_nt(const float* a, const float* b, float* out, int m, int k, int n);         // out = a[m,k] b[n,k]^T

float gelu_tanh(float x);
float gelu_tanh_grad(float x);

void layer_norm(const float* x, const float* g, const float* b, float eps, float* out, float* mean, float* inv,
                int rows, int d);
void layer_norm_bwd(const float* x, const float* g, const float* dy, const float* mean, const float* inv, float* dx,
                    float* dg, float* db, int rows, int d);  // dg/db accumulate
void rms_norm(const float* x, const float* g, float eps, float* out, int rows, int d);
void softmax_rows(float* x, int rows, int cols);
void softmax_bwd(const float* y, const float* dy, float* dx, int rows, int cols);
void rope(float* x, int seq, int n_heads, int head_dim, float base, int pos_start);
void sdpa_causal(const float* q, const float* k, const float* v, float* out, float* attn, int bh, int s, int d);
void sdpa_full(const float* q, const float* k, const float* v, float* out, float* attn, int bh, int s, int d);
void sdpa_causal_bwd(const float* q, const float* k, const float* v, const float* attn, const float* dout, float* dq,
                     float* dk, float* dv, int bh, int s, int d);
float cross_entropy(const float* logits, const int32_t* labels, float* probs, int b, int v);
void cross_entropy_bwd(const float* probs, const int32_t* labels, float* dlogits, int b, int v);
float clip_grad_norm(float* g, float max_norm, size_t n);
void adamw(float* p, const float* g, float* m, float* v, float lr, float b1, float b2, float eps, float wd,
           int64_t step, size_t n);
void flash_attention_v2(const float* q, const float* k, const float* v, float* out, int s, int d);

}  // namespace aether_rt
