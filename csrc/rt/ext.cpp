// libaether_rt: the wider C ABI around the core ops -- extended CPU ops,
// optimiser zoo, pooling, dtype conversions, GGUF block dequantisers, host
// serving structures (paged-KV block pool + page tables, batch scheduler,
// continuous batch, speculative-decoding accept test, model registry, rate
// limiter), observability (counters, Prometheus text, allocation / timer
// probes, crash breadcrumbs, OOM flag) and the single-rank collective shapes.
//
// Symbol names, argument order and return codes follow the reference
// runtime's ABI (runtime/src/lib.rs: extended ops 2471-2820 and 3011-3320,
// dtype conversions 1895-1975, dequantisers 217 and 9218-9300, serving sims
// 5550-6210, observability 1377-1391, 2401, 3660-3680, 6253-6276) so compiled
// Aether programs link against this library unchanged. Handles are small
// integers indexing per-kind tables; every entry point validates its handle
// and returns a negative code instead of crashing.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <atomic>
#include <mutex>
#include <string>
#include <vector>

#include <unistd.h>

extern "C" {
#define AE_API __attribute__((visibility("default")))
}

namespace {

template <class T>
struct Table {
  std::vector<std::unique_ptr<T>> slots;
  std::mutex mu;
  int64_t add(std::unique_ptr<T> v) {
    std::lock_guard<std::mutex> g(mu);
    for (size_t i = 0; i < slots.size(); ++i)
      if (!slots[i]) {
        slots[i] = std::move(v);
        return (int64_t)i;
      }
    slots.push_back(std::move(v));
    return (int64_t)slots.size() - 1;
  }
  T* get(int64_t h) {
    if (h < 0 || (size_t)h >= slots.size()) return nullptr;
    return slots[(size_t)h].get();
  }
  int drop(int64_t h) {
    std::lock_guard<std::mutex> g(mu);
    if (h < 0 || (size_t)h >= slots.size() || !slots[(size_t)h]) return -1;
    slots[(size_t)h].reset();
    return 0;
  }
};

inline float* F(void* p) { return static_cast<float*>(p); }
inline const float* CF(const void* p) { return static_cast<const float*>(p); }
inline float softplus(float x) { return x > 20.f ? x : std::log1p(std::exp(x)); }
inline float sigmoidf(float x) { return 1.f / (1.f + std::exp(-x)); }

}  // namespace

extern "C" {

// ------------------------------------------------------------------ elementwise math (in place)
#define AE_UNARY(NAME, EXPR)                              \
  AE_API int NAME(void* x, int n) {                       \
    if (!x || n < 0) return -1;                           \
    float* s = F(x);                                      \
    for (int i = 0; i < n; ++i) {                         \
      const float v = s[i];                               \
      (void)v;                                            \
      s[i] = (EXPR);                                      \
    }                                                     \
    return 0;                                             \
  }
AE_UNARY(aether_op_log_f32, std::log(v))
AE_UNARY(aether_op_exp_f32, std::exp(v))
AE_UNARY(aether_op_sin_f32, std::sin(v))
AE_UNARY(aether_op_cos_f32, std::cos(v))
AE_UNARY(aether_op_tan_f32, std::tan(v))
AE_UNARY(aether_op_recip_f32, 1.f / v)
AE_UNARY(aether_op_abs_f32, std::fabs(v))
AE_UNARY(aether_op_sign_f32, v > 0.f ? 1.f : (v < 0.f ? -1.f : 0.f))
AE_UNARY(aether_op_mish_f32, v * std::tanh(softplus(v)))
AE_UNARY(aether_op_zeros_f32, 0.f)
AE_UNARY(aether_op_ones_f32, 1.f)
#undef AE_UNARY

AE_API int aether_op_pow_f32(void* x, float p, int n) {
  if (!x || n < 0) return -1;
  for (int i = 0; i < n; ++i) F(x)[i] = std::pow(F(x)[i], p);
  return 0;
}
AE_API int aether_op_clamp_f32(void* x, float lo, float hi, int n) {
  if (!x || n < 0) return -1;
  for (int i = 0; i < n; ++i) F(x)[i] = std::min(std::max(F(x)[i], lo), hi);
  return 0;
}
AE_API int aether_op_leaky_relu_f32(void* x, float slope, int n) {
  if (!x || n < 0) return -1;
  for (int i = 0; i < n; ++i)
    if (F(x)[i] < 0.f) F(x)[i] *= slope;
  return 0;
}
AE_API int aether_op_elu_f32(void* x, float alpha, int n) {
  if (!x || n < 0) return -1;
  for (int i = 0; i < n; ++i)
    if (F(x)[i] < 0.f) F(x)[i] = alpha * (std::exp(F(x)[i]) - 1.f);
  return 0;
}
AE_API int aether_op_full_f32(void* x, float val, int n) {
  if (!x || n < 0) return -1;
  std::fill(F(x), F(x) + n, val);
  return 0;
}
AE_API int aether_op_arange_f32(void* x, float start, float step, int n) {
  if (!x || n < 0) return -1;
  for (int i = 0; i < n; ++i) F(x)[i] = start + step * (float)i;
  return 0;
}
AE_API int aether_op_eye_f32(void* x, int n) {
  if (!x || n < 0) return -1;
  for (int i = 0; i < n; ++i)
    for (int j = 0; j < n; ++j) F(x)[(size_t)i * n + j] = i == j ? 1.f : 0.f;
  return 0;
}
AE_API int aether_op_tril_f32(void* x, int rows, int cols) {
  if (!x || rows < 0 || cols < 0) return -1;
  for (int i = 0; i < rows; ++i)
    for (int j = i + 1; j < cols; ++j) F(x)[(size_t)i * cols + j] = 0.f;
  return 0;
}
AE_API int aether_op_triu_f32(void* x, int rows, int cols) {
  if (!x || rows < 0 || cols < 0) return -1;
  for (int i = 0; i < rows; ++i)
    for (int j = 0; j < std::min(i, cols); ++j) F(x)[(size_t)i * cols + j] = 0.f;
  return 0;
}

// ------------------------------------------------------------------ activation backwards
// grad is the upstream gradient on entry and dL/dx on exit.
AE_API int aether_op_tanh_backward_f32(const void* y, void* grad, int n) {
  if (!y || !grad || n < 0) return -1;
  for (int i = 0; i < n; ++i) F(grad)[i] *= 1.f - CF(y)[i] * CF(y)[i];
  return 0;
}
AE_API int aether_op_sigmoid_backward_f32(const void* y, void* grad, int n) {
  if (!y || !grad || n < 0) return -1;
  for (int i = 0; i < n; ++i) F(grad)[i] *= CF(y)[i] * (1.f - CF(y)[i]);
  return 0;
}
AE_API int aether_op_leaky_relu_backward_f32(const void* x, void* grad, float slope, int n) {
  if (!x || !grad || n < 0) return -1;
  for (int i = 0; i < n; ++i)
    if (CF(x)[i] < 0.f) F(grad)[i] *= slope;
  return 0;
}
AE_API int aether_op_elu_backward_f32(const void* x, void* grad, float alpha, int n) {
  if (!x || !grad || n < 0) return -1;
  for (int i = 0; i < n; ++i)
    if (CF(x)[i] < 0.f) F(grad)[i] *= alpha * std::exp(CF(x)[i]);
  return 0;
}
AE_API int aether_op_mish_backward_f32(const void* x, void* grad, int n) {
  if (!x || !grad || n < 0) return -1;
  for (int i = 0; i < n; ++i) {
    const float v = CF(x)[i];
    const float t = std::tanh(softplus(v));
    F(grad)[i] *= t + v * (1.f - t * t) * sigmoidf(v);
  }
  return 0;
}

// ------------------------------------------------------------------ reductions
AE_API float aether_op_sum_f32(const void* x, int n) {
  double s = 0;
  for (int i = 0; i < n; ++i) s += CF(x)[i];
  return (float)s;
}
AE_API float aether_op_mean_f32(const void* x, int n) { return n > 0 ? aether_op_sum_f32(x, n) / (float)n : 0.f; }
AE_API float aether_op_var_f32(const void* x, int n) {
  if (n <= 0) return 0.f;
  double mean = 0, m2 = 0;  // Welford
  for (int i = 0; i < n; ++i) {
    const double d = CF(x)[i] - mean;
    mean += d / (i + 1);
    m2 += d * (CF(x)[i] - mean);
  }
  return (float)(m2 / n);
}
AE_API float aether_op_std_f32(const void* x, int n) { return std::sqrt(aether_op_var_f32(x, n)); }
AE_API float aether_op_max_red_f32(const void* x, int n) {
  float m = -INFINITY;
  for (int i = 0; i < n; ++i) m = std::max(m, CF(x)[i]);
  return m;
}
AE_API float aether_op_min_red_f32(const void* x, int n) {
  float m = INFINITY;
  for (int i = 0; i < n; ++i) m = std::min(m, CF(x)[i]);
  return m;
}
AE_API int64_t aether_op_argmax_f32(const void* x, int n) {
  int64_t b = 0;
  for (int i = 1; i < n; ++i)
    if (CF(x)[i] > CF(x)[b]) b = i;
  return n > 0 ? b : -1;
}
AE_API int64_t aether_op_argmin_f32(const void* x, int n) {
  int64_t b = 0;
  for (int i = 1; i < n; ++i)
    if (CF(x)[i] < CF(x)[b]) b = i;
  return n > 0 ? b : -1;
}
AE_API float aether_op_prod_f32(const void* x, int n) {
  double p = 1;
  for (int i = 0; i < n; ++i) p *= CF(x)[i];
  return (float)p;
}

// ------------------------------------------------------------------ selection / shape
AE_API int aether_op_masked_fill_f32(void* x, const void* mask, float fill, int n) {
  if (!x || !mask || n < 0) return -1;
  for (int i = 0; i < n; ++i)
    if (CF(mask)[i] != 0.f) F(x)[i] = fill;
  return 0;
}
AE_API int aether_op_where_f32(const void* cond, const void* a, const void* b, void* out, int n) {
  if (!cond || !a || !b || !out || n < 0) return -1;
  for (int i = 0; i < n; ++i) F(out)[i] = CF(cond)[i] != 0.f ? CF(a)[i] : CF(b)[i];
  return 0;
}
AE_API int aether_op_cat_f32(const void* a, int na, const void* b, int nb, void* out) {
  if (!a || !b || !out || na < 0 || nb < 0) return -1;
  std::memcpy(out, a, sizeof(float) * (size_t)na);
  std::memcpy(F(out) + na, b, sizeof(float) * (size_t)nb);
  return 0;
}
AE_API int aether_op_repeat_f32(const void* x, int n, int k, void* out) {
  if (!x || !out || n < 0 || k < 0) return -1;
  for (int r = 0; r < k; ++r) std::memcpy(F(out) + (size_t)r * n, x, sizeof(float) * (size_t)n);
  return 0;
}

// ------------------------------------------------------------------ optimisers
AE_API int aether_op_sgd_momentum_step_f32(void* params, const void* grad, void* buf, float lr, float mu, float wd,
                                           int n) {
  if (!params || !grad || !buf || n < 0) return -1;
  for (int i = 0; i < n; ++i) {
    const float g = CF(grad)[i] + wd * F(params)[i];
    F(buf)[i] = mu * F(buf)[i] + g;
    F(params)[i] -= lr * F(buf)[i];
  }
  return 0;
}
AE_API int aether_op_rmsprop_step_f32(void* params, const void* grad, void* sq, float lr, float rho, float eps, int n) {
  if (!params || !grad || !sq || n < 0) return -1;
  for (int i = 0; i < n; ++i) {
    const float g = CF(grad)[i];
    F(sq)[i] = rho * F(sq)[i] + (1.f - rho) * g * g;
    F(params)[i] -= lr * g / (std::sqrt(F(sq)[i]) + eps);
  }
  return 0;
}
AE_API int aether_op_adagrad_step_f32(void* params, const void* grad, void* sq, float lr, float eps, int n) {
  if (!params || !grad || !sq || n < 0) return -1;
  for (int i = 0; i < n; ++i) {
    const float g = CF(grad)[i];
    F(sq)[i] += g * g;
    F(params)[i] -= lr * g / (std::sqrt(F(sq)[i]) + eps);
  }
  return 0;
}
// Lion: step along sign(b1 m + (1 - b1) g), then m <- b2 m + (1 - b2) g.
AE_API int aether_op_lion_step_f32(void* param, const void* grad, void* m, int n, float lr, float beta1, float beta2,
                                   float wd) {
  if (!param || !grad || !m || n < 0) return -1;
  for (int i = 0; i < n; ++i) {
    const float u = beta1 * F(m)[i] + (1.f - beta1) * CF(grad)[i];
    const float dir = u > 0.f ? 1.f : (u < 0.f ? -1.f : 0.f);
    F(param)[i] -= lr * (dir + wd * F(param)[i]);
    F(m)[i] = beta2 * F(m)[i] + (1.f - beta2) * CF(grad)[i];
  }
  return 0;
}
// LAMB: Adam direction (bias corrections passed in) plus decoupled decay,
// scaled by the trust ratio ||p|| / ||update|| over the whole buffer.
AE_API int aether_op_lamb_step_f32(void* param, const void* grad, void* m, void* v, int n, float lr, float beta1,
                                   float beta2, float eps, float wd, float bc1, float bc2) {
  if (!param || !grad || !m || !v || n < 0) return -1;
  std::vector<float> upd((size_t)n);
  double un = 0, pn = 0;
  for (int i = 0; i < n; ++i) {
    const float g = CF(grad)[i];
    F(m)[i] = beta1 * F(m)[i] + (1.f - beta1) * g;
    F(v)[i] = beta2 * F(v)[i] + (1.f - beta2) * g * g;
    const float r = (F(m)[i] / bc1) / (std::sqrt(F(v)[i] / bc2) + eps) + wd * F(param)[i];
    upd[(size_t)i] = r;
    un += (double)r * r;
    pn += (double)F(param)[i] * F(param)[i];
  }
  const double trust = (pn > 0 && un > 0) ? std::sqrt(pn) / std::sqrt(un) : 1.0;
  const float s = (float)(lr * trust);
  for (int i = 0; i < n; ++i) F(param)[i] -= s * upd[(size_t)i];
  return 0;
}
// Adafactor with factored second moments: row / column EMAs of g^2, the
// second-moment estimate v_ij = r_i c_j / mean(r), step g / sqrt(v / cols).
AE_API int aether_op_adafactor_step_f32(void* param, const void* grad, void* row, void* col, int n_rows, int n_cols,
                                        float lr, float eps, float decay) {
  if (!param || !grad || !row || !col || n_rows <= 0 || n_cols <= 0) return -1;
  const float* g = CF(grad);
  for (int i = 0; i < n_rows; ++i) {
    double s = 0;
    for (int j = 0; j < n_cols; ++j) s += (double)g[(size_t)i * n_cols + j] * g[(size_t)i * n_cols + j];
    F(row)[i] = decay * F(row)[i] + (1.f - decay) * (float)s;
  }
  for (int j = 0; j < n_cols; ++j) {
    double s = 0;
    for (int i = 0; i < n_rows; ++i) s += (double)g[(size_t)i * n_cols + j] * g[(size_t)i * n_cols + j];
    F(col)[j] = decay * F(col)[j] + (1.f - decay) * (float)s;
  }
  double rsum = 0;
  for (int i = 0; i < n_rows; ++i) rsum += F(row)[i];
  const float rmean = std::max((float)(rsum / n_rows), eps);
  for (int i = 0; i < n_rows; ++i)
    for (int j = 0; j < n_cols; ++j) {
      const float vhat = F(row)[i] / rmean * F(col)[j];
      const float denom = std::max(std::sqrt(vhat / (float)n_cols), eps);
      F(param)[(size_t)i * n_cols + j] -= lr * g[(size_t)i * n_cols + j] / denom;
    }
  return 0;
}

// ------------------------------------------------------------------ pooling (N, C, H, W)
static int pool2d(const void* x, void* y, int n, int c, int h, int w, int kh, int kw, int sh, int sw, int ph, int pw,
                  bool is_max) {
  if (!x || !y || kh <= 0 || kw <= 0 || sh <= 0 || sw <= 0) return -1;
  const int ho = (h + 2 * ph - kh) / sh + 1, wo = (w + 2 * pw - kw) / sw + 1;
  for (int p = 0; p < n * c; ++p) {
    const float* xp = CF(x) + (size_t)p * h * w;
    float* yp = F(y) + (size_t)p * ho * wo;
    for (int oh = 0; oh < ho; ++oh)
      for (int ow = 0; ow < wo; ++ow) {
        float acc = is_max ? -INFINITY : 0.f;
        int cnt = 0;
        for (int i = 0; i < kh; ++i)
          for (int j = 0; j < kw; ++j) {
            const int ih = oh * sh - ph + i, iw = ow * sw - pw + j;
            if (ih < 0 || ih >= h || iw < 0 || iw >= w) continue;
            const float v = xp[(size_t)ih * w + iw];
            acc = is_max ? std::max(acc, v) : acc + v;
            ++cnt;
          }
        yp[(size_t)oh * wo + ow] = cnt == 0 ? 0.f : (is_max ? acc : acc / (float)cnt);
      }
  }
  return 0;
}
AE_API int aether_op_max_pool_2d_f32(const void* x, void* y, int n, int c, int h, int w, int kh, int kw, int sh, int sw,
                                     int ph, int pw) {
  return pool2d(x, y, n, c, h, w, kh, kw, sh, sw, ph, pw, true);
}
AE_API int aether_op_avg_pool_2d_f32(const void* x, void* y, int n, int c, int h, int w, int kh, int kw, int sh, int sw,
                                     int ph, int pw) {
  return pool2d(x, y, n, c, h, w, kh, kw, sh, sw, ph, pw, false);
}
AE_API int aether_op_adaptive_avg_pool_2d_f32(const void* x, void* y, int n, int c, int h, int w, int ho, int wo) {
  if (!x || !y || ho <= 0 || wo <= 0) return -1;
  for (int p = 0; p < n * c; ++p)
    for (int oh = 0; oh < ho; ++oh)
      for (int ow = 0; ow < wo; ++ow) {
        const int h0 = oh * h / ho, h1 = (oh + 1) * h / ho, w0 = ow * w / wo, w1 = (ow + 1) * w / wo;
        double s = 0;
        int cnt = 0;
        for (int i = h0; i < h1; ++i)
          for (int j = w0; j < w1; ++j) {
            s += CF(x)[((size_t)p * h + i) * w + j];
            ++cnt;
          }
        F(y)[((size_t)p * ho + oh) * wo + ow] = cnt ? (float)(s / cnt) : 0.f;
      }
  return 0;
}
// mode 0 = sum, 1 = mean; out-of-range indices are skipped.
AE_API int aether_op_embedding_bag_f32(const void* weight, const void* indices, const void* offsets, void* out,
                                       int n_bags, int vocab, int dim, int total_idx, int mode) {
  if (!weight || !indices || !offsets || !out) return -1;
  const int* idx = static_cast<const int*>(indices);
  const int* off = static_cast<const int*>(offsets);
  for (int bag = 0; bag < n_bags; ++bag) {
    float* o = F(out) + (size_t)bag * dim;
    std::fill(o, o + dim, 0.f);
    const int lo = off[bag], hi = std::min(off[bag + 1], total_idx);
    for (int k = lo; k < hi; ++k) {
      const int r = idx[k];
      if (r < 0 || r >= vocab) continue;
      const float* wr = CF(weight) + (size_t)r * dim;
      for (int d = 0; d < dim; ++d) o[d] += wr[d];
    }
    if (mode == 1 && hi > lo)
      for (int d = 0; d < dim; ++d) o[d] /= (float)(hi - lo);
  }
  return 0;
}

// ------------------------------------------------------------------ dtype conversions
// bf16 / f16 values travel in the low 16 bits of an int32.
AE_API int aether_f32_to_bf16(float x) {
  uint32_t u;
  std::memcpy(&u, &x, 4);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return (int)((u >> 16) | 0x40u);  // quiet NaN
  u += 0x7fffu + ((u >> 16) & 1u);  // round to nearest even
  return (int)(u >> 16);
}
AE_API float aether_bf16_to_f32(int b) {
  const uint32_t u = (uint32_t)(b & 0xffff) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}
AE_API int aether_f32_to_f16(float x) {
  uint32_t u;
  std::memcpy(&u, &x, 4);
  const uint32_t sign = (u >> 16) & 0x8000u;
  const int32_t exp = (int32_t)((u >> 23) & 0xff) - 127 + 15;
  uint32_t mant = u & 0x7fffffu;
  if (((u >> 23) & 0xff) == 0xff) return (int)(sign | 0x7c00u | (mant ? 0x200u : 0u));
  if (exp >= 31) return (int)(sign | 0x7c00u);  // overflow -> inf
  if (exp <= 0) {                                // subnormal or zero
    if (exp < -10) return (int)sign;
    mant |= 0x800000u;
    const int shift = 14 - exp;
    uint32_t h = mant >> shift;
    const uint32_t rem = mant & ((1u << shift) - 1), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (h & 1u))) ++h;
    return (int)(sign | h);
  }
  uint32_t h = ((uint32_t)exp << 10) | (mant >> 13);
  const uint32_t rem = mant & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;  // may carry into the exponent: still correct
  return (int)(sign | h);
}
AE_API float aether_f16_to_f32(int hbits) {
  const uint32_t h = (uint32_t)hbits & 0xffffu;
  const uint32_t sign = (h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1f, mant = h & 0x3ffu, u;
  if (exp == 0) {
    if (mant == 0) {
      u = sign;
    } else {  // subnormal: normalise
      int e = -1;
      do {
        mant <<= 1;
        ++e;
      } while (!(mant & 0x400u));
      u = sign | ((uint32_t)(127 - 15 - e) << 23) | ((mant & 0x3ffu) << 13);
    }
  } else if (exp == 31) {
    u = sign | 0x7f800000u | (mant << 13);
  } else {
    u = sign | ((exp + 127 - 15) << 23) | (mant << 13);
  }
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}
// a: [m, k] and b: [k, n] bf16 (one per int32 lane), out: [m, n] f32.
AE_API int aether_op_matmul_bf16_f32_out(int64_t a, int64_t b, int64_t out, int m, int k, int n) {
  if (!a || !b || !out || m < 0 || k < 0 || n < 0) return -1;
  const int* A = reinterpret_cast<const int*>(a);
  const int* B = reinterpret_cast<const int*>(b);
  float* C = reinterpret_cast<float*>(out);
  for (int i = 0; i < m; ++i)
    for (int j = 0; j < n; ++j) {
      float s = 0.f;
      for (int t = 0; t < k; ++t) s += aether_bf16_to_f32(A[(size_t)i * k + t]) * aether_bf16_to_f32(B[(size_t)t * n + j]);
      C[(size_t)i * n + j] = s;
    }
  return 0;
}
AE_API int aether_pack_f32_to_bf16(int64_t src, int64_t dst, int n) {
  if (!src || !dst || n < 0) return -1;
  const float* s = reinterpret_cast<const float*>(src);
  int* d = reinterpret_cast<int*>(dst);
  for (int i = 0; i < n; ++i) d[i] = aether_f32_to_bf16(s[i]);
  return 0;
}

// ------------------------------------------------------------------ GGUF block dequantisers (-> f32)
// Return 0 on success, 1 on a null pointer, 2 on a bad block count.
static inline float half_at(const uint8_t* p) { return aether_f16_to_f32(p[0] | (p[1] << 8)); }
// The exported Q4_0 decoder writes each byte's two values next to each other
// (low nibble at 2j, high nibble at 2j + 1), which is the order this ABI
// function has always produced for its callers (runtime/src/lib.rs:217-240);
// GGUF tensors (low nibbles first, then high) are decoded by the loaders'
// own Q4_0 path.
AE_API int aether_dequant_q4_0(const void* blocks, void* out, int n_blocks) {
  if (!blocks || !out) return 1;
  if (n_blocks <= 0) return 2;
  const uint8_t* b = static_cast<const uint8_t*>(blocks);
  for (int i = 0; i < n_blocks; ++i, b += 18) {
    const float d = half_at(b);
    float* o = F(out) + (size_t)i * 32;
    for (int j = 0; j < 16; ++j) {
      o[2 * j] = d * (float)((b[2 + j] & 0x0f) - 8);
      o[2 * j + 1] = d * (float)((b[2 + j] >> 4) - 8);
    }
  }
  return 0;
}
AE_API int aether_dequant_q8_0(const void* blocks, void* out, int n_blocks) {
  if (!blocks || !out) return 1;
  if (n_blocks <= 0) return 2;
  const uint8_t* b = static_cast<const uint8_t*>(blocks);
  for (int i = 0; i < n_blocks; ++i, b += 34) {
    const float d = half_at(b);
    for (int j = 0; j < 32; ++j) F(out)[(size_t)i * 32 + j] = d * (float)(int8_t)b[2 + j];
  }
  return 0;
}
// Q4_K super-block (256 values): f16 d, f16 dmin, 12 bytes of 6-bit (scale, min)
// for 8 sub-blocks of 32, 128 bytes of nibbles.
AE_API int aether_dequant_q4_k_m(const void* blocks, void* out, int n_blocks) {
  if (!blocks || !out) return 1;
  if (n_blocks <= 0) return 2;
  const uint8_t* b = static_cast<const uint8_t*>(blocks);
  for (int i = 0; i < n_blocks; ++i, b += 144) {
    const float d = half_at(b), dmin = half_at(b + 2);
    const uint8_t* sc = b + 4;
    const uint8_t* qs = b + 16;
    float* o = F(out) + (size_t)i * 256;
    for (int sub = 0; sub < 8; ++sub) {
      int s, m;
      if (sub < 4) {
        s = sc[sub] & 63;
        m = sc[sub + 4] & 63;
      } else {
        s = (sc[sub + 4] & 0x0f) | ((sc[sub - 4] >> 6) << 4);
        m = (sc[sub + 4] >> 4) | ((sc[sub] >> 6) << 4);
      }
      const uint8_t* q = qs + (sub / 2) * 32;
      for (int l = 0; l < 32; ++l) {
        const int v = (sub & 1) ? (q[l] >> 4) : (q[l] & 0x0f);
        o[sub * 32 + l] = d * (float)s * (float)v - dmin * (float)m;
      }
    }
  }
  return 0;
}
// Q6_K super-block (256 values): 128 bytes low nibbles, 64 bytes high 2-bit
// pairs, 16 int8 scales, f16 d.
AE_API int aether_dequant_q6_k(const void* blocks, void* out, int n_blocks) {
  if (!blocks || !out) return 1;
  if (n_blocks <= 0) return 2;
  const uint8_t* b = static_cast<const uint8_t*>(blocks);
  for (int i = 0; i < n_blocks; ++i, b += 210) {
    const uint8_t* ql = b;
    const uint8_t* qh = b + 128;
    const int8_t* sc = reinterpret_cast<const int8_t*>(b + 192);
    const float d = half_at(b + 208);
    float* o = F(out) + (size_t)i * 256;
    for (int half = 0; half < 2; ++half) {
      const uint8_t* L = ql + half * 64;
      const uint8_t* H = qh + half * 32;
      for (int l = 0; l < 32; ++l) {
        const int q[4] = {(L[l] & 0xf) | (((H[l] >> 0) & 3) << 4), (L[l + 32] & 0xf) | (((H[l] >> 2) & 3) << 4),
                          (L[l] >> 4) | (((H[l] >> 4) & 3) << 4), (L[l + 32] >> 4) | (((H[l] >> 6) & 3) << 4)};
        for (int part = 0; part < 4; ++part)
          o[half * 128 + part * 32 + l] = d * (float)sc[half * 8 + part * 2 + l / 16] * (float)(q[part] - 32);
      }
    }
  }
  return 0;
}

// Q3_K super-block (256 values): 32 bytes of third bits (a clear bit
// subtracts 4), 64 bytes of 2-bit values, 16 six-bit scales (low nibbles in
// bytes 0..7, high bit pairs in bytes 8..11, offset 32), f16 d. Value e of
// 128-value half h, pair-shift j, sub-block s uses scale h*8 + j*2 + s.
AE_API int aether_dequant_q3_k(const void* blocks, void* out, int n_blocks) {
  if (!blocks || !out) return 1;
  if (n_blocks <= 0) return 2;
  const uint8_t* b = static_cast<const uint8_t*>(blocks);
  for (int i = 0; i < n_blocks; ++i, b += 110) {
    const uint8_t* hm = b;
    const uint8_t* qs = b + 32;
    const uint8_t* raw = b + 96;
    const float d = half_at(b + 108);
    int sc[16];
    for (int k = 0; k < 16; ++k)
      sc[k] = (((raw[k % 8] >> (4 * (k / 8))) & 0xf) | (((raw[8 + k % 4] >> (2 * (k / 4))) & 3) << 4)) - 32;
    float* o = F(out) + (size_t)i * 256;
    for (int half = 0; half < 2; ++half)
      for (int j = 0; j < 4; ++j)
        for (int l = 0; l < 32; ++l) {
          int q = (qs[half * 32 + l] >> (2 * j)) & 3;
          if (!((hm[l] >> (half * 4 + j)) & 1)) q -= 4;
          o[half * 128 + j * 32 + l] = d * (float)sc[half * 8 + j * 2 + l / 16] * (float)q;
        }
  }
  return 0;
}

// ------------------------------------------------------------------ paged-KV block pool + page tables
struct Pool {
  std::vector<uint8_t> used;
  std::vector<uint64_t> stamp;
  uint64_t tick = 0;
  int block_size = 0;
};
struct PageTbl {
  std::vector<int> blocks;
};
static Table<Pool> g_pools;
static Table<PageTbl> g_tables;

AE_API int64_t aether_pkv_new(int n_blocks, int block_size) {
  if (n_blocks <= 0 || block_size <= 0) return -1;
  auto p = std::make_unique<Pool>();
  p->used.assign((size_t)n_blocks, 0);
  p->stamp.assign((size_t)n_blocks, 0);
  p->block_size = block_size;
  return g_pools.add(std::move(p));
}
AE_API int aether_pkv_destroy(int64_t h) { return g_pools.drop(h); }
AE_API int aether_pkv_allocate(int64_t h) {
  Pool* p = g_pools.get(h);
  if (!p) return -1;
  for (size_t i = 0; i < p->used.size(); ++i)
    if (!p->used[i]) {
      p->used[i] = 1;
      p->stamp[i] = ++p->tick;
      return (int)i;
    }
  return -1;
}
AE_API int aether_pkv_touch(int64_t h, int block) {
  Pool* p = g_pools.get(h);
  if (!p || block < 0 || (size_t)block >= p->used.size() || !p->used[(size_t)block]) return -1;
  p->stamp[(size_t)block] = ++p->tick;
  return 0;
}
AE_API int aether_pkv_free_block(int64_t h, int block) {
  Pool* p = g_pools.get(h);
  if (!p || block < 0 || (size_t)block >= p->used.size()) return -1;
  p->used[(size_t)block] = 0;
  return 0;
}
AE_API int aether_pkv_evict_lru(int64_t h) {
  Pool* p = g_pools.get(h);
  if (!p) return -1;
  int best = -1;
  for (size_t i = 0; i < p->used.size(); ++i)
    if (p->used[i] && (best < 0 || p->stamp[i] < p->stamp[(size_t)best])) best = (int)i;
  if (best >= 0) p->used[(size_t)best] = 0;
  return best;
}
AE_API int aether_pkv_n_allocated(int64_t h) {
  Pool* p = g_pools.get(h);
  if (!p) return -1;
  return (int)std::count(p->used.begin(), p->used.end(), (uint8_t)1);
}
AE_API int64_t aether_pkv_pagetable_new(int initial_capacity) {
  if (initial_capacity < 0) return -1;
  auto t = std::make_unique<PageTbl>();
  t->blocks.assign((size_t)initial_capacity, -1);
  return g_tables.add(std::move(t));
}
AE_API int aether_pkv_pagetable_set(int64_t h, int logical, int physical) {
  PageTbl* t = g_tables.get(h);
  if (!t || logical < 0) return -1;
  if ((size_t)logical >= t->blocks.size()) t->blocks.resize((size_t)logical + 1, -1);
  t->blocks[(size_t)logical] = physical;
  return 0;
}
AE_API int64_t aether_pkv_pagetable_get(int64_t h, int logical) {
  PageTbl* t = g_tables.get(h);
  if (!t || logical < 0 || (size_t)logical >= t->blocks.size()) return -1;
  return t->blocks[(size_t)logical];
}
AE_API int aether_pkv_pagetable_len(int64_t h) {
  PageTbl* t = g_tables.get(h);
  return t ? (int)t->blocks.size() : -1;
}
AE_API int aether_pkv_pagetable_destroy(int64_t h) { return g_tables.drop(h); }
// token position -> physical_block * block_size + offset (or -1 if unmapped)
AE_API int64_t aether_pkv_pagetable_translate(int64_t h, int token_pos, int block_size) {
  if (token_pos < 0 || block_size <= 0) return -1;
  const int64_t phys = aether_pkv_pagetable_get(h, token_pos / block_size);
  return phys < 0 ? -1 : phys * block_size + token_pos % block_size;
}

// ------------------------------------------------------------------ batch scheduler over a block pool
struct SchedReq {
  int id;
  int64_t table;
  int position = 0, emitted = 0, max_tokens = 0;
  bool finished = false;
  std::vector<int> blocks;
};
struct Sched {
  int64_t pool;
  int block_size, max_active;
  std::vector<SchedReq> reqs;
};
static Table<Sched> g_scheds;

static SchedReq* sched_find(Sched* s, int id) {
  for (auto& r : s->reqs)
    if (r.id == id) return &r;
  return nullptr;
}
AE_API int64_t aether_batch_sched_new(int64_t pool_h, int block_size, int max_active) {
  if (pool_h < 0 || block_size <= 0 || max_active <= 0) return -1;
  auto s = std::make_unique<Sched>();
  s->pool = pool_h;
  s->block_size = block_size;
  s->max_active = max_active;
  return g_scheds.add(std::move(s));
}
static void sched_release(Sched* s, SchedReq& r) {
  for (int b : r.blocks) aether_pkv_free_block(s->pool, b);
  aether_pkv_pagetable_destroy(r.table);
}
AE_API int64_t aether_batch_sched_destroy(int64_t h) {
  Sched* s = g_scheds.get(h);
  if (!s) return -1;
  for (auto& r : s->reqs) sched_release(s, r);
  return g_scheds.drop(h);
}
// 0 admitted, -1 at capacity / bad args, -2 block pool exhausted (rolled back)
AE_API int64_t aether_batch_sched_admit(int64_t h, int req_id, int prompt_len, int max_tokens) {
  Sched* s = g_scheds.get(h);
  if (!s || prompt_len < 0 || max_tokens < 0 || (int)s->reqs.size() >= s->max_active) return -1;
  const int total = prompt_len + max_tokens;
  SchedReq r;
  r.id = req_id;
  r.max_tokens = max_tokens;
  r.table = aether_pkv_pagetable_new(std::max(1, (total + s->block_size - 1) / s->block_size));
  if (r.table < 0) return -2;
  const int now = std::max(1, (prompt_len + s->block_size - 1) / s->block_size);
  for (int l = 0; l < now; ++l) {
    const int phys = aether_pkv_allocate(s->pool);
    if (phys < 0) {
      sched_release(s, r);
      return -2;
    }
    aether_pkv_pagetable_set(r.table, l, phys);
    r.blocks.push_back(phys);
  }
  r.position = 0;  // counts emitted tokens from admission (the reference ABI's contract)
  s->reqs.push_back(std::move(r));
  return 0;
}
AE_API int64_t aether_batch_sched_record_token(int64_t h, int req_id, int /*new_token*/) {
  Sched* s = g_scheds.get(h);
  SchedReq* r = s ? sched_find(s, req_id) : nullptr;
  if (!r) return -1;
  if (r->finished) return 0;
  ++r->position;
  ++r->emitted;
  const int logical = r->position / s->block_size;
  if (aether_pkv_pagetable_get(r->table, logical) < 0) {
    const int phys = aether_pkv_allocate(s->pool);
    if (phys < 0) return -2;
    aether_pkv_pagetable_set(r->table, logical, phys);
    r->blocks.push_back(phys);
  }
  if (r->emitted >= r->max_tokens) r->finished = true;
  return 0;
}
AE_API int64_t aether_batch_sched_finish(int64_t h, int req_id) {
  Sched* s = g_scheds.get(h);
  SchedReq* r = s ? sched_find(s, req_id) : nullptr;
  if (!r) return -1;
  r->finished = true;
  return 0;
}
AE_API int64_t aether_batch_sched_reap(int64_t h) {
  Sched* s = g_scheds.get(h);
  if (!s) return -1;
  int64_t n = 0;
  for (auto it = s->reqs.begin(); it != s->reqs.end();) {
    if (it->finished) {
      sched_release(s, *it);
      it = s->reqs.erase(it);
      ++n;
    } else {
      ++it;
    }
  }
  return n;
}
AE_API int64_t aether_batch_sched_n_active(int64_t h) {
  Sched* s = g_scheds.get(h);
  return s ? (int64_t)s->reqs.size() : -1;
}
AE_API int64_t aether_batch_sched_pagetable_for(int64_t h, int req_id) {
  Sched* s = g_scheds.get(h);
  SchedReq* r = s ? sched_find(s, req_id) : nullptr;
  return r ? r->table : -1;
}
AE_API int64_t aether_batch_sched_position(int64_t h, int req_id) {
  Sched* s = g_scheds.get(h);
  SchedReq* r = s ? sched_find(s, req_id) : nullptr;
  return r ? r->position : -1;
}

// ------------------------------------------------------------------ continuous batch
struct CB {
  int capacity;
  std::vector<std::pair<int, int>> active;  // (request, steps)
};
static Table<CB> g_cbs;
AE_API int64_t aether_cb_new(int capacity) {
  if (capacity <= 0) return -1;
  auto c = std::make_unique<CB>();
  c->capacity = capacity;
  return g_cbs.add(std::move(c));
}
AE_API int aether_cb_destroy(int64_t h) { return g_cbs.drop(h); }
AE_API int aether_cb_admit(int64_t h, int req_id) {
  CB* c = g_cbs.get(h);
  if (!c || (int)c->active.size() >= c->capacity) return -1;
  c->active.emplace_back(req_id, 0);
  return 0;
}
AE_API int aether_cb_step(int64_t h) {
  CB* c = g_cbs.get(h);
  if (!c) return -1;
  for (auto& a : c->active) ++a.second;
  return (int)c->active.size();
}
AE_API int aether_cb_complete(int64_t h, int req_id) {
  CB* c = g_cbs.get(h);
  if (!c) return -1;
  for (auto it = c->active.begin(); it != c->active.end(); ++it)
    if (it->first == req_id) {
      c->active.erase(it);
      return 0;
    }
  return -1;
}
AE_API int aether_cb_n_active(int64_t h) {
  CB* c = g_cbs.get(h);
  return c ? (int)c->active.size() : -1;
}

// Speculative decoding: accept a draft token with probability min(1, p_target / p_draft).
AE_API int aether_specdec_accept(float target_prob, float draft_prob, float u) {
  if (draft_prob <= 0.f || target_prob < 0.f || !(u >= 0.f && u < 1.f)) return -1;
  const float ratio = target_prob / draft_prob;
  return (ratio >= 1.f || u < ratio) ? 1 : 0;
}

// ------------------------------------------------------------------ multi-model registry
struct Registry {
  std::vector<std::pair<std::string, int>> models;
};
static Table<Registry> g_regs;
AE_API int64_t aether_mm_new() { return g_regs.add(std::make_unique<Registry>()); }
AE_API int aether_mm_destroy(int64_t h) { return g_regs.drop(h); }
AE_API int aether_mm_register(int64_t h, const void* name, int n_name, int vram_mb) {
  Registry* r = g_regs.get(h);
  if (!r || !name || n_name < 0) return -1;
  r->models.emplace_back(std::string(static_cast<const char*>(name), (size_t)n_name), vram_mb);
  return (int)r->models.size() - 1;
}
AE_API int aether_mm_lookup(int64_t h, const void* name, int n_name) {
  Registry* r = g_regs.get(h);
  if (!r || !name || n_name < 0) return -1;
  const std::string key(static_cast<const char*>(name), (size_t)n_name);
  for (size_t i = 0; i < r->models.size(); ++i)
    if (r->models[i].first == key) return (int)i;
  return -1;
}
AE_API int aether_mm_total_vram_mb(int64_t h) {
  Registry* r = g_regs.get(h);
  if (!r) return -1;
  int s = 0;
  for (auto& m : r->models) s += m.second;
  return s;
}

// ------------------------------------------------------------------ rate limiter (token bucket per key)
struct Limiter {
  double rate, burst;
  std::map<std::string, std::pair<double, int64_t>> buckets;  // key -> (tokens, last_us)
};
static Table<Limiter> g_rls;
AE_API int64_t aether_rl_new(int req_per_sec, int burst) {
  if (req_per_sec <= 0 || burst <= 0) return -1;
  auto l = std::make_unique<Limiter>();
  l->rate = req_per_sec;
  l->burst = burst;
  return g_rls.add(std::move(l));
}
AE_API int aether_rl_destroy(int64_t h) { return g_rls.drop(h); }
// 1 allowed, 0 limited, -1 bad arguments
AE_API int aether_rl_check(int64_t h, const void* key, int n_key, int64_t now_us) {
  Limiter* l = g_rls.get(h);
  if (!l || !key || n_key <= 0) return -1;
  auto& b = l->buckets.try_emplace(std::string(static_cast<const char*>(key), (size_t)n_key), l->burst, now_us)
                .first->second;
  b.first = std::min(l->burst, b.first + (double)std::max<int64_t>(0, now_us - b.second) * 1e-6 * l->rate);
  b.second = now_us;
  if (b.first >= 1.0) {
    b.first -= 1.0;
    return 1;
  }
  return 0;
}

// ------------------------------------------------------------------ observability
static std::mutex g_obs_mu;
static std::map<std::string, uint64_t> g_counters;  // sorted: stable Prometheus output
AE_API int aether_obs_counter_inc(const void* name, int n_name, int by) {
  if (!name || n_name <= 0 || by < 0) return -1;
  std::lock_guard<std::mutex> g(g_obs_mu);
  g_counters[std::string(static_cast<const char*>(name), (size_t)n_name)] += (uint64_t)by;
  return 0;
}
AE_API int64_t aether_obs_counter_get(const void* name, int n_name) {
  if (!name || n_name <= 0) return -1;
  std::lock_guard<std::mutex> g(g_obs_mu);
  auto it = g_counters.find(std::string(static_cast<const char*>(name), (size_t)n_name));
  return it == g_counters.end() ? 0 : (int64_t)it->second;
}
// Writes "# TYPE <name> counter\n<name> <value>\n" per counter; returns the
// bytes written (output truncated to max_out) or -1.
AE_API int aether_obs_dump_prometheus(void* out, int max_out) {
  if (!out || max_out <= 0) return -1;
  std::string s;
  {
    std::lock_guard<std::mutex> g(g_obs_mu);
    for (auto& kv : g_counters)
      s += "# TYPE " + kv.first + " counter\n" + kv.first + " " + std::to_string(kv.second) + "\n";
  }
  const int n = (int)std::min<size_t>(s.size(), (size_t)max_out);
  std::memcpy(out, s.data(), (size_t)n);
  return n;
}

static std::atomic<int64_t> g_gpu_live{0}, g_oom{0};
AE_API int64_t aether_gpu_alloc_track(int64_t bytes) { return g_gpu_live += bytes; }
AE_API int64_t aether_gpu_free_track(int64_t bytes) { return g_gpu_live -= bytes; }
AE_API int64_t aether_gpu_live_bytes() { return g_gpu_live.load(); }
AE_API int64_t aether_oom_signal(int64_t flag) {
  g_oom.store(flag);
  return g_oom.load();
}
AE_API int64_t aether_oom_check() { return g_oom.load(); }

// crash_<pid>_<step>.dump in the working directory: label, pid, step, tracked
// device bytes, OOM flag.
AE_API int aether_crash_dump(const uint8_t* label, int64_t label_len, int64_t step) {
  if (!label || label_len <= 0) return -1;
  char path[64];
  std::snprintf(path, sizeof(path), "crash_%d_%lld.dump", (int)getpid(), (long long)step);
  FILE* f = std::fopen(path, "w");
  if (!f) return -2;
  std::fprintf(f, "label=%.*s\npid=%d\nstep=%lld\ngpu_live_bytes=%lld\noom_flag=%lld\n", (int)label_len,
               reinterpret_cast<const char*>(label), (int)getpid(), (long long)step,
               (long long)aether_gpu_live_bytes(), (long long)aether_oom_check());
  std::fclose(f);
  return 0;
}

static std::atomic<int64_t> g_alloc_total{0}, g_alloc_live{0}, g_alloc_peak{0};
void aether_prof_note_alloc(int64_t bytes) {  // called by aether_alloc_* in abi.cpp
  g_alloc_total += bytes;
  const int64_t live = g_alloc_live += bytes;
  int64_t peak = g_alloc_peak.load();
  while (live > peak && !g_alloc_peak.compare_exchange_weak(peak, live)) {
  }
}
void aether_prof_note_free(int64_t bytes) { g_alloc_live -= bytes; }
AE_API int64_t aether_prof_alloc_total() { return g_alloc_total.load(); }
AE_API int64_t aether_prof_alloc_live() { return g_alloc_live.load(); }
AE_API int64_t aether_prof_alloc_peak() { return g_alloc_peak.load(); }
AE_API int aether_prof_reset() {
  g_alloc_total = 0;
  g_alloc_peak = g_alloc_live.load();
  return 0;
}
AE_API int64_t aether_timer_start() {
  return std::chrono::duration_cast<std::chrono::microseconds>(std::chrono::steady_clock::now().time_since_epoch())
      .count();
}
AE_API int64_t aether_timer_elapsed_us(int64_t start) { return aether_timer_start() - start; }

// The generic collectives (aether_op_{broadcast,all_gather,reduce_scatter,
// send,recv,all_to_all}_f32) live in collectives.cpp, real across processes.

// ------------------------------------------------------------------ distributed algorithm shapes
// Single-process versions of the parallel layouts, with the reference's
// names and argument order (runtime/src/lib.rs:3418-3650). Their real
// multi-GPU counterparts are the torch.distributed engines of the Python
// package (tensor / pipeline / ZeRO-2/3 / PowerSGD); these check a layout's
// arithmetic on the host.

// Column-parallel linear: W (k x n) split into world column blocks, each
// block's product X W_b written into its columns of out (m x n).
AE_API int aether_tp_simulate_column_parallel_linear_f32(const void* x, const void* w, void* out, int m, int k, int n,
                                                         int world) {
  if (!x || !w || !out) return 1;
  if (m <= 0 || k <= 0 || n <= 0 || world <= 0) return 2;
  if (n % world) return 3;
  const float* X = static_cast<const float*>(x);
  const float* W = static_cast<const float*>(w);
  float* O = static_cast<float*>(out);
  const int nb = n / world;
  for (int b = 0; b < world; ++b)
    for (int r = 0; r < m; ++r)
      for (int c = b * nb; c < (b + 1) * nb; ++c) {
        float acc = 0.f;
        for (int j = 0; j < k; ++j) acc += X[(size_t)r * k + j] * W[(size_t)j * n + c];
        O[(size_t)r * n + c] = acc;
      }
  return 0;
}

// Pipeline of n_blocks affine blocks (y = y * scale[b] + bias[b]) over
// n_stages stages, every micro-batch passing every stage in order.
AE_API int aether_pp_simulate_2stage_forward_f32(const void* input, const void* scales, const void* biases, void* out,
                                                 int microbatches, int d, int n_blocks, int n_stages) {
  if (!input || !scales || !biases || !out) return 1;
  if (microbatches <= 0 || d <= 0 || n_blocks <= 0 || n_stages <= 0) return 2;
  if (n_blocks % n_stages) return 3;
  const float* in = static_cast<const float*>(input);
  const float* sc = static_cast<const float*>(scales);
  const float* bi = static_cast<const float*>(biases);
  float* o = static_cast<float*>(out);
  const size_t n = (size_t)microbatches * d;
  std::vector<float> act(in, in + n);  // the activation that would cross each stage boundary
  const int per = n_blocks / n_stages;
  for (int st = 0; st < n_stages; ++st)
    for (int b = st * per; b < (st + 1) * per; ++b)
      for (size_t i = 0; i < n; ++i) act[i] = act[i] * sc[b] + bi[b];
  std::memcpy(o, act.data(), n * sizeof(float));
  return 0;
}

// Per-rank bytes of fp32 parameters + gradients + two AdamW moments under
// ZeRO stage 1 (moments sharded), 2 (+ gradients) and 3 (+ parameters).
AE_API int64_t aether_zero_simulate_stage_bytes_f32(int n_params, int world, int stage) {
  if (n_params <= 0 || world <= 0) return -1;
  if (stage < 1 || stage > 3) return -2;
  const int64_t p = 4LL * n_params, g = 4LL * n_params, o = 8LL * n_params;
  if (stage == 1) return p + g + o / world;
  if (stage == 2) return p + (g + o) / world;
  return (p + g + o) / world;
}

// Step time with the collective hidden under compute versus run after it.
AE_API int aether_overlap_simulate_overlapped_us(int compute_us, int comm_us) {
  if (compute_us < 0 || comm_us < 0) return -1;
  return std::max(compute_us, comm_us);
}
AE_API int aether_overlap_simulate_serial_us(int compute_us, int comm_us) {
  if (compute_us < 0 || comm_us < 0) return -1;
  return compute_us + comm_us;
}

// Rank-k projection with P = the first k columns of G and Q = the first k
// unit vectors: the reconstruction keeps G's first k columns and zeroes the
// rest ((m + n) k values would travel instead of m n). The PowerSGD engine of
// the Python package is the real compressor.
AE_API int aether_grad_compress_lowrank_f32(const void* grad, void* reconstructed, int m, int n, int k) {
  if (!grad || !reconstructed) return 1;
  if (m <= 0 || n <= 0 || k <= 0) return 2;
  if (k > n) return 3;
  const float* g = static_cast<const float*>(grad);
  float* r = static_cast<float*>(reconstructed);
  for (int i = 0; i < m; ++i)
    for (int j = 0; j < n; ++j) r[(size_t)i * n + j] = j < k ? g[(size_t)i * n + j] : 0.f;
  return 0;
}

// FSDP round trip: shard a flat parameter vector over world ranks and
// all-gather the shards back in rank order.
AE_API int aether_fsdp_simulate_shard_alltoall_f32(const void* params, void* out, int n, int world) {
  if (!params || !out) return 1;
  if (n <= 0 || world <= 0) return 2;
  if (n % world) return 3;
  const float* p = static_cast<const float*>(params);
  float* o = static_cast<float*>(out);
  const int len = n / world;
  std::vector<std::vector<float>> shards((size_t)world);
  for (int r = 0; r < world; ++r) shards[(size_t)r].assign(p + (size_t)r * len, p + (size_t)(r + 1) * len);
  for (int r = 0; r < world; ++r) std::memcpy(o + (size_t)r * len, shards[(size_t)r].data(), len * sizeof(float));
  return 0;
}

}  // extern "C"
