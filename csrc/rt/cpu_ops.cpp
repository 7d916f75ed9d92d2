// fp32 CPU operator bodies (see cpu_ops.h). Loops are ordered for unit-stride
// inner accesses and parallelised over rows with OpenMP.
#include "cpu_ops.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

namespace aether_rt {

void matmul(const float* a, const float* b, float* out, int m, int k, int n) {
  std::memset(out, 0, sizeof(float) * (size_t)m * n);
  matmul_acc(a, b, out, m, k, n);
}

void matmul_acc(const float* a, const float* b, float* out, int m, int k, int n) {
#pragma omp parallel for schedule(static) if ((int64_t)m * k * n > 262144)
  for (int i = 0; i < m; ++i) {
    float* o = out + (size_t)i * n;
    const float* ar = a + (size_t)i * k;
    for (int p = 0; p < k; ++p) {
      const float av = ar[p];
      if (av == 0.f) continue;
      const float* br = b + (size_t)p * n;
      for (int j = 0; j < n; ++j) o[j] += av * br[j];
    }
  }
}

void matmul_bwd_lhs(const float* dy, const float* b, float* da, int m, int k, int n) {
  std::memset(da, 0, sizeof(float) * (size_t)m * k);
  matmul_bwd_lhs_acc(dy, b, da, m, k, n);
}

void matmul_bwd_lhs_acc(const float* dy, const float* b, float* da, int m, int k, int n) {
#pragma omp parallel for schedule(static) if ((int64_t)m * k * n > 262144)
  for (int i = 0; i < m; ++i) {
    const float* d = dy + (size_t)i * n;
    float* o = da + (size_t)i * k;
    for (int p = 0; p < k; ++p) {
      const float* br = b + (size_t)p * n;
      float s = 0.f;
      for (int j = 0; j < n; ++j) s += d[j] * br[j];
      o[p] += s;
    }
  }
}

void matmul_bwd_rhs(const float* a, const float* dy, float* db, int m, int k, int n) {
  std::memset(db, 0, sizeof(float) * (size_t)k * n);
  matmul_bwd_rhs_acc(a, dy, db, m, k, n);
}

void matmul_bwd_rhs_acc(const float* a, const float* dy, float* db, int m, int k, int n) {
#pragma omp parallel for schedule(static) if ((int64_t)m * k * n > 262144)
  for (int p = 0; p < k; ++p) {
    float* o = db + (size_t)p * n;
    for (int i = 0; i < m; ++i) {
      const float av = a[(size_t)i * k + p];
      if (av == 0.f) continue;
      const float* d = dy + (size_t)i * n;
      for (int j = 0; j < n; ++j) o[j] += av * d[j];
    }
  }
}

void matmul_nt(const float* a, const float* b, float* out, int m, int k, int n) {
#pragma omp parallel for schedule(static) if ((int64_t)m * k * n > 262144)
  for (int i = 0; i < m; ++i) {
    const float* ar = a + (size_t)i * k;
    for (int j = 0; j < n; ++j) {
      const float* br = b + (size_t)j * k;
      float s = 0.f;
      for (int p = 0; p < k; ++p) s += ar[p] * br[p];
      out[(size_t)i * n + j] = s;
    }
  }
}

float gelu_tanh(float x) {
  const float c = 0.7978845608028654f;
  return 0.5f * x * (1.f + std::tanh(c * (x + 0.044715f * x * x * x)));
}

float gelu_tanh_grad(float x) {
  const float c = 0.7978845608028654f;
  const float u = c * (x + 0.044715f * x * x * x);
  const float t = std::tanh(u);
  return 0.5f * (1.f + t) + 0.5f * x * (1.f - t * t) * c * (1.f + 3.f * 0.044715f * x * x);
}

void layer_norm(const float* x, const float* g, const float* b, float eps, float* out, float* mean, float* inv,
                int rows, int d) {
#pragma omp parallel for schedule(static) if ((int64_t)rows * d > 65536)
  for (int r = 0; r < rows; ++r) {
    const float* xr = x + (size_t)r * d;
    double s = 0.0;
    for (int i = 0; i < d; ++i) s += xr[i];
    const float mu = (float)(s / d);
    double v = 0.0;
    for (int i = 0; i < d; ++i) v += (double)(xr[i] - mu) * (xr[i] - mu);
    const float is = 1.f / std::sqrt((float)(v / d) + eps);
    if (mean) mean[r] = mu;
    if (inv) inv[r] = is;
    float* o = out + (size_t)r * d;
    for (int i = 0; i < d; ++i) o[i] = (xr[i] - mu) * is * g[i] + (b ? b[i] : 0.f);
  }
}

void layer_norm_bwd(const float* x, const float* g, const float* dy, const float* mean, const float* inv, float* dx,
                    float* dg, float* db, int rows, int d) {
  for (int r = 0; r < rows; ++r) {
    const float* xr = x + (size_t)r * d;
    const float* dr = dy + (size_t)r * d;
    const float mu = mean[r], is = inv[r];
    double sg = 0.0, sgx = 0.0;
    for (int i = 0; i < d; ++i) {
      const float xh = (xr[i] - mu) * is;
      const float gw = dr[i] * g[i];
      sg += gw;
      sgx += gw * xh;
      if (dg) dg[i] += dr[i] * xh;
      if (db) db[i] += dr[i];
    }
    const float mg = (float)(sg / d), mgx = (float)(sgx / d);
    float* o = dx + (size_t)r * d;
    for (int i = 0; i < d; ++i) {
      const float xh = (xr[i] - mu) * is;
      o[i] = is * (dr[i] * g[i] - mg - xh * mgx);
    }
  }
}

void rms_norm(const float* x, const float* g, float eps, float* out, int rows, int d) {
  for (int r = 0; r < rows; ++r) {
    const float* xr = x + (size_t)r * d;
    double s = 0.0;
    for (int i = 0; i < d; ++i) s += (double)xr[i] * xr[i];
    const float is = 1.f / std::sqrt((float)(s / d) + eps);
    for (int i = 0; i < d; ++i) out[(size_t)r * d + i] = xr[i] * is * g[i];
  }
}

void softmax_rows(float* x, int rows, int cols) {
  for (int r = 0; r < rows; ++r) {
    float* xr = x + (size_t)r * cols;
    float mx = -INFINITY;
    for (int j = 0; j < cols; ++j) mx = std::max(mx, xr[j]);
    float s = 0.f;
    for (int j = 0; j < cols; ++j) {
      xr[j] = (mx == -INFINITY) ? 0.f : std::exp(xr[j] - mx);
      s += xr[j];
    }
    const float is = s > 0.f ? 1.f / s : 0.f;
    for (int j = 0; j < cols; ++j) xr[j] *= is;
  }
}

void softmax_bwd(const float* y, const float* dy, float* dx, int rows, int cols) {
  for (int r = 0; r < rows; ++r) {
    const float* yr = y + (size_t)r * cols;
    const float* dr = dy + (size_t)r * cols;
    float dot = 0.f;
    for (int j = 0; j < cols; ++j) dot += yr[j] * dr[j];
    for (int j = 0; j < cols; ++j) dx[(size_t)r * cols + j] = yr[j] * (dr[j] - dot);
  }
}

void rope(float* x, int seq, int n_heads, int head_dim, float base, int pos_start) {
  const int half = head_dim / 2;
  for (int t = 0; t < seq; ++t) {
    const float pos = (float)(pos_start + t);
    for (int h = 0; h < n_heads; ++h) {
      float* xr = x + ((size_t)t * n_heads + h) * head_dim;
      for (int i = 0; i < half; ++i) {
        const float theta = pos * std::pow(base, -2.f * i / head_dim);
        const float c = std::cos(theta), s = std::sin(theta);
        const float x0 = xr[i], x1 = xr[i + half];
        xr[i] = x0 * c - x1 * s;
        xr[i + half] = x0 * s + x1 * c;
      }
    }
  }
}

static void sdpa_impl(const float* q, const float* k, const float* v, float* out, float* attn, int bh, int s, int d,
                      bool causal) {
  const float scale = 1.f / std::sqrt((float)d);
#pragma omp parallel for schedule(static) if (bh > 1)
  for (int h = 0; h < bh; ++h) {
    const float* qh = q + (size_t)h * s * d;
    const float* kh = k + (size_t)h * s * d;
    const float* vh = v + (size_t)h * s * d;
    float* ah = attn + (size_t)h * s * s;
    float* oh = out + (size_t)h * s * d;
    for (int i = 0; i < s; ++i) {
      for (int j = 0; j < s; ++j) {
        if (causal && j > i) {
          ah[(size_t)i * s + j] = -INFINITY;
          continue;
        }
        float acc = 0.f;
        for (int e = 0; e < d; ++e) acc += qh[(size_t)i * d + e] * kh[(size_t)j * d + e];
        ah[(size_t)i * s + j] = acc * scale;
      }
    }
    softmax_rows(ah, s, s);
    for (int i = 0; i < s; ++i) {
      float* o = oh + (size_t)i * d;
      for (int e = 0; e < d; ++e) o[e] = 0.f;
      for (int j = 0; j < s; ++j) {
        const float p = ah[(size_t)i * s + j];
        if (p == 0.f) continue;
        for (int e = 0; e < d; ++e) o[e] += p * vh[(size_t)j * d + e];
      }
    }
  }
}

void sdpa_causal(const float* q, const float* k, const float* v, float* out, float* attn, int bh, int s, int d) {
  sdpa_impl(q, k, v, out, attn, bh, s, d, true);
}

void sdpa_full(const float* q, const float* k, const float* v, float* out, float* attn, int bh, int s, int d) {
  sdpa_impl(q, k, v, out, attn, bh, s, d, false);
}

void sdpa_causal_bwd(const float* q, const float* k, const float* v, const float* attn, const float* dout, float* dq,
                     float* dk, float* dv, int bh, int s, int d) {
  const float scale = 1.f / std::sqrt((float)d);
#pragma omp parallel for schedule(static) if (bh > 1)
  for (int h = 0; h < bh; ++h) {
    const float* qh = q + (size_t)h * s * d;
    const float* kh = k + (size_t)h * s * d;
    const float* vh = v + (size_t)h * s * d;
    const float* ah = attn + (size_t)h * s * s;
    const float* doh = dout + (size_t)h * s * d;
    float* dqh = dq + (size_t)h * s * d;
    float* dkh = dk + (size_t)h * s * d;
    float* dvh = dv + (size_t)h * s * d;
    std::fill(dqh, dqh + (size_t)s * d, 0.f);
    std::fill(dkh, dkh + (size_t)s * d, 0.f);
    std::fill(dvh, dvh + (size_t)s * d, 0.f);
    std::vector<float> dp(s), ds(s);
    for (int i = 0; i < s; ++i) {
      const float* a = ah + (size_t)i * s;
      // dV += P^T dO ; dP = dO V^T
      float dot = 0.f;
      for (int j = 0; j <= i; ++j) {
        const float p = a[j];
        float acc = 0.f;
        for (int e = 0; e < d; ++e) {
          dvh[(size_t)j * d + e] += p * doh[(size_t)i * d + e];
          acc += doh[(size_t)i * d + e] * vh[(size_t)j * d + e];
        }
        dp[j] = acc;
        dot += p * acc;
      }
      for (int j = 0; j <= i; ++j) ds[j] = a[j] * (dp[j] - dot) * scale;
      for (int j = 0; j <= i; ++j) {
        for (int e = 0; e < d; ++e) {
          dqh[(size_t)i * d + e] += ds[j] * kh[(size_t)j * d + e];
          dkh[(size_t)j * d + e] += ds[j] * qh[(size_t)i * d + e];
        }
      }
    }
  }
}

float cross_entropy(const float* logits, const int32_t* labels, float* probs, int b, int v) {
  double total = 0.0;
  for (int i = 0; i < b; ++i) {
    const float* l = logits + (size_t)i * v;
    float* p = probs + (size_t)i * v;
    float mx = l[0];
    for (int j = 1; j < v; ++j) mx = std::max(mx, l[j]);
    float s = 0.f;
    for (int j = 0; j < v; ++j) {
      p[j] = std::exp(l[j] - mx);
      s += p[j];
    }
    const float is = 1.f / s;
    for (int j = 0; j < v; ++j) p[j] *= is;
    const float pl = std::max(p[labels[i]], 1e-12f);
    total += -std::log((double)pl);
  }
  return (float)(total / b);
}

void cross_entropy_bwd(const float* probs, const int32_t* labels, float* dlogits, int b, int v) {
  const float ib = 1.f / (float)b;
  for (int i = 0; i < b; ++i) {
    for (int j = 0; j < v; ++j) dlogits[(size_t)i * v + j] = probs[(size_t)i * v + j] * ib;
    dlogits[(size_t)i * v + labels[i]] -= ib;
  }
}

float clip_grad_norm(float* g, float max_norm, size_t n) {
  double sq = 0.0;
  for (size_t i = 0; i < n; ++i) sq += (double)g[i] * g[i];
  const float norm = (float)std::sqrt(sq);
  if (norm > max_norm && norm > 0.f) {
    const float sc = max_norm / norm;
    for (size_t i = 0; i < n; ++i) g[i] *= sc;
  }
  return norm;
}

void adamw(float* p, const float* g, float* m, float* v, float lr, float b1, float b2, float eps, float wd,
           int64_t step, size_t n) {
  const float bc1 = 1.f / (1.f - std::pow(b1, (float)step));
  const float bc2 = 1.f / (1.f - std::pow(b2, (float)step));
  for (size_t i = 0; i < n; ++i) {
    m[i] = b1 * m[i] + (1.f - b1) * g[i];
    v[i] = b2 * v[i] + (1.f - b2) * g[i] * g[i];
    const float mh = m[i] * bc1, vh = v[i] * bc2;
    p[i] -= lr * (mh / (std::sqrt(vh) + eps) + wd * p[i]);
  }
}

// Blockwise causal attention with an online softmax (64-row x 64-column
// blocks): the memory-light formulation, equal to sdpa_causal up to rounding.
void flash_attention_v2(const float* q, const float* k, const float* v, float* out, int s, int d) {
  const int B = 64;
  const float scale = 1.f / std::sqrt((float)d);
  std::vector<float> acc((size_t)B * d), mrow(B), lrow(B), sc(B);
  for (int i0 = 0; i0 < s; i0 += B) {
    const int ib = std::min(B, s - i0);
    std::fill(acc.begin(), acc.end(), 0.f);
    std::fill(mrow.begin(), mrow.end(), -INFINITY);
    std::fill(lrow.begin(), lrow.end(), 0.f);
    for (int j0 = 0; j0 <= i0 + ib - 1 && j0 < s; j0 += B) {
      const int jb = std::min(B, s - j0);
      for (int r = 0; r < ib; ++r) {
        const int i = i0 + r;
        float mx = -INFINITY;
        for (int c = 0; c < jb; ++c) {
          const int j = j0 + c;
          if (j > i) {
            sc[c] = -INFINITY;
            continue;
          }
          float a = 0.f;
          for (int e = 0; e < d; ++e) a += q[(size_t)i * d + e] * k[(size_t)j * d + e];
          sc[c] = a * scale;
          mx = std::max(mx, sc[c]);
        }
        if (mx == -INFINITY) continue;
        const float mn = std::max(mrow[r], mx);
        const float al = std::exp(mrow[r] - mn);
        float ls = 0.f;
        for (int e = 0; e < d; ++e) acc[(size_t)r * d + e] *= al;
        for (int c = 0; c < jb; ++c) {
          if (sc[c] == -INFINITY) continue;
          const float p = std::exp(sc[c] - mn);
          ls += p;
          for (int e = 0; e < d; ++e) acc[(size_t)r * d + e] += p * v[(size_t)(j0 + c) * d + e];
        }
        lrow[r] = lrow[r] * al + ls;
        mrow[r] = mn;
      }
    }
    for (int r = 0; r < ib; ++r)
      for (int e = 0; e < d; ++e) out[(size_t)(i0 + r) * d + e] = acc[(size_t)r * d + e] / lrow[r];
  }
}

}  // namespace aether_rt
