// AetherLM-Nano / -Tiny: the reference trainer's model, trained in fp32 on the
// CPU, with its checkpoint format.
//
// Reference: trainer/src/{config,model,rng,data,sample,main}.rs. Kept alike on
// purpose (so checkpoints and runs are interchangeable):
//   * parameter layout and order of the flat arena (model.rs:14-130) --
//     tok_emb, pos_emb, per block {ln1 g/b, W_qkv [D,3D] + b, W_o + b, ln2 g/b,
//     W_fc1 [D,F] + b, W_fc2 [F,D] + b}, ln_f g/b -- and its init (N(0,0.02),
//     residual projections scaled by 1/sqrt(2L), LN gains 1);
//   * SplitMix64 + Box-Muller RNG (rng.rs) so a seed gives the same weights;
//   * pre-LN GPT block, GELU MLP, learned positions, causal SDPA, tied LM head;
//   * `.weights` = "AETHER01\n" + u64 LE count + raw f32 LE, `.meta` one-line JSON.
// The synthetic corpus is the benchmark's: uniform-random words from a fixed
// seeded vocabulary of lowercase ASCII words, space separated.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <sstream>
#include <string>
#include <vector>

#include "cpu_ops.h"

namespace aether_rt {

struct Rng {
  uint64_t state;
  explicit Rng(uint64_t seed) : state(seed + 0x9E3779B97F4A7C15ull) {}
  uint64_t next_u64() {
    state += 0x9E3779B97F4A7C15ull;
    uint64_t z = state;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
  }
  float next_f32() { return (float)(next_u64() >> 40) / (float)(1ull << 24); }
  float next_normal() {
    for (;;) {
      const float u = next_f32();
      if (u > 1e-10f) {
        const float v = next_f32();
        return std::sqrt(-2.f * std::log(u)) * std::cos(2.f * 3.14159265358979f * v);
      }
    }
  }
  size_t gen_range(size_t hi) { return (size_t)(next_u64() % hi); }
};

struct NanoConfig {
  int vocab, d, L, H, F, S;
};

struct BlockLayout {
  size_t ln1g, ln1b, wqkv, bqkv, wo, bo, ln2g, ln2b, w1, b1, w2, b2;
};

struct BlockAct {
  std::vector<float> x_in, ln1, mean1, inv1, qkv, q, k, v, attn, ao, ao_m, x_mid, ln2, mean2, inv2, fc1, g, x_out;
};

class Nano {
 public:
  NanoConfig c;
  size_t tok, pos, lnfg, lnfb, total;
  std::vector<BlockLayout> blk;
  std::vector<float> p, g, m, v;
  // activations of the last forward
  int B = 0;
  std::vector<BlockAct> acts;
  std::vector<float> x0, xf, lnf, meanf, invf, logits, probs;

  Nano(NanoConfig cfg, uint64_t seed) : c(cfg) {
    size_t off = 0;
    auto take = [&](size_t n) {
      size_t r = off;
      off += n;
      return r;
    };
    tok = take((size_t)c.vocab * c.d);
    pos = take((size_t)c.S * c.d);
    for (int l = 0; l < c.L; ++l) {
      BlockLayout b;
      b.ln1g = take(c.d);
      b.ln1b = take(c.d);
      b.wqkv = take((size_t)c.d * 3 * c.d);
      b.bqkv = take(3 * c.d);
      b.wo = take((size_t)c.d * c.d);
      b.bo = take(c.d);
      b.ln2g = take(c.d);
      b.ln2b = take(c.d);
      b.w1 = take((size_t)c.d * c.F);
      b.b1 = take(c.F);
      b.w2 = take((size_t)c.F * c.d);
      b.b2 = take(c.d);
      blk.push_back(b);
    }
    lnfg = take(c.d);
    lnfb = take(c.d);
    total = off;
    p.assign(total, 0.f);
    g.assign(total, 0.f);
    m.assign(total, 0.f);
    v.assign(total, 0.f);
    Rng rng(seed);
    auto normal = [&](size_t o, size_t n, float std) {
      for (size_t i = 0; i < n; ++i) p[o + i] = rng.next_normal() * std;
    };
    auto fill = [&](size_t o, size_t n, float val) {
      for (size_t i = 0; i < n; ++i) p[o + i] = val;
    };
    normal(tok, (size_t)c.vocab * c.d, 0.02f);
    normal(pos, (size_t)c.S * c.d, 0.02f);
    const float rs = 0.02f / std::sqrt(2.f * c.L);
    for (auto& b : blk) {
      fill(b.ln1g, c.d, 1.f);
      fill(b.ln1b, c.d, 0.f);
      normal(b.wqkv, (size_t)c.d * 3 * c.d, 0.02f);
      fill(b.bqkv, 3 * c.d, 0.f);
      normal(b.wo, (size_t)c.d * c.d, rs);
      fill(b.bo, c.d, 0.f);
      fill(b.ln2g, c.d, 1.f);
      fill(b.ln2b, c.d, 0.f);
      normal(b.w1, (size_t)c.d * c.F, 0.02f);
      fill(b.b1, c.F, 0.f);
      normal(b.w2, (size_t)c.F * c.d, rs);
      fill(b.b2, c.d, 0.f);
    }
    fill(lnfg, c.d, 1.f);
    fill(lnfb, c.d, 0.f);
  }

  // ids/labels: [B, S]; returns mean CE (labels == nullptr: logits only)
  float forward(const int32_t* ids, const int32_t* labels, int Bn, int S) {
    B = Bn;
    const int d = c.d, H = c.H, hd = d / H, T = B * S;
    x0.assign((size_t)T * d, 0.f);
    for (int b = 0; b < B; ++b)
      for (int s = 0; s < S; ++s) {
        const int id = ids[b * S + s];
        for (int i = 0; i < d; ++i)
          x0[((size_t)b * S + s) * d + i] = p[tok + (size_t)id * d + i] + p[pos + (size_t)s * d + i];
      }
    acts.assign(c.L, BlockAct());
    std::vector<float> x = x0;
    for (int l = 0; l < c.L; ++l) {
      const BlockLayout& bl = blk[l];
      BlockAct& a = acts[l];
      a.x_in = x;
      a.ln1.resize((size_t)T * d);
      a.mean1.resize(T);
      a.inv1.resize(T);
      layer_norm(x.data(), &p[bl.ln1g], &p[bl.ln1b], 1e-5f, a.ln1.data(), a.mean1.data(), a.inv1.data(), T, d);
      a.qkv.resize((size_t)T * 3 * d);
      matmul(a.ln1.data(), &p[bl.wqkv], a.qkv.data(), T, d, 3 * d);
      for (int t = 0; t < T; ++t)
        for (int i = 0; i < 3 * d; ++i) a.qkv[(size_t)t * 3 * d + i] += p[bl.bqkv + i];
      // split into [B*H, S, hd]
      a.q.resize((size_t)T * d);
      a.k.resize((size_t)T * d);
      a.v.resize((size_t)T * d);
      for (int b = 0; b < B; ++b)
        for (int s = 0; s < S; ++s)
          for (int h = 0; h < H; ++h)
            for (int e = 0; e < hd; ++e) {
              const size_t src = ((size_t)b * S + s) * 3 * d + (size_t)h * hd + e;
              const size_t dst = (((size_t)b * H + h) * S + s) * hd + e;
              a.q[dst] = a.qkv[src];
              a.k[dst] = a.qkv[src + d];
              a.v[dst] = a.qkv[src + 2 * d];
            }
      a.attn.resize((size_t)B * H * S * S);
      a.ao.resize((size_t)T * d);
      sdpa_causal(a.q.data(), a.k.data(), a.v.data(), a.ao.data(), a.attn.data(), B * H, S, hd);
      a.ao_m.resize((size_t)T * d);  // merged heads [B, S, D]
      for (int b = 0; b < B; ++b)
        for (int h = 0; h < H; ++h)
          for (int s = 0; s < S; ++s)
            for (int e = 0; e < hd; ++e)
              a.ao_m[((size_t)b * S + s) * d + (size_t)h * hd + e] = a.ao[(((size_t)b * H + h) * S + s) * hd + e];
      a.x_mid.resize((size_t)T * d);
      matmul(a.ao_m.data(), &p[bl.wo], a.x_mid.data(), T, d, d);
      for (size_t t = 0; t < (size_t)T; ++t)
        for (int i = 0; i < d; ++i) a.x_mid[t * d + i] += p[bl.bo + i] + x[t * d + i];
      a.ln2.resize((size_t)T * d);
      a.mean2.resize(T);
      a.inv2.resize(T);
      layer_norm(a.x_mid.data(), &p[bl.ln2g], &p[bl.ln2b], 1e-5f, a.ln2.data(), a.mean2.data(), a.inv2.data(), T, d);
      a.fc1.resize((size_t)T * c.F);
      matmul(a.ln2.data(), &p[bl.w1], a.fc1.data(), T, d, c.F);
      a.g.resize((size_t)T * c.F);
      for (size_t t = 0; t < (size_t)T; ++t)
        for (int i = 0; i < c.F; ++i) {
          a.fc1[t * c.F + i] += p[bl.b1 + i];
          a.g[t * c.F + i] = gelu_tanh(a.fc1[t * c.F + i]);
        }
      a.x_out.resize((size_t)T * d);
      matmul(a.g.data(), &p[bl.w2], a.x_out.data(), T, c.F, d);
      for (size_t t = 0; t < (size_t)T; ++t)
        for (int i = 0; i < d; ++i) a.x_out[t * d + i] += p[bl.b2 + i] + a.x_mid[t * d + i];
      x = a.x_out;
    }
    xf = x;
    lnf.resize((size_t)T * d);
    meanf.resize(T);
    invf.resize(T);
    layer_norm(x.data(), &p[lnfg], &p[lnfb], 1e-5f, lnf.data(), meanf.data(), invf.data(), T, d);
    logits.resize((size_t)T * c.vocab);
    matmul_nt(lnf.data(), &p[tok], logits.data(), T, d, c.vocab);  // tied head
    if (!labels) return 0.f;
    probs.resize(logits.size());
    return cross_entropy(logits.data(), labels, probs.data(), T, c.vocab);
  }

  void backward(const int32_t* ids, const int32_t* labels, int S) {
    const int d = c.d, H = c.H, hd = d / H, T = B * S;
    std::fill(g.begin(), g.end(), 0.f);
    std::vector<float> dlog((size_t)T * c.vocab);
    cross_entropy_bwd(probs.data(), labels, dlog.data(), T, c.vocab);
    // logits = lnf tok^T : dlnf = dlog tok ; dtok += dlog^T lnf
    std::vector<float> dlnf((size_t)T * d);
    matmul(dlog.data(), &p[tok], dlnf.data(), T, c.vocab, d);
    matmul_bwd_rhs_acc(dlog.data(), lnf.data(), &g[tok], T, c.vocab, d);
    std::vector<float> dx((size_t)T * d);
    layer_norm_bwd(xf.data(), &p[lnfg], dlnf.data(), meanf.data(), invf.data(), dx.data(), &g[lnfg], &g[lnfb], T, d);
    for (int l = c.L - 1; l >= 0; --l) {
      const BlockLayout& bl = blk[l];
      BlockAct& a = acts[l];
      // x_out = x_mid + g W2 + b2
      std::vector<float> dg((size_t)T * c.F);
      matmul_bwd_lhs(dx.data(), &p[bl.w2], dg.data(), T, c.F, d);
      matmul_bwd_rhs_acc(a.g.data(), dx.data(), &g[bl.w2], T, c.F, d);
      for (size_t t = 0; t < (size_t)T; ++t)
        for (int i = 0; i < d; ++i) g[bl.b2 + i] += dx[t * d + i];
      for (size_t i = 0; i < dg.size(); ++i) dg[i] *= gelu_tanh_grad(a.fc1[i]);
      std::vector<float> dln2((size_t)T * d);
      matmul_bwd_lhs(dg.data(), &p[bl.w1], dln2.data(), T, d, c.F);
      matmul_bwd_rhs_acc(a.ln2.data(), dg.data(), &g[bl.w1], T, d, c.F);
      for (size_t t = 0; t < (size_t)T; ++t)
        for (int i = 0; i < c.F; ++i) g[bl.b1 + i] += dg[t * c.F + i];
      std::vector<float> dmid((size_t)T * d);
      layer_norm_bwd(a.x_mid.data(), &p[bl.ln2g], dln2.data(), a.mean2.data(), a.inv2.data(), dmid.data(),
                     &g[bl.ln2g], &g[bl.ln2b], T, d);
      for (size_t i = 0; i < dmid.size(); ++i) dmid[i] += dx[i];  // residual
      // x_mid = x_in + ao_m Wo + bo
      std::vector<float> dao_m((size_t)T * d);
      matmul_bwd_lhs(dmid.data(), &p[bl.wo], dao_m.data(), T, d, d);
      matmul_bwd_rhs_acc(a.ao_m.data(), dmid.data(), &g[bl.wo], T, d, d);
      for (size_t t = 0; t < (size_t)T; ++t)
        for (int i = 0; i < d; ++i) g[bl.bo + i] += dmid[t * d + i];
      std::vector<float> dao((size_t)T * d), dq((size_t)T * d), dk((size_t)T * d), dv((size_t)T * d);
      for (int b = 0; b < B; ++b)
        for (int h = 0; h < H; ++h)
          for (int s = 0; s < S; ++s)
            for (int e = 0; e < hd; ++e)
              dao[(((size_t)b * H + h) * S + s) * hd + e] = dao_m[((size_t)b * S + s) * d + (size_t)h * hd + e];
      sdpa_causal_bwd(a.q.data(), a.k.data(), a.v.data(), a.attn.data(), dao.data(), dq.data(), dk.data(), dv.data(),
                      B * H, S, hd);
      std::vector<float> dqkv((size_t)T * 3 * d);
      for (int b = 0; b < B; ++b)
        for (int s = 0; s < S; ++s)
          for (int h = 0; h < H; ++h)
            for (int e = 0; e < hd; ++e) {
              const size_t dst = ((size_t)b * S + s) * 3 * d + (size_t)h * hd + e;
              const size_t src = (((size_t)b * H + h) * S + s) * hd + e;
              dqkv[dst] = dq[src];
              dqkv[dst + d] = dk[src];
              dqkv[dst + 2 * d] = dv[src];
            }
      std::vector<float> dln1((size_t)T * d);
      matmul_bwd_lhs(dqkv.data(), &p[bl.wqkv], dln1.data(), T, d, 3 * d);
      matmul_bwd_rhs_acc(a.ln1.data(), dqkv.data(), &g[bl.wqkv], T, d, 3 * d);
      for (size_t t = 0; t < (size_t)T; ++t)
        for (int i = 0; i < 3 * d; ++i) g[bl.bqkv + i] += dqkv[t * 3 * d + i];
      std::vector<float> dxin((size_t)T * d);
      layer_norm_bwd(a.x_in.data(), &p[bl.ln1g], dln1.data(), a.mean1.data(), a.inv1.data(), dxin.data(),
                     &g[bl.ln1g], &g[bl.ln1b], T, d);
      for (size_t i = 0; i < dxin.size(); ++i) dx[i] = dxin[i] + dmid[i];
    }
    // embeddings
    for (int b = 0; b < B; ++b)
      for (int s = 0; s < S; ++s) {
        const int id = ids[b * S + s];
        for (int i = 0; i < d; ++i) {
          const float gv = dx[((size_t)b * S + s) * d + i];
          g[tok + (size_t)id * d + i] += gv;
          g[pos + (size_t)s * d + i] += gv;
        }
      }
  }
};

// ------------------------------------------------------------------ corpus
static std::vector<uint8_t> synthetic_words(size_t n_bytes, uint64_t seed, int n_words) {
  Rng rng(seed);
  std::vector<std::string> vocab;
  for (int w = 0; w < n_words; ++w) {
    const int len = 2 + (int)rng.gen_range(6);
    std::string s;
    for (int i = 0; i < len; ++i) s.push_back((char)('a' + rng.gen_range(26)));
    vocab.push_back(s);
  }
  std::vector<uint8_t> out;
  out.reserve(n_bytes + 16);
  while (out.size() < n_bytes) {
    const std::string& w = vocab[rng.gen_range(vocab.size())];
    out.insert(out.end(), w.begin(), w.end());
    out.push_back(' ');
  }
  out.resize(n_bytes);
  return out;
}

static float cosine_lr(int step, int max_steps, float lr_max, int warmup) {
  if (step < warmup) return lr_max * (step + 1) / (float)std::max(1, warmup);
  const float pr = (step - warmup) / (float)std::max(1, max_steps - warmup);
  return lr_max * 0.5f * (1.f + std::cos(3.14159265358979f * pr));
}

}  // namespace aether_rt

using aether_rt::Nano;
using aether_rt::NanoConfig;

extern "C" {

void* aether_nano_create(int vocab, int d_model, int n_layers, int n_heads, int d_ff, int seq_len, uint64_t seed) {
  if (d_model % n_heads != 0) return nullptr;
  return new Nano(NanoConfig{vocab, d_model, n_layers, n_heads, d_ff, seq_len}, seed);
}

void aether_nano_destroy(void* h) { delete static_cast<Nano*>(h); }

int64_t aether_nano_num_params(void* h) { return (int64_t) static_cast<Nano*>(h)->total; }

float* aether_nano_params(void* h) { return static_cast<Nano*>(h)->p.data(); }
float* aether_nano_grads(void* h) { return static_cast<Nano*>(h)->g.data(); }

// One optimiser step on [B, S] ids/labels. Returns the loss before the update.
float aether_nano_train_step(void* h, const int32_t* ids, const int32_t* labels, int B, float lr, float wd,
                             float clip, int64_t step) {
  Nano* n = static_cast<Nano*>(h);
  const float loss = n->forward(ids, labels, B, n->c.S);
  n->backward(ids, labels, n->c.S);
  if (clip > 0.f) aether_rt::clip_grad_norm(n->g.data(), clip, n->total);
  aether_rt::adamw(n->p.data(), n->g.data(), n->m.data(), n->v.data(), lr, 0.9f, 0.95f, 1e-8f, wd, step, n->total);
  return loss;
}

// Data-parallel halves of a step: forward + backward (gradient left in
// aether_nano_grads, loss returned), and the update once the caller has
// replaced the gradient with its mean over ranks.
float aether_nano_forward_backward(void* h, const int32_t* ids, const int32_t* labels, int B) {
  Nano* n = static_cast<Nano*>(h);
  const float loss = n->forward(ids, labels, B, n->c.S);
  n->backward(ids, labels, n->c.S);
  return loss;
}

void aether_nano_apply_update(void* h, float lr, float wd, float clip, int64_t step) {
  Nano* n = static_cast<Nano*>(h);
  if (clip > 0.f) aether_rt::clip_grad_norm(n->g.data(), clip, n->total);
  aether_rt::adamw(n->p.data(), n->g.data(), n->m.data(), n->v.data(), lr, 0.9f, 0.95f, 1e-8f, wd, step, n->total);
}

float aether_nano_loss(void* h, const int32_t* ids, const int32_t* labels, int B) {
  Nano* n = static_cast<Nano*>(h);
  return n->forward(ids, labels, B, n->c.S);
}

// Greedy continuation: ids [len] -> out [max_new]; context is the last seq_len tokens.
int aether_nano_generate(void* h, const int32_t* prompt, int len, int max_new, int32_t* out) {
  Nano* n = static_cast<Nano*>(h);
  std::vector<int32_t> ctx(prompt, prompt + len);
  for (int t = 0; t < max_new; ++t) {
    const int S = n->c.S;
    std::vector<int32_t> win(S, 0);
    const int L = std::min<int>((int)ctx.size(), S);
    for (int i = 0; i < L; ++i) win[i] = ctx[ctx.size() - L + i];
    n->forward(win.data(), nullptr, 1, S);
    const float* row = n->logits.data() + (size_t)(L - 1) * n->c.vocab;
    int best = 0;
    for (int j = 1; j < n->c.vocab; ++j)
      if (row[j] > row[best]) best = j;
    out[t] = best;
    ctx.push_back(best);
  }
  return max_new;
}

// Synthetic word corpus (bytes) used by the nano benchmark.
int64_t aether_nano_synthetic_corpus(uint8_t* out, int64_t n_bytes, uint64_t seed, int n_words) {
  auto v = aether_rt::synthetic_words((size_t)n_bytes, seed, n_words);
  std::memcpy(out, v.data(), v.size());
  return (int64_t)v.size();
}

// The reference trainer's default smoke corpus: one English sentence repeated
// (trainer/src/data.rs ByteDataset::synthetic). Learnable in tens of steps.
int64_t aether_nano_pattern_corpus(uint8_t* out, int64_t n_bytes) {
  static const char kPat[] = "the quick brown fox jumps over the lazy dog. ";
  const int64_t m = (int64_t)sizeof(kPat) - 1;
  for (int64_t i = 0; i < n_bytes; ++i) out[i] = (uint8_t)kPat[i % m];
  return n_bytes;
}

// Random windows of a byte corpus: ids/labels [B, S].
void aether_nano_sample_batch(const uint8_t* data, int64_t n, int B, int S, uint64_t* rng_state, int32_t* ids,
                              int32_t* labels) {
  aether_rt::Rng rng(0);
  rng.state = *rng_state;
  const size_t starts = (size_t)(n - S - 1);
  for (int b = 0; b < B; ++b) {
    const size_t st = rng.gen_range(starts);
    for (int i = 0; i < S; ++i) {
      ids[b * S + i] = data[st + i];
      labels[b * S + i] = data[st + i + 1];
    }
  }
  *rng_state = rng.state;
}

float aether_nano_cosine_lr(int step, int max_steps, float lr_max, int warmup) {
  return aether_rt::cosine_lr(step, max_steps, lr_max, warmup);
}

// `.weights` ("AETHER01\n" + u64 count + f32 LE) and `.meta` (one-line JSON).
int aether_nano_save(void* h, const char* stem) {
  Nano* n = static_cast<Nano*>(h);
  const std::string s(stem);
  std::ofstream wf(s + ".weights", std::ios::binary);
  if (!wf) return -1;
  wf.write("AETHER01\n", 9);
  const uint64_t cnt = n->total;
  wf.write(reinterpret_cast<const char*>(&cnt), 8);
  wf.write(reinterpret_cast<const char*>(n->p.data()), (std::streamsize)(n->total * 4));
  std::ofstream mf(s + ".meta");
  if (!mf) return -2;
  mf << "{\"vocab\":" << n->c.vocab << ",\"d_model\":" << n->c.d << ",\"n_layers\":" << n->c.L
     << ",\"n_heads\":" << n->c.H << ",\"d_ff\":" << n->c.F << ",\"seq_len\":" << n->c.S
     << ",\"params\":" << n->total << "}\n";
  return 0;
}

int aether_nano_load_weights(void* h, const char* path) {
  Nano* n = static_cast<Nano*>(h);
  std::ifstream f(path, std::ios::binary);
  if (!f) return -1;
  char magic[9];
  f.read(magic, 9);
  if (std::memcmp(magic, "AETHER01\n", 9) != 0) return -2;
  uint64_t cnt = 0;
  f.read(reinterpret_cast<char*>(&cnt), 8);
  if (cnt != n->total) return -3;
  f.read(reinterpret_cast<char*>(n->p.data()), (std::streamsize)(cnt * 4));
  return f ? 0 : -4;
}

}  // extern "C"
