// aether-train: AetherLM-Nano / -Tiny fp32 CPU training through libaether_rt.
// Flags follow the reference CLI (trainer/src/main.rs:25-66):
//   --config nano|tiny --steps N --batch B --seq S --lr LR --seed S
//   --log-every N --data FILE --synth-bytes N --out STEM --warmup N --wd X --clip X
// Without --data the corpus is the synthetic seeded word corpus. Prints
// "[aether-train] step=... loss=... lr=... tok/s=..." lines and writes
// STEM.weights / STEM.meta.
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <string>
#include <vector>

extern "C" {
void* aether_nano_create(int, int, int, int, int, int, uint64_t);
void aether_nano_destroy(void*);
int64_t aether_nano_num_params(void*);
float aether_nano_train_step(void*, const int32_t*, const int32_t*, int, float, float, float, int64_t);
int64_t aether_nano_synthetic_corpus(uint8_t*, int64_t, uint64_t, int);
int64_t aether_nano_pattern_corpus(uint8_t*, int64_t);
void aether_nano_sample_batch(const uint8_t*, int64_t, int, int, uint64_t*, int32_t*, int32_t*);
float aether_nano_cosine_lr(int, int, float, int);
int aether_nano_save(void*, const char*);
int aether_nano_generate(void*, const int32_t*, int, int, int32_t*);
}

int main(int argc, char** argv) {
  std::string config = "nano", data, out = "checkpoints/aether_lm", synthetic = "pattern";
  int steps = 60, batch = 8, seq = 0, log_every = 10, warmup = 10, gen = 60;
  float lr = 3e-3f, wd = 0.f, clip = 1.f;
  uint64_t seed = 42;
  int64_t synth = 1 << 20;
  for (int i = 1; i < argc; ++i) {
    std::string a = argv[i];
    auto next = [&]() { return i + 1 < argc ? std::string(argv[++i]) : std::string(); };
    if (a == "--config") config = next();
    else if (a == "--steps") steps = std::atoi(next().c_str());
    else if (a == "--batch") batch = std::atoi(next().c_str());
    else if (a == "--seq") seq = std::atoi(next().c_str());
    else if (a == "--lr") lr = std::atof(next().c_str());
    else if (a == "--seed") seed = std::strtoull(next().c_str(), nullptr, 10);
    else if (a == "--log-every") log_every = std::max(1, std::atoi(next().c_str()));
    else if (a == "--data") data = next();
    else if (a == "--synth-bytes") synth = std::atoll(next().c_str());
    else if (a == "--synthetic") synthetic = next();  // pattern (reference default) | words
    else if (a == "--out") out = next();
    else if (a == "--warmup") warmup = std::atoi(next().c_str());
    else if (a == "--wd") wd = std::atof(next().c_str());
    else if (a == "--clip") clip = std::atof(next().c_str());
    else if (a == "--gen") gen = std::atoi(next().c_str());
    else if (a == "--world-size") {
      if (std::atoi(next().c_str()) > 1) {
        std::fprintf(stderr, "multi-rank training runs through the torch.distributed engines (aether_b200.train)\n");
        return 2;
      }
    } else {
      std::fprintf(stderr, "unknown flag %s\n", a.c_str());
      return 2;
    }
  }
  int V = 256, D = 64, L = 2, H = 4, F = 128, S = 32;
  if (config == "tiny") {
    D = 320; L = 6; H = 5; F = 1280; S = 256;
  } else if (config != "nano") {
    std::fprintf(stderr, "--config nano|tiny\n");
    return 2;
  }
  if (seq > 0) S = seq;
  std::vector<uint8_t> corpus;
  if (!data.empty()) {
    std::ifstream f(data, std::ios::binary);
    if (!f) {
      std::fprintf(stderr, "cannot read %s\n", data.c_str());
      return 1;
    }
    corpus.assign(std::istreambuf_iterator<char>(f), std::istreambuf_iterator<char>());
  } else {
    corpus.resize((size_t)synth);
    if (synthetic == "words")
      aether_nano_synthetic_corpus(corpus.data(), synth, seed, 200);
    else
      aether_nano_pattern_corpus(corpus.data(), synth);
  }
  void* m = aether_nano_create(V, D, L, H, F, S, seed);
  std::fprintf(stderr, "[aether-train] config=%s params=%lld corpus=%zu bytes\n", config.c_str(),
               (long long)aether_nano_num_params(m), corpus.size());
  std::vector<int32_t> ids((size_t)batch * S), labels((size_t)batch * S);
  uint64_t rng = seed * 7919 + 1;
  auto t0 = std::chrono::steady_clock::now();
  auto tl = t0;
  double run = 0;
  int cnt = 0;
  float first = -1, last = 0;
  for (int step = 0; step < steps; ++step) {
    const float lrs = aether_nano_cosine_lr(step, steps, lr, warmup);
    aether_nano_sample_batch(corpus.data(), (int64_t)corpus.size(), batch, S, &rng, ids.data(), labels.data());
    const float loss = aether_nano_train_step(m, ids.data(), labels.data(), batch, lrs, wd, clip, step + 1);
    if (first < 0) first = loss;
    last = loss;
    run += loss;
    ++cnt;
    if (step % log_every == 0 || step + 1 == steps) {
      auto now = std::chrono::steady_clock::now();
      const double dt = std::chrono::duration<double>(now - tl).count();
      const double el = std::chrono::duration<double>(now - t0).count();
      std::fprintf(stderr, "[aether-train] step=%5d loss=%.4f lr=%.2e tok/s=%.0f elapsed=%.1fs\n", step, run / cnt, lrs,
                   dt > 0 ? (double)batch * S * cnt / dt : 0.0, el);
      tl = now;
      run = 0;
      cnt = 0;
    }
  }
  const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  std::fprintf(stderr, "[aether-train] done in %.1fs\n", el);
  std::string dir = out.substr(0, out.find_last_of('/') == std::string::npos ? 0 : out.find_last_of('/'));
  if (!dir.empty() && std::system(("mkdir -p '" + dir + "'").c_str()) != 0) std::fprintf(stderr, "cannot create %s\n", dir.c_str());
  if (aether_nano_save(m, out.c_str()) != 0) {
    std::fprintf(stderr, "cannot write %s.weights\n", out.c_str());
    return 1;
  }
  std::vector<int32_t> prompt = {corpus[0], corpus[1]}, gen_out(gen);
  aether_nano_generate(m, prompt.data(), 2, gen, gen_out.data());
  std::string txt;
  for (int t : gen_out) txt.push_back((t >= 32 && t < 127) ? (char)t : '?');
  std::printf("{\"first_loss\": %.4f, \"final_loss\": %.4f, \"seconds\": %.2f, \"params\": %lld, \"sample\": \"%c%c%s\"}\n",
              first, last, el, (long long)aether_nano_num_params(m), corpus[0], corpus[1], txt.c_str());
  aether_nano_destroy(m);
  return 0;
}
