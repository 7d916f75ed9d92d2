// aether-train: AetherLM-Nano / -Tiny fp32 CPU training through libaether_rt.
// Flags follow the reference CLI (trainer/src/main.rs:25-66):
//   --config nano|tiny --steps N --batch B --seq S --lr LR --seed S
//   --log-every N --data FILE --synth-bytes N --out STEM --warmup N --wd X --clip X
// Without --data the corpus is the synthetic seeded word corpus. Prints
// "[aether-train] step=... loss=... lr=... tok/s=..." lines and writes
// STEM.weights / STEM.meta.
//
// Data parallelism (reference trainer/src/dp.rs: replicas on the CPU, the
// gradient averaged over ranks, the same AdamW on every rank):
//   --world-size N            N replicas in this process, each sampling its
//                             own batch stream; the mean gradient is applied to all
//   --world-size N --rank r   one replica per process; the ranks meet at
//                             AETHER_COMM_ADDR (host:port) and all-reduce the
//                             gradient through libaether_rt's host communicator
//                             (TCP), so the ranks may sit on different hosts
// Rank r's batches come from its own stream (seed * 7919 + 1 + r * 1000003),
// so both forms train the same model for the same N.
#include <algorithm>
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
float aether_nano_forward_backward(void*, const int32_t*, const int32_t*, int);
void aether_nano_apply_update(void*, float, float, float, int64_t);
float* aether_nano_params(void*);
float* aether_nano_grads(void*);
int64_t aether_nccl_comm_create(int, int);
int aether_nccl_comm_destroy(int64_t);
int aether_nccl_all_reduce_f32(const void*, void*, int, int, int64_t);
int64_t aether_nano_synthetic_corpus(uint8_t*, int64_t, uint64_t, int);
int64_t aether_nano_pattern_corpus(uint8_t*, int64_t);
void aether_nano_sample_batch(const uint8_t*, int64_t, int, int, uint64_t*, int32_t*, int32_t*);
float aether_nano_cosine_lr(int, int, float, int);
int aether_nano_save(void*, const char*);
int aether_nano_generate(void*, const int32_t*, int, int, int32_t*);
}

int main(int argc, char** argv) {
  std::string config = "nano", data, out = "checkpoints/aether_lm", synthetic = "pattern";
  int steps = 60, batch = 8, seq = 0, log_every = 10, warmup = 10, gen = 60, world = 1, rank = -1;
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
    else if (a == "--world-size") world = std::max(1, std::atoi(next().c_str()));
    else if (a == "--rank") rank = std::atoi(next().c_str());
    else {
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
  // replicas held by this process: all of them (in-process DP), or this rank's
  const bool multi_process = world > 1 && rank >= 0;
  if (multi_process && rank >= world) {
    std::fprintf(stderr, "--rank must be below --world-size\n");
    return 2;
  }
  const int local = (world > 1 && !multi_process) ? world : 1;
  std::vector<void*> reps;
  std::vector<uint64_t> rngs;
  for (int r = 0; r < local; ++r) {
    reps.push_back(aether_nano_create(V, D, L, H, F, S, seed));  // identical initial weights
    const int gr = multi_process ? rank : r;
    rngs.push_back(seed * 7919 + 1 + (uint64_t)gr * 1000003ull);
  }
  void* m = reps[0];
  const int64_t np = aether_nano_num_params(m);
  int64_t comm = 0;
  if (multi_process) {
    comm = aether_nccl_comm_create(world, rank);
    if (comm <= 0) {
      std::fprintf(stderr, "[aether-train] rank %d: no rendezvous (set AETHER_COMM_ADDR=host:port)\n", rank);
      return 1;
    }
  }
  std::fprintf(stderr, "[aether-train] config=%s params=%lld corpus=%zu bytes world=%d%s\n", config.c_str(),
               (long long)np, corpus.size(), world,
               multi_process ? " (one rank per process)" : (world > 1 ? " (replicas in-process)" : ""));
  std::vector<int32_t> ids((size_t)batch * S), labels((size_t)batch * S);
  std::vector<float> gsum(world > 1 ? (size_t)np : 0);
  auto t0 = std::chrono::steady_clock::now();
  auto tl = t0;
  double run = 0;
  int cnt = 0;
  float first = -1, last = 0;
  for (int step = 0; step < steps; ++step) {
    const float lrs = aether_nano_cosine_lr(step, steps, lr, warmup);
    float loss = 0.f;
    if (world == 1) {
      aether_nano_sample_batch(corpus.data(), (int64_t)corpus.size(), batch, S, &rngs[0], ids.data(), labels.data());
      loss = aether_nano_train_step(m, ids.data(), labels.data(), batch, lrs, wd, clip, step + 1);
    } else {
      std::fill(gsum.begin(), gsum.end(), 0.f);
      for (int r = 0; r < local; ++r) {  // rank order, so both forms add in the same order
        aether_nano_sample_batch(corpus.data(), (int64_t)corpus.size(), batch, S, &rngs[(size_t)r], ids.data(),
                                 labels.data());
        loss += aether_nano_forward_backward(reps[(size_t)r], ids.data(), labels.data(), batch);
        const float* g = aether_nano_grads(reps[(size_t)r]);
        for (int64_t i = 0; i < np; ++i) gsum[(size_t)i] += g[i];
      }
      if (multi_process) {
        float lbuf = loss;
        if (aether_nccl_all_reduce_f32(gsum.data(), gsum.data(), (int)np, 0, comm) != 0 ||
            aether_nccl_all_reduce_f32(&lbuf, &lbuf, 1, 0, comm) != 0) {
          std::fprintf(stderr, "[aether-train] rank %d: gradient all-reduce failed\n", rank);
          return 1;
        }
        loss = lbuf;
      }
      loss /= (float)world;
      const float inv = 1.f / (float)world;
      for (void* rp : reps) {
        float* g = aether_nano_grads(rp);
        for (int64_t i = 0; i < np; ++i) g[i] = gsum[(size_t)i] * inv;
        aether_nano_apply_update(rp, lrs, wd, clip, step + 1);
      }
    }
    if (first < 0) first = loss;
    last = loss;
    run += loss;
    ++cnt;
    if (step % log_every == 0 || step + 1 == steps) {
      auto now = std::chrono::steady_clock::now();
      const double dt = std::chrono::duration<double>(now - tl).count();
      const double el = std::chrono::duration<double>(now - t0).count();
      std::fprintf(stderr, "[aether-train] step=%5d loss=%.4f lr=%.2e tok/s=%.0f elapsed=%.1fs\n", step, run / cnt, lrs,
                   dt > 0 ? (double)batch * S * cnt * local / dt : 0.0, el);
      tl = now;
      run = 0;
      cnt = 0;
    }
  }
  const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  std::fprintf(stderr, "[aether-train] done in %.1fs\n", el);
  if (local > 1) {  // every replica applied the same updates
    bool same = true;
    for (int r = 1; r < local; ++r)
      same = same && std::memcmp(aether_nano_params(reps[0]), aether_nano_params(reps[(size_t)r]),
                                 sizeof(float) * (size_t)np) == 0;
    std::fprintf(stderr, "[aether-train] replicas %s\n", same ? "identical" : "DIVERGED");
    if (!same) return 1;
  }
  if (multi_process) aether_nccl_comm_destroy(comm);
  if (multi_process && rank != 0) {  // rank 0 writes the checkpoint and the summary
    for (void* rp : reps) aether_nano_destroy(rp);
    return 0;
  }
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
  for (void* rp : reps) aether_nano_destroy(rp);
  return 0;
}
