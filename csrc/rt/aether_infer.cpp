// aether-infer: load STEM.weights/STEM.meta and continue a byte prompt greedily
// (reference CLI: trainer/src/bin/infer.rs -- --ckpt --prompt --max-new).
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <sstream>
#include <string>
#include <vector>

extern "C" {
void* aether_nano_create(int, int, int, int, int, int, uint64_t);
void aether_nano_destroy(void*);
int aether_nano_load_weights(void*, const char*);
int aether_nano_generate(void*, const int32_t*, int, int, int32_t*);
}

static int meta_int(const std::string& s, const std::string& key) {
  const size_t p = s.find("\"" + key + "\":");
  return p == std::string::npos ? -1 : std::atoi(s.c_str() + p + key.size() + 3);
}

int main(int argc, char** argv) {
  std::string ckpt = "checkpoints/aether_lm", prompt = "th";
  int max_new = 60;
  for (int i = 1; i < argc; ++i) {
    std::string a = argv[i];
    auto next = [&]() { return i + 1 < argc ? std::string(argv[++i]) : std::string(); };
    if (a == "--ckpt") ckpt = next();
    else if (a == "--prompt") prompt = next();
    else if (a == "--max-new") max_new = std::atoi(next().c_str());
    else if (a == "--temperature" || a == "--top-k" || a == "--seed") next();  // greedy decoding
  }
  std::ifstream mf(ckpt + ".meta");
  if (!mf) {
    std::fprintf(stderr, "cannot read %s.meta\n", ckpt.c_str());
    return 1;
  }
  std::stringstream ss;
  ss << mf.rdbuf();
  const std::string meta = ss.str();
  void* m = aether_nano_create(meta_int(meta, "vocab"), meta_int(meta, "d_model"), meta_int(meta, "n_layers"),
                               meta_int(meta, "n_heads"), meta_int(meta, "d_ff"), meta_int(meta, "seq_len"), 0);
  if (!m || aether_nano_load_weights(m, (ckpt + ".weights").c_str()) != 0) {
    std::fprintf(stderr, "cannot load %s.weights\n", ckpt.c_str());
    return 1;
  }
  std::vector<int32_t> ids(prompt.begin(), prompt.end()), out(max_new);
  aether_nano_generate(m, ids.data(), (int)ids.size(), max_new, out.data());
  std::string txt = prompt;
  for (int t : out) txt.push_back((t >= 32 && t < 127) ? (char)t : '?');
  std::printf("%s\n", txt.c_str());
  aether_nano_destroy(m);
  return 0;
}
