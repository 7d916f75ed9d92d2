// aether-prepare: turn a text file into the byte-level training corpus the
// AetherLM trainer reads (vocabulary = 256 bytes, so the corpus is the file's
// bytes). Like the reference tool (trainer/src/bin/prepare.rs) it refuses
// inputs over 4 GiB, output paths with "..", and outputs outside the working
// directory, and it writes atomically (temp file + rename).
//
//   aether-prepare --in raw.txt --out data/corpus.bin
#include <sys/stat.h>
#include <unistd.h>

#include <climits>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <string>
#include <vector>

static bool inside_cwd(const std::string& out) {
  if (out.find("..") != std::string::npos) return false;
  char cwd[PATH_MAX];
  if (!getcwd(cwd, sizeof(cwd))) return false;
  std::string dir = out.substr(0, out.find_last_of('/') == std::string::npos ? 0 : out.find_last_of('/'));
  if (dir.empty()) return true;
  if (std::system(("mkdir -p '" + dir + "'").c_str()) != 0) return false;
  char real[PATH_MAX];
  if (!realpath(dir.c_str(), real)) return false;
  const size_t n = std::strlen(cwd);
  return std::strncmp(real, cwd, n) == 0 && (real[n] == '\0' || real[n] == '/');
}

int main(int argc, char** argv) {
  std::string in, out;
  for (int i = 1; i < argc; ++i) {
    const std::string a = argv[i];
    if (a == "--in" && i + 1 < argc) in = argv[++i];
    else if (a == "--out" && i + 1 < argc) out = argv[++i];
    else if (a == "-h" || a == "--help") {
      std::fprintf(stderr, "aether-prepare --in PATH --out PATH\n");
      return 0;
    } else {
      std::fprintf(stderr, "unknown arg: %s\n", a.c_str());
      return 2;
    }
  }
  if (in.empty() || out.empty()) {
    std::fprintf(stderr, "--in and --out are required\n");
    return 2;
  }
  struct stat st {};
  if (stat(in.c_str(), &st) != 0 || !S_ISREG(st.st_mode)) {
    std::fprintf(stderr, "--in must be a regular file\n");
    return 1;
  }
  if ((unsigned long long)st.st_size > (4ull << 30)) {
    std::fprintf(stderr, "input too large (%lld bytes)\n", (long long)st.st_size);
    return 1;
  }
  if (!inside_cwd(out)) {
    std::fprintf(stderr, "output path must stay inside the working directory\n");
    return 1;
  }
  std::ifstream f(in, std::ios::binary);
  std::vector<char> buf((size_t)st.st_size);
  if (!f.read(buf.data(), (std::streamsize)buf.size())) {
    std::fprintf(stderr, "cannot read %s\n", in.c_str());
    return 1;
  }
  const std::string tmp = out + ".tmp";
  {
    std::ofstream o(tmp, std::ios::binary);
    if (!o.write(buf.data(), (std::streamsize)buf.size())) {
      std::fprintf(stderr, "cannot write %s\n", tmp.c_str());
      return 1;
    }
  }
  if (std::rename(tmp.c_str(), out.c_str()) != 0) {
    std::fprintf(stderr, "cannot rename to %s\n", out.c_str());
    return 1;
  }
  std::fprintf(stderr, "[aether-prepare] %zu bytes -> %s\n", buf.size(), out.c_str());
  return 0;
}
