// Developer tools for .aether sources, one binary dispatched on its name:
//
//   aetherfmt [--check] [--reindent] <file>... | -
//       Normalises layout: tabs outside string / char literals become four
//       spaces, trailing whitespace goes, runs of blank lines shrink to one,
//       the file ends in exactly one newline; --reindent also recomputes
//       leading indentation from brace depth (strings and comments skipped).
//       --check rewrites nothing and exits 1 listing the files that would
//       change. Reference: tools/aetherfmt/src/main.rs.
//   aetherclippy [--allow CODE,...] <file>...
//       Line lints, each with a code: AC001 trailing whitespace, AC002 tab
//       indentation, AC003 `let _ =` discards, AC004 integer literal above
//       4096 outside a const declaration, AC005 TODO / FIXME / XXX markers,
//       AC006 line longer than 120 columns, AC007 empty function body.
//       Literals, identifiers and comment text are told apart by a small
//       scanner, so `x_5000` or "5000" is not a magic number. Exit 1 when a
//       lint fires. Reference: tools/aetherclippy/src/main.rs.
//   aetherdoc [--html] <file>...
//       The `///` comment run right above each fn / extern fn / struct / enum
//       / trait / impl / const, as a markdown (or HTML) index grouped by file.
//       Reference: tools/aetherdoc/src/main.rs.
//   aether-audit [--json] [--only sloc|markers|witnesses|conformance|abi] [--root DIR]
//       Repository audit: source lines per component (code / comment /
//       blank), unfinished-work markers in product sources, the .aether
//       witnesses compiled with aetherc and run against their
//       `// expect: exit=N` header, and the C-ABI export count of the built
//       libraries (dlopen + dlsym of every `aether_` name their sources
//       define). Exit 1 when a witness fails or a defined export is missing.
//       Reference: tools/audit/src/*.rs.
//   witness-stamper [--dir DIR] [--tags FILE] [--fresh FILE] [--check]
//       Adds roadmap tags to witnesses (`file tag` lines: the tag is appended
//       to the file's `// roadmap:` line, which is created below the
//       `// expect:` header if absent; tags already there are kept once) and
//       writes fresh witnesses from a spec (`=== name.aether` sections).
//       Idempotent; --check only reports what would change (exit 1 if any).
//       Reference: tools/witness-stamper/src/main.rs.
#include <dirent.h>
#include <dlfcn.h>
#include <sys/stat.h>
#include <sys/wait.h>
#include <unistd.h>

#include <algorithm>
#include <cctype>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <iostream>
#include <map>
#include <set>
#include <sstream>
#include <string>
#include <vector>

namespace {

bool read_file(const std::string& path, std::string& out) {
  std::ifstream f(path, std::ios::binary);
  if (!f) return false;
  std::ostringstream ss;
  ss << f.rdbuf();
  out = ss.str();
  return true;
}

bool write_file(const std::string& path, const std::string& data) {
  const std::string tmp = path + ".tmp~";
  {
    std::ofstream f(tmp, std::ios::binary | std::ios::trunc);
    if (!f) return false;
    f << data;
    if (!f) return false;
  }
  return std::rename(tmp.c_str(), path.c_str()) == 0;
}

std::vector<std::string> split_lines(const std::string& s) {
  std::vector<std::string> out;
  std::string cur;
  for (char c : s) {
    if (c == '\n') {
      if (!cur.empty() && cur.back() == '\r') cur.pop_back();
      out.push_back(cur);
      cur.clear();
    } else {
      cur.push_back(c);
    }
  }
  if (!cur.empty()) out.push_back(cur);
  return out;
}

std::string rtrim(const std::string& s) {
  size_t e = s.size();
  while (e > 0 && (s[e - 1] == ' ' || s[e - 1] == '\t')) --e;
  return s.substr(0, e);
}

std::string ltrim(const std::string& s) {
  size_t b = 0;
  while (b < s.size() && (s[b] == ' ' || s[b] == '\t')) ++b;
  return s.substr(b);
}

bool starts_with(const std::string& s, const char* p) { return s.rfind(p, 0) == 0; }

// ------------------------------------------------------------------ scanner
// Classifies each character of a line as code, string / char literal or
// comment. Block comments carry across lines through `in_block`.
enum Cls : char { CODE = 'c', STR = 's', COMMENT = 'm' };

std::string classify(const std::string& line, bool& in_block) {
  std::string cls(line.size(), CODE);
  size_t i = 0;
  while (i < line.size()) {
    if (in_block) {
      cls[i] = COMMENT;
      if (line[i] == '*' && i + 1 < line.size() && line[i + 1] == '/') {
        cls[i + 1] = COMMENT;
        i += 2;
        in_block = false;
        continue;
      }
      ++i;
      continue;
    }
    const char c = line[i];
    if (c == '/' && i + 1 < line.size() && line[i + 1] == '/') {
      for (size_t j = i; j < line.size(); ++j) cls[j] = COMMENT;
      break;
    }
    if (c == '/' && i + 1 < line.size() && line[i + 1] == '*') {
      cls[i] = cls[i + 1] = COMMENT;
      i += 2;
      in_block = true;
      continue;
    }
    if (c == '"' || c == '\'') {
      // a quote followed by an identifier and no closing quote is a lifetime-like tick: code
      const char q = c;
      size_t j = i + 1;
      bool closed = false;
      while (j < line.size()) {
        if (line[j] == '\\') {
          j += 2;
          continue;
        }
        if (line[j] == q) {
          closed = true;
          break;
        }
        ++j;
      }
      if (q == '\'' && !closed) {
        ++i;
        continue;
      }
      const size_t end = closed ? j : line.size() - 1;
      for (size_t k = i; k <= end && k < line.size(); ++k) cls[k] = STR;
      i = end + 1;
      continue;
    }
    ++i;
  }
  return cls;
}

// ------------------------------------------------------------------ aetherfmt
std::string format_source(const std::string& src, bool reindent) {
  std::vector<std::string> lines = split_lines(src);
  std::vector<std::string> out;
  bool in_block = false;
  int depth = 0;
  int blank_run = 0;
  for (const std::string& raw : lines) {
    const bool was_in_block = in_block;
    const std::string cls = classify(raw, in_block);
    std::string line;
    for (size_t i = 0; i < raw.size(); ++i) {
      if (raw[i] == '\t' && cls[i] != STR) line += "    ";
      else line.push_back(raw[i]);
    }
    line = rtrim(line);
    if (line.empty()) {
      if (++blank_run > 1) continue;
      out.push_back("");
      continue;
    }
    blank_run = 0;
    if (reindent && !was_in_block) {
      // braces of code characters only; a line starting with a closer dedents itself
      int opens = 0, closes = 0, lead_close = 0;
      bool leading = true;
      const std::string t = ltrim(raw);
      const size_t off = raw.size() - t.size();
      for (size_t i = off; i < raw.size(); ++i) {
        if (cls[i] != CODE) {
          leading = false;
          continue;
        }
        const char c = raw[i];
        if (c == '{' || c == '(' || c == '[') {
          ++opens;
          leading = false;
        } else if (c == '}' || c == ')' || c == ']') {
          ++closes;
          if (leading) ++lead_close;
        } else if (c != ' ' && c != '\t') {
          leading = false;
        }
      }
      const int ind = std::max(0, depth - lead_close);
      line = std::string(4 * ind, ' ') + rtrim(ltrim(line));
      depth = std::max(0, depth + opens - closes);
    }
    out.push_back(line);
  }
  while (!out.empty() && out.back().empty()) out.pop_back();
  while (!out.empty() && out.front().empty()) out.erase(out.begin());
  std::string r;
  for (const std::string& l : out) {
    r += l;
    r += '\n';
  }
  return r;
}

int main_fmt(const std::vector<std::string>& args) {
  bool check = false, reindent = false, stdin_mode = false;
  std::vector<std::string> paths;
  for (const std::string& a : args) {
    if (a == "--check") check = true;
    else if (a == "--reindent") reindent = true;
    else if (a == "-") stdin_mode = true;
    else paths.push_back(a);
  }
  if (stdin_mode) {
    std::ostringstream ss;
    ss << std::cin.rdbuf();
    std::fputs(format_source(ss.str(), reindent).c_str(), stdout);
    return 0;
  }
  if (paths.empty()) {
    std::fprintf(stderr, "usage: aetherfmt [--check] [--reindent] <file.aether>... | -\n");
    return 2;
  }
  int changed = 0;
  for (const std::string& p : paths) {
    std::string src;
    if (!read_file(p, src)) {
      std::fprintf(stderr, "aetherfmt: cannot read %s\n", p.c_str());
      return 2;
    }
    const std::string f = format_source(src, reindent);
    if (f == src) continue;
    ++changed;
    if (check) {
      std::printf("%s\n", p.c_str());
    } else if (!write_file(p, f)) {
      std::fprintf(stderr, "aetherfmt: cannot write %s\n", p.c_str());
      return 2;
    }
  }
  if (check && changed) {
    std::fprintf(stderr, "aetherfmt: %d file(s) not formatted\n", changed);
    return 1;
  }
  return 0;
}

// ------------------------------------------------------------------ aetherclippy
struct Lint {
  std::string file;
  int line;
  std::string code, msg;
};

bool is_ident(char c) { return std::isalnum((unsigned char)c) || c == '_'; }

std::vector<Lint> lint_source(const std::string& file, const std::string& src) {
  std::vector<Lint> out;
  const std::vector<std::string> lines = split_lines(src);
  bool in_block = false;
  for (size_t n = 0; n < lines.size(); ++n) {
    const std::string& raw = lines[n];
    const int ln = (int)n + 1;
    const std::string cls = classify(raw, in_block);
    if (!raw.empty() && (raw.back() == ' ' || raw.back() == '\t'))
      out.push_back({file, ln, "AC001", "trailing whitespace"});
    if (!raw.empty() && raw[0] == '\t') out.push_back({file, ln, "AC002", "tab indentation (use four spaces)"});
    const std::string t = ltrim(raw);
    if (starts_with(t, "let _ =") || starts_with(t, "let _=") || starts_with(t, "let _:"))
      out.push_back({file, ln, "AC003", "`let _ = expr;` discards the value: use the expression as a statement"});
    if (!starts_with(t, "const ") && !starts_with(t, "pub const ")) {
      for (size_t i = 0; i < raw.size(); ++i) {
        if (cls[i] != CODE || !std::isdigit((unsigned char)raw[i]) || (i > 0 && is_ident(raw[i - 1]))) continue;
        size_t j = i;
        std::string digits;
        bool hex = false;
        if (raw[i] == '0' && i + 1 < raw.size() && (raw[i + 1] == 'x' || raw[i + 1] == 'X')) {
          hex = true;
          j = i + 2;
        }
        while (j < raw.size() && (std::isxdigit((unsigned char)raw[j]) || raw[j] == '_')) {
          if (raw[j] != '_') {
            if (!hex && !std::isdigit((unsigned char)raw[j])) break;
            digits.push_back(raw[j]);
          }
          ++j;
        }
        const bool is_float = j < raw.size() && raw[j] == '.' && j + 1 < raw.size() && std::isdigit((unsigned char)raw[j + 1]);
        if (!digits.empty() && !is_float) {
          const unsigned long long v = std::strtoull(digits.c_str(), nullptr, hex ? 16 : 10);
          if (v > 4096) out.push_back({file, ln, "AC004", "magic number " + raw.substr(i, j - i) + ": name it with a const"});
        }
        if (is_float) {  // skip the fraction and exponent of a float literal
          ++j;
          while (j < raw.size() && (std::isdigit((unsigned char)raw[j]) || raw[j] == '_')) ++j;
          if (j < raw.size() && (raw[j] == 'e' || raw[j] == 'E')) {
            ++j;
            if (j < raw.size() && (raw[j] == '+' || raw[j] == '-')) ++j;
            while (j < raw.size() && std::isdigit((unsigned char)raw[j])) ++j;
          }
        }
        i = j;
      }
    }
    for (const char* m : {"TODO", "FIXME", "XXX"}) {
      const size_t k = raw.find(m);
      if (k != std::string::npos && cls[k] == COMMENT) {
        out.push_back({file, ln, "AC005", std::string(m) + " marker"});
        break;
      }
    }
    if (raw.size() > 120) out.push_back({file, ln, "AC006", "line longer than 120 columns"});
    if ((starts_with(t, "fn ") || starts_with(t, "pub fn ")) && rtrim(t).size() >= 2) {
      const std::string r = rtrim(t);
      if (r.compare(r.size() - 2, 2, "{}") == 0 && r.find("->") == std::string::npos)
        out.push_back({file, ln, "AC007", "empty function body"});
    }
  }
  return out;
}

int main_clippy(const std::vector<std::string>& args) {
  std::set<std::string> allow;
  std::vector<std::string> paths;
  for (size_t i = 0; i < args.size(); ++i) {
    if (args[i] == "--allow" && i + 1 < args.size()) {
      std::stringstream ss(args[++i]);
      std::string c;
      while (std::getline(ss, c, ',')) allow.insert(c);
    } else {
      paths.push_back(args[i]);
    }
  }
  if (paths.empty()) {
    std::fprintf(stderr, "usage: aetherclippy [--allow CODE,...] <file.aether>...\n");
    return 2;
  }
  int n = 0;
  for (const std::string& p : paths) {
    std::string src;
    if (!read_file(p, src)) {
      std::fprintf(stderr, "aetherclippy: cannot read %s\n", p.c_str());
      return 2;
    }
    for (const Lint& l : lint_source(p, src)) {
      if (allow.count(l.code)) continue;
      std::printf("%s:%d: %s %s\n", l.file.c_str(), l.line, l.code.c_str(), l.msg.c_str());
      ++n;
    }
  }
  if (n) std::fprintf(stderr, "aetherclippy: %d lint(s)\n", n);
  return n ? 1 : 0;
}

// ------------------------------------------------------------------ aetherdoc
struct DocItem {
  std::string file;
  int line;
  std::string kind, name, doc;
};

std::vector<DocItem> extract_docs(const std::string& file, const std::string& src) {
  std::vector<DocItem> out;
  std::string pending;
  bool have = false;
  const std::vector<std::string> lines = split_lines(src);
  for (size_t n = 0; n < lines.size(); ++n) {
    std::string t = ltrim(lines[n]);
    if (starts_with(t, "///")) {
      std::string rest = t.substr(3);
      if (!rest.empty() && rest[0] == ' ') rest.erase(0, 1);
      if (have) pending += '\n';
      pending += rtrim(rest);
      have = true;
      continue;
    }
    if (starts_with(t, "//") || starts_with(t, "#[")) continue;  // plain comments and attributes keep the run
    if (!have) continue;
    std::string s = t;
    if (starts_with(s, "pub ")) s = s.substr(4);
    if (starts_with(s, "unsafe ")) s = s.substr(7);
    std::string kind;
    for (const char* k : {"extern fn ", "fn ", "struct ", "enum ", "trait ", "impl ", "const ", "static ", "type "}) {
      if (starts_with(s, k)) {
        kind = std::string(k);
        kind.pop_back();
        s = s.substr(std::strlen(k));
        break;
      }
    }
    if (!kind.empty()) {
      std::string name;
      for (char c : s) {
        if (is_ident(c) || c == ':' || c == '<' || c == '>' || c == ',' || c == ' ' || c == '&') {
          if (c == ' ' && kind != "impl") break;
          name.push_back(c);
        } else {
          break;
        }
      }
      while (!name.empty() && (name.back() == ' ' || name.back() == '<')) name.pop_back();
      out.push_back({file, (int)n + 1, kind, name, pending});
    }
    pending.clear();
    have = false;
  }
  return out;
}

std::string html_escape(const std::string& s) {
  std::string o;
  for (char c : s) {
    if (c == '<') o += "&lt;";
    else if (c == '>') o += "&gt;";
    else if (c == '&') o += "&amp;";
    else if (c == '"') o += "&quot;";
    else o.push_back(c);
  }
  return o;
}

int main_doc(const std::vector<std::string>& args) {
  bool html = false;
  std::vector<std::string> paths;
  for (const std::string& a : args) {
    if (a == "--html") html = true;
    else paths.push_back(a);
  }
  if (paths.empty()) {
    std::fprintf(stderr, "usage: aetherdoc [--html] <file.aether>...\n");
    return 2;
  }
  std::map<std::string, std::vector<DocItem>> by_file;
  for (const std::string& p : paths) {
    std::string src;
    if (!read_file(p, src)) {
      std::fprintf(stderr, "aetherdoc: cannot read %s\n", p.c_str());
      return 2;
    }
    by_file[p] = extract_docs(p, src);
  }
  std::string o;
  if (html) {
    o += "<!doctype html>\n<html><head><meta charset=\"utf-8\"><title>aetherdoc</title></head><body>\n";
    o += "<h1>API index</h1>\n";
    for (const auto& kv : by_file) {
      o += "<h2><code>" + html_escape(kv.first) + "</code></h2>\n";
      for (const DocItem& d : kv.second) {
        o += "<h3 id=\"" + html_escape(d.name) + "\"><code>" + html_escape(d.kind + " " + d.name) +
             "</code> <small>line " + std::to_string(d.line) + "</small></h3>\n<pre>" + html_escape(d.doc) + "</pre>\n";
      }
    }
    o += "</body></html>\n";
  } else {
    o += "# API index\n\n";
    for (const auto& kv : by_file) {
      o += "## `" + kv.first + "`\n\n";
      for (const DocItem& d : kv.second)
        o += "### `" + d.kind + " " + d.name + "` (line " + std::to_string(d.line) + ")\n\n" + d.doc + "\n\n";
    }
  }
  std::fputs(o.c_str(), stdout);
  return 0;
}

// ------------------------------------------------------------------ aether-audit
std::string json_str(const std::string& s) {
  std::string o = "\"";
  for (unsigned char c : s) {
    if (c == '"') o += "\\\"";
    else if (c == '\\') o += "\\\\";
    else if (c == '\n') o += "\\n";
    else if (c == '\t') o += "\\t";
    else if (c < 0x20) {
      char b[8];
      std::snprintf(b, sizeof b, "\\u%04x", c);
      o += b;
    } else {
      o.push_back((char)c);
    }
  }
  return o + "\"";
}

void walk(const std::string& dir, std::vector<std::string>& files) {
  DIR* d = opendir(dir.c_str());
  if (!d) return;
  while (dirent* e = readdir(d)) {
    const std::string n = e->d_name;
    if (n == "." || n == ".." || n[0] == '.' || n == "__pycache__" || n == "_build" || n == "build" ||
        n == "_work" || (n.size() > 4 && n.compare(n.size() - 4, 4, "_out") == 0) || n == "baseline")
      continue;
    const std::string p = dir + "/" + n;
    struct stat st;
    if (stat(p.c_str(), &st) != 0) continue;
    if (S_ISDIR(st.st_mode)) walk(p, files);
    else if (S_ISREG(st.st_mode)) files.push_back(p);
  }
  closedir(d);
  std::sort(files.begin(), files.end());
}

std::string ext_of(const std::string& p) {
  const size_t k = p.rfind('.');
  return k == std::string::npos ? "" : p.substr(k);
}

struct Sloc {
  long files = 0, code = 0, comment = 0, blank = 0;
};

void count_lines(const std::string& path, Sloc& s) {
  std::string src;
  if (!read_file(path, src)) return;
  const bool py = ext_of(path) == ".py";
  bool in_block = false, in_doc = false;
  ++s.files;
  for (const std::string& raw : split_lines(src)) {
    const std::string t = ltrim(rtrim(raw));
    if (t.empty()) {
      ++s.blank;
      continue;
    }
    if (py) {
      const bool tq = t.find("\"\"\"") != std::string::npos;
      if (in_doc || (tq && starts_with(t, "\"\"\""))) {
        ++s.comment;
        size_t c = 0, k = 0;
        while ((k = t.find("\"\"\"", k)) != std::string::npos) {
          ++c;
          k += 3;
        }
        if (c % 2 == 1) in_doc = !in_doc;
        continue;
      }
      if (t[0] == '#') ++s.comment;
      else ++s.code;
      continue;
    }
    const std::string cls = classify(raw, in_block);
    bool code = false;
    for (size_t i = 0; i < raw.size(); ++i)
      if (cls[i] == CODE && raw[i] != ' ' && raw[i] != '\t') code = true;
    if (code) ++s.code;
    else ++s.comment;
  }
}

int run_cmd(const std::vector<std::string>& argv, std::string* out, int timeout_s) {
  std::string cmd = "timeout " + std::to_string(timeout_s);
  for (const std::string& a : argv) {
    cmd += " '";
    for (char c : a) {
      if (c == '\'') cmd += "'\\''";
      else cmd.push_back(c);
    }
    cmd += "'";
  }
  cmd += " 2>&1";
  FILE* f = popen(cmd.c_str(), "r");
  if (!f) return -1;
  char buf[4096];
  std::string o;
  size_t n;
  while ((n = fread(buf, 1, sizeof buf, f)) > 0) o.append(buf, n);
  const int st = pclose(f);
  if (out) *out = o;
  return WIFEXITED(st) ? WEXITSTATUS(st) : -1;
}

std::string self_dir() {
  char buf[4096];
  const ssize_t n = readlink("/proc/self/exe", buf, sizeof buf - 1);
  if (n <= 0) return ".";
  buf[n] = 0;
  std::string p = buf;
  const size_t k = p.rfind('/');
  return k == std::string::npos ? "." : p.substr(0, k);
}

int main_audit(const std::vector<std::string>& args) {
  bool json = false;
  std::string only, root;
  for (size_t i = 0; i < args.size(); ++i) {
    if (args[i] == "--json") json = true;
    else if (args[i] == "--only" && i + 1 < args.size()) only = args[++i];
    else if (args[i] == "--root" && i + 1 < args.size()) root = args[++i];
  }
  if (root.empty()) {
    // the repository: two levels above aether_b200/bin
    root = self_dir() + "/../..";
  }
  const std::string bin = root + "/aether_b200/bin";
  auto want = [&](const char* s) { return only.empty() || only == s; };
  std::vector<std::string> errors;
  std::string js = "{";
  bool first = true;
  auto key = [&](const std::string& k) {
    js += (first ? "" : ",") + json_str(k) + ":";
    first = false;
  };

  std::vector<std::string> files;
  walk(root + "/csrc", files);
  walk(root + "/aether_b200", files);
  walk(root + "/tests", files);
  if (want("sloc")) {
    std::map<std::string, Sloc> comp;
    for (const std::string& f : files) {
      const std::string e = ext_of(f);
      if (e != ".cpp" && e != ".cu" && e != ".cuh" && e != ".h" && e != ".py" && e != ".aether") continue;
      std::string rel = f.substr(root.size() + 1);
      std::string c = rel.substr(0, rel.find('/'));
      const size_t k = rel.find('/', c.size() + 1);
      if (k != std::string::npos && c != "tests") c = rel.substr(0, k);
      count_lines(f, comp[c]);
    }
    Sloc tot;
    std::fprintf(stderr, "%-28s %6s %8s %8s %7s\n", "component", "files", "code", "comment", "blank");
    key("sloc");
    js += "{";
    bool f1 = true;
    for (const auto& kv : comp) {
      std::fprintf(stderr, "%-28s %6ld %8ld %8ld %7ld\n", kv.first.c_str(), kv.second.files, kv.second.code,
                   kv.second.comment, kv.second.blank);
      js += (f1 ? "" : ",") + json_str(kv.first) + ":{\"files\":" + std::to_string(kv.second.files) +
            ",\"code\":" + std::to_string(kv.second.code) + ",\"comment\":" + std::to_string(kv.second.comment) +
            ",\"blank\":" + std::to_string(kv.second.blank) + "}";
      f1 = false;
      tot.files += kv.second.files;
      tot.code += kv.second.code;
      tot.comment += kv.second.comment;
      tot.blank += kv.second.blank;
    }
    js += "}";
    std::fprintf(stderr, "%-28s %6ld %8ld %8ld %7ld\n", "total", tot.files, tot.code, tot.comment, tot.blank);
  }
  if (want("markers")) {
    // unfinished-work markers in product sources (tests excluded): reported, not fatal
    key("markers");
    js += "[";
    bool f1 = true;
    long n = 0;
    for (const std::string& f : files) {
      const std::string e = ext_of(f);
      if (f.find("/tests/") != std::string::npos || (e != ".cpp" && e != ".cu" && e != ".cuh" && e != ".h" && e != ".py"))
        continue;
      std::string src;
      if (!read_file(f, src)) continue;
      const std::vector<std::string> lines = split_lines(src);
      for (size_t i = 0; i < lines.size(); ++i) {
        for (const char* m : {"TODO", "FIXME", "XXX", "unimplemented", "NotImplementedError"}) {
          if (lines[i].find(m) == std::string::npos) continue;
          const std::string rel = f.substr(root.size() + 1);
          std::fprintf(stderr, "marker %s:%zu: %s\n", rel.c_str(), i + 1, m);
          js += (f1 ? "" : ",") + std::string("{\"file\":") + json_str(rel) + ",\"line\":" + std::to_string(i + 1) +
                ",\"marker\":" + json_str(m) + "}";
          f1 = false;
          ++n;
          break;
        }
      }
    }
    js += "]";
    std::fprintf(stderr, "markers: %ld\n", n);
  }
  if (want("witnesses")) {
    key("witnesses");
    js += "[";
    bool f1 = true;
    std::vector<std::string> progs;
    walk(root + "/tests/aether", progs);
    const std::string aec = bin + "/aetherc";
    const bool have_gpu = access("/dev/nvidia0", F_OK) == 0;
    int pass = 0, fail = 0, skip = 0;
    for (const std::string& p : progs) {
      if (ext_of(p) != ".aether") continue;
      std::string src;
      read_file(p, src);
      const size_t k = src.find("expect: exit=");
      if (k == std::string::npos) continue;
      const int want_rc = std::atoi(src.c_str() + k + 13) & 255;
      const std::string name = p.substr(p.rfind('/') + 1);
      std::string status;
      if (starts_with(name, "gpu_") && !have_gpu) {
        status = "skipped (no GPU)";
        ++skip;
      } else {
        char tmpl[] = "/tmp/aether_audit_XXXXXX";
        const char* td = mkdtemp(tmpl);
        const std::string exe = std::string(td ? td : "/tmp") + "/w";
        std::string log;
        std::vector<std::string> cmd = {aec, p, "-o", exe};
        if (src.find("build-mode: aether-bin-test") != std::string::npos) cmd.push_back("--test");  // #[test] harness
        if (run_cmd(cmd, &log, 300) != 0) {
          status = "compile error";
        } else {
          const int rc = run_cmd({exe}, &log, 600);
          status = rc == want_rc ? "pass" : "exit " + std::to_string(rc) + " != " + std::to_string(want_rc);
        }
        if (status == "pass") ++pass;
        else {
          ++fail;
          errors.push_back("witness " + name + ": " + status);
        }
      }
      std::fprintf(stderr, "witness %-36s %s\n", name.c_str(), status.c_str());
      js += (f1 ? "" : ",") + std::string("{\"name\":") + json_str(name) + ",\"status\":" + json_str(status) + "}";
      f1 = false;
    }
    js += "]";
    std::fprintf(stderr, "witnesses: %d pass, %d fail, %d skipped\n", pass, fail, skip);
  }
  if (want("conformance")) {
    // tests/aether/positive/*.aether must `--check` clean; tests/aether/negative/
    // expect_AE####_*.aether must fail with that code (the reference's
    // conformance layout, tools/audit/src/conformance.rs).
    key("conformance");
    js += "[";
    bool f1 = true;
    const std::string aec = bin + "/aetherc";
    int pass = 0, fail = 0;
    for (const char* kind : {"positive", "negative"}) {
      std::vector<std::string> progs;
      walk(root + "/tests/aether/" + kind, progs);
      std::sort(progs.begin(), progs.end());
      for (const std::string& p : progs) {
        if (ext_of(p) != ".aether") continue;
        const std::string name = p.substr(p.rfind('/') + 1);
        std::string want;
        if (std::string(kind) == "negative") {
          const size_t k = name.find("_AE");
          if (k == std::string::npos || k + 7 > name.size()) continue;
          want = name.substr(k + 1, 6);
        }
        std::string log;
        const int rc = run_cmd({aec, p, "--check", "--json-errors"}, &log, 60);
        std::string status;
        if (want.empty()) status = rc == 0 ? "pass" : "unexpected failure";
        else if (rc == 0) status = "unexpected success";
        else status = log.find("\"code\":\"" + want + "\"") != std::string::npos ? "pass" : "wrong code";
        if (status == "pass") ++pass;
        else {
          ++fail;
          errors.push_back("conformance " + name + ": " + status);
        }
        std::fprintf(stderr, "conformance %-44s %s\n", name.c_str(), status.c_str());
        js += (f1 ? "" : ",") + std::string("{\"name\":") + json_str(name) + ",\"status\":" + json_str(status) + "}";
        f1 = false;
      }
    }
    js += "]";
    std::fprintf(stderr, "conformance: %d pass, %d fail\n", pass, fail);
  }
  if (want("abi")) {
    key("abi");
    js += "{";
    bool f1 = true;
    const std::pair<const char*, std::vector<std::string>> libs[] = {
        {"libaether_rt.so", {}}, {"libaether_dev.so", {}}};
    for (const auto& lib : libs) {
      // exported names the library's sources define: `aether_...(` after `extern "C"` blocks or AETHER_EXPORT
      std::set<std::string> names;
      for (const std::string& f : files) {
        if (f.find("/csrc/rt/") == std::string::npos) continue;
        const std::string e = ext_of(f);
        const bool dev_src = e == ".cu";
        if ((std::string(lib.first) == "libaether_dev.so") != dev_src || (e != ".cpp" && e != ".cu")) continue;
        if (f.find("aether_train.cpp") != std::string::npos || f.find("aether_infer.cpp") != std::string::npos ||
            f.find("aether_prepare.cpp") != std::string::npos || f.find("aether_allreduce.cpp") != std::string::npos)
          continue;
        std::string src;
        read_file(f, src);
        size_t k = 0;
        while ((k = src.find("aether_", k)) != std::string::npos) {
          size_t j = k;
          while (j < src.size() && is_ident(src[j])) ++j;
          size_t q = j;
          while (q < src.size() && src[q] == ' ') ++q;
          // a definition: at line start after a return type, followed by '(' ... ') {'
          const size_t ls = src.rfind('\n', k);
          const std::string before = src.substr(ls == std::string::npos ? 0 : ls + 1, k - (ls == std::string::npos ? 0 : ls + 1));
          const bool at_def = q < src.size() && src[q] == '(' && !before.empty() && before.find('=') == std::string::npos &&
                              before.find("return") == std::string::npos && before.find('(') == std::string::npos &&
                              before.find(',') == std::string::npos && before.find("//") == std::string::npos &&
                              (k == 0 || !is_ident(src[k - 1])) && std::isalpha((unsigned char)before[0]);
          if (at_def) {
            const size_t close = src.find(')', q);
            const size_t brace = close == std::string::npos ? std::string::npos : src.find_first_not_of(" \n", close + 1);
            if (brace != std::string::npos && src[brace] == '{' && before.find("static") == std::string::npos)
              names.insert(src.substr(k, j - k));
          }
          k = j;
        }
      }
      const std::string path = root + "/aether_b200/" + lib.first;
      void* h = dlopen(path.c_str(), RTLD_NOW | RTLD_LOCAL);
      int found = 0;
      std::vector<std::string> missing;
      for (const std::string& n : names) {
        if (h && dlsym(h, n.c_str())) ++found;
        else missing.push_back(n);
      }
      if (!h) errors.push_back(std::string("cannot load ") + lib.first);
      for (const std::string& m : missing) errors.push_back(std::string(lib.first) + " does not export " + m);
      std::fprintf(stderr, "abi %-18s defined %zu exported %d missing %zu\n", lib.first, names.size(), found,
                   missing.size());
      js += (f1 ? "" : ",") + json_str(lib.first) + ":{\"defined\":" + std::to_string(names.size()) +
            ",\"exported\":" + std::to_string(found) + ",\"missing\":" + std::to_string(missing.size()) + "}";
      f1 = false;
      if (h) dlclose(h);
    }
    js += "}";
  }
  key("errors");
  js += "[";
  for (size_t i = 0; i < errors.size(); ++i) js += (i ? "," : "") + json_str(errors[i]);
  js += "]}";
  for (const std::string& e : errors) std::fprintf(stderr, "error: %s\n", e.c_str());
  if (json) std::printf("%s\n", js.c_str());
  return errors.empty() ? 0 : 1;
}

// ------------------------------------------------------------------ witness-stamper
std::string stamp_tags(const std::string& src, const std::vector<std::string>& tags) {
  std::vector<std::string> lines = split_lines(src);
  int road = -1, expect = -1;
  for (size_t i = 0; i < lines.size() && i < 20; ++i) {
    const std::string t = ltrim(lines[i]);
    if (road < 0 && starts_with(t, "// roadmap:")) road = (int)i;
    if (expect < 0 && starts_with(t, "// expect:")) expect = (int)i;
  }
  std::vector<std::string> have;
  if (road >= 0) {
    std::stringstream ss(lines[road].substr(lines[road].find(':') + 1));
    std::string tok;
    while (std::getline(ss, tok, ',')) {
      tok = ltrim(rtrim(tok));
      if (!tok.empty()) have.push_back(tok);
    }
  }
  bool add = false;
  for (const std::string& t : tags)
    if (std::find(have.begin(), have.end(), t) == have.end()) {
      have.push_back(t);
      add = true;
    }
  if (!add) return src;
  std::string line = "// roadmap: ";
  for (size_t i = 0; i < have.size(); ++i) line += (i ? ", " : "") + have[i];
  if (road >= 0) lines[road] = line;
  else lines.insert(lines.begin() + (expect >= 0 ? expect + 1 : 0), line);
  std::string r;
  for (const std::string& l : lines) r += l + "\n";
  return r;
}

int main_stamper(const std::vector<std::string>& args) {
  std::string dir = "tests/aether", tags_file, fresh_file;
  bool check = false;
  for (size_t i = 0; i < args.size(); ++i) {
    if (args[i] == "--dir" && i + 1 < args.size()) dir = args[++i];
    else if (args[i] == "--tags" && i + 1 < args.size()) tags_file = args[++i];
    else if (args[i] == "--fresh" && i + 1 < args.size()) fresh_file = args[++i];
    else if (args[i] == "--check") check = true;
    else {
      std::fprintf(stderr, "usage: witness-stamper [--dir DIR] [--tags FILE] [--fresh FILE] [--check]\n");
      return 2;
    }
  }
  if (tags_file.empty() && fresh_file.empty()) {
    std::fprintf(stderr, "witness-stamper: nothing to do (give --tags and/or --fresh)\n");
    return 2;
  }
  int changed = 0;
  if (!tags_file.empty()) {
    std::string spec;
    if (!read_file(tags_file, spec)) {
      std::fprintf(stderr, "witness-stamper: cannot read %s\n", tags_file.c_str());
      return 2;
    }
    std::map<std::string, std::vector<std::string>> want;
    for (const std::string& raw : split_lines(spec)) {
      const std::string t = ltrim(rtrim(raw));
      if (t.empty() || t[0] == '#') continue;
      std::stringstream ss(t);
      std::string file, tag;
      ss >> file >> tag;
      if (!tag.empty()) want[file].push_back(tag);
    }
    for (const auto& kv : want) {
      const std::string p = dir + "/" + kv.first;
      std::string src;
      if (!read_file(p, src)) {
        std::fprintf(stderr, "witness-stamper: no witness %s\n", p.c_str());
        return 2;
      }
      const std::string out = stamp_tags(src, kv.second);
      if (out == src) continue;
      ++changed;
      std::printf("%s %s\n", check ? "would tag" : "tagged", kv.first.c_str());
      if (!check && !write_file(p, out)) return 2;
    }
  }
  if (!fresh_file.empty()) {
    std::string spec;
    if (!read_file(fresh_file, spec)) {
      std::fprintf(stderr, "witness-stamper: cannot read %s\n", fresh_file.c_str());
      return 2;
    }
    std::string name, body;
    auto flush = [&]() -> bool {
      if (name.empty()) return true;
      if (name.find('/') != std::string::npos || name.size() < 8 ||
          name.compare(name.size() - 7, 7, ".aether") != 0) {
        std::fprintf(stderr, "witness-stamper: bad witness name %s\n", name.c_str());
        return false;
      }
      const std::string p = dir + "/" + name;
      std::string old;
      const bool exists = read_file(p, old);
      if (!exists || old != body) {
        ++changed;
        std::printf("%s %s\n", check ? "would write" : "wrote", name.c_str());
        if (!check && !write_file(p, body)) return false;
      }
      name.clear();
      body.clear();
      return true;
    };
    for (const std::string& raw : split_lines(spec)) {
      if (starts_with(raw, "=== ")) {
        if (!flush()) return 2;
        name = ltrim(rtrim(raw.substr(4)));
        continue;
      }
      if (!name.empty()) body += raw + "\n";
    }
    if (!flush()) return 2;
  }
  return check && changed ? 1 : 0;
}

}  // namespace

int main(int argc, char** argv) {
  std::string prog = argv[0];
  const size_t k = prog.rfind('/');
  if (k != std::string::npos) prog = prog.substr(k + 1);
  std::vector<std::string> args(argv + 1, argv + argc);
  if (prog == "aether-tools" && !args.empty()) {  // aether-tools <tool> args...
    prog = args[0];
    args.erase(args.begin());
  }
  if (prog == "aetherfmt") return main_fmt(args);
  if (prog == "aetherclippy") return main_clippy(args);
  if (prog == "aetherdoc") return main_doc(args);
  if (prog == "aether-audit") return main_audit(args);
  if (prog == "witness-stamper") return main_stamper(args);
  std::fprintf(stderr, "usage: aether-tools {aetherfmt|aetherclippy|aetherdoc|aether-audit|witness-stamper} ...\n");
  return 2;
}
