// libaether_rt: chat templates (a Jinja subset) and tool-call rendering.
//
// Reference ABI (runtime/src/lib.rs:5304-5530, 9694-9725):
//   aether_template_new / _free / _set_var / _push_message / _render /
//   _render_from_file, aether_tool_render_call.
// Supported template language, as in the reference:
//   {{ name }}             a variable set with _set_var ("" when undefined)
//   {{ m.role }} / .content  a field of the message of the enclosing loop
//   {% for m in messages %} ... {% endfor %}
//   {% if expr %} ... {% endif %}   expr is true when it resolves to a
//                          non-empty string other than "0" / "false"
// The template is parsed once into a node tree (text, expression, loop,
// conditional) and the tree is rendered; a malformed template (unclosed
// tag, stray end tag, unknown directive, a loop over anything but
// `messages`) is an error (-1). The full Jinja dialect of Hugging Face chat
// templates is rendered by aether_b200.serving.templates (jinja2).
#include <cctype>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <mutex>
#include <sstream>
#include <string>
#include <utility>
#include <vector>

#define AE_API extern "C" __attribute__((visibility("default")))

namespace {

struct Ctx {
  std::map<std::string, std::string> vars;
  std::vector<std::pair<std::string, std::string>> messages;  // (role, content)
};

std::mutex g_mu;
std::vector<std::unique_ptr<Ctx>> g_ctx;

Ctx* get(int64_t h) {
  if (h < 0 || (size_t)h >= g_ctx.size()) return nullptr;
  return g_ctx[(size_t)h].get();
}

struct Node {
  enum Kind { Text, Expr, For, If } kind;
  std::string s;  // text, expression, or condition
  std::vector<Node> body;
};

std::string trim(const std::string& x) {
  size_t a = 0, b = x.size();
  while (a < b && (x[a] == ' ' || x[a] == '\t' || x[a] == '\n' || x[a] == '\r' || x[a] == '-')) ++a;
  while (b > a && (x[b - 1] == ' ' || x[b - 1] == '\t' || x[b - 1] == '\n' || x[b - 1] == '\r' || x[b - 1] == '-'))
    --b;
  return x.substr(a, b - a);
}

// Parses tpl[pos..] into `out` until an end tag named `until` (or the end of
// the input when `until` is empty). Returns false on a malformed template.
bool parse(const std::string& tpl, size_t& pos, std::vector<Node>& out, const std::string& until) {
  while (pos < tpl.size()) {
    const size_t e = tpl.find("{{", pos), d = tpl.find("{%", pos);
    const size_t next = std::min(e, d);
    if (next == std::string::npos) {
      out.push_back({Node::Text, tpl.substr(pos), {}});
      pos = tpl.size();
      break;
    }
    if (next > pos) out.push_back({Node::Text, tpl.substr(pos, next - pos), {}});
    const bool is_expr = next == e;
    const size_t close = tpl.find(is_expr ? "}}" : "%}", next + 2);
    if (close == std::string::npos) return false;
    const std::string inner = trim(tpl.substr(next + 2, close - next - 2));
    pos = close + 2;
    if (is_expr) {
      out.push_back({Node::Expr, inner, {}});
      continue;
    }
    if (inner == "endfor" || inner == "endif") {
      if (inner != until) return false;
      return true;
    }
    if (inner.rfind("for ", 0) == 0) {
      // only `for <name> in messages`
      const size_t in = inner.find(" in ");
      if (in == std::string::npos || trim(inner.substr(in + 4)) != "messages") return false;
      Node n{Node::For, trim(inner.substr(4, in - 4)), {}};
      if (!parse(tpl, pos, n.body, "endfor")) return false;
      out.push_back(std::move(n));
    } else if (inner.rfind("if ", 0) == 0) {
      Node n{Node::If, trim(inner.substr(3)), {}};
      if (!parse(tpl, pos, n.body, "endif")) return false;
      out.push_back(std::move(n));
    } else {
      return false;  // unknown directive
    }
  }
  return until.empty();
}

std::string resolve(const std::string& expr, const Ctx& c, const std::pair<std::string, std::string>* msg) {
  const size_t dot = expr.find('.');
  if (dot != std::string::npos) {
    if (!msg) return std::string();
    const std::string field = trim(expr.substr(dot + 1));
    if (field == "role") return msg->first;
    if (field == "content") return msg->second;
    return std::string();
  }
  auto it = c.vars.find(expr);
  return it == c.vars.end() ? std::string() : it->second;
}

bool truthy(const std::string& v) {
  if (v.empty() || v == "0") return false;
  std::string l = v;
  for (auto& ch : l) ch = (char)std::tolower((unsigned char)ch);
  return l != "false";
}

void render(const std::vector<Node>& nodes, const Ctx& c, const std::pair<std::string, std::string>* msg,
            std::string& out) {
  for (const Node& n : nodes) {
    switch (n.kind) {
      case Node::Text: out += n.s; break;
      case Node::Expr: out += resolve(n.s, c, msg); break;
      case Node::For:
        for (const auto& m : c.messages) render(n.body, c, &m, out);
        break;
      case Node::If:
        if (truthy(resolve(n.s, c, msg))) render(n.body, c, msg, out);
        break;
    }
  }
}

bool utf8_arg(const void* p, int n, std::string& s, bool allow_empty) {
  if (!p || n < 0 || (!allow_empty && n == 0)) return false;
  s.assign(static_cast<const char*>(p), (size_t)n);
  return true;
}

int render_to(int64_t handle, const std::string& tpl, void* out, int max_out) {
  std::lock_guard<std::mutex> g(g_mu);
  const Ctx* c = get(handle);
  if (!c || !out || max_out <= 0) return -1;
  std::vector<Node> nodes;
  size_t pos = 0;
  if (!parse(tpl, pos, nodes, "")) return -1;
  std::string s;
  render(nodes, *c, nullptr, s);
  if (s.size() > (size_t)max_out) return -1;
  std::memcpy(out, s.data(), s.size());
  return (int)s.size();
}

void json_escape(const std::string& in, std::string& out) {
  for (unsigned char ch : in) {
    switch (ch) {
      case '"': out += "\\\""; break;
      case '\\': out += "\\\\"; break;
      case '\n': out += "\\n"; break;
      case '\r': out += "\\r"; break;
      case '\t': out += "\\t"; break;
      default:
        if (ch < 0x20) {
          char buf[8];
          std::snprintf(buf, sizeof(buf), "\\u%04x", ch);
          out += buf;
        } else {
          out += (char)ch;
        }
    }
  }
}

}  // namespace

extern "C" {

AE_API int64_t aether_template_new() {
  std::lock_guard<std::mutex> g(g_mu);
  for (size_t i = 0; i < g_ctx.size(); ++i)
    if (!g_ctx[i]) {
      g_ctx[i] = std::make_unique<Ctx>();
      return (int64_t)i;
    }
  g_ctx.push_back(std::make_unique<Ctx>());
  return (int64_t)g_ctx.size() - 1;
}

AE_API int aether_template_free(int64_t handle) {
  std::lock_guard<std::mutex> g(g_mu);
  if (!get(handle)) return -1;
  g_ctx[(size_t)handle].reset();
  return 0;
}

AE_API int aether_template_set_var(int64_t handle, const void* name, int n_name, const void* value, int n_value) {
  std::string k, v;
  if (!utf8_arg(name, n_name, k, false) || !utf8_arg(value, n_value, v, true)) return -1;
  std::lock_guard<std::mutex> g(g_mu);
  Ctx* c = get(handle);
  if (!c) return -1;
  c->vars[k] = v;
  return 0;
}

AE_API int aether_template_push_message(int64_t handle, const void* role, int n_role, const void* content,
                                        int n_content) {
  std::string r, t;
  if (!utf8_arg(role, n_role, r, false) || !utf8_arg(content, n_content, t, true)) return -1;
  std::lock_guard<std::mutex> g(g_mu);
  Ctx* c = get(handle);
  if (!c) return -1;
  c->messages.emplace_back(r, t);
  return 0;
}

AE_API int aether_template_render(int64_t handle, const void* tpl, int n_tpl, void* out, int max_out) {
  std::string t;
  if (!utf8_arg(tpl, n_tpl, t, false)) return -1;
  return render_to(handle, t, out, max_out);
}

AE_API int aether_template_render_from_file(int64_t handle, int64_t path, int n_path, void* out, int max_out) {
  std::string p;
  if (path == 0 || !utf8_arg(reinterpret_cast<const void*>(path), n_path, p, false)) return -1;
  std::ifstream f(p, std::ios::binary);
  if (!f) return -1;
  std::stringstream ss;
  ss << f.rdbuf();
  const std::string t = ss.str();
  if (t.empty()) return -1;
  return render_to(handle, t, out, max_out);
}

// {"type":"function","function":{"name":NAME,"arguments":ARGS}} with ARGS (a
// JSON text) carried as a JSON string, the OpenAI tool-call shape.
AE_API int aether_tool_render_call(const void* name, int n_name, const void* args, int n_args, void* out,
                                   int max_out) {
  std::string n, a;
  if (!utf8_arg(name, n_name, n, false) || !utf8_arg(args, n_args, a, true) || !out || max_out <= 0) return -1;
  std::string s = "{\"type\":\"function\",\"function\":{\"name\":\"";
  json_escape(n, s);
  s += "\",\"arguments\":\"";
  json_escape(a, s);
  s += "\"}}";
  if (s.size() > (size_t)max_out) return -1;
  std::memcpy(out, s.data(), s.size());
  return (int)s.size();
}

}  // extern "C"
