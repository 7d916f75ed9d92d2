// HTTP/2 (RFC 9113) server sessions for cleartext connections with prior
// knowledge (h2c), and HPACK (RFC 7541) header compression. Transport-agnostic
// like the TLS sessions: the caller feeds received bytes in, pops complete
// requests, answers them (headers, then body chunks) and takes bytes to send.
// Flow control in both directions: received DATA is credited back at once;
// outgoing DATA waits for the peer's connection and stream windows, queued per
// stream until WINDOW_UPDATE frames open them.
//
// HPACK: the 61-entry static table, a dynamic table with eviction, every
// representation on decode; the encoder emits literals without indexing
// (Huffman-coded when that is shorter), so it never depends on the peer's
// table state. The Huffman code (RFC 7541 Appendix B) is canonical; its
// table below was read off an HTTP/2 client's encoder output for every byte
// a header value can carry and completed through the canonical ordering (NUL,
// LF, CR, EOS); a test checks that it is a complete prefix code.
//
// Names of the reference's export (runtime/src/http2.rs: the loopback smoke)
// are kept; the session ABI and the code are this library's own.
#include <cstdint>
#include <cstring>
#include <deque>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

namespace {

struct Sym {
  uint32_t code;
  uint8_t len;
};
const Sym HUFF[257] = {
    {0x1ff8u, 13}, {0x7fffd8u, 23}, {0xfffffe2u, 28}, {0xfffffe3u, 28}, {0xfffffe4u, 28}, {0xfffffe5u, 28},
    {0xfffffe6u, 28}, {0xfffffe7u, 28}, {0xfffffe8u, 28}, {0xffffeau, 24}, {0x3ffffffcu, 30}, {0xfffffe9u, 28},
    {0xfffffeau, 28}, {0x3ffffffdu, 30}, {0xfffffebu, 28}, {0xfffffecu, 28}, {0xfffffedu, 28}, {0xfffffeeu, 28},
    {0xfffffefu, 28}, {0xffffff0u, 28}, {0xffffff1u, 28}, {0xffffff2u, 28}, {0x3ffffffeu, 30}, {0xffffff3u, 28},
    {0xffffff4u, 28}, {0xffffff5u, 28}, {0xffffff6u, 28}, {0xffffff7u, 28}, {0xffffff8u, 28}, {0xffffff9u, 28},
    {0xffffffau, 28}, {0xffffffbu, 28}, {0x14u, 6}, {0x3f8u, 10}, {0x3f9u, 10}, {0xffau, 12},
    {0x1ff9u, 13}, {0x15u, 6}, {0xf8u, 8}, {0x7fau, 11}, {0x3fau, 10}, {0x3fbu, 10},
    {0xf9u, 8}, {0x7fbu, 11}, {0xfau, 8}, {0x16u, 6}, {0x17u, 6}, {0x18u, 6},
    {0x0u, 5}, {0x1u, 5}, {0x2u, 5}, {0x19u, 6}, {0x1au, 6}, {0x1bu, 6},
    {0x1cu, 6}, {0x1du, 6}, {0x1eu, 6}, {0x1fu, 6}, {0x5cu, 7}, {0xfbu, 8},
    {0x7ffcu, 15}, {0x20u, 6}, {0xffbu, 12}, {0x3fcu, 10}, {0x1ffau, 13}, {0x21u, 6},
    {0x5du, 7}, {0x5eu, 7}, {0x5fu, 7}, {0x60u, 7}, {0x61u, 7}, {0x62u, 7},
    {0x63u, 7}, {0x64u, 7}, {0x65u, 7}, {0x66u, 7}, {0x67u, 7}, {0x68u, 7},
    {0x69u, 7}, {0x6au, 7}, {0x6bu, 7}, {0x6cu, 7}, {0x6du, 7}, {0x6eu, 7},
    {0x6fu, 7}, {0x70u, 7}, {0x71u, 7}, {0x72u, 7}, {0xfcu, 8}, {0x73u, 7},
    {0xfdu, 8}, {0x1ffbu, 13}, {0x7fff0u, 19}, {0x1ffcu, 13}, {0x3ffcu, 14}, {0x22u, 6},
    {0x7ffdu, 15}, {0x3u, 5}, {0x23u, 6}, {0x4u, 5}, {0x24u, 6}, {0x5u, 5},
    {0x25u, 6}, {0x26u, 6}, {0x27u, 6}, {0x6u, 5}, {0x74u, 7}, {0x75u, 7},
    {0x28u, 6}, {0x29u, 6}, {0x2au, 6}, {0x7u, 5}, {0x2bu, 6}, {0x76u, 7},
    {0x2cu, 6}, {0x8u, 5}, {0x9u, 5}, {0x2du, 6}, {0x77u, 7}, {0x78u, 7},
    {0x79u, 7}, {0x7au, 7}, {0x7bu, 7}, {0x7ffeu, 15}, {0x7fcu, 11}, {0x3ffdu, 14},
    {0x1ffdu, 13}, {0xffffffcu, 28}, {0xfffe6u, 20}, {0x3fffd2u, 22}, {0xfffe7u, 20}, {0xfffe8u, 20},
    {0x3fffd3u, 22}, {0x3fffd4u, 22}, {0x3fffd5u, 22}, {0x7fffd9u, 23}, {0x3fffd6u, 22}, {0x7fffdau, 23},
    {0x7fffdbu, 23}, {0x7fffdcu, 23}, {0x7fffddu, 23}, {0x7fffdeu, 23}, {0xffffebu, 24}, {0x7fffdfu, 23},
    {0xffffecu, 24}, {0xffffedu, 24}, {0x3fffd7u, 22}, {0x7fffe0u, 23}, {0xffffeeu, 24}, {0x7fffe1u, 23},
    {0x7fffe2u, 23}, {0x7fffe3u, 23}, {0x7fffe4u, 23}, {0x1fffdcu, 21}, {0x3fffd8u, 22}, {0x7fffe5u, 23},
    {0x3fffd9u, 22}, {0x7fffe6u, 23}, {0x7fffe7u, 23}, {0xffffefu, 24}, {0x3fffdau, 22}, {0x1fffddu, 21},
    {0xfffe9u, 20}, {0x3fffdbu, 22}, {0x3fffdcu, 22}, {0x7fffe8u, 23}, {0x7fffe9u, 23}, {0x1fffdeu, 21},
    {0x7fffeau, 23}, {0x3fffddu, 22}, {0x3fffdeu, 22}, {0xfffff0u, 24}, {0x1fffdfu, 21}, {0x3fffdfu, 22},
    {0x7fffebu, 23}, {0x7fffecu, 23}, {0x1fffe0u, 21}, {0x1fffe1u, 21}, {0x3fffe0u, 22}, {0x1fffe2u, 21},
    {0x7fffedu, 23}, {0x3fffe1u, 22}, {0x7fffeeu, 23}, {0x7fffefu, 23}, {0xfffeau, 20}, {0x3fffe2u, 22},
    {0x3fffe3u, 22}, {0x3fffe4u, 22}, {0x7ffff0u, 23}, {0x3fffe5u, 22}, {0x3fffe6u, 22}, {0x7ffff1u, 23},
    {0x3ffffe0u, 26}, {0x3ffffe1u, 26}, {0xfffebu, 20}, {0x7fff1u, 19}, {0x3fffe7u, 22}, {0x7ffff2u, 23},
    {0x3fffe8u, 22}, {0x1ffffecu, 25}, {0x3ffffe2u, 26}, {0x3ffffe3u, 26}, {0x3ffffe4u, 26}, {0x7ffffdeu, 27},
    {0x7ffffdfu, 27}, {0x3ffffe5u, 26}, {0xfffff1u, 24}, {0x1ffffedu, 25}, {0x7fff2u, 19}, {0x1fffe3u, 21},
    {0x3ffffe6u, 26}, {0x7ffffe0u, 27}, {0x7ffffe1u, 27}, {0x3ffffe7u, 26}, {0x7ffffe2u, 27}, {0xfffff2u, 24},
    {0x1fffe4u, 21}, {0x1fffe5u, 21}, {0x3ffffe8u, 26}, {0x3ffffe9u, 26}, {0xffffffdu, 28}, {0x7ffffe3u, 27},
    {0x7ffffe4u, 27}, {0x7ffffe5u, 27}, {0xfffecu, 20}, {0xfffff3u, 24}, {0xfffedu, 20}, {0x1fffe6u, 21},
    {0x3fffe9u, 22}, {0x1fffe7u, 21}, {0x1fffe8u, 21}, {0x7ffff3u, 23}, {0x3fffeau, 22}, {0x3fffebu, 22},
    {0x1ffffeeu, 25}, {0x1ffffefu, 25}, {0xfffff4u, 24}, {0xfffff5u, 24}, {0x3ffffeau, 26}, {0x7ffff4u, 23},
    {0x3ffffebu, 26}, {0x7ffffe6u, 27}, {0x3ffffecu, 26}, {0x3ffffedu, 26}, {0x7ffffe7u, 27}, {0x7ffffe8u, 27},
    {0x7ffffe9u, 27}, {0x7ffffeau, 27}, {0x7ffffebu, 27}, {0xffffffeu, 28}, {0x7ffffecu, 27}, {0x7ffffedu, 27},
    {0x7ffffeeu, 27}, {0x7ffffefu, 27}, {0x7fffff0u, 27}, {0x3ffffeeu, 26}, {0x3fffffffu, 30},
};

const char* STATIC[62][2] = {
    {"", ""},
    {":authority", ""}, {":method", "GET"}, {":method", "POST"}, {":path", "/"}, {":path", "/index.html"},
    {":scheme", "http"}, {":scheme", "https"}, {":status", "200"}, {":status", "204"}, {":status", "206"},
    {":status", "304"}, {":status", "400"}, {":status", "404"}, {":status", "500"}, {"accept-charset", ""},
    {"accept-encoding", "gzip, deflate"}, {"accept-language", ""}, {"accept-ranges", ""}, {"accept", ""},
    {"access-control-allow-origin", ""}, {"age", ""}, {"allow", ""}, {"authorization", ""},
    {"cache-control", ""}, {"content-disposition", ""}, {"content-encoding", ""}, {"content-language", ""},
    {"content-length", ""}, {"content-location", ""}, {"content-range", ""}, {"content-type", ""},
    {"cookie", ""}, {"date", ""}, {"etag", ""}, {"expect", ""}, {"expires", ""}, {"from", ""}, {"host", ""},
    {"if-match", ""}, {"if-modified-since", ""}, {"if-none-match", ""}, {"if-range", ""},
    {"if-unmodified-since", ""}, {"last-modified", ""}, {"link", ""}, {"location", ""}, {"max-forwards", ""},
    {"proxy-authenticate", ""}, {"proxy-authorization", ""}, {"range", ""}, {"referer", ""}, {"refresh", ""},
    {"retry-after", ""}, {"server", ""}, {"set-cookie", ""}, {"strict-transport-security", ""},
    {"transfer-encoding", ""}, {"user-agent", ""}, {"vary", ""}, {"via", ""}, {"www-authenticate", ""}};

typedef std::vector<uint8_t> Bytes;
typedef std::vector<std::pair<std::string, std::string>> Headers;

// ------------------------------------------------------------------------------------------------ Huffman
// Canonical decoding: symbols sorted by (length, symbol); per length the first
// code and its position in that order.
struct HuffDec {
  uint16_t order[257];
  uint32_t first[31];
  int first_pos[31], count[31];
  HuffDec() {
    int n = 0;
    for (int L = 1; L <= 30; ++L) {
      first_pos[L] = n;
      count[L] = 0;
      for (int s = 0; s < 257; ++s)
        if (HUFF[s].len == L) {
          if (!count[L]) first[L] = HUFF[s].code;
          order[n++] = (uint16_t)s;
          ++count[L];
        }
    }
  }
};
const HuffDec& huff_dec() {
  static HuffDec d;
  return d;
}

bool huff_decode(const uint8_t* p, size_t n, std::string& out) {
  const HuffDec& d = huff_dec();
  uint32_t code = 0;
  int len = 0;
  for (size_t i = 0; i < n; ++i)
    for (int b = 7; b >= 0; --b) {
      code = code << 1 | ((p[i] >> b) & 1);
      ++len;
      if (len > 30) return false;
      if (d.count[len] && code >= d.first[len] && code < d.first[len] + (uint32_t)d.count[len]) {
        const int s = d.order[d.first_pos[len] + (code - d.first[len])];
        if (s == 256) return false;  // EOS inside a string
        out.push_back((char)s);
        code = 0;
        len = 0;
      }
    }
  // at most 7 padding bits, all ones (a prefix of EOS)
  return len <= 7 && code == (1u << len) - 1;
}

Bytes huff_encode(const std::string& s) {
  Bytes out;
  uint64_t acc = 0;
  int bits = 0;
  for (unsigned char c : s) {
    acc = acc << HUFF[c].len | HUFF[c].code;
    bits += HUFF[c].len;
    while (bits >= 8) {
      out.push_back((uint8_t)(acc >> (bits - 8)));
      bits -= 8;
    }
  }
  if (bits) out.push_back((uint8_t)((acc << (8 - bits)) | ((1u << (8 - bits)) - 1)));
  return out;
}

size_t huff_len(const std::string& s) {
  size_t b = 0;
  for (unsigned char c : s) b += HUFF[c].len;
  return (b + 7) / 8;
}

// ------------------------------------------------------------------------------------------------ HPACK
void put_int(Bytes& b, uint8_t first, int prefix, uint64_t v) {
  const uint64_t m = (1u << prefix) - 1;
  if (v < m) {
    b.push_back((uint8_t)(first | v));
    return;
  }
  b.push_back((uint8_t)(first | m));
  v -= m;
  while (v >= 128) {
    b.push_back((uint8_t)(v & 127) | 128);
    v >>= 7;
  }
  b.push_back((uint8_t)v);
}
void put_str(Bytes& b, const std::string& s) {
  if (huff_len(s) < s.size()) {
    const Bytes h = huff_encode(s);
    put_int(b, 0x80, 7, h.size());
    b.insert(b.end(), h.begin(), h.end());
  } else {
    put_int(b, 0, 7, s.size());
    b.insert(b.end(), s.begin(), s.end());
  }
}
int static_name(const std::string& name) {
  for (int i = 1; i <= 61; ++i)
    if (name == STATIC[i][0]) return i;
  return 0;
}
// Header block: indexed fields for exact static matches, otherwise literals without indexing.
Bytes hpack_encode(const Headers& hs) {
  Bytes b;
  for (auto& h : hs) {
    int exact = 0;
    for (int i = 1; i <= 61 && !exact; ++i)
      if (h.first == STATIC[i][0] && h.second == STATIC[i][1]) exact = i;
    if (exact) {
      put_int(b, 0x80, 7, exact);
      continue;
    }
    const int ni = static_name(h.first);
    put_int(b, 0x00, 4, ni);
    if (!ni) put_str(b, h.first);
    put_str(b, h.second);
  }
  return b;
}

struct HpackDecoder {
  std::deque<std::pair<std::string, std::string>> dyn;  // newest first
  size_t size = 0, max_size = 4096, limit = 4096;
  void evict() {
    while (size > max_size && !dyn.empty()) {
      size -= dyn.back().first.size() + dyn.back().second.size() + 32;
      dyn.pop_back();
    }
  }
  void add(const std::string& n, const std::string& v) {
    const size_t s = n.size() + v.size() + 32;
    if (s > max_size) {
      dyn.clear();
      size = 0;
      return;
    }
    dyn.emplace_front(n, v);
    size += s;
    evict();
  }
  bool entry(uint64_t i, std::string& n, std::string& v) {
    if (i >= 1 && i <= 61) {
      n = STATIC[i][0];
      v = STATIC[i][1];
      return true;
    }
    if (i > 61 && i - 62 < dyn.size()) {
      n = dyn[i - 62].first;
      v = dyn[i - 62].second;
      return true;
    }
    return false;
  }
  static bool get_int(const uint8_t* p, size_t n, size_t& i, int prefix, uint64_t& v) {
    if (i >= n) return false;
    const uint64_t m = (1u << prefix) - 1;
    v = p[i++] & m;
    if (v < m) return true;
    for (int sh = 0; sh < 56; sh += 7) {
      if (i >= n) return false;
      const uint8_t x = p[i++];
      v += (uint64_t)(x & 127) << sh;
      if (!(x & 128)) return true;
    }
    return false;
  }
  static bool get_str(const uint8_t* p, size_t n, size_t& i, std::string& s) {
    if (i >= n) return false;
    const bool h = p[i] & 0x80;
    uint64_t len;
    if (!get_int(p, n, i, 7, len) || len > n - i) return false;
    s.clear();
    const bool ok = h ? huff_decode(p + i, len, s) : (s.assign((const char*)p + i, len), true);
    i += len;
    return ok;
  }
  bool decode(const uint8_t* p, size_t n, Headers& out) {
    size_t i = 0;
    while (i < n) {
      const uint8_t b = p[i];
      uint64_t idx;
      std::string name, value;
      if (b & 0x80) {
        if (!get_int(p, n, i, 7, idx) || !entry(idx, name, value)) return false;
        out.emplace_back(name, value);
      } else if ((b & 0xE0) == 0x20) {
        if (!get_int(p, n, i, 5, idx) || idx > limit) return false;
        max_size = idx;
        evict();
      } else {
        const bool incr = b & 0x40;
        if (!get_int(p, n, i, incr ? 6 : 4, idx)) return false;
        if (idx) {
          std::string unused;
          if (!entry(idx, name, unused)) return false;
        } else if (!get_str(p, n, i, name)) {
          return false;
        }
        if (!get_str(p, n, i, value)) return false;
        if (incr) add(name, value);
        out.emplace_back(name, value);
      }
    }
    return true;
  }
};

// ------------------------------------------------------------------------------------------------ frames
enum : uint8_t { F_DATA = 0, F_HEADERS = 1, F_PRIORITY = 2, F_RST = 3, F_SETTINGS = 4, F_PUSH = 5, F_PING = 6,
                 F_GOAWAY = 7, F_WINDOW = 8, F_CONT = 9 };
const char PREFACE[] = "PRI * HTTP/2.0\r\n\r\nSM\r\n\r\n";

struct Stream {
  Headers req;
  Bytes block, body;
  bool headers_done = false, complete = false, queued = false;
  int64_t send_window = 65535;
  Bytes pending;  // response DATA waiting for window
  bool end_after_pending = false;
};

struct Session {
  Bytes in, out;
  bool preface = false, failed = false, goaway = false;
  HpackDecoder dec;
  std::map<uint32_t, Stream> streams;
  std::deque<uint32_t> ready;
  uint32_t cont_stream = 0, last_stream = 0;
  int64_t conn_window = 65535, init_window = 65535;
  uint32_t max_frame = 16384;

  void frame(uint8_t type, uint8_t flags, uint32_t sid, const uint8_t* p, size_t n) {
    out.push_back((uint8_t)(n >> 16));
    out.push_back((uint8_t)(n >> 8));
    out.push_back((uint8_t)n);
    out.push_back(type);
    out.push_back(flags);
    for (int s = 24; s >= 0; s -= 8) out.push_back((uint8_t)(sid >> s));
    out.insert(out.end(), p, p + n);
  }
  void window_update(uint32_t sid, uint32_t inc) {
    const uint8_t b[4] = {(uint8_t)(inc >> 24), (uint8_t)(inc >> 16), (uint8_t)(inc >> 8), (uint8_t)inc};
    frame(F_WINDOW, 0, sid, b, 4);
  }
  void fail(uint32_t code) {
    uint8_t b[8] = {(uint8_t)(last_stream >> 24), (uint8_t)(last_stream >> 16), (uint8_t)(last_stream >> 8),
                    (uint8_t)last_stream, (uint8_t)(code >> 24), (uint8_t)(code >> 16), (uint8_t)(code >> 8),
                    (uint8_t)code};
    frame(F_GOAWAY, 0, 0, b, 8);
    failed = true;
  }
  void start() {
    const uint8_t s[] = {0, 3, 0, 0, 0, 100};  // MAX_CONCURRENT_STREAMS 100
    frame(F_SETTINGS, 0, 0, s, sizeof(s));
  }
  // Sends as much pending DATA of stream sid as the windows allow.
  void flush(uint32_t sid) {
    auto it = streams.find(sid);
    if (it == streams.end()) return;
    Stream& st = it->second;
    while (!st.pending.empty()) {
      const int64_t room = std::min<int64_t>(std::min(conn_window, st.send_window), max_frame);
      if (room <= 0) return;
      const size_t n = std::min<size_t>(st.pending.size(), (size_t)room);
      const bool last = n == st.pending.size() && st.end_after_pending;
      frame(F_DATA, last ? 1 : 0, sid, st.pending.data(), n);
      st.pending.erase(st.pending.begin(), st.pending.begin() + n);
      conn_window -= n;
      st.send_window -= n;
      if (last) {
        streams.erase(it);
        return;
      }
    }
    if (st.end_after_pending) {  // an empty final chunk
      frame(F_DATA, 1, sid, nullptr, 0);
      streams.erase(it);
    }
  }
  void flush_all() {
    std::vector<uint32_t> ids;
    for (auto& kv : streams) ids.push_back(kv.first);
    for (uint32_t id : ids) flush(id);
  }
  bool headers_complete(uint32_t sid, Stream& st, bool end_stream) {
    Headers hs;
    if (!dec.decode(st.block.data(), st.block.size(), hs)) return false;
    st.block.clear();
    st.req.insert(st.req.end(), hs.begin(), hs.end());
    st.headers_done = true;
    if (end_stream) mark_complete(sid, st);
    return true;
  }
  void mark_complete(uint32_t sid, Stream& st) {
    st.complete = true;
    if (!st.queued) {
      st.queued = true;
      ready.push_back(sid);
    }
  }
  bool on_frame(uint8_t type, uint8_t flags, uint32_t sid, const uint8_t* p, size_t n) {
    if (cont_stream && (type != F_CONT || sid != cont_stream)) return false;
    switch (type) {
      case F_SETTINGS: {
        if (sid) return false;
        if (flags & 1) return n == 0;
        if (n % 6) return false;
        for (size_t i = 0; i < n; i += 6) {
          const uint16_t id = (uint16_t)(p[i] << 8 | p[i + 1]);
          const uint32_t v = (uint32_t)p[i + 2] << 24 | (uint32_t)p[i + 3] << 16 | (uint32_t)p[i + 4] << 8 | p[i + 5];
          if (id == 4) {  // initial window: shifts every open stream's window
            if (v > 0x7fffffff) return false;
            for (auto& kv : streams) kv.second.send_window += (int64_t)v - init_window;
            init_window = v;
          } else if (id == 5) {
            if (v < 16384 || v > 16777215) return false;
            max_frame = v;
          }
        }
        frame(F_SETTINGS, 1, 0, nullptr, 0);
        flush_all();
        return true;
      }
      case F_PING:
        if (sid || n != 8) return false;
        if (!(flags & 1)) frame(F_PING, 1, 0, p, 8);
        return true;
      case F_WINDOW: {
        if (n != 4) return false;
        const uint32_t inc = ((uint32_t)p[0] << 24 | (uint32_t)p[1] << 16 | (uint32_t)p[2] << 8 | p[3]) & 0x7fffffff;
        if (!inc) return false;
        if (sid == 0) {
          conn_window += inc;
          flush_all();
        } else if (streams.count(sid)) {
          streams[sid].send_window += inc;
          flush(sid);
        }
        return true;
      }
      case F_HEADERS: {
        if (!sid || !(sid & 1)) return false;
        size_t off = 0, pad = 0;
        if (flags & 0x8) {
          if (n < 1) return false;
          pad = p[0];
          off = 1;
        }
        if (flags & 0x20) off += 5;
        if (off + pad > n) return false;
        if (!streams.count(sid)) {
          if (sid <= last_stream) return false;  // stream ids only increase
          last_stream = sid;
          streams[sid].send_window = init_window;
        }
        Stream& st = streams[sid];
        st.block.insert(st.block.end(), p + off, p + n - pad);
        if (flags & 0x4) return headers_complete(sid, st, flags & 1);
        cont_stream = sid;
        if (flags & 1) st.end_after_pending = true;  // END_STREAM arrives before the CONTINUATIONs end
        return true;
      }
      case F_CONT: {
        if (sid != cont_stream) return false;
        Stream& st = streams[sid];
        st.block.insert(st.block.end(), p, p + n);
        if (!(flags & 0x4)) return true;
        cont_stream = 0;
        const bool end = st.end_after_pending;
        st.end_after_pending = false;
        return headers_complete(sid, st, end);
      }
      case F_DATA: {
        if (!sid) return false;
        size_t off = 0, pad = 0;
        if (flags & 0x8) {
          if (n < 1) return false;
          pad = p[0];
          off = 1;
        }
        if (off + pad > n) return false;
        if (n) {
          window_update(0, (uint32_t)n);
          if (!(flags & 1)) window_update(sid, (uint32_t)n);
        }
        auto it = streams.find(sid);
        if (it == streams.end() || !it->second.headers_done) return true;  // closed or reset: drop
        it->second.body.insert(it->second.body.end(), p + off, p + n - pad);
        if (flags & 1) mark_complete(sid, it->second);
        return true;
      }
      case F_RST:
        streams.erase(sid);
        return true;
      case F_GOAWAY:
        goaway = true;
        return true;
      case F_PRIORITY:
        return true;
      default:
        return true;  // unknown frame types are ignored
    }
  }
  bool drain() {
    if (!preface) {
      if (in.size() < 24) return true;
      if (memcmp(in.data(), PREFACE, 24)) return false;
      in.erase(in.begin(), in.begin() + 24);
      preface = true;
    }
    size_t i = 0;
    while (in.size() - i >= 9) {
      const size_t n = (size_t)in[i] << 16 | (size_t)in[i + 1] << 8 | in[i + 2];
      if (n > 16384) return false;  // we never raise SETTINGS_MAX_FRAME_SIZE
      if (in.size() - i < 9 + n) break;
      const uint32_t sid =
          ((uint32_t)in[i + 5] << 24 | (uint32_t)in[i + 6] << 16 | (uint32_t)in[i + 7] << 8 | in[i + 8]) & 0x7fffffff;
      if (!on_frame(in[i + 3], in[i + 4], sid, in.data() + i + 9, n)) return false;
      i += 9 + n;
    }
    in.erase(in.begin(), in.begin() + i);
    return true;
  }
  void respond_headers(uint32_t sid, const Headers& hs, bool end) {
    const Bytes block = hpack_encode(hs);
    size_t off = 0;
    bool first = true;
    do {  // HEADERS, then CONTINUATION frames of at most max_frame bytes
      const size_t n = std::min<size_t>(block.size() - off, max_frame);
      const bool last = off + n == block.size();
      const uint8_t flags = (uint8_t)((last ? 4 : 0) | (first && end ? 1 : 0));
      frame(first ? F_HEADERS : F_CONT, flags, sid, block.data() + off, n);
      off += n;
      first = false;
    } while (off < block.size());
  }
};

std::mutex g_mu;
std::vector<std::unique_ptr<Session>> g_sessions;

Session* get(int64_t h) {
  std::lock_guard<std::mutex> l(g_mu);
  return (h >= 0 && (size_t)h < g_sessions.size()) ? g_sessions[h].get() : nullptr;
}

// "name: value\n" lines -> header list (lower-cased names, as HTTP/2 requires).
bool parse_lines(const char* p, int n, Headers& out) {
  std::string s(p ? p : "", p ? n : 0);
  size_t i = 0;
  while (i < s.size()) {
    size_t e = s.find('\n', i);
    if (e == std::string::npos) e = s.size();
    const std::string line = s.substr(i, e - i);
    i = e + 1;
    if (line.empty()) continue;
    const size_t c = line.find(':', 1);
    if (c == std::string::npos) return false;
    std::string name = line.substr(0, c), value = line.substr(c + 1);
    while (!value.empty() && value[0] == ' ') value.erase(0, 1);
    for (auto& ch : name) ch = (char)tolower((unsigned char)ch);
    out.emplace_back(name, value);
  }
  return true;
}

}  // namespace

extern "C" {

// A server session for one h2c connection; its SETTINGS are queued at once.
int64_t aether_h2_server_new() {
  auto s = std::make_unique<Session>();
  s->start();
  std::lock_guard<std::mutex> l(g_mu);
  for (size_t i = 0; i < g_sessions.size(); ++i)
    if (!g_sessions[i]) {
      g_sessions[i] = std::move(s);
      return (int64_t)i;
    }
  g_sessions.push_back(std::move(s));
  return (int64_t)g_sessions.size() - 1;
}
int aether_h2_server_free(int64_t h) {
  std::lock_guard<std::mutex> l(g_mu);
  if (h < 0 || (size_t)h >= g_sessions.size() || !g_sessions[h]) return -1;
  g_sessions[h].reset();
  return 0;
}
// Received bytes in; returns the number of complete requests waiting, -1 on a
// protocol error (a GOAWAY is queued and the session is dead), -2 on a bad handle.
int aether_h2_server_feed(int64_t h, const void* in, int n) {
  Session* s = get(h);
  if (!s) return -2;
  if (s->failed || n < 0 || (n && !in)) return -1;
  s->in.insert(s->in.end(), (const uint8_t*)in, (const uint8_t*)in + n);
  if (!s->drain()) {
    s->fail(1);  // PROTOCOL_ERROR
    return -1;
  }
  return (int)s->ready.size();
}
// Pops the oldest complete request: its stream id, "METHOD PATH\n" followed by
// "name: value\n" lines (":authority" as "host"), and its body. 1 when one was
// popped, 0 when none waits, -1 when a buffer is too small (nothing popped).
int aether_h2_server_next_request(int64_t h, int* stream, char* head, int max_head, int* head_len, void* body,
                                  int max_body, int* body_len) {
  Session* s = get(h);
  if (!s) return -2;
  if (!stream || !head || !head_len || !body_len || (max_body > 0 && !body)) return -1;
  if (s->ready.empty()) return 0;
  const uint32_t sid = s->ready.front();
  Stream& st = s->streams[sid];
  std::string method, path, lines;
  for (auto& kv : st.req) {
    if (kv.first == ":method") method = kv.second;
    else if (kv.first == ":path") path = kv.second;
    else if (kv.first == ":authority") lines += "host: " + kv.second + "\n";
    else if (kv.first[0] != ':') lines += kv.first + ": " + kv.second + "\n";
  }
  const std::string text = method + " " + path + "\n" + lines;
  if ((int)text.size() > max_head || (int)st.body.size() > max_body) return -1;
  memcpy(head, text.data(), text.size());
  if (!st.body.empty()) memcpy(body, st.body.data(), st.body.size());
  *stream = (int)sid;
  *head_len = (int)text.size();
  *body_len = (int)st.body.size();
  s->ready.pop_front();
  st.req.clear();
  st.body.clear();
  return 1;
}
// Response headers for a stream: status and "name: value\n" lines; end = 1
// when no body follows.
int aether_h2_server_respond(int64_t h, int stream, int status, const char* headers, int n_headers, int end) {
  Session* s = get(h);
  if (!s) return -2;
  auto it = s->streams.find((uint32_t)stream);
  if (it == s->streams.end() || status < 100 || status > 999 || n_headers < 0) return -1;
  Headers hs{{":status", std::to_string(status)}};
  if (!parse_lines(headers, n_headers, hs)) return -1;
  s->respond_headers((uint32_t)stream, hs, end != 0);
  if (end) s->streams.erase(it);
  return 0;
}
// A body chunk for a stream (end = 1 on the last one); sent as the windows allow.
int aether_h2_server_data(int64_t h, int stream, const void* data, int n, int end) {
  Session* s = get(h);
  if (!s) return -2;
  auto it = s->streams.find((uint32_t)stream);
  if (it == s->streams.end() || n < 0 || (n && !data)) return -1;
  it->second.pending.insert(it->second.pending.end(), (const uint8_t*)data, (const uint8_t*)data + n);
  if (end) it->second.end_after_pending = true;
  s->flush((uint32_t)stream);
  return n;
}
int aether_h2_server_take_outbound(int64_t h, void* out, int max_out) {
  Session* s = get(h);
  if (!s) return -2;
  if (!out || max_out < 0) return -1;
  const int n = (int)std::min<size_t>(s->out.size(), (size_t)max_out);
  memcpy(out, s->out.data(), n);
  s->out.erase(s->out.begin(), s->out.begin() + n);
  return n;
}

// HPACK Huffman coding of a byte string; returns the output length or -1.
int aether_hpack_huffman_encode(const void* in, int n, void* out, int max_out) {
  if (n < 0 || (n && !in) || !out) return -1;
  const Bytes b = huff_encode(std::string((const char*)in, n));
  if ((int)b.size() > max_out) return -1;
  memcpy(out, b.data(), b.size());
  return (int)b.size();
}
int aether_hpack_huffman_decode(const void* in, int n, void* out, int max_out) {
  if (n < 0 || (n && !in) || !out) return -1;
  std::string s;
  if (!huff_decode((const uint8_t*)in, n, s) || (int)s.size() > max_out) return -1;
  memcpy(out, s.data(), s.size());
  return (int)s.size();
}
// The code of one symbol (0..256) and its length in bits.
int aether_hpack_huffman_code(int sym, uint32_t* code) {
  if (sym < 0 || sym > 256 || !code) return -1;
  *code = HUFF[sym].code;
  return HUFF[sym].len;
}
// Header block of "name: value\n" lines -> HPACK bytes; and back (a fresh
// decoder each call). Return lengths, -1 on errors.
int aether_hpack_encode(const char* lines, int n, void* out, int max_out) {
  Headers hs;
  if (n < 0 || !out || !parse_lines(lines, n, hs)) return -1;
  const Bytes b = hpack_encode(hs);
  if ((int)b.size() > max_out) return -1;
  memcpy(out, b.data(), b.size());
  return (int)b.size();
}
int aether_hpack_decode(const void* in, int n, char* out, int max_out) {
  if (n < 0 || (n && !in) || !out) return -1;
  HpackDecoder d;
  Headers hs;
  if (!d.decode((const uint8_t*)in, n, hs)) return -1;
  std::string s;
  for (auto& kv : hs) s += kv.first + ": " + kv.second + "\n";
  if ((int)s.size() > max_out) return -1;
  memcpy(out, s.data(), s.size());
  return (int)s.size();
}

// In-process client bytes -> server session -> response -> parsed back: 42 on success.
int aether_http2_self_loopback_smoke() {
  const int64_t h = aether_h2_server_new();
  Bytes c(PREFACE, PREFACE + 24);
  auto frame = [&](uint8_t type, uint8_t flags, uint32_t sid, const Bytes& p) {
    c.push_back((uint8_t)(p.size() >> 16));
    c.push_back((uint8_t)(p.size() >> 8));
    c.push_back((uint8_t)p.size());
    c.push_back(type);
    c.push_back(flags);
    for (int s = 24; s >= 0; s -= 8) c.push_back((uint8_t)(sid >> s));
    c.insert(c.end(), p.begin(), p.end());
  };
  frame(F_SETTINGS, 0, 0, {});
  frame(F_HEADERS, 4, 1,
        hpack_encode({{":method", "POST"}, {":scheme", "http"}, {":path", "/v1/echo"}, {":authority", "local"}}));
  frame(F_DATA, 1, 1, Bytes{'p', 'i', 'n', 'g'});
  int rc = 1;
  if (aether_h2_server_feed(h, c.data(), (int)c.size()) == 1) {
    int sid, hl, bl;
    char head[256];
    char body[64];
    if (aether_h2_server_next_request(h, &sid, head, sizeof(head), &hl, body, sizeof(body), &bl) == 1 && bl == 4 &&
        !memcmp(body, "ping", 4) && std::string(head, hl).rfind("POST /v1/echo\n", 0) == 0) {
      aether_h2_server_respond(h, sid, 200, "content-type: text/plain\n", 25, 0);
      aether_h2_server_data(h, sid, "pong", 4, 1);
      uint8_t out[4096];
      const int n = aether_h2_server_take_outbound(h, out, sizeof(out));
      // the last frame is DATA "pong" with END_STREAM on stream 1
      rc = (n >= 13 && out[n - 13 + 3] == F_DATA && (out[n - 13 + 4] & 1) && !memcmp(out + n - 4, "pong", 4)) ? 42 : 3;
    } else {
      rc = 2;
    }
  }
  aether_h2_server_free(h);
  return rc;
}

}  // extern "C"
