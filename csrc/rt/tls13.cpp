// TLS 1.3 (RFC 8446) client and server sessions, transport-agnostic: the
// caller feeds received bytes in and takes bytes to send out. Profile:
// TLS_CHACHA20_POLY1305_SHA256, X25519 key exchange, Ed25519 signatures, no
// HelloRetryRequest / PSK / 0-RTT. The server presents a self-signed Ed25519
// X.509 certificate that it builds itself (DER); the client reads the Ed25519
// key from the server's certificate and checks CertificateVerify and
// Finished, but validates no chain. Change-cipher-spec records (middlebox
// compatibility) are skipped and post-handshake messages (session tickets,
// key updates) are ignored.
//
// Every primitive is an export of this library (SHA-256, HMAC, HKDF and the
// TLS 1.3 label expansion, ChaCha20-Poly1305, X25519, Ed25519).
// Names and arguments of the session calls follow the reference's exports
// (runtime/src/tls13.rs:1027-1140); the code is this library's own.
#include <cstdint>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

extern "C" {
int aether_sha256(const void* msg, int n, void* out);
int aether_hmac_sha256(const void* key, int nk, const void* msg, int nm, void* out);
int aether_hkdf_extract(const void* salt, int ns, const void* ikm, int ni, void* out);
int aether_tls13_hkdf_expand_label(const void* secret, int ns, const void* label, int nl, const void* ctx, int nc,
                                   void* out, int n);
int aether_chacha20_poly1305_encrypt(const void* key, const void* nonce, const void* aad, int na, const void* plain,
                                     int np, void* out, int max_out);
int aether_chacha20_poly1305_decrypt(const void* key, const void* nonce, const void* aad, int na, const void* in, int n,
                                     void* out, int max_out);
int aether_x25519_derive_public(const void* scalar, void* out);
int aether_x25519_shared_secret(const void* scalar, const void* peer, void* out);
int aether_ed25519_derive_public(const void* seed, void* out_pub);
int aether_ed25519_sign(const void* seed, const void* pub, const void* msg, int n, void* out_sig);
int aether_ed25519_verify(const void* pub, const void* msg, int n, const void* sig);
}

namespace {

typedef std::vector<uint8_t> Bytes;

enum : uint8_t { REC_CCS = 20, REC_ALERT = 21, REC_HS = 22, REC_APP = 23 };
enum : uint8_t { HS_CH = 1, HS_SH = 2, HS_NST = 4, HS_EE = 8, HS_CERT = 11, HS_CV = 15, HS_FIN = 20, HS_KU = 24 };
const uint16_t SUITE = 0x1303, GROUP_X25519 = 0x001d, SIG_ED25519 = 0x0807, TLS13 = 0x0304;

void put8(Bytes& b, uint32_t v) { b.push_back((uint8_t)v); }
void put16(Bytes& b, uint32_t v) {
  b.push_back((uint8_t)(v >> 8));
  b.push_back((uint8_t)v);
}
void put24(Bytes& b, uint32_t v) {
  b.push_back((uint8_t)(v >> 16));
  put16(b, v);
}
void put(Bytes& b, const uint8_t* p, size_t n) { b.insert(b.end(), p, p + n); }
void put(Bytes& b, const Bytes& x) { b.insert(b.end(), x.begin(), x.end()); }

// A bounds-checked reader; any short read marks it bad.
struct Rd {
  const uint8_t* p;
  size_t n, i = 0;
  bool ok = true;
  uint32_t u(int w) {
    if (i + w > n) {
      ok = false;
      return 0;
    }
    uint32_t v = 0;
    for (int k = 0; k < w; ++k) v = v << 8 | p[i++];
    return v;
  }
  Rd sub(size_t len) {
    if (i + len > n) {
      ok = false;
      return Rd{p, 0};
    }
    Rd r{p + i, len};
    i += len;
    return r;
  }
  Bytes take(size_t len) {
    if (i + len > n) {
      ok = false;
      return {};
    }
    Bytes b(p + i, p + i + len);
    i += len;
    return b;
  }
  bool end() const { return i == n; }
};

Bytes sha256(const Bytes& m) {
  Bytes h(32);
  aether_sha256(m.empty() ? (const void*)"" : m.data(), (int)m.size(), h.data());
  return h;
}
Bytes expand_label(const Bytes& secret, const char* label, const Bytes& ctx, int n) {
  Bytes out(n);
  aether_tls13_hkdf_expand_label(secret.data(), 32, label, (int)strlen(label), ctx.empty() ? nullptr : ctx.data(),
                                 (int)ctx.size(), out.data(), n);
  return out;
}
Bytes extract(const Bytes& salt, const Bytes& ikm) {
  Bytes out(32);
  aether_hkdf_extract(salt.data(), (int)salt.size(), ikm.data(), (int)ikm.size(), out.data());
  return out;
}
Bytes hmac(const Bytes& key, const Bytes& msg) {
  Bytes out(32);
  aether_hmac_sha256(key.data(), (int)key.size(), msg.empty() ? (const void*)"" : msg.data(), (int)msg.size(),
                     out.data());
  return out;
}

// ------------------------------------------------------------------------------------------------ DER certificate
Bytes der(uint8_t tag, const Bytes& body) {
  Bytes b{tag};
  const size_t n = body.size();
  if (n < 128) {
    b.push_back((uint8_t)n);
  } else if (n < 256) {
    b.push_back(0x81);
    b.push_back((uint8_t)n);
  } else {
    b.push_back(0x82);
    b.push_back((uint8_t)(n >> 8));
    b.push_back((uint8_t)n);
  }
  put(b, body);
  return b;
}
Bytes cat(std::initializer_list<Bytes> parts) {
  Bytes b;
  for (auto& p : parts) put(b, p);
  return b;
}
// Self-signed v3 certificate: subject = issuer = CN, Ed25519 key and signature.
Bytes make_cert(const uint8_t seed[32], const uint8_t pub[32], const std::string& cn, const Bytes& serial_in) {
  const Bytes ed_alg = der(0x30, der(0x06, {0x2B, 0x65, 0x70}));  // id-Ed25519 (1.3.101.112)
  Bytes serial = serial_in.empty() ? Bytes{1} : serial_in;
  if (serial[0] & 0x80) serial.insert(serial.begin(), 0);  // keep the INTEGER positive
  const Bytes name =
      der(0x30, der(0x31, der(0x30, cat({der(0x06, {0x55, 0x04, 0x03}), der(0x0C, Bytes(cn.begin(), cn.end()))}))));
  const std::string nb = "250101000000Z", na = "20991231235959Z";
  const Bytes validity = der(0x30, cat({der(0x17, Bytes(nb.begin(), nb.end())), der(0x18, Bytes(na.begin(), na.end()))}));
  Bytes bits{0};
  put(bits, pub, 32);
  const Bytes spki = der(0x30, cat({ed_alg, der(0x03, bits)}));
  const Bytes tbs = der(0x30, cat({der(0xA0, der(0x02, {2})), der(0x02, serial), ed_alg, name, validity, name, spki}));
  uint8_t sig[64];
  aether_ed25519_sign(seed, pub, tbs.data(), (int)tbs.size(), sig);
  Bytes sigbits{0};
  put(sigbits, sig, 64);
  return der(0x30, cat({tbs, ed_alg, der(0x03, sigbits)}));
}
// The Ed25519 key of a certificate: the SubjectPublicKeyInfo
// SEQUENCE { SEQUENCE { OID 1.3.101.112 } BIT STRING (0 unused bits, 32 bytes) }.
bool cert_ed25519_key(const Bytes& c, uint8_t out[32]) {
  static const uint8_t pat[] = {0x30, 0x2A, 0x30, 0x05, 0x06, 0x03, 0x2B, 0x65, 0x70, 0x03, 0x21, 0x00};
  for (size_t i = 0; i + sizeof(pat) + 32 <= c.size(); ++i)
    if (!memcmp(&c[i], pat, sizeof(pat))) {
      memcpy(out, &c[i + sizeof(pat)], 32);
      return true;
    }
  return false;
}

// ------------------------------------------------------------------------------------------------ session
struct Keys {
  Bytes key, iv;
  uint64_t seq = 0;
  bool on = false;
  void set(const Bytes& secret) {
    key = expand_label(secret, "key", {}, 32);
    iv = expand_label(secret, "iv", {}, 12);
    seq = 0;
    on = true;
  }
  Bytes nonce() {
    Bytes n = iv;
    for (int i = 0; i < 8; ++i) n[11 - i] ^= (uint8_t)(seq >> (8 * i));
    ++seq;
    return n;
  }
};

enum State { WAIT_CH, WAIT_SH, WAIT_EE, WAIT_CERT, WAIT_CV, WAIT_FIN, WAIT_CLIENT_FIN, CONNECTED, FAILED };

struct Session {
  bool server;
  State st;
  uint8_t x_priv[32], x_pub[32], random[32];
  Bytes session_id;
  // server identity
  uint8_t ed_seed[32], ed_pub[32];
  Bytes cert;
  bool alpn_h2 = false;  // server: the client offered "h2" and it was selected
  uint8_t peer_ed[32];
  Bytes transcript, in, out, hs_buf;
  Bytes hs_secret, c_hs, s_hs, c_ap, s_ap, master;
  Keys rd, wr;

  void record(uint8_t type, const Bytes& payload) {  // plaintext or protected, by the write keys
    if (!wr.on) {
      put8(out, type);
      put16(out, 0x0303);
      put16(out, (uint32_t)payload.size());
      put(out, payload);
      return;
    }
    Bytes inner = payload;
    inner.push_back(type);
    Bytes hdr{REC_APP, 0x03, 0x03};
    put16(hdr, (uint32_t)inner.size() + 16);
    Bytes ct(inner.size() + 16);
    const Bytes n = wr.nonce();
    aether_chacha20_poly1305_encrypt(wr.key.data(), n.data(), hdr.data(), 5, inner.data(), (int)inner.size(), ct.data(),
                                     (int)ct.size());
    put(out, hdr);
    put(out, ct);
  }
  void hs_msg(uint8_t type, const Bytes& body) {
    Bytes m{type};
    put24(m, (uint32_t)body.size());
    put(m, body);
    put(transcript, m);
    record(REC_HS, m);
  }
  void derive_handshake(const uint8_t shared[32]) {
    const Bytes zeros(32, 0);
    const Bytes early = extract(zeros, zeros);
    const Bytes derived = expand_label(early, "derived", sha256({}), 32);
    hs_secret = extract(derived, Bytes(shared, shared + 32));
    const Bytes th = sha256(transcript);
    c_hs = expand_label(hs_secret, "c hs traffic", th, 32);
    s_hs = expand_label(hs_secret, "s hs traffic", th, 32);
    master = extract(expand_label(hs_secret, "derived", sha256({}), 32), zeros);
  }
  void derive_app() {  // transcript through the server Finished
    const Bytes th = sha256(transcript);
    c_ap = expand_label(master, "c ap traffic", th, 32);
    s_ap = expand_label(master, "s ap traffic", th, 32);
  }
  Bytes finished(const Bytes& base) { return hmac(expand_label(base, "finished", {}, 32), sha256(transcript)); }
  static Bytes cv_content(bool server_side, const Bytes& th) {
    Bytes m(64, 0x20);
    const char* ctx = server_side ? "TLS 1.3, server CertificateVerify" : "TLS 1.3, client CertificateVerify";
    put(m, (const uint8_t*)ctx, strlen(ctx));
    m.push_back(0);
    put(m, th);
    return m;
  }

  // -------------------------------------------------------------------------------------------- client
  void client_hello() {
    Bytes b;
    put16(b, 0x0303);
    put(b, random, 32);
    put8(b, (uint32_t)session_id.size());
    put(b, session_id);
    put16(b, 2);
    put16(b, SUITE);
    put8(b, 1);
    put8(b, 0);
    Bytes ext;
    put16(ext, 43);  // supported_versions
    put16(ext, 3);
    put8(ext, 2);
    put16(ext, TLS13);
    put16(ext, 10);  // supported_groups
    put16(ext, 4);
    put16(ext, 2);
    put16(ext, GROUP_X25519);
    put16(ext, 13);  // signature_algorithms
    put16(ext, 4);
    put16(ext, 2);
    put16(ext, SIG_ED25519);
    put16(ext, 51);  // key_share
    put16(ext, 2 + 4 + 32);
    put16(ext, 4 + 32);
    put16(ext, GROUP_X25519);
    put16(ext, 32);
    put(ext, x_pub, 32);
    put16(b, (uint32_t)ext.size());
    put(b, ext);
    hs_msg(HS_CH, b);
    st = WAIT_SH;
  }
  bool on_server_hello(Rd& r) {
    if (r.u(2) != 0x0303) return false;
    r.take(32);
    r.take(r.u(1));  // session id echo
    if (r.u(2) != SUITE || r.u(1) != 0) return false;
    Rd ext = r.sub(r.u(2));
    bool v13 = false;
    Bytes share;
    while (ext.ok && !ext.end()) {
      const uint32_t t = ext.u(2);
      Rd e = ext.sub(ext.u(2));
      if (t == 43) v13 = e.u(2) == TLS13;
      if (t == 51 && e.u(2) == GROUP_X25519) share = e.take(e.u(2));
    }
    if (!r.ok || !ext.ok || !v13 || share.size() != 32) return false;
    uint8_t shared[32];
    aether_x25519_shared_secret(x_priv, share.data(), shared);
    derive_handshake(shared);
    rd.set(s_hs);
    wr.set(c_hs);
    wr.on = false;  // the client keeps writing in the clear until its Finished
    st = WAIT_EE;
    return true;
  }
  bool client_handshake(uint8_t type, const Bytes& msg, Rd& r) {
    if (st == WAIT_EE && type == HS_EE) {
      put(transcript, msg);
      st = WAIT_CERT;
      return true;
    }
    if (st == WAIT_CERT && type == HS_CERT) {
      r.take(r.u(1));
      Rd list = r.sub(r.u(3));
      const Bytes first = list.take(list.u(3));
      if (!list.ok || !cert_ed25519_key(first, peer_ed)) return false;
      put(transcript, msg);
      st = WAIT_CV;
      return true;
    }
    if (st == WAIT_CV && type == HS_CV) {
      if (r.u(2) != SIG_ED25519) return false;
      const Bytes sig = r.take(r.u(2));
      const Bytes content = cv_content(true, sha256(transcript));
      if (sig.size() != 64 || aether_ed25519_verify(peer_ed, content.data(), (int)content.size(), sig.data()) != 0)
        return false;
      put(transcript, msg);
      st = WAIT_FIN;
      return true;
    }
    if (st == WAIT_FIN && type == HS_FIN) {
      const Bytes want = finished(s_hs);
      const Bytes got = r.take(32);
      if (got != want) return false;
      put(transcript, msg);
      derive_app();
      wr.set(c_hs);  // client Finished under the client handshake key
      hs_msg(HS_FIN, finished(c_hs));
      rd.set(s_ap);
      wr.set(c_ap);
      st = CONNECTED;
      return true;
    }
    if (st == CONNECTED && (type == HS_NST || type == HS_KU)) return true;  // tickets / key updates: ignored
    return false;
  }

  // -------------------------------------------------------------------------------------------- server
  bool on_client_hello(const Bytes& msg, Rd& r) {
    if (r.u(2) != 0x0303) return false;
    r.take(32);
    session_id = r.take(r.u(1));
    Rd suites = r.sub(r.u(2));
    bool have_suite = false;
    while (suites.ok && !suites.end()) have_suite |= suites.u(2) == SUITE;
    r.take(r.u(1));  // compression methods
    Rd ext = r.sub(r.u(2));
    bool v13 = false, ed = false;
    Bytes share;
    while (ext.ok && !ext.end()) {
      const uint32_t t = ext.u(2);
      Rd e = ext.sub(ext.u(2));
      if (t == 43) {
        Rd v = e.sub(e.u(1));
        while (v.ok && !v.end()) v13 |= v.u(2) == TLS13;
      } else if (t == 13) {
        Rd v = e.sub(e.u(2));
        while (v.ok && !v.end()) ed |= v.u(2) == SIG_ED25519;
      } else if (t == 51) {
        Rd v = e.sub(e.u(2));
        while (v.ok && !v.end()) {
          const uint32_t g = v.u(2);
          Bytes k = v.take(v.u(2));
          if (g == GROUP_X25519 && k.size() == 32) share = k;
        }
      } else if (t == 16) {  // ALPN: select "h2" when offered
        Rd v = e.sub(e.u(2));
        while (v.ok && !v.end()) {
          const Bytes proto = v.take(v.u(1));
          if (proto.size() == 2 && proto[0] == 'h' && proto[1] == '2') alpn_h2 = true;
        }
      }
    }
    if (!r.ok || !ext.ok || !have_suite || !v13 || !ed || share.empty()) return false;
    put(transcript, msg);
    Bytes b;
    put16(b, 0x0303);
    put(b, random, 32);
    put8(b, (uint32_t)session_id.size());
    put(b, session_id);
    put16(b, SUITE);
    put8(b, 0);
    Bytes e;
    put16(e, 43);
    put16(e, 2);
    put16(e, TLS13);
    put16(e, 51);
    put16(e, 36);
    put16(e, GROUP_X25519);
    put16(e, 32);
    put(e, x_pub, 32);
    put16(b, (uint32_t)e.size());
    put(b, e);
    hs_msg(HS_SH, b);
    if (!session_id.empty()) record(REC_CCS, {1});  // middlebox compatibility
    uint8_t shared[32];
    aether_x25519_shared_secret(x_priv, share.data(), shared);
    derive_handshake(shared);
    wr.set(s_hs);
    if (alpn_h2) {  // EncryptedExtensions carrying the selected protocol
      hs_msg(HS_EE, {0, 9, 0, 16, 0, 5, 0, 3, 2, 'h', '2'});
    } else {
      hs_msg(HS_EE, {0, 0});
    }
    Bytes c;
    put8(c, 0);
    Bytes entry;
    put24(entry, (uint32_t)cert.size());
    put(entry, cert);
    put16(entry, 0);
    put24(c, (uint32_t)entry.size());
    put(c, entry);
    hs_msg(HS_CERT, c);
    const Bytes content = cv_content(true, sha256(transcript));
    uint8_t sig[64];
    aether_ed25519_sign(ed_seed, ed_pub, content.data(), (int)content.size(), sig);
    Bytes cv;
    put16(cv, SIG_ED25519);
    put16(cv, 64);
    put(cv, sig, 64);
    hs_msg(HS_CV, cv);
    hs_msg(HS_FIN, finished(s_hs));
    derive_app();
    rd.set(c_hs);
    wr.set(s_ap);
    st = WAIT_CLIENT_FIN;
    return true;
  }
  bool server_handshake(uint8_t type, const Bytes& msg, Rd& r) {
    if (st == WAIT_CLIENT_FIN && type == HS_FIN) {
      if (r.take(32) != finished(c_hs)) return false;
      put(transcript, msg);
      rd.set(c_ap);
      st = CONNECTED;
      return true;
    }
    if (st == CONNECTED && type == HS_KU) return true;
    return false;
  }

  // -------------------------------------------------------------------------------------------- input
  bool handshake_bytes(const Bytes& data) {
    put(hs_buf, data);
    size_t off = 0;
    while (hs_buf.size() - off >= 4) {
      const uint32_t len = (uint32_t)hs_buf[off + 1] << 16 | (uint32_t)hs_buf[off + 2] << 8 | hs_buf[off + 3];
      if (hs_buf.size() - off < 4 + len) break;
      const Bytes msg(hs_buf.begin() + off, hs_buf.begin() + off + 4 + len);
      Rd r{msg.data() + 4, len};
      const uint8_t type = msg[0];
      bool ok;
      if (server && st == WAIT_CH) ok = type == HS_CH && on_client_hello(msg, r);
      else if (!server && st == WAIT_SH) ok = type == HS_SH && (put(transcript, msg), on_server_hello(r));
      else ok = server ? server_handshake(type, msg, r) : client_handshake(type, msg, r);
      if (!ok) return false;
      off += 4 + len;
    }
    hs_buf.erase(hs_buf.begin(), hs_buf.begin() + off);
    return true;
  }
  // Consumes whole records from `in`; decrypted application data goes to app.
  bool drain(Bytes& app) {
    while (in.size() >= 5) {
      const uint8_t type = in[0];
      const size_t len = (size_t)in[3] << 8 | in[4];
      if (len > (1 << 14) + 256) return false;
      if (in.size() < 5 + len) break;
      const Bytes hdr(in.begin(), in.begin() + 5), body(in.begin() + 5, in.begin() + 5 + len);
      in.erase(in.begin(), in.begin() + 5 + len);
      if (type == REC_CCS) continue;
      if (type == REC_ALERT && !rd.on) return false;
      uint8_t inner_type = type;
      Bytes plain = body;
      if (rd.on && type == REC_APP) {
        if (len < 17) return false;
        plain.resize(len - 16);
        const Bytes n = rd.nonce();
        if (aether_chacha20_poly1305_decrypt(rd.key.data(), n.data(), hdr.data(), 5, body.data(), (int)len,
                                             plain.data(), (int)plain.size()) < 0)
          return false;
        while (!plain.empty() && plain.back() == 0) plain.pop_back();
        if (plain.empty()) return false;
        inner_type = plain.back();
        plain.pop_back();
      } else if (rd.on) {
        return false;  // plaintext after keys are set
      }
      if (inner_type == REC_HS) {
        if (!handshake_bytes(plain)) return false;
      } else if (inner_type == REC_APP && st == CONNECTED) {
        put(app, plain);
      } else if (inner_type == REC_ALERT) {
        return false;
      } else {
        return false;
      }
    }
    return true;
  }
};

std::mutex g_mu;
std::vector<std::unique_ptr<Session>> g_sessions;

int64_t add(std::unique_ptr<Session> s) {
  std::lock_guard<std::mutex> l(g_mu);
  for (size_t i = 0; i < g_sessions.size(); ++i)
    if (!g_sessions[i]) {
      g_sessions[i] = std::move(s);
      return (int64_t)i;
    }
  g_sessions.push_back(std::move(s));
  return (int64_t)g_sessions.size() - 1;
}
Session* get(int64_t h, bool server) {
  std::lock_guard<std::mutex> l(g_mu);
  if (h < 0 || (size_t)h >= g_sessions.size() || !g_sessions[h] || g_sessions[h]->server != server) return nullptr;
  return g_sessions[h].get();
}

int feed(int64_t h, bool server, const void* in, int n, void* out_app, int max_app) {
  Session* s = get(h, server);
  if (!s) return -2;
  if (s->st == FAILED || n < 0 || (n && !in)) return -1;
  put(s->in, (const uint8_t*)in, n);
  Bytes app;
  if (!s->drain(app)) {
    s->st = FAILED;
    return -1;
  }
  if ((int)app.size() > max_app || (!app.empty() && !out_app)) return -1;
  if (!app.empty()) memcpy(out_app, app.data(), app.size());
  return (int)app.size();
}
int take(int64_t h, bool server, void* out, int max_out) {
  Session* s = get(h, server);
  if (!s) return -2;
  if (!out || max_out < 0) return -1;
  const int n = (int)std::min<size_t>(s->out.size(), (size_t)max_out);
  memcpy(out, s->out.data(), n);
  s->out.erase(s->out.begin(), s->out.begin() + n);
  return n;
}
int send_app(int64_t h, bool server, const void* app, int n) {
  Session* s = get(h, server);
  if (!s) return -2;
  if (s->st != CONNECTED || n < 0 || (n && !app)) return -1;
  for (int off = 0; off < n || (n == 0 && off == 0); off += 16384) {  // records of at most 2^14 bytes
    const int c = std::min(16384, n - off);
    s->record(REC_APP, Bytes((const uint8_t*)app + off, (const uint8_t*)app + off + c));
    if (n == 0) break;
  }
  return n;
}
int release(int64_t h, bool server) {
  std::lock_guard<std::mutex> l(g_mu);
  if (h < 0 || (size_t)h >= g_sessions.size() || !g_sessions[h] || g_sessions[h]->server != server) return -1;
  g_sessions[h].reset();
  return 0;
}

}  // namespace

extern "C" {

// Server session: Ed25519 identity seed, server random, X25519 private key, and
// the CN / serial of the self-signed certificate it presents. Handle >= 0 or -1.
int64_t aether_tls13_server_new(const void* ed_seed, const void* random, const void* x_priv, const void* cn, int n_cn,
                                const void* serial, int n_serial) {
  if (!ed_seed || !random || !x_priv || n_cn < 0 || n_cn > 64 || n_serial < 0 || n_serial > 20 || (n_cn && !cn) ||
      (n_serial && !serial))
    return -1;
  auto s = std::make_unique<Session>();
  s->server = true;
  s->st = WAIT_CH;
  memcpy(s->ed_seed, ed_seed, 32);
  memcpy(s->random, random, 32);
  memcpy(s->x_priv, x_priv, 32);
  aether_x25519_derive_public(s->x_priv, s->x_pub);
  aether_ed25519_derive_public(s->ed_seed, s->ed_pub);
  s->cert = make_cert(s->ed_seed, s->ed_pub, std::string((const char*)cn, n_cn),
                      Bytes((const uint8_t*)serial, (const uint8_t*)serial + n_serial));
  return add(std::move(s));
}
// Client session: X25519 private key, client random, legacy session id (0..32
// bytes). The ClientHello is queued at once (take_outbound).
int64_t aether_tls13_client_new(const void* x_priv, const void* random, const void* session_id, int n_sid) {
  if (!x_priv || !random || n_sid < 0 || n_sid > 32 || (n_sid && !session_id)) return -1;
  auto s = std::make_unique<Session>();
  s->server = false;
  memcpy(s->x_priv, x_priv, 32);
  memcpy(s->random, random, 32);
  aether_x25519_derive_public(s->x_priv, s->x_pub);
  s->session_id.assign((const uint8_t*)session_id, (const uint8_t*)session_id + n_sid);
  s->client_hello();
  return add(std::move(s));
}
// Received bytes in (any split); application data decrypted by them out.
// Returns its length, -1 on a protocol error (the session is then dead), -2 on a bad handle.
int aether_tls13_server_feed(int64_t h, const void* in, int n, void* out_app, int max_app) {
  return feed(h, true, in, n, out_app, max_app);
}
int aether_tls13_client_feed(int64_t h, const void* in, int n, void* out_app, int max_app) {
  return feed(h, false, in, n, out_app, max_app);
}
int aether_tls13_server_take_outbound(int64_t h, void* out, int max_out) { return take(h, true, out, max_out); }
int aether_tls13_client_take_outbound(int64_t h, void* out, int max_out) { return take(h, false, out, max_out); }
// Queue application data (after the handshake); returns its length.
int aether_tls13_server_send(int64_t h, const void* app, int n) { return send_app(h, true, app, n); }
int aether_tls13_client_send(int64_t h, const void* app, int n) { return send_app(h, false, app, n); }
int aether_tls13_server_is_done(int64_t h) {
  Session* s = get(h, true);
  return s ? s->st == CONNECTED : -2;
}
int aether_tls13_client_is_done(int64_t h) {
  Session* s = get(h, false);
  return s ? s->st == CONNECTED : -2;
}
int aether_tls13_server_free(int64_t h) { return release(h, true); }
// 1 when ALPN selected "h2" on this server session, 0 otherwise.
int aether_tls13_server_alpn_h2(int64_t h) {
  Session* s = get(h, true);
  return s ? (int)s->alpn_h2 : -2;
}
int aether_tls13_client_free(int64_t h) { return release(h, false); }

// Client and server in one process, fixed keys: handshake and one exchange of
// application data each way. 42 on success.
int aether_tls13_self_loopback_smoke() {
  uint8_t a[32], b[32], c[32], d[32], e[32];
  for (int i = 0; i < 32; ++i) {
    a[i] = (uint8_t)(i + 1);
    b[i] = (uint8_t)(2 * i + 3);
    c[i] = (uint8_t)(5 * i + 7);
    d[i] = (uint8_t)(11 * i + 13);
    e[i] = (uint8_t)(17 * i + 19);
  }
  const int64_t sv = aether_tls13_server_new(a, b, c, "aether", 6, "\x01", 1);
  const int64_t cl = aether_tls13_client_new(d, e, e, 32);
  if (sv < 0 || cl < 0) return 1;
  uint8_t buf[65536], app[256];
  int rc = 2;
  for (int round = 0; round < 8; ++round) {
    int n = aether_tls13_client_take_outbound(cl, buf, sizeof(buf));
    if (n > 0 && aether_tls13_server_feed(sv, buf, n, app, sizeof(app)) < 0) break;
    n = aether_tls13_server_take_outbound(sv, buf, sizeof(buf));
    if (n > 0 && aether_tls13_client_feed(cl, buf, n, app, sizeof(app)) < 0) break;
    if (aether_tls13_client_is_done(cl) == 1 && aether_tls13_server_is_done(sv) == 1) {
      rc = 3;
      break;
    }
  }
  if (rc == 3) {
    int n;
    aether_tls13_client_send(cl, "ping", 4);
    n = aether_tls13_client_take_outbound(cl, buf, sizeof(buf));
    if (aether_tls13_server_feed(sv, buf, n, app, sizeof(app)) == 4 && !memcmp(app, "ping", 4)) {
      aether_tls13_server_send(sv, "pong", 4);
      n = aether_tls13_server_take_outbound(sv, buf, sizeof(buf));
      if (aether_tls13_client_feed(cl, buf, n, app, sizeof(app)) == 4 && !memcmp(app, "pong", 4)) rc = 42;
    }
  }
  aether_tls13_server_free(sv);
  aether_tls13_client_free(cl);
  return rc;
}

}  // extern "C"
