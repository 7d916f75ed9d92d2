// Cryptographic and wire codecs of the core C ABI, written from their
// specifications: SHA-256 / SHA-512 (FIPS 180-4), HMAC-SHA256 (RFC 2104),
// HKDF (RFC 5869) and the TLS 1.3 HKDF-Expand-Label (RFC 8446 7.1),
// ChaCha20-Poly1305 AEAD (RFC 8439), X25519 (RFC 7748), Ed25519 (RFC 8032),
// WebSocket frames (RFC 6455 5.2), a minimal HTTP/1.1 request parser and 200
// response writer, and the OpenAI chat-completion body.
//
// Field arithmetic mod 2^255 - 19 uses five 51-bit limbs with 128-bit
// products; Ed25519 scalars are reduced mod the group order by binary long
// division; the curve constants (d, sqrt(-1), the base point) are derived at
// first use from their definitions. The ladder and the Ed25519 scalar
// multiplication select with masks instead of branches on secret bits.
//
// Names, argument orders and return conventions follow the reference's
// exports (runtime/src/lib.rs:6587-7903); the code is this library's own.
#include <sys/random.h>

#include <cerrno>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

namespace {

// ================================================================================================ SHA-2
// Fractional bits of the cube roots (K) and square roots (H) of the first
// primes, as FIPS 180-4 4.2.2 / 4.2.3 / 5.3.3 / 5.3.5 define them; generated
// with exact integer roots.
const uint32_t K256[64] = {
    0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u, 0x923f82a4u, 0xab1c5ed5u,
    0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u, 0x72be5d74u, 0x80deb1feu, 0x9bdc06a7u, 0xc19bf174u,
    0xe49b69c1u, 0xefbe4786u, 0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu, 0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau,
    0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u, 0xc6e00bf3u, 0xd5a79147u, 0x06ca6351u, 0x14292967u,
    0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu, 0x53380d13u, 0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u,
    0xa2bfe8a1u, 0xa81a664bu, 0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u,
    0x19a4c116u, 0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au, 0x5b9cca4fu, 0x682e6ff3u,
    0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u, 0x90befffau, 0xa4506cebu, 0xbef9a3f7u, 0xc67178f2u,
};
const uint32_t H256[8] = {
    0x6a09e667u, 0xbb67ae85u, 0x3c6ef372u, 0xa54ff53au, 0x510e527fu, 0x9b05688cu, 0x1f83d9abu, 0x5be0cd19u,
};
const uint64_t K512[80] = {
    0x428a2f98d728ae22ull, 0x7137449123ef65cdull, 0xb5c0fbcfec4d3b2full, 0xe9b5dba58189dbbcull,
    0x3956c25bf348b538ull, 0x59f111f1b605d019ull, 0x923f82a4af194f9bull, 0xab1c5ed5da6d8118ull,
    0xd807aa98a3030242ull, 0x12835b0145706fbeull, 0x243185be4ee4b28cull, 0x550c7dc3d5ffb4e2ull,
    0x72be5d74f27b896full, 0x80deb1fe3b1696b1ull, 0x9bdc06a725c71235ull, 0xc19bf174cf692694ull,
    0xe49b69c19ef14ad2ull, 0xefbe4786384f25e3ull, 0x0fc19dc68b8cd5b5ull, 0x240ca1cc77ac9c65ull,
    0x2de92c6f592b0275ull, 0x4a7484aa6ea6e483ull, 0x5cb0a9dcbd41fbd4ull, 0x76f988da831153b5ull,
    0x983e5152ee66dfabull, 0xa831c66d2db43210ull, 0xb00327c898fb213full, 0xbf597fc7beef0ee4ull,
    0xc6e00bf33da88fc2ull, 0xd5a79147930aa725ull, 0x06ca6351e003826full, 0x142929670a0e6e70ull,
    0x27b70a8546d22ffcull, 0x2e1b21385c26c926ull, 0x4d2c6dfc5ac42aedull, 0x53380d139d95b3dfull,
    0x650a73548baf63deull, 0x766a0abb3c77b2a8ull, 0x81c2c92e47edaee6ull, 0x92722c851482353bull,
    0xa2bfe8a14cf10364ull, 0xa81a664bbc423001ull, 0xc24b8b70d0f89791ull, 0xc76c51a30654be30ull,
    0xd192e819d6ef5218ull, 0xd69906245565a910ull, 0xf40e35855771202aull, 0x106aa07032bbd1b8ull,
    0x19a4c116b8d2d0c8ull, 0x1e376c085141ab53ull, 0x2748774cdf8eeb99ull, 0x34b0bcb5e19b48a8ull,
    0x391c0cb3c5c95a63ull, 0x4ed8aa4ae3418acbull, 0x5b9cca4f7763e373ull, 0x682e6ff3d6b2b8a3ull,
    0x748f82ee5defb2fcull, 0x78a5636f43172f60ull, 0x84c87814a1f0ab72ull, 0x8cc702081a6439ecull,
    0x90befffa23631e28ull, 0xa4506cebde82bde9ull, 0xbef9a3f7b2c67915ull, 0xc67178f2e372532bull,
    0xca273eceea26619cull, 0xd186b8c721c0c207ull, 0xeada7dd6cde0eb1eull, 0xf57d4f7fee6ed178ull,
    0x06f067aa72176fbaull, 0x0a637dc5a2c898a6ull, 0x113f9804bef90daeull, 0x1b710b35131c471bull,
    0x28db77f523047d84ull, 0x32caab7b40c72493ull, 0x3c9ebe0a15c9bebcull, 0x431d67c49c100d4cull,
    0x4cc5d4becb3e42b6ull, 0x597f299cfc657e2aull, 0x5fcb6fab3ad6faecull, 0x6c44198c4a475817ull,
};
const uint64_t H512[8] = {
    0x6a09e667f3bcc908ull, 0xbb67ae8584caa73bull, 0x3c6ef372fe94f82bull, 0xa54ff53a5f1d36f1ull,
    0x510e527fade682d1ull, 0x9b05688c2b3e6c1full, 0x1f83d9abfb41bd6bull, 0x5be0cd19137e2179ull,
};

inline uint32_t ror32(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }
inline uint64_t ror64(uint64_t x, int n) { return (x >> n) | (x << (64 - n)); }
inline uint32_t be32(const uint8_t* p) { return (uint32_t)p[0] << 24 | (uint32_t)p[1] << 16 | (uint32_t)p[2] << 8 | p[3]; }
inline uint64_t be64(const uint8_t* p) { return (uint64_t)be32(p) << 32 | be32(p + 4); }
inline uint32_t le32(const uint8_t* p) { return (uint32_t)p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24; }
inline uint64_t le64(const uint8_t* p) { return (uint64_t)le32(p) | (uint64_t)le32(p + 4) << 32; }
inline void put_be32(uint8_t* p, uint32_t v) {
  for (int i = 0; i < 4; ++i) p[i] = (uint8_t)(v >> (24 - 8 * i));
}
inline void put_be64(uint8_t* p, uint64_t v) {
  for (int i = 0; i < 8; ++i) p[i] = (uint8_t)(v >> (56 - 8 * i));
}
inline void put_le32(uint8_t* p, uint32_t v) {
  for (int i = 0; i < 4; ++i) p[i] = (uint8_t)(v >> (8 * i));
}
inline void put_le64(uint8_t* p, uint64_t v) {
  for (int i = 0; i < 8; ++i) p[i] = (uint8_t)(v >> (8 * i));
}

// Message padding shared by both hashes: 0x80, zeros, then the bit length
// big-endian in the last `lenbytes` bytes of a block of `block` bytes.
std::vector<uint8_t> sha_pad(const uint8_t* m, size_t n, size_t block, size_t lenbytes) {
  std::vector<uint8_t> b(m, m + n);
  b.push_back(0x80);
  while (b.size() % block != block - lenbytes) b.push_back(0);
  for (size_t i = 0; i < lenbytes - 8; ++i) b.push_back(0);
  uint8_t l[8];
  put_be64(l, (uint64_t)n * 8);
  b.insert(b.end(), l, l + 8);
  return b;
}

void sha256(const uint8_t* m, size_t n, uint8_t out[32]) {
  uint32_t h[8];
  memcpy(h, H256, sizeof(h));
  const std::vector<uint8_t> b = sha_pad(m, n, 64, 8);
  uint32_t w[64];
  for (size_t off = 0; off < b.size(); off += 64) {
    for (int t = 0; t < 16; ++t) w[t] = be32(&b[off + 4 * t]);
    for (int t = 16; t < 64; ++t) {
      const uint32_t s0 = ror32(w[t - 15], 7) ^ ror32(w[t - 15], 18) ^ (w[t - 15] >> 3);
      const uint32_t s1 = ror32(w[t - 2], 17) ^ ror32(w[t - 2], 19) ^ (w[t - 2] >> 10);
      w[t] = w[t - 16] + s0 + w[t - 7] + s1;
    }
    uint32_t a = h[0], bb = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
    for (int t = 0; t < 64; ++t) {
      const uint32_t t1 = hh + (ror32(e, 6) ^ ror32(e, 11) ^ ror32(e, 25)) + ((e & f) ^ (~e & g)) + K256[t] + w[t];
      const uint32_t t2 = (ror32(a, 2) ^ ror32(a, 13) ^ ror32(a, 22)) + ((a & bb) ^ (a & c) ^ (bb & c));
      hh = g; g = f; f = e; e = d + t1; d = c; c = bb; bb = a; a = t1 + t2;
    }
    h[0] += a; h[1] += bb; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
  }
  for (int i = 0; i < 8; ++i) put_be32(out + 4 * i, h[i]);
}

void sha512(const uint8_t* m, size_t n, uint8_t out[64]) {
  uint64_t h[8];
  memcpy(h, H512, sizeof(h));
  const std::vector<uint8_t> b = sha_pad(m, n, 128, 16);
  uint64_t w[80];
  for (size_t off = 0; off < b.size(); off += 128) {
    for (int t = 0; t < 16; ++t) w[t] = be64(&b[off + 8 * t]);
    for (int t = 16; t < 80; ++t) {
      const uint64_t s0 = ror64(w[t - 15], 1) ^ ror64(w[t - 15], 8) ^ (w[t - 15] >> 7);
      const uint64_t s1 = ror64(w[t - 2], 19) ^ ror64(w[t - 2], 61) ^ (w[t - 2] >> 6);
      w[t] = w[t - 16] + s0 + w[t - 7] + s1;
    }
    uint64_t a = h[0], bb = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
    for (int t = 0; t < 80; ++t) {
      const uint64_t t1 = hh + (ror64(e, 14) ^ ror64(e, 18) ^ ror64(e, 41)) + ((e & f) ^ (~e & g)) + K512[t] + w[t];
      const uint64_t t2 = (ror64(a, 28) ^ ror64(a, 34) ^ ror64(a, 39)) + ((a & bb) ^ (a & c) ^ (bb & c));
      hh = g; g = f; f = e; e = d + t1; d = c; c = bb; bb = a; a = t1 + t2;
    }
    h[0] += a; h[1] += bb; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
  }
  for (int i = 0; i < 8; ++i) put_be64(out + 8 * i, h[i]);
}

void sha512_cat(std::initializer_list<std::pair<const uint8_t*, size_t>> parts, uint8_t out[64]) {
  std::vector<uint8_t> m;
  for (auto& p : parts) m.insert(m.end(), p.first, p.first + p.second);
  sha512(m.data(), m.size(), out);
}

void hmac256(const uint8_t* key, size_t nk, const uint8_t* msg, size_t nm, uint8_t out[32]) {
  uint8_t k[64] = {0};
  if (nk > 64) sha256(key, nk, k);
  else if (nk) memcpy(k, key, nk);
  std::vector<uint8_t> in(64 + nm), outer(64 + 32);
  for (int i = 0; i < 64; ++i) {
    in[i] = k[i] ^ 0x36;
    outer[i] = k[i] ^ 0x5c;
  }
  if (nm) memcpy(&in[64], msg, nm);
  sha256(in.data(), in.size(), &outer[64]);
  sha256(outer.data(), outer.size(), out);
}

void hkdf_expand(const uint8_t* prk, size_t np, const uint8_t* info, size_t ni, uint8_t* out, size_t n) {
  std::vector<uint8_t> t;
  uint8_t block[32];
  size_t done = 0;
  for (uint8_t i = 1; done < n; ++i) {
    std::vector<uint8_t> m(t);
    m.insert(m.end(), info, info + ni);
    m.push_back(i);
    hmac256(prk, np, m.data(), m.size(), block);
    const size_t c = std::min<size_t>(32, n - done);
    memcpy(out + done, block, c);
    done += c;
    t.assign(block, block + 32);
  }
}

// ================================================================================================ ChaCha20-Poly1305
inline uint32_t rol32(uint32_t x, int n) { return (x << n) | (x >> (32 - n)); }

void chacha_block(const uint8_t key[32], uint32_t counter, const uint8_t nonce[12], uint8_t out[64]) {
  uint32_t s[16];
  // the four words of the ASCII string "expand 32-byte k"
  s[0] = le32((const uint8_t*)"expa");
  s[1] = le32((const uint8_t*)"nd 3");
  s[2] = le32((const uint8_t*)"2-by");
  s[3] = le32((const uint8_t*)"te k");
  for (int i = 0; i < 8; ++i) s[4 + i] = le32(key + 4 * i);
  s[12] = counter;
  for (int i = 0; i < 3; ++i) s[13 + i] = le32(nonce + 4 * i);
  uint32_t x[16];
  memcpy(x, s, sizeof(x));
  auto qr = [&](int a, int b, int c, int d) {
    x[a] += x[b]; x[d] = rol32(x[d] ^ x[a], 16);
    x[c] += x[d]; x[b] = rol32(x[b] ^ x[c], 12);
    x[a] += x[b]; x[d] = rol32(x[d] ^ x[a], 8);
    x[c] += x[d]; x[b] = rol32(x[b] ^ x[c], 7);
  };
  for (int r = 0; r < 10; ++r) {
    qr(0, 4, 8, 12); qr(1, 5, 9, 13); qr(2, 6, 10, 14); qr(3, 7, 11, 15);
    qr(0, 5, 10, 15); qr(1, 6, 11, 12); qr(2, 7, 8, 13); qr(3, 4, 9, 14);
  }
  for (int i = 0; i < 16; ++i) put_le32(out + 4 * i, x[i] + s[i]);
}

void chacha_xor(const uint8_t key[32], uint32_t counter, const uint8_t nonce[12], const uint8_t* in, uint8_t* out,
                size_t n) {
  uint8_t ks[64];
  for (size_t off = 0; off < n; off += 64, ++counter) {
    chacha_block(key, counter, nonce, ks);
    const size_t c = std::min<size_t>(64, n - off);
    for (size_t i = 0; i < c; ++i) out[off + i] = in[off + i] ^ ks[i];
  }
}

// Poly1305 over 2^130 - 5 with five 26-bit limbs; 2^130 = 5 (mod p) folds the top.
void poly1305(const uint8_t key[32], const uint8_t* m, size_t n, uint8_t tag[16]) {
  unsigned __int128 rr = (unsigned __int128)le64(key + 8) << 64 | le64(key);
  rr &= ((unsigned __int128)0x0ffffffc0ffffffcull << 64) | 0x0ffffffc0fffffffull;  // clamp
  const uint64_t M = 0x3ffffff;
  uint64_t r[5], s5[5], h[5] = {0, 0, 0, 0, 0};
  for (int i = 0; i < 5; ++i) {
    r[i] = (uint64_t)(rr >> (26 * i)) & M;
    s5[i] = r[i] * 5;
  }
  for (size_t off = 0; off < n; off += 16) {
    uint8_t blk[17] = {0};
    const size_t c = std::min<size_t>(16, n - off);
    memcpy(blk, m + off, c);
    blk[c] = 1;  // the appended one bit (2^128 for a full block)
    const unsigned __int128 lo = (unsigned __int128)le64(blk + 8) << 64 | le64(blk);
    h[0] += (uint64_t)lo & M;
    h[1] += (uint64_t)(lo >> 26) & M;
    h[2] += (uint64_t)(lo >> 52) & M;
    h[3] += (uint64_t)(lo >> 78) & M;
    h[4] += (uint64_t)(lo >> 104) | ((uint64_t)blk[16] << 24);
    const uint64_t d0 = h[0] * r[0] + h[1] * s5[4] + h[2] * s5[3] + h[3] * s5[2] + h[4] * s5[1];
    const uint64_t d1 = h[0] * r[1] + h[1] * r[0] + h[2] * s5[4] + h[3] * s5[3] + h[4] * s5[2];
    const uint64_t d2 = h[0] * r[2] + h[1] * r[1] + h[2] * r[0] + h[3] * s5[4] + h[4] * s5[3];
    const uint64_t d3 = h[0] * r[3] + h[1] * r[2] + h[2] * r[1] + h[3] * r[0] + h[4] * s5[4];
    const uint64_t d4 = h[0] * r[4] + h[1] * r[3] + h[2] * r[2] + h[3] * r[1] + h[4] * r[0];
    uint64_t cc = d0 >> 26;
    h[0] = d0 & M;
    uint64_t t = d1 + cc; cc = t >> 26; h[1] = t & M;
    t = d2 + cc; cc = t >> 26; h[2] = t & M;
    t = d3 + cc; cc = t >> 26; h[3] = t & M;
    t = d4 + cc; cc = t >> 26; h[4] = t & M;
    h[0] += cc * 5;
    cc = h[0] >> 26; h[0] &= M; h[1] += cc;
  }
  // full carry, then subtract p once if h >= p
  uint64_t cc = 0;
  for (int k = 0; k < 2; ++k) {
    for (int i = 0; i < 5; ++i) {
      h[i] += cc;
      cc = h[i] >> 26;
      h[i] &= M;
    }
    h[0] += cc * 5;
    cc = 0;
  }
  uint64_t g[5];
  cc = 5;
  for (int i = 0; i < 5; ++i) {
    g[i] = h[i] + cc;
    cc = g[i] >> 26;
    g[i] &= M;
  }
  const uint64_t use_g = 0 - cc;  // all ones when h + 5 reached 2^130
  for (int i = 0; i < 5; ++i) h[i] = (g[i] & use_g) | (h[i] & ~use_g);
  unsigned __int128 acc = (unsigned __int128)h[0] | (unsigned __int128)h[1] << 26 | (unsigned __int128)h[2] << 52 |
                          (unsigned __int128)h[3] << 78 | (unsigned __int128)h[4] << 104;
  acc += (unsigned __int128)le64(key + 24) << 64 | le64(key + 16);
  put_le64(tag, (uint64_t)acc);
  put_le64(tag + 8, (uint64_t)(acc >> 64));
}

void aead_tag(const uint8_t key[32], const uint8_t nonce[12], const uint8_t* aad, size_t na, const uint8_t* ct,
              size_t nc, uint8_t tag[16]) {
  uint8_t otk[64];
  chacha_block(key, 0, nonce, otk);
  std::vector<uint8_t> mac(aad, aad + na);
  mac.resize((mac.size() + 15) / 16 * 16, 0);
  mac.insert(mac.end(), ct, ct + nc);
  mac.resize((mac.size() + 15) / 16 * 16, 0);
  uint8_t l[16];
  put_le64(l, na);
  put_le64(l + 8, nc);
  mac.insert(mac.end(), l, l + 16);
  poly1305(otk, mac.data(), mac.size(), tag);
}

// ================================================================================================ GF(2^255 - 19)
typedef uint64_t fe[5];
typedef unsigned __int128 u128;
const uint64_t M51 = (1ull << 51) - 1;

void fe_copy(fe r, const fe a) { memcpy(r, a, sizeof(fe)); }
void fe_set(fe r, uint64_t v) {
  r[0] = v;
  r[1] = r[2] = r[3] = r[4] = 0;
}
void fe_carry(fe r) {
  for (int k = 0; k < 2; ++k) {
    uint64_t c = 0;
    for (int i = 0; i < 5; ++i) {
      r[i] += c;
      c = r[i] >> 51;
      r[i] &= M51;
    }
    r[0] += c * 19;
  }
}
void fe_add(fe r, const fe a, const fe b) {
  for (int i = 0; i < 5; ++i) r[i] = a[i] + b[i];
  fe_carry(r);
}
void fe_sub(fe r, const fe a, const fe b) {  // a + 4p - b keeps every limb positive
  const uint64_t p0 = 4 * (M51 - 18), pi = 4 * M51;
  r[0] = a[0] + p0 - b[0];
  for (int i = 1; i < 5; ++i) r[i] = a[i] + pi - b[i];
  fe_carry(r);
}
void fe_mul(fe r, const fe a, const fe b) {
  const uint64_t b19[5] = {b[0] * 19, b[1] * 19, b[2] * 19, b[3] * 19, b[4] * 19};
  u128 t[5];
  t[0] = (u128)a[0] * b[0] + (u128)a[1] * b19[4] + (u128)a[2] * b19[3] + (u128)a[3] * b19[2] + (u128)a[4] * b19[1];
  t[1] = (u128)a[0] * b[1] + (u128)a[1] * b[0] + (u128)a[2] * b19[4] + (u128)a[3] * b19[3] + (u128)a[4] * b19[2];
  t[2] = (u128)a[0] * b[2] + (u128)a[1] * b[1] + (u128)a[2] * b[0] + (u128)a[3] * b19[4] + (u128)a[4] * b19[3];
  t[3] = (u128)a[0] * b[3] + (u128)a[1] * b[2] + (u128)a[2] * b[1] + (u128)a[3] * b[0] + (u128)a[4] * b19[4];
  t[4] = (u128)a[0] * b[4] + (u128)a[1] * b[3] + (u128)a[2] * b[2] + (u128)a[3] * b[1] + (u128)a[4] * b[0];
  u128 c = 0;
  for (int i = 0; i < 5; ++i) {
    t[i] += c;
    c = t[i] >> 51;
    r[i] = (uint64_t)t[i] & M51;
  }
  r[0] += (uint64_t)c * 19;
  fe_carry(r);
}
void fe_sq(fe r, const fe a) { fe_mul(r, a, a); }
void fe_mul_small(fe r, const fe a, uint64_t s) {
  u128 c = 0;
  for (int i = 0; i < 5; ++i) {
    const u128 t = (u128)a[i] * s + c;
    r[i] = (uint64_t)t & M51;
    c = t >> 51;
  }
  r[0] += (uint64_t)c * 19;
  fe_carry(r);
}
// a^e for a 32-byte little-endian exponent
void fe_pow(fe r, const fe a, const uint8_t e[32]) {
  fe acc, base;
  fe_set(acc, 1);
  fe_copy(base, a);
  for (int i = 0; i < 256; ++i) {
    if ((e[i >> 3] >> (i & 7)) & 1) fe_mul(acc, acc, base);
    fe_sq(base, base);
  }
  fe_copy(r, acc);
}
// p - 2 and (p + 3) / 8 and (p - 1) / 4, little-endian
void exp_bytes(uint8_t e[32], int which) {
  // p = 2^255 - 19 = 0x7fff..ffed
  uint8_t p[32];
  memset(p, 0xff, 32);
  p[0] = 0xed;
  p[31] = 0x7f;
  memcpy(e, p, 32);
  if (which == 0) {  // p - 2
    e[0] = 0xeb;
  } else if (which == 1) {  // (p + 3) / 8 = 2^252 - 2
    memset(e, 0xff, 32);
    e[0] = 0xfe;
    e[31] = 0x0f;
  } else {  // (p - 1) / 4 = 2^253 - 5
    memset(e, 0xff, 32);
    e[0] = 0xfb;
    e[31] = 0x1f;
  }
}
void fe_inv(fe r, const fe a) {
  uint8_t e[32];
  exp_bytes(e, 0);
  fe_pow(r, a, e);
}
void fe_frombytes(fe h, const uint8_t s[32]) {
  h[0] = le64(s) & M51;
  h[1] = (le64(s + 6) >> 3) & M51;
  h[2] = (le64(s + 12) >> 6) & M51;
  h[3] = (le64(s + 19) >> 1) & M51;
  h[4] = (le64(s + 24) >> 12) & M51;
}
void fe_tobytes(uint8_t s[32], const fe a) {
  fe h;
  fe_copy(h, a);
  fe_carry(h);
  uint64_t q = (h[0] + 19) >> 51;
  for (int i = 1; i < 5; ++i) q = (h[i] + q) >> 51;  // 1 exactly when h >= p
  h[0] += 19 * q;
  uint64_t c = 0;
  for (int i = 0; i < 5; ++i) {
    h[i] += c;
    c = h[i] >> 51;
    h[i] &= M51;
  }
  put_le64(s, h[0] | h[1] << 51);
  put_le64(s + 8, h[1] >> 13 | h[2] << 38);
  put_le64(s + 16, h[2] >> 26 | h[3] << 25);
  put_le64(s + 24, h[3] >> 39 | h[4] << 12);
}
bool fe_iszero(const fe a) {
  uint8_t s[32];
  fe_tobytes(s, a);
  uint8_t o = 0;
  for (int i = 0; i < 32; ++i) o |= s[i];
  return o == 0;
}
bool fe_isodd(const fe a) {
  uint8_t s[32];
  fe_tobytes(s, a);
  return s[0] & 1;
}
bool fe_eq(const fe a, const fe b) {
  fe d;
  fe_sub(d, a, b);
  return fe_iszero(d);
}
void fe_neg(fe r, const fe a) {
  fe z;
  fe_set(z, 0);
  fe_sub(r, z, a);
}
void fe_cswap(fe a, fe b, uint64_t bit) {
  const uint64_t m = 0 - bit;
  for (int i = 0; i < 5; ++i) {
    const uint64_t t = m & (a[i] ^ b[i]);
    a[i] ^= t;
    b[i] ^= t;
  }
}

// X25519 Montgomery ladder (RFC 7748 5) on a clamped scalar.
void x25519(uint8_t out[32], const uint8_t scalar[32], const uint8_t u_in[32]) {
  uint8_t k[32];
  memcpy(k, scalar, 32);
  k[0] &= 248;
  k[31] &= 127;
  k[31] |= 64;
  uint8_t ub[32];
  memcpy(ub, u_in, 32);
  ub[31] &= 127;
  fe x1, x2, z2, x3, z3, A, AA, B, BB, E, C, D, DA, CB, t;
  fe_frombytes(x1, ub);
  fe_set(x2, 1);
  fe_set(z2, 0);
  fe_copy(x3, x1);
  fe_set(z3, 1);
  uint64_t swap = 0;
  for (int i = 254; i >= 0; --i) {
    const uint64_t bit = (k[i >> 3] >> (i & 7)) & 1;
    swap ^= bit;
    fe_cswap(x2, x3, swap);
    fe_cswap(z2, z3, swap);
    swap = bit;
    fe_add(A, x2, z2);
    fe_sq(AA, A);
    fe_sub(B, x2, z2);
    fe_sq(BB, B);
    fe_sub(E, AA, BB);
    fe_add(C, x3, z3);
    fe_sub(D, x3, z3);
    fe_mul(DA, D, A);
    fe_mul(CB, C, B);
    fe_add(t, DA, CB);
    fe_sq(x3, t);
    fe_sub(t, DA, CB);
    fe_sq(t, t);
    fe_mul(z3, x1, t);
    fe_mul(x2, AA, BB);
    fe_mul_small(t, E, 121665);
    fe_add(t, AA, t);
    fe_mul(z2, E, t);
  }
  fe_cswap(x2, x3, swap);
  fe_cswap(z2, z3, swap);
  fe_inv(z2, z2);
  fe_mul(x2, x2, z2);
  fe_tobytes(out, x2);
}

// ================================================================================================ Ed25519
struct Pt {
  fe X, Y, Z, T;
};
struct EdConst {
  fe d, d2, sqrtm1;
  Pt B;
  bool ready = false;
};
EdConst g_ed;

void pt_add(Pt& r, const Pt& p, const Pt& q) {  // complete for a = -1 (doubling included)
  fe a, b, c, d, e, f, g, h, t;
  fe_sub(a, p.Y, p.X);
  fe_sub(t, q.Y, q.X);
  fe_mul(a, a, t);
  fe_add(b, p.Y, p.X);
  fe_add(t, q.Y, q.X);
  fe_mul(b, b, t);
  fe_mul(c, p.T, q.T);
  fe_mul(c, c, g_ed.d2);
  fe_mul(d, p.Z, q.Z);
  fe_add(d, d, d);
  fe_sub(e, b, a);
  fe_sub(f, d, c);
  fe_add(g, d, c);
  fe_add(h, b, a);
  fe_mul(r.X, e, f);
  fe_mul(r.Y, g, h);
  fe_mul(r.T, e, h);
  fe_mul(r.Z, f, g);
}
void pt_zero(Pt& p) {
  fe_set(p.X, 0);
  fe_set(p.Y, 1);
  fe_set(p.Z, 1);
  fe_set(p.T, 0);
}
void pt_cswap(Pt& a, Pt& b, uint64_t bit) {
  fe_cswap(a.X, b.X, bit);
  fe_cswap(a.Y, b.Y, bit);
  fe_cswap(a.Z, b.Z, bit);
  fe_cswap(a.T, b.T, bit);
}
// [k]P for a 32-byte little-endian scalar, ladder-style (same operations for every bit)
void pt_mul(Pt& r, const Pt& P, const uint8_t k[32]) {
  Pt r0, r1 = P;
  pt_zero(r0);
  for (int i = 255; i >= 0; --i) {
    const uint64_t bit = (k[i >> 3] >> (i & 7)) & 1;
    pt_cswap(r0, r1, bit);
    pt_add(r1, r0, r1);
    pt_add(r0, r0, r0);
    pt_cswap(r0, r1, bit);
  }
  r = r0;
}
void pt_encode(uint8_t s[32], const Pt& p) {
  fe zi, x, y;
  fe_inv(zi, p.Z);
  fe_mul(x, p.X, zi);
  fe_mul(y, p.Y, zi);
  fe_tobytes(s, y);
  s[31] |= (uint8_t)(fe_isodd(x) << 7);
}
// x from y and the sign bit (RFC 8032 5.1.3); false when no point has this y.
bool recover_x(fe x, const fe y, int sign) {
  fe y2, u, v, x2, one, t;
  fe_set(one, 1);
  fe_sq(y2, y);
  fe_sub(u, y2, one);
  fe_mul(v, g_ed.d, y2);
  fe_add(v, v, one);
  fe_inv(t, v);
  fe_mul(x2, u, t);
  if (fe_iszero(x2)) {
    if (sign) return false;
    fe_set(x, 0);
    return true;
  }
  uint8_t e[32];
  exp_bytes(e, 1);
  fe_pow(x, x2, e);
  fe_sq(t, x);
  if (!fe_eq(t, x2)) fe_mul(x, x, g_ed.sqrtm1);
  fe_sq(t, x);
  if (!fe_eq(t, x2)) return false;
  if ((int)fe_isodd(x) != sign) fe_neg(x, x);
  return true;
}
bool pt_decode(Pt& p, const uint8_t s[32]) {
  uint8_t b[32];
  memcpy(b, s, 32);
  const int sign = b[31] >> 7;
  b[31] &= 127;
  fe_frombytes(p.Y, b);
  uint8_t chk[32];
  fe_tobytes(chk, p.Y);
  if (memcmp(chk, b, 32) != 0) return false;  // y >= p is not canonical
  if (!recover_x(p.X, p.Y, sign)) return false;
  fe_set(p.Z, 1);
  fe_mul(p.T, p.X, p.Y);
  return true;
}
void ed_init() {
  if (g_ed.ready) return;
  fe a, b;
  fe_set(a, 121665);
  fe_neg(a, a);
  fe_set(b, 121666);
  fe_inv(b, b);
  fe_mul(g_ed.d, a, b);  // d = -121665 / 121666
  fe_add(g_ed.d2, g_ed.d, g_ed.d);
  fe two;
  fe_set(two, 2);
  uint8_t e[32];
  exp_bytes(e, 2);
  fe_pow(g_ed.sqrtm1, two, e);  // 2^((p-1)/4) squares to -1
  fe four, five;
  fe_set(four, 4);
  fe_set(five, 5);
  fe_inv(five, five);
  fe_mul(g_ed.B.Y, four, five);  // base point: y = 4/5, x even
  recover_x(g_ed.B.X, g_ed.B.Y, 0);
  fe_set(g_ed.B.Z, 1);
  fe_mul(g_ed.B.T, g_ed.B.X, g_ed.B.Y);
  g_ed.ready = true;
}

// Scalars mod L = 2^252 + 27742317777372353535851937790883648493, as 32-bit limbs.
const uint32_t L_LIMBS[8] = {0x5cf5d3ed, 0x5812631a, 0xa2f79cd6, 0x14def9de, 0, 0, 0, 0x10000000};

bool ge_L(const uint32_t r[9]) {
  if (r[8]) return true;
  for (int i = 7; i >= 0; --i) {
    if (r[i] != L_LIMBS[i]) return r[i] > L_LIMBS[i];
  }
  return true;
}
// x (n little-endian bytes) mod L, by binary long division from the top bit.
void mod_L(uint8_t out[32], const uint8_t* x, size_t n) {
  uint32_t r[9] = {0};
  for (int i = (int)n * 8 - 1; i >= 0; --i) {
    uint32_t c = (x[i >> 3] >> (i & 7)) & 1;
    for (int j = 0; j < 9; ++j) {
      const uint32_t nc = r[j] >> 31;
      r[j] = (r[j] << 1) | c;
      c = nc;
    }
    if (ge_L(r)) {
      uint64_t borrow = 0;
      for (int j = 0; j < 9; ++j) {
        const uint64_t s = (uint64_t)r[j] - (j < 8 ? L_LIMBS[j] : 0) - borrow;
        r[j] = (uint32_t)s;
        borrow = (s >> 63) & 1;
      }
    }
  }
  for (int j = 0; j < 8; ++j) put_le32(out + 4 * j, r[j]);
}
// (a * b + c) mod L for 32-byte scalars
void muladd_L(uint8_t out[32], const uint8_t a[32], const uint8_t b[32], const uint8_t c[32]) {
  uint64_t t[17] = {0};
  for (int i = 0; i < 8; ++i) {
    uint64_t carry = 0;
    const uint64_t ai = le32(a + 4 * i);
    for (int j = 0; j < 8; ++j) {
      const u128 s = (u128)ai * le32(b + 4 * j) + t[i + j] + carry;
      t[i + j] = (uint64_t)s & 0xffffffffu;
      carry = (uint64_t)(s >> 32);
    }
    t[i + 8] += carry;
  }
  uint64_t carry = 0;
  for (int i = 0; i < 17; ++i) {
    const uint64_t s = t[i] + (i < 8 ? le32(c + 4 * i) : 0) + carry;
    t[i] = s & 0xffffffffu;
    carry = s >> 32;
  }
  uint8_t buf[68];
  for (int i = 0; i < 17; ++i) put_le32(buf + 4 * i, (uint32_t)t[i]);
  mod_L(out, buf, 68);
}

void ed_expand(const uint8_t seed[32], uint8_t a[32], uint8_t prefix[32]) {
  uint8_t h[64];
  sha512(seed, 32, h);
  memcpy(a, h, 32);
  a[0] &= 248;
  a[31] &= 127;
  a[31] |= 64;
  memcpy(prefix, h + 32, 32);
}

}  // namespace

extern "C" {

// ================================================================================================ hashes, MACs, KDFs
int aether_sha256(const void* msg, int n, void* out) {
  if (!msg || !out || n < 0) return -1;
  sha256((const uint8_t*)msg, n, (uint8_t*)out);
  return 32;
}
int aether_sha512(const void* msg, int n, void* out) {
  if (!msg || !out || n < 0) return -1;
  sha512((const uint8_t*)msg, n, (uint8_t*)out);
  return 64;
}
int aether_hmac_sha256(const void* key, int nk, const void* msg, int nm, void* out) {
  if (!key || !msg || !out || nk < 0 || nm < 0) return -1;
  hmac256((const uint8_t*)key, nk, (const uint8_t*)msg, nm, (uint8_t*)out);
  return 32;
}
// PRK = HMAC(salt, ikm); an absent salt is 32 zero bytes (the same key after HMAC's padding).
int aether_hkdf_extract(const void* salt, int ns, const void* ikm, int ni, void* out) {
  if (!ikm || !out || ns < 0 || ni < 0) return -1;
  static const uint8_t zero = 0;
  hmac256(salt ? (const uint8_t*)salt : &zero, salt ? ns : 0, (const uint8_t*)ikm, ni, (uint8_t*)out);
  return 32;
}
int aether_hkdf_expand(const void* prk, int np, const void* info, int ni, void* out, int n) {
  if (!prk || !out || np != 32 || ni < 0 || n <= 0 || n > 255 * 32 || (ni > 0 && !info)) return -1;
  hkdf_expand((const uint8_t*)prk, np, (const uint8_t*)info, ni, (uint8_t*)out, n);
  return n;
}
// HKDF-Expand(secret, HkdfLabel{length, "tls13 " + label, context}, length)
int aether_tls13_hkdf_expand_label(const void* secret, int ns, const void* label, int nl, const void* ctx, int nc,
                                   void* out, int n) {
  if (!secret || !label || !out || ns != 32 || nl <= 0 || nl > 255 || nc < 0 || nc > 255 || n <= 0 || n > 0xffff)
    return -1;
  if (nc > 0 && !ctx) return -1;
  const std::string full = "tls13 " + std::string((const char*)label, nl);
  if (full.size() > 255) return -1;
  std::vector<uint8_t> info = {(uint8_t)(n >> 8), (uint8_t)n, (uint8_t)full.size()};
  info.insert(info.end(), full.begin(), full.end());
  info.push_back((uint8_t)nc);
  if (nc) info.insert(info.end(), (const uint8_t*)ctx, (const uint8_t*)ctx + nc);
  if (n > 255 * 32) return -1;
  hkdf_expand((const uint8_t*)secret, 32, info.data(), info.size(), (uint8_t*)out, n);
  return n;
}

// ================================================================================================ AEAD
// out = ciphertext || 16-byte tag; returns n_plain + 16.
int aether_chacha20_poly1305_encrypt(const void* key, const void* nonce, const void* aad, int na, const void* plain,
                                     int np, void* out, int max_out) {
  if (!key || !nonce || !out || na < 0 || np < 0 || (na && !aad) || (np && !plain) || np + 16 > max_out) return -1;
  uint8_t* o = (uint8_t*)out;
  chacha_xor((const uint8_t*)key, 1, (const uint8_t*)nonce, (const uint8_t*)plain, o, np);
  aead_tag((const uint8_t*)key, (const uint8_t*)nonce, (const uint8_t*)aad, na, o, np, o + np);
  return np + 16;
}
// Checks the tag first (constant-time compare); -2 on mismatch, else the plaintext length.
int aether_chacha20_poly1305_decrypt(const void* key, const void* nonce, const void* aad, int na, const void* in,
                                     int n, void* out, int max_out) {
  if (!key || !nonce || !in || !out || na < 0 || n < 16 || (na && !aad) || n - 16 > max_out) return -1;
  const uint8_t* c = (const uint8_t*)in;
  uint8_t tag[16];
  aead_tag((const uint8_t*)key, (const uint8_t*)nonce, (const uint8_t*)aad, na, c, n - 16, tag);
  uint8_t diff = 0;
  for (int i = 0; i < 16; ++i) diff |= tag[i] ^ c[n - 16 + i];
  if (diff) return -2;
  chacha_xor((const uint8_t*)key, 1, (const uint8_t*)nonce, c, (uint8_t*)out, n - 16);
  return n - 16;
}

// ================================================================================================ curves
int aether_x25519_derive_public(const void* scalar, void* out) {
  if (!scalar || !out) return -1;
  uint8_t base[32] = {9};
  x25519((uint8_t*)out, (const uint8_t*)scalar, base);
  return 32;
}
int aether_x25519_shared_secret(const void* scalar, const void* peer, void* out) {
  if (!scalar || !peer || !out) return -1;
  x25519((uint8_t*)out, (const uint8_t*)scalar, (const uint8_t*)peer);
  return 32;
}
int aether_ed25519_derive_public(const void* seed, void* out_pub) {
  if (!seed || !out_pub) return -1;
  ed_init();
  uint8_t a[32], prefix[32];
  ed_expand((const uint8_t*)seed, a, prefix);
  Pt A;
  pt_mul(A, g_ed.B, a);
  pt_encode((uint8_t*)out_pub, A);
  return 32;
}
int aether_ed25519_sign(const void* seed, const void* pub, const void* msg, int n, void* out_sig) {
  if (!seed || !pub || !msg || !out_sig || n < 0) return -1;
  ed_init();
  uint8_t a[32], prefix[32], h[64], r[32], k[32];
  ed_expand((const uint8_t*)seed, a, prefix);
  const uint8_t* m = (const uint8_t*)msg;
  sha512_cat({{prefix, 32}, {m, (size_t)n}}, h);
  mod_L(r, h, 64);
  Pt R;
  pt_mul(R, g_ed.B, r);
  uint8_t* sig = (uint8_t*)out_sig;
  pt_encode(sig, R);
  sha512_cat({{sig, 32}, {(const uint8_t*)pub, 32}, {m, (size_t)n}}, h);
  mod_L(k, h, 64);
  muladd_L(sig + 32, k, a, r);  // S = r + k a
  return 64;
}
// 0 when the signature verifies, -1 otherwise.
int aether_ed25519_verify(const void* pub, const void* msg, int n, const void* sig) {
  if (!pub || !msg || !sig || n < 0) return -1;
  ed_init();
  const uint8_t* s = (const uint8_t*)sig;
  Pt A, R;
  if (!pt_decode(A, (const uint8_t*)pub) || !pt_decode(R, s)) return -1;
  uint32_t S[9] = {0};
  for (int i = 0; i < 8; ++i) S[i] = le32(s + 32 + 4 * i);
  if (ge_L(S)) return -1;  // S must be reduced
  uint8_t h[64], k[32];
  sha512_cat({{s, 32}, {(const uint8_t*)pub, 32}, {(const uint8_t*)msg, (size_t)n}}, h);
  mod_L(k, h, 64);
  Pt sB, kA, rhs;
  pt_mul(sB, g_ed.B, s + 32);
  pt_mul(kA, A, k);
  pt_add(rhs, R, kA);
  uint8_t e1[32], e2[32];
  pt_encode(e1, sB);
  pt_encode(e2, rhs);
  return memcmp(e1, e2, 32) == 0 ? 0 : -1;
}
int aether_random_bytes(void* out, int n) {
  if (!out || n < 0) return -1;
  int done = 0;
  while (done < n) {
    const ssize_t r = getrandom((uint8_t*)out + done, n - done, 0);
    if (r < 0) {
      if (errno == EINTR) continue;
      return -1;
    }
    done += (int)r;
  }
  return n;
}

// ================================================================================================ wire codecs
// One unmasked FIN text frame (server to client).
int aether_ws_encode_text_frame(const void* payload, int n, void* out, int max_out) {
  if (!payload || !out || n < 0 || max_out <= 0) return -1;
  uint8_t hdr[10];
  int h = 0;
  hdr[h++] = 0x81;
  if (n < 126) {
    hdr[h++] = (uint8_t)n;
  } else if (n < 65536) {
    hdr[h++] = 126;
    hdr[h++] = (uint8_t)(n >> 8);
    hdr[h++] = (uint8_t)n;
  } else {
    hdr[h++] = 127;
    put_be64(hdr + h, (uint64_t)n);
    h += 8;
  }
  if (h + n > max_out) return -1;
  memcpy(out, hdr, h);
  memcpy((uint8_t*)out + h, payload, n);
  return h + n;
}
// The payload of one frame (unmasked when the mask bit is set).
int aether_ws_decode_frame_payload(const void* buf, int n, void* out, int max_out) {
  if (!buf || !out || n < 2 || max_out <= 0) return -1;
  const uint8_t* b = (const uint8_t*)buf;
  const bool masked = b[1] & 0x80;
  uint64_t len = b[1] & 0x7f;
  size_t off = 2;
  if (len == 126) {
    if (n < 4) return -1;
    len = (uint64_t)b[2] << 8 | b[3];
    off = 4;
  } else if (len == 127) {
    if (n < 10) return -1;
    len = be64(b + 2);
    off = 10;
  }
  uint8_t mask[4] = {0, 0, 0, 0};
  if (masked) {
    if ((size_t)n < off + 4) return -1;
    memcpy(mask, b + off, 4);
    off += 4;
  }
  if (len > (uint64_t)n - off || len > (uint64_t)max_out) return -1;
  for (uint64_t i = 0; i < len; ++i) ((uint8_t*)out)[i] = b[off + i] ^ mask[i & 3];
  return (int)len;
}
// Request line "METHOD SP PATH SP VERSION": method and path are copied back to
// back into out_strings; returns the offset of the body (after the blank line).
int aether_http_parse_request(const void* buf, int n, void* out_strings, int max_strings, int* out_method_len,
                              int* out_path_len) {
  if (!buf || !out_strings || !out_method_len || !out_path_len || n <= 0) return -1;
  const char* b = (const char*)buf;
  const std::string s(b, n);
  const size_t end = s.find("\r\n\r\n");
  const size_t eol = s.find("\r\n");
  if (end == std::string::npos) return -1;
  const size_t sp1 = s.find(' ');
  if (sp1 == std::string::npos || sp1 == 0 || sp1 > eol) return -1;
  const size_t sp2 = s.find(' ', sp1 + 1);
  if (sp2 == std::string::npos || sp2 > eol || sp2 == sp1 + 1) return -1;
  const int ml = (int)sp1, pl = (int)(sp2 - sp1 - 1);
  if (ml + pl > max_strings) return -1;
  memcpy(out_strings, b, ml);
  memcpy((char*)out_strings + ml, b + sp1 + 1, pl);
  *out_method_len = ml;
  *out_path_len = pl;
  return (int)(end + 4);
}
int aether_http_write_response_200(const void* body, int n, void* out, int max_out) {
  if (!out || n < 0 || (n && !body)) return -1;
  char hdr[96];
  const int h = snprintf(hdr, sizeof(hdr), "HTTP/1.1 200 OK\r\nContent-Length: %d\r\n\r\n", n);
  if (h + n > max_out) return -1;
  memcpy(out, hdr, h);
  if (n) memcpy((char*)out + h, body, n);
  return h + n;
}
// The /v1/chat/completions success body; strings are copied as given (the
// caller escapes them).
int aether_openai_render_completion(const void* id, int nid, const void* model, int nm, const void* content, int nc,
                                    int prompt_tokens, int completion_tokens, void* out, int max_out) {
  if (!id || !model || !content || !out || nid < 0 || nm < 0 || nc < 0) return -1;
  std::string s = "{\"id\":\"" + std::string((const char*)id, nid) +
                  "\",\"object\":\"chat.completion\",\"model\":\"" + std::string((const char*)model, nm) +
                  "\",\"choices\":[{\"index\":0,\"message\":{\"role\":\"assistant\",\"content\":\"" +
                  std::string((const char*)content, nc) + "\"},\"finish_reason\":\"stop\"}],\"usage\":{" +
                  "\"prompt_tokens\":" + std::to_string(prompt_tokens) +
                  ",\"completion_tokens\":" + std::to_string(completion_tokens) + "}}";
  if ((int)s.size() > max_out) return -1;
  memcpy(out, s.data(), s.size());
  return (int)s.size();
}

}  // extern "C"
