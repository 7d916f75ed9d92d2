"""Crypto and wire codecs of libaether_rt against independent implementations
(hashlib, hmac, the `cryptography` package) and RFC test vectors."""
import ctypes as C
import hashlib
import hmac
import json
import os

import pytest

from aether_b200 import runtime as rt

crypto = pytest.importorskip("cryptography")
from cryptography.hazmat.primitives import hashes, serialization  # noqa: E402
from cryptography.hazmat.primitives.asymmetric import ed25519, x25519  # noqa: E402
from cryptography.hazmat.primitives.ciphers.aead import ChaCha20Poly1305  # noqa: E402
from cryptography.hazmat.primitives.kdf.hkdf import HKDF, HKDFExpand  # noqa: E402


def _buf(n):
    return C.create_string_buffer(n)


def _raw(pub):
    return pub.public_bytes(serialization.Encoding.Raw, serialization.PublicFormat.Raw)


def test_group_order_limbs():
    L = 2 ** 252 + 27742317777372353535851937790883648493
    limbs = [0x5CF5D3ED, 0x5812631A, 0xA2F79CD6, 0x14DEF9DE, 0, 0, 0, 0x10000000]
    assert sum(v << (32 * i) for i, v in enumerate(limbs)) == L


@pytest.mark.parametrize("n", [0, 1, 55, 56, 63, 64, 111, 112, 127, 128, 1000])
def test_sha2_and_hmac(n):
    m = os.urandom(n) if n else b""
    o = _buf(64)
    assert rt.call("aether_sha256", m or b"\0", n, o) == 32 and o.raw[:32] == hashlib.sha256(m).digest()
    assert rt.call("aether_sha512", m or b"\0", n, o) == 64 and o.raw == hashlib.sha512(m).digest()
    for key in (b"k", os.urandom(64), os.urandom(100)):
        assert rt.call("aether_hmac_sha256", key, len(key), m or b"\0", n, o) == 32
        assert o.raw[:32] == hmac.new(key, m, hashlib.sha256).digest()


def test_hkdf_and_tls13_label():
    salt, ikm, info = os.urandom(13), os.urandom(40), b"context info"
    prk = _buf(32)
    assert rt.call("aether_hkdf_extract", salt, len(salt), ikm, len(ikm), prk) == 32
    assert prk.raw == hmac.new(salt, ikm, hashlib.sha256).digest()
    out = _buf(100)
    assert rt.call("aether_hkdf_expand", prk, 32, info, len(info), out, 100) == 100
    want = HKDF(algorithm=hashes.SHA256(), length=100, salt=salt, info=info).derive(ikm)
    assert out.raw == want
    assert rt.call("aether_hkdf_extract", None, 0, ikm, len(ikm), prk) == 32  # absent salt = zeros
    assert prk.raw == hmac.new(b"\0" * 32, ikm, hashlib.sha256).digest()
    secret, ctx = os.urandom(32), hashlib.sha256(b"hello").digest()
    out = _buf(16)
    assert rt.call("aether_tls13_hkdf_expand_label", secret, 32, b"key", 3, ctx, 32, out, 16) == 16
    full = b"tls13 key"
    label = (16).to_bytes(2, "big") + bytes([len(full)]) + full + bytes([32]) + ctx
    assert out.raw == HKDFExpand(algorithm=hashes.SHA256(), length=16, info=label).derive(secret)
    assert rt.call("aether_hkdf_expand", prk, 31, info, len(info), out, 16) == -1


def test_chacha20_poly1305():
    # RFC 8439 2.8.2
    key = bytes(range(0x80, 0xA0))
    nonce = bytes.fromhex("070000004041424344454647")
    aad = bytes.fromhex("50515253c0c1c2c3c4c5c6c7")
    pt = (b"Ladies and Gentlemen of the class of '99: If I could offer you only one tip for the future, "
          b"sunscreen would be it.")
    out = _buf(len(pt) + 16)
    assert rt.call("aether_chacha20_poly1305_encrypt", key, nonce, aad, len(aad), pt, len(pt), out,
                   len(pt) + 16) == len(pt) + 16
    assert out.raw[-16:].hex() == "1ae10b594f09e26a7e902ecbd0600691"
    assert out.raw == ChaCha20Poly1305(key).encrypt(nonce, pt, aad)
    back = _buf(len(pt))
    assert rt.call("aether_chacha20_poly1305_decrypt", key, nonce, aad, len(aad), out.raw, len(pt) + 16, back,
                   len(pt)) == len(pt)
    assert back.raw == pt
    bad = bytearray(out.raw)
    bad[3] ^= 1
    assert rt.call("aether_chacha20_poly1305_decrypt", key, nonce, aad, len(aad), bytes(bad), len(bad), back,
                   len(pt)) == -2
    for n in (0, 1, 15, 16, 17, 64, 65, 300):  # block and padding edges, empty AAD
        k, nn, m = os.urandom(32), os.urandom(12), os.urandom(n)
        o = _buf(n + 16)
        assert rt.call("aether_chacha20_poly1305_encrypt", k, nn, None, 0, m or b"\0", n, o, n + 16) == n + 16
        assert o.raw == ChaCha20Poly1305(k).encrypt(nn, m, None)


def test_x25519():
    for _ in range(5):
        a, b = os.urandom(32), os.urandom(32)
        pa, pb, s1, s2 = _buf(32), _buf(32), _buf(32), _buf(32)
        assert rt.call("aether_x25519_derive_public", a, pa) == 32
        assert pa.raw == _raw(x25519.X25519PrivateKey.from_private_bytes(a).public_key())
        rt.call("aether_x25519_derive_public", b, pb)
        rt.call("aether_x25519_shared_secret", a, pb.raw, s1)
        rt.call("aether_x25519_shared_secret", b, pa.raw, s2)
        want = x25519.X25519PrivateKey.from_private_bytes(a).exchange(x25519.X25519PublicKey.from_public_bytes(pb.raw))
        assert s1.raw == s2.raw == want
    # RFC 7748 5.2 first vector
    k = bytes.fromhex("a546e36bf0527c9d3b16154b82465edd62144c0ac1fc5a18506a2244ba449ac4")
    u = bytes.fromhex("e6db6867583030db3594c1a424b15f7c726624ec26b3353b10a903a6d0ab1c4c")
    o = _buf(32)
    rt.call("aether_x25519_shared_secret", k, u, o)
    assert o.raw.hex() == "c3da55379de9c6908e94ea4df28d084f32eccf03491c71f754b4075577a28552"


def test_ed25519():
    for n in (0, 1, 100, 1000):
        seed, msg = os.urandom(32), os.urandom(n)
        pub, sig = _buf(32), _buf(64)
        assert rt.call("aether_ed25519_derive_public", seed, pub) == 32
        sk = ed25519.Ed25519PrivateKey.from_private_bytes(seed)
        assert pub.raw == _raw(sk.public_key())
        assert rt.call("aether_ed25519_sign", seed, pub.raw, msg or b"\0", n, sig) == 64
        assert sig.raw == sk.sign(msg)  # deterministic signatures: byte-identical
        assert rt.call("aether_ed25519_verify", pub.raw, msg or b"\0", n, sig.raw) == 0
        bad = bytearray(sig.raw)
        bad[10] ^= 4
        assert rt.call("aether_ed25519_verify", pub.raw, msg or b"\0", n, bytes(bad)) == -1
        if n:
            assert rt.call("aether_ed25519_verify", pub.raw, bytes([msg[0] ^ 1]) + msg[1:], n, sig.raw) == -1
    # RFC 8032 7.1 test 1 (empty message)
    seed = bytes.fromhex("9d61b19deffd5a60ba844af492ec2cc44449c5697b326919703bac031cae7f60")
    pub, sig = _buf(32), _buf(64)
    rt.call("aether_ed25519_derive_public", seed, pub)
    assert pub.raw.hex() == "d75a980182b10ab7d54bfed3c964073a0ee172f3daa62325af021a68f707511a"
    rt.call("aether_ed25519_sign", seed, pub.raw, b"\0", 0, sig)
    assert sig.raw.hex().startswith("e5564300c360ac729086e2cc806e828a84877f1eb8e5d974d873e06522490155")


def test_random_and_wire_codecs():
    a, b = _buf(64), _buf(64)
    assert rt.call("aether_random_bytes", a, 64) == 64 and rt.call("aether_random_bytes", b, 64) == 64
    assert a.raw != b.raw
    for n in (5, 200, 70000):
        payload = os.urandom(n)
        frame = _buf(n + 10)
        m = rt.call("aether_ws_encode_text_frame", payload, n, frame, n + 10)
        assert m == n + (2 if n < 126 else 4 if n < 65536 else 10) and frame.raw[0] == 0x81
        out = _buf(n)
        assert rt.call("aether_ws_decode_frame_payload", frame.raw, m, out, n) == n and out.raw == payload
    # a masked client frame (RFC 6455 5.7: "Hello")
    masked = bytes.fromhex("818537fa213d7f9f4d5158")
    out = _buf(16)
    assert rt.call("aether_ws_decode_frame_payload", masked, len(masked), out, 16) == 5 and out.raw[:5] == b"Hello"
    assert rt.call("aether_ws_decode_frame_payload", masked[:8], 8, out, 16) == -1  # truncated

    req = b"POST /v1/chat/completions HTTP/1.1\r\nHost: x\r\nContent-Length: 2\r\n\r\n{}"
    strings, ml, pl = _buf(64), C.c_int(), C.c_int()
    body = rt.call("aether_http_parse_request", req, len(req), strings, 64, C.byref(ml), C.byref(pl))
    assert req[body:] == b"{}"
    assert strings.raw[: ml.value] == b"POST" and strings.raw[ml.value : ml.value + pl.value] == b"/v1/chat/completions"
    assert rt.call("aether_http_parse_request", b"GET /\r\n", 7, strings, 64, C.byref(ml), C.byref(pl)) == -1
    out = _buf(128)
    n = rt.call("aether_http_write_response_200", b"hi", 2, out, 128)
    assert out.raw[:n] == b"HTTP/1.1 200 OK\r\nContent-Length: 2\r\n\r\nhi"
    out = _buf(512)
    n = rt.call("aether_openai_render_completion", b"cmpl-1", 6, b"qwen", 4, b"Hello there", 11, 7, 3, out, 512)
    doc = json.loads(out.raw[:n])
    assert doc["choices"][0]["message"]["content"] == "Hello there" and doc["usage"]["completion_tokens"] == 3
    assert rt.call("aether_openai_render_completion", b"a", 1, b"m", 1, b"c", 1, 1, 1, out, 10) == -1
