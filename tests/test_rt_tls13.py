"""TLS 1.3 sessions of libaether_rt: the in-process loopback, our server with
OpenSSL as the client, and our client with OpenSSL as the server (Python's ssl
module over memory BIOs, no sockets)."""
import ctypes as C
import datetime
import os
import ssl

import pytest

from aether_b200 import runtime as rt

crypto = pytest.importorskip("cryptography")
from cryptography import x509  # noqa: E402
from cryptography.hazmat.primitives import serialization  # noqa: E402
from cryptography.hazmat.primitives.asymmetric import ed25519  # noqa: E402
from cryptography.x509.oid import NameOID  # noqa: E402

L = C.c_int64


def _lib():
    lb = rt.lib()
    lb.aether_tls13_server_new.restype = L
    lb.aether_tls13_client_new.restype = L
    for n in ("server_feed", "client_feed", "server_take_outbound", "client_take_outbound", "server_send",
              "client_send", "server_is_done", "client_is_done", "server_free", "client_free"):
        getattr(lb, "aether_tls13_" + n).argtypes = [L] + [C.c_void_p, C.c_int] * (
            2 if n.endswith("feed") else 1 if ("send" in n or "take" in n) else 0)
    return lb


def _take(lb, side, h):
    buf = C.create_string_buffer(1 << 17)
    n = getattr(lb, f"aether_tls13_{side}_take_outbound")(L(h), buf, 1 << 17)
    assert n >= 0
    return buf.raw[:n]


def _feed(lb, side, h, data):
    app = C.create_string_buffer(1 << 16)
    n = getattr(lb, f"aether_tls13_{side}_feed")(L(h), data or b"\0", len(data), app, 1 << 16)
    assert n >= 0, (side, n)
    return app.raw[:n]


def _ssl_step(obj):
    try:
        obj.do_handshake()
        return True
    except ssl.SSLWantReadError:
        return False


def test_loopback_smoke():
    assert rt.lib().aether_tls13_self_loopback_smoke() == 42


def test_our_server_with_openssl_client():
    lb = _lib()
    seed = os.urandom(32)
    h = lb.aether_tls13_server_new(seed, os.urandom(32), os.urandom(32), b"aether.test", 11, b"\x9a\x01", 2)
    assert h >= 0
    ctx = ssl.SSLContext(ssl.PROTOCOL_TLS_CLIENT)
    ctx.check_hostname = False
    ctx.verify_mode = ssl.CERT_NONE
    ctx.minimum_version = ssl.TLSVersion.TLSv1_3
    inc, outg = ssl.MemoryBIO(), ssl.MemoryBIO()
    cli = ctx.wrap_bio(inc, outg, server_side=False)
    done = False
    for _ in range(10):
        done = _ssl_step(cli)
        data = outg.read()
        if data:
            _feed(lb, "server", h, data)
        back = _take(lb, "server", h)
        if back:
            inc.write(back)
        if done and lb.aether_tls13_server_is_done(L(h)) == 1:
            break
    assert done and lb.aether_tls13_server_is_done(L(h)) == 1
    assert cli.version() == "TLSv1.3" and cli.cipher()[0] == "TLS_CHACHA20_POLY1305_SHA256"
    # the certificate OpenSSL received: our self-signed Ed25519 one, with a valid signature
    cert = x509.load_der_x509_certificate(cli.getpeercert(binary_form=True))
    assert cert.subject.get_attributes_for_oid(NameOID.COMMON_NAME)[0].value == "aether.test"
    assert cert.serial_number == 0x9A01
    pub = cert.public_key()
    pub.verify(cert.signature, cert.tbs_certificate_bytes)
    want = ed25519.Ed25519PrivateKey.from_private_bytes(seed).public_key()
    assert pub.public_bytes_raw() == want.public_bytes_raw()
    # application data both ways, including a record larger than 2^14 bytes
    cli.write(b"hello server")
    assert _feed(lb, "server", h, outg.read()) == b"hello server"
    big = os.urandom(40000)
    assert lb.aether_tls13_server_send(L(h), big, len(big)) == len(big)
    inc.write(_take(lb, "server", h))
    got = b""
    while len(got) < len(big):
        got += cli.read(65536)
    assert got == big
    assert lb.aether_tls13_server_free(L(h)) == 0


def test_our_client_with_openssl_server(tmp_path):
    key = ed25519.Ed25519PrivateKey.generate()
    name = x509.Name([x509.NameAttribute(NameOID.COMMON_NAME, "openssl.test")])
    now = datetime.datetime.now(datetime.timezone.utc)
    cert = (x509.CertificateBuilder().subject_name(name).issuer_name(name).public_key(key.public_key())
            .serial_number(7).not_valid_before(now - datetime.timedelta(days=1))
            .not_valid_after(now + datetime.timedelta(days=1)).sign(key, None))
    cf, kf = tmp_path / "c.pem", tmp_path / "k.pem"
    cf.write_bytes(cert.public_bytes(serialization.Encoding.PEM))
    kf.write_bytes(key.private_bytes(serialization.Encoding.PEM, serialization.PrivateFormat.PKCS8,
                                     serialization.NoEncryption()))
    ctx = ssl.SSLContext(ssl.PROTOCOL_TLS_SERVER)
    ctx.minimum_version = ssl.TLSVersion.TLSv1_3
    ctx.load_cert_chain(str(cf), str(kf))
    inc, outg = ssl.MemoryBIO(), ssl.MemoryBIO()
    srv = ctx.wrap_bio(inc, outg, server_side=True)
    lb = _lib()
    h = lb.aether_tls13_client_new(os.urandom(32), os.urandom(32), os.urandom(32), 32)
    assert h >= 0
    done = False
    for _ in range(10):
        data = _take(lb, "client", h)
        if data:
            inc.write(data)
        done = _ssl_step(srv)
        back = outg.read()
        if back:
            _feed(lb, "client", h, back)
        if done and lb.aether_tls13_client_is_done(L(h)) == 1:
            break
    assert done and lb.aether_tls13_client_is_done(L(h)) == 1
    data = _take(lb, "client", h)  # anything still queued (nothing, or alerts)
    if data:
        inc.write(data)
    assert srv.cipher()[0] == "TLS_CHACHA20_POLY1305_SHA256"
    assert lb.aether_tls13_client_send(L(h), b"GET / please", 12) == 12
    inc.write(_take(lb, "client", h))
    assert srv.read(100) == b"GET / please"
    srv.write(b"pong from openssl")
    got = _feed(lb, "client", h, outg.read())  # session tickets ride along and are ignored
    assert got == b"pong from openssl"
    # a tampered record kills the session
    lb.aether_tls13_client_send(L(h), b"x", 1)
    srv.write(b"more")
    rec = bytearray(outg.read())
    rec[-1] ^= 1
    app = C.create_string_buffer(64)
    assert lb.aether_tls13_client_feed(L(h), bytes(rec), len(rec), app, 64) == -1
    assert lb.aether_tls13_client_free(L(h)) == 0
