"""HTTP/2 and HPACK: the Huffman table is a complete canonical prefix code that
round-trips every byte string; HPACK blocks round-trip; the native session
answers an in-process client; and curl (nghttp2) talks h2c to an ASGI app
served through serving.h2, including streamed bodies, large bodies that need
flow-control window updates, and concurrent streams."""
import asyncio
import ctypes as C
import json
import os
import shutil
import socket
import subprocess
import threading
from fractions import Fraction

import pytest

from aether_b200 import runtime as rt


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_huffman_table_is_complete_canonical_prefix_code():
    lb = rt.lib()
    codes = {}
    for s in range(257):
        c = C.c_uint32()
        n = lb.aether_hpack_huffman_code(s, C.byref(c))
        assert 5 <= n <= 30
        codes[s] = format(c.value, f"0{n}b")
    assert sum(Fraction(1, 2 ** len(c)) for c in codes.values()) == 1  # Kraft equality: complete
    items = sorted(codes.items(), key=lambda kv: (len(kv[1]), kv[0]))
    for (_, a), (_, b) in zip(items, items[1:]):  # canonical, hence prefix-free
        assert int(b, 2) == (int(a, 2) + 1) << (len(b) - len(a))
    assert codes[256] == "1" * 30  # EOS
    assert codes[ord("0")] == "00000" and codes[ord("a")] == "00011"
    for data in (b"", b"www.example.com", bytes(range(256)), os.urandom(1000)):
        enc = C.create_string_buffer(4 * len(data) + 8)
        n = lb.aether_hpack_huffman_encode(data or b"\0", len(data), enc, len(enc))
        dec = C.create_string_buffer(len(data) + 8)
        m = lb.aether_hpack_huffman_decode(enc.raw[:n] or b"\0", n, dec, len(dec))
        assert dec.raw[:m] == data
    # RFC 7541 C.4.1: "www.example.com" Huffman-coded
    enc = C.create_string_buffer(32)
    n = lb.aether_hpack_huffman_encode(b"www.example.com", 15, enc, 32)
    assert enc.raw[:n].hex() == "f1e3c2e5f23a6ba0ab90f4ff"
    # padding longer than 7 bits or not all ones is refused
    assert lb.aether_hpack_huffman_decode(b"\xff\xff", 2, dec, 8) == -1


def test_hpack_round_trip_and_static_table():
    lb = rt.lib()
    lines = b":method: GET\n:path: /v1/models\n:scheme: http\nuser-agent: aether\nx-custom: a b c\n"
    enc = C.create_string_buffer(512)
    n = lb.aether_hpack_encode(lines, len(lines), enc, 512)
    assert enc.raw[0] == 0x82  # indexed :method GET
    out = C.create_string_buffer(512)
    m = lb.aether_hpack_decode(enc.raw[:n], n, out, 512)
    assert out.raw[:m] == lines
    # a block with incremental indexing then a dynamic-table reference (RFC 7541 C.3.1 / C.3.2 style)
    blk = bytes.fromhex("828684410f7777772e6578616d706c652e636f6d") + bytes.fromhex("be")
    m = lb.aether_hpack_decode(blk, len(blk), out, 512)
    assert out.raw[:m].decode().splitlines() == [":method: GET", ":scheme: http", ":path: /",
                                                 ":authority: www.example.com", ":authority: www.example.com"]


def test_loopback_smoke():
    assert rt.lib().aether_http2_self_loopback_smoke() == 42


@pytest.fixture(scope="module")
def h2_server():
    if not shutil.which("curl"):
        pytest.skip("curl not available")
    from aether_b200.serving.h2 import serve

    async def app(scope, receive, send):
        msg = await receive()
        body = msg.get("body", b"")
        path = scope["path"]
        if path == "/stream":
            await send({"type": "http.response.start", "status": 200, "headers": [(b"content-type", b"text/event-stream")]})
            for i in range(5):
                await send({"type": "http.response.body", "body": f"data: {i}\n\n".encode(), "more_body": True})
                await asyncio.sleep(0.01)
            await send({"type": "http.response.body", "body": b"", "more_body": False})
            return
        if path == "/big":
            payload = bytes(range(256)) * 1024  # 256 KiB: needs window updates from the client
        else:
            payload = json.dumps({"method": scope["method"], "path": path, "query": scope["query_string"].decode(),
                                  "len": len(body), "ua": dict(scope["headers"]).get(b"user-agent", b"").decode(),
                                  "version": scope["http_version"]}).encode()
        await send({"type": "http.response.start", "status": 200 if path != "/missing" else 404,
                    "headers": [(b"content-type", b"application/json"), (b"x-served-by", b"aether")]})
        await send({"type": "http.response.body", "body": payload, "more_body": False})

    port = _free_port()
    loop = asyncio.new_event_loop()
    ready = threading.Event()

    def run():
        asyncio.set_event_loop(loop)
        ev = asyncio.Event()

        async def main():
            task = asyncio.ensure_future(serve(app, "127.0.0.1", port, ev))
            await ev.wait()
            ready.set()
            await task

        try:
            loop.run_until_complete(main())
        except BaseException:  # cancelled at teardown
            pass

    th = threading.Thread(target=run, daemon=True)
    th.start()
    assert ready.wait(10)
    yield port
    for t in asyncio.all_tasks(loop):
        loop.call_soon_threadsafe(t.cancel)


def _curl(port, *args):
    out = subprocess.run(["curl", "-s", "--http2-prior-knowledge", "--max-time", "10", *args],
                         capture_output=True, timeout=30)
    assert out.returncode == 0, out.stderr
    return out.stdout


def test_curl_h2c_requests(h2_server):
    port = h2_server
    doc = json.loads(_curl(port, f"http://127.0.0.1:{port}/v1/models?x=1"))
    assert doc == {"method": "GET", "path": "/v1/models", "query": "x=1", "len": 0, "ua": doc["ua"], "version": "2"}
    assert doc["ua"].startswith("curl/")
    body = json.dumps({"prompt": "hi" * 5000}).encode()
    post = subprocess.run(["curl", "-s", "--http2-prior-knowledge", "--max-time", "10", "-X", "POST",
                           "--data-binary", "@-", f"http://127.0.0.1:{port}/v1/completions"],
                          input=body, capture_output=True, timeout=30)
    doc = json.loads(post.stdout)
    assert doc["method"] == "POST" and doc["len"] == len(body)
    head = _curl(port, "-D", "-", "-o", "/dev/null", f"http://127.0.0.1:{port}/missing").decode()
    assert head.startswith("HTTP/2 404") and "x-served-by: aether" in head
    big = _curl(port, f"http://127.0.0.1:{port}/big")
    assert big == bytes(range(256)) * 1024
    assert _curl(port, "-N", f"http://127.0.0.1:{port}/stream") == b"".join(f"data: {i}\n\n".encode() for i in range(5))
    # several requests multiplexed on one connection
    urls = [f"http://127.0.0.1:{port}/r{i}" for i in range(6)]
    out = _curl(port, "--parallel", "--parallel-immediate", *urls)
    assert out.count(b'"version": "2"') == 6


def test_curl_h2_over_native_tls():
    """curl (OpenSSL + nghttp2) negotiates TLS 1.3 and ALPN h2 with the
    library's own TLS server session, then speaks HTTP/2 through it."""
    if not shutil.which("curl"):
        pytest.skip("curl not available")
    from aether_b200.serving.h2 import serve

    async def app(scope, receive, send):
        await receive()
        body = (b"tls h2 " + scope["path"].encode()) * (1 if scope["path"] != "/big" else 20000)
        await send({"type": "http.response.start", "status": 200, "headers": [(b"content-type", b"text/plain")]})
        await send({"type": "http.response.body", "body": body, "more_body": False})

    port = _free_port()
    loop = asyncio.new_event_loop()
    ready = threading.Event()

    def run():
        asyncio.set_event_loop(loop)
        ev = asyncio.Event()

        async def main():
            task = asyncio.ensure_future(serve(app, "127.0.0.1", port, ev, tls=True))
            await ev.wait()
            ready.set()
            await task

        try:
            loop.run_until_complete(main())
        except BaseException:  # cancelled at the end of the test
            pass

    threading.Thread(target=run, daemon=True).start()
    assert ready.wait(10)
    try:
        out = subprocess.run(["curl", "-s", "-k", "--http2", "--tlsv1.3", "-w", "\\n%{http_version}",
                              f"https://127.0.0.1:{port}/hello"], capture_output=True, timeout=30)
        assert out.returncode == 0, out.stderr
        body, version = out.stdout.rsplit(b"\n", 1)
        assert body == b"tls h2 /hello" and version == b"2"
        big = subprocess.run(["curl", "-s", "-k", "--http2", f"https://127.0.0.1:{port}/big"], capture_output=True,
                             timeout=30)
        assert big.stdout == b"tls h2 /big" * 20000
    finally:
        for t in asyncio.all_tasks(loop):
            loop.call_soon_threadsafe(t.cancel)
