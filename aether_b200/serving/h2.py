"""HTTP/2 over cleartext with prior knowledge (h2c) in front of an ASGI app:
the framing, HPACK and flow control run in the native session of
libaether_rt (``aether_h2_server_*``); this module owns the sockets and turns
each complete request into one ASGI call, so the OpenAI-compatible FastAPI
app of ``serving.server`` is served unchanged. Response bodies are sent chunk
by chunk as the app produces them (server-sent events stream), and requests
on different streams of one connection run concurrently.

    python -m aether_b200.serving.server --model 7b --h2c --port 8000
    curl --http2-prior-knowledge http://127.0.0.1:8000/v1/models

With ``tls=True`` the same sessions run inside the library's own TLS 1.3
server sessions (ChaCha20-Poly1305, X25519, a self-signed Ed25519
certificate generated at start-up, ALPN "h2"):

    python -m aether_b200.serving.server --model 7b --h2-tls --port 8443
    curl -k --http2 https://127.0.0.1:8443/v1/models

Reference: the h2 path of aether-serve (trainer/src/bin/serve.rs:1059-1207,
runtime/src/http2.rs).
"""
from __future__ import annotations

import asyncio
import ctypes as C

from .. import runtime as rt

_MAX_HEAD, _MAX_BODY = 1 << 16, 1 << 24


def _lib():
    lb = rt.lib()
    L, P, I = C.c_int64, C.c_void_p, C.c_int
    lb.aether_h2_server_new.restype = L
    lb.aether_h2_server_new.argtypes = []
    lb.aether_h2_server_free.argtypes = [L]
    lb.aether_h2_server_feed.argtypes = [L, P, I]
    lb.aether_h2_server_next_request.argtypes = [L, C.POINTER(I), P, I, C.POINTER(I), P, I, C.POINTER(I)]
    lb.aether_h2_server_respond.argtypes = [L, I, I, C.c_char_p, I, I]
    lb.aether_h2_server_data.argtypes = [L, I, P, I, I]
    lb.aether_h2_server_take_outbound.argtypes = [L, P, I]
    return lb


class H2Connection:
    """One client connection: bytes in, ASGI calls, bytes out."""

    def __init__(self, app, reader, writer, server_addr=("127.0.0.1", 0)):
        self.app, self.reader, self.writer = app, reader, writer
        self.lib = _lib()
        self.h = self.lib.aether_h2_server_new()
        self.server_addr = server_addr
        self.out = C.create_string_buffer(1 << 20)
        self.tasks: set = set()

    def _flush(self) -> None:
        while True:
            n = self.lib.aether_h2_server_take_outbound(self.h, self.out, len(self.out))
            if n <= 0:
                return
            self.writer.write(self.out.raw[:n])

    async def run(self) -> None:
        head = C.create_string_buffer(_MAX_HEAD)
        body = C.create_string_buffer(_MAX_BODY)
        sid, hl, bl = C.c_int(), C.c_int(), C.c_int()
        try:
            self._flush()  # our SETTINGS
            await self.writer.drain()
            while True:
                data = await self.reader.read(65536)
                if not data:
                    break
                n = self.lib.aether_h2_server_feed(self.h, data, len(data))
                self._flush()
                if n < 0:
                    break
                while self.lib.aether_h2_server_next_request(self.h, C.byref(sid), head, _MAX_HEAD, C.byref(hl), body,
                                                             _MAX_BODY, C.byref(bl)) == 1:
                    t = asyncio.ensure_future(self._serve(sid.value, head.raw[: hl.value], body.raw[: bl.value]))
                    self.tasks.add(t)
                    t.add_done_callback(self.tasks.discard)
                await self.writer.drain()
        finally:
            for t in list(self.tasks):
                t.cancel()
            self.lib.aether_h2_server_free(self.h)
            self.writer.close()

    async def _serve(self, stream: int, head: bytes, body: bytes) -> None:
        lines = head.decode("latin-1").split("\n")
        method, _, target = lines[0].partition(" ")
        path, _, query = target.partition("?")
        headers = []
        for line in lines[1:]:
            if line:
                k, _, v = line.partition(": ")
                headers.append((k.encode("latin-1"), v.encode("latin-1")))
        peer = self.writer.get_extra_info("peername") or ("", 0)
        scope = {"type": "http", "asgi": {"version": "3.0"}, "http_version": "2", "method": method,
                 "scheme": "http", "path": path, "raw_path": path.encode(), "query_string": query.encode(),
                 "root_path": "", "headers": headers, "client": peer[:2], "server": self.server_addr}
        sent_body = False

        async def receive():
            nonlocal sent_body
            if not sent_body:
                sent_body = True
                return {"type": "http.request", "body": body, "more_body": False}
            await asyncio.Event().wait()  # the client cannot disconnect mid-request here

        async def send(msg):
            if msg["type"] == "http.response.start":
                hs = "".join(f"{k.decode('latin-1')}: {v.decode('latin-1')}\n" for k, v in msg.get("headers", []))
                enc = hs.encode("latin-1")
                self.lib.aether_h2_server_respond(self.h, stream, int(msg["status"]), enc, len(enc), 0)
            elif msg["type"] == "http.response.body":
                chunk = msg.get("body", b"")
                more = msg.get("more_body", False)
                self.lib.aether_h2_server_data(self.h, stream, chunk or b"\0", len(chunk), 0 if more else 1)
            self._flush()
            await self.writer.drain()

        await self.app(scope, receive, send)


class _TlsStream:
    """Reader / writer pair over a native TLS 1.3 server session: reads return
    decrypted application data, writes are encrypted into records."""

    def __init__(self, reader, writer, cn: bytes):
        import os

        lb = rt.lib()
        L, P, I = C.c_int64, C.c_void_p, C.c_int
        lb.aether_tls13_server_new.restype = L
        lb.aether_tls13_server_new.argtypes = [P, P, P, P, I, P, I]
        lb.aether_tls13_server_feed.argtypes = [L, P, I, P, I]
        lb.aether_tls13_server_take_outbound.argtypes = [L, P, I]
        lb.aether_tls13_server_send.argtypes = [L, P, I]
        lb.aether_tls13_server_free.argtypes = [L]
        lb.aether_tls13_server_is_done.argtypes = [L]
        self.lib, self.reader, self.writer = lb, reader, writer
        self.early = bytearray()  # plaintext written before the handshake completed
        self.h = lb.aether_tls13_server_new(os.urandom(32), os.urandom(32), os.urandom(32), cn, len(cn),
                                            os.urandom(8), 8)
        self.buf = C.create_string_buffer(1 << 17)
        self.app = C.create_string_buffer(1 << 17)

    def _flush(self):
        while True:
            n = self.lib.aether_tls13_server_take_outbound(self.h, self.buf, len(self.buf))
            if n <= 0:
                return
            self.writer.write(self.buf.raw[:n])

    async def read(self, n: int) -> bytes:
        while True:
            data = await self.reader.read(65536)
            if not data:
                return b""
            got = self.lib.aether_tls13_server_feed(self.h, data, len(data), self.app, len(self.app))
            if self.early and self.lib.aether_tls13_server_is_done(self.h) == 1:
                early, self.early = bytes(self.early), bytearray()
                self.lib.aether_tls13_server_send(self.h, early, len(early))
            self._flush()
            await self.writer.drain()
            if got < 0:
                return b""
            if got:
                return self.app.raw[:got]

    def write(self, data: bytes) -> None:
        if self.lib.aether_tls13_server_is_done(self.h) != 1:
            self.early += data
            return
        if self.lib.aether_tls13_server_send(self.h, data, len(data)) >= 0:
            self._flush()

    async def drain(self) -> None:
        await self.writer.drain()

    def close(self) -> None:
        self.lib.aether_tls13_server_free(self.h)
        self.writer.close()

    def get_extra_info(self, key):
        return self.writer.get_extra_info(key)


async def serve(app, host: str = "127.0.0.1", port: int = 8000, ready: asyncio.Event | None = None,
                tls: bool = False):
    """Serve `app` over h2c (or HTTP/2 over the native TLS 1.3 with tls=True) until cancelled."""

    async def on_conn(reader, writer):
        if tls:
            stream = _TlsStream(reader, writer, host.encode())
            await H2Connection(app, stream, stream, (host, port)).run()
        else:
            await H2Connection(app, reader, writer, (host, port)).run()

    server = await asyncio.start_server(on_conn, host, port)
    if ready is not None:
        ready.set()
    async with server:
        await server.serve_forever()
