"""OpenAI-compatible HTTP server.

Reference: aether-serve (trainer/src/bin/serve.rs): routes GET /v1/models,
POST /v1/chat/completions, POST /v1/completions, POST /v1/embeddings, SSE
streaming, Prometheus metrics; its own HTTP/1.1 + h2 + TLS 1.3 stack. Here the
HTTP layer is FastAPI/uvicorn (HTTP/1.1; TLS via uvicorn's ssl options) in
front of the continuous-batching ``Engine``.

    python -m aether_b200.serving.server --model 1.5b --max-concurrent 8 --port 8000
"""
from __future__ import annotations

import argparse
import asyncio
import json
import time
import uuid

from fastapi import FastAPI, HTTPException, Request as HTTPRequest
from fastapi.responses import JSONResponse, PlainTextResponse, StreamingResponse

from .sampling import SamplingParams
from .tokenizer import chat_template


class RateLimiter:
    """Token bucket per client address: ``rate`` requests per second with
    bursts of ``burst`` (reference: the rate limiter of
    runtime/src/lib.rs:6186-6210)."""

    def __init__(self, rate: float, burst: int, clock=time.monotonic):
        self.rate, self.burst, self.clock = rate, burst, clock
        self.buckets: dict = {}

    def allow(self, key: str) -> bool:
        now = self.clock()
        tokens, last = self.buckets.get(key, (float(self.burst), now))
        tokens = min(float(self.burst), tokens + (now - last) * self.rate)
        ok = tokens >= 1.0
        self.buckets[key] = (tokens - 1.0 if ok else tokens, now)
        return ok


def build_app(engine, model_name: str = "aether-qwen", embedder=None, template="chatml",
              vision=None, rate_limit: RateLimiter | None = None) -> FastAPI:
    """template: a built-in style name ("chatml", "llama3", ...) or a
    ``templates.JinjaChatTemplate`` (the model's own chat template, which also
    renders ``tools`` and tool-call turns)."""
    app = FastAPI(title="aether_b200")

    if rate_limit is not None:
        @app.middleware("http")
        async def _limit(req: HTTPRequest, call_next):
            if req.method == "POST" and not rate_limit.allow(req.client.host if req.client else "?"):
                engine.metrics.inc("rate_limited")
                return JSONResponse({"error": {"message": "rate limit exceeded", "type": "rate_limit"}},
                                    status_code=429)
            return await call_next(req)

    @app.get("/health")
    def health():
        return {"status": "ok", "active": len(engine.active), "queue": engine.pending.qsize()}

    @app.get("/v1/models")
    def models():
        data = [{"id": model_name, "object": "model", "owned_by": "aether_b200", "created": 0}]
        if embedder is not None:
            data.append({"id": embedder.name, "object": "model", "owned_by": "aether_b200", "created": 0})
        return {"object": "list", "data": data}

    @app.get("/metrics")
    def metrics():
        return PlainTextResponse(engine.metrics.prometheus())

    def _usage(r):
        return {"prompt_tokens": len(r.prompt_ids), "completion_tokens": len(r.tokens),
                "total_tokens": len(r.prompt_ids) + len(r.tokens)}

    async def _collect(r):
        loop = asyncio.get_running_loop()
        toks = []
        while True:
            t = await loop.run_in_executor(None, r.out.get)
            if t is None:
                return toks
            toks.append(t)

    def _trim(text: str, stops) -> str:
        for s in stops or []:
            i = text.find(s)
            if i >= 0:
                text = text[:i]
        return text

    async def _sse(r, make_chunk, stops):
        loop = asyncio.get_running_loop()
        sent = ""
        toks = []
        while True:
            t = await loop.run_in_executor(None, r.out.get)
            if t is None:
                break
            toks.append(t)
            text = _trim(engine.tok.decode(toks), stops)
            delta, sent = text[len(sent):], text
            if delta:
                yield f"data: {json.dumps(make_chunk(delta, None))}\n\n"
        yield f"data: {json.dumps(make_chunk('', r.finish_reason or 'stop'))}\n\n"
        yield "data: [DONE]\n\n"

    @app.post("/v1/completions")
    async def completions(req: HTTPRequest):
        body = await req.json()
        prompt = body.get("prompt", "")
        if isinstance(prompt, list):
            prompt = prompt[0] if prompt and isinstance(prompt[0], str) else prompt
        ids = engine.tok.encode(prompt) if isinstance(prompt, str) else list(prompt)
        params = SamplingParams.from_openai(body)
        try:
            r = engine.submit(ids, params)
        except ValueError as e:
            raise HTTPException(400, str(e)) from e
        cid = f"cmpl-{uuid.uuid4().hex[:24]}"
        created = int(time.time())
        if body.get("stream"):
            def chunk(delta, fin):
                return {"id": cid, "object": "text_completion", "created": created, "model": model_name,
                        "choices": [{"index": 0, "text": delta, "finish_reason": fin}]}
            return StreamingResponse(_sse(r, chunk, params.stop), media_type="text/event-stream")
        toks = await _collect(r)
        text = _trim(engine.tok.decode(toks), params.stop)
        return {"id": cid, "object": "text_completion", "created": created, "model": model_name,
                "choices": [{"index": 0, "text": text, "finish_reason": r.finish_reason or "stop"}],
                "usage": _usage(r)}

    @app.post("/v1/chat/completions")
    async def chat(req: HTTPRequest):
        body = await req.json()
        messages = body.get("messages") or []
        if not messages:
            raise HTTPException(400, "messages required")
        tools = body.get("tools")
        if isinstance(template, str):
            prompt = chat_template(messages, template)
        else:
            try:
                prompt = template.render(messages, tools=tools, add_generation_prompt=True)
            except Exception as e:  # a template's raise_exception or a sandbox violation
                raise HTTPException(400, f"chat template: {e}") from e
        ids = engine.tok.encode(prompt)
        params = SamplingParams.from_openai(body)
        try:
            r = engine.submit(ids, params)
        except ValueError as e:
            raise HTTPException(400, str(e)) from e
        cid = f"chatcmpl-{uuid.uuid4().hex[:24]}"
        created = int(time.time())
        if body.get("stream"):
            def chunk(delta, fin):
                d = {"content": delta} if delta else {}
                return {"id": cid, "object": "chat.completion.chunk", "created": created, "model": model_name,
                        "choices": [{"index": 0, "delta": d, "finish_reason": fin}]}
            return StreamingResponse(_sse(r, chunk, params.stop), media_type="text/event-stream")
        toks = await _collect(r)
        text = _trim(engine.tok.decode(toks), params.stop)
        msg = {"role": "assistant", "content": text}
        finish = r.finish_reason or "stop"
        if tools:
            from .templates import parse_tool_calls

            content, calls = parse_tool_calls(text)
            if calls:
                msg = {"role": "assistant", "content": content or None, "tool_calls": calls}
                finish = "tool_calls"
        return {"id": cid, "object": "chat.completion", "created": created, "model": model_name,
                "choices": [{"index": 0, "message": msg, "finish_reason": finish}],
                "usage": _usage(r)}

    @app.post("/v1/embeddings")
    async def embeddings(req: HTTPRequest):
        if embedder is None:
            return JSONResponse({"error": {"message": "no embedding model loaded"}}, status_code=501)
        body = await req.json()
        inputs = body.get("input", [])
        if isinstance(inputs, str):
            inputs = [inputs]
        vecs = embedder.embed_texts(inputs)
        return {"object": "list", "model": embedder.name,
                "data": [{"object": "embedding", "index": i, "embedding": v} for i, v in enumerate(vecs)],
                "usage": {"prompt_tokens": 0, "total_tokens": 0}}

    @app.post("/v1/vision/embed")
    async def vision_embed(req: HTTPRequest):
        """Body: {"image": [3][H][W] floats}, {"image_b64": raw little-endian
        float32 bytes, "shape": [3, H, W]}, or {"image_u8_b64": raw 8-bit RGB
        bytes, "shape": [H, W, 3]} (normalised with the ImageNet mean / std
        per channel) -> L2-normalised CLS embedding."""
        if vision is None:
            return JSONResponse({"error": {"message": "no vision model loaded"}}, status_code=501)
        import base64

        import numpy as np
        import torch

        body = await req.json()
        if "image_u8_b64" in body:
            from ..runtime import call, ptr

            hwc = np.frombuffer(base64.b64decode(body["image_u8_b64"]), dtype=np.uint8).reshape(body["shape"])
            if hwc.ndim != 3 or hwc.shape[2] != 3:
                raise HTTPException(400, "image_u8_b64 must be [H, W, 3] uint8")
            chw = np.empty((3, hwc.shape[0], hwc.shape[1]), np.float32)
            for c, (mu, sd) in enumerate(((0.485, 0.229), (0.456, 0.224), (0.406, 0.225))):
                plane = np.ascontiguousarray(hwc[:, :, c])
                call("aether_img_normalize_f32", ptr(plane), ptr(chw[c]), plane.size, mu, sd)
            img = torch.from_numpy(chw)
        elif "image_b64" in body:
            arr = np.frombuffer(base64.b64decode(body["image_b64"]), dtype="<f4").reshape(body["shape"])
            img = torch.from_numpy(arr.copy())
        else:
            img = torch.tensor(body["image"], dtype=torch.float32)
        if tuple(img.shape) != (3, vision.cfg.img, vision.cfg.img):
            raise HTTPException(400, f"image must be [3, {vision.cfg.img}, {vision.cfg.img}]")
        return {"object": "embedding", "model": vision.name, "embedding": vision.embed(img).tolist()}

    return app


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="1.5b",
                    choices=["1.5b", "7b", "qwen3-8b", "llama3-8b", "mistral-7b", "mistral-7b-v0.1", "qwen2-moe",
                             "mixtral", "deepseek-v2-lite", "tiny"])
    ap.add_argument("--tokenizer", default=None, help="tokenizer.json (default: byte tokenizer)")
    ap.add_argument("--max-concurrent", type=int, default=8)
    ap.add_argument("--max-seq", type=int, default=4096)
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--h2c", action="store_true", help="serve HTTP/2 over cleartext (prior knowledge) instead of HTTP/1.1")
    ap.add_argument("--h2-tls", action="store_true",
                    help="serve HTTP/2 over the native TLS 1.3 (self-signed Ed25519 certificate, ALPN h2)")
    ap.add_argument("--device", default="cuda")
    ap.add_argument("--embeddings", action="store_true", help="also serve a BGE-large-shape /v1/embeddings model")
    ap.add_argument("--vision", action="store_true", help="also serve a DINOv3 ViT-L/16-shape /v1/vision/embed")
    ap.add_argument("--rate-limit", type=float, default=0.0, help="POST requests per second per client (0 = off)")
    ap.add_argument("--gguf", default=None, help="load Qwen2 weights (and tokenizer) from a GGUF file")
    ap.add_argument("--keep-quant", action="store_true",
                    help="with --gguf: keep the projections in the file's quantised blocks on the device (the "
                    "file's size in memory) and expand each right before its GEMM")
    ap.add_argument("--hf", default=None, help="load Qwen2 weights from a Hugging Face directory")
    ap.add_argument("--tp", type=int, default=1,
                    help="tensor-parallel degree; launch with torchrun --nproc-per-node N (rank 0 serves HTTP)")
    args = ap.parse_args()
    import uvicorn

    from ..models.qwen import QwenConfig, QwenModel, QwenWeights
    from .engine import Engine
    from .tokenizer import BPETokenizer, ByteTokenizer

    from ..models.moe import MoEConfig, MoEQwenModel

    from ..models.deepseek import DeepSeekConfig, DeepSeekModel

    presets = {"7b": QwenConfig.qwen25_7b, "qwen3-8b": QwenConfig.qwen3_8b, "llama3-8b": QwenConfig.llama3_8b,
               "mistral-7b": QwenConfig.mistral_7b, "mistral-7b-v0.1": QwenConfig.mistral_7b_v01,
               "qwen2-moe": MoEConfig.qwen2_moe_a2_7b, "mixtral": MoEConfig.mixtral_8x7b,
               "deepseek-v2-lite": DeepSeekConfig.deepseek_v2_lite, "1.5b": QwenConfig.qwen25_1_5b}
    if args.model == "tiny":
        cfg = QwenConfig(vocab=1024, d_model=256, n_layers=2, n_heads=2, n_kv_heads=1, d_ff=512, max_seq=args.max_seq)
    else:
        cfg = presets[args.model]()
    tok = BPETokenizer.from_file(args.tokenizer) if args.tokenizer else ByteTokenizer()
    weights = None
    template = "chatml"
    if args.gguf:
        from ..formats import gguf
        from .templates import JinjaChatTemplate

        g = gguf.GGUFFile(args.gguf)
        load_dev = "cpu" if args.tp > 1 else args.device  # TP: each rank moves only its shard
        if g.meta.get("general.architecture") == "deepseek2":  # DeepSeek-V2 / GLM-4.7-flash (MLA + MoE)
            if args.tp > 1:
                raise SystemExit("--tp with a deepseek2 GGUF is not supported yet (random-init presets are)")
            cfg, weights = gguf.load_deepseek_weights(args.gguf, device=args.device)
        else:
            if args.keep_quant and args.tp > 1:
                raise SystemExit("--keep-quant serves one GPU (the TP shards are bf16)")
            cfg, weights = gguf.load_qwen_weights(args.gguf, device=load_dev, keep_quant=args.keep_quant)
        if not args.tokenizer:
            tok = gguf.tokenizer_from_gguf(g)
        template = JinjaChatTemplate.from_gguf(g) or template
    elif args.hf:
        import os

        from ..formats import hf

        from .templates import JinjaChatTemplate

        cfg, weights = hf.load_qwen_hf(args.hf, device="cpu" if args.tp > 1 else args.device)
        if not args.tokenizer and os.path.exists(os.path.join(args.hf, "tokenizer.json")):
            tok = BPETokenizer.from_file(os.path.join(args.hf, "tokenizer.json"))
        template = JinjaChatTemplate.from_hf_dir(args.hf) or template
    tp = None
    if args.tp > 1:  # one process per GPU; every rank builds its shard, rank 0 serves
        import torch.distributed as dist

        from ..parallel import dist as D
        from ..parallel.tp import TensorParallel
        from .tp_serve import BroadcastModel, follow

        info = D.init(timeout_s=600)
        if info.world != args.tp:
            raise SystemExit(f"--tp {args.tp} needs {args.tp} processes (got {info.world})")
        args.device = str(info.device)
        tp = TensorParallel(info)
        ctrl = dist.new_group(backend="gloo")
        if weights is not None and not isinstance(cfg, (DeepSeekConfig, MoEConfig)):
            weights = QwenWeights.shard(weights, info.rank, info.world, info.device)
    if isinstance(cfg, DeepSeekConfig):
        model = DeepSeekModel(cfg, device=args.device, max_batch=args.max_concurrent, max_seq=args.max_seq,
                              weights=weights, tp=tp)
    elif isinstance(cfg, MoEConfig):
        model = MoEQwenModel(cfg, device=args.device, max_batch=args.max_concurrent, max_seq=args.max_seq, tp=tp)
    else:
        model = QwenModel(cfg, device=args.device, max_batch=args.max_concurrent, max_seq=args.max_seq,
                          weights=weights, tp=tp)
    if tp is not None:
        if info.rank != 0:
            follow(model, ctrl)  # until rank 0 stops
            tp.close()
            D.shutdown()
            return
        model = BroadcastModel(model, ctrl)
    engine = Engine(model, tok, max_concurrent=args.max_concurrent, use_graph=args.device != "cpu")
    embedder = vision = None
    if args.embeddings:
        from ..models.encoders import BertConfig, BertEncoder, TextEmbedder

        embedder = TextEmbedder(BertEncoder(BertConfig.bge_large(), device=args.device), tok)
    if args.vision:
        from ..models.encoders import VitConfig, VitEncoder

        vision = VitEncoder(VitConfig.vitl16(), device=args.device)
    limiter = RateLimiter(args.rate_limit, max(1, int(args.rate_limit))) if args.rate_limit > 0 else None
    app = build_app(engine, f"qwen2.5-{args.model}", embedder=embedder, template=template, vision=vision,
                    rate_limit=limiter)
    try:
        if args.h2c or args.h2_tls:
            import asyncio

            from .h2 import serve as serve_h2

            asyncio.run(serve_h2(app, args.host, args.port, tls=args.h2_tls))
        else:
            uvicorn.run(app, host=args.host, port=args.port, log_level="warning")
    finally:
        engine.shutdown()
        if tp is not None:  # release the replaying ranks, then the process group
            model.stop()
            tp.close()
            D.shutdown()


if __name__ == "__main__":
    main()
