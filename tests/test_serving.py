"""Serving stack on CPU with a tiny random Qwen: tokenizers, the continuous
batching engine (results equal per-request greedy generation), sampling
parameters, and the OpenAI-compatible HTTP routes on a live server."""
import json
import socket
import threading
import time
import urllib.request

import pytest
import torch

from aether_b200.models.qwen import QwenConfig, QwenModel
from aether_b200.serving.engine import Engine
from aether_b200.serving.sampling import SamplingParams
from aether_b200.serving.tokenizer import BPETokenizer, ByteTokenizer, bytes_to_unicode, chat_template

TINY = dict(vocab=300, d_model=128, n_layers=2, n_heads=2, n_kv_heads=1, d_ff=256, max_seq=128, init_std=0.08)


def _model(seed=0, max_batch=4):
    return QwenModel(QwenConfig(**TINY), device="cpu", seed=seed, max_batch=max_batch, max_seq=128)


def test_byte_tokenizer_roundtrip():
    t = ByteTokenizer()
    s = "héllo <|im_start|>user\nhi<|im_end|>"
    ids = t.encode(s)
    assert t.special["<|im_start|>"] in ids
    assert t.decode(ids) == s


def test_bpe_tokenizer_merges():
    be = bytes_to_unicode()
    sp = be[ord(" ")]
    vocab = {c: i for i, c in enumerate(sorted(set(be.values())))}
    n = len(vocab)
    vocab.update({"h" + "e": n, "he" + "l": n + 1, "hel" + "l": n + 2, "hell" + "o": n + 3, sp + "w": n + 4})
    merges = ["h e", "he l", "hel l", "hell o", sp + " w"]
    tok = BPETokenizer(vocab, merges, {"<|endoftext|>": n + 10})
    ids = tok.encode("hello world<|endoftext|>")
    assert ids[0] == n + 3 and ids[1] == n + 4 and ids[-1] == n + 10
    assert tok.decode(ids) == "hello world<|endoftext|>"


def test_chat_template():
    p = chat_template([{"role": "user", "content": "hi"}])
    assert p == "<|im_start|>user\nhi<|im_end|>\n<|im_start|>assistant\n"


def test_engine_matches_individual_generation():
    m = _model(seed=3, max_batch=4)
    ref = _model(seed=3, max_batch=4)
    eng = Engine(m, ByteTokenizer(), max_concurrent=3, eos_ids=[], use_graph=False)
    prompts = [list(range(5, 5 + n)) for n in (7, 11, 4, 9)]
    reqs = [eng.submit(p, SamplingParams(max_tokens=6)) for p in prompts]
    outs = []
    for r in reqs:
        toks = list(eng.stream(r, timeout=120))
        outs.append(toks)
    eng.shutdown()
    for p, got in zip(prompts, outs):
        want = ref.generate(torch.tensor([p]), 6, use_graph=False)[0].tolist()
        assert got == want, (p, got, want)
    assert eng.metrics.counters["requests_finished"] == 4


def test_sampling_params():
    m = _model(seed=4)
    eng = Engine(m, ByteTokenizer(), max_concurrent=2, eos_ids=[], use_graph=False)
    prompt = list(range(20, 30))
    a = eng.generate(prompt, SamplingParams(temperature=0.8, top_k=20, seed=123, max_tokens=5))[1]
    b = eng.generate(prompt, SamplingParams(temperature=0.8, top_k=20, seed=123, max_tokens=5))[1]
    assert a == b
    g = eng.generate(prompt, SamplingParams(max_tokens=5))[1]
    k1 = eng.generate(prompt, SamplingParams(temperature=1.0, top_k=1, seed=1, max_tokens=5))[1]
    assert g == k1
    forced = eng.generate(prompt, SamplingParams(temperature=0.7, logit_bias={42: 100.0}, seed=1, max_tokens=3))[1]
    assert forced == [42, 42, 42]
    eng.shutdown()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _post(url, body):
    req = urllib.request.Request(url, data=json.dumps(body).encode(), headers={"Content-Type": "application/json"})
    with urllib.request.urlopen(req, timeout=60) as r:
        return r.read().decode()


def test_http_server_routes():
    import uvicorn

    from aether_b200.serving.server import build_app

    from aether_b200.models.encoders import BertConfig, BertEncoder, TextEmbedder, VitConfig, VitEncoder

    m = _model(seed=5)
    eng = Engine(m, ByteTokenizer(), max_concurrent=2, use_graph=False)
    emb = TextEmbedder(BertEncoder(BertConfig(vocab=500, d_model=64, n_layers=1, n_heads=2, d_ff=128, max_pos=64),
                                   device="cpu"), ByteTokenizer())
    vis = VitEncoder(VitConfig(d=64, n_layers=1, n_heads=2, d_ff=128, patch=8, img=16), device="cpu")
    port = _free_port()
    app = build_app(eng, "tiny", embedder=emb, vision=vis)
    server = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="error"))
    th = threading.Thread(target=server.run, daemon=True)
    th.start()
    base = f"http://127.0.0.1:{port}"
    for _ in range(200):
        try:
            urllib.request.urlopen(base + "/health", timeout=1)
            break
        except Exception:  # noqa: BLE001
            time.sleep(0.05)
    try:
        models = json.loads(urllib.request.urlopen(base + "/v1/models", timeout=10).read())
        assert models["data"][0]["id"] == "tiny"
        out = json.loads(_post(base + "/v1/completions", {"prompt": "abc", "max_tokens": 4}))
        assert out["object"] == "text_completion" and out["usage"]["completion_tokens"] >= 1
        chat = json.loads(_post(base + "/v1/chat/completions",
                                {"messages": [{"role": "user", "content": "hi"}], "max_tokens": 3}))
        assert chat["choices"][0]["message"]["role"] == "assistant"
        sse = _post(base + "/v1/chat/completions",
                    {"messages": [{"role": "user", "content": "hi"}], "max_tokens": 3, "stream": True})
        assert sse.strip().endswith("data: [DONE]")
        metrics = urllib.request.urlopen(base + "/metrics", timeout=10).read().decode()
        assert "aether_requests_total" in metrics
        e = json.loads(_post(base + "/v1/embeddings", {"input": ["hello", "world"]}))
        assert len(e["data"]) == 2 and len(e["data"][0]["embedding"]) == 64
        v = json.loads(_post(base + "/v1/vision/embed", {"image": torch.randn(3, 16, 16).tolist()}))
        assert len(v["embedding"]) == 64
        import base64

        import numpy as np

        raw = np.random.default_rng(0).integers(0, 256, (16, 16, 3), dtype=np.uint8)
        v8 = json.loads(_post(base + "/v1/vision/embed", {"image_u8_b64": base64.b64encode(raw.tobytes()).decode(),
                                                          "shape": [16, 16, 3]}))
        assert len(v8["embedding"]) == 64 and abs(sum(x * x for x in v8["embedding"]) - 1.0) < 1e-3
    finally:
        server.should_exit = True
        th.join(timeout=10)
        eng.shutdown()


@pytest.mark.gpu
def test_gpu_engine_batched_graph_decode():
    cfg = QwenConfig(**dict(TINY, d_model=256, n_heads=2, n_kv_heads=1, d_ff=512))
    m = QwenModel(cfg, device="cuda", seed=6, max_batch=4, max_seq=128)
    ref = QwenModel(cfg, device="cuda", seed=6, max_batch=4, max_seq=128)
    eng = Engine(m, ByteTokenizer(), max_concurrent=4, eos_ids=[], use_graph=True)
    prompts = [list(range(3, 3 + n)) for n in (5, 13, 8)]
    reqs = [eng.submit(p, SamplingParams(max_tokens=8)) for p in prompts]
    outs = [list(eng.stream(r, timeout=120)) for r in reqs]
    eng.shutdown()
    assert not eng.errors, eng.errors
    assert all(r.finish_reason == "length" for r in reqs), [r.finish_reason for r in reqs]
    agree = 0
    for p, got in zip(prompts, outs):
        want = ref.generate(torch.tensor([p], device="cuda"), 8, use_graph=False)[0].tolist()
        agree += sum(int(a == b) for a, b in zip(got, want))
    assert agree >= 0.9 * 24, (outs,)


def test_rate_limiter_token_bucket():
    from aether_b200.serving.server import RateLimiter

    now = [0.0]
    rl = RateLimiter(rate=2.0, burst=3, clock=lambda: now[0])
    assert [rl.allow("x") for _ in range(4)] == [True, True, True, False]
    assert rl.allow("y")  # buckets are per client
    now[0] += 0.5  # one token back at 2/s
    assert rl.allow("x") and not rl.allow("x")


QWEN_STYLE = (
    "{%- if tools %}<|im_start|>system\n# Tools\n<tools>\n{%- for tool in tools %}\n{{ tool | tojson }}\n{%- endfor %}\n"
    "</tools><|im_end|>\n{%- endif %}\n"
    "{%- for message in messages %}\n"
    "{%- if message.role == 'assistant' and message.tool_calls %}<|im_start|>assistant\n"
    "{%- for tc in message.tool_calls %}<tool_call>\n{\"name\": \"{{ tc.function.name }}\", \"arguments\": "
    "{{ tc.function.arguments }}}\n</tool_call>{%- endfor %}<|im_end|>\n"
    "{%- elif message.role == 'tool' %}<|im_start|>user\n<tool_response>\n{{ message.content }}\n</tool_response>"
    "<|im_end|>\n"
    "{%- else %}<|im_start|>{{ message.role }}\n{{ message.content }}<|im_end|>\n{%- endif %}\n"
    "{%- endfor %}\n{%- if add_generation_prompt %}<|im_start|>assistant\n{%- endif %}")


def test_jinja_chat_template_tools_and_tool_call_parsing():
    from aether_b200.serving.templates import JinjaChatTemplate, TemplateError, parse_tool_calls

    t = JinjaChatTemplate(QWEN_STYLE)
    tools = [{"type": "function", "function": {"name": "get_weather", "parameters": {"type": "object"}}}]
    msgs = [{"role": "user", "content": "weather in Paris?"},
            {"role": "assistant", "content": None,
             "tool_calls": [{"type": "function", "function": {"name": "get_weather",
                                                               "arguments": "{\"city\": \"Paris\"}"}}]},
            {"role": "tool", "content": "18C"}]
    out = t.render(msgs, tools=tools)
    assert '"name": "get_weather"' in out and "<tool_response>\n18C" in out
    assert out.endswith("<|im_start|>assistant")  # "{%-" also strips the newline before it
    gen = 'Let me check.<tool_call>\n{"name": "get_weather", "arguments": {"city": "Oslo"}}\n</tool_call>'
    content, calls = parse_tool_calls(gen)
    assert content == "Let me check." and len(calls) == 1
    assert calls[0]["function"]["name"] == "get_weather"
    assert json.loads(calls[0]["function"]["arguments"]) == {"city": "Oslo"}
    assert parse_tool_calls("no calls here") == ("no calls here", [])
    bad = JinjaChatTemplate("{{ raise_exception('only user/assistant roles') }}")
    with pytest.raises(TemplateError):
        bad.render(msgs)
    # the sandbox refuses attribute access into Python internals
    with pytest.raises(Exception):
        JinjaChatTemplate("{{ messages.__class__.__mro__ }}").render(msgs)


def test_http2_server_routes():
    """The same OpenAI app over h2c (prior knowledge), driven by curl."""
    import asyncio
    import shutil
    import subprocess

    from aether_b200.serving.h2 import serve
    from aether_b200.serving.server import build_app

    if not shutil.which("curl"):
        pytest.skip("curl not available")
    eng = Engine(_model(seed=6), ByteTokenizer(), max_concurrent=2, use_graph=False)
    app = build_app(eng, "tiny-h2")
    port = _free_port()
    loop = asyncio.new_event_loop()
    started = threading.Event()

    def run():
        asyncio.set_event_loop(loop)
        ev = asyncio.Event()

        async def main():
            task = asyncio.ensure_future(serve(app, "127.0.0.1", port, ev))
            await ev.wait()
            started.set()
            await task

        try:
            loop.run_until_complete(main())
        except BaseException:  # cancelled at the end of the test
            pass

    th = threading.Thread(target=run, daemon=True)
    th.start()
    assert started.wait(10)
    base = f"http://127.0.0.1:{port}"

    def curl(*args, data=None):
        out = subprocess.run(["curl", "-s", "--http2-prior-knowledge", "--max-time", "60", *args], input=data,
                             capture_output=True, timeout=90)
        assert out.returncode == 0, out.stderr
        return out.stdout

    try:
        assert json.loads(curl(base + "/v1/models"))["data"][0]["id"] == "tiny-h2"
        body = json.dumps({"prompt": "abc", "max_tokens": 4}).encode()
        out = json.loads(curl("-H", "content-type: application/json", "--data-binary", "@-", base + "/v1/completions",
                              data=body))
        assert out["object"] == "text_completion" and out["usage"]["completion_tokens"] >= 1
        body = json.dumps({"messages": [{"role": "user", "content": "hi"}], "max_tokens": 3, "stream": True}).encode()
        sse = curl("-N", "-H", "content-type: application/json", "--data-binary", "@-", base + "/v1/chat/completions",
                   data=body).decode()
        assert sse.count("data: ") >= 2 and sse.rstrip().endswith("data: [DONE]")
    finally:
        eng.shutdown()
        for t in asyncio.all_tasks(loop):
            loop.call_soon_threadsafe(t.cancel)
