"""QLoRA over a GGUF-quantised Qwen2 base (models/qlora_gguf.py): the base's
projections stay in the file's blocks (mixed Q8_0 / Q4_0 / F16 parts here)
and expand per use; the adapted model matches a plain bf16 GPT loaded with
the same dequantised weights, the chunked LM-head loss matches the unchunked
one (loss and adapter gradients), the adapters train, and the device block
decoder matches the host dequantiser for every type it handles."""
import numpy as np
import pytest
import torch

from aether_b200.formats import gguf as G
from aether_b200.models.gpt import GPT
from aether_b200.models.lora import LoRAConfig
from aether_b200.models.qlora_gguf import PROJ, config_from_gguf, qlora_from_gguf
from aether_b200.optim import FlatAdamW

V, D, L, H, HKV, FF = 256, 128, 2, 2, 1, 256


def _write_base(path, seed=0, D=D, H=H, HKV=HKV, FF=FF):
    g = torch.Generator().manual_seed(seed)
    rnd = lambda *s: torch.randn(*s, generator=g) * 0.05  # noqa: E731
    hd = D // H
    t = {"token_embd.weight": (rnd(V, D), G.F16), "output_norm.weight": (1 + 0.1 * rnd(D), G.F32),
         "output.weight": (rnd(V, D), G.Q8_0)}
    for i in range(L):
        p = f"blk.{i}."
        t.update({
            p + "attn_norm.weight": (1 + 0.1 * rnd(D), G.F32), p + "ffn_norm.weight": (1 + 0.1 * rnd(D), G.F32),
            p + "attn_q.weight": (rnd(H * hd, D), G.Q8_0), p + "attn_k.weight": (rnd(HKV * hd, D), G.Q4_0),
            p + "attn_v.weight": (rnd(HKV * hd, D), G.F16), p + "attn_q.bias": (rnd(H * hd), G.F32),
            p + "attn_k.bias": (rnd(HKV * hd), G.F32), p + "attn_v.bias": (rnd(HKV * hd), G.F32),
            p + "attn_output.weight": (rnd(D, H * hd), G.Q8_0), p + "ffn_gate.weight": (rnd(FF, D), G.Q4_0),
            p + "ffn_up.weight": (rnd(FF, D), G.Q8_0), p + "ffn_down.weight": (rnd(D, FF), G.F16)})
    meta = {"general.architecture": "qwen2", "qwen2.embedding_length": D, "qwen2.block_count": L,
            "qwen2.attention.head_count": H, "qwen2.attention.head_count_kv": HKV, "qwen2.feed_forward_length": FF,
            "qwen2.rope.freq_base": 1e6, "qwen2.attention.layer_norm_rms_epsilon": 1e-6,
            "tokenizer.ggml.tokens": [f"t{i}" for i in range(V)]}
    G.write_gguf(path, meta, t)
    return path


def _dense_gpt(path, device="cpu"):
    """A plain bf16 GPT holding the same (dequantised) weights."""
    gf = G.GGUFFile(path)
    cfg = config_from_gguf(gf, max_seq=64)
    m = GPT(cfg, device=device)
    a = m.arena
    t = lambda n: gf.tensor(n, dtype=torch.float32)  # noqa: E731
    with torch.no_grad():
        a.set_full("tok_emb", t("token_embd.weight"))
        a.set_full("final_norm", t("output_norm.weight"))
        a.set_full("lm_head", t("output.weight"))
        for i in range(L):
            p = f"blk.{i}."
            a.set_full(f"l{i}.attn_norm", t(p + "attn_norm.weight"))
            a.set_full(f"l{i}.mlp_norm", t(p + "ffn_norm.weight"))
            a.set_full(f"l{i}.bqkv", torch.cat([t(p + "attn_q.bias"), t(p + "attn_k.bias"), t(p + "attn_v.bias")]))
            a.set_full(f"l{i}.wqkv", torch.cat([t(p + "attn_q.weight"), t(p + "attn_k.weight"), t(p + "attn_v.weight")]))
            a.set_full(f"l{i}.wo", t(p + "attn_output.weight"))
            a.set_full(f"l{i}.wgu", torch.cat([t(p + "ffn_gate.weight"), t(p + "ffn_up.weight")]))
            a.set_full(f"l{i}.wd", t(p + "ffn_down.weight"))
        a.sync_bf16_from_master()
    return m


def _batch(seed=1, B=2, S=16):
    g = torch.Generator().manual_seed(seed)
    tok = torch.randint(0, V, (B, S + 1), generator=g)
    return tok[:, :-1].contiguous(), tok[:, 1:].contiguous()


def test_qlora_gguf_base_matches_dense_and_keeps_blocks(tmp_path):
    path = _write_base(str(tmp_path / "base.gguf"))
    m = qlora_from_gguf(path, device="cpu", lora=LoRAConfig(rank=8), max_seq=64, loss_chunk=0)
    assert m.cfg.qkv_bias and not m.cfg.tie_embeddings
    # the projections are not in the base arena; they stay in the file's blocks
    assert not any(n.split(".")[-1] in PROJ for n in m.base.arena.names())
    parts = [p for w in m.qweights.values() for p in w.parts]
    assert {p.typ for p in parts} == {G.Q8_0, G.Q4_0, G.F16} and all(p.blocks is not None for p in parts)
    dense_bytes = sum(2 * w.shape[0] * w.shape[1] for w in m.qweights.values())
    assert m.base_bytes < 0.8 * dense_bytes
    ids, tgt = _batch()
    ref = _dense_gpt(path)
    with torch.no_grad():
        a, b = float(m.loss(ids, tgt)), float(ref.loss(ids, tgt))
    assert abs(a - b) < 1e-4 * abs(b), (a, b)


def test_chunked_head_loss_matches_and_adapters_train(tmp_path):
    path = _write_base(str(tmp_path / "base.gguf"))
    ids, tgt = _batch(S=24)
    runs = []
    for chunk in (0, 7):
        m = qlora_from_gguf(path, device="cpu", lora=LoRAConfig(rank=8), max_seq=64, loss_chunk=chunk)
        with torch.no_grad():  # a non-zero update, so the adapter gradients are non-trivial
            for n in m.arena.names():
                if n.endswith(".B"):
                    m.arena.master_view(n).normal_(0, 0.01, generator=torch.Generator().manual_seed(5))
            m.arena.sync_bf16_from_master()
        m.arena.zero_grad()
        loss = m.loss(ids, tgt)
        loss.backward()
        runs.append((float(loss.detach()), m.arena.grad.clone()))
    (l0, g0), (l1, g1) = runs
    assert abs(l0 - l1) < 1e-5 * abs(l0), (l0, l1)
    assert float((g0 - g1).abs().max()) <= 1e-3 * float(g0.abs().max()) + 1e-8
    # a few optimiser steps on one batch lower its loss
    m = qlora_from_gguf(path, device="cpu", lora=LoRAConfig(rank=8), max_seq=64, loss_chunk=7)
    opt = FlatAdamW(m.arena, lr=1e-2, weight_decay=0.0)
    first = None
    for _ in range(6):
        m.arena.zero_grad()
        loss = m.loss(ids, tgt)
        loss.backward()
        opt.step()
        first = float(loss) if first is None else first
    assert float(m.loss(ids, tgt)) < first - 0.05


def test_pipeline_stage_of_gguf_base(tmp_path):
    """A layer range of the base (a pipeline stage) loads only its layers."""
    path = _write_base(str(tmp_path / "base.gguf"))
    s0 = qlora_from_gguf(path, device="cpu", lora=LoRAConfig(rank=8), layers=[0], first=True, last=False)
    s1 = qlora_from_gguf(path, device="cpu", lora=LoRAConfig(rank=8), layers=[1], first=False, last=True)
    assert {k[0] for k in s0.qweights} == {0} and {k[0] for k in s1.qweights} == {1}
    assert "lm_head" not in s0.base.arena.names() and "tok_emb" not in s1.base.arena.names()
    ids, tgt = _batch()
    whole = qlora_from_gguf(path, device="cpu", lora=LoRAConfig(rank=8), loss_chunk=0)
    with torch.no_grad():
        h = s0.base.forward_hidden(ids)
        a = float(s1.loss(None, tgt, x=h))
        b = float(whole.loss(ids, tgt))
    assert abs(a - b) < 1e-5 * abs(b)


def _random_blocks(typ, rows, K, seed=0):
    """Random bytes as GGUF blocks of `typ`, with sane fp16 scale fields."""
    ne, nb = G.BLOCKS[typ]
    rng = np.random.default_rng(seed)
    b = rng.integers(0, 256, size=(rows * K // ne, nb), dtype=np.uint8)
    h = lambda v: np.frombuffer(np.float16(v).tobytes(), np.uint8)  # noqa: E731
    if typ in (G.Q8_0, G.Q4_0, G.Q5_0):
        b[:, 0:2] = h(0.01)
    elif typ in (G.Q4_K, G.Q5_K):
        b[:, 0:2], b[:, 2:4] = h(0.01), h(0.004)
    elif typ == G.Q6_K:
        b[:, 208:210] = h(0.01)
    elif typ == G.F16:
        b = np.frombuffer(rng.standard_normal(rows * K).astype(np.float16).tobytes(), np.uint8).reshape(-1, 2)
    elif typ == G.F32:
        b = np.frombuffer(rng.standard_normal(rows * K).astype(np.float32).tobytes(), np.uint8).reshape(-1, 4)
    return np.ascontiguousarray(b.reshape(-1))


@pytest.mark.gpu
@pytest.mark.parametrize("typ", ["F32", "F16", "Q4_0", "Q5_0", "Q8_0", "Q4_K", "Q5_K", "Q6_K"])
def test_gpu_gguf_block_decoder_matches_host(typ):
    from aether_b200.ops import functional as F

    t = getattr(G, typ)
    rows, K = 7, 512
    blocks = _random_blocks(t, rows, K)
    want = torch.from_numpy(G.dequantize(blocks, t, rows * K).reshape(rows, K)).to(torch.bfloat16)
    out = torch.zeros(rows, K + 64, dtype=torch.bfloat16, device="cuda")
    F.gguf_dequant(torch.from_numpy(blocks).cuda(), t, rows, K, out)
    got = out[:, :K].cpu()
    assert float((got.float() - want.float()).abs().max()) <= 1e-2 * float(want.float().abs().max()) + 1e-6
    assert float(out[:, K:].abs().max()) == 0.0  # nothing past K of each row


@pytest.mark.gpu
def test_gpu_qlora_gguf_matches_cpu(tmp_path):
    path = _write_base(str(tmp_path / "base.gguf"))
    ids, tgt = _batch()
    cpu = qlora_from_gguf(path, device="cpu", lora=LoRAConfig(rank=8), max_seq=64, loss_chunk=0)
    gpu = qlora_from_gguf(path, device="cuda", lora=LoRAConfig(rank=8), max_seq=64, loss_chunk=8)
    a = float(cpu.loss(ids, tgt))
    gpu.arena.zero_grad()
    lg = gpu.loss(ids.cuda(), tgt.cuda())
    lg.backward()
    assert abs(float(lg) - a) < 2e-2 * abs(a), (float(lg), a)
    assert float(gpu.arena.grad.abs().sum()) > 0  # the adapters receive gradients


def test_qlora_smoke_command_line(tmp_path):
    """qlora-smoke over a layer range: loss falls, adapters grow; bad ranges exit 2."""
    from aether_b200 import qlora_smoke

    path = _write_base(str(tmp_path / "base.gguf"))
    assert qlora_smoke.main(["--gguf", path, "--lo", "0", "--hi", "2", "--steps", "8", "--device", "cpu"]) == 0
    assert qlora_smoke.main(["--gguf", path, "--lo", "1", "--hi", "2", "--steps", "8", "--device", "cpu"]) == 0
    assert qlora_smoke.main(["--gguf", path, "--lo", "1", "--hi", "5", "--device", "cpu"]) == 2


def _serve_pair(path, device):
    from aether_b200.models.qwen import QwenModel

    cfg_d, w_d = G.load_qwen_weights(path, device=device)
    cfg_q, w_q = G.load_qwen_weights(path, device=device, keep_quant=True)
    assert not isinstance(w_q.wqkv[0], torch.Tensor) and w_q.wqkv[0].parts[0].blocks is not None
    md = QwenModel(cfg_d, device=device, weights=w_d, max_batch=2, max_seq=64)
    mq = QwenModel(cfg_q, device=device, weights=w_q, max_batch=2, max_seq=64)
    return md, mq


def test_serving_keeps_gguf_weights_quantised(tmp_path):
    """Serving a GGUF model with its projections kept in the file's blocks
    (expanded per GEMM) gives the same logits and tokens as serving the
    dequantised bf16 weights."""
    path = _write_base(str(tmp_path / "base.gguf"), seed=5)
    md, mq = _serve_pair(path, "cpu")
    toks = torch.randint(0, V, (2, 11), generator=torch.Generator().manual_seed(6))
    _, ld = md.prefill(toks, return_logits=True)
    _, lq = mq.prefill(toks, return_logits=True)
    assert torch.equal(ld, lq)
    assert torch.equal(md.generate(toks, 4, use_graph=False), mq.generate(toks, 4, use_graph=False))


@pytest.mark.gpu
def test_gpu_serving_keeps_gguf_weights_quantised(tmp_path):
    """The same on the device, with CUDA-graph decode (the per-projection
    expansions are captured with the GEMMs); head_dim 128, as the decode
    attention kernel needs."""
    path = _write_base(str(tmp_path / "base.gguf"), seed=7, D=256, H=2, HKV=1, FF=512)
    md, mq = _serve_pair(path, "cuda")
    toks = torch.randint(0, V, (2, 11), generator=torch.Generator().manual_seed(8)).cuda()
    _, ld = md.prefill(toks, return_logits=True)
    _, lq = mq.prefill(toks, return_logits=True)
    assert float((ld.float() - lq.float()).abs().max()) < 1e-2 * float(ld.float().abs().max())
    gd, gq = md.generate(toks, 6, use_graph=True), mq.generate(toks, 6, use_graph=True)
    assert float((gd == gq).float().mean()) >= 0.9
