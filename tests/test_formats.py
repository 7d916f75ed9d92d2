"""Model file formats: safetensors, AetherLM .weights/.meta, GGUF (reader,
writer, block dequantisers against per-element restatements of the published
block layouts), HF-directory and GGUF loaders for Qwen2 weights."""
import os

import numpy as np
import pytest
import torch

from aether_b200.formats import aether_weights, gguf, hf
from aether_b200.formats import safetensors as st
from aether_b200.models.qwen import QwenConfig, QwenModel, QwenWeights

TINYQ = dict(vocab=256, d_model=128, n_layers=2, n_heads=2, n_kv_heads=1, d_ff=256, max_seq=64, init_std=0.05)


def test_safetensors_roundtrip(tmp_path):
    g = torch.Generator().manual_seed(0)
    t = {"a": torch.randn(3, 5, generator=g), "b": torch.randn(7, generator=g).to(torch.bfloat16),
         "c": torch.arange(10, dtype=torch.int64).view(2, 5), "d": torch.randn(4, generator=g).half(),
         "e": torch.tensor([True, False])}
    p = str(tmp_path / "x.safetensors")
    st.save_file(t, p, metadata={"k": "v"})
    back = st.load_file(p)
    assert set(back) == set(t)
    for k in t:
        assert back[k].dtype == t[k].dtype and torch.equal(back[k], t[k]), k
    assert st.metadata(p) == {"k": "v"}
    hdr, base = st.read_header(p)
    assert base % 8 == 0 and hdr["a"]["shape"] == [3, 5]
    assert not os.path.exists(p + ".tmp")


def test_aether_weights_byte_format(tmp_path):
    p = np.arange(85504, dtype=np.float32) * 0.5
    stem = str(tmp_path / "aether_lm")
    meta = dict(vocab=256, d_model=64, n_layers=2, n_heads=4, d_ff=128, seq_len=32)
    aether_weights.save(stem, p, meta)
    raw = open(stem + ".weights", "rb").read()
    assert raw[:9] == b"AETHER01\n" and int.from_bytes(raw[9:17], "little") == p.size and len(raw) == 17 + 4 * p.size
    assert open(stem + ".meta").read() == ('{"vocab":256,"d_model":64,"n_layers":2,"n_heads":4,"d_ff":128,'
                                           '"seq_len":32,"params":85504}\n')
    back, m = aether_weights.load(stem)
    assert np.array_equal(back, p) and m["params"] == 85504


# ---------------------------------------------------------------- GGUF dequantisers
def _f16(b):
    return float(np.frombuffer(bytes(b), dtype=np.float16)[0])


def _q4k_scalar(block):
    d, dmin = _f16(block[0:2]), _f16(block[2:4])
    sc, qs = block[4:16], block[16:144]

    def scale_min(j):
        if j < 4:
            return sc[j] & 63, sc[j + 4] & 63
        return (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4), (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4)

    y = []
    for grp in range(4):
        q = qs[grp * 32 : grp * 32 + 32]
        s1, m1 = scale_min(2 * grp)
        s2, m2 = scale_min(2 * grp + 1)
        y += [d * s1 * (v & 0xF) - dmin * m1 for v in q]
        y += [d * s2 * (v >> 4) - dmin * m2 for v in q]
    return y


def _q6k_scalar(block):
    ql, qh = block[0:128], block[128:192]
    sc = [int(x) for x in np.frombuffer(bytes(block[192:208]), dtype=np.int8)]
    d = _f16(block[208:210])
    y = [0.0] * 256
    for half in range(2):
        L, H, S = ql[half * 64 :], qh[half * 32 :], sc[half * 8 :]
        for l in range(32):
            i = l // 16
            q1 = ((L[l] & 0xF) | (((H[l] >> 0) & 3) << 4)) - 32
            q2 = ((L[l + 32] & 0xF) | (((H[l] >> 2) & 3) << 4)) - 32
            q3 = ((L[l] >> 4) | (((H[l] >> 4) & 3) << 4)) - 32
            q4 = ((L[l + 32] >> 4) | (((H[l] >> 6) & 3) << 4)) - 32
            b = half * 128
            y[b + l], y[b + l + 32] = d * S[i] * q1, d * S[i + 2] * q2
            y[b + l + 64], y[b + l + 96] = d * S[i + 4] * q3, d * S[i + 6] * q4
    return y


def _rand_blocks(nb, size, f16_at, seed):
    rng = np.random.default_rng(seed)
    b = rng.integers(0, 256, size=(nb, size), dtype=np.uint8)
    for off in f16_at:  # keep the f16 scales finite and modest
        b[:, off : off + 2] = np.frombuffer(rng.uniform(0.01, 0.1, nb).astype(np.float16).tobytes(),
                                            dtype=np.uint8).reshape(nb, 2)
    return b


@pytest.mark.parametrize("typ", ["q4k", "q6k"])
def test_kquant_dequant_matches_scalar(typ):
    if typ == "q4k":
        b = _rand_blocks(3, 144, [0, 2], 1)
        got = gguf.dequantize(b.reshape(-1), gguf.Q4_K, 3 * 256)
        ref = sum((_q4k_scalar([int(x) for x in r]) for r in b), [])
    else:
        b = _rand_blocks(3, 210, [208], 2)
        got = gguf.dequantize(b.reshape(-1), gguf.Q6_K, 3 * 256)
        ref = sum((_q6k_scalar([int(x) for x in r]) for r in b), [])
    np.testing.assert_allclose(got, np.array(ref, dtype=np.float32), rtol=1e-6, atol=1e-6)


def test_gguf_roundtrip_quant_types(tmp_path):
    g = torch.Generator().manual_seed(0)
    w = torch.randn(64, 96, generator=g)
    p = str(tmp_path / "t.gguf")
    meta = {"general.architecture": "test", "test.block_count": 3, "test.eps": 1e-5, "general.name": "x",
            "tokenizer.ggml.tokens": ["a", "b", "c"], "test.ids": [1, -2, 3]}
    gguf.write_gguf(p, meta, {"f32": (w, gguf.F32), "f16": (w, gguf.F16), "q8": (w, gguf.Q8_0), "q4": (w, gguf.Q4_0)})
    f = gguf.GGUFFile(p)
    assert f.meta["test.block_count"] == 3 and f.meta["general.name"] == "x"
    assert f.meta["tokenizer.ggml.tokens"] == ["a", "b", "c"] and f.meta["test.ids"] == [1, -2, 3]
    assert abs(f.meta["test.eps"] - 1e-5) < 1e-10
    assert torch.equal(f.tensor("f32", torch.float32), w)
    assert torch.equal(f.tensor("f16", torch.float32), w.half().float())
    e8 = float((f.tensor("q8", torch.float32) - w).abs().max())
    e4 = float((f.tensor("q4", torch.float32) - w).abs().max())
    amax = float(w.abs().max())
    assert e8 < amax / 127 and e4 < amax / 7, (e8, e4)


def _qwen_weights():
    cfg = QwenConfig(**TINYQ)
    return cfg, QwenWeights(cfg, "cpu", seed=4)


def _same_weights(a, b):
    for name in ("embed", "lm_head", "final_norm"):
        assert torch.equal(getattr(a, name), getattr(b, name)), name
    for name in ("attn_norm", "mlp_norm", "wqkv", "bqkv", "wo", "wgu", "wd"):
        for x, y in zip(getattr(a, name), getattr(b, name)):
            assert torch.equal(x, y), name


def test_hf_directory_roundtrip(tmp_path):
    cfg, w = _qwen_weights()
    hf.save_qwen_hf(cfg, w, str(tmp_path))
    cfg2, w2 = hf.load_qwen_hf(str(tmp_path), device="cpu")
    assert (cfg2.d_model, cfg2.n_layers, cfg2.n_kv_heads, cfg2.d_ff, cfg2.tie_embeddings) == (128, 2, 1, 256, True)
    _same_weights(w, w2)


def test_gguf_qwen_loader_logits(tmp_path):
    cfg, w = _qwen_weights()
    t = {"token_embd.weight": (w.embed, gguf.F32), "output_norm.weight": (w.final_norm, gguf.F32)}
    D = cfg.head_dim
    q, kv = cfg.n_heads * D, cfg.n_kv_heads * D
    for i in range(cfg.n_layers):
        p = f"blk.{i}."
        wq, wk, wv = w.wqkv[i].split([q, kv, kv])
        bq, bk, bv = w.bqkv[i].split([q, kv, kv])
        gt, up = w.wgu[i].split([cfg.d_ff, cfg.d_ff])
        t.update({p + "attn_norm.weight": (w.attn_norm[i], gguf.F32), p + "ffn_norm.weight": (w.mlp_norm[i], gguf.F32),
                  p + "attn_q.weight": (wq, gguf.F32), p + "attn_k.weight": (wk, gguf.F32),
                  p + "attn_v.weight": (wv, gguf.F32), p + "attn_q.bias": (bq, gguf.F32),
                  p + "attn_k.bias": (bk, gguf.F32), p + "attn_v.bias": (bv, gguf.F32),
                  p + "attn_output.weight": (w.wo[i], gguf.F32), p + "ffn_gate.weight": (gt, gguf.F32),
                  p + "ffn_up.weight": (up, gguf.F32), p + "ffn_down.weight": (w.wd[i], gguf.F32)})
    meta = {"general.architecture": "qwen2", "qwen2.embedding_length": 128, "qwen2.block_count": 2,
            "qwen2.attention.head_count": 2, "qwen2.attention.head_count_kv": 1, "qwen2.feed_forward_length": 256,
            "qwen2.rope.freq_base": 1e6, "qwen2.attention.layer_norm_rms_epsilon": 1e-6,
            "tokenizer.ggml.tokens": [f"t{i}" for i in range(256)]}
    path = str(tmp_path / "q.gguf")
    gguf.write_gguf(path, meta, t)
    cfg2, w2 = gguf.load_qwen_weights(path, device="cpu")
    assert cfg2.vocab == 256 and cfg2.tie_embeddings and cfg2.qkv_bias
    _same_weights(w, w2)
    toks = torch.randint(0, 256, (1, 9), generator=torch.Generator().manual_seed(3))
    a = QwenModel(cfg, device="cpu", weights=w, max_batch=1).reference_logits(toks)
    b = QwenModel(cfg2, device="cpu", weights=w2, max_batch=1).reference_logits(toks)
    assert torch.equal(a, b)


def test_tokenizer_from_gguf_metadata(tmp_path):
    toks = ["a", "b", "c", "ab", "abc", "<|im_end|>"]
    meta = {"general.architecture": "qwen2", "tokenizer.ggml.tokens": toks, "tokenizer.ggml.merges": ["a b", "ab c"],
            "tokenizer.ggml.token_type": [1, 1, 1, 1, 1, 3]}
    p = str(tmp_path / "tok.gguf")
    gguf.write_gguf(p, meta, {"x": (torch.zeros(8), gguf.F32)})
    tok = gguf.tokenizer_from_gguf(gguf.GGUFFile(p))
    assert tok.encode("abc<|im_end|>") == [4, 5]
    assert tok.decode([3, 2]) == "abc" and tok.eos_id == 5
