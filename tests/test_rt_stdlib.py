"""Host pieces of the C ABI in libaether_rt: the extra losses against plain
PyTorch autograd, the bf16 host matmul, scalar helpers, witness exits and
print formats, the BPE table and tokenizer.json loader, safetensors header
queries and the GGUF reader against files written by this package."""
import ctypes as C
import json

import numpy as np
import pytest
import torch

from aether_b200 import runtime as rt
from aether_b200.formats import gguf as G
from aether_b200.formats import safetensors as ST


def _p(a):
    return rt.ptr(a)


def _f(*shape, seed=0):
    return np.random.default_rng(seed).standard_normal(shape).astype(np.float32)


def test_losses_match_autograd():
    n = 64
    pred = (1 / (1 + np.exp(-_f(n, seed=1)))).astype(np.float32)
    tgt = (np.random.default_rng(2).random(n) > 0.5).astype(np.float32)
    g = np.zeros(n, np.float32)
    tp = torch.from_numpy(pred.astype(np.float64)).requires_grad_()
    ref = torch.nn.functional.binary_cross_entropy(tp, torch.from_numpy(tgt.astype(np.float64)))
    ref.backward()
    assert abs(rt.call("aether_op_bce_f32", _p(pred), _p(tgt), n) - float(ref)) < 1e-5
    rt.call("aether_op_bce_backward_f32", _p(pred), _p(tgt), _p(g), n)
    np.testing.assert_allclose(g, tp.grad.numpy(), rtol=1e-4, atol=1e-7)

    p = np.random.default_rng(3).dirichlet(np.ones(n)).astype(np.float32)
    t = np.random.default_rng(4).dirichlet(np.ones(n)).astype(np.float32)
    tp = torch.from_numpy(p.astype(np.float64)).requires_grad_()
    ref = (torch.from_numpy(t.astype(np.float64)) * (torch.log(torch.from_numpy(t.astype(np.float64))) - torch.log(tp))).mean()
    ref.backward()
    assert abs(rt.call("aether_op_kl_div_f32", _p(p), _p(t), n) - float(ref)) < 1e-6
    rt.call("aether_op_kl_div_backward_f32", _p(p), _p(t), _p(g), n)
    np.testing.assert_allclose(g, tp.grad.numpy(), rtol=1e-4)

    a, b = _f(16, seed=5), _f(16, seed=6)
    for y, margin in ((1.0, 1.0), (0.0, 10.0)):
        ta = torch.from_numpy(a.astype(np.float64)).requires_grad_()
        dist = (ta - torch.from_numpy(b.astype(np.float64))).norm()
        ref = y * dist ** 2 + (1 - y) * torch.clamp(margin - dist, min=0) ** 2
        ref.backward()
        got = rt.call("aether_op_contrastive_f32", _p(a), _p(b), C.c_float(y), 16, C.c_float(margin))
        assert abs(got - float(ref)) < 1e-3 * max(1.0, abs(float(ref)))
        g16 = np.zeros(16, np.float32)
        rt.call("aether_op_contrastive_backward_f32", _p(a), _p(b), _p(g16), C.c_float(y), 16, C.c_float(margin))
        np.testing.assert_allclose(g16, ta.grad.numpy(), rtol=1e-3, atol=1e-5)

    x, t2 = _f(n, seed=7), _f(n, seed=8)
    tx = torch.from_numpy(x.astype(np.float64)).requires_grad_()
    ref = torch.nn.functional.smooth_l1_loss(tx, torch.from_numpy(t2.astype(np.float64)), beta=0.5)
    ref.backward()
    assert abs(rt.call("aether_op_smooth_l1_f32", _p(x), _p(t2), n, C.c_float(0.5)) - float(ref)) < 1e-5
    rt.call("aether_op_smooth_l1_backward_f32", _p(x), _p(t2), _p(g), n, C.c_float(0.5))
    np.testing.assert_allclose(g, tx.grad.numpy(), rtol=1e-5, atol=1e-8)

    an, po, ne = _f(8, seed=9), _f(8, seed=10), _f(8, seed=11)
    ta = torch.from_numpy(an.astype(np.float64)).requires_grad_()
    ref = torch.clamp(((ta - torch.from_numpy(po.astype(np.float64))) ** 2).sum()
                      - ((ta - torch.from_numpy(ne.astype(np.float64))) ** 2).sum() + 5.0, min=0)
    ref.backward()
    assert abs(rt.call("aether_op_triplet_f32", _p(an), _p(po), _p(ne), 8, C.c_float(5.0)) - float(ref)) < 1e-4
    g8 = np.zeros(8, np.float32)
    rt.call("aether_op_triplet_backward_f32", _p(an), _p(po), _p(ne), _p(g8), 8, C.c_float(5.0))
    np.testing.assert_allclose(g8, ta.grad.numpy(), rtol=1e-5, atol=1e-6)


def test_bf16_matmul_scalars_and_witnesses(capfd):
    m, k, n = 5, 33, 7
    a = torch.randn(m, k, generator=torch.Generator().manual_seed(0)).bfloat16()
    b = torch.randn(k, n, generator=torch.Generator().manual_seed(1)).bfloat16()
    out = np.zeros((m, n), np.uint16)
    an, bn = a.view(torch.int16).numpy().copy(), b.view(torch.int16).numpy().copy()
    assert rt.call("aether_op_matmul_bf16", _p(an), _p(bn), _p(out), m, k, n) == 0
    got = torch.from_numpy(out.view(np.int16)).view(torch.bfloat16).float()
    want = (a.float() @ b.float()).bfloat16().float()
    assert float((got - want).abs().max()) <= float(want.abs().max()) * 2 ** -7

    x = np.arange(10, dtype=np.float32)
    assert rt.call("aether_sum_f32", _p(x), 10) == 45.0
    assert rt.call("aether_dot_f32_scalar", _p(x), _p(x), 10) == 285.0
    assert rt.call("aether_max_f32", C.c_float(2.0), C.c_float(3.0)) == 3.0
    assert rt.call("aether_min_i64", -5, 4) == -5 and rt.call("aether_abs_i64", -7) == 7
    assert abs(rt.call("aether_sqrt_f32", C.c_float(2.0)) - 2 ** 0.5) < 1e-6
    assert rt.call("aether_f32_close_exit", C.c_float(1.0), C.c_float(1.0005)) == 42
    assert rt.call("aether_f32_close_exit", C.c_float(1.0), C.c_float(1.1)) == 1
    assert rt.call("aether_f32_in_band_exit", C.c_float(0.5), C.c_float(0.1), C.c_float(1.0)) == 42
    assert rt.call("aether_f32_in_band_exit", C.c_float(float("nan")), C.c_float(0.1), C.c_float(1.0)) == 1
    buf = np.zeros(4, np.float32)
    rt.call("aether_fill_f32", _p(buf), 4, C.c_float(1.5))
    assert (buf == 1.5).all()
    rt.call("aether_print_loss", 7, C.c_float(1.25))
    rt.call("aether_print_kv_i64", b"tokens", 12)
    rt.call("aether_print_newline")
    out = capfd.readouterr().out
    assert "step=7 loss=1.250000\n" in out and "tokens: 12\n" in out

    # the reference's 4-argument normal fill: N(0, scale^2), deterministic in the seed
    h = np.zeros(4096, np.float32)
    rt.call("aether_init_normal_f32", _p(h), 4096, C.c_float(0.5), 7)
    assert abs(float(h.std()) - 0.5) < 0.03 and abs(float(h.mean())) < 0.03
    h2 = np.zeros(4096, np.float32)
    rt.call("aether_init_normal_f32", _p(h2), 4096, C.c_float(0.5), 7)
    np.testing.assert_array_equal(h, h2)


def _ids(out, n):
    return list(out[:n])


def test_bpe_table_and_tokenizer_json():
    h = rt.call("aether_bpe_tokenizer_new")
    assert h >= 0
    ab = rt.call("aether_bpe_add_merge", h, ord("a"), ord("b"), 0, b"ab", 2)
    abc = rt.call("aether_bpe_add_merge", h, ab, ord("c"), 1, b"abc", 3)
    assert (ab, abc) == (256, 257)
    assert rt.call("aether_bpe_add_merge", h, ord("a"), ord("b"), 5, b"ab", 2) == -1  # duplicate pair
    out = np.zeros(16, np.int32)
    text = b"abcabx"
    n = rt.call("aether_bpe_encode", h, text, len(text), _p(out), 16)
    assert _ids(out, n) == [abc, ab, ord("x")]
    dec = C.create_string_buffer(32)
    m = rt.call("aether_bpe_decode", h, _p(out), n, dec, 32)
    assert dec.raw[:m] == text
    assert rt.call("aether_bpe_encode", h, text, len(text), _p(out), 2) == -1  # overflow
    assert rt.call("aether_bpe_lookup_bytes", h, b"abc", 3) == abc
    assert rt.call("aether_bpe_tokenizer_free", h) == 0

    # a tokenizer.json with surface-string vocab, both merge spellings and an added token
    tj = {"model": {"type": "BPE",
                    "vocab": {"h": 0, "e": 1, "l": 2, "o": 3, "Ġ": 4, "he": 5, "ll": 6, "hell": 7, "hello": 8},
                    "merges": ["h e", ["l", "l"], "he ll", "hell o"]},
          "added_tokens": [{"id": 9, "content": "<|end|>"}]}
    blob = json.dumps(tj).encode()
    h = rt.call("aether_bpe_tokenizer_new")
    assert rt.call("aether_tokenizer_json_load", h, blob, len(blob)) == 4
    init = np.array([0, 1, 2, 2, 3, 4, 0], np.int32)  # h e l l o Ġ h
    n = rt.call("aether_bpe_encode_ids", h, _p(init), len(init), _p(out), 16)
    assert _ids(out, n) == [8, 4, 0]
    assert rt.call("aether_bpe_lookup_bytes", h, "Ġ".encode(), 2) == 4
    assert rt.call("aether_bpe_lookup_bytes", h, b"<|end|>", 7) == 9
    bad = json.dumps({"model": {"vocab": {"a": 0}, "merges": ["a b"]}}).encode()
    h2 = rt.call("aether_bpe_tokenizer_new")
    assert rt.call("aether_tokenizer_json_load", h2, bad, len(bad)) == -2
    assert rt.call("aether_tokenizer_json_load", h2, b"{oops", 5) == -1


def test_safetensors_header_queries(tmp_path):
    path = str(tmp_path / "m.safetensors")
    ST.save_file({"w": torch.zeros(3, 4, dtype=torch.bfloat16), "b": torch.zeros(5, dtype=torch.float32),
                  "i": torch.zeros(2, 2, 2, dtype=torch.int64)}, path)
    raw = np.fromfile(path, np.uint8)
    L = raw.size
    assert rt.call("aether_safetensors_n_tensors", _p(raw), L) == 3
    assert rt.call("aether_safetensors_get_dtype", _p(raw), L, b"w", 1) == 2
    assert rt.call("aether_safetensors_get_dtype", _p(raw), L, b"b", 1) == 0
    assert rt.call("aether_safetensors_get_dtype", _p(raw), L, b"i", 1) == 6
    assert rt.call("aether_safetensors_get_dtype", _p(raw), L, b"zz", 2) == -1
    dims = np.zeros(4, np.int64)
    assert rt.call("aether_safetensors_get_shape", _p(raw), L, b"i", 1, _p(dims), 4) == 3
    assert list(dims[:3]) == [2, 2, 2]
    assert rt.call("aether_safetensors_n_tensors", _p(raw), 4) == -1  # truncated


def test_gguf_reader(tmp_path):
    path = str(tmp_path / "t.gguf")
    w = torch.randn(4, 64, generator=torch.Generator().manual_seed(0))
    e = torch.randn(3, 32, generator=torch.Generator().manual_seed(1))
    G.write_gguf(path, {"general.architecture": "qwen2", "qwen2.block_count": 2, "qwen2.rope.freq_base": 1e6,
                        "tokenizer.ggml.tokens": ["a", "bb", "ccc"], "flag": True},
                 {"blk.0.w": (w, G.Q8_0), "emb": (e, G.F32)})
    pb = path.encode()
    h = rt.call("aether_gguf_open", pb, len(pb))
    assert h >= 0
    assert rt.call("aether_gguf_version", h) == 3
    assert rt.call("aether_gguf_n_tensors", h) == 2
    k = b"qwen2.block_count"
    assert rt.call("aether_gguf_get_metadata_u32", h, k, len(k)) == 2
    k = b"qwen2.rope.freq_base"
    assert rt.call("aether_gguf_get_metadata_f32", h, k, len(k)) == pytest.approx(1e6)
    k = b"flag"
    assert rt.call("aether_gguf_get_metadata_bool", h, k, len(k)) == 1
    k = b"general.architecture"
    s = C.create_string_buffer(64)
    assert rt.call("aether_gguf_get_metadata_string", h, k, len(k), s, 64) == 5 and s.raw[:5] == b"qwen2"
    assert rt.call("aether_gguf_get_metadata_string", h, k, len(k), s, 2) == -2
    k = b"tokenizer.ggml.tokens"
    assert rt.call("aether_gguf_get_metadata_array_string_n", h, k, len(k)) == 3
    assert rt.call("aether_gguf_get_metadata_array_string_get", h, k, len(k), 2, s, 64) == 3 and s.raw[:3] == b"ccc"
    assert rt.call("aether_gguf_get_metadata_u32", h, b"missing", 7) == -1
    i = rt.call("aether_gguf_find_tensor_by_name", h, b"emb", 3)
    assert i == 1
    assert rt.call("aether_gguf_get_tensor_dtype", h, i) == G.F32
    dims = np.zeros(4, np.int64)
    assert rt.call("aether_gguf_get_tensor_shape", h, i, _p(dims), 4) == 2 and list(dims[:2]) == [32, 3]
    assert rt.call("aether_gguf_get_tensor_n_elems", h, i) == 96
    ptr = rt.call("aether_gguf_get_tensor_data_ptr", h, i)
    got = np.ctypeslib.as_array((C.c_float * 96).from_address(ptr))
    np.testing.assert_array_equal(got, e.numpy().reshape(-1))
    # the Q8_0 tensor's blocks, read through the absolute offset, dequantise to the same values
    j = rt.call("aether_gguf_find_tensor_by_name", h, b"blk.0.w", 7)
    off = rt.call("aether_gguf_get_tensor_abs_offset", h, j)
    raw = np.fromfile(path, np.uint8)[off : off + 8 * 34]
    np.testing.assert_allclose(G.dequantize(raw, G.Q8_0, 256).reshape(4, 64), w.numpy(), atol=0.02)
    n = C.create_string_buffer(16)
    assert rt.call("aether_gguf_get_tensor_name", h, j, n, 16) == 7 and n.raw[:7] == b"blk.0.w"
    assert rt.call("aether_gguf_close", h) == 0
    assert rt.call("aether_gguf_n_tensors", h) == -1
    bad = str(tmp_path / "bad.gguf")
    open(bad, "wb").write(b"NOPE" + b"\0" * 40)
    assert rt.call("aether_gguf_open", bad.encode(), len(bad)) == -2


def test_unprefixed_file_format_exports(tmp_path):
    """gguf_* header queries on an in-memory image and the one-tensor
    safetensors save / load / lookup exports (the runtime module declares
    them without the aether_ prefix)."""
    lib = rt.lib()
    for n in ("gguf_parse_magic", "gguf_version", "gguf_tensor_count", "gguf_metadata_count",
              "safetensors_parse_header", "safetensors_get_tensor_f32"):
        getattr(lib, n).restype = C.c_int64
    for n in ("safetensors_save_f32", "safetensors_load_f32"):
        getattr(lib, n).restype = C.c_int
    head = np.frombuffer(b"GGUF" + (3).to_bytes(4, "little") + (7).to_bytes(8, "little") + (11).to_bytes(8, "little"),
                         np.uint8).copy()
    p, n = C.c_int64(head.ctypes.data), C.c_int64(head.size)
    assert lib.gguf_parse_magic(p, n) == 1 and lib.gguf_version(p, n) == 3
    assert lib.gguf_tensor_count(p, n) == 7 and lib.gguf_metadata_count(p, n) == 11
    assert lib.gguf_tensor_count(p, C.c_int64(12)) == -1  # too short for the field
    vals = np.arange(6, dtype=np.float32) * 1.5
    path = str(tmp_path / "w.safetensors").encode()
    assert lib.safetensors_save_f32(C.c_int64(C.cast(C.c_char_p(path), C.c_void_p).value),
                                    C.c_int64(vals.ctypes.data), C.c_int64(6)) == 0
    got = np.zeros(6, np.float32)
    assert lib.safetensors_load_f32(C.c_int64(C.cast(C.c_char_p(path), C.c_void_p).value),
                                    C.c_int64(got.ctypes.data), C.c_int64(6)) == 0
    assert np.array_equal(got, vals)
    blob = np.frombuffer(open(path.decode(), "rb").read(), np.uint8).copy()
    b, bn = C.c_int64(blob.ctypes.data), C.c_int64(blob.size)
    hdr = lib.safetensors_parse_header(b, bn)
    assert hdr > 0 and json.loads(bytes(blob[8:8 + hdr]))["data"]["shape"] == [6]
    name = b"data"
    addr = lib.safetensors_get_tensor_f32(b, bn, C.c_int64(C.cast(C.c_char_p(name), C.c_void_p).value), C.c_int64(4))
    assert addr == blob.ctypes.data + 8 + hdr
    assert np.array_equal(np.frombuffer((C.c_float * 6).from_address(addr), np.float32), vals)
    miss = b"nope"
    assert lib.safetensors_get_tensor_f32(b, bn, C.c_int64(C.cast(C.c_char_p(miss), C.c_void_p).value), C.c_int64(4)) == 0
