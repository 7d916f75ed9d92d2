"""Device-ABI decode-step, MLA, encoder and q8_1 ops on a B200, each against a
numpy / PyTorch fp32 reference or the existing entry point it generalises
(contiguous vs paged caches, one sequence vs a batch, one split vs many)."""
import ctypes as C
import math

import numpy as np
import pytest
import torch

from aether_b200.formats import gguf as G
from aether_b200.runtime import device as D

pytestmark = pytest.mark.gpu
f = C.c_float


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    return D.Dev()


def _r(*shape, seed=0):
    return np.random.default_rng(seed).standard_normal(shape).astype(np.float32)


def _close(got, want, tol=1e-4):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    err = np.abs(got - want).max() / max(np.abs(want).max(), 1e-6)
    assert err < tol, err


def _rope_half(x, pos, base, rd=None, off=0, factor=None):
    """Half-split RoPE of dims [off, off + rd) of the last axis at positions pos (per row)."""
    x = x.astype(np.float64).copy()
    rd = rd or x.shape[-1]
    half = rd // 2
    j = np.arange(half)
    fac = np.ones(half) if factor is None else factor
    ang = np.asarray(pos, np.float64).reshape(-1, *([1] * (x.ndim - 1)))[..., :1] * fac * base ** (-2.0 * j / rd)
    c, s = np.cos(ang), np.sin(ang)
    a, b = x[..., off : off + half].copy(), x[..., off + half : off + rd].copy()
    x[..., off : off + half] = a * c - b * s
    x[..., off + half : off + rd] = a * s + b * c
    return x


def _attn(q, K, V, scale):
    """q [H, dk], K [T, Hkv, dk], V [T, Hkv, dv] -> [H, dv]."""
    H, Hkv = q.shape[0], K.shape[1]
    Kr, Vr = np.repeat(K, H // Hkv, 1), np.repeat(V, H // Hkv, 1)
    s = np.einsum("hd,thd->ht", q.astype(np.float64), Kr) * scale
    p = np.exp(s - s.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    return np.einsum("ht,thd->hd", p, Vr)


def test_rope_variants():
    d = _dev()
    x = _r(3, 4, 16, seed=1)
    hx, st = d.upload(x), d.upload(np.array([7, 0], np.int32))
    d.call("aether_op_rope_apply_devarg_f32_cuda", hx, 3, 4, 16, f(10000.0), st)
    _close(d.download(hx, x.shape), _rope_half(x, [7, 8, 9], 10000.0))
    pos = np.array([3, 100, 0], np.int32)
    hx = d.upload(x)
    d.call("aether_op_batched_rope_apply_devarg_f32_cuda", hx, 3, 4, 16, f(10000.0), d.upload(pos))
    _close(d.download(hx, x.shape), _rope_half(x, pos, 10000.0))
    hq, hkv, hd = 4, 2, 16
    q, k, v = _r(hq, hd, seed=2), _r(hkv, hd, seed=3), _r(hkv, hd, seed=4)
    bq, bk, bv = _r(hq, hd, seed=5), _r(hkv, hd, seed=6), _r(hkv, hd, seed=7)
    hs = [d.upload(t) for t in (q, k, v, bq, bk, bv)]
    d.call("aether_op_qkv_bias_rope_devarg_f32_cuda", *hs, hq, hkv, hd, f(1e6), st)
    _close(d.download(hs[0], q.shape), _rope_half((q + bq)[None], [7], 1e6)[0])
    _close(d.download(hs[1], k.shape), _rope_half((k + bk)[None], [7], 1e6)[0])
    _close(d.download(hs[2], v.shape), v + bv)


def test_contiguous_paged_batched_and_split_attention():
    d = _dev()
    hq, hkv, hd, bs, T = 8, 2, 64, 16, 50
    dkv = hkv * hd
    ks, vs = _r(T, hkv, hd, seed=10), _r(T, hkv, hd, seed=11)
    q = _r(hq, hd, seed=12)
    scale = 1 / math.sqrt(hd)
    want = _attn(q, ks, vs, scale)
    # contiguous cache filled through the step-argument append
    kc, vc = d.alloc_f32(64 * dkv), d.alloc_f32(64 * dkv)
    step = np.zeros(2, np.int32)
    hst = d.upload(step)
    for t in range(T):
        step[:] = (t, t + 1)
        d.call("aether_dev_h2d_i32", step.ctypes.data, hst, 2)
        d.call("aether_op_append_kv_devarg_f32_cuda", d.upload(ks[t].ravel()), d.upload(vs[t].ravel()), kc, vc, dkv,
               hst)
    hqd, out = d.upload(q), d.alloc_f32(hq * hd)
    d.call("aether_op_attention_seq1_devarg_f32_cuda", hqd, kc, vc, out, hq, hkv, hd, f(scale), 64, hst)
    _close(d.download(out, (hq, hd)), want)
    # paged pool with a shuffled page table
    n_pages = 8
    table = np.random.default_rng(0).permutation(n_pages).astype(np.int32)
    kp, vp, hpt = d.alloc_f32(n_pages * bs * dkv), d.alloc_f32(n_pages * bs * dkv), d.upload(table)
    for t in range(T):
        step[:] = (t, t + 1)
        d.call("aether_dev_h2d_i32", step.ctypes.data, hst, 2)
        d.call("aether_op_paged_append_kv_devarg_f32_cuda", d.upload(ks[t].ravel()), d.upload(vs[t].ravel()), kp, vp,
               hpt, dkv, bs, hst)
    for v in ("", "_v2", "_v3"):
        d.call(f"aether_op_paged_attention_seq1{v}_devarg_f32_cuda", hqd, kp, vp, hpt, out, hq, hkv, hd, bs, f(scale),
               128, hst)
        _close(d.download(out, (hq, hd)), want)
    d.call("aether_op_paged_attention_flex_devarg_f32_cuda", hqd, kp, vp, hpt, out, hq, hkv, hd, bs, 20, f(scale), 128,
           hst)
    _close(d.download(out, (hq, hd)), _attn(q, ks[T - 20 :], vs[T - 20 :], scale))
    n_split = 4
    sm, sl, sv = d.alloc_f32(hq * n_split), d.alloc_f32(hq * n_split), d.alloc_f32(hq * n_split * hd)
    d.call("aether_op_paged_attention_seq1_v4_devarg_f32_cuda", hqd, kp, vp, hpt, out, sm, sl, sv, hq, hkv, hd, bs,
           f(scale), 128, n_split, hst)
    _close(d.download(out, (hq, hd)), want)
    # a table entry pointing past the pool is masked, not read
    bad = table.copy()
    bad[0] = 10**6
    d.call("aether_op_paged_attention_seq1_devarg_f32_cuda", hqd, kp, vp, d.upload(bad), out, hq, hkv, hd, bs,
           f(scale), 128, hst)
    _close(d.download(out, (hq, hd)), _attn(q, ks[bs:], vs[bs:], scale))

    # two sequences in one pool: seqB (shared step) and hetero (own lengths)
    B, stride = 2, 4
    tables = np.array([[0, 1, 2, 3], [4, 5, 6, 7]], np.int32)
    kpb, vpb, hptb = d.alloc_f32(n_pages * bs * dkv), d.alloc_f32(n_pages * bs * dkv), d.upload(tables)
    kb, vb = _r(T, B, dkv, seed=13), _r(T, B, dkv, seed=14)
    for t in range(T):
        step[:] = (t, t + 1)
        d.call("aether_dev_h2d_i32", step.ctypes.data, hst, 2)
        d.call("aether_op_batched_paged_append_kv_seqB_devarg_f32_cuda", d.upload(kb[t]), d.upload(vb[t]), kpb, vpb,
               hptb, B, dkv, bs, stride, hst)
    qb = _r(B, hq, hd, seed=15)
    outb = d.alloc_f32(B * hq * hd)
    d.call("aether_op_batched_paged_attention_seqB_devarg_f32_cuda", d.upload(qb), kpb, vpb, hptb, outb, B, hq, hkv, hd,
           bs, stride, f(scale), 128, hst)
    got = d.download(outb, (B, hq, hd))
    for b in range(B):
        _close(got[b], _attn(qb[b], kb[:, b].reshape(T, hkv, hd), vb[:, b].reshape(T, hkv, hd), scale))
    lens = np.array([T, 17], np.int32)
    d.call("aether_op_batched_paged_attention_hetero_devarg_f32_cuda", d.upload(qb), kpb, vpb, hptb, outb, B, hq, hkv,
           hd, bs, stride, f(scale), 128, d.upload(lens))
    got = d.download(outb, (B, hq, hd))
    for b in range(B):
        n = lens[b]
        _close(got[b], _attn(qb[b], kb[:n, b].reshape(n, hkv, hd), vb[:n, b].reshape(n, hkv, hd), scale))
    # hetero append: each sequence writes at its own position
    pos = np.array([5, 40], np.int32)
    newk, newv = _r(B, dkv, seed=16), _r(B, dkv, seed=17)
    d.call("aether_op_batched_paged_append_kv_hetero_devarg_f32_cuda", d.upload(newk), d.upload(newv), kpb, vpb, hptb, B,
           dkv, bs, stride, d.upload(pos))
    pool = d.download(kpb, (n_pages * bs, dkv))
    for b in range(B):
        row = tables[b, pos[b] // bs] * bs + pos[b] % bs
        _close(pool[row], newk[b], 1e-7)


def test_mla_ops():
    d = _dev()
    H, nope, rope, vhd, lora = 4, 32, 16, 24, 64
    qk = nope + rope
    kv_a = _r(lora + rope, seed=20)
    hc, hr = d.alloc_f32(lora), d.alloc_f32(rope)
    d.call("aether_op_mla_split_kv_a_f32_cuda", d.upload(kv_a), hc, hr, lora, rope)
    _close(d.download(hc, lora), kv_a[:lora], 1e-7)
    _close(d.download(hr, rope), kv_a[lora:], 1e-7)
    kvb = _r(H, nope + vhd, seed=21)
    krow, vrow = d.alloc_f32(H * qk), d.alloc_f32(H * vhd)
    d.call("aether_op_mla_assemble_k_f32_cuda", d.upload(kvb), hr, krow, H, nope, rope, vhd)
    _close(d.download(krow, (H, qk)), np.concatenate([kvb[:, :nope], np.tile(kv_a[lora:], (H, 1))], 1), 1e-7)
    d.call("aether_op_mla_extract_v_f32_cuda", d.upload(kvb), vrow, H, nope, vhd)
    _close(d.download(vrow, (H, vhd)), kvb[:, nope:], 1e-7)
    bk, bv = d.alloc_f32(H * (lora + rope)), d.alloc_f32(H * lora)
    d.call("aether_op_mla_broadcast_kv_for_mqa_f32_cuda", hc, hr, bk, bv, H, lora, rope)
    _close(d.download(bk, (H, lora + rope)), np.tile(kv_a, (H, 1)), 1e-7)
    _close(d.download(bv, (H, lora)), np.tile(kv_a[:lora], (H, 1)), 1e-7)

    st = d.upload(np.array([37, 38], np.int32))
    q = _r(H, qk, seed=22)
    hq = d.upload(q)
    d.call("aether_op_mla_rope_q_partial_f32_cuda", hq, H, qk, nope, f(10000.0), st)
    _close(d.download(hq, (H, qk)), _rope_half(q[None], [37], 10000.0, rope, nope)[0])
    kr = _r(rope, seed=23)
    hk = d.upload(kr)
    d.call("aether_op_mla_rope_k_shared_f32_cuda", hk, rope, f(10000.0), st)
    _close(d.download(hk, rope), _rope_half(kr[None, None], [37], 10000.0)[0, 0])
    # YaRN: per-pair factor ramp / s + (1 - ramp) between the beta_fast / beta_slow corrections
    s_, ctx, bf, bsl, base = 40.0, 4096.0, 32.0, 1.0, 10000.0
    corr = lambda rot: rope * math.log(ctx / (rot * 2 * math.pi)) / (2 * math.log(base))  # noqa: E731
    lo, hi = max(math.floor(corr(bf)), 0), min(math.ceil(corr(bsl)), rope - 1)
    ramp = np.clip((np.arange(rope // 2) - lo) / (hi - lo), 0, 1)
    fac = ramp / s_ + (1 - ramp)
    hq = d.upload(q)
    d.call("aether_op_mla_rope_q_partial_yarn_f32_cuda", hq, H, qk, nope, f(base), f(s_), f(ctx), f(bf), f(bsl), st)
    _close(d.download(hq, (H, qk)), _rope_half(q[None], [37], base, rope, nope, fac)[0])
    hk = d.upload(kr)
    d.call("aether_op_mla_rope_k_shared_yarn_f32_cuda", hk, rope, f(base), f(s_), f(ctx), f(bf), f(bsl), st)
    _close(d.download(hk, rope), _rope_half(kr[None, None], [37], base, factor=fac)[0, 0])

    # non-absorbed MLA paged attention: K rows of H * qk, V rows of H * vhd
    T, bs = 30, 8
    Ks, Vs = _r(T, H, qk, seed=24), _r(T, H, vhd, seed=25)
    table = np.array([3, 0, 2, 1], np.int32)
    kp, vp, hpt = d.alloc_f32(4 * bs * H * qk), d.alloc_f32(4 * bs * H * vhd), d.upload(table)
    step = np.zeros(2, np.int32)
    hst = d.upload(step)
    for t in range(T):
        step[:] = (t, t + 1)
        d.call("aether_dev_h2d_i32", step.ctypes.data, hst, 2)
        d.call("aether_op_paged_append_kv_mla_devarg_f32_cuda", d.upload(Ks[t].ravel()), d.upload(Vs[t].ravel()), kp,
               vp, hpt, H * qk, H * vhd, bs, hst)
    out = d.alloc_f32(H * vhd)
    d.call("aether_op_paged_attention_mla_devarg_f32_cuda", d.upload(q), kp, vp, hpt, out, H, qk, vhd, bs, f(0.1), 64,
           hst)
    _close(d.download(out, (H, vhd)), _attn(q, Ks, Vs, 0.1))

    # absorbed MLA: Q8_0 and F16 per-head weights
    key_mla = qk
    wq = _r(H * lora, nope, seed=26) * 0.1
    wv = _r(H * vhd, lora, seed=27) * 0.1
    for name, typ in (("q8_0", G.Q8_0), ("f16", G.F16)):
        if typ == G.Q8_0:
            bq_ = np.frombuffer(G._quant_q8_0(wq.ravel()), np.uint8).copy()
            bv_ = np.frombuffer(G._quant_q8_0(wv.ravel()), np.uint8).copy()
            wq_d = G.dequantize(bq_, typ, wq.size).reshape(wq.shape)
            wv_d = G.dequantize(bv_, typ, wv.size).reshape(wv.shape)
            bpr_q, bpr_v = nope // 32, lora // 32
        else:
            bq_ = np.frombuffer(wq.astype(np.float16).tobytes(), np.uint8).copy()
            bv_ = np.frombuffer(wv.astype(np.float16).tobytes(), np.uint8).copy()
            wq_d, wv_d = wq.astype(np.float16).astype(np.float64), wv.astype(np.float16).astype(np.float64)
            bpr_q, bpr_v = nope, lora
        qo = d.alloc_f32(H * (lora + rope))
        d.call(f"aether_op_mla_absorb_q_{name}_cuda", d.upload(q), d.upload(bq_), qo, H, key_mla, rope, lora, bpr_q)
        want = np.concatenate([np.einsum("hcj,hj->hc", wq_d.reshape(H, lora, nope), q[:, :nope]), q[:, nope:]], 1)
        _close(d.download(qo, (H, lora + rope)), want)
        av = _r(H, lora, seed=28)
        ao = d.alloc_f32(H * vhd)
        d.call(f"aether_op_mla_absorb_v_{name}_cuda", d.upload(av), d.upload(bv_), ao, H, lora, vhd, bpr_v)
        _close(d.download(ao, (H, vhd)), np.einsum("hvc,hc->hv", wv_d.reshape(H, vhd, lora), av))


def test_bert_and_dinov3():
    d = _dev()
    S, H, hd = 33, 4, 32
    q, k, v = _r(S, H, hd, seed=30), _r(S, H, hd, seed=31), _r(S, H, hd, seed=32)
    out = d.alloc_f32(S * H * hd)
    d.call("aether_op_bert_self_attention_fwd_f32_cuda", d.upload(q), d.upload(k), d.upload(v), out, S, H, hd,
           f(hd ** -0.5))
    ref = torch.nn.functional.scaled_dot_product_attention(*(torch.from_numpy(t).transpose(0, 1) for t in (q, k, v)))
    _close(d.download(out, (S, H, hd)), ref.transpose(0, 1).numpy())
    V, P, Dm = 100, 64, 48
    word, pos, typ = _r(V, Dm, seed=33), _r(P, Dm, seed=34), _r(2, Dm, seed=35)
    ids = np.random.default_rng(0).integers(0, V, S).astype(np.int32)
    tt = (np.arange(S) >= 20).astype(np.int32)
    eo = d.alloc_f32(S * Dm)
    d.call("aether_op_bert_embed_sum_f32_cuda", d.upload(ids), d.upload(tt), d.upload(word), d.upload(pos),
           d.upload(typ), eo, S, Dm)
    _close(d.download(eo, (S, Dm)), word[ids] + pos[:S] + typ[tt], 1e-6)
    n_prefix, n_patch = 5, 16
    buf = _r(n_prefix + n_patch, H, hd, seed=36)
    cs, sn = np.cos(_r(n_patch, hd, seed=37)), np.sin(_r(n_patch, hd, seed=38))
    hb = d.upload(buf)
    d.call("aether_op_dinov3_rope2d_f32_cuda", hb, d.upload(cs.astype(np.float32)), d.upload(sn.astype(np.float32)),
           n_prefix + n_patch, n_prefix, H, hd, n_patch)
    x = buf[n_prefix:]
    rot = np.concatenate([-x[..., hd // 2 :], x[..., : hd // 2]], -1)
    want = buf.copy()
    want[n_prefix:] = x * cs[:, None, :] + rot * sn[:, None, :]
    _close(d.download(hb, buf.shape), want)


def test_q8_1_activations_and_batched_quant_matvec():
    d = _dev()
    rows, bpr = 16, 2
    k = bpr * 256
    blk = np.random.default_rng(40).integers(0, 256, size=(rows * bpr, 144), dtype=np.uint8)
    blk[:, 0:2] = np.frombuffer(np.float16(0.02).tobytes(), np.uint8)
    blk[:, 2:4] = np.frombuffer(np.float16(0.01).tobytes(), np.uint8)
    w = G.dequantize(blk.ravel(), G.Q4_K, rows * k).reshape(rows, k).astype(np.float64)
    x = _r(k, seed=41)
    aq, ad, as_ = d.alloc_u8(k), d.alloc_f32(k // 32), d.alloc_f32(k // 32)
    d.call("aether_op_quantize_q8_1_llama_cuda", d.upload(x), aq, ad, as_, k)
    qv = d.download(aq, k, np.uint8).view(np.int8).astype(np.float64)
    sc = d.download(ad, k // 32).astype(np.float64)
    xq = (qv.reshape(-1, 32) * sc[:, None]).ravel()
    assert np.abs(xq - x).max() <= sc.max() * 0.5 + 1e-6  # round-to-nearest of x / d
    _close(d.download(as_, k // 32), (qv.reshape(-1, 32).sum(1) * sc), 1e-5)
    hw, out = d.upload(blk.ravel()), d.alloc_f32(rows)
    d.call("aether_op_mmvq_q4k_q8_1_single_cuda", hw, aq, ad, out, rows, bpr)
    _close(d.download(out, rows), w @ xq)
    d.call("aether_op_mmvq_q4k_q8_1_swiglu_cuda", hw, hw, aq, ad, out, rows, bpr)
    z = w @ xq
    _close(d.download(out, rows), z / (1 + np.exp(-z)) * z)
    B = 3
    xb = _r(B, k, seed=42)
    ob = d.alloc_f32(B * rows)
    for name in ("q4k_matmul_seqB_v3", "q4k_matmul_seqB_fp16"):
        d.call(f"aether_op_fused_{name}_cuda", d.upload(xb), hw, ob, rows, bpr, B)
        _close(d.download(ob, (B, rows)), xb.astype(np.float64) @ w.T)
    d.call("aether_op_fused_q4k_membw_probe_cuda", d.upload(x), hw, out, rows, bpr)
    _close(d.download(out, rows), w @ x)
