"""The device-handle C ABI (libaether_dev.so): every export is bound, bad
handles and extents are refused without launching (CPU), and on a B200 every
op matches a plain fp32 PyTorch / numpy reference of the same op."""
import ctypes as C

import numpy as np
import pytest
import torch

from aether_b200.formats import gguf as G
from aether_b200.runtime import device as D


def test_exports_bound_and_bad_handles_refused():
    lb = D.lib()
    for name in D.SIGNATURES:
        assert hasattr(lb, name), name
    bogus = 10**9  # never handed out
    assert lb.aether_dev_alloc_f32(0) == 0
    assert lb.aether_op_add_f32_cuda(bogus, bogus, bogus, 4) == -1
    assert lb.aether_op_matmul_f32_cuda(bogus, bogus, bogus, 2, 2, 2) == -1
    assert lb.aether_op_sdpa_causal_forward_f32_cuda(bogus, bogus, bogus, bogus, bogus, 1, 4, 8) == -1
    assert lb.aether_op_fused_q4k_matmul_seq1_cuda(bogus, bogus, bogus, 4, 1) == -1
    assert lb.aether_dev_h2d_f32(0, bogus, 4) == -1
    assert np.isnan(lb.aether_op_cross_entropy_f32_cuda(bogus, bogus, bogus, 2, 4))
    assert lb.aether_wall_us() > 0
    assert lb.aether_op_paged_attention_seq1_devarg_f32_cuda(bogus, bogus, bogus, bogus, bogus, 8, 2, 64, 16, 1.0,
                                                             128, bogus) == -1
    assert lb.aether_op_paged_attention_seq1_v4_devarg_f32_cuda(bogus, bogus, bogus, bogus, bogus, bogus, bogus, bogus,
                                                                8, 2, 64, 16, 1.0, 128, 0, bogus) == -1
    assert lb.aether_op_mla_absorb_q_q4_k_cuda(bogus, bogus, bogus, 4, 192, 64, 512, 1) == -1
    assert lb.aether_op_quantize_q8_1_llama_cuda(bogus, bogus, bogus, bogus, 33) == -1
    if not torch.cuda.is_available():  # the GPU benches say -1 without a device
        assert lb.aether_llm_inference_bench_tps_cuda(3, 64, 2, 256, 8) == -1.0
        assert lb.aether_llm_inference_bench_tps_cuda_resident(3, 64, 2, 256, 8) == -1.0
    assert lb.aether_nccl_real_get_handle(0) == 0  # no clique yet
    assert lb.aether_nccl_real_all_reduce_f32(bogus, bogus, 4, 0, 1) == -1
    assert lb.aether_nccl_real_comm_world_size(5) == -1


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    return D.Dev()


def _rand(*shape, seed=0, scale=1.0):
    return (np.random.default_rng(seed).standard_normal(shape) * scale).astype(np.float32)


def _close(got, want, tol=1e-4):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    err = np.abs(got - want).max() / max(np.abs(want).max(), 1e-6)
    assert err < tol, err


@pytest.mark.gpu
def test_registry_copies_and_refusals():
    d = _dev()
    x = _rand(1000)
    h = d.upload(x)
    np.testing.assert_array_equal(d.download(h, 1000), x)
    # first-n copies and device-to-device copies with offsets
    y = d.alloc_f32(1000)
    d.call("aether_dev_d2d_f32_offset", h, 100, y, 0, 50)
    np.testing.assert_array_equal(d.download(y, 50), x[100:150])
    # an extent past the allocation is refused, not launched
    assert d.lib.aether_op_add_f32_cuda(h, h, y, 1001) == -1
    assert d.lib.aether_dev_d2d_f32_offset(h, 990, y, 0, 20) == -1
    # kinds are checked: an f32 handle is not an i32 buffer
    assert d.lib.aether_op_embed_lookup_f32_cuda(h, h, y, 4, 8) == -1
    assert d.lib.aether_dev_mem_free_bytes() > 0
    d.free(h)
    d.free(y)
    assert d.lib.aether_op_scale_f32_cuda(h, C.c_float(2.0), 10) == -1  # freed


@pytest.mark.gpu
@pytest.mark.parametrize("m,k,n,tol", [
    (67, 129, 45, 1e-5),      # small: the SIMT kernel
    (300, 190, 257, 2e-5),    # tensor cores (tf32 x3), every dimension ragged against the 128 / 32 tiles
    (1024, 1024, 1024, 2e-5),
])
def test_gemm_family(m, k, n, tol):
    """The f32 GEMM family against fp64 numpy. A single tf32 pass would be off
    by ~1e-3 relative; the three-term hi / lo split must stay at fp32 level."""
    d = _dev()
    a, b = _rand(m, k, seed=1), _rand(k, n, seed=2)
    ha, hb, ho = d.upload(a), d.upload(b), d.alloc_f32(m * n)
    d.call("aether_op_matmul_f32_cuda", ha, hb, ho, m, k, n)
    _close(d.download(ho, (m, n)), a.astype(np.float64) @ b, tol)
    d.call("aether_op_matmul_gelu_f32_cuda", ha, hb, ho, m, k, n)
    ref = torch.nn.functional.gelu(torch.from_numpy(a.astype(np.float64) @ b), approximate="tanh").numpy()
    _close(d.download(ho, (m, n)), ref, max(tol, 1e-5))
    at = d.upload(np.ascontiguousarray(a.T))  # [k, m]
    d.call("aether_op_matmul_tn_f32_cuda", at, hb, ho, m, k, n)
    _close(d.download(ho, (m, n)), a.astype(np.float64) @ b, tol)
    bt = d.upload(np.ascontiguousarray(b.T))  # [n, k]
    d.call("aether_op_matmul_nt_f32_cuda", ha, bt, ho, m, k, n)
    _close(d.download(ho, (m, n)), a.astype(np.float64) @ b, tol)
    dy = _rand(m, n, seed=3)
    hdy, hdb, hda = d.upload(dy), d.alloc_f32(k * n), d.alloc_f32(m * k)
    d.call("aether_op_matmul_backward_rhs_f32_cuda", ha, hdy, hdb, m, k, n)
    _close(d.download(hdb, (k, n)), a.T.astype(np.float64) @ dy, tol)
    d.call("aether_op_matmul_backward_lhs_f32_cuda", hdy, hb, hda, m, k, n)
    _close(d.download(hda, (m, k)), dy.astype(np.float64) @ b.T, tol)
    d.call("aether_bench_matmul_batch", ha, hb, ho, m, k, n, 3)
    d.call("aether_op_matmul_f32_cuda_profile", ha, hb, ho, m, k, n)


@pytest.mark.gpu
def test_elementwise_and_rows():
    d = _dev()
    n = 5000
    x, y = _rand(n, seed=4), _rand(n, seed=5)
    hx, hy, ho = d.upload(x), d.upload(y), d.alloc_f32(n)
    d.call("aether_op_add_f32_cuda", hx, hy, ho, n)
    _close(d.download(ho, n), x + y)
    tx = torch.from_numpy(x).requires_grad_()
    g = torch.nn.functional.gelu(tx, approximate="tanh")
    g.backward(torch.from_numpy(y))
    d.call("aether_op_gelu_f32_cuda", hx, ho, n)
    _close(d.download(ho, n), g.detach().numpy())
    d.call("aether_op_gelu_backward_f32_cuda", hx, hy, ho, n)
    _close(d.download(ho, n), tx.grad.numpy())
    d.call("aether_op_gelu_erf_f32_cuda", hx, ho, n)
    _close(d.download(ho, n), torch.nn.functional.gelu(torch.from_numpy(x)).numpy())
    tx = torch.from_numpy(x).requires_grad_()
    s = torch.nn.functional.silu(tx)
    s.backward(torch.from_numpy(y))
    d.call("aether_op_silu_backward_f32_cuda", hx, hy, ho, n)
    _close(d.download(ho, n), tx.grad.numpy())
    hs = d.upload(x)
    d.call("aether_op_silu_f32_cuda", hs, n)
    _close(d.download(hs, n), s.detach().numpy())
    d.call("aether_op_mul_inplace_f32_cuda", hs, hy, n)
    _close(d.download(hs, n), s.detach().numpy() * y)
    d.call("aether_op_add_inplace_f32_cuda", hs, hx, n)
    d.call("aether_op_scale_f32_cuda", hs, C.c_float(0.5), n)
    _close(d.download(hs, n), (s.detach().numpy() * y + x) * 0.5)
    rows, cols = 50, 100
    hb = d.upload(y[:cols])
    hm = d.upload(x[: rows * cols])
    d.call("aether_op_bias_add_f32_cuda", hm, hb, rows, cols)
    _close(d.download(hm, (rows, cols)), x[: rows * cols].reshape(rows, cols) + y[:cols])
    t3 = _rand(3, 5, 7, seed=6)
    ht, ho3 = d.upload(t3), d.alloc_f32(t3.size)
    d.call("aether_op_transpose_021_f32_cuda", ht, ho3, 3, 5, 7)
    _close(d.download(ho3, (5, 3, 7)), t3.transpose(1, 0, 2))

    # row ops
    b, dd = 37, 777
    x, dy = _rand(b, dd, seed=7), _rand(b, dd, seed=8)
    gam, bet = _rand(dd, seed=9), _rand(dd, seed=10)
    hx, hdy, hg, hbt = d.upload(x), d.upload(dy), d.upload(gam), d.upload(bet)
    hy, hmean, hrstd, hdx = d.alloc_f32(b * dd), d.alloc_f32(b), d.alloc_f32(b), d.alloc_f32(b * dd)
    d.call("aether_op_softmax_f32_cuda", hx, hy, b, dd)
    sm = torch.softmax(torch.from_numpy(x), -1)
    _close(d.download(hy, (b, dd)), sm.numpy())
    ts = torch.from_numpy(x).requires_grad_()
    torch.softmax(ts, -1).backward(torch.from_numpy(dy))
    d.call("aether_op_softmax_backward_scaled_f32_cuda", hy, hdy, hdx, C.c_float(0.5), b, dd)
    _close(d.download(hdx, (b, dd)), 0.5 * ts.grad.numpy(), 1e-3)

    tx, tg, tb = (torch.from_numpy(v).clone().requires_grad_() for v in (x, gam, bet))
    ln = torch.nn.functional.layer_norm(tx, (dd,), tg, tb, 1e-5)
    ln.backward(torch.from_numpy(dy))
    d.call("aether_op_layer_norm_f32_cuda", hx, hg, hbt, hy, hmean, hrstd, C.c_float(1e-5), b, dd)
    _close(d.download(hy, (b, dd)), ln.detach().numpy())
    d.call("aether_op_layer_norm_backward_dx_f32_cuda", hx, hg, hmean, hrstd, hdy, hdx, b, dd)
    _close(d.download(hdx, (b, dd)), tx.grad.numpy(), 1e-3)
    hdg, hdb = d.alloc_f32(dd), d.alloc_f32(dd)
    d.call("aether_op_layer_norm_backward_params_f32_cuda", hx, hmean, hrstd, hdy, hdg, hdb, b, dd)
    _close(d.download(hdg, dd), tg.grad.numpy(), 1e-3)
    _close(d.download(hdb, dd), tb.grad.numpy(), 1e-3)
    res = _rand(b, dd, seed=11)
    hres = d.upload(res)
    d.call("aether_op_add_layer_norm_f32_cuda", hx, hres, hg, hbt, hy, hmean, hrstd, C.c_float(1e-5), b, dd)
    _close(d.download(hy, (b, dd)),
           torch.nn.functional.layer_norm(torch.from_numpy(x + res), (dd,), torch.from_numpy(gam),
                                          torch.from_numpy(bet), 1e-5).numpy())

    tx, tg = (torch.from_numpy(v).clone().requires_grad_() for v in (x, gam))
    rms = tx * torch.rsqrt(tx.pow(2).mean(-1, keepdim=True) + 1e-6) * tg
    rms.backward(torch.from_numpy(dy))
    d.call("aether_op_rms_norm_f32_cuda", hx, hg, hy, C.c_float(1e-6), b, dd)
    _close(d.download(hy, (b, dd)), rms.detach().numpy())
    hinv = d.alloc_f32(b)
    d.call("aether_op_rms_norm_backward_dx_f32_cuda", hx, hg, hdy, hdx, hinv, C.c_float(1e-6), b, dd)
    _close(d.download(hdx, (b, dd)), tx.grad.numpy(), 1e-3)
    d.call("aether_op_rms_norm_backward_gamma_f32_cuda", hx, hdy, hinv, hdg, b, dd)
    _close(d.download(hdg, dd), tg.grad.numpy(), 1e-3)
    hx2 = d.upload(x)
    d.call("aether_op_fused_add_rmsnorm_f32_cuda", hx2, hres, hg, hy, C.c_float(1e-6), b, dd)
    s2 = x + res
    _close(d.download(hx2, (b, dd)), s2)
    _close(d.download(hy, (b, dd)), s2 / np.sqrt((s2 ** 2).mean(-1, keepdims=True) + 1e-6) * gam)


@pytest.mark.gpu
def test_cross_entropy_adamw_embedding_gqa_rope():
    d = _dev()
    b, v = 19, 1000
    logits = _rand(b, v, seed=12, scale=3.0)
    labels = np.random.default_rng(13).integers(0, v, b).astype(np.int32)
    hl, ht, hp, hd = d.upload(logits), d.upload(labels), d.alloc_f32(b * v), d.alloc_f32(b * v)
    loss = d.lib.aether_op_cross_entropy_f32_cuda(hl, ht, hp, b, v)
    tl = torch.from_numpy(logits).requires_grad_()
    ref = torch.nn.functional.cross_entropy(tl, torch.from_numpy(labels).long())
    ref.backward()
    assert abs(loss - float(ref)) < 1e-4 * abs(float(ref))
    d.call("aether_op_cross_entropy_backward_f32_cuda", hp, ht, hd, b, v)
    _close(d.download(hd, (b, v)), tl.grad.numpy(), 1e-3)

    n = 3000
    p, g = _rand(n, seed=14), _rand(n, seed=15)
    hp_, hg_, hm_, hv_ = d.upload(p), d.upload(g), d.alloc_f32(n), d.alloc_f32(n)
    tp = torch.from_numpy(p.copy()).requires_grad_()
    opt = torch.optim.AdamW([tp], lr=1e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.0)
    for step in (1, 2):
        d.call("aether_op_adamw_step_f32_cuda", hp_, hg_, hm_, hv_, C.c_float(1e-2), C.c_float(0.9), C.c_float(0.95),
               C.c_float(1e-8), C.c_float(0.0), step, n)
        tp.grad = torch.from_numpy(g)
        opt.step()
    _close(d.download(hp_, n), tp.detach().numpy(), 1e-5)

    V, Dm, T = 50, 16, 30
    table = _rand(V, Dm, seed=16)
    ids = np.random.default_rng(17).integers(0, V, T).astype(np.int32)
    htab, hid, hout = d.upload(table), d.upload(ids), d.alloc_f32(T * Dm)
    d.call("aether_op_embed_lookup_f32_cuda", htab, hid, hout, T, Dm)
    _close(d.download(hout, (T, Dm)), table[ids])
    dout = _rand(T, Dm, seed=18)
    hdo, hdt = d.upload(dout), d.alloc_f32(V * Dm)
    d.call("aether_op_embed_scatter_add_f32_cuda", hdo, hid, hdt, T, Dm)
    want = np.zeros((V, Dm), np.float32)
    np.add.at(want, ids, dout)
    _close(d.download(hdt, (V, Dm)), want, 1e-5)

    S, Hkv, Hq, hd = 5, 2, 6, 8
    kv = _rand(S, Hkv, hd, seed=19)
    hkv, hrep = d.upload(kv), d.alloc_f32(S * Hq * hd)
    d.call("aether_op_gqa_repeat_kv_f32_cuda", hkv, hrep, S, Hkv, hd, Hq)
    rep = np.repeat(kv, Hq // Hkv, axis=1)
    _close(d.download(hrep, (S, Hq, hd)), rep)
    grad = _rand(S, Hq, hd, seed=20)
    hgr, hred = d.upload(grad), d.alloc_f32(S * Hkv * hd)
    d.call("aether_op_gqa_reduce_kv_grad_f32_cuda", hgr, hred, S, Hkv, hd, Hq)
    _close(d.download(hred, (S, Hkv, hd)), grad.reshape(S, Hkv, Hq // Hkv, hd).sum(2))

    seq, heads, hd = 7, 3, 16
    xr = _rand(seq, heads, hd, seed=21)
    hx = d.upload(xr)
    d.call("aether_op_rope_apply_f32_cuda", hx, seq, heads, hd, C.c_float(10000.0), 5)
    half = hd // 2
    pos = np.arange(5, 5 + seq, dtype=np.float64)[:, None]
    ang = pos * 10000.0 ** (-2.0 * np.arange(half) / hd)[None, :]
    c, s = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]
    a0, a1 = xr[..., :half], xr[..., half:]
    want = np.concatenate([a0 * c - a1 * s, a0 * s + a1 * c], -1)
    _close(d.download(hx, (seq, heads, hd)), want, 1e-4)
    d.call("aether_op_rope_apply_backward_f32_cuda", hx, seq, heads, hd, C.c_float(10000.0), 5)
    _close(d.download(hx, (seq, heads, hd)), xr, 1e-4)  # the backward rotation undoes the forward


@pytest.mark.gpu
def test_sdpa_and_decode_attention_and_graphs():
    d = _dev()
    bh, s, hd = 3, 37, 16
    q, k, v, do = (_rand(bh, s, hd, seed=30 + i) for i in range(4))
    hq, hk, hv, hdo = d.upload(q), d.upload(k), d.upload(v), d.upload(do)
    ho, ha = d.alloc_f32(bh * s * hd), d.alloc_f32(bh * s * s)
    d.call("aether_op_sdpa_causal_forward_f32_cuda", hq, hk, hv, ho, ha, bh, s, hd)
    tq, tk, tv = (torch.from_numpy(t).requires_grad_() for t in (q, k, v))
    ref = torch.nn.functional.scaled_dot_product_attention(tq, tk, tv, is_causal=True)
    ref.backward(torch.from_numpy(do))
    _close(d.download(ho, (bh, s, hd)), ref.detach().numpy(), 1e-4)
    hdq, hdk, hdv, hds = (d.alloc_f32(n) for n in (bh * s * hd, bh * s * hd, bh * s * hd, bh * s * s))
    d.call("aether_op_sdpa_causal_backward_f32_cuda", hq, hk, hv, ha, hdo, hdq, hdk, hdv, hds, bh, s, hd)
    _close(d.download(hdq, (bh, s, hd)), tq.grad.numpy(), 1e-3)
    _close(d.download(hdk, (bh, s, hd)), tk.grad.numpy(), 1e-3)
    _close(d.download(hdv, (bh, s, hd)), tv.grad.numpy(), 1e-3)

    # one-token decode against a KV cache filled through append_kv
    max_seq, hq_, hkv_, hd_ = 64, 8, 2, 32
    dkv = hkv_ * hd_
    kc, vc = d.alloc_f32(max_seq * dkv), d.alloc_f32(max_seq * dkv)
    ks, vs = _rand(20, dkv, seed=40), _rand(20, dkv, seed=41)
    for t in range(20):
        hk1, hv1 = d.upload(ks[t]), d.upload(vs[t])
        d.call("aether_op_append_kv_f32_cuda", hk1, hv1, kc, vc, t, dkv)
    assert d.lib.aether_op_append_kv_f32_cuda(hk1, hv1, kc, vc, max_seq, dkv) == -1  # past the cache
    qd = _rand(hq_ * hd_, seed=42)
    hqd, hod = d.upload(qd), d.alloc_f32(hq_ * hd_)
    scale = 1.0 / np.sqrt(hd_)
    d.call("aether_op_attention_seq1_f32_cuda", hqd, kc, vc, hod, 20, hq_, hkv_, hd_, C.c_float(scale))
    qt = torch.from_numpy(qd).view(hq_, 1, hd_)
    kt = torch.from_numpy(ks).view(20, hkv_, hd_).transpose(0, 1).repeat_interleave(hq_ // hkv_, 0)
    vt = torch.from_numpy(vs).view(20, hkv_, hd_).transpose(0, 1).repeat_interleave(hq_ // hkv_, 0)
    want = torch.softmax(qt @ kt.transpose(1, 2) * scale, -1) @ vt
    _close(d.download(hod, hq_ * hd_), want.reshape(-1).numpy(), 1e-4)

    # a captured graph replays the same launches
    n = 1024
    x = _rand(n, seed=43)
    hx, hy = d.upload(x), d.upload(np.ones(n, np.float32))
    d.call("aether_dev_graph_begin")
    d.call("aether_op_add_inplace_f32_cuda", hx, hy, n)
    d.call("aether_op_scale_f32_cuda", hx, C.c_float(2.0), n)
    d.call("aether_dev_graph_end")
    d.call("aether_dev_graph_launch")
    d.call("aether_dev_graph_launch")
    d.call("aether_dev_sync")
    _close(d.download(hx, n), ((x + 1) * 2 + 1) * 2)
    d.call("aether_dev_graph_destroy")


_HALVES = {G.Q4_0: (0,), G.Q8_0: (0,), G.Q5_0: (0,), G.IQ4_NL: (0,), G.Q4_K: (0, 2), G.Q5_K: (0, 2), G.Q3_K: (108,),
           G.Q6_K: (208,), G.IQ4_XS: (0,), G.IQ3_XXS: (0,), G.IQ3_S: (0,)}


def _qblocks(typ, n, seed):
    ne, nb = G.BLOCKS[typ]
    rng = np.random.default_rng(seed)
    b = rng.integers(0, 256, size=(n, nb), dtype=np.uint8)
    for o in _HALVES[typ]:  # sane f16 scales
        b[:, o : o + 2] = np.frombuffer(np.float16(rng.uniform(0.01, 0.1)).tobytes(), np.uint8)
    return b


@pytest.mark.gpu
@pytest.mark.parametrize("typ,name", [(G.Q4_0, "q4_0"), (G.Q5_0, "q5_0"), (G.Q8_0, "q8_0"), (G.IQ4_NL, "iq4_nl"),
                                      (G.Q3_K, "q3_k"), (G.Q4_K, "q4k"), (G.Q5_K, "q5_k"), (G.Q6_K, "q6k"),
                                      (G.IQ4_XS, "iq4_xs"), (G.IQ3_XXS, "iq3_xxs"), (G.IQ3_S, "iq3_s")])
def test_quantised_dequant_and_matvec(typ, name):
    """Device dequantisation and the fused mat-vec against the load-time
    dequantiser of the same GGUF blocks (numpy, or the native host decoders of
    the IQ3 codebook formats)."""
    d = _dev()
    ne, nb = G.BLOCKS[typ]
    rows, bpr = 24, (4 if ne == 256 else 32)
    blk = _qblocks(typ, rows * bpr, seed=typ)
    k = bpr * ne
    w = G.dequantize(blk.reshape(-1), typ, rows * k).reshape(rows, k)
    hw, hout = d.upload(blk.reshape(-1)), d.alloc_f32(rows * k)
    d.call("aether_op_dequant_f32_cuda", typ, hw, hout, rows * bpr)
    _close(d.download(hout, (rows, k)), w, 1e-6)
    x = _rand(k, seed=50)
    hx, hy = d.upload(x), d.alloc_f32(rows)
    fn = f"aether_op_fused_{name}_matmul_seq1_cuda" if name != "q6k" else "aether_op_fused_q6k_matmul_seq1_v2_cuda"
    d.call(fn, hx, hw, hy, rows, bpr)
    _close(d.download(hy, rows), w.astype(np.float64) @ x, 1e-4)
    if typ == G.Q4_K:
        # gate/up SwiGLU in one pass, experts, and the frozen-weight input gradient
        hy2 = d.alloc_f32(rows)
        d.call("aether_op_fused_q4k_ffn_gate_up_silu_mul_cuda", hx, hw, hw, hy2, rows, bpr)
        z = w.astype(np.float64) @ x
        _close(d.download(hy2, rows), z / (1 + np.exp(-z)) * z, 1e-4)
        blk1 = _qblocks(typ, rows * bpr, seed=99).reshape(-1)
        two = d.upload(np.concatenate([blk.reshape(-1), blk1]))
        w1 = G.dequantize(blk1, typ, rows * k).reshape(rows, k)
        d.call("aether_op_fused_q4k_expert_matmul_seq1_cuda", hx, two, hy, rows, bpr, 1)
        _close(d.download(hy, rows), w1.astype(np.float64) @ x, 1e-4)
        dyv = _rand(rows, seed=51)
        hdy, hdx = d.upload(dyv), d.alloc_f32(k)
        d.call("aether_op_quant_matmul_backward_lhs_f32_cuda", hw, typ, hdy, hdx, rows, k)
        _close(d.download(hdx, k), w.T.astype(np.float64) @ dyv, 1e-4)
    if typ in (G.Q4_K, G.Q6_K, G.IQ3_XXS):
        fn = {G.Q4_K: "aether_op_dequant_q4_k_m_f32_cuda", G.Q6_K: "aether_op_dequant_q6_k_f32_cuda",
              G.IQ3_XXS: "aether_op_dequant_iq3_xxs_f32_cuda"}[typ]
        d.call(fn, hw, hout, rows * bpr)
        _close(d.download(hout, (rows, k)), w, 1e-6)
    if typ in (G.IQ3_XXS, G.IQ3_S):  # expert e = 1 of a stacked pair
        blk1 = _qblocks(typ, rows * bpr, seed=98).reshape(-1)
        two = d.upload(np.concatenate([blk.reshape(-1), blk1]))
        w1 = G.dequantize(blk1, typ, rows * k).reshape(rows, k)
        d.call(f"aether_op_fused_{name}_expert_matmul_seq1_cuda", hx, two, hy, rows, bpr, 1)
        _close(d.download(hy, rows), w1.astype(np.float64) @ x, 1e-4)


@pytest.mark.gpu
def test_f16_f32_weight_matvec():
    d = _dev()
    n_in, n_out = 256, 40
    w = _rand(n_out, n_in, seed=60)
    x = _rand(n_in, seed=61)
    hx, hy = d.upload(x), d.alloc_f32(n_out)
    hw16 = d.upload(np.frombuffer(w.astype(np.float16).tobytes(), np.uint8).copy())
    d.call("aether_op_fused_f16_matmul_seq1_cuda", hx, hw16, hy, n_in, n_out)
    _close(d.download(hy, n_out), w.astype(np.float16).astype(np.float64) @ x, 1e-4)
    hw32 = d.upload(np.frombuffer(w.tobytes(), np.uint8).copy())
    d.call("aether_op_fused_f32_matmul_seq1_cuda", hx, hw32, hy, n_in, n_out)
    _close(d.download(hy, n_out), w.astype(np.float64) @ x, 1e-4)


@pytest.mark.gpu
def test_cuda_train_tiny_witness_matches_host_ops():
    """The reference's cuda_train_tiny program (B=8, K=16, N=4 linear
    classifier, 50 AdamW steps) driven through the device ABI, against the
    same steps on the host ops of libaether_rt."""
    from aether_b200 import runtime as rt

    d = _dev()
    B, K, N = 8, 16, 4
    x = np.zeros(B * K, np.float32)
    w0 = np.zeros(K * N, np.float32)
    lab = np.zeros(B, np.int32)
    rt.call("aether_init_normal_f32", rt.ptr(x), B * K, C.c_float(1.0), 1)
    rt.call("aether_init_normal_f32", rt.ptr(w0), K * N, C.c_float(0.1), 7)
    rt.call("aether_fill_labels_i32", rt.ptr(lab), B, N, 13)
    hx, hw, hl = d.upload(x), d.upload(w0), d.upload(lab)
    hy, hp, hdy, hdw, hm, hv = (d.alloc_f32(n) for n in (B * N, B * N, B * N, K * N, K * N, K * N))
    dev_losses = []
    for s in range(1, 51):
        d.call("aether_op_matmul_f32_cuda", hx, hw, hy, B, K, N)
        dev_losses.append(d.lib.aether_op_cross_entropy_f32_cuda(hy, hl, hp, B, N))
        d.call("aether_op_cross_entropy_backward_f32_cuda", hp, hl, hdy, B, N)
        d.call("aether_op_matmul_backward_rhs_f32_cuda", hx, hdy, hdw, B, K, N)
        d.call("aether_op_adamw_step_f32_cuda", hw, hdw, hm, hv, C.c_float(0.05), C.c_float(0.9), C.c_float(0.999),
               C.c_float(1e-8), C.c_float(0.0), s, K * N)
    d.call("aether_dev_sync")
    assert dev_losses[-1] < dev_losses[0]
    # host ops, same program
    w = w0.copy()
    y, p, dy, dw, m, v = (np.zeros(n, np.float32) for n in (B * N, B * N, B * N, K * N, K * N, K * N))
    lib = rt.lib()
    for f in ("aether_op_cross_entropy_f32",):
        getattr(lib, f).restype = C.c_float
    lib.aether_op_adamw_step_f32.argtypes = [C.c_void_p] * 4 + [C.c_float] * 5 + [C.c_int64, C.c_int]
    host_losses = []
    for s in range(1, 51):
        lib.aether_op_matmul_f32(rt.ptr(x), rt.ptr(w), rt.ptr(y), B, K, N)
        host_losses.append(lib.aether_op_cross_entropy_f32(rt.ptr(y), rt.ptr(lab), rt.ptr(p), B, N))
        lib.aether_op_cross_entropy_backward_f32(rt.ptr(p), rt.ptr(lab), rt.ptr(dy), B, N)
        lib.aether_op_matmul_backward_rhs_f32(rt.ptr(x), rt.ptr(dy), rt.ptr(dw), B, K, N)
        lib.aether_op_adamw_step_f32(rt.ptr(w), rt.ptr(dw), rt.ptr(m), rt.ptr(v), 0.05, 0.9, 0.999, 1e-8, 0.0, s, K * N)
    np.testing.assert_allclose(dev_losses, host_losses, rtol=1e-4)
    np.testing.assert_allclose(d.download(hw, K * N), w, rtol=1e-3, atol=1e-5)


@pytest.mark.gpu
def test_nccl_clique_on_the_visible_gpus():
    """ncclCommInitAll over every visible GPU; each rank's buffer holds rank + 1
    and the queued per-rank calls run as one group (a 1-GPU clique at once)."""
    d = _dev()
    n = d.lib.aether_dev_count()
    assert d.lib.aether_nccl_real_init_multi_gpu(n) == n
    sends, recvs = [], []
    for r in range(n):
        d.call("aether_dev_set_device", r)
        sends.append(d.upload(np.full(1000, r + 1, np.float32)))
        recvs.append(d.alloc_f32(1000))
    assert d.lib.aether_nccl_real_all_reduce_f32(sends[0], recvs[0], 1000, 9, 1) == -1  # bad op
    for r in range(n):
        h = d.lib.aether_nccl_real_get_handle(r)
        assert d.lib.aether_nccl_real_comm_rank(h) == r and d.lib.aether_nccl_real_comm_world_size(h) == n
        d.call("aether_nccl_real_all_reduce_f32", sends[r], recvs[r], 1000, 0, h)
    want = n * (n + 1) / 2
    for r in range(n):
        d.call("aether_dev_set_device", r)
        d.call("aether_dev_sync")
        assert (d.download(recvs[r], 1000) == want).all()
    d.call("aether_nccl_real_finalize")
    d.call("aether_dev_set_device", 0)


@pytest.mark.gpu
def test_tiny_lm_benches(capsys):
    """The reference witnesses' tiny decoder (2 layers, d 64, ff 256, 8
    tokens): per-call routing and the device-resident graph replay."""
    d = _dev()
    per_call = d.lib.aether_llm_inference_bench_tps_cuda(50, 64, 2, 256, 8)
    resident = d.lib.aether_llm_inference_bench_tps_cuda_resident(2000, 64, 2, 256, 8)
    with capsys.disabled():
        print(f"\ntiny LM iterations/s: per-call {per_call:.0f}, resident {resident:.0f}")
    assert per_call > 0 and resident > per_call
