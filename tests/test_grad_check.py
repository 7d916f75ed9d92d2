"""Gradient checks of the f32 C ABIs: a LayerNorm -> matmul -> GELU -> matmul
-> cross-entropy block and a causal attention block, differentiated with the
libraries' own backward ops and compared with central finite differences of
their forward ops, on the host ops of libaether_rt (CPU) and the device ops of
libaether_dev (GPU)."""
import ctypes as C

import numpy as np
import pytest
import torch

from aether_b200 import runtime as rt
from aether_b200.runtime import device as D

B, DM, FF, V = 6, 16, 24, 10
EPS, PROBES = 1e-2, 6


def _params(seed=0):
    g = np.random.default_rng(seed)
    return {
        "x": g.standard_normal((B, DM)).astype(np.float32),
        "gamma": (1 + 0.1 * g.standard_normal(DM)).astype(np.float32),
        "beta": (0.1 * g.standard_normal(DM)).astype(np.float32),
        "w1": (0.3 * g.standard_normal((DM, FF))).astype(np.float32),
        "w2": (0.3 * g.standard_normal((FF, V))).astype(np.float32),
    }, g.integers(0, V, B).astype(np.int32)


def _check(loss_fn, grads, params, seed=1):
    """Central differences at a few random entries of every tensor."""
    g = np.random.default_rng(seed)
    for name, p in params.items():
        for _ in range(PROBES):
            i = tuple(int(g.integers(0, s)) for s in p.shape)
            old = p[i]
            p[i] = old + EPS
            lp = loss_fn(params)
            p[i] = old - EPS
            lm = loss_fn(params)
            p[i] = old
            fd = (lp - lm) / (2 * EPS)
            an = float(grads[name][i])
            assert abs(fd - an) <= 2e-3 + 3e-2 * abs(an), (name, i, fd, an)


# ------------------------------------------------------------------------------------------------ host ops
def _host_block(params, labels, backward=False):
    lb = rt.lib()
    lb.aether_op_cross_entropy_f32.restype = C.c_float
    p = rt.ptr
    ln, mean, inv = (np.zeros(s, np.float32) for s in ((B, DM), B, B))
    lb.aether_op_layer_norm_f32(p(params["x"]), p(params["gamma"]), p(params["beta"]), C.c_float(1e-5), p(ln), p(mean),
                                p(inv), B, DM)
    h1 = np.zeros((B, FF), np.float32)
    lb.aether_op_matmul_f32(p(ln), p(params["w1"]), p(h1), B, DM, FF)
    a1 = h1.copy()
    lb.aether_op_gelu_f32(p(a1), B * FF)
    logits, probs = np.zeros((B, V), np.float32), np.zeros((B, V), np.float32)
    lb.aether_op_matmul_f32(p(a1), p(params["w2"]), p(logits), B, FF, V)
    loss = lb.aether_op_cross_entropy_f32(p(logits), p(labels), p(probs), B, V)
    if not backward:
        return loss
    dl, dw2, da1, dh1, dw1, dln = (np.zeros(s, np.float32) for s in ((B, V), (FF, V), (B, FF), (B, FF), (DM, FF), (B, DM)))
    lb.aether_op_cross_entropy_backward_f32(p(probs), p(labels), p(dl), B, V)
    lb.aether_op_matmul_backward_rhs_f32(p(a1), p(dl), p(dw2), B, FF, V)
    lb.aether_op_matmul_backward_lhs_f32(p(dl), p(params["w2"]), p(da1), B, FF, V)
    lb.aether_op_gelu_backward_f32(p(h1), p(da1), p(dh1), B * FF)
    lb.aether_op_matmul_backward_rhs_f32(p(ln), p(dh1), p(dw1), B, DM, FF)
    lb.aether_op_matmul_backward_lhs_f32(p(dh1), p(params["w1"]), p(dln), B, DM, FF)
    dx, dg, db = np.zeros((B, DM), np.float32), np.zeros(DM, np.float32), np.zeros(DM, np.float32)
    lb.aether_op_layer_norm_backward_f32(p(params["x"]), p(params["gamma"]), p(dln), p(mean), p(inv), p(dx), p(dg),
                                         p(db), B, DM)
    return loss, {"x": dx, "gamma": dg, "beta": db, "w1": dw1, "w2": dw2}


def test_host_block_gradients():
    params, labels = _params()
    _, grads = _host_block(params, labels, backward=True)
    _check(lambda ps: _host_block(ps, labels), grads, params)


def test_host_causal_attention_gradients():
    lb = rt.lib()
    bh, s, d = 2, 5, 8
    g = np.random.default_rng(3)
    qkv = {n: g.standard_normal((bh, s, d)).astype(np.float32) for n in ("q", "k", "v")}
    w = g.standard_normal((bh, s, d)).astype(np.float32)  # loss = sum(out * w)
    p = rt.ptr

    def fwd(ps):
        out, att = np.zeros((bh, s, d), np.float32), np.zeros((bh, s, s), np.float32)
        lb.aether_op_sdpa_causal_f32(p(ps["q"]), p(ps["k"]), p(ps["v"]), p(out), p(att), bh, s, d)
        return float((out.astype(np.float64) * w).sum()), att

    _, att = fwd(qkv)
    dq, dk, dv = (np.zeros((bh, s, d), np.float32) for _ in range(3))
    lb.aether_op_sdpa_causal_backward_f32(p(qkv["q"]), p(qkv["k"]), p(qkv["v"]), p(att), p(w), p(dq), p(dk), p(dv), bh,
                                          s, d)
    _check(lambda ps: fwd(ps)[0], {"q": dq, "k": dk, "v": dv}, qkv)


# ------------------------------------------------------------------------------------------------ device ops
def _dev_block(d, params, labels, backward=False):
    f = C.c_float
    h = {n: d.upload(v) for n, v in params.items()}
    hl = d.upload(labels)
    ln, mean, rstd = d.alloc_f32(B * DM), d.alloc_f32(B), d.alloc_f32(B)
    d.call("aether_op_layer_norm_f32_cuda", h["x"], h["gamma"], h["beta"], ln, mean, rstd, f(1e-5), B, DM)
    h1, a1 = d.alloc_f32(B * FF), d.alloc_f32(B * FF)
    d.call("aether_op_matmul_f32_cuda", ln, h["w1"], h1, B, DM, FF)
    d.call("aether_op_gelu_f32_cuda", h1, a1, B * FF)
    logits, probs = d.alloc_f32(B * V), d.alloc_f32(B * V)
    d.call("aether_op_matmul_f32_cuda", a1, h["w2"], logits, B, FF, V)
    loss = d.lib.aether_op_cross_entropy_f32_cuda(logits, hl, probs, B, V)
    if not backward:
        return loss
    dl, dw2, da1, dh1, dw1, dln = (d.alloc_f32(n) for n in (B * V, FF * V, B * FF, B * FF, DM * FF, B * DM))
    d.call("aether_op_cross_entropy_backward_f32_cuda", probs, hl, dl, B, V)
    d.call("aether_op_matmul_backward_rhs_f32_cuda", a1, dl, dw2, B, FF, V)
    d.call("aether_op_matmul_backward_lhs_f32_cuda", dl, h["w2"], da1, B, FF, V)
    d.call("aether_op_gelu_backward_f32_cuda", h1, da1, dh1, B * FF)
    d.call("aether_op_matmul_backward_rhs_f32_cuda", ln, dh1, dw1, B, DM, FF)
    d.call("aether_op_matmul_backward_lhs_f32_cuda", dh1, h["w1"], dln, B, DM, FF)
    dx, dg, db = d.alloc_f32(B * DM), d.alloc_f32(DM), d.alloc_f32(DM)
    d.call("aether_op_layer_norm_backward_dx_f32_cuda", h["x"], h["gamma"], mean, rstd, dln, dx, B, DM)
    d.call("aether_op_layer_norm_backward_params_f32_cuda", h["x"], mean, rstd, dln, dg, db, B, DM)
    return loss, {"x": d.download(dx, (B, DM)), "gamma": d.download(dg, DM), "beta": d.download(db, DM),
                  "w1": d.download(dw1, (DM, FF)), "w2": d.download(dw2, (FF, V))}


@pytest.mark.gpu
def test_device_block_gradients():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    d = D.Dev()
    params, labels = _params(seed=5)
    _, grads = _dev_block(d, params, labels, backward=True)
    _check(lambda ps: _dev_block(d, ps, labels), grads, params, seed=6)


@pytest.mark.gpu
def test_device_causal_attention_gradients():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    d = D.Dev()
    bh, s, hd = 2, 7, 16
    g = np.random.default_rng(7)
    qkv = {n: g.standard_normal((bh, s, hd)).astype(np.float32) for n in ("q", "k", "v")}
    w = g.standard_normal((bh, s, hd)).astype(np.float32)
    hw = d.upload(w)

    def fwd(ps, keep=False):
        hs = [d.upload(ps[n]) for n in ("q", "k", "v")]
        out, att = d.alloc_f32(bh * s * hd), d.alloc_f32(bh * s * s)
        d.call("aether_op_sdpa_causal_forward_f32_cuda", *hs, out, att, bh, s, hd)
        loss = float((d.download(out, (bh, s, hd)).astype(np.float64) * w).sum())
        return (loss, hs, att) if keep else loss

    _, hs, att = fwd(qkv, keep=True)
    dq, dk, dv, ds = (d.alloc_f32(n) for n in (bh * s * hd, bh * s * hd, bh * s * hd, bh * s * s))
    d.call("aether_op_sdpa_causal_backward_f32_cuda", *hs, att, hw, dq, dk, dv, ds, bh, s, hd)
    grads = {n: d.download(h, (bh, s, hd)) for n, h in (("q", dq), ("k", dk), ("v", dv))}
    _check(fwd, grads, qkv, seed=8)
