"""Numerics of every sm_100a kernel against the plain-PyTorch fp32 reference
(aether_b200.ops.reference), the way the reference runtime checks its CUDA
kernels against ops.rs (runtime/tests/cuda_*_parity.rs)."""
import math

import pytest
import torch

from aether_b200 import _ext
from aether_b200.ops import functional as F
from aether_b200.ops import reference as ref
from tests.util import assert_close

pytestmark = pytest.mark.gpu
dev = "cuda"


@pytest.fixture(autouse=True)
def _status():
    _ext.C()
    yield
    torch.cuda.synchronize()
    assert _ext.check_status() == 0


def bf(*shape, scale=1.0, seed=0):
    g = torch.Generator(device=dev).manual_seed(seed)
    return (torch.randn(*shape, device=dev, generator=g) * scale).to(torch.bfloat16)


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 1024), (300, 264, 200), (1000, 776, 328), (2048, 2048, 2048)])
def test_gemm_nt(M, N, K):
    a, b = bf(M, K, seed=1), bf(N, K, seed=2)
    out = F.gemm(a, b)
    assert_close(out, ref.gemm(a, b), 1e-2, "gemm nt")


@pytest.mark.parametrize("a_mn,b_mn", [(False, True), (True, True), (True, False)])
@pytest.mark.parametrize("M,N,K", [(256, 256, 128), (384, 520, 264), (1024, 2048, 512)])
def test_gemm_layouts(a_mn, b_mn, M, N, K):
    a = bf(K, M, seed=3) if a_mn else bf(M, K, seed=3)
    b = bf(K, N, seed=4) if b_mn else bf(N, K, seed=4)
    out = F.gemm(a, b, a_mn=a_mn, b_mn=b_mn)
    assert_close(out, ref.gemm(a, b, a_mn, b_mn), 1e-2, f"gemm a_mn={a_mn} b_mn={b_mn}")


def test_gemm_epilogues():
    M, N, K = 520, 384, 256
    a, b = bf(M, K, seed=5), bf(N, K, seed=6)
    bias, res = bf(N, seed=7), bf(M, N, seed=8)
    out = F.gemm(a, b, bias=bias, residual=res, alpha=0.5)
    assert_close(out, ref.gemm(a, b, bias=bias, residual=res, alpha=0.5), 1e-2, "gemm epilogue")
    acc = torch.randn(M, N, device=dev)
    acc0 = acc.clone()
    F.gemm(a, b, out=acc, accumulate=True)
    assert_close(acc, acc0 + ref.gemm(a, b), 1e-3, "gemm fp32 accumulate")
    f32 = F.gemm(a, b, out_dtype=torch.float32)
    assert_close(f32, ref.gemm(a, b), 1e-4, "gemm fp32 out")
    at = torch.tensor([2.0], device=dev)
    o2 = F.gemm(a, b, out_dtype=torch.float32, alpha_t=at)
    assert_close(o2, 2 * ref.gemm(a, b), 1e-4, "gemm alpha_t")


def test_gemm_large_persistent():
    a, b = bf(8192, 2048, seed=9), bf(5632, 2048, seed=10)
    out = F.gemm(a, b)
    # check a sample of rows against fp32
    idx = torch.randint(0, 8192, (64,), device=dev)
    assert_close(out[idx], ref.gemm(a[idx], b), 1e-2, "gemm large")


@pytest.mark.parametrize("d", [64, 1536, 2048, 3584, 4096])
def test_rmsnorm(d):
    x, w, r = bf(257, d, seed=1), bf(d, seed=2), bf(257, d, seed=3)
    y, h, rstd = F.rmsnorm(x, w, 1e-6)
    yr, _, rr = ref.rmsnorm(x, w, 1e-6)
    assert_close(y, yr, 1e-2, "rmsnorm")
    assert_close(rstd, rr, 1e-5, "rstd")
    y2, h2, _ = F.rmsnorm(x, w, 1e-6, res=r)
    yr2, hr2, _ = ref.rmsnorm(x, w, 1e-6, res=r)
    assert_close(h2, hr2, 1e-2, "rmsnorm residual stream")
    assert_close(y2, yr2, 1e-2, "rmsnorm+res")
    # backward
    dy = bf(257, d, seed=4)
    dw = torch.zeros(d, device=dev)
    dx = F.rmsnorm_bwd(dy, x, w, rstd, dw, accumulate=True)
    xf = x.float().requires_grad_(True)
    wf = w.float().requires_grad_(True)
    yf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * wf
    yf.backward(dy.float())
    assert_close(dx, xf.grad, 2e-2, "rmsnorm dx")
    assert_close(dw, wf.grad, 1e-3, "rmsnorm dw")


@pytest.mark.parametrize("d", [768, 4096])
def test_layernorm(d):
    x, w, b = bf(130, d, seed=1), bf(d, seed=2), bf(d, seed=3)
    y, h, mean, rstd = F.layernorm(x, w, b, 1e-5)
    yr, _ = ref.layernorm(x, w, b, 1e-5)
    assert_close(y, yr, 1e-2, "layernorm")
    dy = bf(130, d, seed=4)
    dw, db = torch.zeros(d, device=dev), torch.zeros(d, device=dev)
    dx = F.layernorm_bwd(dy, x, w, mean, rstd, dw, db)
    xf, wf, bfp = (t.float().requires_grad_(True) for t in (x, w, b))
    torch.nn.functional.layer_norm(xf, (d,), wf, bfp, 1e-5).backward(dy.float())
    assert_close(dx, xf.grad, 2e-2, "ln dx")
    assert_close(dw, wf.grad, 1e-3, "ln dw")
    assert_close(db, bfp.grad, 1e-3, "ln db")


@pytest.mark.parametrize("d", [512, 4096])
def test_softmax(d):
    x = bf(100, d, scale=3.0)
    y = F.softmax(x, 0.7)
    assert_close(y, ref.softmax(x, 0.7), 1e-2, "softmax")
    dy = bf(100, d, seed=5)
    dx = F.softmax_bwd(y, dy, 0.7)
    xf = x.float().requires_grad_(True)
    torch.softmax(xf * 0.7, -1).backward(dy.float())
    assert_close(dx, xf.grad, 3e-2, "softmax bwd")


def test_swiglu_gelu():
    h = bf(333, 2 * 1024)
    assert_close(F.swiglu(h), ref.swiglu(h), 1e-2, "swiglu")
    da = bf(333, 1024, seed=3)
    hf = h.float().requires_grad_(True)
    ref.swiglu(hf).backward(da.float())
    assert_close(F.swiglu_bwd(h, da), hf.grad, 2e-2, "swiglu bwd")
    x = bf(4096, 8, seed=4)
    assert_close(F.gelu(x), ref.gelu_tanh(x), 1e-2, "gelu")
    dy = bf(4096, 8, seed=5)
    xf = x.float().requires_grad_(True)
    ref.gelu_tanh(xf).backward(dy.float())
    assert_close(F.gelu_bwd(x, dy), xf.grad, 2e-2, "gelu bwd")


def test_rope():
    T, H, D = 300, 6, 128
    cos, sin = ref.rope_tables(512, D, 1e6, device=dev)
    x = bf(T, (H + 4) * D)
    pos = torch.randint(0, 512, (T,), device=dev, dtype=torch.int32)
    y = x.clone()
    F.rope_(y, pos, cos, sin, H, D)
    assert_close(y, ref.rope(x, pos, cos, sin, H, D), 1e-2, "rope")
    F.rope_(y, pos, cos, sin, H, D, inverse=True)
    assert_close(y, x, 2e-2, "rope inverse")


def test_embedding():
    table = bf(1000, 256)
    ids = torch.randint(0, 1000, (4, 77), device=dev)
    out = F.embedding(table, ids)
    assert torch.equal(out, table[ids])
    dy = bf(4, 77, 256, seed=3)
    g = torch.zeros(1000, 256, device=dev)
    F.embedding_bwd(dy, ids, g)
    gr = torch.zeros(1000, 256, device=dev).index_add_(0, ids.reshape(-1), dy.reshape(-1, 256).float())
    assert_close(g, gr, 1e-5, "embedding bwd")


@pytest.mark.parametrize("V", [32000, 151936, 1003])
def test_cross_entropy(V):
    T = 64
    logits = bf(T, V, scale=2.0)
    tgt = torch.randint(0, V, (T,), device=dev)
    tgt[3] = -100
    lr_, lse_r = ref.cross_entropy(logits, tgt)
    gr = ref.cross_entropy_grad(logits, tgt, 1.0 / T)
    buf = logits.clone()
    loss, lse = F.cross_entropy_fused(buf, tgt, grad_scale=1.0 / T)
    assert_close(loss, lr_, 1e-4, "ce loss")
    assert float(loss[3]) == 0.0
    assert_close(buf, gr, 1e-2, "ce grad (in place)")


def test_argmax():
    x = bf(7, 151936)
    assert torch.equal(F.argmax(x), x.float().argmax(-1))
    y = torch.randn(3, 152064, device=dev)  # fp32, vectorised path
    assert torch.equal(F.argmax(y), y.argmax(-1))
    z = torch.randn(3, 1003, device=dev)[:, :1001]  # odd stride: scalar path
    assert torch.equal(F.argmax(z), z.argmax(-1))
    t = torch.zeros(2, 70000, device=dev)
    t[0, 5] = t[0, 60000] = 1.0  # ties go to the lowest index
    assert F.argmax(t).tolist() == [5, 0]


def test_adamw():
    n = 100003
    p = torch.randn(n, device=dev)
    g = torch.randn(n, device=dev)
    m, v = torch.zeros(n, device=dev), torch.zeros(n, device=dev)
    pb = torch.empty(n, device=dev, dtype=torch.bfloat16)
    p2, m2, v2 = p.clone(), m.clone(), v.clone()
    for step in (1, 2, 3):
        F.adamw_(p, g, m, v, pb, lr=1e-3, beta1=0.9, beta2=0.95, eps=1e-8, wd=0.1, step=step, gscale=0.5)
        ref.adamw(p2, g, m2, v2, 1e-3, 0.9, 0.95, 1e-8, 0.1, step, 0.5)
    assert_close(p, p2, 1e-6, "adamw p")
    assert_close(pb, p2, 1e-2, "adamw bf16 copy")
    norm, clip = F.grad_norm(g, pre_scale=1.0, max_norm=1.0)
    assert abs(float(norm) - float(g.norm())) / float(g.norm()) < 1e-5
    assert abs(float(clip) - 1.0 / float(g.norm())) < 1e-5


@pytest.mark.parametrize("B,Sq,Sk,Hq,Hkv,D,causal", [
    (2, 256, 256, 4, 4, 128, True),
    (1, 300, 300, 4, 2, 128, True),
    (2, 128, 384, 6, 2, 128, True),    # prefill on top of a cache (offset)
    (1, 200, 333, 2, 1, 64, False),
    (2, 1024, 1024, 8, 8, 128, True),
])
def test_attention_fwd_bwd(B, Sq, Sk, Hq, Hkv, D, causal):
    q, k, v = bf(B, Sq, Hq, D, seed=1), bf(B, Sk, Hkv, D, seed=2), bf(B, Sk, Hkv, D, seed=3)
    scale = 1.0 / math.sqrt(D)
    off = Sk - Sq
    o, lse = F.attention(q, k, v, scale, causal, off)
    o_r, lse_r = ref.attention(q, k, v, scale, causal, off)
    assert_close(o, o_r, 1e-2, "attention out")
    assert_close(lse, lse_r, 1e-4, "attention lse")
    do = bf(B, Sq, Hq, D, seed=4)
    dq, dk, dv = F.attention_bwd(q, k, v, o, do, lse, scale, causal, off)
    qf, kf, vf = (t.float().requires_grad_(True) for t in (q, k, v))
    of, _ = ref.attention(qf, kf, vf, scale, causal, off)
    of.backward(do.float())
    assert_close(dq, qf.grad, 2e-2, "dq")
    assert_close(dk, kf.grad, 2e-2, "dk")
    assert_close(dv, vf.grad, 2e-2, "dv")


@pytest.mark.parametrize("impl", ["tc", "fa2"])
@pytest.mark.parametrize("B,Sq,Sk,Hq,Hkv,causal", [
    (2, 256, 256, 4, 4, True), (1, 300, 300, 4, 2, True), (2, 128, 384, 6, 2, True), (1, 200, 333, 2, 1, False),
    (1, 1000, 1000, 2, 2, True),
])
def test_attention_fwd_impls(impl, B, Sq, Sk, Hq, Hkv, causal):
    D = 128
    q, k, v = bf(B, Sq, Hq, D, seed=5), bf(B, Sk, Hkv, D, seed=6), bf(B, Sk, Hkv, D, seed=7)
    off = Sk - Sq
    o, lse = F.attention(q, k, v, D ** -0.5, causal, off, impl=impl)
    o_r, lse_r = ref.attention(q, k, v, D ** -0.5, causal, off)
    assert_close(o, o_r, 1e-2, f"attention {impl}")
    assert_close(lse, lse_r, 1e-4, f"lse {impl}")


@pytest.mark.parametrize("impl", ["tc", "fa2"])
@pytest.mark.parametrize("B,Sq,Sk,Hq,Hkv,causal", [
    (2, 256, 256, 4, 4, True), (1, 300, 300, 4, 2, True), (2, 128, 384, 6, 2, True), (1, 200, 333, 2, 1, False),
    (1, 700, 700, 2, 2, True),
])
def test_attention_bwd_impls(impl, B, Sq, Sk, Hq, Hkv, causal):
    D = 128
    q, k, v = bf(B, Sq, Hq, D, seed=8), bf(B, Sk, Hkv, D, seed=9), bf(B, Sk, Hkv, D, seed=10)
    off = Sk - Sq
    o, lse = F.attention(q, k, v, D ** -0.5, causal, off)
    do = bf(B, Sq, Hq, D, seed=11)
    dq, dk, dv = F.attention_bwd(q, k, v, o, do, lse, D ** -0.5, causal, off, impl=impl)
    qf, kf, vf = (t.float().requires_grad_(True) for t in (q, k, v))
    of, _ = ref.attention(qf, kf, vf, D ** -0.5, causal, off)
    of.backward(do.float())
    assert_close(dq, qf.grad, 2e-2, f"dq {impl}")
    assert_close(dk, kf.grad, 2e-2, f"dk {impl}")
    assert_close(dv, vf.grad, 2e-2, f"dv {impl}")


def test_attention_packed_strided():
    """q/k/v as strided views of one packed qkv buffer (the model's layout)."""
    B, S, H, D = 2, 512, 4, 128
    qkv = bf(B, S, 3 * H * D)
    q = qkv[:, :, : H * D].view(B, S, H, D)
    k = qkv[:, :, H * D : 2 * H * D].view(B, S, H, D)
    v = qkv[:, :, 2 * H * D :].view(B, S, H, D)
    o, _ = F.attention(q, k, v, 1 / math.sqrt(D), True)
    o_r, _ = ref.attention(q, k, v, 1 / math.sqrt(D), True)
    assert_close(o, o_r, 1e-2, "packed attention")


@pytest.fixture
def pair_gemm():
    """Every GEMM of M, N >= 256 on the CTA-pair (cta_group::2) kernel."""
    old = _ext.C().gemm_pair_mode(1)
    yield
    _ext.C().gemm_pair_mode(old)


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True), (True, False)])
@pytest.mark.parametrize("M,N,K", [(256, 256, 64), (312, 520, 200), (1000, 776, 328), (2048, 1536, 1024)])
def test_gemm_pair_layouts(pair_gemm, a_mn, b_mn, M, N, K):
    a = bf(K, M, seed=1) if a_mn else bf(M, K, seed=1)
    b = bf(K, N, seed=2) if b_mn else bf(N, K, seed=2)
    out = F.gemm(a, b, a_mn=a_mn, b_mn=b_mn)
    assert_close(out, ref.gemm(a, b, a_mn, b_mn), 1e-2, f"pair gemm a_mn={a_mn} b_mn={b_mn} {M}x{N}x{K}")


def test_gemm_pair_epilogues(pair_gemm):
    M, N, K = 520, 1032, 264
    a, b = bf(M, K, seed=3), bf(N, K, seed=4)
    bias, res = bf(N, seed=5), bf(M, N, seed=6)
    out = F.gemm(a, b, bias=bias, residual=res, alpha=0.5)
    assert_close(out, ref.gemm(a, b, bias=bias, residual=res, alpha=0.5), 1e-2, "pair gemm epilogue")
    acc0 = torch.randn(M, N, device=dev)
    acc = acc0.clone()
    F.gemm(a, b, out=acc, accumulate=True)
    assert_close(acc, acc0 + ref.gemm(a, b), 1e-3, "pair gemm fp32 accumulate")
    f32 = F.gemm(a, b, out_dtype=torch.float32)
    assert_close(f32, ref.gemm(a, b), 1e-4, "pair gemm fp32 out")
    # a problem with more 256 x 256 tiles than SM pairs: every pair walks several tiles
    a, b = bf(4096, 512, seed=7), bf(3072, 512, seed=8)
    out = F.gemm(a, b)
    idx = torch.arange(0, 4096, 61, device=dev)
    assert_close(out[idx], ref.gemm(a[idx], b), 1e-2, "pair gemm persistent")


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True)])
def test_gemm_one_cta_large(a_mn, b_mn):
    """The one-CTA kernel on a problem the default would give to the pair kernel."""
    old = _ext.C().gemm_pair_mode(0)
    try:
        M, N, K = 1536, 1280, 520
        a = bf(K, M, seed=9) if a_mn else bf(M, K, seed=9)
        b = bf(K, N, seed=10) if b_mn else bf(N, K, seed=10)
        out = F.gemm(a, b, a_mn=a_mn, b_mn=b_mn)
        assert_close(out, ref.gemm(a, b, a_mn, b_mn), 1e-2, f"one-CTA gemm a_mn={a_mn} b_mn={b_mn}")
    finally:
        _ext.C().gemm_pair_mode(old)
