"""Flex attention (sliding window, logit softcap, per-layer window pattern):
the CPU oracle against explicit truncation, the model against its fp32
reference, and the GPU kernels (tcgen05 / mma.sync prefill, split-K decode)
against the oracle."""
import math

import pytest
import torch

from aether_b200.models.qwen import QwenConfig, QwenModel
from aether_b200.ops import functional as F
from aether_b200.ops import reference as ref


def _qkv(B, Sq, Sk, Hq, Hkv, D, seed=0, device="cpu"):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Sq, Hq, D, generator=g).bfloat16()
    k = torch.randn(B, Sk, Hkv, D, generator=g).bfloat16()
    v = torch.randn(B, Sk, Hkv, D, generator=g).bfloat16()
    return q.to(device), k.to(device), v.to(device)


def test_window_equals_truncated_context():
    """Row i with window W attends to exactly keys (i - W, i]."""
    q, k, v = _qkv(1, 12, 12, 2, 1, 16)
    W = 4
    o, _ = ref.attention(q, k, v, 0.25, True, 0, W)
    for i in (0, 3, 7, 11):
        lo = max(0, i - W + 1)
        oi, _ = ref.attention(q[:, i : i + 1], k[:, lo : i + 1], v[:, lo : i + 1], 0.25, False)
        assert torch.allclose(o[:, i], oi[:, 0], atol=1e-5)


def test_softcap_bounds_logits():
    q, k, v = _qkv(1, 4, 4, 1, 1, 16)
    q = q * 50  # large logits
    _, lse_c = ref.attention(q, k, v, 1.0, False, 0, 0, 5.0)
    assert bool((lse_c <= 5.0 + math.log(4) + 1e-4).all())  # every capped logit <= 5


def test_layer_window_pattern():
    cfg = QwenConfig(n_layers=6, sliding_window=512, sliding_window_pattern=3, rope_theta_swa=1e4)
    assert [cfg.layer_window(i)[0] for i in range(6)] == [512, 512, 0, 512, 512, 0]
    assert cfg.layer_window(0)[1] == 1e4 and cfg.layer_window(2)[1] == cfg.rope_theta
    assert QwenConfig.mistral_7b_v01().layer_window(5) == (4096, 1e4)


FLEX = dict(vocab=256, d_model=128, n_layers=3, n_heads=2, n_kv_heads=1, d_ff=256, max_seq=64, init_std=0.05,
            sliding_window=5, sliding_window_pattern=3, rope_theta_swa=1e4, attn_softcap=20.0)


def test_flex_model_cpu():
    m = QwenModel(QwenConfig(**FLEX), device="cpu", seed=1, max_batch=2, max_seq=64)
    toks = torch.randint(0, 256, (2, 13), generator=torch.Generator().manual_seed(2))
    _, logits = m.prefill(toks, return_logits=True)
    ref_l = m.reference_logits(toks)[:, -1]
    assert float((logits - ref_l).norm() / ref_l.norm()) < 3e-2
    # decode one token and compare with the reference over the extended sequence
    nxt = m.generate(toks, 2, use_graph=False)
    full = torch.cat([toks, nxt[:, :1]], 1)
    want = m.reference_logits(full)[:, -1].argmax(-1)
    assert float((want == nxt[:, 1]).float().mean()) >= 0.5


@pytest.mark.gpu
@pytest.mark.parametrize("D,impl", [(128, "tc"), (128, "fa2"), (64, "fa2")])
@pytest.mark.parametrize("window,softcap", [(0, 30.0), (100, 0.0), (37, 15.0)])
def test_gpu_prefill_flex(D, impl, window, softcap):
    q, k, v = _qkv(2, 300, 300, 4, 2, D, seed=3, device="cuda")
    o, lse = F.attention(q, k, v, 1 / math.sqrt(D), True, 0, impl=impl, window=window, softcap=softcap)
    ro, _ = ref.attention(q.cpu(), k.cpu(), v.cpu(), 1 / math.sqrt(D), True, 0, window, softcap)
    err = float((o.float().cpu() - ro).norm() / ro.norm())
    assert err < 2e-2, err


@pytest.mark.gpu
@pytest.mark.parametrize("window,softcap", [(0, 30.0), (64, 0.0), (300, 10.0)])
def test_gpu_decode_flex(window, softcap):
    B, Hq, Hkv, D, L = 3, 8, 2, 128, 700
    g = torch.Generator().manual_seed(5)
    kc = torch.randn(B + 1, 1024, Hkv, D, generator=g).bfloat16().cuda()
    vc = torch.randn(B + 1, 1024, Hkv, D, generator=g).bfloat16().cuda()
    q = torch.randn(B, Hq * D, generator=g).bfloat16().cuda()
    slot = torch.tensor([2, 0, 1], dtype=torch.int32, device="cuda")
    seqlen = torch.tensor([L, 65, 1], dtype=torch.int32, device="cuda")
    out = torch.empty(B, Hq * D, dtype=torch.bfloat16, device="cuda")
    for splits in (1, 8):
        F.decode_attention(q, kc, vc, slot, seqlen, out, Hq, 1 / math.sqrt(D), splits=splits, window=window,
                           softcap=softcap)
        want = torch.empty_like(out).cpu()
        F.decode_attention(q.cpu(), kc.cpu(), vc.cpu(), slot.cpu(), seqlen.cpu(), want, Hq, 1 / math.sqrt(D),
                           window=window, softcap=softcap)
        err = float((out.float().cpu() - want.float()).norm() / want.float().norm())
        assert err < 2e-2, (splits, err)


@pytest.mark.gpu
def test_gpu_flex_model_prefill_and_graph_decode():
    cfg = QwenConfig(**dict(FLEX, d_model=256, n_heads=2, n_kv_heads=1))
    m = QwenModel(cfg, device="cuda", seed=1, max_batch=2, max_seq=64)
    toks = torch.randint(0, 256, (2, 20), generator=torch.Generator().manual_seed(2)).cuda()
    _, logits = m.prefill(toks, return_logits=True)
    ref_l = m.reference_logits(toks)[:, -1]
    assert float((logits - ref_l).norm() / ref_l.norm()) < 3e-2
    eager = m.generate(toks, 6, use_graph=False)
    graph = m.generate(toks, 6, use_graph=True)
    assert float((eager == graph).float().mean()) > 0.9


def _fp32_grads(q, k, v, do, scale, window, softcap):
    qf, kf, vf = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    o, _ = ref.attention(qf, kf, vf, scale, True, 0, window, softcap)
    return torch.autograd.grad(o, (qf, kf, vf), do.float())


@pytest.mark.parametrize("window,softcap", [(0, 30.0), (48, 0.0), (33, 15.0)])
def test_backward_flex_cpu(window, softcap):
    """The CPU path of attention_bwd is autograd through the fp32 oracle with
    the same window / softcap."""
    q, k, v = _qkv(1, 40, 40, 2, 1, 16, seed=5)
    do = torch.randn(1, 40, 2, 16, generator=torch.Generator().manual_seed(6)).bfloat16()
    o, lse = F.attention(q, k, v, 0.25, True, window=window, softcap=softcap)
    dq, dk, dv = F.attention_bwd(q, k, v, o, do, lse, 0.25, True, window=window, softcap=softcap)
    for got, want in zip((dq, dk, dv), _fp32_grads(q, k, v, do, 0.25, window, softcap)):
        assert float((got.float() - want).norm() / want.norm()) < 2e-2


@pytest.mark.gpu
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("window,softcap", [(0, 30.0), (96, 0.0), (77, 20.0)])
def test_gpu_backward_flex(D, window, softcap):
    """Training backward with a sliding window and / or soft-capped logits (the
    mma.sync kernel) against fp32 autograd through the oracle: GQA 4:2, a
    ragged key count."""
    q, k, v = _qkv(2, 200, 200, 4, 2, D, seed=7, device="cuda")
    do = torch.randn(2, 200, 4, D, generator=torch.Generator().manual_seed(8)).bfloat16().cuda()
    scale = D ** -0.5
    o, lse = F.attention(q, k, v, scale, True, window=window, softcap=softcap)
    dq, dk, dv = F.attention_bwd(q, k, v, o, do, lse, scale, True, window=window, softcap=softcap)
    torch.cuda.synchronize()
    for name, got, want in zip("qkv", (dq, dk, dv), _fp32_grads(q, k, v, do, scale, window, softcap)):
        err = float((got.float() - want).norm() / want.norm())
        assert err < 2e-2, (name, err)
