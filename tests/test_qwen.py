"""Qwen2 serving path: prefill + CUDA-graph greedy decode against an fp32
eager forward of the same random weights (top-1 agreement and logits)."""
import pytest
import torch

from aether_b200.models.qwen import QwenConfig, QwenModel
from aether_b200.ops import functional as F

TINY = dict(vocab=1024, d_model=256, n_layers=2, n_heads=4, n_kv_heads=2, d_ff=512, max_seq=256, init_std=0.05)


def test_cpu_prefill_matches_reference():
    cfg = QwenConfig(**TINY)
    m = QwenModel(cfg, device="cpu", seed=0, max_batch=2, max_seq=128)
    toks = torch.randint(0, cfg.vocab, (2, 16), generator=torch.Generator().manual_seed(0))
    nxt = m.prefill(toks)
    ref = m.reference_logits(toks)[:, -1].argmax(-1)
    assert torch.equal(nxt.cpu(), ref.cpu())


def test_cpu_decode_matches_full_forward():
    cfg = QwenConfig(**TINY)
    m = QwenModel(cfg, device="cpu", seed=1, max_batch=2, max_seq=128)
    toks = torch.randint(0, cfg.vocab, (2, 12), generator=torch.Generator().manual_seed(1))
    out = m.generate(toks, 4, use_graph=False)
    seq = torch.cat([toks, out[:, :3]], dim=1)
    ref = m.reference_logits(seq)[:, -1].argmax(-1)
    assert torch.equal(out[:, 3], ref)


@pytest.mark.gpu
def test_gpu_prefill_and_graph_decode():
    cfg = QwenConfig(**dict(TINY, d_model=512, n_heads=4, n_kv_heads=2, d_ff=1024))
    m = QwenModel(cfg, device="cuda", seed=2, max_batch=8, max_seq=256)
    toks = torch.randint(0, cfg.vocab, (3, 40), device="cuda")
    out_g = m.generate(toks, 6, use_graph=True)
    m2 = QwenModel(cfg, device="cuda", seed=2, max_batch=8, max_seq=256)
    out_e = m2.generate(toks, 6, use_graph=False)
    assert torch.equal(out_g, out_e)
    seq = torch.cat([toks, out_g[:, :5]], dim=1)
    logits = m.reference_logits(seq)[:, -1]
    top = logits.argmax(-1)
    agree = (top == out_g[:, 5]).float().mean().item()
    assert agree >= 2 / 3, (top, out_g[:, 5])


@pytest.mark.gpu
def test_gpu_skinny_gemm_and_decode_attention():
    from aether_b200.ops import reference as ref
    for M in (1, 2, 3, 4, 7, 16, 33, 64):
        x = torch.randn(M, 3584, device="cuda").bfloat16()
        w = torch.randn(1000, 3584, device="cuda").bfloat16()
        acc = torch.zeros(M, 1024, device="cuda")
        F.skinny_gemm(x, w, acc)
        r = x.float() @ w.float().t()
        err = (acc[:, :1000] - r).norm() / r.norm()
        assert err < 1e-3, (M, float(err))
        y = torch.empty(M, 1000, dtype=torch.bfloat16, device="cuda")
        b = torch.randn(1000, device="cuda").bfloat16()
        F.skinny_finalize(acc, y, bias=b)
        assert float((y.float() - (r + b.float())).norm() / r.norm()) < 1e-2
        assert float(acc.abs().max()) == 0.0
    B, Hq, Hkv, D, S = 3, 28, 4, 128, 700
    kc = torch.randn(B + 1, 1024, Hkv, D, device="cuda").bfloat16()
    vc = torch.randn(B + 1, 1024, Hkv, D, device="cuda").bfloat16()
    q = torch.randn(B, Hq * D, device="cuda").bfloat16()
    slot = torch.tensor([2, 0, 1], dtype=torch.int32, device="cuda")
    seqlen = torch.tensor([S, 1, 129], dtype=torch.int32, device="cuda")
    out = torch.empty(B, Hq * D, dtype=torch.bfloat16, device="cuda")
    F.decode_attention(q, kc, vc, slot, seqlen, out, Hq, D ** -0.5, splits=8)
    for bi in range(B):
        L, s = int(seqlen[bi]), int(slot[bi])
        o, _ = ref.attention(q[bi].view(1, 1, Hq, D), kc[s, :L][None], vc[s, :L][None], D ** -0.5, causal=False)
        e = (out[bi].float() - o.reshape(-1)).norm() / o.norm()
        assert e < 1e-2, (bi, float(e))


@pytest.mark.gpu
def test_gpu_fused_gemm_epilogues_match_separate_kernels():
    """The decode GEMMs that finish QKV (bias + RoPE + KV append) and SwiGLU
    inside their tiles give the same caches, activations and tokens as the
    GEMM + finalize-kernel path, on contiguous and paged caches and at batch
    sizes that exercise one and several 16-row MMA columns."""
    from aether_b200.ops import reference as ref

    # fused-epilogue GEMMs against the separate kernels, one call each
    for M in (1, 5, 33):
        Hq, Hkv, D, K = 4, 2, 128, 512
        x = torch.randn(M, K, device="cuda").bfloat16()
        w = (torch.randn((Hq + 2 * Hkv) * D, K, device="cuda") * 0.05).bfloat16()
        bias = torch.randn((Hq + 2 * Hkv) * D, device="cuda").bfloat16()
        cos, sin = ref.rope_tables(64, D, 1e4, device="cuda")
        pos = torch.randint(0, 64, (M,), dtype=torch.int32, device="cuda")
        slot = torch.randperm(M + 1, device="cuda")[:M].int()
        outs = []
        for fused in (True, False):
            kc = torch.zeros(M + 1, 64, Hkv, D, dtype=torch.bfloat16, device="cuda")
            vc = torch.zeros_like(kc)
            qkv = torch.zeros(M, (Hq + 2 * Hkv) * D, dtype=torch.bfloat16, device="cuda")
            acc = torch.zeros(M, (Hq + 2 * Hkv) * D, device="cuda")
            tiles = torch.zeros(64, dtype=torch.int32, device="cuda")
            if fused:
                F.skinny_gemm_qkv(x, w, acc, tiles, bias, qkv, pos, slot, cos.contiguous(), sin.contiguous(), kc, vc,
                                  Hq, Hkv)
                assert int(tiles.abs().sum()) == 0 and float(acc.abs().max()) == 0.0
            else:
                F.skinny_gemm(x, w, acc)
                F.qkv_finalize_rope(acc, bias, qkv, pos, slot, cos.contiguous(), sin.contiguous(), kc, vc, Hq, Hkv, D)
            outs.append((qkv, kc, vc))
        for a, b in zip(*outs):
            assert float((a.float() - b.float()).abs().max()) <= 2e-2 * float(b.float().abs().max()) + 1e-6
        Fh = 192
        wgu = (torch.randn(2 * Fh, K, device="cuda") * 0.05).bfloat16()
        acc = torch.zeros(M, 2 * Fh, device="cuda")
        tiles = torch.zeros(64, dtype=torch.int32, device="cuda")
        act = torch.empty(M, Fh, dtype=torch.bfloat16, device="cuda")
        F.skinny_gemm_swiglu(x, wgu, acc, act, tiles)
        z = x.float() @ wgu.float().t()
        want = torch.nn.functional.silu(z[:, :Fh]) * z[:, Fh:]
        assert float((act.float() - want).norm() / want.norm()) < 1e-2
        assert int(tiles.abs().sum()) == 0 and float(acc.abs().max()) == 0.0
    # and the whole decode step with and without them (contiguous and paged caches)
    cfg = QwenConfig(**dict(TINY, d_model=512, n_heads=4, n_kv_heads=2, d_ff=1024))
    toks = torch.randint(0, cfg.vocab, (3, 40), device="cuda")
    for pages in (0, 64):
        m1 = QwenModel(cfg, device="cuda", seed=2, max_batch=8, max_seq=256, kv_pages=pages)
        m2 = QwenModel(cfg, device="cuda", seed=2, max_batch=8, max_seq=256, kv_pages=pages)
        m1.fused_epilogues, m2.fused_epilogues = True, False
        m1.mega = m2.mega = False  # exercise the kernel chain (the one-kernel step has its own tests)
        assert torch.equal(m1.generate(toks, 8), m2.generate(toks, 8))


QWEN3 = dict(TINY, qkv_bias=False, qk_norm=True, head_dim_=128, tie_embeddings=False)  # head_dim != d / H


def _random_qk_norms(m, seed):
    g = torch.Generator().manual_seed(seed)
    for lst in (m.w.q_norm, m.w.k_norm):
        for t in lst:
            t.copy_((1 + 0.3 * torch.randn(t.shape, generator=g)).to(t.dtype))


def test_cpu_qwen3_qk_norm_decode_matches_full_forward():
    cfg = QwenConfig(**QWEN3)
    m = QwenModel(cfg, device="cpu", seed=3, max_batch=2, max_seq=128)
    _random_qk_norms(m, 0)
    toks = torch.randint(0, cfg.vocab, (2, 10), generator=torch.Generator().manual_seed(4))
    nxt, logits = m.prefill(toks, return_logits=True)
    ref = m.reference_logits(toks)[:, -1]
    assert float((logits - ref).norm() / ref.norm()) < 2e-2
    out = m.generate(toks, 4, use_graph=False)
    seq = torch.cat([toks, out[:, :3]], dim=1)
    assert torch.equal(out[:, 3], m.reference_logits(seq)[:, -1].argmax(-1))


def test_model_family_presets():
    for cfg, params in ((QwenConfig.qwen3_8b(), 8.19e9), (QwenConfig.llama3_8b(), 8.03e9),
                        (QwenConfig.mistral_7b(), 7.24e9)):
        assert abs(cfg.n_params() - params) / params < 0.02, (cfg, cfg.n_params())


@pytest.mark.gpu
def test_gpu_qwen3_qk_norm_graph_decode():
    cfg = QwenConfig(**QWEN3)
    m = QwenModel(cfg, device="cuda", seed=3, max_batch=4, max_seq=256)
    _random_qk_norms(m, 0)
    toks = torch.randint(0, cfg.vocab, (2, 24), generator=torch.Generator().manual_seed(5)).cuda()
    _, logits = m.prefill(toks, return_logits=True)
    ref = m.reference_logits(toks)[:, -1]
    assert float((logits - ref).norm() / ref.norm()) < 3e-2
    out_g = m.generate(toks, 5, use_graph=True)
    out_e = m.generate(toks, 5, use_graph=False)
    assert float((out_g == out_e).float().mean()) > 0.9


def test_shard_of_full_weights_equals_random_init_shard():
    """QwenWeights.shard of the unsplit weights gives the same tensors as the
    random-init TP shard (the path checkpoints take into TP serving)."""
    from aether_b200.models.qwen import QwenConfig, QwenWeights

    cfg = QwenConfig(vocab=256, d_model=128, n_layers=2, n_heads=4, n_kv_heads=2, d_ff=256, max_seq=32)
    full = QwenWeights(cfg, "cpu", seed=5)
    for r in range(2):
        a = QwenWeights(cfg, "cpu", seed=5, tp_rank=r, tp_size=2)
        b = QwenWeights.shard(full, r, 2, "cpu")
        for name in ("wqkv", "bqkv", "wo", "wgu", "wd"):
            for x, y in zip(getattr(a, name), getattr(b, name)):
                assert (x is None and y is None) or torch.equal(x, y), (r, name)
        assert (a.hq, a.hkv, a.f) == (b.hq, b.hkv, b.f)
