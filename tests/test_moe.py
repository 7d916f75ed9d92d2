"""Mixture-of-experts: routing, expert permutation and the grouped GEMM
against plain references, and an MoE decoder's prefill / decode against the
fp32 per-token reference (CPU, and the tcgen05 path on the GPU)."""
import pytest
import torch

from aether_b200.models.moe import MoEConfig, MoEQwenModel
from aether_b200.ops import functional as F

TINY = dict(vocab=256, d_model=128, n_layers=2, n_heads=2, n_kv_heads=1, d_ff=8, max_seq=64, init_std=0.05,
            n_experts=6, top_k=2, d_expert=64, shared_ff=128)


def test_route_and_permute_cpu():
    g = torch.Generator().manual_seed(0)
    logits = torch.randn(9, 6, generator=g)
    idx, wt = F.moe_route(logits, 2, softmax_all=True, renorm=True)
    assert torch.allclose(wt.sum(-1), torch.ones(9))
    row_of, src_row, tile_group = F.moe_permute(idx, 6)
    assert src_row.numel() % 128 == 0
    for i, r in enumerate(row_of.tolist()):
        assert int(src_row[r]) == i // 2 and int(tile_group[r // 128]) == int(idx.view(-1)[i])


@pytest.mark.parametrize("cfg_kw", [dict(), dict(shared_ff=0, router_softmax_all=False)])
def test_moe_model_matches_reference_cpu(cfg_kw):
    cfg = MoEConfig(**dict(TINY, **cfg_kw))
    m = MoEQwenModel(cfg, device="cpu", seed=1, max_batch=2, max_seq=64)
    toks = torch.randint(0, 256, (2, 11), generator=torch.Generator().manual_seed(2))
    _, logits = m.prefill(toks, return_logits=True)
    ref = m.reference_logits(toks)[:, -1]
    err = float((logits - ref).norm() / ref.norm())
    assert err < 3e-2, err
    out = m.generate(toks, 4, use_graph=False)
    assert out.shape == (2, 4)


@pytest.mark.gpu
def test_gpu_moe_kernels_match_cpu():
    g = torch.Generator().manual_seed(0)
    T, E, k, d, N = 37, 8, 2, 256, 192
    logits = torch.randn(T, E, generator=g)
    for softmax_all in (True, False):
        ic, wc = F.moe_route(logits, k, softmax_all, renorm=True)
        ig, wg = F.moe_route(logits.cuda(), k, softmax_all, renorm=True)
        assert torch.equal(ig.cpu(), ic) and torch.allclose(wg.cpu(), wc, atol=1e-5)
    x = (torch.randn(T, d, generator=g) * 0.5).bfloat16()
    w = (torch.randn(E, N, d, generator=g) * 0.05).bfloat16()
    row_of, src_row, tile_group = F.moe_permute(ig, E)
    X = F.moe_gather(x.cuda(), src_row)
    Y = F.gemm_grouped(X, w.cuda(), tile_group)
    wt = wg
    out = F.moe_combine(Y, row_of, wt)
    ref = torch.zeros(T, N)
    for t in range(T):
        for j in range(k):
            ref[t] += float(wt[t, j]) * (x[t].float() @ w[int(ig[t, j])].float().t())
    err = float((out.float().cpu() - ref).norm() / ref.norm())
    assert err < 1e-2, err


@pytest.mark.gpu
def test_gpu_moe_model_prefill_and_graph_decode():
    cfg = MoEConfig(**dict(TINY, d_model=256, n_heads=2, n_kv_heads=1, shared_ff=256))
    m = MoEQwenModel(cfg, device="cuda", seed=1, max_batch=2, max_seq=64)
    toks = torch.randint(0, 256, (2, 16), generator=torch.Generator().manual_seed(2)).cuda()
    _, logits = m.prefill(toks, return_logits=True)
    ref = m.reference_logits(toks)[:, -1]
    assert float((logits - ref).norm() / ref.norm()) < 3e-2
    eager = m.generate(toks, 6, use_graph=False)
    graph = m.generate(toks, 6, use_graph=True)
    assert float((eager == graph).float().mean()) > 0.9
