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


def test_permute_expert_range_cpu():
    """Expert parallelism: the pairs of experts [e0, e0 + E) are permuted, the rest get row -1."""
    g = torch.Generator().manual_seed(3)
    idx, wt = F.moe_route(torch.randn(13, 8, generator=g), 2)
    row_of, src_row, tile_group = F.moe_permute(idx, 4, 4)
    flat = idx.view(-1)
    for i, r in enumerate(row_of.tolist()):
        e = int(flat[i])
        if e < 4:
            assert r == -1
        else:
            assert int(src_row[r]) == i // 2 and int(tile_group[r // 128]) == e - 4
    Y = torch.randn(src_row.numel(), 16).bfloat16()
    out = F.moe_combine(Y, row_of, wt)
    want = torch.zeros(13, 16)
    for i, r in enumerate(row_of.tolist()):
        if r >= 0:
            want[i // 2] += float(wt.view(-1)[i]) * Y[r].float()
    assert torch.allclose(out.float(), want, atol=2e-2)


def _ep_worker(rank, world, port, q):
    import os

    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=world)

    class GlooTP:
        def __init__(self):
            self.rank, self.world = rank, world

        def all_reduce_(self, t):
            f = t.float()
            dist.all_reduce(f)
            t.copy_(f)
            return t

    cfg = MoEConfig(**dict(TINY, n_heads=2, n_kv_heads=2))
    m = MoEQwenModel(cfg, device="cpu", seed=1, max_batch=2, max_seq=64, tp=GlooTP())
    toks = torch.randint(0, 256, (2, 11), generator=torch.Generator().manual_seed(2))
    _, logits = m.prefill(toks, return_logits=True)
    q.put((rank, logits))
    dist.destroy_process_group()


def test_expert_parallel_matches_one_rank_cpu():
    """Experts split over 2 gloo ranks (with the TP-sharded attention and shared
    expert) give the single-rank logits."""
    import multiprocessing as mp
    import socket

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_ep_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=300) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    cfg = MoEConfig(**dict(TINY, n_heads=2, n_kv_heads=2))
    m = MoEQwenModel(cfg, device="cpu", seed=1, max_batch=2, max_seq=64)
    toks = torch.randint(0, 256, (2, 11), generator=torch.Generator().manual_seed(2))
    _, ref = m.prefill(toks, return_logits=True)
    for r in (0, 1):
        err = float((got[r] - ref).norm() / ref.norm())
        assert err < 3e-2, (r, err)


@pytest.mark.gpu
def test_gpu_permute_expert_range_and_combine():
    g = torch.Generator().manual_seed(4)
    T, E, k, d, N = 41, 8, 2, 128, 64
    idx, wt = F.moe_route(torch.randn(T, E, generator=g).cuda(), k)
    x = (torch.randn(T, d, generator=g) * 0.5).bfloat16().cuda()
    w = (torch.randn(E, N, d, generator=g) * 0.05).bfloat16().cuda()
    full = torch.zeros(T, N, device="cuda")
    for e0, e1 in ((0, 3), (3, 8)):
        row_of, src_row, tile_group = F.moe_permute(idx, e1 - e0, e0)
        flat = idx.view(-1)
        local = (flat >= e0) & (flat < e1)
        assert bool(((row_of >= 0) == local).all())
        Y = F.gemm_grouped(F.moe_gather(x, src_row), w[e0:e1].contiguous(), tile_group)
        full += F.moe_combine(Y, row_of, wt).float()
    row_of, src_row, tile_group = F.moe_permute(idx, E)
    want = F.moe_combine(F.gemm_grouped(F.moe_gather(x, src_row), w, tile_group), row_of, wt).float()
    assert float((full - want).norm() / want.norm()) < 1e-2
