"""Host-side logic of the backward-overlapped data-parallel engine: the
per-bucket chunking of the flat arena, and the gradient-ready hooks of the GPT
model (each fires once per backward, in backward order, when its bucket's
gradients are already final). The device path is checked against the NCCL
engine by the multi-GPU worker."""
import torch

from aether_b200.models.gpt import GPT, GPTConfig
from aether_b200.parallel.dp import bucket_chunks

CFG = GPTConfig(vocab=256, d_model=64, n_layers=3, n_heads=2, n_kv_heads=2, d_ff=128, max_seq=32)


def _bucket_ranges(arena):
    # world 1: every bucket is one chunk covering the whole bucket
    return {k: (b, e) for k, (b, e, _) in bucket_chunks(arena, 1, 0).items()}


def test_buckets_cover_the_arena_in_backward_order():
    m = GPT(CFG, device="cpu", seed=0, pad_multiple=4)
    full = _bucket_ranges(m.arena)
    assert list(full) == ["head", "l2", "l1", "l0", "embed"]
    spans = sorted(full.values())
    assert spans[0][0] == 0 and spans[-1][1] == m.arena.numel
    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))


def test_bucket_chunks_partition_every_bucket():
    m = GPT(CFG, device="cpu", seed=0, pad_multiple=8)
    full = _bucket_ranges(m.arena)
    for world in (1, 2, 3, 4, 8):
        per_rank = [bucket_chunks(m.arena, world, r) for r in range(world)]
        for k, (b, e) in full.items():
            cover = sorted((c[k][0], c[k][1]) for c in per_rank if c[k][1] > c[k][0])
            assert cover[0][0] == b and cover[-1][1] == e, (world, k)
            assert all(x[1] == y[0] for x, y in zip(cover, cover[1:])), (world, k)
            assert all(x[0] % 128 == 0 for x in cover)
        for c in per_rank:  # state offsets pack the chunks back to back
            offs = [(o, ce - cb) for cb, ce, o in c.values()]
            assert [o for o, _ in offs] == [sum(n for _, n in offs[:i]) for i in range(len(offs))]


def test_grad_ready_hooks_fire_in_backward_order_with_final_gradients():
    m = GPT(CFG, device="cpu", seed=1)
    a = m.arena
    ranges = _bucket_ranges(a)
    seen = []
    snap = {}

    def ready(key):
        b, e = ranges[key]
        seen.append(key)
        snap[key] = a.grad[b:e].clone()

    m.grad_ready_hook = ready
    toks = torch.randint(0, CFG.vocab, (2, 17), generator=torch.Generator().manual_seed(3))
    a.zero_grad()
    loss = m.loss(toks[:, :-1].contiguous(), toks[:, 1:].contiguous())
    loss.backward()
    assert seen == ["head", "l2", "l1", "l0"]  # the embedding is final only when backward returns
    for k in seen:
        b, e = ranges[k]
        assert torch.equal(snap[k], a.grad[b:e]), k
        assert float(a.grad[b:e].abs().sum()) > 0, k
