"""Paged KV cache: page allocator (reference counts, prefix sharing, LRU
reuse), paged decode/prefill against the contiguous cache on CPU, and on the
GPU the paged kernels (KV append through the page table, split-K decode
attention reading pages) against the contiguous ones."""
import pytest
import torch

from aether_b200.models.qwen import QwenConfig, QwenModel
from aether_b200.ops import functional as F
from aether_b200.serving.engine import Engine
from aether_b200.serving.kv import NoPages, PageAllocator, prefix_keys
from aether_b200.serving.sampling import SamplingParams
from aether_b200.serving.tokenizer import ByteTokenizer

TINY = dict(vocab=300, d_model=128, n_layers=2, n_heads=2, n_kv_heads=1, d_ff=256, max_seq=128, init_std=0.08)


def test_page_allocator_refcounts_prefix_and_lru():
    a = PageAllocator(5, 4, reserved=1)
    p1, p2 = a.allocate(), a.allocate()
    assert {p1, p2} <= {1, 2, 3, 4} and a.available() == 2
    a.register(p1, "k1")
    assert a.lookup("k1") == p1 and a.ref[p1] == 2 and a.hits == 1
    a.release(p1)
    a.release(p1)  # now cached (keyed), not free
    assert a.available() == 3 and "k1" in a.cached
    assert a.lookup("k1") == p1  # a later request still hits it
    a.release(p1)
    a.release(p2)  # unkeyed -> straight back to the free list
    got = [a.allocate() for _ in range(4)]
    assert sorted(got) == [1, 2, 3, 4] and "k1" not in a.key_page  # the cached page was evicted last
    with pytest.raises(NoPages):
        a.allocate()


def test_prefix_keys_chain():
    k1 = prefix_keys([1, 2, 3, 4, 5, 6, 7, 8, 9], 4)
    k2 = prefix_keys([1, 2, 3, 4, 5, 6, 7, 8, 0], 4)
    k3 = prefix_keys([0, 2, 3, 4, 5, 6, 7, 8], 4)  # same second page, different history
    assert len(k1) == 2 and k1 == k2 and k3[1] != k1[1]


def test_paged_generate_matches_contiguous_cpu():
    cfg = QwenConfig(**TINY)
    a = QwenModel(cfg, device="cpu", seed=2, max_batch=2, max_seq=64)
    b = QwenModel(cfg, device="cpu", seed=2, max_batch=2, max_seq=64, kv_pages=16, page_size=8)
    prompts = torch.randint(0, 300, (2, 13), generator=torch.Generator().manual_seed(1))
    assert torch.equal(a.generate(prompts, 6, use_graph=False), b.generate(prompts, 6, use_graph=False))


def _engine_outputs(model, prompts, n):
    eng = Engine(model, ByteTokenizer(), max_concurrent=2, eos_ids=[], use_graph=model.device.type == "cuda")
    outs = []
    for p in prompts:  # one after another, so the second can hit the first one's cached pages
        r = eng.submit(p, SamplingParams(max_tokens=n))
        outs.append(list(eng.stream(r, timeout=120)))
    eng.shutdown()
    assert not eng.errors, eng.errors
    return outs, eng


def _prefix_prompts():
    g = torch.Generator().manual_seed(3)
    shared = torch.randint(0, 300, (21,), generator=g).tolist()
    return [shared + [5, 6, 7], shared + [9]]


def test_engine_prefix_sharing_cpu():
    cfg = QwenConfig(**TINY)
    prompts = _prefix_prompts()
    want, _ = _engine_outputs(QwenModel(cfg, device="cpu", seed=4, max_batch=2, max_seq=64), prompts, 5)
    paged = QwenModel(cfg, device="cpu", seed=4, max_batch=2, max_seq=64, kv_pages=20, page_size=8)
    got, eng = _engine_outputs(paged, prompts, 5)
    assert got == want
    assert eng.metrics.counters.get("prefix_cached_tokens", 0) == 16  # two full pages of the shared 21 tokens


@pytest.mark.gpu
def test_gpu_paged_kernels_match_contiguous():
    g = torch.Generator(device="cuda").manual_seed(0)
    B, Hq, Hkv, D, P, S = 3, 8, 2, 128, 16, 200
    npages = (S + P - 1) // P
    Tq = (Hq + 2 * Hkv) * D
    kc = torch.zeros(B, 256, Hkv, D, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    kp = torch.zeros(B * npages + 1, P, Hkv, D, dtype=torch.bfloat16, device="cuda")
    vp = torch.zeros_like(kp)
    perm = torch.randperm(B * npages, generator=torch.Generator().manual_seed(0)) + 1  # scattered pages
    table = perm.view(B, npages).to(torch.int32).cuda()
    cos, sin = torch.rand(256, D // 2, device="cuda"), torch.rand(256, D // 2, device="cuda")
    qkv = torch.randn(B * S, Tq, device="cuda", generator=g).bfloat16()
    pos = torch.arange(S, dtype=torch.int32, device="cuda").repeat(B)
    slot = torch.arange(B, dtype=torch.int32, device="cuda").repeat_interleave(S)
    q1, q2 = qkv.clone(), qkv.clone()
    F.rope_kv_append(q1, pos, slot, cos, sin, kc, vc, Hq, Hkv, D)
    F.rope_kv_append(q2, pos, slot, cos, sin, kp, vp, Hq, Hkv, D, page_table=table)
    assert torch.equal(q1, q2)
    for b in range(B):
        assert torch.equal(F.gather_kv(kp, b, S, table), kc[b, :S])
        assert torch.equal(F.gather_kv(vp, b, S, table), vc[b, :S])
    q = torch.randn(B, Hq * D, device="cuda", generator=g).bfloat16()
    seqlen = torch.tensor([S, 37, 129], dtype=torch.int32, device="cuda")
    rows = torch.arange(B, dtype=torch.int32, device="cuda")
    o1 = torch.empty(B, Hq * D, dtype=torch.bfloat16, device="cuda")
    o2 = torch.empty_like(o1)
    cnt = torch.zeros(B * Hkv, dtype=torch.int32, device="cuda")
    F.decode_attention(q, kc, vc, rows, seqlen, o1, Hq, D ** -0.5, splits=4, counters=cnt)
    F.decode_attention(q, kp, vp, rows, seqlen, o2, Hq, D ** -0.5, splits=4, counters=cnt, page_table=table)
    assert torch.equal(o1, o2)


@pytest.mark.gpu
def test_gpu_engine_paged_prefix_sharing():
    cfg = QwenConfig(**dict(TINY, d_model=256, n_heads=2, n_kv_heads=1, d_ff=512))
    prompts = _prefix_prompts()
    want, _ = _engine_outputs(QwenModel(cfg, device="cuda", seed=4, max_batch=2, max_seq=128), prompts, 6)
    paged = QwenModel(cfg, device="cuda", seed=4, max_batch=2, max_seq=128, kv_pages=24, page_size=8)
    got, eng = _engine_outputs(paged, prompts, 6)
    agree = sum(int(a == b) for x, y in zip(got, want) for a, b in zip(x, y))
    assert agree >= 0.9 * 12, (got, want)
    assert eng.metrics.counters.get("prefix_cached_tokens", 0) == 16
