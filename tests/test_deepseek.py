"""DeepSeek-V2 family: absorbed multi-head latent attention against the
standard (decompressed) MLA oracle, YaRN tables, DeepSeek MoE routing; CPU
and the GPU kernels."""
import math

import pytest
import torch

from aether_b200.models.deepseek import DeepSeekConfig, DeepSeekModel, yarn_rope_tables
from aether_b200.ops import functional as F

TINY = dict(vocab=256, d_model=128, n_layers=2, n_heads=4, d_ff=256, first_dense=1, n_experts=8, top_k=2,
            d_expert=64, n_shared=1, max_seq=64, init_std=0.05, yarn_factor=4.0, yarn_orig_ctx=16,
            yarn_mscale=0.707, yarn_mscale_all_dim=0.707)


def test_yarn_tables():
    plain = DeepSeekConfig(**dict(TINY, yarn_factor=0.0))
    c0, s0 = yarn_rope_tables(plain, 8)
    assert torch.allclose(c0[:, 0], torch.cos(torch.arange(8.0)), atol=1e-6)
    cfg = DeepSeekConfig(**TINY)
    c, s = yarn_rope_tables(cfg, 64)
    # the highest frequency keeps its original rate, the lowest is divided by the factor
    assert torch.allclose(c[:, 0], c0[:, 0].new_tensor(torch.cos(torch.arange(64.0)).tolist()), atol=1e-5)
    inv_last = 10000.0 ** (-(62 / 64))
    assert torch.allclose(s[:8, -1], torch.sin(torch.arange(8.0) * inv_last / 4.0), atol=1e-6)
    assert cfg.softmax_scale() > 1 / math.sqrt(192)


@pytest.mark.parametrize("kw", [dict(), dict(q_lora_rank=64, router="sigmoid", norm_topk=True, routed_scale=1.8)])
def test_mla_model_matches_oracle_cpu(kw):
    cfg = DeepSeekConfig(**dict(TINY, **kw))
    m = DeepSeekModel(cfg, device="cpu", seed=1, max_batch=2, max_seq=64)
    toks = torch.randint(0, 256, (2, 9), generator=torch.Generator().manual_seed(2))
    _, logits = m.prefill(toks, return_logits=True)
    ref = m.reference_logits(toks)[:, -1]
    err = float((logits - ref).norm() / ref.norm())
    assert err < 3e-2, err
    out = m.generate(toks, 3, use_graph=False)
    full = torch.cat([toks, out[:, :1]], 1)
    ref2 = m.reference_logits(full)[:, -1]
    _, l2 = DeepSeekModel(cfg, device="cpu", seed=1, max_batch=2, max_seq=64).prefill(full, return_logits=True)
    assert float((l2 - ref2).norm() / ref2.norm()) < 3e-2


def test_sigmoid_route_cpu():
    lg = torch.randn(5, 8, generator=torch.Generator().manual_seed(0))
    idx, wt = F.moe_route(lg, 3, sigmoid=True, renorm=True, scale=2.0)
    want = torch.topk(torch.sigmoid(lg), 3, -1)
    assert torch.equal(idx.long(), want.indices)
    assert torch.allclose(wt, 2.0 * want.values / want.values.sum(-1, keepdim=True), atol=1e-6)


@pytest.mark.gpu
@pytest.mark.parametrize("H,splits", [(16, 1), (16, 4), (20, 3), (4, 1)])
def test_gpu_mla_attention_matches_cpu(H, splits):
    g = torch.Generator().manual_seed(H + splits)
    N = 5
    cache = (torch.randn(3, 300, 576, generator=g) * 0.5).bfloat16()
    q = (torch.randn(N, H, 576, generator=g) * 0.5).bfloat16()
    slot = torch.tensor([0, 2, 1, 0, 2], dtype=torch.int32)
    seqlen = torch.tensor([300, 1, 65, 128, 200], dtype=torch.int32)
    out = torch.empty(N, H, 512, dtype=torch.bfloat16)
    F.mla_attention(q, cache, slot, seqlen, out, 0.07)
    og = torch.empty(N, H, 512, dtype=torch.bfloat16, device="cuda")
    F.mla_attention(q.cuda(), cache.cuda(), slot.cuda(), seqlen.cuda(), og, 0.07, splits=splits)
    err = float((og.float().cpu() - out.float()).norm() / out.float().norm())
    assert err < 1e-2, err


@pytest.mark.gpu
def test_gpu_mla_prep_and_sigmoid_route():
    g = torch.Generator().manual_seed(7)
    T, H = 6, 4
    kv_a = torch.randn(T, 576, generator=g).bfloat16()
    q = torch.randn(T, H * 192, generator=g).bfloat16()
    w = torch.rand(512, generator=g) + 0.5
    pos = torch.tensor([0, 1, 2, 5, 9, 3], dtype=torch.int32)
    slot = torch.tensor([0, 0, 0, 1, 1, 2], dtype=torch.int32)
    cfg = DeepSeekConfig(**TINY)
    cos, sin = yarn_rope_tables(cfg, 16)
    outs = []
    for dev in ("cpu", "cuda"):
        cache = torch.zeros(3, 16, 576, dtype=torch.bfloat16, device=dev)
        q_abs = torch.zeros(T, H, 576, dtype=torch.bfloat16, device=dev)
        F.mla_prep(kv_a.to(dev), w.to(dev), 1e-6, q.to(dev), H, 192, 128, pos.to(dev), slot.to(dev), cos.to(dev),
                   sin.to(dev), cache, q_abs)
        outs.append((cache.float().cpu(), q_abs.float().cpu()))
    assert torch.allclose(outs[0][0], outs[1][0], atol=2e-2, rtol=2e-2)
    assert torch.allclose(outs[0][1], outs[1][1], atol=2e-2, rtol=2e-2)
    lg = torch.randn(33, 64, generator=g)
    ic, wc = F.moe_route(lg, 6, sigmoid=True, renorm=True, scale=1.8)
    ig, wg = F.moe_route(lg.cuda(), 6, sigmoid=True, renorm=True, scale=1.8)
    assert torch.equal(ig.cpu(), ic) and torch.allclose(wg.cpu(), wc, atol=1e-5)


@pytest.mark.gpu
@pytest.mark.parametrize("kw", [dict(n_heads=16), dict(n_heads=4, q_lora_rank=64, router="sigmoid", norm_topk=True)])
def test_gpu_mla_model_prefill_and_graph_decode(kw):
    cfg = DeepSeekConfig(**dict(TINY, d_model=256, **kw))
    m = DeepSeekModel(cfg, device="cuda", seed=1, max_batch=2, max_seq=64)
    toks = torch.randint(0, 256, (2, 20), generator=torch.Generator().manual_seed(2)).cuda()
    _, logits = m.prefill(toks, return_logits=True)
    ref = m.reference_logits(toks)[:, -1]
    assert float((logits - ref).norm() / ref.norm()) < 3e-2
    eager = m.generate(toks, 6, use_graph=False)
    graph = m.generate(toks, 6, use_graph=True)
    assert float((eager == graph).float().mean()) > 0.9


def test_deepseek_gguf_roundtrip(tmp_path):
    """A deepseek2 GGUF written with llama.cpp tensor names and interleaved
    RoPE rows loads back into the same model (same logits)."""
    from aether_b200.formats import gguf as G

    cfg = DeepSeekConfig(**dict(TINY, q_lora_rank=64, router="sigmoid", norm_topk=True, routed_scale=1.5))
    m = DeepSeekModel(cfg, device="cpu", seed=3, max_batch=2, max_seq=64)
    w = m.w
    inv = torch.argsort(G._rope_rows_to_halves(64))  # back to interleaved rows

    def unfix_q(wq):
        v = wq.view(cfg.n_heads, cfg.qk_head, -1)
        return torch.cat([v[:, : cfg.qk_nope], v[:, cfg.qk_nope :][:, inv]], 1).reshape(wq.shape)

    T = {"token_embd.weight": w.embed, "output_norm.weight": w.final_norm, "output.weight": w.lm_head}
    for i in range(cfg.n_layers):
        p = f"blk.{i}."
        T[p + "attn_norm.weight"] = w.attn_norm[i]
        T[p + "ffn_norm.weight"] = w.mlp_norm[i]
        T[p + "attn_q_a.weight"] = w.wq_a[i]
        T[p + "attn_q_a_norm.weight"] = w.q_a_norm[i]
        T[p + "attn_q_b.weight"] = unfix_q(w.wq_b[i])
        T[p + "attn_kv_a_mqa.weight"] = torch.cat([w.wkv_a[i][:512], w.wkv_a[i][512:][inv]])
        T[p + "attn_kv_a_norm.weight"] = w.kv_norm[i]
        T[p + "attn_kv_b.weight"] = torch.cat([w.w_uk[i], w.w_uv[i]], 1).reshape(-1, 512)
        T[p + "attn_output.weight"] = w.wo[i]
        if i < cfg.first_dense:
            g_, u_ = w.dense_gu[i].chunk(2)
            T[p + "ffn_gate.weight"], T[p + "ffn_up.weight"], T[p + "ffn_down.weight"] = g_, u_, w.dense_d[i]
        else:
            T[p + "ffn_gate_inp.weight"] = w.router[i][: cfg.n_experts]
            g_, u_ = w.exp_gu[i].chunk(2, 1)
            T[p + "ffn_gate_exps.weight"], T[p + "ffn_up_exps.weight"] = g_, u_
            T[p + "ffn_down_exps.weight"] = w.exp_d[i]
            g_, u_ = w.sh_gu[i].chunk(2)
            T[p + "ffn_gate_shexp.weight"], T[p + "ffn_up_shexp.weight"] = g_, u_
            T[p + "ffn_down_shexp.weight"] = w.sh_d[i]
    a = "deepseek2."
    meta = {"general.architecture": "deepseek2", a + "block_count": cfg.n_layers, a + "embedding_length": 128,
            a + "feed_forward_length": cfg.d_ff, a + "attention.head_count": cfg.n_heads,
            a + "attention.q_lora_rank": 64, a + "attention.kv_lora_rank": 512, a + "attention.key_length": 192,
            a + "attention.value_length": 128, a + "rope.dimension_count": 64, a + "leading_dense_block_count": 1,
            a + "expert_count": 8, a + "expert_used_count": 2, a + "expert_feed_forward_length": 64,
            a + "expert_shared_count": 1, a + "expert_gating_func": 2, a + "expert_weights_norm": True,
            a + "expert_weights_scale": 1.5, a + "rope.freq_base": 10000.0, a + "rope.scaling.type": "yarn",
            a + "rope.scaling.factor": 4.0, a + "rope.scaling.original_context_length": 16,
            a + "rope.scaling.yarn_log_multiplier": 0.0707, a + "attention.layer_norm_rms_epsilon": 1e-6}
    path = str(tmp_path / "ds.gguf")
    G.write_gguf(path, meta, {k: (v, G.F32) for k, v in T.items()})
    cfg2, w2 = G.load_deepseek_weights(path, device="cpu")
    assert (cfg2.q_lora_rank, cfg2.router, cfg2.routed_scale, cfg2.n_shared) == (64, "sigmoid", 1.5, 1)
    assert abs(cfg2.yarn_mscale_all_dim - 0.707) < 1e-4 and cfg2.yarn_factor == 4.0
    m2 = DeepSeekModel(cfg2, device="cpu", max_batch=2, max_seq=64, weights=w2)
    toks = torch.randint(0, 256, (2, 7), generator=torch.Generator().manual_seed(5))
    _, l1 = m.prefill(toks, return_logits=True)
    _, l2 = m2.prefill(toks, return_logits=True)
    assert float((l1 - l2).norm() / l1.norm()) < 1e-2


def test_engine_serves_mla_model_cpu():
    """The continuous-batching engine drives the MLA model (prefill per slot, batched decode)."""
    from aether_b200.serving.engine import Engine
    from aether_b200.serving.sampling import SamplingParams
    from aether_b200.serving.tokenizer import ByteTokenizer

    cfg = DeepSeekConfig(**TINY)
    m = DeepSeekModel(cfg, device="cpu", seed=1, max_batch=2, max_seq=64)
    eng = Engine(m, ByteTokenizer(), max_concurrent=2, use_graph=False)
    try:
        rs = [eng.submit(list(b"hello"), SamplingParams(max_tokens=4)),
              eng.submit(list(b"abc"), SamplingParams(max_tokens=3, temperature=0.7, seed=1))]
        for r in rs:  # each request streams its tokens, then None
            while r.out.get(timeout=120) is not None:
                pass
        assert len(rs[0].tokens) == 4 and len(rs[1].tokens) == 3
        want = m.generate(torch.tensor([list(b"hello")]), 4, use_graph=False)[0].tolist()
        assert rs[0].tokens == want
    finally:
        eng.shutdown()


def _tp_worker(rank, world, port, kw, q):
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

    cfg = DeepSeekConfig(**dict(TINY, **kw))
    m = DeepSeekModel(cfg, device="cpu", seed=1, max_batch=2, max_seq=64, tp=GlooTP())
    toks = torch.randint(0, 256, (2, 9), generator=torch.Generator().manual_seed(2))
    _, logits = m.prefill(toks, return_logits=True)
    nxt = m.generate(toks, 3, use_graph=False)
    q.put((rank, logits, nxt))
    dist.destroy_process_group()


@pytest.mark.parametrize("kw", [dict(), dict(q_lora_rank=64, router="sigmoid", norm_topk=True)])
def test_mla_tensor_parallel_matches_one_rank_cpu(kw):
    """Heads, experts and FFN slices over 2 gloo ranks give the single-rank logits."""
    import multiprocessing as mp
    import socket

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_tp_worker, args=(r, 2, port, kw, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = {r: (lg, nx) for r, lg, nx in (q.get(timeout=300) for _ in ps)}
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    cfg = DeepSeekConfig(**dict(TINY, **kw))
    m = DeepSeekModel(cfg, device="cpu", seed=1, max_batch=2, max_seq=64)
    toks = torch.randint(0, 256, (2, 9), generator=torch.Generator().manual_seed(2))
    _, ref = m.prefill(toks, return_logits=True)
    for r in (0, 1):
        lg, nx = got[r]
        assert float((lg - ref).norm() / ref.norm()) < 3e-2, r
    assert torch.equal(got[0][1], got[1][1])  # ranks agree on the generated tokens
