"""The GPT training model (with and without Qwen3 q/k norm) against a plain
fp32 PyTorch re-implementation of the same architecture on the same weights:
loss and every parameter gradient (CPU)."""
import math

import pytest
import torch

from aether_b200.models.gpt import GPT, GPTConfig
from aether_b200.ops import reference as ref


def _torch_loss(m: GPT, ids, tgt, params):
    cfg = m.cfg
    B, S = ids.shape
    D, Hq, Hkv = cfg.head_dim, cfg.n_heads, cfg.n_kv_heads
    g = Hq // Hkv
    rms = lambda x, w: x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + cfg.norm_eps) * w  # noqa: E731
    x = params["tok_emb"][ids.reshape(-1)]
    pos = torch.arange(S).repeat(B)
    for i in range(cfg.n_layers):
        h = rms(x, params[f"l{i}.attn_norm"])
        qkv = h @ params[f"l{i}.wqkv"].t()
        q, k, v = qkv[:, : Hq * D], qkv[:, Hq * D : (Hq + Hkv) * D], qkv[:, (Hq + Hkv) * D :]
        if cfg.qk_norm:
            q = rms(q.reshape(-1, Hq, D), params[f"l{i}.q_norm"]).reshape(-1, Hq * D)
            k = rms(k.reshape(-1, Hkv, D), params[f"l{i}.k_norm"]).reshape(-1, Hkv * D)
        qk = ref.rope(torch.cat([q, k], 1), pos, m.rope_cos, m.rope_sin, Hq + Hkv, D)
        q4 = qk[:, : Hq * D].reshape(B, S, Hq, D).transpose(1, 2)
        k4 = qk[:, Hq * D :].reshape(B, S, Hkv, D).transpose(1, 2).repeat_interleave(g, 1)
        v4 = v.reshape(B, S, Hkv, D).transpose(1, 2).repeat_interleave(g, 1)
        s = q4 @ k4.transpose(-1, -2) / math.sqrt(D)
        s = s.masked_fill(torch.ones(S, S, dtype=torch.bool).triu(1), float("-inf"))
        o = (torch.softmax(s, -1) @ v4).transpose(1, 2).reshape(B * S, Hq * D)
        x = x + o @ params[f"l{i}.wo"].t()
        h = rms(x, params[f"l{i}.mlp_norm"])
        gt, up = (h @ params[f"l{i}.wgu"].t()).chunk(2, -1)
        x = x + (torch.nn.functional.silu(gt) * up) @ params[f"l{i}.wd"].t()
    h = rms(x, params["final_norm"])
    logits = h @ params["lm_head"].t()
    return torch.nn.functional.cross_entropy(logits, tgt.reshape(-1))


@pytest.mark.parametrize("qk_norm", [False, True])
def test_gpt_matches_plain_torch(qk_norm):
    cfg = GPTConfig(vocab=96, d_model=64, n_layers=2, n_heads=4, n_kv_heads=2, d_ff=96, max_seq=32, qk_norm=qk_norm)
    m = GPT(cfg, device="cpu", seed=2)
    if qk_norm:  # non-trivial norm weights
        with torch.no_grad():
            for i in range(cfg.n_layers):
                for n in ("q_norm", "k_norm"):
                    m.arena.master_view(f"l{i}.{n}").uniform_(0.5, 1.5, generator=torch.Generator().manual_seed(i))
            m.arena.sync_bf16_from_master()
    toks = torch.randint(0, 96, (2, 17), generator=torch.Generator().manual_seed(3))
    ids, tgt = toks[:, :-1].contiguous(), toks[:, 1:].contiguous()
    loss = m.loss(ids, tgt)
    loss.backward()
    params = {n: m.arena[n].detach().float().clone().requires_grad_(True) for n in m.arena.names()}
    lr = _torch_loss(m, ids, tgt, params)
    lr.backward()
    assert abs(float(loss) - float(lr)) < 2e-3 * float(lr), (float(loss), float(lr))
    for n, p in params.items():
        s = m.arena.slots[n]
        g = m.arena.grad[s.offset : s.offset + s.numel].view(s.shape)
        err = float((g - p.grad).norm() / p.grad.norm().clamp(min=1e-12))
        assert err < 2e-2, (n, err)


@pytest.mark.gpu
def test_gpu_qk_norm_gpt_matches_plain_torch():
    """The q/k-norm path on the GPU kernels (head rows through the RMSNorm
    kernels, tcgen05 GEMMs and attention) against the fp32 re-implementation."""
    cfg = GPTConfig(vocab=256, d_model=256, n_layers=2, n_heads=2, n_kv_heads=1, d_ff=512, max_seq=128, qk_norm=True)
    m = GPT(cfg, device="cuda", seed=2)
    toks = torch.randint(0, 256, (2, 129), generator=torch.Generator().manual_seed(3))
    ids, tgt = toks[:, :-1].contiguous(), toks[:, 1:].contiguous()
    loss = m.loss(ids.cuda(), tgt.cuda())
    loss.backward()
    cpu = GPT(cfg, device="cpu", seed=2)
    params = {n: cpu.arena[n].detach().float().clone().requires_grad_(True) for n in cpu.arena.names()}
    lr = _torch_loss(cpu, ids, tgt, params)
    lr.backward()
    assert abs(float(loss) - float(lr)) < 1e-2 * float(lr)
    for n, p in params.items():
        s = m.arena.slots[n]
        g = m.arena.grad[s.offset : s.offset + s.numel].view(s.shape).float().cpu()
        assert float((g - p.grad).norm() / p.grad.norm().clamp(min=1e-12)) < 5e-2, n
