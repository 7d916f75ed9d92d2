"""LoRA / QLoRA: adapter gradients against torch autograd of the same formula,
zero initial update, training moves only the adapters, merge reproduces the
adapted model, quantised base (Q8_0/Q4_0) GPU kernels agree byte-for-byte with
the CPU quantiser, and LoRA training on the GPU matches the CPU path."""
import pytest
import torch

from aether_b200.models.gpt import GPT, GPTConfig
from aether_b200.models.lora import LoRAConfig, LoRAGPT, LoRALinearFn
from aether_b200.ops import functional as F
from aether_b200.parallel import dist as D
from aether_b200.train import Trainer

TINY = dict(vocab=128, d_model=64, n_layers=2, n_heads=2, n_kv_heads=2, d_ff=128, max_seq=32)


def _param(t):
    t = t.detach().clone().to(torch.bfloat16).requires_grad_(True)
    t.main_grad = torch.zeros(t.shape, dtype=torch.float32)
    return t


def test_lora_linear_grads_match_autograd():
    g = torch.Generator().manual_seed(0)
    T, K, N, r, s = 24, 64, 48, 8, 2.0
    x = torch.randn(T, K, generator=g).bfloat16()
    w = (torch.randn(N, K, generator=g) * 0.1).bfloat16()
    a = _param(torch.randn(r, K, generator=g) * 0.1)
    b = _param(torch.randn(N, r, generator=g) * 0.1)
    res = torch.randn(T, N, generator=g).bfloat16()
    dy = torch.randn(T, N, generator=g).bfloat16()
    xr = x.clone().requires_grad_(True)
    y = LoRALinearFn.apply(xr, a, b, res, w, s)
    y.backward(dy)
    # fp32 autograd of the same function
    xf = x.float().requires_grad_(True)
    af = a.detach().float().requires_grad_(True)
    bf = b.detach().float().requires_grad_(True)
    yf = xf @ w.float().t() + s * (xf @ af.t()) @ bf.t() + res.float()
    yf.backward(dy.float())
    assert (y.float() - yf).abs().max() < 0.05
    assert torch.allclose(xr.grad.float(), xf.grad, atol=0.05, rtol=0.02)
    assert torch.allclose(a.main_grad, af.grad, atol=0.05, rtol=0.02)
    assert torch.allclose(b.main_grad, bf.grad, atol=0.05, rtol=0.02)


def _batch(seed):
    return torch.randint(0, 128, (4, 17), generator=torch.Generator().manual_seed(seed))


def test_lora_gpt_trains_only_adapters_and_merges():
    base = GPT(GPTConfig(**TINY), device="cpu", seed=1)
    w0 = base.arena.master.clone()
    toks = _batch(0)
    ids, tgt = toks[:, :-1].contiguous(), toks[:, 1:].contiguous()
    with torch.no_grad():
        l0 = float(base.loss(ids, tgt))
    m = LoRAGPT(base, LoRAConfig(rank=8, alpha=16.0), seed=3)
    with torch.no_grad():
        assert abs(float(m.loss(ids, tgt)) - l0) < 1e-6  # B = 0: the update starts at exactly zero
    tr = Trainer(m, D.DistInfo(), lr=1e-2, weight_decay=0.0, micro_batch=4)
    first = float(tr.train_step(toks))
    for _ in range(15):
        last = float(tr.train_step(toks))
    assert last < first - 0.3, (first, last)
    assert torch.equal(base.arena.master, w0)  # the base never moves
    with torch.no_grad():
        adapted = base.logits(ids).float()
        m.merge()
        base._linear = GPT._linear.__get__(base)  # plain base forward, adapters folded in
        merged = base.logits(ids).float()
    assert (adapted - merged).abs().max() < 0.05 * adapted.abs().max()


def test_qlora_cpu_close_to_bf16_base():
    toks = _batch(1)
    ids, tgt = toks[:, :-1].contiguous(), toks[:, 1:].contiguous()
    ref = LoRAGPT(GPT(GPTConfig(**TINY), device="cpu", seed=1), LoRAConfig(rank=8), seed=3)
    q8 = LoRAGPT(GPT(GPTConfig(**TINY), device="cpu", seed=1), LoRAConfig(rank=8), seed=3, quant="q8_0")
    with torch.no_grad():
        a, b = float(ref.loss(ids, tgt)), float(q8.loss(ids, tgt))
    assert abs(a - b) < 0.02 * a and q8.base_bytes_saved > 0


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", [F.Q8_0, F.Q4_0])
@pytest.mark.parametrize("shape", [(96, 256), (37, 96)])  # whole 32-block warp spans; a ragged last span
def test_gpu_block_quant_matches_cpu(fmt, shape):
    x = (torch.randn(*shape, generator=torch.Generator().manual_seed(0)) * 0.05).bfloat16()
    qc = F.quantize_blocks(x, fmt)
    qg = F.quantize_blocks(x.cuda(), fmt)
    assert torch.equal(qg.cpu(), qc)
    yc = F.dequantize_blocks(qc, x.shape, fmt)
    yg = F.dequantize_blocks(qg, x.shape, fmt)
    assert torch.equal(yg.cpu(), yc)


@pytest.mark.gpu
@pytest.mark.parametrize("quant", [None, "q4_0"])
def test_gpu_lora_matches_cpu(quant):
    cfg = GPTConfig(vocab=512, d_model=256, n_layers=2, n_heads=2, n_kv_heads=2, d_ff=512, max_seq=128)
    toks = torch.randint(0, 512, (2, 129), generator=torch.Generator().manual_seed(1))
    ids, tgt = toks[:, :-1].contiguous(), toks[:, 1:].contiguous()
    out = []
    for dev in ("cuda", "cpu"):
        m = LoRAGPT(GPT(cfg, device=dev, seed=3), LoRAConfig(rank=16), seed=5, quant=quant)
        with torch.no_grad():  # give B a nonzero value so dA is exercised
            m.arena.master.copy_(torch.randn(m.arena.numel, generator=torch.Generator().manual_seed(7)) * 0.01)
            m.arena.sync_bf16_from_master()
        loss = m.loss(ids.to(dev), tgt.to(dev))
        loss.backward()
        out.append((float(loss), m.arena.grad.float().cpu()))
    (lg, gg), (lc, gc) = out
    assert abs(lg - lc) < 2e-2 * abs(lc)
    assert float((gg - gc).norm() / gc.norm()) < 5e-2
