"""GPT model: CPU training converges; on the GPU the native path matches the
fp32 CPU path on loss and gradients (same random init)."""
import pytest
import torch

from aether_b200.models.gpt import GPT, GPTConfig
from aether_b200.parallel import dist as D
from aether_b200.train import Trainer
from tests.util import rel_err

TINY = dict(vocab=256, d_model=128, n_layers=2, n_heads=2, n_kv_heads=1, d_ff=256, max_seq=64)


def test_cpu_training_loss_falls():
    cfg = GPTConfig(**TINY)
    m = GPT(cfg, device="cpu", seed=0)
    tr = Trainer(m, D.DistInfo(), lr=3e-3, weight_decay=0.0, micro_batch=2)
    g = torch.Generator().manual_seed(0)
    tokens = torch.randint(0, 256, (4, 33), generator=g)
    first = float(tr.train_step(tokens))
    for _ in range(25):
        last = float(tr.train_step(tokens))
    assert first > 5.0 and last < first - 2.0, (first, last)


def test_param_count_24l():
    cfg = GPTConfig.gpt_24l()
    assert 1.3e9 < cfg.n_params() < 1.45e9


@pytest.mark.gpu
def test_gpu_matches_cpu_grads():
    cfg = GPTConfig(vocab=512, d_model=256, n_layers=2, n_heads=2, n_kv_heads=2, d_ff=512, max_seq=128)
    gm = GPT(cfg, device="cuda", seed=3)
    cm = GPT(cfg, device="cpu", seed=3)
    tokens = torch.randint(0, 512, (2, 129), generator=torch.Generator().manual_seed(1))
    ids, tgt = tokens[:, :-1].contiguous(), tokens[:, 1:].contiguous()
    lg = gm.loss(ids.cuda(), tgt.cuda())
    lg.backward()
    lc = cm.loss(ids, tgt)
    lc.backward()
    assert abs(float(lg) - float(lc)) < 2e-2 * abs(float(lc))
    for name in gm.arena.names():
        a = gm.arena[name].main_grad.cpu()
        b = cm.arena[name].main_grad
        assert rel_err(a, b) < 8e-2, name


@pytest.mark.gpu
def test_gpu_training_step_decreases_loss():
    cfg = GPTConfig(vocab=1024, d_model=256, n_layers=2, n_heads=2, n_kv_heads=2, d_ff=512, max_seq=256)
    m = GPT(cfg, device="cuda", seed=0)
    tr = Trainer(m, D.DistInfo(device=torch.device("cuda")), lr=2e-3, weight_decay=0.0, micro_batch=2)
    tokens = torch.randint(0, 1024, (4, 257), device="cuda")
    l0 = float(tr.train_step(tokens))
    for _ in range(10):
        l1 = float(tr.train_step(tokens))
    assert l1 < l0 - 1.0, (l0, l1)
