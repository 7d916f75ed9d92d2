"""AdamW over the flat fp32 master buffer of a ParamArena.

Reference: the decoupled AdamW of runtime/src/cuda.rs:6924-6942
(p -= lr * (m_hat / (sqrt(v_hat) + eps) + wd * p)), the global-norm clip of
trainer/src/model.rs:686 and the warmup+cosine schedule of
trainer/src/main.rs:159-163. The arena is split into a weight-decay range and
a no-decay range per contiguous run of slots, so an update is a handful of
launches that each stream p/g/m/v and write the bf16 compute copy.

``shard`` (start, end) restricts the update to one data-parallel shard
(ZeRO-1); optimiser state is then only allocated for that range.
"""
from __future__ import annotations

import math

import torch

from ..ops import functional as F


def cosine_lr(step: int, base_lr: float, warmup: int, total: int, min_ratio: float = 0.1) -> float:
    if warmup > 0 and step < warmup:
        return base_lr * (step + 1) / warmup
    if total <= warmup:
        return base_lr
    prog = min(1.0, (step - warmup) / max(1, total - warmup))
    return base_lr * (min_ratio + (1 - min_ratio) * 0.5 * (1 + math.cos(math.pi * prog)))


def _runs(mask: torch.Tensor, start: int, end: int):
    """Contiguous runs [(a, b, value)] of a bool mask over [start, end)."""
    m = mask[start:end]
    if m.numel() == 0:
        return []
    change = torch.nonzero(m[1:] != m[:-1]).flatten().tolist()
    bounds = [0] + [c + 1 for c in change] + [m.numel()]
    return [(start + a, start + b, bool(m[a])) for a, b in zip(bounds[:-1], bounds[1:])]


class FlatAdamW:
    def __init__(self, arena, lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, max_grad_norm=0.0,
                 shard: tuple[int, int] | None = None):
        self.arena = arena
        self.lr = lr
        self.beta1, self.beta2 = betas
        self.eps = eps
        self.wd = weight_decay
        self.max_grad_norm = max_grad_norm
        self.start, self.end = shard if shard is not None else (0, arena.numel)
        n = self.end - self.start
        self.m = torch.zeros(n, dtype=torch.float32, device=arena.device)
        self.v = torch.zeros(n, dtype=torch.float32, device=arena.device)
        self.runs = _runs(arena.decay_mask, self.start, self.end)
        self.step_count = 0

    def step(self, lr: float | None = None, grad: torch.Tensor | None = None, gscale: float = 1.0,
             gscale_tensor: torch.Tensor | None = None) -> None:
        """grad: the gradient for [start, end) (defaults to the arena's)."""
        self.step_count += 1
        lr = self.lr if lr is None else lr
        a = self.arena
        g_all = grad if grad is not None else a.grad[self.start : self.end]
        for s, e, decay in self.runs:
            o = s - self.start
            F.adamw_(a.master[s:e], g_all[o : o + (e - s)], self.m[o : o + (e - s)], self.v[o : o + (e - s)],
                     a.bf16[s:e], lr=lr, beta1=self.beta1, beta2=self.beta2, eps=self.eps,
                     wd=self.wd if decay else 0.0, step=self.step_count, gscale=gscale, gscale_tensor=gscale_tensor)

    def state_dict(self) -> dict:
        return {"m": self.m.cpu(), "v": self.v.cpu(), "step": self.step_count, "shard": (self.start, self.end)}

    def load_state_dict(self, sd: dict) -> None:
        self.m.copy_(sd["m"].to(self.m.device))
        self.v.copy_(sd["v"].to(self.v.device))
        self.step_count = int(sd["step"])
