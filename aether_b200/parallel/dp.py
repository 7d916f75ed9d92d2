"""Data parallelism with ZeRO-1 sharding of the optimiser.

The reference DP (trainer/src/dp.rs:1-169) computes on the CPU, copies every
gradient to the device, all-reduces the full fp32 vector and runs identical
AdamW on every rank. Here each rank owns 1/world of the flat arena:

    grads (fp32, flat)  --reduce-scatter-->  shard grad (sum)
    AdamW on the shard (gradient scaled by 1/world inside the kernel)
    bf16 shard          --all-gather------>  full bf16 compute copy

so optimiser state and optimiser traffic shrink by the world size. The
collectives run on NCCL here; ``fused_dp.py`` provides the single-kernel
NVLink version of reduce-scatter + AdamW.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..optim import FlatAdamW


class DataParallel:
    def __init__(self, arena, info, lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, max_grad_norm=0.0,
                 group=None):
        self.arena = arena
        self.info = info
        self.group = group
        self.world = info.world
        self.rank = info.rank
        assert arena.numel % max(1, self.world) == 0, "arena must be padded to a multiple of the world size"
        self.shard_len = arena.numel // self.world
        self.start = self.rank * self.shard_len
        self.end = self.start + self.shard_len
        self.opt = FlatAdamW(arena, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay,
                             max_grad_norm=max_grad_norm, shard=(self.start, self.end))
        self.grad_shard = torch.empty(self.shard_len, dtype=torch.float32, device=arena.device) if self.world > 1 else None

    def broadcast_params(self) -> None:
        if self.world > 1:
            dist.broadcast(self.arena.master, src=0, group=self.group)
            self.arena.sync_bf16_from_master()

    def step(self, lr: float | None = None) -> None:
        a = self.arena
        if self.world == 1:
            self.opt.step(lr=lr)
            return
        dist.reduce_scatter_tensor(self.grad_shard, a.grad, op=dist.ReduceOp.SUM, group=self.group)
        self.opt.step(lr=lr, grad=self.grad_shard, gscale=1.0 / self.world)
        shard_bf16 = a.bf16[self.start : self.end]
        dist.all_gather_into_tensor(a.bf16, shard_bf16, group=self.group)
