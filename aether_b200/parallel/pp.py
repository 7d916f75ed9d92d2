"""Pipeline parallelism: 1F1B schedule with point-to-point activation and
gradient transfers over torch.distributed (NCCL on GPUs, gloo on CPU).

Reference: trainer/src/pipeline.rs -- ``trait Stage {forward, backward, step}``
(:180) and ``run_1f1b`` (:199-290): rank r runs (world-1-r) warm-up forwards,
then alternates one forward and one backward, then drains the remaining
backwards; activations travel device -> host -> TCP -> host -> device. Here
activations and gradients stay on the GPU and move with NCCL isend / irecv
(a rank's send overlaps its next compute, and every receive is posted one
micro-batch ahead); the schedule and the stage contract are the same.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..optim import FlatAdamW


class GPTPipelineStage:
    """One stage of a GPT model: its layer range, the embedding on the first
    stage and the final norm + LM head + loss on the last."""

    def __init__(self, cfg, rank: int, world: int, device, seed: int = 0, lr: float = 3e-4, weight_decay: float = 0.1,
                 betas=(0.9, 0.95)):
        from ..models.gpt import GPT

        L = cfg.n_layers
        bounds = [round(L * i / world) for i in range(world + 1)]
        self.layers = list(range(bounds[rank], bounds[rank + 1]))
        self.rank, self.world = rank, world
        self.first, self.last = rank == 0, rank == world - 1
        self.model = GPT(cfg, device=device, seed=seed, layers=self.layers, first=self.first, last=self.last)
        self.opt = FlatAdamW(self.model.arena, lr=lr, betas=betas, weight_decay=weight_decay)
        self.device = torch.device(device)
        self.cfg = cfg

    def forward(self, ids, targets, x_in, loss_scale):
        B, S = targets.shape
        if self.last:
            return self.model.loss(ids if self.first else None, targets, loss_scale, x=x_in)
        return self.model.forward_hidden(ids if self.first else None, x=x_in, B=B, S=S)

    def step(self, lr=None):
        self.opt.step(lr=lr)

    def zero_grad(self):
        self.model.arena.zero_grad()


def run_1f1b(stage: GPTPipelineStage, batches: list, group=None) -> torch.Tensor | None:
    """One optimiser step over ``batches`` (a list of (ids [b, S], targets [b, S])
    micro-batches, identical on every rank). Returns the summed loss on the last
    stage (None elsewhere). Gradients accumulate in the stage's arena."""
    rank, world = stage.rank, stage.world
    n = len(batches)
    d = stage.cfg.d_model
    dev = stage.device
    act_dtype = stage.model.arena.bf16.dtype  # activations travel in the compute dtype
    n_tok = sum(t.numel() for _, t in batches)
    loss_scale = 1.0 / n_tok
    inputs, outputs = {}, {}
    pending = []
    total = torch.zeros((), dtype=torch.float32, device=dev)
    prev, nxt = rank - 1, rank + 1

    # Receives are posted one micro-batch ahead (irecv), so the transfer of the
    # next activation / gradient overlaps the compute of the current one. Per
    # peer the posts stay in schedule order, matching the sender's isends.
    posted = {}

    def post(kind, i):
        if i >= n or (kind, i) in posted or (stage.first if kind == "x" else stage.last):
            return
        t = torch.empty(batches[i][1].numel(), d, dtype=act_dtype, device=dev)
        posted[(kind, i)] = (t, dist.irecv(t, src=prev if kind == "x" else nxt, group=group))

    def take(kind, i):
        post(kind, i)
        t, work = posted.pop((kind, i))
        work.wait()
        return t

    def fwd(i):
        ids, tgt = batches[i]
        ids, tgt = ids.to(dev), tgt.to(dev)
        x = None
        if not stage.first:
            x = take("x", i)
            post("x", i + 1)
            x.requires_grad_(True)
            inputs[i] = x
        out = stage.forward(ids, tgt, x, loss_scale)
        outputs[i] = out
        if not stage.last:
            pending.append(dist.isend(out.detach().contiguous(), dst=nxt, group=group))

    def bwd(i):
        nonlocal total
        out = outputs.pop(i)
        if stage.last:
            out.backward()
            total = total + out.detach()
        else:
            g = take("g", i)
            post("g", i + 1)
            out.backward(g)
        if not stage.first:
            x = inputs.pop(i)
            pending.append(dist.isend(x.grad.contiguous(), dst=prev, group=group))

    warm = min(world - 1 - rank, n)
    for i in range(warm):
        fwd(i)
    for i in range(n - warm):
        fwd(warm + i)
        bwd(i)
    for i in range(n - warm, n):
        bwd(i)
    for h in pending:
        h.wait()
    return total if stage.last else None
