"""Data parallelism with ZeRO-1 sharding of the optimiser.

The reference DP (trainer/src/dp.rs:1-169) computes on the CPU, copies every
gradient to the device, all-reduces the full fp32 vector and runs identical
AdamW on every rank. Here each rank owns 1/world of the flat arena:

    grads (fp32, flat)  --reduce-scatter-->  shard grad (sum)
    AdamW on the shard (gradient scaled by 1/world inside the kernel)
    bf16 shard          --all-gather------>  full bf16 compute copy

Three implementations with the same interface:
  * ``DataParallel``       -- the baseline: NCCL reduce-scatter, AdamW kernel,
                              NCCL all-gather (gloo on CPU);
  * ``FusedDataParallel``  -- the arena's gradient and bf16 buffers live in
                              symmetric memory, and ONE kernel per step reduces
                              the shard across GPUs (NVLS multimem.ld_reduce or
                              P2P loads), applies AdamW, and writes the new bf16
                              parameters into every GPU's copy (multimem.st or
                              P2P stores), bracketed by two device barriers.
  * ``OverlappedDataParallel`` -- the same fused kernel per gradient bucket
                              (one bucket per layer, plus the head and the
                              embedding), launched on a side stream as soon as
                              the last micro-batch's backward has finished that
                              layer, so the reduction and the optimiser step of
                              layer i run under the backward of layers i-1..0.
                              Every bucket is split over all ranks (each rank
                              owns 1/world of every layer); the step ends with
                              one device barrier.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .._ext import C
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

    def _reduce_scatter(self) -> None:
        a = self.arena
        if a.grad.is_cuda:
            dist.reduce_scatter_tensor(self.grad_shard, a.grad, op=dist.ReduceOp.SUM, group=self.group)
        else:  # gloo has no reduce-scatter
            full = a.grad.clone()
            dist.all_reduce(full, group=self.group)
            self.grad_shard.copy_(full[self.start : self.end])

    def step(self, lr: float | None = None) -> None:
        a = self.arena
        if self.world == 1:
            self.opt.step(lr=lr)
            return
        self._reduce_scatter()
        self.opt.step(lr=lr, grad=self.grad_shard, gscale=1.0 / self.world)
        shard_bf16 = a.bf16[self.start : self.end].clone()
        if a.bf16.is_cuda:
            dist.all_gather_into_tensor(a.bf16, shard_bf16, group=self.group)
        else:
            parts = [torch.empty_like(shard_bf16) for _ in range(self.world)]
            dist.all_gather(parts, shard_bf16, group=self.group)
            a.bf16.copy_(torch.cat(parts))

    def state_dict(self) -> dict:
        return {"opt": self.opt.state_dict()}


class FusedDataParallel:
    """One-kernel DP step over symmetric memory (see module docstring).

    The model must be built with ``alloc=team_alloc(team)`` so its arena's
    gradient and bf16 buffers are symmetric."""

    def __init__(self, arena, team, lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1):
        self.arena, self.team = arena, team
        self.world, self.rank = team.world, team.rank
        self.lr, (self.beta1, self.beta2), self.eps, self.wd = lr, betas, eps, weight_decay
        assert arena.numel % (self.world * 128) == 0
        self.shard_len = arena.numel // self.world
        self.start = self.rank * self.shard_len
        self.end = self.start + self.shard_len
        dev = arena.device
        self.m = torch.zeros(self.shard_len, dtype=torch.float32, device=dev)
        self.v = torch.zeros(self.shard_len, dtype=torch.float32, device=dev)
        blocks = arena.decay_mask.view(-1, 128)[:, 0]
        self.decay_blocks = blocks.to(torch.uint8).to(dev)
        self.grad_buf = team.find(arena.grad)
        self.param_buf = team.find(arena.bf16)
        self.step_count = 0

    def broadcast_params(self) -> None:
        if self.world > 1:
            dist.broadcast(self.arena.master, src=0)
            self.arena.sync_bf16_from_master()

    def step(self, lr: float | None = None) -> None:
        self.step_count += 1
        a = self.arena
        gb, pb = self.grad_buf, self.param_buf
        self.team.barrier()  # every rank's gradient is final
        C().dp_reduce_adamw(gb.peers_dev, gb.mc_ptr, pb.peers_dev, pb.mc_ptr, a.master[self.start : self.end],
                            self.m, self.v, self.decay_blocks, self.start, self.shard_len, self.world,
                            float(lr if lr is not None else self.lr), self.beta1, self.beta2, self.eps, self.wd,
                            self.step_count, 1.0 / self.world, None)
        self.team.barrier()  # every rank's new parameters have landed everywhere

    def state_dict(self) -> dict:
        return {"m": self.m.cpu(), "v": self.v.cpu(), "step": self.step_count, "shard": (self.start, self.end)}


def team_alloc(team):
    """Allocator for ParamArena that places buffers in the team's symmetric memory."""

    def alloc(numel, dtype):
        return team.alloc(numel, dtype).tensor

    return alloc


def _bucket_key(name: str) -> str:
    head = name.split(".", 1)[0]
    if head.startswith("l") and head[1:].isdigit():
        return head
    return "embed" if name == "tok_emb" else "head"


def bucket_chunks(arena, world: int, rank: int) -> dict:
    """{bucket key: (arena begin, arena end, state offset)} of rank's chunk of
    every gradient bucket, in backward order of the keys (head, l{L-1} .. l0,
    embed follow from the arena order reversed). A bucket is a contiguous run
    of slots with the same key (the padding after the last slot belongs to the
    last bucket); it splits into ``world`` chunks of whole 128-element blocks,
    and the state offsets pack this rank's chunks back to back."""
    slots = sorted(arena.slots.values(), key=lambda s: s.offset)
    starts, keys = [], []
    for s in slots:
        k = _bucket_key(s.name)
        if not keys or keys[-1] != k:
            keys.append(k)
            starts.append(s.offset)
    assert len(set(keys)) == len(keys), "bucket members must be contiguous in the arena"
    ends = starts[1:] + [arena.numel]
    out, off = {}, 0
    for k, b, e in reversed(list(zip(keys, starts, ends))):
        chunk = -(-(e - b) // (world * 128)) * 128
        cb = min(e, b + rank * chunk)
        ce = min(e, cb + chunk)
        out[k] = (cb, ce, off)
        off += ce - cb
    return out


class OverlappedDataParallel:
    """Bucketed, backward-overlapped fused DP step (see module docstring).

    Use with a model that calls ``grad_ready(key)`` when a bucket's gradients
    are final (``GPT`` does, through the ``grad_ready_hook`` the Trainer
    installs with ``attach``): ``arm()`` before the last micro-batch's
    backward, ``step()`` after it. Buckets are contiguous arena ranges in
    backward order: the head (final norm + LM head), layers L-1 .. 0, the
    embedding. Each is split into ``world`` chunks of whole 128-element
    blocks; rank r reduces and updates chunk r of every bucket."""

    def __init__(self, arena, team, lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1):
        self.arena, self.team = arena, team
        self.world, self.rank = team.world, team.rank
        self.lr, (self.beta1, self.beta2), self.eps, self.wd = lr, betas, eps, weight_decay
        dev = arena.device
        self.buckets = bucket_chunks(arena, self.world, self.rank)
        off = sum(e - b for b, e, _ in self.buckets.values())
        self.state_len = off
        self.m = torch.zeros(max(1, off), dtype=torch.float32, device=dev)
        self.v = torch.zeros(max(1, off), dtype=torch.float32, device=dev)
        self.decay_blocks = arena.decay_mask.view(-1, 128)[:, 0].to(torch.uint8).to(dev)
        self.grad_buf = team.find(arena.grad)
        self.param_buf = team.find(arena.bf16)
        self.step_count = 0
        self.side = torch.cuda.Stream(dev) if dev.type == "cuda" else None
        self._armed = False
        self._done: set = set()
        self._lr = lr

    @property
    def slices(self):
        """[(arena begin, arena end, state offset)] of this rank's chunks."""
        return sorted(self.buckets.values())

    def broadcast_params(self) -> None:
        if self.world > 1:
            dist.broadcast(self.arena.master, src=0)
            self.arena.sync_bf16_from_master()

    def attach(self, model) -> None:
        # tensor parallelism sums some gradients after the backward (finish_grads),
        # which a bucket reduced during the backward would miss
        assert getattr(model, "tp", None) is None, "the overlapped DP engine is for pure data parallelism"
        model.grad_ready_hook = self.grad_ready

    def arm(self, lr: float | None = None) -> None:
        """The next backward is the step's last: reduce buckets as they finish."""
        self.step_count += 1
        self._lr = float(lr if lr is not None else self.lr)
        self._armed = True
        self._done = set()

    def grad_ready(self, key: str) -> None:
        """Called (on the autograd thread, with the compute stream current)
        when bucket ``key``'s gradients are final for this step."""
        if not self._armed or key in self._done or key not in self.buckets:
            return
        self._done.add(key)
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.arena.device))
        self.side.wait_event(ev)
        with torch.cuda.stream(self.side):
            self._reduce_bucket(key)

    def _reduce_bucket(self, key: str) -> None:
        a = self.arena
        gb, pb = self.grad_buf, self.param_buf
        cb, ce, so = self.buckets[key]
        self.team.barrier()  # every rank's gradients of this bucket are final
        if ce > cb:
            C().dp_reduce_adamw(gb.peers_dev, gb.mc_ptr, pb.peers_dev, pb.mc_ptr, a.master[cb:ce],
                                self.m[so : so + ce - cb], self.v[so : so + ce - cb], self.decay_blocks, cb, ce - cb,
                                self.world, self._lr, self.beta1, self.beta2, self.eps, self.wd, self.step_count,
                                1.0 / self.world, None)

    def step(self, lr: float | None = None) -> None:
        """After the last backward: the buckets whose hooks did not fire (the
        embedding, or all of them without ``arm``), then one barrier so no rank
        starts the next step before every rank's new parameters have landed."""
        if not self._armed:
            self.arm(lr)
        main = torch.cuda.current_stream(self.arena.device)
        self.side.wait_stream(main)
        with torch.cuda.stream(self.side):
            for key in self.buckets:  # ranks visit the remaining buckets in the same order
                if key not in self._done:
                    self._done.add(key)
                    self._reduce_bucket(key)
        main.wait_stream(self.side)
        self.team.barrier()
        self._armed = False

    def state_dict(self) -> dict:
        return {"m": self.m.cpu(), "v": self.v.cpu(), "step": self.step_count, "slices": self.slices}
