"""Tensor parallelism for training (Megatron layout) and the 2-D TP x DP mesh.

Per layer, with T token rows replicated on every TP rank:
  wqkv, wgu   column-parallel: each rank holds the rows of its heads / of its
              slice of the SwiGLU intermediate (gate and up halves alike)
  wo, wd      row-parallel: each rank holds the matching input columns and
              produces a partial sum that is all-reduced over the TP group
  norms, embedding, LM head  replicated (their inputs and output gradients
              are identical on every TP rank, so their gradients are too)
Autograd: ``tp_copy`` (identity forward, all-reduce of the input gradient in
backward) sits in front of each column-parallel projection, ``tp_reduce``
(all-reduce forward, identity backward) after each row-parallel one; the
residual is added by TP rank 0's GEMM epilogue only, so the sum carries it
once. Two all-reduces per layer forward and two backward.

The all-reduce is pluggable: NCCL over the TP process group (the baseline), or
the in-kernel symmetric-memory all-reduce (``parallel.symm.SymmTeam``, NVLS
``multimem.ld_reduce`` / ``multimem.st`` or one-shot peer loads).

Reference: the Megatron plan of runtime/src/tensor_parallel.rs:8-29
(column-parallel QKV and gate/up, row-parallel o_proj and down_proj, 2
all-reduces per block, KV heads replicated below TP = n_kv) -- which the
reference only executes on one GPU -- and the TP4 x DP2 training target.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass
class TPGroup:
    rank: int
    world: int
    group: object = None
    team: object = None  # SymmTeam for the in-kernel all-reduce (None: NCCL / gloo)
    _bufs: dict = None

    def all_reduce_(self, t: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return t
        if self.team is not None and t.is_cuda and t.is_contiguous():
            if self._bufs is None:
                self._bufs = {}
            key = (t.dtype, t.numel())
            if key not in self._bufs:
                self._bufs[key] = self.team.alloc(t.numel(), t.dtype)
            buf = self._bufs[key]
            buf.tensor.copy_(t.view(-1))
            self.team.all_reduce_(buf)
            t.view(-1).copy_(buf.tensor)
            return t
        dist.all_reduce(t, group=self.group)
        return t


@dataclass
class Mesh:
    """rank = dp_rank * tp + tp_rank: TP groups are runs of consecutive ranks."""

    tp: TPGroup
    dp_rank: int
    dp_world: int
    dp_group: object


def make_mesh(tp_size: int, use_symm: bool = False) -> Mesh:
    world = dist.get_world_size() if dist.is_initialized() else 1
    rank = dist.get_rank() if dist.is_initialized() else 0
    assert world % tp_size == 0, "world size must be a multiple of the TP degree"
    dp_size = world // tp_size
    tp_group = dp_group = None
    if world > 1:
        for d in range(dp_size):  # every rank creates every group, in the same order
            g = dist.new_group(list(range(d * tp_size, (d + 1) * tp_size)))
            if d == rank // tp_size:
                tp_group = g
        for t in range(tp_size):
            g = dist.new_group(list(range(t, world, tp_size)))
            if t == rank % tp_size:
                dp_group = g
    team = None
    if use_symm and tp_size > 1:
        from .symm import SymmTeam
        from .dist import DistInfo

        info = DistInfo(rank, world, rank, torch.device("cuda", torch.cuda.current_device()), "nccl")
        team = SymmTeam(info, group=tp_group)
    return Mesh(TPGroup(rank % tp_size, tp_size, tp_group, team), rank // tp_size, dp_size, dp_group)


class _Copy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, tp):
        ctx.tp = tp
        return x

    @staticmethod
    def backward(ctx, dx):
        return ctx.tp.all_reduce_(dx.contiguous().clone()), None


class _Reduce(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y, tp):
        ctx.mark_dirty(y)
        return tp.all_reduce_(y)

    @staticmethod
    def backward(ctx, dy):
        return dy, None


class _ReduceResidual(torch.autograd.Function):
    """out = all_reduce(y) where TP rank 0's y already holds the residual r;
    r's gradient is the output gradient on every rank."""

    @staticmethod
    def forward(ctx, y, r, tp):
        ctx.has_r = r is not None
        ctx.mark_dirty(y)
        return tp.all_reduce_(y)

    @staticmethod
    def backward(ctx, dy):
        return dy, (dy if ctx.has_r else None), None


def tp_reduce_residual(y, r, tp):
    return _ReduceResidual.apply(y, r, tp)


def tp_copy(x, tp):
    return _Copy.apply(x, tp) if tp is not None and tp.world > 1 else x


def tp_reduce(y, tp):
    return _Reduce.apply(y, tp) if tp is not None and tp.world > 1 else y


# ---------------------------------------------------------------------------- sharding of full tensors
COLUMN = ("wqkv", "wgu")
ROW = ("wo", "wd")


def shard_shape(cfg, name: str, shape: tuple, tp_size: int) -> tuple:
    base = name.split(".")[-1]
    if tp_size == 1 or base not in COLUMN + ROW:
        return shape
    if base == "wqkv":
        hq, hkv = cfg.n_heads // tp_size, cfg.n_kv_heads // tp_size
        return ((hq + 2 * hkv) * cfg.head_dim, shape[1])
    if base == "wgu":
        return (shape[0] // tp_size, shape[1])
    return (shape[0], shape[1] // tp_size)  # wo, wd: input columns


def shard_tensor(cfg, name: str, full: torch.Tensor, tp_rank: int, tp_size: int) -> torch.Tensor:
    base = name.split(".")[-1]
    if tp_size == 1 or base not in COLUMN + ROW:
        return full
    r = tp_rank
    if base == "wqkv":
        D, Hq, Hkv = cfg.head_dim, cfg.n_heads, cfg.n_kv_heads
        hq, hkv = Hq // tp_size, Hkv // tp_size
        q = full[r * hq * D : (r + 1) * hq * D]
        k = full[(Hq + r * hkv) * D : (Hq + (r + 1) * hkv) * D]
        v = full[(Hq + Hkv + r * hkv) * D : (Hq + Hkv + (r + 1) * hkv) * D]
        return torch.cat([q, k, v], 0)
    if base == "wgu":
        f = full.shape[0] // 2
        fl = f // tp_size
        return torch.cat([full[r * fl : (r + 1) * fl], full[f + r * fl : f + (r + 1) * fl]], 0)
    cols = full.shape[1] // tp_size
    return full[:, r * cols : (r + 1) * cols]
