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

Sequence parallelism (``make_mesh(..., sequence_parallel=True)``): between
the projections the [T, d] residual stream, its norms and their saved
activations are split by token over the TP ranks; each all-reduce becomes a
reduce-scatter after the row-parallel GEMM plus an all-gather before the next
column-parallel one (the column GEMM keeps only its local rows and gathers them
again in backward, overlapped with the input-gradient GEMM). The per-layer norm
weights then see only their rank's tokens, so ``GPT.finish_grads`` sums their
gradients over the TP group; the embedding output is split after the lookup
and the final norm, LM head and loss run on the all-gathered rows.

The all-reduce is pluggable: NCCL over the TP process group (the baseline), or
the in-kernel symmetric-memory all-reduce (``parallel.symm.SymmTeam``, NVLS
``multimem.ld_reduce`` / ``multimem.st`` or one-shot peer loads). With
``make_mesh(..., sequence_parallel=True, fused=True)`` each sequence-parallel
projection is instead one ``gemm_tp`` kernel (``parallel.tp_fused``): the
all-gather or reduce-scatter runs inside the GEMM over NVLink, tile by tile.

Reference: the Megatron plan of runtime/src/tensor_parallel.rs:8-29
(column-parallel QKV and gate/up, row-parallel o_proj and down_proj, 2
all-reduces per block, KV heads replicated below TP = n_kv) -- which the
reference only executes on one GPU -- and the TP4 x DP2 training target. The
reference has no sequence parallelism (its long-context features are paged KV
and split-K decode attention); the split here is Megatron's.
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
    sp: bool = False  # sequence parallelism: the residual stream split by token
    fused: object = None  # parallel.tp_fused.FusedTP: projections with the collective inside the GEMM

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


def make_mesh(tp_size: int, use_symm: bool = False, sequence_parallel: bool = False, fused: bool = False) -> Mesh:
    """fused: (with sequence_parallel) every projection is one gemm_tp kernel with
    its all-gather / reduce-scatter over NVLink inside it -- no NCCL call per layer."""
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
    assert not fused or sequence_parallel, "the fused projections work on token-split rows (sequence parallelism)"
    team = None
    if (use_symm or fused) and tp_size > 1:
        from .symm import SymmTeam
        from .dist import DistInfo

        info = DistInfo(rank, world, rank, torch.device("cuda", torch.cuda.current_device()), "nccl")
        team = SymmTeam(info, group=tp_group)
    fused_tp = None
    if fused and tp_size > 1:
        from .tp_fused import FusedTP

        fused_tp = FusedTP(team)
    return Mesh(TPGroup(rank % tp_size, tp_size, tp_group, team if use_symm else None,
                        sp=sequence_parallel and tp_size > 1, fused=fused_tp),
                rank // tp_size, dp_size, dp_group)


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


# ---------------------------------------------------------------------------- sequence parallelism
# The residual stream (and with it the norms and their saved activations) is
# split by token over the TP ranks: rank r holds rows [r*Tl, (r+1)*Tl) of the
# [T, d] hidden state. A column-parallel projection all-gathers its input rows
# (and reduce-scatters the input gradient), a row-parallel one reduce-scatters
# its partial sums (and all-gathers the output gradient): the same bytes as the
# two all-reduces, split into their halves, with 1/tp of the activations kept.
def _gather_tokens(t: torch.Tensor, tp: TPGroup, async_op: bool = False):
    """[Tl, ...] on every TP rank -> [tp*Tl, ...] (rank r's rows at r*Tl)."""
    t = t.contiguous()
    out = torch.empty((tp.world * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
    if t.is_cuda:
        work = dist.all_gather_into_tensor(out, t, group=tp.group, async_op=async_op)
    else:
        work = dist.all_gather(list(out.chunk(tp.world)), t, group=tp.group, async_op=async_op)
    return out, work


def _scatter_tokens(t: torch.Tensor, tp: TPGroup, async_op: bool = False):
    """[tp*Tl, ...] partial sums on every rank -> this rank's rows of the sum."""
    t = t.contiguous()
    Tl = t.shape[0] // tp.world
    if t.is_cuda:
        out = torch.empty((Tl,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        work = dist.reduce_scatter_tensor(out, t, group=tp.group, async_op=async_op)
        return out, work
    full = t.clone()  # gloo has no reduce-scatter
    dist.all_reduce(full, group=tp.group)
    return full[tp.rank * Tl : (tp.rank + 1) * Tl].clone(), None


def _wgrad(dy, x, w):
    """dW = dy^T x, accumulated into w's fp32 main gradient when it has one."""
    from ..ops import functional as F
    from ..ops.autograd import _main_grad

    mg = _main_grad(w)
    if mg is not None:
        F.gemm(dy, x, a_mn=True, b_mn=True, out=mg, accumulate=True)
        return None
    return F.gemm(dy, x, a_mn=True, b_mn=True, out_dtype=torch.float32).to(w.dtype)


class _SPColumnLinear(torch.autograd.Function):
    """y = all_gather(h) @ w^T. Only the local rows h are saved: backward
    gathers them again on the communication stream while the input-gradient
    GEMM runs, and reduce-scatters that gradient while the weight-gradient
    GEMM runs."""

    @staticmethod
    def forward(ctx, h, w, tp):
        from ..ops import functional as F

        hf, _ = _gather_tokens(h, tp)
        ctx.tp = tp
        ctx.save_for_backward(h, w)
        return F.gemm(hf, w)

    @staticmethod
    def backward(ctx, dy):
        from ..ops import functional as F

        h, w = ctx.saved_tensors
        tp = ctx.tp
        dy = dy.contiguous()
        hf, gwork = _gather_tokens(h, tp, async_op=True)
        dhf = F.gemm(dy, w, b_mn=True)
        dh, swork = _scatter_tokens(dhf, tp, async_op=True)
        if gwork is not None:
            gwork.wait()
        dw = _wgrad(dy, hf, w) if ctx.needs_input_grad[1] else None
        if swork is not None:
            swork.wait()
        return dh, dw, None


class _SPRowLinear(torch.autograd.Function):
    """x_out = reduce_scatter(o @ w^T) + r: o holds this rank's heads / FFN
    columns for all T tokens, r and x_out this rank's token rows."""

    @staticmethod
    def forward(ctx, o, w, r, tp):
        from ..ops import functional as F

        y, _ = _scatter_tokens(F.gemm(o, w), tp)
        ctx.tp = tp
        ctx.has_r = r is not None
        ctx.save_for_backward(o, w)
        return y.add_(r) if r is not None else y

    @staticmethod
    def backward(ctx, dx):
        from ..ops import functional as F

        o, w = ctx.saved_tensors
        dyf, _ = _gather_tokens(dx, ctx.tp)
        do = F.gemm(dyf, w, b_mn=True) if ctx.needs_input_grad[0] else None
        dw = _wgrad(dyf, o, w) if ctx.needs_input_grad[1] else None
        return do, dw, (dx if ctx.has_r else None), None


class _SPSplit(torch.autograd.Function):
    """Full rows computed identically on every rank -> this rank's rows; the
    gradient of the full tensor is the all-gather of the row gradients."""

    @staticmethod
    def forward(ctx, x, tp):
        ctx.tp = tp
        Tl = x.shape[0] // tp.world
        return x[tp.rank * Tl : (tp.rank + 1) * Tl].clone()

    @staticmethod
    def backward(ctx, dx):
        return _gather_tokens(dx, ctx.tp)[0], None


class _SPGather(torch.autograd.Function):
    """This rank's rows -> all rows, followed by work that every rank repeats
    on the full tensor (final norm, LM head, loss): the incoming gradient is
    the same on every rank, so each keeps its own rows of it."""

    @staticmethod
    def forward(ctx, x, tp):
        ctx.tp = tp
        return _gather_tokens(x, tp)[0]

    @staticmethod
    def backward(ctx, dx):
        tp = ctx.tp
        Tl = dx.shape[0] // tp.world
        return dx[tp.rank * Tl : (tp.rank + 1) * Tl].contiguous(), None


def sp_column_linear(h, w, tp):
    if tp.fused is not None and h.is_cuda and tp.fused.supports(h.shape[0]):
        from .tp_fused import fused_column_linear

        return fused_column_linear(h, w, tp)
    return _SPColumnLinear.apply(h, w, tp)


def sp_row_linear(o, w, r, tp):
    if tp.fused is not None and o.is_cuda and tp.fused.supports(o.shape[0] // tp.world):
        from .tp_fused import fused_row_linear

        return fused_row_linear(o, w, r, tp)
    return _SPRowLinear.apply(o, w, r, tp)


def sp_split(x, tp):
    return _SPSplit.apply(x, tp)


def sp_gather(x, tp):
    return _SPGather.apply(x, tp)


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
