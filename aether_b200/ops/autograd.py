"""Autograd functions over the native kernels.

Weights are bf16 views into a flat arena and carry a ``main_grad`` attribute
(an fp32 view into the arena's flat gradient). Backward passes accumulate the
weight gradient straight into ``main_grad`` from the GEMM / reduction epilogue
(fp32, across micro-batches) and return ``None`` for the weight, so no bf16
weight-gradient tensor is ever materialised and the flat gradient is ready for
one data-parallel reduce-scatter.
"""
from __future__ import annotations

import weakref

import torch

from . import functional as F


# Gradient buffers of parameters that autograd re-creates on unpack (sharded
# parameters gathered again by a saved-tensor hook): the unpacked tensor is a
# new object, so its buffer is found by (data_ptr, numel).
MAIN_GRADS: dict = {}


def _main_grad(w: torch.Tensor) -> torch.Tensor | None:
    mg = getattr(w, "main_grad", None)
    if mg is None and MAIN_GRADS:
        mg = MAIN_GRADS.get((w.data_ptr(), w.numel()))
    return mg


# ZeRO-3 arenas in fused mode (parallel.fsdp): a weight whose memory lies in
# one of their unit buffers with a gather still pending is gathered by the GEMM
# that reads it. Looked up by address: autograd hands backward new tensor
# objects over the saved memory, so nothing set on the forward's view survives.
PG_ARENAS = weakref.WeakSet()


def _gemm_w(x, w, b_mn=False, residual=None):
    """x . w^T (b_mn: x . w) where w may be a ZeRO-3 weight whose unit is still
    to be gathered: then this GEMM is the unit's first consumer and gathers it
    inside the same kernel (parallel.fsdp, fused mode)."""
    for arena in list(PG_ARENAS):
        u = arena.pending_at(w)
        if u is not None:
            y = arena.pg_gemm(u, x, w, b_mn=b_mn, residual=residual)
            if y is not None:
                return y
            break
    return F.gemm(x, w, b_mn=b_mn, residual=residual)


class LinearFn(torch.autograd.Function):
    """y = x @ w^T (+ residual). x: [T, K], w: [N, K]."""

    @staticmethod
    def forward(ctx, x, w, residual=None):
        y = _gemm_w(x, w, residual=residual)
        ctx.save_for_backward(x, w)
        ctx.has_res = residual is not None
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        dy = dy.contiguous()
        dx = _gemm_w(dy, w, b_mn=True) if ctx.needs_input_grad[0] else None
        mg = _main_grad(w)
        dw = None
        if mg is not None:
            F.gemm(dy, x, a_mn=True, b_mn=True, out=mg, accumulate=True)
        elif ctx.needs_input_grad[1]:
            dw = F.gemm(dy, x, a_mn=True, b_mn=True, out_dtype=torch.float32).to(w.dtype)
        return dx, dw, (dy if ctx.has_res else None)


def linear(x, w, residual=None):
    return LinearFn.apply(x, w, residual)


class AddBiasFn(torch.autograd.Function):
    """y = x + b (b broadcast over rows); the bias gradient (column sums of
    dy, fp32) accumulates into b's main_grad like every arena weight."""

    @staticmethod
    def forward(ctx, x, b):
        ctx.b = b
        return x + b

    @staticmethod
    def backward(ctx, dy):
        b = ctx.b
        mg = _main_grad(b)
        db = None
        if mg is not None:
            mg.add_(dy.float().sum(0))
        elif ctx.needs_input_grad[1]:
            db = dy.float().sum(0).to(b.dtype)
        return dy, db


def add_bias(x, b):
    return AddBiasFn.apply(x, b)


class RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        y, _, rstd = F.rmsnorm(x, w, eps)
        ctx.save_for_backward(x, w, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, rstd = ctx.saved_tensors
        mg = _main_grad(w)
        tmp = None
        if mg is None:
            tmp = torch.zeros(w.shape, dtype=torch.float32, device=w.device)
        dx = F.rmsnorm_bwd(dy.contiguous(), x, w, rstd, mg if mg is not None else tmp, accumulate=True)
        return dx, (tmp.to(w.dtype) if tmp is not None and ctx.needs_input_grad[1] else None), None


def rmsnorm(x, w, eps=1e-6):
    return RMSNormFn.apply(x, w, eps)


class RMSNormResidualFn(torch.autograd.Function):
    """(rmsnorm(x) * w, x) for a pre-norm residual block: the second output
    is the residual branch (an alias of x). In backward both gradients arrive
    in one call and the kernel adds the residual gradient into dx as it
    writes it, so autograd never runs a separate [T, d] add for the two uses
    of x."""

    @staticmethod
    def forward(ctx, x, w, eps):
        y, _, rstd = F.rmsnorm(x, w, eps)
        ctx.save_for_backward(x, w, rstd)
        return y, x.view(x.shape)

    @staticmethod
    def backward(ctx, dy, dres):
        x, w, rstd = ctx.saved_tensors
        mg = _main_grad(w)
        tmp = None
        if mg is None:
            tmp = torch.zeros(w.shape, dtype=torch.float32, device=w.device)
        if dy is None:
            dy = torch.zeros_like(x)
        dx = F.rmsnorm_bwd(dy.contiguous(), x, w, rstd, mg if mg is not None else tmp,
                           dres=dres.contiguous() if dres is not None else None, accumulate=True)
        return dx, (tmp.to(w.dtype) if tmp is not None and ctx.needs_input_grad[1] else None), None


def rmsnorm_residual(x, w, eps=1e-6):
    """-> (normed, residual alias of x); see RMSNormResidualFn."""
    return RMSNormResidualFn.apply(x, w, eps)


class LayerNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, eps):
        y, _, mean, rstd = F.layernorm(x, w, b, eps)
        ctx.save_for_backward(x, w, mean, rstd)
        ctx.b = b
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, mean, rstd = ctx.saved_tensors
        b = ctx.b
        mgw = _main_grad(w)
        mgb = _main_grad(b) if b is not None else None
        tw = mgw if mgw is not None else torch.zeros(w.shape, dtype=torch.float32, device=w.device)
        tb = mgb if mgb is not None else torch.zeros(w.shape, dtype=torch.float32, device=w.device)
        dx = F.layernorm_bwd(dy.contiguous(), x, w, mean, rstd, tw, tb, accumulate=True)
        dw = tw.to(w.dtype) if mgw is None and ctx.needs_input_grad[1] else None
        db = tb.to(w.dtype) if b is not None and mgb is None and ctx.needs_input_grad[2] else None
        return dx, dw, db, None


def layernorm(x, w, b=None, eps=1e-5):
    return LayerNormFn.apply(x, w, b, eps)


class RopeFn(torch.autograd.Function):
    """In-place RoPE on the first n_heads heads of each row of a [T, row] tensor."""

    @staticmethod
    def forward(ctx, x2d, pos, cos_t, sin_t, n_heads, head_dim):
        F.rope_(x2d, pos, cos_t, sin_t, n_heads, head_dim)
        ctx.mark_dirty(x2d)
        ctx.save_for_backward(pos, cos_t, sin_t)
        ctx.n_heads, ctx.head_dim = n_heads, head_dim
        return x2d

    @staticmethod
    def backward(ctx, dy):
        pos, cos_t, sin_t = ctx.saved_tensors
        dy = dy.contiguous().clone() if not dy.is_contiguous() else dy
        F.rope_(dy, pos, cos_t, sin_t, ctx.n_heads, ctx.head_dim, inverse=True)
        return dy, None, None, None, None, None


def rope_(x2d, pos, cos_t, sin_t, n_heads, head_dim):
    return RopeFn.apply(x2d, pos, cos_t, sin_t, n_heads, head_dim)


class AttentionFn(torch.autograd.Function):
    """Causal attention over a packed qkv [B*S, (Hq + 2*Hkv) * D] buffer -> o [B*S, Hq*D]."""

    @staticmethod
    def forward(ctx, qkv, B, S, Hq, Hkv, D, scale, causal, window=0, softcap=0.0):
        row = qkv.shape[1]
        q = qkv.view(B, S, row)[:, :, : Hq * D].view(B, S, Hq, D)
        k = qkv.view(B, S, row)[:, :, Hq * D : (Hq + Hkv) * D].view(B, S, Hkv, D)
        v = qkv.view(B, S, row)[:, :, (Hq + Hkv) * D :].view(B, S, Hkv, D)
        o = torch.empty(B, S, Hq, D, dtype=qkv.dtype, device=qkv.device)
        o, lse = F.attention(q, k, v, scale, causal, 0, out=o, window=window, softcap=softcap)
        ctx.save_for_backward(qkv, o, lse)
        ctx.cfg = (B, S, Hq, Hkv, D, scale, causal, window, softcap)
        return o.view(B * S, Hq * D)

    @staticmethod
    def backward(ctx, do):
        qkv, o, lse = ctx.saved_tensors
        B, S, Hq, Hkv, D, scale, causal, window, softcap = ctx.cfg
        row = qkv.shape[1]
        v3 = qkv.view(B, S, row)
        q = v3[:, :, : Hq * D].view(B, S, Hq, D)
        k = v3[:, :, Hq * D : (Hq + Hkv) * D].view(B, S, Hkv, D)
        v = v3[:, :, (Hq + Hkv) * D :].view(B, S, Hkv, D)
        dqkv = torch.empty_like(qkv)
        d3 = dqkv.view(B, S, row)
        dq = d3[:, :, : Hq * D].view(B, S, Hq, D)
        dk = d3[:, :, Hq * D : (Hq + Hkv) * D].view(B, S, Hkv, D)
        dv = d3[:, :, (Hq + Hkv) * D :].view(B, S, Hkv, D)
        F.attention_bwd(q, k, v, o, do.contiguous().view(B, S, Hq, D), lse, scale, causal, 0, dq=dq, dk=dk, dv=dv,
                        window=window, softcap=softcap)
        return dqkv, None, None, None, None, None, None, None, None, None


def attention_packed(qkv, B, S, Hq, Hkv, D, scale, causal=True, window=0, softcap=0.0):
    """window > 0: sliding-window attention; softcap > 0: soft-capped logits
    (forward and backward)."""
    return AttentionFn.apply(qkv, B, S, Hq, Hkv, D, scale, causal, window, softcap)


class SwiGLUFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h):
        ctx.save_for_backward(h)
        return F.swiglu(h)

    @staticmethod
    def backward(ctx, dact):
        (h,) = ctx.saved_tensors
        return F.swiglu_bwd(h, dact.contiguous())


def swiglu(h):
    return SwiGLUFn.apply(h)


class GeluFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        ctx.save_for_backward(x)
        return F.gelu(x)

    @staticmethod
    def backward(ctx, dy):
        (x,) = ctx.saved_tensors
        return F.gelu_bwd(x, dy.contiguous())


def gelu(x):
    return GeluFn.apply(x)


class EmbeddingFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, table, ids):
        ctx.save_for_backward(ids)
        ctx.table = table
        return F.embedding(table, ids)

    @staticmethod
    def backward(ctx, dy):
        (ids,) = ctx.saved_tensors
        table = ctx.table
        mg = _main_grad(table)
        if mg is not None:
            F.embedding_bwd(dy.contiguous(), ids, mg)
            return None, None
        g = torch.zeros(table.shape, dtype=torch.float32, device=table.device)
        F.embedding_bwd(dy.contiguous(), ids, g)
        return g.to(table.dtype), None


def embedding(table, ids):
    return EmbeddingFn.apply(table, ids)


class LMHeadCrossEntropyFn(torch.autograd.Function):
    """loss = sum_t CE(x_t @ w^T, target_t) * loss_scale, with the logits
    gradient computed in the forward pass (written over the logits buffer) and
    scaled on the device by the incoming gradient during backward."""

    @staticmethod
    def forward(ctx, x, w, targets, loss_scale, ignore_index):
        logits = F.gemm(x, w)
        loss_rows, _ = F.cross_entropy_fused(logits, targets, grad_scale=loss_scale, ignore_index=ignore_index,
                                             write_grad=True)
        ctx.save_for_backward(x, w, logits)
        return loss_rows.sum() * loss_scale

    @staticmethod
    def backward(ctx, dloss):
        x, w, dlogits = ctx.saved_tensors
        g = dloss.reshape(1).float().contiguous()
        dx = F.gemm(dlogits, w, b_mn=True, alpha_t=g)
        mg = _main_grad(w)
        dw = None
        if mg is not None:
            F.gemm(dlogits, x, a_mn=True, b_mn=True, out=mg, accumulate=True, alpha_t=g)
        elif ctx.needs_input_grad[1]:
            dw = F.gemm(dlogits, x, a_mn=True, b_mn=True, out_dtype=torch.float32, alpha_t=g).to(w.dtype)
        return dx, dw, None, None, None


def lm_head_cross_entropy(x, w, targets, loss_scale, ignore_index=-100):
    return LMHeadCrossEntropyFn.apply(x, w, targets, float(loss_scale), ignore_index)


class ChunkedLMHeadCrossEntropyFn(torch.autograd.Function):
    """LMHeadCrossEntropyFn over ``chunk`` tokens at a time: each chunk's
    logits [chunk, V] are computed, turned into their gradient by the fused
    cross-entropy kernel and consumed at once -- the input gradient of the
    chunk (dlogits W) and, when the head trains, its weight gradient
    (dlogits^T x, accumulated in fp32) -- so no [tokens, V] tensor exists.
    Backward scales the stored gradients by the incoming one. Reference: the
    QLoRA stage's chunked LM-head loss (trainer/src/qwen_qlora_stage.rs)."""

    @staticmethod
    def forward(ctx, x, w, targets, loss_scale, chunk, ignore_index):
        T = x.shape[0]
        dx = torch.empty_like(x)
        train_w = ctx.needs_input_grad[1]
        dw = torch.zeros(w.shape, dtype=torch.float32, device=w.device) if train_w else None
        total = torch.zeros((), dtype=torch.float32, device=x.device)
        for t0 in range(0, T, chunk):
            xs, ts = x[t0 : t0 + chunk], targets[t0 : t0 + chunk]
            logits = F.gemm(xs, w)
            rows, _ = F.cross_entropy_fused(logits, ts, grad_scale=loss_scale, ignore_index=ignore_index,
                                            write_grad=True)
            total = total + rows.sum()
            F.gemm(logits, w, b_mn=True, out=dx[t0 : t0 + chunk])
            if train_w:
                F.gemm(logits, xs, a_mn=True, b_mn=True, out=dw, accumulate=True)
            del logits
        ctx.save_for_backward(dx, dw if train_w else torch.empty(0))
        ctx.train_w, ctx.wref = train_w, w
        return total * loss_scale

    @staticmethod
    def backward(ctx, dloss):
        dx, dw = ctx.saved_tensors
        g = dloss.float()
        gx = (dx.float() * g).to(dx.dtype)
        gw = None
        if ctx.train_w:
            w = ctx.wref
            mg = _main_grad(w)
            if mg is not None:
                mg.add_(dw * g)
            else:
                gw = (dw * g).to(w.dtype)
        return gx, gw, None, None, None, None


def lm_head_cross_entropy_chunked(x, w, targets, loss_scale, chunk, ignore_index=-100):
    return ChunkedLMHeadCrossEntropyFn.apply(x, w, targets, float(loss_scale), int(chunk), ignore_index)
