"""Context parallelism for long-sequence training: the sequence is split into
contiguous chunks, one per rank of the CP group, and every attention layer
all-gathers K and V over NVLink.

Per layer on CP rank r (chunk length Sl, queries at global positions
[r*Sl, (r+1)*Sl)):
    K, V      = all_gather over the CP group ([B, S, Hkv, D], S = cp * Sl)
    O, lse    = causal attention of the local queries against all keys with
                causal offset r*Sl (one flash-attention launch)
  backward:
    dQ, dK*, dV* = attention backward against the gathered K/V (same offset)
    dK, dV    = reduce-scatter of dK*, dV* over the group (each rank keeps the
                sum of every rank's contribution to its own chunk)
Weights are replicated over the CP group, so their gradients are averaged
with the data-parallel engines (each rank's loss is the mean over its own
tokens, and the chunks are equal). RoPE uses global positions.

The reference has no sequence / context parallelism (long context comes only
from paged KV and split-K decode there); this is the all-gather form of
context parallelism, which on NVSwitch moves 2 * (cp - 1) / cp of a layer's
K/V per rank per layer -- small next to the attention FLOPs at long S -- and
keeps one causal attention launch per layer instead of a ring of cp launches.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from ..ops import functional as F


@dataclass
class CPGroup:
    rank: int
    world: int
    group: object = None


def all_gather_seq(t: torch.Tensor, cp: CPGroup) -> torch.Tensor:
    """[B, Sl, ...] on every rank -> [B, cp * Sl, ...] (chunk r at r*Sl)."""
    parts = [torch.empty_like(t) for _ in range(cp.world)]
    dist.all_gather(parts, t.contiguous(), group=cp.group)
    return torch.cat(parts, dim=1)


def reduce_scatter_seq(t: torch.Tensor, cp: CPGroup) -> torch.Tensor:
    """[B, cp * Sl, ...] partial sums on every rank -> this rank's chunk of the sum."""
    Sl = t.shape[1] // cp.world
    chunks = [c.contiguous() for c in t.split(Sl, dim=1)]
    if t.is_cuda:
        out = torch.empty_like(chunks[0])
        dist.reduce_scatter(out, chunks, group=cp.group)
        return out
    full = torch.stack(chunks)  # gloo has no reduce-scatter
    dist.all_reduce(full, group=cp.group)
    return full[cp.rank].clone()


class CPAttentionFn(torch.autograd.Function):
    """Causal attention of a packed local qkv [B*Sl, (Hq + 2 Hkv) D] against the
    whole sequence's keys -> o [B*Sl, Hq*D]."""

    @staticmethod
    def forward(ctx, qkv, B, Sl, Hq, Hkv, D, scale, cp):
        row = qkv.shape[1]
        v3 = qkv.view(B, Sl, row)
        q = v3[:, :, : Hq * D].view(B, Sl, Hq, D)
        k = v3[:, :, Hq * D : (Hq + Hkv) * D].view(B, Sl, Hkv, D)
        v = v3[:, :, (Hq + Hkv) * D :].view(B, Sl, Hkv, D)
        kf, vf = all_gather_seq(k, cp), all_gather_seq(v, cp)
        off = cp.rank * Sl
        o = torch.empty(B, Sl, Hq, D, dtype=qkv.dtype, device=qkv.device)
        o, lse = F.attention(q, kf, vf, scale, True, off, out=o)
        ctx.save_for_backward(qkv, kf, vf, o, lse)
        ctx.cfg = (B, Sl, Hq, Hkv, D, scale, cp, off)
        return o.view(B * Sl, Hq * D)

    @staticmethod
    def backward(ctx, do):
        qkv, kf, vf, o, lse = ctx.saved_tensors
        B, Sl, Hq, Hkv, D, scale, cp, off = ctx.cfg
        row = qkv.shape[1]
        q = qkv.view(B, Sl, row)[:, :, : Hq * D].view(B, Sl, Hq, D)
        dqkv = torch.empty_like(qkv)
        d3 = dqkv.view(B, Sl, row)
        dq = d3[:, :, : Hq * D].view(B, Sl, Hq, D)
        _, dkf, dvf = F.attention_bwd(q, kf, vf, o, do.contiguous().view(B, Sl, Hq, D), lse, scale, True, off, dq=dq)
        d3[:, :, Hq * D : (Hq + Hkv) * D] = reduce_scatter_seq(dkf, cp).view(B, Sl, Hkv * D)
        d3[:, :, (Hq + Hkv) * D :] = reduce_scatter_seq(dvf, cp).view(B, Sl, Hkv * D)
        return dqkv, None, None, None, None, None, None, None


def cp_attention(qkv, B, Sl, Hq, Hkv, D, scale, cp: CPGroup):
    return CPAttentionFn.apply(qkv, B, Sl, Hq, Hkv, D, scale, cp)


def shard_sequence(tokens: torch.Tensor, cp: CPGroup):
    """tokens [b, S+1] -> this rank's (ids, targets), each [b, S / cp]."""
    S = tokens.shape[1] - 1
    Sl = S // cp.world
    a = cp.rank * Sl
    return tokens[:, a : a + Sl].contiguous(), tokens[:, a + 1 : a + Sl + 1].contiguous()
