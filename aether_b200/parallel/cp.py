"""Context parallelism for long-sequence training: the sequence is split into
contiguous chunks, one per rank of the CP group. Three attention schemes
(``CPGroup.mode``):

  * ``allgather`` (default): every attention layer all-gathers K and V over
    NVLink and runs one causal flash-attention launch (described below);
  * ``ring``: ring attention -- K/V chunks travel around the group with
    point-to-point transfers that overlap the attention of the chunk in hand;
    partial outputs merge by log-sum-exp, so a rank never holds more than two
    K/V chunks (memory O(S / cp) per rank). Backward sends each chunk around
    again with its dK / dV accumulators, which arrive back at the owner;
  * ``ulysses``: all-to-all from sequence-sharded to head-sharded q / k / v,
    full-sequence causal attention on H / cp heads, all-to-all back (needs
    H and Hkv divisible by cp).

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
    mode: str = "allgather"  # "allgather" | "ring" | "ulysses"

    def peer(self, r: int) -> int:
        """Global rank of group rank r (the group may be a sub-group)."""
        return r if self.group is None else dist.get_global_rank(self.group, r)


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


def _split_qkv(t, B, Sl, Hq, Hkv, D):
    v3 = t.view(B, Sl, t.shape[1])
    return (v3[:, :, : Hq * D].view(B, Sl, Hq, D), v3[:, :, Hq * D : (Hq + Hkv) * D].view(B, Sl, Hkv, D),
            v3[:, :, (Hq + Hkv) * D :].view(B, Sl, Hkv, D))


def _partial_attention_bwd(q, k, v, o, do, lse, scale, causal):
    """Gradients of one K/V chunk's share of an attention whose normaliser
    (lse [B, Hq, Sq], natural log) and output o cover more keys than this chunk:
    P = exp(s - lse), dV = P^T dO, dS = P * (dO V^T - rowsum(dO * O)),
    dQ = scale dS K, dK = scale dS^T Q. The device path is the flash kernel
    (which takes lse and o as given); this is its host form."""
    if q.is_cuda:
        return F.attention_bwd(q, k, v, o, do, lse, scale, causal, 0)
    B, Sq, Hq, D = q.shape
    Sk, Hkv = k.shape[1], k.shape[2]
    g = Hq // Hkv
    qf, of, dof = (t.float().permute(0, 2, 1, 3) for t in (q, o, do))
    kf = k.float().permute(0, 2, 1, 3).repeat_interleave(g, dim=1)
    vf = v.float().permute(0, 2, 1, 3).repeat_interleave(g, dim=1)
    sc = (qf @ kf.transpose(-1, -2)) * scale
    if causal:
        i = torch.arange(Sq)[:, None]
        j = torch.arange(Sk)[None, :]
        sc = sc.masked_fill(j > i, float("-inf"))
    pr = torch.exp(sc - lse.float()[..., None])
    dv = pr.transpose(-1, -2) @ dof
    ds = pr * (dof @ vf.transpose(-1, -2) - (dof * of).sum(-1, keepdim=True))
    dq = (ds @ kf) * scale
    dk = (ds.transpose(-1, -2) @ qf) * scale

    def back(t, groups):  # [B, H, S, D] -> [B, S, H / groups, D], summing each GQA group
        t = t.view(B, t.shape[1] // groups, groups, t.shape[2], D).sum(2) if groups > 1 else t
        return t.permute(0, 2, 1, 3)

    return back(dq, 1).to(q.dtype), back(dk, g).to(k.dtype), back(dv, g).to(v.dtype)


def _ring_exchange(cp: CPGroup, send: list, recv: list):
    """Sends the tensors to the next rank and receives as many from the
    previous one (asynchronously); returns the requests."""
    nxt, prv = cp.peer((cp.rank + 1) % cp.world), cp.peer((cp.rank - 1) % cp.world)
    ops = [dist.P2POp(dist.isend, t, nxt, cp.group) for t in send]
    ops += [dist.P2POp(dist.irecv, t, prv, cp.group) for t in recv]
    return dist.batch_isend_irecv(ops)


class RingAttentionFn(torch.autograd.Function):
    """Causal ring attention of a packed local qkv [B*Sl, (Hq + 2 Hkv) D]."""

    @staticmethod
    def forward(ctx, qkv, B, Sl, Hq, Hkv, D, scale, cp):
        q, k, v = _split_qkv(qkv, B, Sl, Hq, Hkv, D)
        r, W = cp.rank, cp.world
        cur = [k.contiguous(), v.contiguous()]
        o_acc = torch.zeros(B, Sl, Hq, D, dtype=torch.float32, device=qkv.device)
        lse_acc = torch.full((B, Hq, Sl), float("-inf"), dtype=torch.float32, device=qkv.device)
        for j in range(W):
            src = (r - j) % W  # owner of the chunk in hand
            reqs, nxt = [], None
            if j < W - 1:
                nxt = [torch.empty_like(t) for t in cur]
                reqs = _ring_exchange(cp, cur, nxt)
            if src <= r:  # chunks after this rank's are fully masked
                o_s, lse_s = F.attention(q, cur[0], cur[1], scale, src == r, 0)
                lse_s = lse_s.float()
                new = torch.logaddexp(lse_acc, lse_s)
                wa = torch.exp(lse_acc - new).permute(0, 2, 1)[..., None]
                wb = torch.exp(lse_s - new).permute(0, 2, 1)[..., None]
                o_acc = o_acc * wa + o_s.float() * wb
                lse_acc = new
            for rq in reqs:
                rq.wait()
            if nxt is not None:
                cur = nxt
        o = o_acc.to(qkv.dtype)
        ctx.save_for_backward(qkv, o, lse_acc)
        ctx.cfg = (B, Sl, Hq, Hkv, D, scale, cp)
        return o.view(B * Sl, Hq * D)

    @staticmethod
    def backward(ctx, do):
        qkv, o, lse = ctx.saved_tensors
        B, Sl, Hq, Hkv, D, scale, cp = ctx.cfg
        q, k, v = _split_qkv(qkv, B, Sl, Hq, Hkv, D)
        do = do.contiguous().view(B, Sl, Hq, D)
        r, W = cp.rank, cp.world
        dq = torch.zeros(B, Sl, Hq, D, dtype=torch.float32, device=qkv.device)
        cur = [k.contiguous(), v.contiguous(), torch.zeros(k.shape, dtype=torch.float32, device=qkv.device),
               torch.zeros(v.shape, dtype=torch.float32, device=qkv.device)]
        for j in range(W):
            src = (r - j) % W
            if src <= r:
                dq_s, dk_s, dv_s = _partial_attention_bwd(q, cur[0], cur[1], o, do, lse, scale, src == r)
                dq += dq_s.float()
                cur[2] += dk_s.float()
                cur[3] += dv_s.float()
            # pass the chunk on with its gradient sums; after W hops each is home again
            send = cur if j < W - 1 else cur[2:]
            nxt = [torch.empty_like(t) for t in send]
            for rq in _ring_exchange(cp, send, nxt):
                rq.wait()
            cur = nxt if j < W - 1 else [None, None] + nxt
        dqkv = torch.empty_like(qkv)
        d3 = dqkv.view(B, Sl, qkv.shape[1])
        d3[:, :, : Hq * D] = dq.view(B, Sl, Hq * D).to(qkv.dtype)
        d3[:, :, Hq * D : (Hq + Hkv) * D] = cur[2].view(B, Sl, Hkv * D).to(qkv.dtype)
        d3[:, :, (Hq + Hkv) * D :] = cur[3].view(B, Sl, Hkv * D).to(qkv.dtype)
        return dqkv, None, None, None, None, None, None, None


def _seq_to_heads(t: torch.Tensor, cp: CPGroup) -> torch.Tensor:
    """[B, Sl, H, D] sequence-sharded -> [B, W*Sl, H/W, D] head-sharded (all-to-all)."""
    B, Sl, H, D = t.shape
    W = cp.world
    src = t.reshape(B, Sl, W, H // W, D).permute(2, 0, 1, 3, 4).contiguous()  # [W(dest), B, Sl, H/W, D]
    out = torch.empty_like(src)                                              # [W(source chunk), ...]
    dist.all_to_all_single(out, src, group=cp.group)
    return out.permute(1, 0, 2, 3, 4).reshape(B, W * Sl, H // W, D)


def _heads_to_seq(t: torch.Tensor, cp: CPGroup) -> torch.Tensor:
    """Inverse of _seq_to_heads: [B, W*Sl, H/W, D] -> [B, Sl, H, D]."""
    B, S, Hl, D = t.shape
    W = cp.world
    Sl = S // W
    src = t.reshape(B, W, Sl, Hl, D).permute(1, 0, 2, 3, 4).contiguous()   # [W(dest chunk), B, Sl, Hl, D]
    out = torch.empty_like(src)                                              # [W(source head group), ...]
    dist.all_to_all_single(out, src, group=cp.group)
    return out.permute(1, 2, 0, 3, 4).reshape(B, Sl, W * Hl, D)


class UlyssesAttentionFn(torch.autograd.Function):
    """Causal attention of a packed local qkv with the heads spread over the
    group and the whole sequence on every rank (two all-to-alls each way)."""

    @staticmethod
    def forward(ctx, qkv, B, Sl, Hq, Hkv, D, scale, cp):
        q, k, v = (_seq_to_heads(t.contiguous(), cp) for t in _split_qkv(qkv, B, Sl, Hq, Hkv, D))
        o, lse = F.attention(q, k, v, scale, True, 0)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.cfg = (B, Sl, Hq, Hkv, D, scale, cp, qkv.shape[1])
        return _heads_to_seq(o, cp).reshape(B * Sl, Hq * D)

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        B, Sl, Hq, Hkv, D, scale, cp, row = ctx.cfg
        doh = _seq_to_heads(do.contiguous().view(B, Sl, Hq, D), cp)
        dq, dk, dv = F.attention_bwd(q, k, v, o, doh, lse, scale, True, 0)
        dqkv = torch.empty(B * Sl, row, dtype=q.dtype, device=q.device)
        d3 = dqkv.view(B, Sl, row)
        d3[:, :, : Hq * D] = _heads_to_seq(dq, cp).reshape(B, Sl, Hq * D)
        d3[:, :, Hq * D : (Hq + Hkv) * D] = _heads_to_seq(dk, cp).reshape(B, Sl, Hkv * D)
        d3[:, :, (Hq + Hkv) * D :] = _heads_to_seq(dv, cp).reshape(B, Sl, Hkv * D)
        return dqkv, None, None, None, None, None, None, None


def cp_attention(qkv, B, Sl, Hq, Hkv, D, scale, cp: CPGroup):
    if cp.mode == "ring":
        return RingAttentionFn.apply(qkv, B, Sl, Hq, Hkv, D, scale, cp)
    if cp.mode == "ulysses":
        assert Hq % cp.world == 0 and Hkv % cp.world == 0, "Ulysses needs the heads divisible by the CP degree"
        return UlyssesAttentionFn.apply(qkv, B, Sl, Hq, Hkv, D, scale, cp)
    return CPAttentionFn.apply(qkv, B, Sl, Hq, Hkv, D, scale, cp)


def shard_sequence(tokens: torch.Tensor, cp: CPGroup):
    """tokens [b, S+1] -> this rank's (ids, targets), each [b, S / cp]."""
    S = tokens.shape[1] - 1
    Sl = S // cp.world
    a = cp.rank * Sl
    return tokens[:, a : a + Sl].contiguous(), tokens[:, a + 1 : a + Sl + 1].contiguous()
