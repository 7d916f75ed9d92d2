"""Fused tensor-parallel training projections (sequence parallelism).

Each Megatron projection of a layer is one ``gemm_tp`` kernel (csrc/gemm_tp.cu)
whose collective runs inside it, tile by tile, over NVLink:

  forward   column (qkv, gate_up)   y  = all_gather(h) . W^T      ag_mode 1
            row    (o_proj, down)   x  = reduce_scatter(o . W^T) + r   rs
  backward  column                  dh = reduce_scatter(dy . W), and h's rows
                                         gathered alongside for dW = dy^T . h_full
            row                     do = all_gather(dx) . W  (the gathered dY
                                         also kept locally for dW = dY^T . o)

so a layer's hot path issues no NCCL call. The buffers live in symmetric
memory (every rank maps every peer's; the rows are pushed with P2P stores,
each rank receiving (tp - 1) / tp of them either way): per activation shape [M, d] a two-slot gather ring ([M, d] bf16 plus
per-chunk flags) and a two-slot receive ring ([tp, M / tp, d] bf16 plus
per-slab counters). Flags only grow (the kernel compares them with the
number of uses of the slot), so they are zeroed once, at allocation.

Reference: runtime/src/tensor_parallel.rs:8-29 (the Megatron plan, executed
there on one GPU with two all-reduces per block).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import functional as F

BM = 128
BN = 256


class _Ring:
    def __init__(self, team, M: int, d: int):
        tp = team.world
        self.M, self.d, self.Ml = M, d, M // tp
        mt = self.Ml // BM
        num_n = (d + BN - 1) // BN
        self.ag = [team.alloc(M * d, torch.bfloat16) for _ in range(2)]
        self.agf = [team.alloc(tp * mt, torch.int32) for _ in range(2)]
        self.rs = [team.alloc(tp * self.Ml * d, torch.bfloat16) for _ in range(2)]
        self.rsf = [team.alloc(mt * num_n * 4, torch.int32) for _ in range(2)]
        for f in self.agf + self.rsf:
            f.tensor.zero_()
        self.n_ag = 0
        self.n_rs = 0

    def next_ag(self):
        slot, ep = self.n_ag & 1, (self.n_ag >> 1) + 1
        self.n_ag += 1
        return slot, ep

    def next_rs(self):
        slot, ep = self.n_rs & 1, (self.n_rs >> 1) + 1
        self.n_rs += 1
        return slot, ep


class FusedTP:
    """The fused projections of one TP group (a ``parallel.symm.SymmTeam``
    over it). Rings are created per activation shape on first use; every rank
    makes the same calls in the same order, so their use counts agree."""

    def __init__(self, team, timeout_s: float = 10.0):
        self.team = team
        self.rank, self.tp = team.rank, team.world
        self.timeout_s = timeout_s
        self.rings: dict[tuple, _Ring] = {}

    def ring(self, M: int, d: int) -> _Ring:
        key = (M, d)
        r = self.rings.get(key)
        if r is None:
            r = _Ring(self.team, M, d)
            torch.cuda.synchronize(self.team.device)
            dist.barrier(group=self.team.group)  # every rank's flags are zero before anyone signals
            self.rings[key] = r
        return r

    def supports(self, rows_local: int) -> bool:
        return rows_local % BM == 0 and rows_local > 0

    def _call(self, a_local, a_ag, b, out, residual, push_src, b_mn, ag_mode, rs, local_copy, ring,
              ag_slot=0, ag_ep=0, rs_slot=0, rs_ep=0):
        ag = ring.ag[ag_slot]
        agf = ring.agf[ag_slot]
        rsb = ring.rs[rs_slot]
        rsf = ring.rsf[rs_slot]
        use_ag = ag_mode != 0
        F.gemm_tp([a_local], [a_ag] if a_ag is not None else [], [b], [out],
                    [residual] if residual is not None else [], [push_src] if push_src is not None else [],
                    [self.rank], self.tp, ring.Ml, b_mn, ag_mode, rs, local_copy,
                    ag.peers_host if use_ag else [], agf.peers_host if use_ag else [],
                    0,  # P2P pushes (the own rows are read back locally; see the kernel's note on multicast)
                    rsb.peers_host if rs else [], rsf.peers_host if rs else [], ag_ep, rs_ep, self.timeout_s)

    # ------------------------------------------------------------------ forward
    def column(self, h: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """y[M, N] = all_gather(h)[M, d] . w[N, d]^T; h is this rank's [M / tp, d]."""
        Ml, d = h.shape
        ring = self.ring(Ml * self.tp, d)
        slot, ep = ring.next_ag()
        y = torch.empty(Ml * self.tp, w.shape[0], dtype=torch.bfloat16, device=h.device)
        self._call(h, ring.ag[slot].tensor.view(ring.M, d), w, y, None, h, False, 1, False, False, ring,
                   ag_slot=slot, ag_ep=ep)
        return y

    def row(self, o: torch.Tensor, w: torch.Tensor, r: torch.Tensor | None) -> torch.Tensor:
        """x[M / tp, d] = this rank's rows of sum_ranks(o . w^T) + r."""
        M = o.shape[0]
        d = w.shape[0]
        ring = self.ring(M, d)
        slot, ep = ring.next_rs()
        x = torch.empty(ring.Ml, d, dtype=torch.bfloat16, device=o.device)
        self._call(o, None, w, x, r, None, False, 0, True, False, ring, rs_slot=slot, rs_ep=ep)
        return x

    # ------------------------------------------------------------------ backward
    def column_bwd(self, dy: torch.Tensor, w: torch.Tensor, h: torch.Tensor):
        """(dh, h_full): dh[M / tp, d] = this rank's rows of sum_ranks(dy . w)
        and h_full[M, d] = all_gather(h), gathered while the GEMM runs."""
        M = dy.shape[0]
        d = w.shape[1]
        ring = self.ring(M, d)
        a_slot, a_ep = ring.next_ag()
        r_slot, r_ep = ring.next_rs()
        dh = torch.empty(ring.Ml, d, dtype=torch.bfloat16, device=dy.device)
        self._call(dy, None, w, dh, None, h, True, 2, True, True, ring, ag_slot=a_slot, ag_ep=a_ep,
                   rs_slot=r_slot, rs_ep=r_ep)
        return dh, ring.ag[a_slot].tensor.view(M, d)

    def row_bwd(self, dx: torch.Tensor, w: torch.Tensor):
        """(do, dy_full): do[M, n] = all_gather(dx) . w with w [d, n], and the
        gathered dy_full[M, d] (this rank's rows copied in as well)."""
        Ml, d = dx.shape
        ring = self.ring(Ml * self.tp, d)
        slot, ep = ring.next_ag()
        g = ring.ag[slot].tensor.view(ring.M, d)
        do = torch.empty(ring.M, w.shape[1], dtype=torch.bfloat16, device=dx.device)
        self._call(dx, g, w, do, None, dx, True, 1, False, True, ring, ag_slot=slot, ag_ep=ep)
        return do, g


class _FusedColumn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, w, tp):
        h = h.contiguous()
        ctx.tp = tp
        ctx.save_for_backward(h, w)
        return tp.fused.column(h, w)

    @staticmethod
    def backward(ctx, dy):
        from .tp_train import _wgrad

        h, w = ctx.saved_tensors
        dy = dy.contiguous()
        dh, hf = ctx.tp.fused.column_bwd(dy, w, h)
        dw = _wgrad(dy, hf, w) if ctx.needs_input_grad[1] else None
        return dh, dw, None


class _FusedRow(torch.autograd.Function):
    @staticmethod
    def forward(ctx, o, w, r, tp):
        o = o.contiguous()
        ctx.tp = tp
        ctx.has_r = r is not None
        ctx.save_for_backward(o, w)
        return tp.fused.row(o, w, r.contiguous() if r is not None else None)

    @staticmethod
    def backward(ctx, dx):
        from .tp_train import _wgrad

        o, w = ctx.saved_tensors
        dx = dx.contiguous()
        do, dyf = ctx.tp.fused.row_bwd(dx, w)
        dw = _wgrad(dyf, o, w) if ctx.needs_input_grad[1] else None
        return do, dw, (dx if ctx.has_r else None), None


def fused_column_linear(h, w, tp):
    return _FusedColumn.apply(h, w, tp)


def fused_row_linear(o, w, r, tp):
    return _FusedRow.apply(o, w, r, tp)
