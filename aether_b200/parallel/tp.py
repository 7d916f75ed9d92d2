"""Tensor parallelism for the Qwen serving model.

Megatron layout (reference plan: runtime/src/tensor_parallel.rs:8-29, which
executes on one GPU only): q/k/v heads and gate/up rows column-parallel,
o_proj and down_proj row-parallel, two reductions of [tokens, d_model] per
block. The LM head is split by vocabulary rows (the reference replicates it):
each rank computes the logits of its slice and one kernel merges the ranks'
(max, index) candidates through symmetric memory, so no rank streams the whole
[vocab, d_model] head per token.

Decode reductions, two modes (``AETHER_TP_REDUCE``):
  * ``push`` (default): the row-parallel GEMM accumulates locally; ONE small
    kernel then pushes this rank's fp32 partial row into every rank's inbox
    (NVLS ``multimem.st`` or P2P stores), raises per-row epoch flags, waits
    for every peer's flag and sums -- fused with the residual add and the
    next RMSNorm (``csrc/tp_decode.cu``). No barrier launch, no remote atomics.
  * ``multimem``: the GEMM epilogue reduces its partials through the NVSwitch
    multicast address (``multimem.red``) into every rank's accumulator; at two
    ranks its last CTA signals completion to every peer, at more a device
    barrier kernel follows; then the finalising kernel reads.
Without multicast the push mode uses P2P stores and the multimem mode falls
back to a P2P one-shot all-reduce. Prefill uses the NVLS two-shot all-reduce.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from .._ext import C
from ..ops import functional as F
from .symm import SymmTeam


class TensorParallel:
    def __init__(self, info, timeout_s: float = 30.0, use_multicast: bool | None = None):
        self.info = info
        self.team = SymmTeam(info, timeout_s=timeout_s, use_multicast=use_multicast)
        self.rank, self.world = self.team.rank, self.team.world
        self.device = info.device
        self._stage = None
        self._acc = []
        self._done = torch.zeros(4, dtype=torch.int32, device=self.device)  # CTA counters of the signalling GEMMs
        # Completion signal from the GEMM's last CTA instead of a separate barrier
        # launch. Measured (7B o_proj, batch 1): TP2 16.9 vs 19.0 us per reduction,
        # TP8 26.8 vs 19.7 us -- the signalling GEMM's tail waits for its multimem
        # reductions to reach all 8 ranks -- so it is the default up to 2 ranks.
        env = os.environ.get("AETHER_TP_SIGNAL")  # multimem mode only
        self.signal = (env == "1") if env is not None else self.world <= 2
        t = self.team
        # finalize kernels pass this to F.skinny_finalize / F.finalize_residual_norm(wait=...)
        self.wait = (t.sig.tensor, t.epoch, self.rank, self.world, float(t.timeout_s)) if self.world > 1 else None
        self.mode = os.environ.get("AETHER_TP_REDUCE", "push")
        assert self.mode in ("push", "multimem"), "AETHER_TP_REDUCE: push or multimem"
        self._rows_cap = 0

    # ------------------------------------------------------------------ decode exchange buffers
    def prepare_decode(self, rows_cap: int, width: int, vocab_cols: int) -> None:
        """Allocates (collectively: every rank calls this with the same sizes)
        the symmetric areas of the push reduction and the vocab-parallel head:
        inbox fp32 [2][8][rows_cap][width], flags, argmax records, and a
        full-width logits buffer [rows_cap, vocab_cols]."""
        if self._rows_cap >= rows_cap or self.world == 1:
            return
        t = self.team
        self._rows_cap = rows_cap
        self._width = (width + 3) // 4 * 4
        self._inbox = t.alloc(2 * 8 * rows_cap * self._width, torch.float32)
        self._inflags = t.alloc(2 * 8 * rows_cap, torch.int32)
        self._vrec = t.alloc(2 * 8 * rows_cap * 4, torch.int32)
        self._vfull = t.alloc(rows_cap * vocab_cols, torch.float32)
        self._vcols = vocab_cols
        for b in (self._inbox, self._inflags, self._vrec, self._vfull):
            b.tensor.zero_()
        self._inbox_peers = torch.tensor(self._inbox.peers_host, dtype=torch.int64)
        self._inflag_peers = torch.tensor(self._inflags.peers_host, dtype=torch.int64)
        self._vrec_peers = torch.tensor(self._vrec.peers_host, dtype=torch.int64)
        self._vfull_peers = torch.tensor(self._vfull.peers_host, dtype=torch.int64)
        self._push_ctr = torch.zeros(rows_cap, dtype=torch.int32, device=self.device)
        self._vctr = torch.zeros(rows_cap, dtype=torch.int32, device=self.device)
        torch.cuda.synchronize(self.device)
        dist.barrier()

    def push_reduce(self, acc, y, res=None, bias=None, w=None, h=None, eps=1e-6):
        """y = bf16(sum over ranks of acc[:rows, :N] + bias + res), acc zeroed;
        with w: h = rmsnorm(y) * w. One kernel (see module docstring)."""
        rows = y.shape[0]
        assert rows <= self._rows_cap and y.shape[1] <= self._width, "prepare_decode first"
        C().tp_push_reduce(acc, y, bias, res, w, h, float(eps), self._inbox_peers, int(self._inbox.mc_ptr),
                           self._width, self._inflag_peers, self._push_ctr, self._rows_cap, self.rank, self.world,
                           float(self.team.timeout_s))
        return y

    def vocab_argmax(self, logits, n_loc: int, col0: int, out=None):
        """Greedy token per row over every rank's vocabulary slice: logits
        [rows, >= n_loc] fp32 hold this rank's columns col0 .. col0 + n_loc."""
        rows = logits.shape[0]
        if out is None:
            out = torch.empty(rows, dtype=torch.long, device=logits.device)
        assert rows <= self._rows_cap, "prepare_decode first"
        C().tp_vocab_argmax(logits, int(n_loc), int(col0), self._vrec_peers, self._vctr, self._rows_cap, out,
                            self.rank, self.world, float(self.team.timeout_s))
        return out

    def gather_vocab(self, logits, n_loc: int, col0: int, V: int, out=None):
        """Full [rows, V] fp32 logits from every rank's slice (P2P stores into
        every rank's buffer, then a device barrier)."""
        rows = logits.shape[0]
        assert rows <= self._rows_cap and V <= self._vcols, "prepare_decode first"
        C().tp_put_cols(logits, int(n_loc), int(col0), self._vfull_peers, self._vcols, self.rank, self.world)
        self.team.barrier()
        full = self._vfull.tensor.view(self._rows_cap, self._vcols)[:rows, :V]
        out = full.clone() if out is None else out.copy_(full)
        # no rank may overwrite this rank's buffer before it has been read
        self.team.barrier()
        return out

    # ------------------------------------------------------------------ prefill
    def all_reduce_(self, t: torch.Tensor) -> torch.Tensor:
        n = t.numel()
        if self._stage is None or self._stage.tensor.numel() < n or self._stage.tensor.dtype != t.dtype:
            cap = max(n, 1 << 20)
            self._stage = self.team.alloc(cap, t.dtype)
        buf = self._stage
        buf.tensor[:n].copy_(t.reshape(-1))
        self.team.all_reduce_(buf, n)
        t.copy_(buf.tensor[:n].view_as(t))
        return t

    # ------------------------------------------------------------------ decode
    def _acc_buf(self, which: int, rows: int, cols: int):
        b, r, c = self._acc[which % 2]
        assert rows <= r and cols <= c
        return b, c

    def reduce_gemm(self, x: torch.Tensor, w: torch.Tensor, which: int) -> torch.Tensor:
        """fp32 [M, N] = sum over ranks of x @ w^T, in a symmetric accumulator
        that the following skinny_finalize reads and re-zeroes."""
        M, N = x.shape[0], w.shape[0]
        if not self._acc:
            self._init_acc(M, N)
        b, cols = self._acc_buf(which, M, N)
        acc = b.tensor.view(-1, cols)
        if b.mc_ptr and self.signal:
            t = self.team
            F.skinny_gemm(x, w, acc, acc_mc=b.mc_ptr,
                          signal=(t.peer_sig, t.epoch, self._done[which % 2], self.rank, self.world))
        elif b.mc_ptr:
            F.skinny_gemm(x, w, acc, acc_mc=b.mc_ptr)
            self.team.barrier()
        else:
            F.skinny_gemm(x, w, acc)
            self.team.all_reduce_(b, acc.numel())
        return acc[:M]

    def finalize_wait(self):
        """The ``wait`` argument for the kernel that consumes reduce_gemm's
        output: with multicast the GEMM signals completion itself; without,
        the all-reduce already synchronised."""
        return self.wait if (self.signal and self._acc and self._acc[0][0].mc_ptr) else None

    def _init_acc(self, M: int, N: int) -> None:
        rows = max(M, 64)
        cols = max(N, 8192)
        for _ in range(2):
            b = self.team.alloc(rows * cols, torch.float32)
            b.tensor.zero_()
            self._acc.append((b, rows, cols))
        torch.cuda.synchronize(self.device)
        dist.barrier()

    def max_over_ranks(self, x: float) -> float:
        t = torch.tensor([x], dtype=torch.float64, device=self.device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def close(self) -> None:
        torch.cuda.synchronize(self.device)
        dist.barrier()
