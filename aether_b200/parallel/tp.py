"""Tensor parallelism for the Qwen serving model.

Megatron layout (reference plan: runtime/src/tensor_parallel.rs:8-29, which
executes on one GPU only): q/k/v heads and gate/up rows column-parallel,
o_proj and down_proj row-parallel, two reductions of [tokens, d_model] per
block. Decode runs each row-parallel layer as ONE kernel: the split-K
swap-AB tcgen05 GEMM's epilogue reduces its fp32 partials through the
NVSwitch multicast address (``multimem.red``) into every rank's accumulator;
at two ranks its last CTA then raises this rank's epoch in every peer's signal
slot and the finalising kernel (bias / residual (+ RMSNorm) -> bf16) waits for
all ranks' slots before it reads (no separate barrier launch); at more ranks a
device barrier kernel sits between the two, which measured faster there. Without multicast
the partials go to a local accumulator and a P2P one-shot all-reduce. Prefill
uses the NVLS two-shot all-reduce kernel.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

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
        import os

        env = os.environ.get("AETHER_TP_SIGNAL")
        self.signal = (env == "1") if env is not None else self.world <= 2
        t = self.team
        # finalize kernels pass this to F.skinny_finalize / F.finalize_residual_norm(wait=...)
        self.wait = (t.sig.tensor, t.epoch, self.rank, self.world, float(t.timeout_s)) if self.world > 1 else None

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
