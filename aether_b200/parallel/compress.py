"""Gradient compression for data parallelism: rank-r PowerSGD with error
feedback (Vogels, Karimireddy, Jaggi, "PowerSGD: Practical Low-Rank Gradient
Compression for Distributed Optimization", NeurIPS 2019).

For every weight matrix M (m x n) of the arena's gradient, with this rank's
error e from the previous step:
    M  <- M + e
    P  = M Q                   all-reduce (mean) -> orthonormalise columns
    Q  = M^T P                 all-reduce (mean)
    G  = P Q^T                 the rank-r estimate of the mean gradient
    e  = M - G                 (kept locally; fed back next step)
Each matrix moves (m + n) r values instead of m n. The P's of all matrices
travel in one all-reduce and the Q's in a second. Vectors and matrices too
small to gain are averaged uncompressed in a third. Q is warm-started from
the previous step (one power iteration per step), seeded identically on
every rank.

``CompressedDataParallel`` then runs the same AdamW on every rank over the
whole arena (the compressed estimate is identical everywhere).

Reference: aether_grad_compress_lowrank_f32 (runtime/src/lib.rs:3588) is a
shape-only stand-in (first k columns, identity Q); this is the algorithm
that stub names.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..optim import FlatAdamW


def _orthonormalise_(P: torch.Tensor, tol: float = 1e-5) -> torch.Tensor:
    """Modified Gram-Schmidt over the r columns of P (r small). A column whose
    residual is below ``tol`` of its norm (P has lower rank than r) is set to
    zero: normalising round-off would add a direction that is not orthogonal."""
    for j in range(P.shape[1]):
        c = P[:, j]
        n0 = c.norm()
        for i in range(j):
            c -= torch.dot(P[:, i], c) * P[:, i]
        n = c.norm()
        c *= torch.where(n > tol * n0, 1.0 / n.clamp(min=1e-30), torch.zeros_like(n))
    return P


class PowerSGD:
    def __init__(self, arena, world: int, group=None, rank: int = 4, seed: int = 0):
        self.arena, self.world, self.group, self.r = arena, world, group, rank
        dev = arena.device
        self.mats, self.plain = [], []
        for name, s in arena.slots.items():
            if len(s.shape) == 2:
                m, n = s.shape
                r = min(rank, m, n)
                if (m + n) * r < m * n // 2:
                    self.mats.append((name, s.offset, m, n, r))
                    continue
            self.plain.append((s.offset, s.numel))
        self._gen = torch.Generator(device="cpu").manual_seed(seed)  # same stream on every rank
        self.Q = [torch.randn(n, r, generator=self._gen).to(dev) for _, _, _, n, r in self.mats]
        self.err = [torch.zeros(m, n, dtype=torch.float32, device=dev) for _, _, m, n, _ in self.mats]
        self.p_len = sum(m * r for _, _, m, _, r in self.mats)
        self.q_len = sum(n * r for _, _, _, n, r in self.mats)
        self.plain_len = sum(n for _, n in self.plain)
        self.bytes_dense = 4 * sum(s.numel for s in arena.slots.values())
        self.bytes_sent = 4 * (self.p_len + self.q_len + self.plain_len)

    def _mean_(self, t: torch.Tensor) -> None:
        if self.world > 1:
            dist.all_reduce(t, group=self.group)
            t /= self.world

    def all_reduce_(self) -> None:
        """Replace the arena's gradient with the compressed estimate of the mean over ranks."""
        grad, dev = self.arena.grad, self.arena.device
        Ms = []
        P_all = torch.empty(self.p_len, dtype=torch.float32, device=dev)
        o = 0
        for (name, off, m, n, r), Q, e in zip(self.mats, self.Q, self.err):
            M = grad[off : off + m * n].view(m, n)
            M += e
            Ms.append(M)
            torch.mm(M, Q, out=P_all[o : o + m * r].view(m, r))
            o += m * r
        self._mean_(P_all)
        Q_all = torch.empty(self.q_len, dtype=torch.float32, device=dev)
        o = p = 0
        Ps = []
        for (name, off, m, n, r), M in zip(self.mats, Ms):
            P = _orthonormalise_(P_all[p : p + m * r].view(m, r))
            Ps.append(P)
            torch.mm(M.t(), P, out=Q_all[o : o + n * r].view(n, r))
            o += n * r
            p += m * r
        self._mean_(Q_all)
        o = 0
        for i, ((name, off, m, n, r), M, P) in enumerate(zip(self.mats, Ms, Ps)):
            Q = Q_all[o : o + n * r].view(n, r)
            o += n * r
            G = P @ Q.t()
            torch.sub(M, G, out=self.err[i])
            M.copy_(G)
            self.Q[i].copy_(Q)  # warm start; columns of a rank-deficient step are drawn again
            dead = Q.norm(dim=0) == 0
            if bool(dead.any()):
                self.Q[i][:, dead] = torch.randn(n, int(dead.sum()), generator=self._gen).to(Q.device)
        if self.plain:
            flat = torch.cat([grad[off : off + n] for off, n in self.plain])
            self._mean_(flat)
            o = 0
            for off, n in self.plain:
                grad[off : off + n].copy_(flat[o : o + n])
                o += n


class CompressedDataParallel:
    """DP engine: PowerSGD all-reduce of the gradient, then AdamW on the full
    arena on every rank (same interface as ``parallel.dp.DataParallel``)."""

    def __init__(self, arena, info, rank: int = 4, lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1,
                 group=None):
        self.arena, self.info = arena, info
        self.world = info.world
        self.comp = PowerSGD(arena, info.world, group, rank)
        self.opt = FlatAdamW(arena, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay)
        self.group = group

    def broadcast_params(self) -> None:
        if self.world > 1:
            dist.broadcast(self.arena.master, src=0, group=self.group)
            self.arena.sync_bf16_from_master()

    def step(self, lr: float | None = None) -> None:
        self.comp.all_reduce_()
        self.opt.step(lr=lr)

    def state_dict(self) -> dict:
        return {"opt": self.opt.state_dict(), "powersgd_q": [q.cpu() for q in self.comp.Q],
                "powersgd_err": [e.cpu() for e in self.comp.err]}
