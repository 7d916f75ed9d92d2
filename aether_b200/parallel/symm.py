"""Symmetric-memory team: buffers every rank maps into every peer (P2P) plus,
where NVSwitch multicast is available, one NVLS multicast address per buffer.

Built on ``torch.distributed._symmetric_memory`` for allocation and the
exchange of handles; all data movement on the hot paths is done by this
library's own kernels (``csrc/comm.cu``): a bounded cross-GPU barrier, NVLS /
P2P all-reduce, the fused data-parallel reduce + AdamW + broadcast, and the
multicast-reduce epilogue of the tensor-parallel decode GEMM.
"""
from __future__ import annotations

import os
from dataclasses import dataclass

import torch
import torch.distributed as dist

from .._ext import C

MAX_WORLD = 8


@dataclass
class SymmBuffer:
    tensor: torch.Tensor          # this rank's local view
    peers_dev: torch.Tensor       # CUDA int64 [world] peer base pointers
    peers_host: list              # same, host ints
    mc_ptr: int                   # multicast base address (0 if unavailable)
    handle: object

    def mc_at(self, elem_offset: int) -> int:
        return self.mc_ptr + elem_offset * self.tensor.element_size() if self.mc_ptr else 0


class SymmTeam:
    def __init__(self, info, group=None, timeout_s: float = 10.0, use_multicast: bool | None = None):
        import torch.distributed._symmetric_memory as symm_mem

        self._symm = symm_mem
        assert dist.is_initialized(), "SymmTeam needs an initialised process group"
        self.group = group or dist.group.WORLD
        self.group_name = self.group.group_name
        self.rank = dist.get_rank(self.group)
        self.world = dist.get_world_size(self.group)
        assert self.world <= MAX_WORLD
        self.device = info.device
        self.timeout_s = timeout_s
        if use_multicast is None:
            use_multicast = os.environ.get("AETHER_NO_MULTICAST", "0") != "1"
        self.use_multicast = use_multicast
        self.buffers: list[SymmBuffer] = []
        sig = self.alloc(MAX_WORLD * 32, torch.int32)  # signal slots (first MAX_WORLD used)
        sig.tensor.zero_()
        self.sig = sig
        self.peer_sig = torch.tensor(sig.peers_host, dtype=torch.int64)
        self.epoch = torch.zeros(1, dtype=torch.int32, device=self.device)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)

    def alloc(self, numel: int, dtype) -> SymmBuffer:
        t = self._symm.empty(numel, dtype=dtype, device=self.device)
        h = self._symm.rendezvous(t, self.group_name)
        ptrs = [int(p) for p in h.buffer_ptrs]
        mc = int(getattr(h, "multicast_ptr", 0) or 0) if self.use_multicast else 0
        b = SymmBuffer(t, torch.tensor(ptrs, dtype=torch.int64, device=self.device), ptrs, mc, h)
        self.buffers.append(b)
        return b

    def find(self, t: torch.Tensor) -> SymmBuffer:
        for b in self.buffers:
            if b.tensor.data_ptr() == t.data_ptr():
                return b
        raise KeyError("tensor is not a symmetric buffer of this team")

    @property
    def has_multicast(self) -> bool:
        return all(b.mc_ptr != 0 for b in self.buffers[:1])

    def barrier(self) -> None:
        """Device-side barrier on the current stream (graph-capturable)."""
        C().team_barrier(self.peer_sig, self.sig.tensor, self.epoch, self.rank, self.world, self.timeout_s)

    def all_reduce_(self, buf: SymmBuffer, numel: int | None = None) -> torch.Tensor:
        """In-place sum across ranks of the first numel elements of a symmetric buffer."""
        n = numel or buf.tensor.numel()
        self.barrier()
        if buf.mc_ptr:
            C().allreduce_nvls(buf.mc_ptr, n, buf.tensor.dtype == torch.bfloat16, self.rank, self.world)
            self.barrier()
            return buf.tensor[:n]
        tmp = torch.empty(n, dtype=buf.tensor.dtype, device=self.device)
        C().allreduce_oneshot(buf.peers_dev, tmp, self.world)
        self.barrier()
        buf.tensor[:n].copy_(tmp)
        return buf.tensor[:n]
