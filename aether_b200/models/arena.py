"""Flat parameter arena: one fp32 master buffer, one bf16 compute copy, one
fp32 gradient buffer (plus optimiser state owned by the optimiser).

The reference trainer keeps params/grads/adam_m/adam_v in one flat f32 arena
with an offset ``Layout`` (trainer/src/model.rs:14-130); this keeps that idea
and adds the bf16 compute copy. Every tensor starts on a 128-element boundary
(256 B in bf16), which the TMA descriptors of the GEMM need, and the total is
padded so it splits evenly into data-parallel shards.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

ALIGN = 128


@dataclass
class Slot:
    name: str
    shape: tuple
    offset: int
    numel: int
    decay: bool


class ParamArena:
    def __init__(self, specs, device, pad_multiple: int = 1, alloc=None):
        """specs: list of (name, shape, decay: bool). ``alloc(numel, dtype)``
        (optional) provides the bf16 and gradient buffers, e.g. from symmetric
        memory so the data-parallel kernels can reach them from every GPU."""
        self.slots: dict[str, Slot] = {}
        off = 0
        for name, shape, decay in specs:
            n = 1
            for s in shape:
                n *= int(s)
            self.slots[name] = Slot(name, tuple(int(s) for s in shape), off, n, decay)
            off += (n + ALIGN - 1) // ALIGN * ALIGN
        unit = ALIGN * max(1, int(pad_multiple))
        self.numel = (off + unit - 1) // unit * unit
        self.n_params = sum(s.numel for s in self.slots.values())
        self.device = torch.device(device)
        self.master = torch.zeros(self.numel, dtype=torch.float32, device=self.device)
        if alloc is None:
            self.bf16 = torch.zeros(self.numel, dtype=torch.bfloat16, device=self.device)
            self.grad = torch.zeros(self.numel, dtype=torch.float32, device=self.device)
        else:
            self.bf16 = alloc(self.numel, torch.bfloat16)
            self.grad = alloc(self.numel, torch.float32)
            self.bf16.zero_()
            self.grad.zero_()
        self.decay_mask = torch.zeros(self.numel, dtype=torch.bool)
        for s in self.slots.values():
            if s.decay:
                self.decay_mask[s.offset : s.offset + s.numel] = True
        self._views: dict[str, torch.Tensor] = {}
        for s in self.slots.values():
            v = self.bf16[s.offset : s.offset + s.numel].view(s.shape)
            v.requires_grad_(True)
            v.main_grad = self.grad[s.offset : s.offset + s.numel].view(s.shape)
            self._views[s.name] = v

    def __getitem__(self, name: str) -> torch.Tensor:
        return self._views[name]

    def master_view(self, name: str) -> torch.Tensor:
        s = self.slots[name]
        return self.master[s.offset : s.offset + s.numel].view(s.shape)

    def set_full(self, name: str, t: torch.Tensor) -> None:
        """Initialise parameter ``name`` from its full fp32 value."""
        self.master_view(name).copy_(t.to(self.device, torch.float32))

    def names(self):
        return list(self.slots.keys())

    def sync_bf16_from_master(self) -> None:
        with torch.no_grad():
            self.bf16.copy_(self.master.to(torch.bfloat16))

    def zero_grad(self) -> None:
        self.grad.zero_()

    def state_dict(self) -> dict:
        return {n: self.master_view(n).detach().cpu().clone() for n in self.names()}

    def load_state_dict(self, sd: dict) -> None:
        with torch.no_grad():
            for n in self.names():
                self.master_view(n).copy_(sd[n].to(self.master.device, torch.float32))
        self.sync_bf16_from_master()
