"""Sharded data parallelism: ZeRO-2 (gradients and optimiser state sharded)
and ZeRO-3 / FSDP (parameters sharded too), one unit per transformer layer.

Layout. Every layer is a unit; the embeddings, final norm and LM head form the
root unit. A unit's parameters are laid out flat (each on a 128-element
boundary, the unit padded to a multiple of world * 128), and rank r holds the
slice [r L / w, (r+1) L / w) of every unit: fp32 master, AdamW m / v, fp32
gradient and bf16 copy, concatenated over units into one flat shard that
``FlatAdamW`` updates like any arena.

Parameters (stage 3). A layer's bf16 parameters are all-gathered into one of
two rotating unit buffers when the layer first touches them, and the gather
of the next layer is issued at the same time (async NCCL, so it overlaps this
layer's GEMMs). Autograd does not keep the gathered weights alive: a
saved-tensor hook replaces every parameter view by its (unit, name) key, and
backward gathers the unit again when its first op unpacks a weight,
prefetching the unit below. The root unit stays gathered from its first use to
the optimiser step. Stage 2 keeps a full bf16 copy instead, refreshed by one
all-gather per unit after each step.

Gradients (stages 2 and 3). A unit's weight gradients accumulate into one of
two rotating fp32 unit buffers (the GEMM epilogues reduce into ``main_grad``).
When backward reaches the next unit, the finished buffer is reduce-scattered
asynchronously into a shard-sized scratch, added into the gradient shard when
the buffer is next needed; a callback at the end of backward flushes the last
units. Micro-batches accumulate into the shard.

Per-rank bytes per parameter: 18 / world (master, m, v, gradient, bf16) plus
two layer units of bf16 and fp32 buffers and the root unit; stage 2 adds the
full bf16 copy (2 bytes per parameter).

Reference: the ZeRO-1/2/3 byte accounting (runtime/src/lib.rs:3525) and the
FSDP shard / all-gather / reduce-scatter round trip (runtime/src/lib.rs:3627)
are in-process simulations there; this is the engine they model.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from ..models.arena import ALIGN, Slot
from ..ops import autograd as A
from ..optim import FlatAdamW

ROOT = -1


@dataclass
class ShardSpec:
    rank: int
    world: int
    stage: int = 3  # 2: gradients + optimiser state sharded; 3: parameters too
    group: object = None
    # stage 3 on GPUs: a parallel.symm.SymmTeam over `group`. Each layer's
    # parameter all-gather then runs inside its first consuming GEMM (the
    # gemm_param_gather kernel) instead of an NCCL call.
    fused: object = None


# elements per flag of the fused parameter gather (a layer unit is padded to
# a multiple of world * FUSED_CHUNK)
FUSED_CHUNK = 16384


def _unit_of(name: str, fused: bool = False) -> int:
    if fused and name.split(".")[-1].endswith("norm"):
        return ROOT  # norm weights are read by row kernels before any GEMM: keep them gathered
    if name.startswith("l") and "." in name:
        head = name.split(".", 1)[0][1:]
        if head.isdigit():
            return int(head)
    return ROOT


class _Unit:
    def __init__(self, uid: int, specs, world: int, quantum: int = ALIGN):
        self.uid = uid
        self.slots: dict[str, Slot] = {}
        off = 0
        for name, shape, decay in specs:
            n = 1
            for s in shape:
                n *= int(s)
            self.slots[name] = Slot(name, tuple(int(s) for s in shape), off, n, decay)
            off += (n + ALIGN - 1) // ALIGN * ALIGN
        unit = quantum * world
        self.numel = max(unit, (off + unit - 1) // unit * unit)
        self.shard = self.numel // world
        self.offset = 0  # of this unit's slice inside the rank's flat shard


class _StreamWork:
    """Completion of work queued on a side stream (the wait is on the device)."""

    def __init__(self, event):
        self.event = event

    def wait(self):
        torch.cuda.current_stream().wait_event(self.event)


class ShardedArena:
    """The arena of a ZeRO-2 / ZeRO-3 model. ``master`` / ``bf16`` / ``grad`` /
    ``decay_mask`` cover this rank's flat shard (what the optimiser updates);
    ``arena[name]`` is the full bf16 parameter, gathered on demand."""

    def __init__(self, specs, device, spec: ShardSpec):
        self.spec = spec
        self.rank, self.world, self.stage, self.group = spec.rank, spec.world, spec.stage, spec.group
        assert self.stage in (2, 3)
        self.device = torch.device(device)
        self.team = spec.fused if (spec.fused is not None and self.stage == 3 and self.world > 1
                                   and self.device.type == "cuda") else None
        fused = self.team is not None
        by_unit: dict[int, list] = {}
        for sp in specs:
            by_unit.setdefault(_unit_of(sp[0], fused), []).append(sp)
        order = sorted(u for u in by_unit if u != ROOT) + ([ROOT] if ROOT in by_unit else [])
        self.units: dict[int, _Unit] = {}
        off = 0
        for u in order:
            unit = _Unit(u, by_unit[u], self.world, FUSED_CHUNK if (fused and u != ROOT) else ALIGN)
            unit.offset = off
            off += unit.shard
            self.units[u] = unit
        self.layer_ids = [u for u in order if u != ROOT]
        self.unit_of = {name: u for u, unit in self.units.items() for name in unit.slots}
        self.slots = {name: unit.slots[name] for unit in self.units.values() for name in unit.slots}
        self.numel = off
        self.n_params = sum(s.numel for s in self.slots.values())
        dev = self.device
        self.master = torch.zeros(off, dtype=torch.float32, device=dev)
        self.bf16 = torch.zeros(off, dtype=torch.bfloat16, device=dev)
        self.grad = torch.zeros(off, dtype=torch.float32, device=dev)
        self.decay_mask = torch.zeros(off, dtype=torch.bool)
        for unit in self.units.values():
            lo = self.rank * unit.shard
            for s in unit.slots.values():
                a, b = max(s.offset, lo), min(s.offset + s.numel, lo + unit.shard)
                if s.decay and a < b:
                    self.decay_mask[unit.offset + a - lo : unit.offset + b - lo] = True
        layer_max = max([self.units[u].numel for u in self.layer_ids], default=ALIGN)
        root_n = self.units[ROOT].numel if ROOT in self.units else 0
        # parameter storage: stage 2 keeps every unit; stage 3 two rotating layer buffers + the root
        if self.stage == 2:
            self._full = torch.zeros(sum(u.numel for u in self.units.values()), dtype=torch.bfloat16, device=dev)
            base = 0
            self._pbuf = {}
            for u, unit in self.units.items():
                self._pbuf[u] = self._full[base : base + unit.numel]
                base += unit.numel
        elif fused:
            # symmetric memory: every rank's unit buffers, gather flags and
            # readiness words, mapped into every peer
            t = self.team
            self._psym = [t.alloc(layer_max, torch.bfloat16) for _ in range(2)]
            self._pslots = [b.tensor for b in self._psym]
            self._pflags = [t.alloc(max(1, layer_max // FUSED_CHUNK), torch.int32) for _ in range(2)]
            self._pready = [t.alloc(self.world, torch.int32) for _ in range(2)]
            for b in self._pflags + self._pready:
                b.tensor.zero_()
            self._pctr = [torch.zeros(2, dtype=torch.int32, device=dev) for _ in range(2)]
            self._puses = [0, 0]
            A.PG_ARENAS.add(self)  # its pending gathers run inside the GEMMs that read them
            self._proot = torch.zeros(root_n, dtype=torch.bfloat16, device=dev)
            torch.cuda.synchronize(dev)
            dist.barrier(group=self.group)  # every rank's flags are zero before anyone signals
        else:
            self._pslots = [torch.zeros(layer_max, dtype=torch.bfloat16, device=dev) for _ in range(2)]
            self._proot = torch.zeros(root_n, dtype=torch.bfloat16, device=dev)
        if fused:
            # layer gradients in symmetric memory: each rank sums its shard range
            # out of every peer's buffer with its own kernel (no NCCL per layer)
            self._gsym = [self.team.alloc(layer_max, torch.float32) for _ in range(2)]
            self._gslots = [b.tensor for b in self._gsym]
            for g in self._gslots:
                g.zero_()
            self._rs_stream = torch.cuda.Stream(device=dev)
            self._rs_peers = {}
        else:
            self._gslots = [torch.zeros(layer_max, dtype=torch.float32, device=dev) for _ in range(2)]
        self._groot = torch.zeros(root_n, dtype=torch.float32, device=dev)
        # AETHER_FSDP_FUSED_RS=0 keeps the fused parameter gathers but reduces
        # gradients with NCCL (to tell the two apart)
        import os as _os

        self._fused_rs = fused and _os.environ.get("AETHER_FSDP_FUSED_RS", "1") != "0"
        self._scratch = {i: torch.zeros(layer_max // self.world, dtype=torch.float32, device=dev) for i in (0, 1)}
        self._scratch[ROOT] = torch.zeros(max(1, root_n // self.world), dtype=torch.float32, device=dev)
        self._reset_state()

    # ------------------------------------------------------------ bookkeeping
    def _reset_state(self):
        self._resident = {}  # unit -> (param buffer, pending gather work or None)
        self._pending = {}  # fused mode: unit -> slot whose gather waits for the unit's first GEMM
        self._pslot_owner = [None, None]
        self._cur_fwd = None
        self._gslot_owner = [None, None]  # unit whose gradient sits in the slot
        self._gslot_seq = [0, 0]  # assignment order, to recycle the older slot
        self._seq = 0
        self._gpending = {}  # slot key -> (work, unit)
        self._groot_live = False
        self._bwd_unit = None
        self._bwd_active = False
        self._views = {}
        self._grad_keys = {}  # unit -> keys it registered in the autograd gradient-buffer table

    def names(self):
        return list(self.slots.keys())

    def _shard_of(self, u: int, buf: torch.Tensor) -> torch.Tensor:
        unit = self.units[u]
        return buf[unit.offset : unit.offset + unit.shard]

    def set_full(self, name: str, t: torch.Tensor) -> None:
        """Initialise parameter ``name`` from its full fp32 value (every rank
        passes the same tensor and keeps its slice)."""
        self.scatter_full(name, t, self.master)

    def scatter_full(self, name: str, t: torch.Tensor, buf: torch.Tensor) -> None:
        """Write this rank's slice of parameter ``name`` (full value ``t``) into
        ``buf``, a shard-layout buffer (master weights or optimiser moments)."""
        u = self.unit_of[name]
        unit, s = self.units[u], self.slots[name]
        lo = self.rank * unit.shard
        flat = t.reshape(-1).to(torch.float32)
        a, b = max(s.offset, lo), min(s.offset + s.numel, lo + unit.shard)
        if a < b:
            buf[unit.offset + a - lo : unit.offset + b - lo].copy_(flat[a - s.offset : b - s.offset].to(buf.device))

    def layout(self) -> dict:
        """Unit id -> [offset in this rank's shard, shard length, unit length,
        {name: [shape, offset in unit, numel, decay]}] (checkpoint metadata)."""
        return {str(u): [unit.offset, unit.shard, unit.numel,
                         {n: [list(sl.shape), sl.offset, sl.numel, sl.decay] for n, sl in unit.slots.items()}]
                for u, unit in self.units.items()}

    def sync_bf16_from_master(self) -> None:
        with torch.no_grad():
            self.bf16.copy_(self.master.to(torch.bfloat16))
        self.params_updated()

    def zero_grad(self) -> None:
        self.grad.zero_()

    # ------------------------------------------------------------ collectives
    def _all_gather(self, out: torch.Tensor, shard: torch.Tensor, async_op: bool):
        if self.world == 1:
            out.copy_(shard)
            return None
        if out.is_cuda:
            return dist.all_gather_into_tensor(out, shard, group=self.group, async_op=async_op)
        parts = [torch.empty_like(shard) for _ in range(self.world)]
        dist.all_gather(parts, shard, group=self.group)
        out.copy_(torch.cat(parts))
        return None

    def _reduce_scatter(self, out: torch.Tensor, full: torch.Tensor):
        if self.world == 1:
            out.copy_(full)
            return None
        if full.is_cuda:
            return dist.reduce_scatter_tensor(out, full, group=self.group, async_op=True)
        t = full.clone()
        dist.all_reduce(t, group=self.group)
        out.copy_(t[self.rank * out.numel() : (self.rank + 1) * out.numel()])
        return None

    # ------------------------------------------------------------ parameters
    def params_updated(self) -> None:
        """The bf16 shard changed (optimiser step, load): refresh / invalidate the gathered copies."""
        self._finish_grads()
        self._reset_state()
        if self.stage == 2:
            for u in self.units:
                self._all_gather(self._pbuf[u][: self.units[u].numel], self._shard_of(u, self.bf16), False)

    def _gather(self, u: int, async_op: bool):
        unit = self.units[u]
        if u == ROOT:
            buf = self._proot
        else:
            k = 0 if self._pslot_owner[0] is None else 1 if self._pslot_owner[1] is None else None
            if k is None:  # evict the slot that does not hold the unit in use
                busy = {self._cur_fwd, self._bwd_unit}
                k = 0 if self._pslot_owner[0] not in busy else 1
            old = self._pslot_owner[k]
            if old is not None:
                self._resident.pop(old, None)
                self._pending.pop(old, None)
            self._pslot_owner[k] = u
            buf = self._pslots[k]
            if self.team is not None:
                # no transfer now: the unit's first GEMM gathers it (pg_gemm)
                self._pending[u] = k
                self._resident[u] = (buf, None)
                return
        work = self._all_gather(buf[: unit.numel], self._shard_of(u, self.bf16), async_op)
        self._resident[u] = (buf, work)

    def _ensure(self, u: int) -> torch.Tensor:
        if self.stage == 2:
            return self._pbuf[u]
        if u not in self._resident:
            self._gather(u, async_op=False)
        buf, work = self._resident[u]
        if work is not None:
            work.wait()
            self._resident[u] = (buf, None)
        return buf

    def _prefetch(self, u: int | None) -> None:
        if self.team is not None:
            return  # fused mode gathers inside the consuming GEMM, overlapped there
        if self.stage == 3 and u is not None and u not in self._resident:
            self._gather(u, async_op=self.device.type == "cuda")

    def pending_at(self, w: torch.Tensor):
        """The unit whose still-pending gather covers w's memory, or None
        (ops.autograd._gemm_w asks before every linear GEMM)."""
        if not self._pending or not w.is_cuda:
            return None
        p = w.data_ptr()
        for u, k in self._pending.items():
            base = self._pslots[k].data_ptr()
            if base <= p < base + self.units[u].numel * 2:
                return u
        return None

    def pg_gemm(self, u: int, x: torch.Tensor, w: torch.Tensor, b_mn: bool = False, residual=None):
        """x . w^T (b_mn: x . w) as the first consumer of unit u's still-pending
        gather: one kernel moves every rank's shard into every rank's unit
        buffer and multiplies as the weight's chunks arrive. None when u is
        already gathered (the caller runs a plain GEMM)."""
        k = self._pending.get(u)
        if k is None:
            return None
        if residual is not None or not x.is_contiguous():
            self._complete(u)  # a form the gather kernel does not take: plain gather first
            return None
        del self._pending[u]
        from ..ops import functional as F

        unit = self.units[u]
        self._puses[k] += 1
        out = torch.empty(x.shape[0], w.shape[1] if b_mn else w.shape[0], dtype=torch.bfloat16, device=x.device)
        sym, fl, rd = self._psym[k], self._pflags[k], self._pready[k]
        F.gemm_param_gather([x], [w], [out], [self._shard_of(u, self.bf16)], [self._pctr[k]], [self.rank],
                              self.world, FUSED_CHUNK, b_mn, sym.peers_host, fl.peers_host, rd.peers_host,
                              0, self._puses[k], 10.0)  # P2P pushes: this rank reads its own chunks back
        return out

    def _complete(self, u: int) -> None:
        """Gathers a pending unit without a GEMM (NCCL) -- for consumers the
        fused kernel does not cover."""
        k = self._pending.pop(u, None)
        if k is not None:
            unit = self.units[u]
            self._all_gather(self._pslots[k][: unit.numel], self._shard_of(u, self.bf16), False)

    def _view(self, name: str, buf: torch.Tensor) -> torch.Tensor:
        s = self.slots[name]
        v = buf[s.offset : s.offset + s.numel].view(s.shape)
        v.requires_grad_(True)
        v._fsdp_name = name
        return v

    def __getitem__(self, name: str) -> torch.Tensor:
        u = self.unit_of[name]
        if self.stage == 2:
            v = self._views.get(name)
            if v is None:
                v = self._views[name] = self._view(name, self._pbuf[u])
            return v
        if u != ROOT and u != self._cur_fwd:
            self._cur_fwd = u
            buf = self._ensure(u)
            i = self.layer_ids.index(u)
            self._prefetch(self.layer_ids[i + 1] if i + 1 < len(self.layer_ids) else None)
            return self._view(name, buf)
        key = (u, name)
        v = self._views.get(key)
        if v is None or u != ROOT:
            v = self._view(name, self._ensure(u))
            if u == ROOT:
                self._views[key] = v
        return v

    # ------------------------------------------------------------ gradients
    def _grad_buf(self, u: int) -> torch.Tensor:
        """The fp32 buffer unit u's gradients accumulate into during this backward."""
        if u == ROOT:
            if not self._groot_live:
                self._drain(ROOT)  # the previous micro-batch's root gradient
                self._groot.zero_()
                self._groot_live = True
            return self._groot
        for k in (0, 1):
            if self._gslot_owner[k] == u and k not in self._gpending:
                return self._gslots[k]
        k = 0 if self._gslot_owner[0] is None else 1 if self._gslot_owner[1] is None else None
        if k is None:  # recycle the slot assigned longer ago (its reduce-scatter started first)
            k = 0 if self._gslot_seq[0] < self._gslot_seq[1] else 1
        self._drain(k)
        self._seq += 1
        self._gslot_owner[k] = u
        self._gslot_seq[k] = self._seq
        g = self._gslots[k]
        g[: self.units[u].numel].zero_()
        return g

    def _flush(self, u: int) -> None:
        """Start the reduce-scatter of unit u's finished gradient buffer."""
        for key in self._grad_keys.pop(u, ()):
            A.MAIN_GRADS.pop(key, None)
        unit = self.units[u]
        if u == ROOT:
            if not self._groot_live:
                return
            key, full = ROOT, self._groot
            self._groot_live = False
        else:
            ks = [k for k in (0, 1) if self._gslot_owner[k] == u and k not in self._gpending]
            if not ks:
                return
            key, full = ks[0], self._gslots[ks[0]]
        out = self._scratch[key][: unit.shard]
        if self.team is not None and key != ROOT and self._fused_rs:
            self._gpending[key] = (self._reduce_scatter_fused(key, u, out), u)
            return
        self._gpending[key] = (self._reduce_scatter(out, full[: unit.numel]), u)

    def _reduce_scatter_fused(self, key: int, u: int, out: torch.Tensor) -> "_StreamWork":
        """Unit u's gradient (slot `key`) reduce-scattered by this library's
        kernels on a side stream, overlapped with the backward of the layers
        below: a bounded barrier (every rank's unit gradient is complete), a
        one-shot sum of this rank's shard range over every peer's buffer (P2P
        loads), a second barrier (every peer has read this rank's buffer, so
        the slot may be zeroed again)."""
        from .._ext import C

        unit = self.units[u]
        tab = self._rs_peers.get((key, u))
        if tab is None:
            off = self.rank * unit.shard * 4
            tab = torch.tensor([p + off for p in self._gsym[key].peers_host], dtype=torch.int64, device=self.device)
            self._rs_peers[(key, u)] = tab
        ready = torch.cuda.Event()
        ready.record(torch.cuda.current_stream(self.device))
        side = self._rs_stream
        with torch.cuda.stream(side):
            side.wait_event(ready)
            self.team.barrier()
            C().allreduce_oneshot(tab, out, self.world)
            self.team.barrier()
            done = torch.cuda.Event()
            done.record(side)
        out.record_stream(side)
        return _StreamWork(done)

    def _drain(self, key) -> None:
        """Wait for slot ``key``'s reduce-scatter and add it into the gradient shard."""
        p = self._gpending.pop(key, None)
        if p is None:
            if key != ROOT:
                self._gslot_owner[key] = None
            return
        work, u = p
        if work is not None:
            work.wait()
        unit = self.units[u]
        self._shard_of(u, self.grad).add_(self._scratch[key][: unit.shard])
        if key != ROOT:
            self._gslot_owner[key] = None

    def _finish_grads(self) -> None:
        for k in (0, 1):
            if self._gslot_owner[k] is not None and k not in self._gpending:
                self._flush(self._gslot_owner[k])
        self._flush(ROOT)
        for key in list(self._gpending):
            self._drain(key)
        self._gslot_owner = [None, None]

    def _end_backward(self) -> None:
        self._bwd_active = False
        self._bwd_unit = None
        for k in (0, 1):
            if self._gslot_owner[k] is not None and k not in self._gpending:
                self._flush(self._gslot_owner[k])
        self._flush(ROOT)
        self._cur_fwd = None

    def _unpack_param(self, name: str) -> torch.Tensor:
        u = self.unit_of[name]
        if not self._bwd_active:
            self._bwd_active = True
            self._cur_fwd = None
            torch.autograd.Variable._execution_engine.queue_callback(self._end_backward)
        if u != ROOT and u != self._bwd_unit:
            if self._bwd_unit is not None:
                self._flush(self._bwd_unit)
            self._bwd_unit = u
            if self.stage == 3:
                buf = self._ensure(u)
                i = self.layer_ids.index(u)
                self._prefetch(self.layer_ids[i - 1] if i > 0 else None)
        g = self._grad_buf(u)
        s = self.slots[name]
        if u == ROOT or self.stage == 2:
            v = self[name]
        else:
            v = self._view(name, self._ensure(u))
        # autograd hands backward a new tensor over the same memory: register
        # the gradient buffer by address
        key = (v.data_ptr(), v.numel())
        A.MAIN_GRADS[key] = g[s.offset : s.offset + s.numel].view(s.shape)
        self._grad_keys.setdefault(u, []).append(key)
        return v

    def autograd_hooks(self):
        """Context for the forward pass: parameter views are saved as keys and
        re-materialised (gathered, with their gradient buffer) in backward."""

        def pack(t):
            name = getattr(t, "_fsdp_name", None)
            return t if name is None else ("fsdp", name)

        def unpack(p):
            if isinstance(p, tuple) and len(p) == 2 and p[0] == "fsdp":
                return self._unpack_param(p[1])
            return p

        self._cur_fwd = None
        if ROOT in self.units:
            self._root_main_grad()
        return torch.autograd.graph.saved_tensors_hooks(pack, unpack)

    def _root_main_grad(self) -> None:
        """Root parameters whose backward reads ``main_grad`` from the tensor
        the forward saw (the embedding keeps its table on ctx) get the root
        gradient buffer attached up front."""
        g = self._grad_buf(ROOT)
        for name, s in self.units[ROOT].slots.items():
            v = self[name]
            v.main_grad = g[s.offset : s.offset + s.numel].view(s.shape)

    # ------------------------------------------------------------ state
    def full_state(self) -> dict:
        """Every parameter's full fp32 master value (collective: all ranks call)."""
        out = {}
        for u, unit in self.units.items():
            full = torch.empty(unit.numel, dtype=torch.float32, device=self.device)
            self._all_gather(full, self._shard_of(u, self.master).contiguous(), False)
            for name, s in unit.slots.items():
                out[name] = full[s.offset : s.offset + s.numel].view(s.shape).cpu().clone()
        return out


class ShardedDataParallel:
    """Optimiser engine for a model built with ``shard=ShardSpec(...)``: AdamW
    on this rank's shard (gradient x 1/world), then refresh the parameters."""

    def __init__(self, arena: ShardedArena, lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1):
        self.arena = arena
        self.world = arena.world
        self.opt = FlatAdamW(arena, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay)

    def broadcast_params(self) -> None:
        self.arena.sync_bf16_from_master()

    def step(self, lr: float | None = None) -> None:
        a = self.arena
        a._finish_grads()
        self.opt.step(lr=lr, gscale=1.0 / self.world)
        a.params_updated()

    def state_dict(self) -> dict:
        return {"opt": self.opt.state_dict()}


def stage_bytes(n_params: int, world: int, stage: int) -> int:
    """Per-rank bytes of persistent training state under ZeRO stage 1 / 2 / 3
    in this package (fp32 master, AdamW m / v, fp32 gradient, bf16 copy),
    excluding the per-unit working buffers."""
    n, w = n_params, world
    if stage == 1:
        return 2 * n + 4 * n + (4 + 4 + 4) * n // w
    if stage == 2:
        return 2 * n + (4 + 4 + 4 + 4 + 2) * n // w
    if stage == 3:
        return (4 + 4 + 4 + 4 + 2) * n // w
    raise ValueError("stage must be 1, 2 or 3")

