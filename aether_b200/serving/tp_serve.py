"""Serving a tensor-parallel model: rank 0 runs the HTTP server and the
continuous-batching engine; every model call the engine makes (prefill of one
request, one batched decode step) is first broadcast over a CPU control group
(a fixed-size int64 message, no pickling) and then executed, and ranks 1..N-1 replay the same calls on their shard. All
ranks thus launch the same kernels and collectives in the same order (the TP
reductions, NVLS or NCCL, pair up), while sampling, tokenisation and HTTP stay
on rank 0.

The KV cache is the per-slot contiguous one (the paged pool's host-side page
bookkeeping lives in the engine and is not mirrored).

    torchrun --nproc-per-node 8 -m aether_b200.serving.server --model 7b --tp 8

Reference: the tensor-parallel serving session (TpSession,
runtime/src/tensor_parallel.rs) driven by aether-serve.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


_STOP, _PREFILL, _DECODE = 0, 1, 2
_SLOT = 256  # int64 words of the fixed control message: header + inline payload
_HDR = 8


class _Control:
    """The per-call control message, without pickling: one fixed-size int64
    broadcast (header + inline payload) per call, plus one exact-size
    broadcast when the payload does not fit (long prompts). Header:
    [command, B, S, start_pos, flags, payload length, 0, 0]; flags bit 0
    use_graph, bit 1 want_logits, bit 2 slots present, bit 3 return_logits.
    Payload: tokens (B * S), then positions (decode: B), then slots (B)."""

    def __init__(self, group=None):
        self.group = group
        self.buf = torch.zeros(_SLOT, dtype=torch.int64)

    def send(self, cmd: int, B: int = 0, S: int = 0, start: int = 0, flags: int = 0, payload=()) -> None:
        parts = [p.detach().to("cpu", torch.int64).reshape(-1) for p in payload if p is not None]
        data = torch.cat(parts) if parts else torch.zeros(0, dtype=torch.int64)
        n = int(data.numel())
        self.buf.zero_()
        self.buf[:_HDR] = torch.tensor([cmd, B, S, start, flags, n, 0, 0], dtype=torch.int64)
        inline = n <= _SLOT - _HDR
        if inline:
            self.buf[_HDR : _HDR + n] = data
        dist.broadcast(self.buf, src=0, group=self.group)
        if not inline:
            dist.broadcast(data.contiguous(), src=0, group=self.group)

    def recv(self):
        dist.broadcast(self.buf, src=0, group=self.group)
        cmd, B, S, start, flags, n = (int(v) for v in self.buf[:6])
        if n <= _SLOT - _HDR:
            data = self.buf[_HDR : _HDR + n].clone()
        else:
            data = torch.empty(n, dtype=torch.int64)
            dist.broadcast(data, src=0, group=self.group)
        return cmd, B, S, start, flags, data


class BroadcastModel:
    """Rank 0's handle on a TP model: forwards ``prefill`` / ``decode_step`` to
    every rank (``follow``) before running them locally; every other
    attribute is the wrapped model's."""

    def __init__(self, model, group=None):
        self.model = model
        self.ctl = _Control(group)

    def prefill(self, tokens, slots=None, start_pos: int = 0, return_logits: bool = False):
        B, S = tokens.shape
        flags = (4 if slots is not None else 0) | (8 if return_logits else 0)
        self.ctl.send(_PREFILL, B, S, int(start_pos), flags, (tokens, slots))
        return self.model.prefill(tokens, slots=slots, start_pos=start_pos, return_logits=return_logits)

    def decode_step(self, tokens, pos, slots=None, use_graph: bool = True, want_logits: bool = False):
        B = tokens.shape[0]
        flags = (1 if use_graph else 0) | (2 if want_logits else 0) | (4 if slots is not None else 0)
        self.ctl.send(_DECODE, B, 1, 0, flags, (tokens, pos, slots))
        return self.model.decode_step(tokens, pos, slots, use_graph=use_graph, want_logits=want_logits)

    def stop(self) -> None:
        self.ctl.send(_STOP)

    def __getattr__(self, name):
        return getattr(self.model, name)


def follow(model, group=None) -> int:
    """Replay rank 0's model calls on this rank's shard until it sends stop;
    returns the number of calls replayed."""
    dev = model.device
    ctl = _Control(group)
    n = 0
    while True:
        cmd, B, S, start, flags, data = ctl.recv()
        if cmd == _STOP:
            return n
        slots = data[-B:].to(dev, torch.int32) if flags & 4 else None
        if cmd == _PREFILL:
            toks = data[: B * S].view(B, S).to(dev)
            model.prefill(toks, slots=slots, start_pos=start, return_logits=bool(flags & 8))
        elif cmd == _DECODE:
            toks, pos = data[:B].to(dev), data[B : 2 * B].to(dev, torch.int32)
            model.decode_step(toks, pos, slots, use_graph=bool(flags & 1), want_logits=bool(flags & 2))
        else:
            raise ValueError(f"unknown command {cmd}")
        n += 1
