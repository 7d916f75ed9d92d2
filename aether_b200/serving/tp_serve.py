"""Serving a tensor-parallel model: rank 0 runs the HTTP server and the
continuous-batching engine; every model call the engine makes (prefill of one
request, one batched decode step) is first broadcast over a CPU control group
and then executed, and ranks 1..N-1 replay the same calls on their shard. All
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


def _cpu(t):
    return t.detach().to("cpu") if isinstance(t, torch.Tensor) else t


class BroadcastModel:
    """Rank 0's handle on a TP model: forwards ``prefill`` / ``decode_step`` to
    every rank (``follow``) before running them locally; every other
    attribute is the wrapped model's."""

    def __init__(self, model, group=None):
        self.model = model
        self.group = group

    def _send(self, cmd) -> None:
        dist.broadcast_object_list([cmd], src=0, group=self.group)

    def prefill(self, tokens, slots=None, start_pos: int = 0, return_logits: bool = False):
        self._send(("prefill", _cpu(tokens), _cpu(slots), int(start_pos), bool(return_logits)))
        return self.model.prefill(tokens, slots=slots, start_pos=start_pos, return_logits=return_logits)

    def decode_step(self, tokens, pos, slots=None, use_graph: bool = True, want_logits: bool = False):
        self._send(("decode", _cpu(tokens), _cpu(pos), _cpu(slots), bool(use_graph), bool(want_logits)))
        return self.model.decode_step(tokens, pos, slots, use_graph=use_graph, want_logits=want_logits)

    def stop(self) -> None:
        self._send(("stop",))

    def __getattr__(self, name):
        return getattr(self.model, name)


def follow(model, group=None) -> int:
    """Replay rank 0's model calls on this rank's shard until it sends stop;
    returns the number of calls replayed."""
    dev = model.device
    n = 0
    while True:
        box = [None]
        dist.broadcast_object_list(box, src=0, group=group)
        cmd = box[0]
        if cmd[0] == "stop":
            return n
        if cmd[0] == "prefill":
            _, toks, slots, start, want = cmd
            model.prefill(toks.to(dev), slots=None if slots is None else slots.to(dev), start_pos=start,
                          return_logits=want)
        elif cmd[0] == "decode":
            _, toks, pos, slots, use_graph, want = cmd
            model.decode_step(toks.to(dev), pos.to(dev), None if slots is None else slots.to(dev),
                              use_graph=use_graph, want_logits=want)
        else:
            raise ValueError(f"unknown command {cmd[0]!r}")
        n += 1
