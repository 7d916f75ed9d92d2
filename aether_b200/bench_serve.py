"""Serving benchmark: Qwen2.5 decode tokens/s and p50 time-to-first-token.

Configs (random-init bf16 weights, uniform-random prompt ids, greedy):
  1.5b : Qwen2.5-1.5B shape, prompt 512, 256 new tokens, batch 1/8/32
  7b   : Qwen2.5-7B shape,   prompt 2048, 256 new tokens, batch 1/16/64
KV cache preallocated to 4096 positions; decode runs as one CUDA graph per
step. TTFT = prefill of the batch's prompts + the first greedy token (CUDA
events, p50 over --ttft-reps); decode tok/s = batch * steps / device time of
``steps`` graph replays. One JSON line per (config, batch).

    python -m aether_b200.bench_serve --model 7b --batches 1,16,64
    torchrun --nproc-per-node N -m aether_b200.bench_serve --model 7b --tp N
"""
from __future__ import annotations

import argparse
import json
import os
import statistics

import torch

from . import _ext
from .models.qwen import QwenConfig, QwenModel


class EmulatedTP:
    """One tensor-parallel rank's share of the work on a single GPU, with the
    cross-rank exchanges replaced by their local halves: the model holds rank
    ``rank`` of ``world``'s shards and runs the same kernels as in a real TP
    run (push-reduce mode), except that a reduction sums only this rank's
    partial and the vocabulary argmax sees only this rank's slice. The time
    per step is the TP compute floor; a real TP run minus it is the cost of
    communication. Numerics are not those of the full model."""

    mode = "push"

    def __init__(self, rank: int, world: int):
        self.rank, self.world = rank, world
        self._acc = None

    def prepare_decode(self, rows_cap, width, vocab_cols):
        pass

    def all_reduce_(self, t):
        return t

    def reduce_gemm(self, x, w, which):
        """This rank's partial only (the multicast-reduce path without the exchange)."""
        from .ops import functional as F

        if self._acc is None or self._acc.shape[1] < w.shape[0]:
            self._acc = torch.zeros(64, max(w.shape[0], 8192), dtype=torch.float32, device=x.device)
        F.skinny_gemm(x, w, self._acc)
        return self._acc[: x.shape[0]]

    def finalize_wait(self):
        return None

    def push_reduce(self, acc, y, res=None, bias=None, w=None, h=None, eps=1e-6):
        from .ops import functional as F

        if w is None:
            return F.skinny_finalize(acc, y, bias=bias, res=res)
        F.finalize_residual_norm(acc, y, w, h, bias=bias, res=res, eps=eps)
        return y

    def vocab_argmax(self, logits, n_loc, col0, out=None):
        from .ops import functional as F

        r = F.argmax(logits[:, :n_loc].contiguous()) + col0
        if out is None:
            return r
        out.copy_(r)
        return out

    def gather_vocab(self, logits, n_loc, col0, V, out=None):
        raise NotImplementedError("the emulation keeps one vocabulary slice")

    def max_over_ranks(self, x):
        return x


def events():
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def run(model_name: str, batches, prompt: int, new_tokens: int, ttft_reps: int, tp=None, rank0=True):
    cfg = QwenConfig.qwen25_7b() if model_name == "7b" else QwenConfig.qwen25_1_5b()
    maxb = max(batches)
    dev = torch.device("cuda", torch.cuda.current_device())
    m = QwenModel(cfg, device=dev, seed=0, max_batch=maxb, max_seq=4096, tp=tp)
    g = torch.Generator(device="cpu").manual_seed(7)
    out = []
    for B in batches:
        prompts = torch.randint(0, cfg.vocab, (B, prompt), generator=g).to(dev)
        # warm-up: prefill + graph capture
        m.prefill(prompts)
        tok = torch.zeros(B, dtype=torch.long, device=dev)
        pos = torch.full((B,), prompt, dtype=torch.int32, device=dev)
        for _ in range(3):
            m.decode_step(tok, pos)
        torch.cuda.synchronize()
        # TTFT
        tt = []
        for _ in range(ttft_reps):
            e0, e1 = events()
            e0.record()
            nxt = m.prefill(prompts)
            e1.record()
            torch.cuda.synchronize()
            tt.append(e0.elapsed_time(e1))
        # decode
        tok = nxt.clone()
        pos = torch.full((B,), prompt, dtype=torch.int32, device=dev)
        steps = new_tokens - 1
        e0, e1 = events()
        e0.record()
        for _ in range(steps):
            tok = m.decode_step(tok, pos)
            pos += 1
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        ms_step = ms / steps
        if tp is not None:
            ms_step = tp.max_over_ranks(ms_step)
            tt = [tp.max_over_ranks(t) for t in tt]
        rec = {
            "metric": "decode_tokens_per_s", "model": f"Qwen2.5-{model_name.upper()} shape", "tp": tp.world if tp else 1, "emulated_tp": isinstance(tp, EmulatedTP),
            "batch": B, "prompt": prompt, "new_tokens": new_tokens, "value": B / (ms_step / 1e3), "unit": "tokens/s",
            "ms_per_decode_step": ms_step, "ttft_p50_ms": statistics.median(tt), "ttft_all_ms": tt,
            "decode_splits": m.decode_splits, "graph": True, "dtype": "bf16",
            "data": "synthetic uniform-random prompts, random-init weights",
            "kv_cache_gb": m.cache.bytes() / 1e9,
        }
        if rank0:
            print(json.dumps(rec), flush=True)
        out.append(rec)
    assert _ext.check_status() == 0
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="1.5b", choices=["1.5b", "7b"])
    ap.add_argument("--batches", default=None)
    ap.add_argument("--prompt", type=int, default=None)
    ap.add_argument("--new-tokens", type=int, default=256)
    ap.add_argument("--ttft-reps", type=int, default=5)
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--emulate-tp", type=int, default=0,
                    help="one GPU runs one TP rank's shards without communication (the TP compute floor)")
    args = ap.parse_args()
    _ext.C()
    batches = [int(b) for b in (args.batches or ("1,8,32" if args.model == "1.5b" else "1,16,64")).split(",")]
    prompt = args.prompt or (512 if args.model == "1.5b" else 2048)
    tp = None
    rank0 = True
    if args.emulate_tp > 1:
        tp = EmulatedTP(0, args.emulate_tp)
    elif args.tp > 1 or int(os.environ.get("WORLD_SIZE", "1")) > 1:
        from .parallel import dist as D
        from .parallel.tp import TensorParallel

        info = D.init()
        tp = TensorParallel(info)
        rank0 = info.is_main
    run(args.model, batches, prompt, args.new_tokens, args.ttft_reps, tp, rank0)
    if tp is not None and hasattr(tp, "close"):
        tp.close()


if __name__ == "__main__":
    main()
