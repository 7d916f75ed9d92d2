"""Pipeline-parallel training worker: one rank per process.

    python -m aether_b200.pp_worker --rank R --world-size W --layers L \\
        [--base-port P] [--host H] [--epochs N] [--seed S] [--lr LR] [--microbatch M] [--qlora q8_0|q4_0]
        [--gguf MODEL.gguf]

Ranks meet at ``host:base-port`` (torch.distributed rendezvous; NCCL on GPUs,
gloo on the CPU), each takes its contiguous share of ``--layers`` Qwen3-style
blocks (RMSNorm, fused QKV with per-head q/k RMSNorm, RoPE, causal attention,
SwiGLU; the first rank embeds, the last owns the final norm, LM head and loss)
and trains them with the 1F1B schedule over synthetic token batches. With
``--qlora`` the stage's base projections are frozen and kept as GGUF Q8_0 /
Q4_0 blocks, and only LoRA adapters train (the QLoRA stage); with ``--gguf``
the stage is that GGUF model's share of layers, in the file's own blocks
(``--layers`` is then the model's). The last rank
prints ``EPOCH <e> <mean loss>`` per epoch, every rank prints a checksum of
its trained parameters, and the last rank ends with
``RESULT rank=<R> world=<W> final_loss=<x>``. A ``--world-size 1`` run holds
every layer in one process -- the reference the pipelined run must
reproduce (same seed: the same weights and batches).

Reference: pp_qwen_worker / pp_qlora_worker (trainer/src/bin/pp_qwen_worker.rs,
pp_qlora_worker.rs: the same flags and output lines) over run_1f1b
(trainer/src/pipeline.rs:199-290) with QwenBlockStage / QwenQLoraStage.
"""
from __future__ import annotations

import argparse
import os
import sys

import torch


def model_config(layers: int):
    from .models.gpt import GPTConfig

    # small Qwen3-style blocks (fast on one GPU or CPU; the flags scale the depth)
    return GPTConfig(vocab=512, d_model=128, n_layers=layers, n_heads=4, n_kv_heads=2, d_ff=256, max_seq=64,
                     qk_norm=True, rope_theta=1e6, norm_eps=1e-6)


class QLoRAPipelineStage:
    """A pipeline stage whose base projections are frozen GGUF blocks and whose
    LoRA adapters train (the QLoRA stage), with the GPTPipelineStage contract.
    The base is a random GPT re-quantised to ``quant`` (Q8_0 / Q4_0), or --
    with ``gguf`` -- this stage's layers of a GGUF model file, kept in the
    file's own blocks (models/qlora_gguf.py)."""

    def __init__(self, cfg, rank, world, device, seed=0, lr=1e-3, quant="q8_0", lora_rank=8, gguf=None):
        from .models.gpt import GPT
        from .models.lora import LoRAConfig, LoRAGPT
        from .optim import FlatAdamW

        L = cfg.n_layers
        bounds = [round(L * i / world) for i in range(world + 1)]
        self.layers = list(range(bounds[rank], bounds[rank + 1]))
        self.rank, self.world = rank, world
        self.first, self.last = rank == 0, rank == world - 1
        lcfg = LoRAConfig(rank=lora_rank, alpha=2.0 * lora_rank)
        if gguf is not None:
            from .models.qlora_gguf import qlora_from_gguf

            self.lora = qlora_from_gguf(gguf, device=device, lora=lcfg, seed=seed, layers=self.layers,
                                        first=self.first, last=self.last, max_seq=cfg.max_seq)
        else:
            base = GPT(cfg, device=device, seed=seed, layers=self.layers, first=self.first, last=self.last)
            self.lora = LoRAGPT(base, lcfg, seed=seed + 1, quant=quant)
        self.model = self.lora
        self.opt = FlatAdamW(self.lora.arena, lr=lr, weight_decay=0.0)
        self.device = torch.device(device)
        self.cfg = cfg

    def forward(self, ids, targets, x_in, loss_scale):
        B, S = targets.shape
        if self.last:
            return self.lora.loss(ids if self.first else None, targets, loss_scale, x=x_in)
        return self.lora.base.forward_hidden(ids if self.first else None, x=x_in, B=B, S=S)

    def step(self, lr=None):
        self.opt.step(lr=lr)

    def zero_grad(self):
        self.lora.arena.zero_grad()


def batches_for(epoch: int, n_micro: int, microbatch: int, seq: int, vocab: int, seed: int):
    """Identical on every rank: epoch e's micro-batches of (ids, targets)."""
    g = torch.Generator().manual_seed(seed * 7919 + epoch)
    toks = torch.randint(0, vocab, (n_micro, microbatch, seq + 1), generator=g)
    return [(t[:, :-1].contiguous(), t[:, 1:].contiguous()) for t in toks]


def checksum(arena) -> float:
    return float(arena.master.double().abs().sum())


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--rank", type=int, required=True)
    ap.add_argument("--world-size", type=int, required=True)
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--base-port", type=int, default=29600)
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--epochs", type=int, default=3)
    ap.add_argument("--seed", type=int, default=42)
    ap.add_argument("--lr", type=float, default=3e-3)
    ap.add_argument("--microbatch", type=int, default=2)
    ap.add_argument("--micro-batches", type=int, default=4, help="micro-batches per optimiser step")
    ap.add_argument("--seq", type=int, default=32)
    ap.add_argument("--qlora", choices=["q8_0", "q4_0"], default=None)
    ap.add_argument("--gguf", default=None, help="QLoRA over this GGUF model's layers (its quantised blocks)")
    ap.add_argument("--device", default=None, help="cpu or cuda (default: cuda when available)")
    a = ap.parse_args(argv)
    if not 0 <= a.rank < a.world_size:
        ap.error("--rank must be in [0, world-size)")
    if a.layers < a.world_size:
        ap.error("--layers must be at least --world-size")

    from .parallel import dist as D
    from .parallel.pp import GPTPipelineStage, run_1f1b

    os.environ.update(RANK=str(a.rank), WORLD_SIZE=str(a.world_size), MASTER_ADDR=a.host,
                      MASTER_PORT=str(a.base_port), LOCAL_RANK=os.environ.get("LOCAL_RANK", str(a.rank)))
    use_cuda = (a.device or ("cuda" if torch.cuda.is_available() else "cpu")) == "cuda"
    info = D.init(device=None if use_cuda else "cpu", timeout_s=120)
    dev = info.device
    cfg = model_config(a.layers)
    if a.gguf:
        from .formats.gguf import GGUFFile
        from .models.qlora_gguf import config_from_gguf

        cfg = config_from_gguf(GGUFFile(a.gguf), max_seq=max(64, a.seq))
        if cfg.n_layers < a.world_size:
            ap.error("the GGUF model has fewer layers than --world-size")
        stage = QLoRAPipelineStage(cfg, a.rank, a.world_size, dev, seed=a.seed, lr=a.lr, gguf=a.gguf)
    elif a.qlora:
        stage = QLoRAPipelineStage(cfg, a.rank, a.world_size, dev, seed=a.seed, lr=a.lr, quant=a.qlora)
    else:
        stage = GPTPipelineStage(cfg, a.rank, a.world_size, dev, seed=a.seed, lr=a.lr, weight_decay=0.0)
    final = None
    for e in range(a.epochs):
        stage.zero_grad()
        if a.world_size > 1:
            loss = run_1f1b(stage, batches_for(e, a.micro_batches, a.microbatch, a.seq, cfg.vocab, a.seed))
        else:  # one process holds every layer: plain gradient accumulation over the micro-batches
            mbs = batches_for(e, a.micro_batches, a.microbatch, a.seq, cfg.vocab, a.seed)
            n_tok = sum(t.numel() for _, t in mbs)
            loss = torch.zeros((), device=dev)
            for ids, tgt in mbs:
                out = stage.forward(ids.to(dev), tgt.to(dev), None, 1.0 / n_tok)
                out.backward()
                loss = loss + out.detach()
        stage.step()
        if stage.last:
            final = float(loss)
            print(f"EPOCH {e} {final:.6f}", flush=True)
    arena = stage.model.arena
    print(f"CHECKSUM rank={a.rank} layers={stage.layers[0]}-{stage.layers[-1]} value={checksum(arena):.9e}", flush=True)
    if stage.last:
        print(f"RESULT rank={a.rank} world={a.world_size} final_loss={final:.6f}", flush=True)
    D.shutdown()
    return 0


if __name__ == "__main__":
    sys.exit(main())
