"""QLoRA smoke test over a real GGUF model: one process, a layer range.

    python -m aether_b200.qlora_smoke --gguf MODEL.gguf [--lo 0 --hi 2 --t 8 --steps 30 --rank 8 --lr 5e-3]
        [--device cuda|cpu]

Loads layers [lo, hi) of the GGUF model as a QLoRA stage (frozen base in the
file's quantised blocks + trainable LoRA adapters, models/qlora_gguf.py) and
trains the adapters against a synthetic loss head -- unit-weight RMSNorm, a
fixed random [256, d_model] projection and cross-entropy over 256 synthetic
classes with targets (i * 37 + 11) mod 256 -- which only turns the stage's
hidden states into a scalar. The stage sees the model's token embeddings when
lo is 0 and fixed random hidden states otherwise. Prints one ``STEP k loss``
line per step and a ``RESULT`` line; exits 0 when the loss is finite and
decreased and the adapters' B matrices (zero at start) have grown, 1
otherwise, 2 on bad arguments.

Reference: trainer/src/bin/qlora_smoke.rs (same flags, same synthetic head and
pass criteria).
"""
from __future__ import annotations

import argparse
import math
import sys

import torch

VS = 256  # synthetic loss-head classes


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--gguf", required=True)
    ap.add_argument("--lo", type=int, default=0)
    ap.add_argument("--hi", type=int, default=2)
    ap.add_argument("--t", type=int, default=8, help="tokens per step")
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--rank", type=int, default=8)
    ap.add_argument("--lr", type=float, default=5e-3)
    ap.add_argument("--device", default=None)
    a = ap.parse_args(argv)

    from .formats.gguf import GGUFFile
    from .models.lora import LoRAConfig
    from .models.qlora_gguf import config_from_gguf, qlora_from_gguf
    from .ops import autograd as A
    from .optim import FlatAdamW

    cfg = config_from_gguf(GGUFFile(a.gguf))
    if not 0 <= a.lo < a.hi <= cfg.n_layers or a.t < 1 or a.rank % 8:
        print(f"bad range / sizes: model has {cfg.n_layers} layers; rank must be a multiple of 8", file=sys.stderr)
        return 2
    dev = torch.device(a.device or ("cuda" if torch.cuda.is_available() else "cpu"))
    m = qlora_from_gguf(a.gguf, device=dev, lora=LoRAConfig(rank=a.rank, alpha=2.0 * a.rank),
                        layers=list(range(a.lo, a.hi)), first=a.lo == 0, last=False, max_seq=max(64, a.t))
    g = torch.Generator().manual_seed(0x105)
    w_head = (torch.randn(VS, cfg.d_model, generator=g) * 0.02).to(dev, torch.bfloat16)
    g_norm = torch.ones(cfg.d_model, dtype=torch.bfloat16, device=dev)
    targets = torch.tensor([(i * 37 + 11) % VS for i in range(a.t)], dtype=torch.long, device=dev)
    ids = torch.arange(a.t, dtype=torch.long, device=dev).view(1, a.t) % cfg.vocab
    x_in = None
    if a.lo > 0:
        x_in = (torch.randn(a.t, cfg.d_model, generator=g) * 0.5).to(dev, torch.bfloat16)
    opt = FlatAdamW(m.arena, lr=a.lr, weight_decay=0.0)
    losses = []
    for k in range(a.steps):
        m.arena.zero_grad()
        h = m.base.forward_hidden(ids if a.lo == 0 else None, x=x_in, B=1, S=a.t)
        hn = A.rmsnorm(h, g_norm, 1e-5)
        loss = A.lm_head_cross_entropy(hn, w_head, targets, 1.0 / a.t)
        loss.backward()
        opt.step()
        losses.append(float(loss.detach()))
        print(f"STEP {k} {losses[-1]:.6f}", flush=True)
    b_norm = sum(float(m.arena.master_view(n).abs().sum()) for n in m.arena.names() if n.endswith(".B"))
    ok = all(math.isfinite(v) for v in losses) and losses[-1] < losses[0] and b_norm > 0.0
    print(f"RESULT layers={a.lo}-{a.hi - 1} first={losses[0]:.6f} last={losses[-1]:.6f} adapter_B_l1={b_norm:.6e} "
          f"ok={ok}", flush=True)
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
