"""LoRA and QLoRA fine-tuning of the GPT / Qwen-style decoder.

Every targeted projection y = x W^T of the frozen base gains a low-rank
update, y = x W^T + s (x A^T) B^T with s = alpha / rank, A [rank, in] ~
N(0, 1/sqrt(rank)) and B [out, rank] = 0 (the initial update is exactly zero).
Only A and B train: they live in their own ``ParamArena`` (fp32 master, bf16
compute copy, fp32 gradient), so ``FlatAdamW`` and the data-parallel engines
(ZeRO-1 shard + reduce) work on the adapters unchanged -- that is LoRA-DP.

QLoRA keeps the frozen base weights as GGUF Q8_0 or Q4_0 blocks on the GPU
and expands each one to bf16 into a shared scratch buffer right before its
GEMM (and again in backward for the input gradient), so a 7B base takes 4-8
GB instead of 15 GB.

Reference: the LoRA adapter (trainer/src/lora.rs:31-230: init, forward,
backward, AdamW, flat gradients for DP), LoRA-DP (trainer/src/lora_dp.rs),
and the QLoRA stage over a frozen quantised GGUF base with seven adapters per
layer (trainer/src/qwen_qlora_stage.rs:118-712). Here q/k/v are one fused
projection and gate/up another, so a layer has four adapted projections
(wqkv, wo, wgu, wd) that cover the same seven matrices.

GEMMs per adapted projection (all on the tcgen05 kernel):
  forward   u = x A^T;  z = s u B^T (+ residual);  y = x W^T + z
  backward  g = dy B;   dx = dy W + s g A;  dB += s dy^T u;  dA += s g^T x
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from ..ops import functional as F
from .arena import ParamArena


@dataclass
class LoRAConfig:
    rank: int = 16
    alpha: float = 32.0
    targets: tuple = ("wqkv", "wo", "wgu", "wd")

    @property
    def scale(self) -> float:
        return self.alpha / self.rank


class _QuantWeight:
    """A frozen base weight held as GGUF blocks; ``bf16()`` expands it into
    the owner's shared scratch buffer."""

    def __init__(self, w: torch.Tensor, fmt: int, scratch):
        self.shape = tuple(w.shape)
        self.fmt = fmt
        self.blocks = F.quantize_blocks(w.detach().contiguous(), fmt)
        self.scratch = scratch

    def bf16(self) -> torch.Tensor:
        n = self.shape[0] * self.shape[1]
        return F.dequantize_blocks(self.blocks, self.shape, self.fmt, out=self.scratch(n).view(self.shape))


def _weight(w):
    """A frozen weight object (quantised blocks) expanded to bf16, or the tensor itself."""
    return w.bf16() if hasattr(w, "bf16") and not isinstance(w, torch.Tensor) else w


def _acc(mg, a, b, a_mn, b_mn, alpha):
    F.gemm(a, b, a_mn=a_mn, b_mn=b_mn, out=mg, accumulate=True, alpha=alpha)


class FrozenLinearFn(torch.autograd.Function):
    """y = x W^T (+ residual) for a frozen base weight object that expands to
    bf16 on demand (it is expanded again in backward: the shared scratch it
    expands into holds another weight by then)."""

    @staticmethod
    def forward(ctx, x, residual, w):
        ctx.w, ctx.has_res = w, residual is not None
        return F.gemm(x, _weight(w), residual=residual)

    @staticmethod
    def backward(ctx, dy):
        dx = F.gemm(dy.contiguous(), _weight(ctx.w), b_mn=True)
        return dx, (dy if ctx.has_res else None), None


class LoRALinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, a, b, residual, w, scale):
        u = F.gemm(x, a)                                      # [T, r]
        z = F.gemm(u, b, alpha=scale, residual=residual)      # [T, out]
        y = F.gemm(x, _weight(w), residual=z)
        ctx.save_for_backward(x, a, b, u)
        ctx.w, ctx.scale, ctx.has_res = w, scale, residual is not None
        return y

    @staticmethod
    def backward(ctx, dy):
        x, a, b, u = ctx.saved_tensors
        s = ctx.scale
        dy = dy.contiguous()
        g = F.gemm(dy, b, b_mn=True)                          # [T, r] = dy B
        dx = None
        if ctx.needs_input_grad[0]:
            base = F.gemm(dy, _weight(ctx.w), b_mn=True)      # dy W
            dx = F.gemm(g, a, b_mn=True, alpha=s, residual=base)
        _acc(b.main_grad, dy, u, True, True, s)                # dB += s dy^T u
        _acc(a.main_grad, g, x, True, True, s)                 # dA += s g^T x
        return dx, None, None, (dy if ctx.has_res else None), None, None


class LoRAGPT:
    """Adapters over a frozen ``GPT`` (its weights bf16, or quantised with
    ``quant="q8_0"|"q4_0"``). Exposes ``arena`` (the adapters), ``loss`` and
    ``device`` so ``Trainer`` and the DP engines drive it like a full model."""

    def __init__(self, base, cfg: LoRAConfig = LoRAConfig(), seed: int = 0, pad_multiple: int = 1, alloc=None,
                 quant: str | None = None, weights: dict | None = None):
        """weights: prebuilt frozen base weights {(layer, target): weight} for
        projections that live outside the base arena (a GGUF base kept in its
        own quantised blocks, see ``models.qlora_gguf``)."""
        self.base, self.lcfg = base, cfg
        self.cfg, self.device = base.cfg, base.device
        assert cfg.rank % 8 == 0, "LoRA rank must be a multiple of 8 (tensor-core tile granularity)"
        base.freeze()
        ext = getattr(base, "external_shapes", {})
        specs = []
        for i in base.layers:
            for t in cfg.targets:
                key = f"l{i}.{t}"
                out, inp = ext[key] if key in ext else base.arena.slots[key].shape
                specs += [(f"l{i}.{t}.A", (cfg.rank, inp), False), (f"l{i}.{t}.B", (out, cfg.rank), False)]
        self.arena = ParamArena(specs, self.device, pad_multiple=pad_multiple, alloc=alloc)
        with torch.no_grad():
            for name, slot in self.arena.slots.items():
                mv = self.arena.master_view(name)
                if name.endswith(".A"):
                    # one generator per (layer, target): any pipeline split draws the same adapters
                    layer, target = name.split(".")[:2]
                    key = int(layer[1:]) * len(cfg.targets) + cfg.targets.index(target)
                    g = torch.Generator(device="cpu").manual_seed(seed * 1000003 + key)
                    mv.copy_((torch.randn(slot.shape, generator=g) / math.sqrt(cfg.rank)).to(self.device))
                else:
                    mv.zero_()
        self.arena.sync_bf16_from_master()
        self._scratch = None
        self.qweights: dict = dict(weights or {})
        for w in self.qweights.values():
            if hasattr(w, "scratch") and w.scratch is None:
                w.scratch = self._scratch_buf
        if quant is not None:
            fmt = {"q8_0": F.Q8_0, "q4_0": F.Q4_0}[quant]
            for i in base.layers:
                for t in cfg.targets:
                    self.qweights[(i, t)] = _QuantWeight(base.arena[f"l{i}.{t}"], fmt, self._scratch_buf)
            # the bf16 copies of the quantised projections are no longer needed
            self.base_bytes_saved = sum(2 * q.shape[0] * q.shape[1] - q.blocks.numel() for q in self.qweights.values())
        base._linear = self._linear

    def _scratch_buf(self, n: int) -> torch.Tensor:
        if self._scratch is None or self._scratch.numel() < n:
            self._scratch = torch.empty(n, dtype=torch.bfloat16, device=self.device)
        return self._scratch[:n]

    def _linear(self, i, name, x, residual=None):
        if name not in self.lcfg.targets:
            from ..ops import autograd as A

            w = self.qweights.get((i, name))
            if w is not None:
                return FrozenLinearFn.apply(x, residual, w)
            return A.linear(x, self.base.arena[f"l{i}.{name}"], residual=residual)
        w = self.qweights.get((i, name))
        if w is None:
            w = self.base.arena[f"l{i}.{name}"]
        a, b = self.arena[f"l{i}.{name}.A"], self.arena[f"l{i}.{name}.B"]
        return LoRALinearFn.apply(x, a, b, residual, w, self.lcfg.scale)

    def loss(self, ids, targets, loss_scale=None, x=None):
        return self.base.loss(ids, targets, loss_scale, x=x)

    @torch.no_grad()
    def merge(self) -> None:
        """Folds s B A into the base bf16 weights (for serving without adapters)."""
        for i in self.base.layers:
            for t in self.lcfg.targets:
                w = self.base.arena.master_view(f"l{i}.{t}")
                a = self.arena.master_view(f"l{i}.{t}.A")
                b = self.arena.master_view(f"l{i}.{t}.B")
                w += self.lcfg.scale * (b @ a)
        self.base.arena.sync_bf16_from_master()

    def save_adapters(self, path: str) -> None:
        from ..formats import safetensors as st

        st.save_file(self.arena.state_dict(), path, metadata={"rank": self.lcfg.rank, "alpha": self.lcfg.alpha,
                                                              "targets": ",".join(self.lcfg.targets)})

    def load_adapters(self, path: str) -> None:
        from ..formats import safetensors as st

        self.arena.load_state_dict(st.load_file(path))
