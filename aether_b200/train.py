"""Training API: ``Trainer.train_step`` runs one optimiser step over a batch of
token sequences (host or device), split into micro-batches with fp32
gradient accumulation, then the data-parallel reduction and AdamW.

Reference: the aether-train hot loop (trainer/src/main.rs:125-150:
cosine_lr, sample_batch, forward, backward, clip, adamw_step) and the DP
driver (trainer/src/dp.rs:34-169).
"""
from __future__ import annotations

import torch

from .optim import cosine_lr
from .parallel.dp import DataParallel


class Trainer:
    def __init__(self, model, info, *, lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1,
                 micro_batch: int = 8, warmup_steps: int = 0, total_steps: int = 0, max_grad_norm: float = 0.0,
                 dp=None, tracer=None, crash_dir: str | None = None):
        """tracer: optional ``utils.trace.Tracer`` (sections fwd_bwd / optimizer);
        crash_dir: write ``crash_<pid>_<step>.dump`` there if a step raises."""
        self.model = model
        self.tracer = tracer
        self.crash_dir = crash_dir
        self.info = info
        self.micro_batch = micro_batch
        self.base_lr = lr
        self.warmup = warmup_steps
        self.total = total_steps
        self.dp = dp if dp is not None else DataParallel(model.arena, info, lr=lr, betas=betas, eps=eps,
                                                         weight_decay=weight_decay, max_grad_norm=max_grad_norm)
        self.step_idx = 0
        self._loss_acc = torch.zeros(1, dtype=torch.float32, device=model.device)
        if hasattr(self.dp, "attach"):  # engines that reduce gradient buckets during the backward
            self.dp.attach(model)

    def lr_at(self, step: int) -> float:
        if self.total <= 0:
            return self.base_lr
        return cosine_lr(step, self.base_lr, self.warmup, self.total)

    def train_step(self, tokens: torch.Tensor) -> torch.Tensor:
        """tokens: [b, S+1] int64 (this rank's sequences). Returns the mean loss
        of this rank as a device tensor (no host sync)."""
        if self.crash_dir is None:
            return self._train_step(tokens)
        from .utils.crash import crash_guard

        with crash_guard(lambda: self.step_idx, self.crash_dir):
            return self._train_step(tokens)

    def _section(self, name):
        import contextlib

        return self.tracer.section(name) if self.tracer is not None else contextlib.nullcontext()

    def _train_step(self, tokens: torch.Tensor) -> torch.Tensor:
        dev = self.model.device
        b = tokens.shape[0]
        mb = min(self.micro_batch, b)
        n_mb = (b + mb - 1) // mb
        n_tok = b * (tokens.shape[1] - 1)
        self.model.arena.zero_grad()
        self._loss_acc.zero_()
        arm = getattr(self.dp, "arm", None)
        with self._section("fwd_bwd"):
            for i in range(n_mb):
                chunk = tokens[i * mb : (i + 1) * mb]
                if chunk.device != dev:
                    chunk = chunk.to(dev, non_blocking=True)
                ids = chunk[:, :-1]
                tgt = chunk[:, 1:]
                loss = self.model.loss(ids.contiguous(), tgt.contiguous(), loss_scale=1.0 / n_tok)
                if arm is not None and i == n_mb - 1:
                    arm(self.lr_at(self.step_idx))  # the last backward reduces buckets as layers finish
                loss.backward()
                self._loss_acc += loss.detach()
            finish = getattr(self.model, "finish_grads", None)
            if finish is not None:  # gradients that the model reduces itself (sequence parallelism)
                finish()
        with self._section("optimizer"):
            self.dp.step(lr=self.lr_at(self.step_idx))
        self.step_idx += 1
        return self._loss_acc
