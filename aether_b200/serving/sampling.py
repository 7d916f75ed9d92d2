"""Sampling parameters and on-device token selection.

Reference: SamplingParams and the sampler of runtime/src/serving.rs:4835-5040
(greedy / temperature / top-k / top-p, presence and frequency penalties,
OpenAI logit_bias, seeded RNG, stop strings). Here selection runs on the GPU
over a [B, vocab] logits tensor; greedy rows never leave the decode graph.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch


@dataclass
class SamplingParams:
    temperature: float = 0.0
    top_p: float = 1.0
    top_k: int = 0
    presence_penalty: float = 0.0
    frequency_penalty: float = 0.0
    repetition_penalty: float = 1.0
    seed: int | None = None
    logit_bias: dict = field(default_factory=dict)
    max_tokens: int = 256
    stop: list = field(default_factory=list)          # stop strings
    stop_token_ids: list = field(default_factory=list)

    @property
    def greedy(self) -> bool:
        return (self.temperature <= 0.0 and not self.logit_bias and self.presence_penalty == 0.0
                and self.frequency_penalty == 0.0 and self.repetition_penalty == 1.0)

    @staticmethod
    def from_openai(body: dict) -> "SamplingParams":
        stop = body.get("stop") or []
        if isinstance(stop, str):
            stop = [stop]
        bias = {int(k): float(v) for k, v in (body.get("logit_bias") or {}).items()}
        return SamplingParams(
            temperature=float(body.get("temperature", 0.0) or 0.0),
            top_p=float(body.get("top_p", 1.0) or 1.0),
            top_k=int(body.get("top_k", 0) or 0),
            presence_penalty=float(body.get("presence_penalty", 0.0) or 0.0),
            frequency_penalty=float(body.get("frequency_penalty", 0.0) or 0.0),
            repetition_penalty=float(body.get("repetition_penalty", 1.0) or 1.0),
            seed=body.get("seed"),
            logit_bias=bias,
            max_tokens=int(body.get("max_tokens", body.get("max_completion_tokens", 256)) or 256),
            stop=list(stop),
        )


def sample_rows(logits: torch.Tensor, params: list, history: list, generators: list) -> torch.Tensor:
    """Selects one token per row of logits [B, V] (fp32) according to each
    row's SamplingParams; history[i] is the list of tokens generated so far."""
    B, V = logits.shape
    out = torch.empty(B, dtype=torch.long, device=logits.device)
    for i in range(B):
        p = params[i]
        row = logits[i]
        if p.greedy:
            out[i] = row.argmax()
            continue
        row = row.clone()
        for tok, b in p.logit_bias.items():
            if 0 <= tok < V:
                row[tok] += b
        if history[i] and (p.presence_penalty or p.frequency_penalty or p.repetition_penalty != 1.0):
            ids = torch.tensor(history[i], device=row.device)
            counts = torch.bincount(ids, minlength=V).to(row.dtype)
            seen = counts > 0
            row -= p.frequency_penalty * counts + p.presence_penalty * seen.to(row.dtype)
            if p.repetition_penalty != 1.0:
                rp = p.repetition_penalty
                row = torch.where(seen, torch.where(row > 0, row / rp, row * rp), row)
        if p.temperature <= 0.0:
            out[i] = row.argmax()
            continue
        row = row / p.temperature
        if p.top_k and p.top_k > 0:
            k = min(p.top_k, V)
            kth = torch.topk(row, k).values[-1]
            row = torch.where(row < kth, torch.full_like(row, float("-inf")), row)
        probs = torch.softmax(row, dim=-1)
        if p.top_p < 1.0:
            sp, si = torch.sort(probs, descending=True)
            cum = torch.cumsum(sp, dim=-1)
            keep = cum - sp < p.top_p
            keep[0] = True
            mask = torch.zeros_like(probs, dtype=torch.bool)
            mask[si[keep]] = True
            probs = torch.where(mask, probs, torch.zeros_like(probs))
            probs = probs / probs.sum()
        out[i] = torch.multinomial(probs, 1, generator=generators[i]).squeeze()
    return out
