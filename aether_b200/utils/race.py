"""Race detection by repetition: a kernel whose result depends on thread
timing (a missing barrier, an unordered read of a buffer another CTA is
writing, a stale pipeline stage) rarely gives the same bits twice. With
`compute-sanitizer` unavailable, kernels that are deterministic by design
(every reduction in a fixed order: the GEMMs, attention forward, decode
attention, norms, MoE routing) are rerun on identical inputs and their
outputs compared bit for bit; kernels that add with atomics or TMA reduce
(attention dQ, wgrad accumulation into a shared buffer) are checked against a
tolerance instead.

    report = repeat_check(lambda: F.gemm(a, b), runs=5)
    assert report.deterministic, report
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch


@dataclass
class RepeatReport:
    runs: int
    deterministic: bool
    max_abs_diff: float = 0.0
    differing_elements: int = 0
    first_bad_index: tuple | None = None
    notes: list = field(default_factory=list)


def _flatten(out):
    if isinstance(out, torch.Tensor):
        return [out]
    if isinstance(out, (list, tuple)):
        return [t for o in out for t in _flatten(o)]
    if out is None:
        return []
    raise TypeError(f"unsupported output type {type(out)}")


def repeat_check(fn, runs: int = 3, atol: float = 0.0) -> RepeatReport:
    """Run ``fn()`` ``runs`` times and compare every tensor it returns with
    the first run's: bitwise when atol == 0, else within atol."""
    assert runs >= 2
    first = [t.detach().clone() for t in _flatten(fn())]
    rep = RepeatReport(runs=runs, deterministic=True)
    for r in range(1, runs):
        outs = _flatten(fn())
        if len(outs) != len(first):
            rep.deterministic = False
            rep.notes.append(f"run {r}: {len(outs)} outputs, first run had {len(first)}")
            continue
        for j, (a, b) in enumerate(zip(first, outs)):
            if a.shape != b.shape or a.dtype != b.dtype:
                rep.deterministic = False
                rep.notes.append(f"run {r} output {j}: shape / dtype changed")
                continue
            if atol == 0.0:  # compare the bytes of each element (NaNs and -0.0 included)
                ab, bb = a.reshape(-1), b.detach().reshape(-1)
                if a.is_floating_point():
                    ab, bb = ab.contiguous().view(torch.uint8), bb.contiguous().view(torch.uint8)
                bad = (ab != bb).reshape(a.numel(), -1).any(-1)
            else:
                bad = ((a.float() - b.detach().float()).abs() > atol).reshape(-1)
            n_bad = int(bad.sum())
            if n_bad:
                rep.deterministic = False
                rep.differing_elements += n_bad
                d = float((a.float() - b.detach().float()).abs().nan_to_num(float("inf")).max())
                rep.max_abs_diff = max(rep.max_abs_diff, d)
                if rep.first_bad_index is None:
                    flat = int(torch.nonzero(bad)[0])
                    rep.first_bad_index = (r, j, tuple(int(i) for i in torch.unravel_index(torch.tensor(flat), a.shape)))
    return rep
