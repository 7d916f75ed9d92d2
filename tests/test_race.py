"""Repeat-run race detection: the checker itself (CPU), and the kernels that
are deterministic by design giving identical bits run after run (GPU)."""
import itertools
import math

import pytest
import torch

from aether_b200.ops import functional as F
from aether_b200.utils.race import repeat_check


def test_repeat_check_detects_nondeterminism():
    x = torch.randn(64, 64, generator=torch.Generator().manual_seed(0))
    assert repeat_check(lambda: x @ x, runs=3).deterministic
    flip = itertools.count()

    def racy():
        y = x.clone()
        if next(flip) == 1:  # the second run differs in one element
            y[3, 5] += 1e-3
        return y, x.sum()

    rep = repeat_check(racy, runs=3)
    assert not rep.deterministic and rep.differing_elements == 1 and rep.first_bad_index == (1, 0, (3, 5))
    assert repeat_check(racy, runs=2, atol=1e-2).deterministic


def _bf(*shape, seed=0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * 0.5).bfloat16().cuda()


@pytest.mark.gpu
def test_gpu_deterministic_kernels_repeat_bitwise():
    a, b = _bf(1000, 512, seed=1), _bf(768, 512, seed=2)
    assert repeat_check(lambda: F.gemm(a, b), runs=4).deterministic
    q, k, v = _bf(2, 700, 4, 128, seed=3), _bf(2, 700, 2, 128, seed=4), _bf(2, 700, 2, 128, seed=5)
    rep = repeat_check(lambda: F.attention(q, k, v, 1 / math.sqrt(128), True, 0, impl="tc"), runs=4)
    assert rep.deterministic, rep
    x, w = _bf(333, 2048, seed=6), _bf(2048, seed=7)
    assert repeat_check(lambda: F.rmsnorm(x, w)[0], runs=4).deterministic
    kc, vc = _bf(3, 512, 2, 128, seed=8), _bf(3, 512, 2, 128, seed=9)
    qd = _bf(3, 8 * 128, seed=10)
    slot = torch.tensor([0, 1, 2], dtype=torch.int32, device="cuda")
    seqlen = torch.tensor([512, 77, 300], dtype=torch.int32, device="cuda")

    def dec():
        out = torch.empty(3, 8 * 128, dtype=torch.bfloat16, device="cuda")
        return F.decode_attention(qd, kc, vc, slot, seqlen, out, 8, 1 / math.sqrt(128), splits=4)

    assert repeat_check(dec, runs=4).deterministic


@pytest.mark.gpu
def test_gpu_attention_backward_repeats_within_tolerance():
    """dQ is reduce-added by key blocks in an order the scheduler picks, so
    repeats agree to rounding, not to the bit; dK / dV have one writer."""
    q, k, v = _bf(1, 512, 4, 128, seed=11), _bf(1, 512, 4, 128, seed=12), _bf(1, 512, 4, 128, seed=13)
    do = _bf(1, 512, 4, 128, seed=14)
    o, lse = F.attention(q, k, v, 1 / math.sqrt(128), True, 0, impl="tc")
    run = lambda: F.attention_bwd(q, k, v, o, do, lse, 1 / math.sqrt(128), True, 0, impl="tc")  # noqa: E731
    dq, dk, dv = run()
    assert repeat_check(lambda: run()[1:], runs=3).deterministic  # dK, dV bitwise
    assert repeat_check(lambda: run()[0], runs=3, atol=float(dq.float().abs().max()) * 1e-2).deterministic
