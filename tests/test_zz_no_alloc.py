"""The allocation-free decode-attention entry point, called through its
exported C symbol, matches the regular entry point (fused-combine path) on two
calls in a row, and rejects problems larger than its static scratch."""
import ctypes

import pytest
import torch

from aether_b200 import _ext
from aether_b200.ops import functional as F

pytestmark = pytest.mark.gpu


def _fn():
    lib = ctypes.CDLL(_ext.so_path())
    f = lib.aether_decode_attention_noalloc
    i64, i32, vp = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p
    f.argtypes = [vp, i64, vp, vp, i64, i64, vp, vp, vp, i64, i32, i32, i32, i32, i32, ctypes.c_float, vp]
    f.restype = ctypes.c_int
    return f


def _call(f, q, kc, vc, slot, seqlen, out, Hq, splits, scale):
    B, D, Hkv = q.shape[0], kc.shape[3], kc.shape[2]
    stream = torch.cuda.current_stream().cuda_stream
    return f(q.data_ptr(), q.stride(0), kc.data_ptr(), vc.data_ptr(), kc.stride(0), kc.stride(1), slot.data_ptr(),
             seqlen.data_ptr(), out.data_ptr(), out.stride(0), B, Hq, Hkv, D, splits, scale, stream)


def test_noalloc_decode_attention_matches_regular_entry_point():
    f = _fn()
    g = torch.Generator(device="cuda").manual_seed(7)
    B, Hq, Hkv, D, splits = 3, 28, 4, 128, 8
    kc = torch.randn(B + 1, 1024, Hkv, D, device="cuda", generator=g).bfloat16()
    vc = torch.randn(B + 1, 1024, Hkv, D, device="cuda", generator=g).bfloat16()
    q = torch.randn(B, Hq * D, device="cuda", generator=g).bfloat16()
    slot = torch.tensor([2, 0, 1], dtype=torch.int32, device="cuda")
    seqlen = torch.tensor([700, 1, 129], dtype=torch.int32, device="cuda")
    scale = D ** -0.5
    want = torch.empty(B, Hq * D, dtype=torch.bfloat16, device="cuda")
    counters = torch.zeros(B * Hkv, dtype=torch.int32, device="cuda")
    F.decode_attention(q, kc, vc, slot, seqlen, want, Hq, scale, splits=splits, counters=counters)
    for _ in range(2):  # twice in a row: the counters must come back to zero
        got = torch.full_like(want, float("nan"))
        assert _call(f, q, kc, vc, slot, seqlen, got, Hq, splits, scale) == 0
        torch.cuda.synchronize()
        err = float((got.float() - want.float()).abs().max())
        assert err <= 1e-2 * float(want.float().abs().max()), err


def test_noalloc_rejects_oversized_problem():
    f = _fn()
    B, Hq, Hkv, D = 64, 32, 8, 128
    q = torch.zeros(B, Hq * D, dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros(B, 16, Hkv, D, dtype=torch.bfloat16, device="cuda")
    slot = torch.arange(B, dtype=torch.int32, device="cuda")
    seqlen = torch.ones(B, dtype=torch.int32, device="cuda")
    out = torch.empty_like(q)
    assert _call(f, q, kc, kc, slot, seqlen, out, Hq, 8, 1.0) == -2  # 64*32*8 partial rows > 8192
    assert _call(f, q, kc, kc, slot, seqlen, out, Hq, 8, 1.0) == -2
    assert _call(f, q[:2], kc, kc, slot, seqlen, out, Hq, 65, 1.0) == -1  # more splits than the kernel allows
