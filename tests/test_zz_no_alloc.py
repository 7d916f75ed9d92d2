"""The allocation-free decode-attention entry point, called through its
exported C symbol, matches the regular entry point (fused-combine path) on two
calls in a row, and rejects problems larger than its static scratch."""
import ctypes

import pytest
import torch

from aether_b200 import _ext
from aether_b200.ops import functional as F

gpu = pytest.mark.gpu


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


@gpu
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


@gpu
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
    # only the counters limit: B * Hkv = 1025 > 1024 while B * Hq * splits fits the partial rows
    qb = torch.zeros(1025, D, dtype=torch.bfloat16, device="cuda")
    kb = torch.zeros(1025, 4, 1, D, dtype=torch.bfloat16, device="cuda")
    sb = torch.arange(1025, dtype=torch.int32, device="cuda")
    lb = torch.ones(1025, dtype=torch.int32, device="cuda")
    ob = torch.empty_like(qb)
    assert _call(f, qb, kb, kb, sb, lb, ob, 1, 1, 1.0) == -2
    # an empty batch (B = 0, valid pointers) launches nothing and succeeds
    stream = torch.cuda.current_stream().cuda_stream
    assert f(qb.data_ptr(), qb.stride(0), kb.data_ptr(), kb.data_ptr(), kb.stride(0), kb.stride(1), sb.data_ptr(),
             lb.data_ptr(), ob.data_ptr(), ob.stride(0), 0, 1, 1, D, 1, 1.0, stream) == 0


def _raw(f, q=0x10000, q_rs=3584, kc=0x20000, vc=0x30000, slot_stride=4096 * 4 * 128, pos_stride=4 * 128,
         out=0x40000, out_rs=3584, B=1, Hq=28, Hkv=4, D=128, splits=4):
    """A call with plain integer addresses: every case below is rejected by
    the argument checks, which run before any CUDA call, so nothing is read
    from these addresses and nothing is launched."""
    return f(q, q_rs, kc, vc, slot_stride, pos_stride, 0x50000, 0x60000, out, out_rs, B, Hq, Hkv, D, splits, 1.0, None)


def test_noalloc_rejects_misaligned_arguments_without_launching():
    if not _ext.available():
        pytest.skip("native extension not built")
    f = _fn()
    assert _raw(f, kc=0x20008) == -1           # K cache not 16-byte aligned
    assert _raw(f, vc=0x30004) == -1           # V cache not 16-byte aligned
    assert _raw(f, slot_stride=4096 * 4 * 128 + 4) == -1  # slot stride not a multiple of 8 elements
    assert _raw(f, pos_stride=4 * 128 + 2) == -1          # position stride not a multiple of 8 elements
    assert _raw(f, q=0x10002) == -1            # q not 4-byte aligned
    assert _raw(f, q_rs=3583) == -1            # odd q row stride
    assert _raw(f, out=0x40004) == -1          # out not 8-byte aligned
    assert _raw(f, out_rs=3582) == -1          # out row stride not a multiple of 4
    assert _raw(f, D=64) == -1                 # head dim other than 128
    assert _raw(f, Hq=27) == -1                # Hq not a multiple of Hkv
