"""GGUF block formats Q4_1, Q5_0, Q5_1, Q2_K, Q3_K, Q5_K, IQ4_NL, IQ4_XS: the
vectorised load-time dequantiser against element-by-element decoders written
straight from the block layouts, on random blocks; the native Q3_K decoder of
the C ABI against both."""
import numpy as np
import pytest

from aether_b200.formats import gguf as G


def _blocks(typ, n, seed):
    ne, nb = G.BLOCKS[typ]
    rng = np.random.default_rng(seed)
    b = rng.integers(0, 256, size=(n, nb), dtype=np.uint8)
    halves = {G.Q4_1: (0, 2), G.Q5_1: (0, 2), G.Q5_0: (0,), G.IQ4_NL: (0,), G.Q2_K: (80, 82), G.Q3_K: (108,),
              G.Q5_K: (0, 2), G.IQ4_XS: (0,)}[typ]
    for o in halves:  # sane f16 scales
        b[:, o : o + 2] = np.frombuffer(np.float16(rng.uniform(0.01, 0.1)).tobytes(), np.uint8)
    return b


def _f16(b, o):
    return float(np.frombuffer(bytes(b[o : o + 2]), np.float16)[0])


def _scalar(typ, blk):
    out = []
    if typ in (G.Q4_1, G.Q5_0, G.Q5_1, G.IQ4_NL):
        d = _f16(blk, 0)
        m = _f16(blk, 2) if typ in (G.Q4_1, G.Q5_1) else 0.0
        o = 4 if typ in (G.Q4_1, G.Q5_1) else 2
        qh = int.from_bytes(bytes(blk[o : o + 4]), "little") if typ in (G.Q5_0, G.Q5_1) else 0
        qs = blk[o + 4 : o + 20] if typ in (G.Q5_0, G.Q5_1) else blk[o : o + 16]
        for e in range(32):
            q = int(qs[e % 16]) & 0xF if e < 16 else int(qs[e % 16]) >> 4
            if typ == G.IQ4_NL:
                out.append(d * float(G.IQ4_LEVELS[q]))
            elif typ == G.Q4_1:
                out.append(q * d + m)
            else:
                q |= ((qh >> e) & 1) << 4
                out.append((q - 16) * d if typ == G.Q5_0 else q * d + m)
        return out
    if typ == G.Q2_K:
        sc, qs, d, dm = blk[0:16], blk[16:80], _f16(blk, 80), _f16(blk, 82)
        for e in range(256):
            half, r = divmod(e, 128)
            j, r2 = divmod(r, 32)
            si = half * 8 + j * 2 + r2 // 16
            q = (int(qs[half * 32 + r2]) >> (2 * j)) & 3
            out.append(d * (int(sc[si]) & 0xF) * q - dm * (int(sc[si]) >> 4))
        return out
    if typ == G.Q3_K:
        hm, qs, d = blk[0:32], blk[32:96], _f16(blk, 108)
        raw = [int(x) for x in blk[96:108]]
        sc = []
        for i in range(16):  # 4 low bits from bytes 0..7, 2 high bits from bytes 8..11
            lo = (raw[i % 8] >> (4 * (i // 8))) & 0xF
            hi = (raw[8 + i % 4] >> (2 * (i // 4))) & 3
            sc.append((lo | (hi << 4)) - 32)
        for e in range(256):
            half, r = divmod(e, 128)
            j, r2 = divmod(r, 32)
            si = half * 8 + j * 2 + r2 // 16
            q = (int(qs[half * 32 + r2]) >> (2 * j)) & 3
            if not (int(hm[r2]) >> (half * 4 + j)) & 1:
                q -= 4
            out.append(d * sc[si] * q)
        return out
    if typ == G.Q5_K:
        d, dm = _f16(blk, 0), _f16(blk, 2)
        sc, mn = G._k4_scales(blk[4:16][None, :])
        qh, qs = blk[16:48], blk[48:176]
        for e in range(256):
            g, r = divmod(e, 64)
            sub, l = divmod(r, 32)
            q = (int(qs[g * 32 + l]) >> (4 * sub)) & 0xF
            q += 16 if (int(qh[l]) >> (2 * g + sub)) & 1 else 0
            out.append(d * sc[0, 2 * g + sub] * q - dm * mn[0, 2 * g + sub])
        return out
    if typ == G.IQ4_XS:
        d = _f16(blk, 0)
        sh = int.from_bytes(bytes(blk[2:4]), "little")
        for e in range(256):
            ib, r = divmod(e, 32)
            ls = ((int(blk[4 + ib // 2]) >> (4 * (ib % 2))) & 0xF) | (((sh >> (2 * ib)) & 3) << 4)
            q = int(blk[8 + ib * 16 + r % 16])
            q = q & 0xF if r < 16 else q >> 4
            out.append(d * (ls - 32) * float(G.IQ4_LEVELS[q]))
        return out
    raise AssertionError(typ)


@pytest.mark.parametrize("typ", [G.Q4_1, G.Q5_0, G.Q5_1, G.IQ4_NL, G.Q2_K, G.Q3_K, G.Q5_K, G.IQ4_XS])
def test_block_dequant_matches_scalar_decoder(typ):
    ne, nb = G.BLOCKS[typ]
    b = _blocks(typ, 3, typ)
    got = G.dequantize(b.reshape(-1), typ, 3 * ne)
    want = np.array([v for blk in b for v in _scalar(typ, blk)], np.float32)
    assert np.allclose(got, want, rtol=1e-5, atol=1e-6)


def test_native_q3_k_matches():
    from aether_b200 import runtime as R

    b = _blocks(G.Q3_K, 4, 1)
    out = np.zeros(4 * 256, np.float32)
    assert R.call("aether_dequant_q3_k", R.ptr(b), R.ptr(out), 4) == 0
    assert np.allclose(out, G.dequantize(b.reshape(-1), G.Q3_K, 1024), rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("name", ["IQ3_XXS", "IQ3_S"])
def test_iq3_matches_the_gguf_package(name):
    """The IQ3 codebook formats through the load-time dequantiser, against the
    pure-Python dequantiser of the `gguf` package on random blocks."""
    gq = pytest.importorskip("gguf.quants")
    gt = pytest.importorskip("gguf").GGMLQuantizationType
    typ = getattr(G, name)
    ne, nb = G.BLOCKS[typ]
    rng = np.random.default_rng(typ)
    b = rng.integers(0, 256, size=(40, nb), dtype=np.uint8)
    b[:, 0:2] = np.frombuffer(np.float16(rng.uniform(0.01, 0.1)).tobytes(), np.uint8)
    want = gq.dequantize(b.reshape(-1), getattr(gt, name)).reshape(-1)
    got = G.dequantize(b.reshape(-1), typ, 40 * ne - 7)
    np.testing.assert_array_equal(got, want[: 40 * ne - 7])
