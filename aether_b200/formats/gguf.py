"""GGUF reader, writer (for tests and exports) and load-time dequantisation.

Reference: aether_gguf_* (runtime/src/lib.rs:8647-9030 -- header, metadata
key/values including arrays, tensor table), the CPU dequantisers
(lib.rs:217, 9218-9404) and GGUF-metadata-driven model configs
(runtime/src/serving.rs:459-900). The reference keeps weights quantised on the
GPU and multiplies with per-format GEMV kernels; this build dequantises at
load time to bf16 (the tensor-core GEMMs want bf16 operands), so the block
formats only need a correct unpacking, done here in vectorised numpy.

Block layouts (the published GGUF/ggml formats, reproduced because files must
decode identically):
  Q8_0  32 values: f16 d, 32 x int8            x = d * q
  Q4_0  32 values: f16 d, 16 bytes of nibbles  x = d * (q - 8); low nibbles are
        elements 0..15, high nibbles 16..31
  Q4_K  256 values: f16 d, f16 dmin, 12 bytes of 6-bit (scale, min) pairs for 8
        sub-blocks of 32, 128 bytes of nibbles; x = d*sc*q - dmin*mn
  Q6_K  256 values: 128 bytes low 4 bits, 64 bytes high 2 bits, 16 x int8
        scales, f16 d; x = d * scale * (q - 32) over 16 sub-blocks of 16
  IQ3_XXS / IQ3_S  256 values: codebook indices (4 magnitudes each), sign
        patterns and 4-bit scales; decoded by the native library, which holds
        the format's codebooks
"""
from __future__ import annotations

import struct

import numpy as np
import torch

GGUF_MAGIC = 0x46554747
(T_U8, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64, T_I64, T_F64) = range(13)
_SCALAR = {T_U8: "<B", T_I8: "<b", T_U16: "<H", T_I16: "<h", T_U32: "<I", T_I32: "<i", T_F32: "<f", T_BOOL: "<?",
           T_U64: "<Q", T_I64: "<q", T_F64: "<d"}

F32, F16, Q4_0, Q8_0, Q4_K, Q6_K, BF16 = 0, 1, 2, 8, 12, 14, 30
Q4_1, Q5_0, Q5_1, Q2_K, Q3_K, Q5_K, IQ4_NL, IQ4_XS = 3, 6, 7, 10, 11, 13, 20, 23
IQ3_XXS, IQ3_S = 18, 21
# (block elements, block bytes) of every type the load-time dequantiser reads
BLOCKS = {F32: (1, 4), F16: (1, 2), BF16: (1, 2), Q4_0: (32, 18), Q4_1: (32, 20), Q5_0: (32, 22), Q5_1: (32, 24),
          Q8_0: (32, 34), Q2_K: (256, 84), Q3_K: (256, 110), Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210),
          IQ4_NL: (32, 18), IQ4_XS: (256, 136), IQ3_XXS: (256, 98), IQ3_S: (256, 110)}
# the 16 non-uniform levels of the IQ4_NL / IQ4_XS formats
IQ4_LEVELS = np.array([-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113], np.float32)
# (block elements, block bytes)
_BLOCK = BLOCKS


class GGUFFile:
    def __init__(self, path: str):
        self.path = path
        with open(path, "rb") as f:
            self.data = f.read()
        self.pos = 0
        magic, self.version = self._u("<I"), self._u("<I")
        if magic != GGUF_MAGIC:
            raise ValueError(f"{path}: not a GGUF file")
        n_tensors, n_kv = self._u("<Q"), self._u("<Q")
        self.meta = {}
        for _ in range(n_kv):
            k = self._str()
            self.meta[k] = self._val(self._u("<I"))
        self.tensors = {}
        for _ in range(n_tensors):
            name = self._str()
            nd = self._u("<I")
            dims = [self._u("<Q") for _ in range(nd)]
            typ = self._u("<I")
            off = self._u("<Q")
            self.tensors[name] = (dims, typ, off)
        align = int(self.meta.get("general.alignment", 32))
        self.data_start = (self.pos + align - 1) // align * align

    def _u(self, fmt):
        v = struct.unpack_from(fmt, self.data, self.pos)[0]
        self.pos += struct.calcsize(fmt)
        return v

    def _str(self):
        n = self._u("<Q")
        s = self.data[self.pos : self.pos + n].decode("utf-8", errors="replace")
        self.pos += n
        return s

    def _val(self, t):
        if t == T_STR:
            return self._str()
        if t == T_ARR:
            et, n = self._u("<I"), self._u("<Q")
            return [self._val(et) for _ in range(n)]
        return self._u(_SCALAR[t])

    def raw(self, name: str) -> tuple:
        dims, typ, off = self.tensors[name]
        n = int(np.prod(dims)) if dims else 1
        be, bb = _BLOCK[typ]
        nbytes = n // be * bb
        start = self.data_start + off
        return np.frombuffer(self.data, dtype=np.uint8, count=nbytes, offset=start), dims, typ

    def tensor(self, name: str, dtype=torch.bfloat16) -> torch.Tensor:
        """Dequantised tensor in torch (row-major) shape: GGUF dims are listed
        fastest-first, so dims [K, N] become [N, K]."""
        buf, dims, typ = self.raw(name)
        x = dequantize(buf, typ, int(np.prod(dims)))
        return torch.from_numpy(x.reshape(list(reversed(dims)))).to(dtype)


def _f16(b):
    return b.view(np.float16).astype(np.float32)


def dequantize(buf: np.ndarray, typ: int, n: int) -> np.ndarray:
    if typ == F32:
        return buf.view(np.float32)[:n].copy()
    if typ == F16:
        return buf.view(np.float16)[:n].astype(np.float32)
    if typ == BF16:
        u = buf.view(np.uint16)[:n].astype(np.uint32) << 16
        return u.view(np.float32)
    if typ == Q8_0:
        b = buf.reshape(-1, 34)
        d = _f16(b[:, :2].copy())
        q = b[:, 2:].view(np.int8).astype(np.float32)
        return (q * d).reshape(-1)[:n]
    if typ == Q4_0:
        b = buf.reshape(-1, 18)
        d = _f16(b[:, :2].copy())
        qs = b[:, 2:]
        q = np.concatenate([qs & 0x0F, qs >> 4], axis=1).astype(np.float32) - 8.0
        return (q * d).reshape(-1)[:n]
    if typ == Q4_K:
        b = buf.reshape(-1, 144)
        d = _f16(b[:, 0:2].copy())
        dmin = _f16(b[:, 2:4].copy())
        sc = b[:, 4:16].astype(np.uint32)
        qs = b[:, 16:144]
        scales = np.empty((b.shape[0], 8), np.float32)
        mins = np.empty((b.shape[0], 8), np.float32)
        for j in range(8):
            if j < 4:
                s, m = sc[:, j] & 63, sc[:, j + 4] & 63
            else:
                s = (sc[:, j + 4] & 0x0F) | ((sc[:, j - 4] >> 6) << 4)
                m = (sc[:, j + 4] >> 4) | ((sc[:, j] >> 6) << 4)
            scales[:, j], mins[:, j] = s, m
        out = np.empty((b.shape[0], 256), np.float32)
        for g in range(4):  # 4 groups of 64: low nibbles -> sub-block 2g, high -> 2g+1
            q = qs[:, g * 32 : (g + 1) * 32]
            lo, hi = (q & 0x0F).astype(np.float32), (q >> 4).astype(np.float32)
            out[:, g * 64 : g * 64 + 32] = d * scales[:, 2 * g : 2 * g + 1] * lo - dmin * mins[:, 2 * g : 2 * g + 1]
            out[:, g * 64 + 32 : g * 64 + 64] = d * scales[:, 2 * g + 1 : 2 * g + 2] * hi - dmin * mins[:, 2 * g + 1 : 2 * g + 2]
        return out.reshape(-1)[:n]
    if typ == Q6_K:
        b = buf.reshape(-1, 210)
        ql, qh = b[:, 0:128], b[:, 128:192]
        scales = b[:, 192:208].view(np.int8).astype(np.float32)
        d = _f16(b[:, 208:210].copy())
        out = np.empty((b.shape[0], 256), np.float32)
        for half in range(2):  # two 128-value halves
            l = ql[:, half * 64 : half * 64 + 64]
            h = qh[:, half * 32 : half * 32 + 32]
            for part in range(4):
                if part == 0:
                    q = (l[:, 0:32] & 0xF) | (((h >> 0) & 3) << 4)
                elif part == 1:
                    q = (l[:, 32:64] & 0xF) | (((h >> 2) & 3) << 4)
                elif part == 2:
                    q = (l[:, 0:32] >> 4) | (((h >> 4) & 3) << 4)
                else:
                    q = (l[:, 32:64] >> 4) | (((h >> 6) & 3) << 4)
                q = q.astype(np.float32) - 32.0
                base = half * 128 + part * 32
                for sub in range(2):  # each 32-run spans two 16-value sub-blocks
                    si = half * 8 + part * 2 + sub
                    out[:, base + sub * 16 : base + sub * 16 + 16] = d * scales[:, si : si + 1] * q[:, sub * 16 : sub * 16 + 16]
        return out.reshape(-1)[:n]
    if typ in (Q4_1, Q5_0, Q5_1, IQ4_NL):
        return _dequant_32(buf, typ)[:n]
    if typ in (Q2_K, Q3_K, Q5_K, IQ4_XS):
        return _dequant_k(buf, typ)[:n]
    if typ in (IQ3_XXS, IQ3_S):  # codebook formats: the native dequantisers hold the grids
        from .. import runtime as rt

        b = np.ascontiguousarray(buf, dtype=np.uint8)
        nblk = b.size // BLOCKS[typ][1]
        out = np.empty(nblk * 256, np.float32)
        rt.call("aether_dequant_iq3_xxs" if typ == IQ3_XXS else "aether_dequant_iq3_s", rt.ptr(b), rt.ptr(out), nblk)
        return out[:n]
    raise NotImplementedError(f"GGUF tensor type {typ} is not supported by the load-time dequantiser")


def _k4_scales(sc: np.ndarray):
    """The 8 six-bit (scale, min) pairs packed in 12 bytes (Q4_K / Q5_K)."""
    sc = sc.astype(np.uint32)
    scales = np.empty((sc.shape[0], 8), np.float32)
    mins = np.empty((sc.shape[0], 8), np.float32)
    for j in range(8):
        if j < 4:
            s_, m_ = sc[:, j] & 63, sc[:, j + 4] & 63
        else:
            s_ = (sc[:, j + 4] & 0x0F) | ((sc[:, j - 4] >> 6) << 4)
            m_ = (sc[:, j + 4] >> 4) | ((sc[:, j] >> 6) << 4)
        scales[:, j], mins[:, j] = s_, m_
    return scales, mins


def _dequant_32(buf: np.ndarray, typ: int) -> np.ndarray:
    """32-element blocks: Q4_1 (d, m, nibbles), Q5_0 (d, 32 high bits, nibbles;
    offset 16), Q5_1 (d, m, high bits, nibbles), IQ4_NL (d, nibbles indexing
    the 16 IQ4 levels). Nibble j of byte i is element i (low) / i + 16 (high)."""
    ne, nb = BLOCKS[typ]
    b = buf.reshape(-1, nb)
    d = _f16(b[:, 0:2].copy())
    if typ == IQ4_NL:
        qs = b[:, 2:18]
        q = np.concatenate([qs & 0x0F, qs >> 4], axis=1)
        return (IQ4_LEVELS[q] * d).reshape(-1)
    has_m = typ in (Q4_1, Q5_1)
    m = _f16(b[:, 2:4].copy()) if has_m else 0.0
    o = 4 if has_m else 2
    if typ == Q4_1:
        qs = b[:, o : o + 16]
        q = np.concatenate([qs & 0x0F, qs >> 4], axis=1).astype(np.float32)
        return (q * d + m).reshape(-1)
    qh = b[:, o : o + 4].copy().view(np.uint32)  # [blocks, 1]
    qs = b[:, o + 4 : o + 20]
    bits = (qh >> np.arange(32, dtype=np.uint32)[None, :]) & 1  # bit j -> element j
    q = np.concatenate([qs & 0x0F, qs >> 4], axis=1).astype(np.uint32) | (bits << 4)
    q = q.astype(np.float32)
    if typ == Q5_0:
        return ((q - 16.0) * d).reshape(-1)
    return (q * d + m).reshape(-1)


def _dequant_k(buf: np.ndarray, typ: int) -> np.ndarray:
    """256-element super-blocks: Q2_K, Q3_K, Q5_K, IQ4_XS."""
    ne, nb = BLOCKS[typ]
    b = buf.reshape(-1, nb)
    nbk = b.shape[0]
    out = np.empty((nbk, 256), np.float32)
    if typ == Q2_K:
        # scales[16] (low nibble scale, high nibble min), qs[64] (2 bits), d, dmin
        sc, qs = b[:, 0:16], b[:, 16:80]
        d, dmin = _f16(b[:, 80:82].copy()), _f16(b[:, 82:84].copy())
        dl = d * (sc & 0x0F).astype(np.float32)
        ml = dmin * (sc >> 4).astype(np.float32)
        for half in range(2):
            q = qs[:, half * 32 : half * 32 + 32]
            for j in range(4):  # shift 2j
                v = ((q >> (2 * j)) & 3).astype(np.float32)
                for part in range(2):
                    si = half * 8 + j * 2 + part
                    o = half * 128 + j * 32 + part * 16
                    out[:, o : o + 16] = dl[:, si : si + 1] * v[:, part * 16 : part * 16 + 16] - ml[:, si : si + 1]
        return out.reshape(-1)
    if typ == Q3_K:
        # hmask[32] (third bit, 0 means -4), qs[64] (low 2 bits), 16 six-bit scales in 12 bytes, d
        hm, qs, sb = b[:, 0:32], b[:, 32:96], b[:, 96:108].astype(np.uint32)
        d = _f16(b[:, 108:110].copy())
        a = [sb[:, 4 * i] | (sb[:, 4 * i + 1] << 8) | (sb[:, 4 * i + 2] << 16) | (sb[:, 4 * i + 3] << 24)
             for i in range(3)]
        k1, k2 = np.uint32(0x03030303), np.uint32(0x0F0F0F0F)
        words = [(a[0] & k2) | (((a[2] >> 0) & k1) << 4), (a[1] & k2) | (((a[2] >> 2) & k1) << 4),
                 ((a[0] >> 4) & k2) | (((a[2] >> 4) & k1) << 4), ((a[1] >> 4) & k2) | (((a[2] >> 6) & k1) << 4)]
        scales = np.stack([((w >> (8 * k)) & 0xFF) for w in words for k in range(4)], 1).astype(np.float32) - 32.0
        for half in range(2):
            q = qs[:, half * 32 : half * 32 + 32]
            for j in range(4):
                m = 1 << (half * 4 + j)
                v = ((q >> (2 * j)) & 3).astype(np.float32) - np.where(hm & m, 0.0, 4.0)
                for part in range(2):
                    si = half * 8 + j * 2 + part
                    o = half * 128 + j * 32 + part * 16
                    out[:, o : o + 16] = d * scales[:, si : si + 1] * v[:, part * 16 : part * 16 + 16]
        return out.reshape(-1)
    if typ == Q5_K:
        d, dmin = _f16(b[:, 0:2].copy()), _f16(b[:, 2:4].copy())
        scales, mins = _k4_scales(b[:, 4:16])
        qh, qs = b[:, 16:48], b[:, 48:176]
        for g in range(4):
            q = qs[:, g * 32 : g * 32 + 32]
            lo = (q & 0x0F).astype(np.float32) + np.where(qh & (1 << (2 * g)), 16.0, 0.0)
            hi = (q >> 4).astype(np.float32) + np.where(qh & (1 << (2 * g + 1)), 16.0, 0.0)
            out[:, g * 64 : g * 64 + 32] = d * scales[:, 2 * g : 2 * g + 1] * lo - dmin * mins[:, 2 * g : 2 * g + 1]
            out[:, g * 64 + 32 : g * 64 + 64] = (d * scales[:, 2 * g + 1 : 2 * g + 2] * hi
                                                 - dmin * mins[:, 2 * g + 1 : 2 * g + 2])
        return out.reshape(-1)
    if typ == IQ4_XS:
        # d, scales_h (u16: 2 high bits per sub-block), scales_l[4] (nibbles), qs[128]
        d = _f16(b[:, 0:2].copy())
        sh = b[:, 2:4].copy().view(np.uint16).astype(np.uint32)
        sl, qs = b[:, 4:8], b[:, 8:136]
        for ib in range(8):
            ls = ((sl[:, ib // 2] >> (4 * (ib % 2))) & 0x0F).astype(np.uint32) | (((sh[:, 0] >> (2 * ib)) & 3) << 4)
            dl = d[:, 0] * (ls.astype(np.float32) - 32.0)
            q = qs[:, ib * 16 : ib * 16 + 16]
            out[:, ib * 32 : ib * 32 + 16] = dl[:, None] * IQ4_LEVELS[q & 0x0F]
            out[:, ib * 32 + 16 : ib * 32 + 32] = dl[:, None] * IQ4_LEVELS[q >> 4]
        return out.reshape(-1)
    raise NotImplementedError(typ)


# ---------------------------------------------------------------------------- writer
def _quant_q8_0(x: np.ndarray) -> bytes:
    b = x.reshape(-1, 32).astype(np.float32)
    d = np.abs(b).max(axis=1) / 127.0
    d16 = d.astype(np.float16)
    inv = np.where(d16.astype(np.float32) > 0, 1.0 / d16.astype(np.float32), 0.0)
    q = np.clip(np.rint(b * inv[:, None]), -127, 127).astype(np.int8)
    out = np.empty((b.shape[0], 34), np.uint8)
    out[:, :2] = d16.view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.tobytes()


def _quant_q4_0(x: np.ndarray) -> bytes:
    b = x.reshape(-1, 32).astype(np.float32)
    idx = np.abs(b).argmax(axis=1)
    mx = b[np.arange(b.shape[0]), idx]
    d = mx / -8.0
    d16 = d.astype(np.float16)
    inv = np.where(d16.astype(np.float32) != 0, 1.0 / d16.astype(np.float32), 0.0)
    q = np.clip(np.rint(b * inv[:, None]) + 8, 0, 15).astype(np.uint8)
    out = np.empty((b.shape[0], 18), np.uint8)
    out[:, :2] = d16.view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q[:, :16] | (q[:, 16:] << 4)
    return out.tobytes()


def write_gguf(path: str, metadata: dict, tensors: dict, alignment: int = 32) -> None:
    """tensors: name -> (torch tensor [.., K], ggml type in {F32, F16, Q8_0, Q4_0})."""
    def s(x: str) -> bytes:
        e = x.encode()
        return struct.pack("<Q", len(e)) + e

    def val(v) -> bytes:
        if isinstance(v, bool):
            return struct.pack("<I", T_BOOL) + struct.pack("<?", v)
        if isinstance(v, int):
            return struct.pack("<I", T_U32) + struct.pack("<I", v) if 0 <= v < 2**32 else struct.pack("<I", T_I64) + struct.pack("<q", v)
        if isinstance(v, float):
            return struct.pack("<I", T_F32) + struct.pack("<f", v)
        if isinstance(v, str):
            return struct.pack("<I", T_STR) + s(v)
        if isinstance(v, list):
            if all(isinstance(i, str) for i in v):
                return struct.pack("<I", T_ARR) + struct.pack("<IQ", T_STR, len(v)) + b"".join(s(i) for i in v)
            if any(isinstance(i, float) for i in v):  # e.g. tokenizer.ggml.scores
                return struct.pack("<I", T_ARR) + struct.pack("<IQ", T_F32, len(v)) + b"".join(
                    struct.pack("<f", float(i)) for i in v)
            return struct.pack("<I", T_ARR) + struct.pack("<IQ", T_I32, len(v)) + b"".join(struct.pack("<i", i) for i in v)
        raise TypeError(type(v))

    meta = dict(metadata)
    meta["general.alignment"] = alignment
    head = struct.pack("<IIQQ", GGUF_MAGIC, 3, len(tensors), len(meta))
    head += b"".join(s(k) + val(v) for k, v in meta.items())
    blobs, infos, off = [], b"", 0
    for name, (t, typ) in tensors.items():
        x = t.detach().float().cpu().numpy().reshape(-1)
        if typ == F32:
            raw = x.astype(np.float32).tobytes()
        elif typ == F16:
            raw = x.astype(np.float16).tobytes()
        elif typ == Q8_0:
            raw = _quant_q8_0(x)
        elif typ == Q4_0:
            raw = _quant_q4_0(x)
        else:
            raise NotImplementedError(typ)
        dims = list(reversed(t.shape))
        infos += s(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        infos += struct.pack("<IQ", typ, off)
        pad = (-len(raw)) % alignment
        blobs.append(raw + b"\0" * pad)
        off += len(raw) + pad
    body = head + infos
    body += b"\0" * ((-len(body)) % alignment)
    with open(path, "wb") as f:
        f.write(body)
        for b in blobs:
            f.write(b)


# ---------------------------------------------------------------------------- Qwen2 mapping
def qwen_config_from_gguf(g: GGUFFile):
    from ..models.qwen import QwenConfig

    arch = g.meta.get("general.architecture", "qwen2")
    m = lambda k, d=None: g.meta.get(f"{arch}.{k}", d)  # noqa: E731
    vocab = len(g.meta.get("tokenizer.ggml.tokens", [])) or int(g.tensors["token_embd.weight"][0][1])
    d, H = int(m("embedding_length")), int(m("attention.head_count"))
    head_dim = int(m("attention.key_length", d // H))
    return QwenConfig(vocab=vocab, d_model=d, n_layers=int(m("block_count")), n_heads=H,
                      n_kv_heads=int(m("attention.head_count_kv", H)),
                      d_ff=int(m("feed_forward_length")), rope_theta=float(m("rope.freq_base", 1e6)),
                      norm_eps=float(m("attention.layer_norm_rms_epsilon", 1e-6)),
                      tie_embeddings="output.weight" not in g.tensors,
                      qkv_bias="blk.0.attn_q.bias" in g.tensors,
                      qk_norm="blk.0.attn_q_norm.weight" in g.tensors,
                      head_dim_=head_dim if head_dim != d // H else 0,
                      sliding_window=int(m("attention.sliding_window", 0)),
                      sliding_window_pattern=int(m("attention.sliding_window_pattern", 0)),
                      rope_theta_swa=float(m("rope.freq_base_swa", 0.0)),
                      attn_softcap=float(m("attn_logit_softcapping", 0.0)))


def load_qwen_weights(path: str, device="cuda", keep_quant: bool = False):
    """GGUF (llama.cpp tensor names; architectures qwen2, qwen3, llama, mistral)
    -> QwenWeights on `device` (bf16). keep_quant: the four projection groups
    of every layer stay in the file's own blocks on the device (each part its
    own type) and are expanded to bf16 into one shared scratch right before
    each GEMM -- the weights take the file's size in memory, at the cost of an
    expansion per use; embeddings, norms, biases and the LM head are bf16."""
    from ..models.qwen import QwenWeights

    g = GGUFFile(path)
    cfg = qwen_config_from_gguf(g)
    w = QwenWeights.__new__(QwenWeights)
    w.cfg, w.device, w.tp_rank, w.tp_size = cfg, torch.device(device), 0, 1
    w.hq, w.hkv, w.f = cfg.n_heads, cfg.n_kv_heads, cfg.d_ff
    t = lambda n: g.tensor(n).to(device)  # noqa: E731
    if keep_quant:
        from ..models.qlora_gguf import GGUFPart, GGUFWeight

        holder = {}

        def scratch(n):
            buf = holder.get("buf")
            if buf is None or buf.numel() < n:
                buf = holder["buf"] = torch.empty(n, dtype=torch.bfloat16, device=device)
            return buf[:n]

        def q(*names):
            return GGUFWeight([GGUFPart(g, nm, device) for nm in names], scratch)
    else:
        def q(*names):
            return torch.cat([t(nm) for nm in names]).contiguous() if len(names) > 1 else t(names[0])
    w.embed = t("token_embd.weight")
    w.lm_head = w.embed if cfg.tie_embeddings else t("output.weight")
    w.final_norm = t("output_norm.weight")
    w.attn_norm, w.mlp_norm, w.wqkv, w.bqkv, w.wo, w.wgu, w.wd = [], [], [], [], [], [], []
    w.q_norm = [] if cfg.qk_norm else None
    w.k_norm = [] if cfg.qk_norm else None
    for i in range(cfg.n_layers):
        p = f"blk.{i}."
        if cfg.qk_norm:
            w.q_norm.append(t(p + "attn_q_norm.weight"))
            w.k_norm.append(t(p + "attn_k_norm.weight"))
        w.attn_norm.append(t(p + "attn_norm.weight"))
        w.mlp_norm.append(t(p + "ffn_norm.weight"))
        w.wqkv.append(q(p + "attn_q.weight", p + "attn_k.weight", p + "attn_v.weight"))
        w.bqkv.append(torch.cat([t(p + "attn_q.bias"), t(p + "attn_k.bias"), t(p + "attn_v.bias")]).contiguous()
                      if cfg.qkv_bias else None)
        w.wo.append(q(p + "attn_output.weight"))
        w.wgu.append(q(p + "ffn_gate.weight", p + "ffn_up.weight"))
        w.wd.append(q(p + "ffn_down.weight"))
    return cfg, w


def tokenizer_from_gguf(g: GGUFFile):
    """The GGUF file's own tokenizer: SentencePiece (``tokenizer.ggml.model``
    "llama": pieces, scores, token types, BOS / EOS, add-BOS and space-prefix
    flags) or byte-level BPE (``gpt2``: tokens + merges)."""
    from ..serving.tokenizer import BPETokenizer, SPMTokenizer

    if g.meta.get("tokenizer.ggml.model") == "llama":
        toks = g.meta.get("tokenizer.ggml.tokens", [])
        scores = g.meta.get("tokenizer.ggml.scores", [0.0] * len(toks))
        types = g.meta.get("tokenizer.ggml.token_type", [1] * len(toks))
        get = lambda k: (int(g.meta[k]) if k in g.meta else None)  # noqa: E731
        return SPMTokenizer(toks, scores, types, bos_id=get("tokenizer.ggml.bos_token_id"),
                            eos_id=get("tokenizer.ggml.eos_token_id"), unk_id=get("tokenizer.ggml.unknown_token_id"),
                            add_bos=bool(g.meta.get("tokenizer.ggml.add_bos_token", True)),
                            add_space_prefix=bool(g.meta.get("tokenizer.ggml.add_space_prefix", True)))
    toks = g.meta.get("tokenizer.ggml.tokens", [])
    merges = g.meta.get("tokenizer.ggml.merges", [])
    types = g.meta.get("tokenizer.ggml.token_type", [1] * len(toks))
    vocab, added = {}, {}
    for i, (tok, ty) in enumerate(zip(toks, types)):
        (added if ty in (3, 4) else vocab)[tok] = i
    return BPETokenizer(vocab, merges, added)


# ---------------------------------------------------------------------------- DeepSeek-V2 / GLM-4.7-flash mapping
def _rope_rows_to_halves(n: int = 64) -> torch.Tensor:
    """Row order that turns interleaved RoPE pairs (0,1), (2,3), ... -- the
    GGUF / Hugging Face layout of DeepSeek-V2's q_pe / k_pe -- into the
    half-split pairs (i, i + n/2) the kernels rotate: dot products of q_pe and
    k_pe are unchanged when both are reordered the same way."""
    return torch.cat([torch.arange(0, n, 2), torch.arange(1, n, 2)])


def deepseek_config_from_gguf(g: GGUFFile):
    from ..models.deepseek import DeepSeekConfig

    arch = g.meta.get("general.architecture", "deepseek2")
    m = lambda k, d=None: g.meta.get(f"{arch}.{k}", d)  # noqa: E731
    vocab = len(g.meta.get("tokenizer.ggml.tokens", [])) or int(g.tensors["token_embd.weight"][0][1])
    H = int(m("attention.head_count"))
    rope_d = int(m("rope.dimension_count", 64))
    qk = int(m("attention.key_length", 192))
    gating = int(m("expert_gating_func", 1))
    factor = float(m("rope.scaling.factor", 0.0))
    log_mul = float(m("rope.scaling.yarn_log_multiplier", 0.0))  # 0.1 * mscale_all_dim
    return DeepSeekConfig(
        vocab=vocab, d_model=int(m("embedding_length")), n_layers=int(m("block_count")), n_heads=H,
        q_lora_rank=int(m("attention.q_lora_rank", 0)), kv_lora_rank=int(m("attention.kv_lora_rank", 512)),
        qk_nope=qk - rope_d, qk_rope=rope_d, v_head=int(m("attention.value_length", 128)),
        d_ff=int(m("feed_forward_length")), first_dense=int(m("leading_dense_block_count", 1)),
        n_experts=int(m("expert_count", 0)), top_k=int(m("expert_used_count", 0)),
        d_expert=int(m("expert_feed_forward_length", 0)), n_shared=int(m("expert_shared_count", 0)),
        router="sigmoid" if gating == 2 else "softmax", norm_topk=bool(m("expert_weights_norm", False)),
        routed_scale=float(m("expert_weights_scale", 1.0)), rope_theta=float(m("rope.freq_base", 10000.0)),
        yarn_factor=factor if m("rope.scaling.type", "yarn") == "yarn" else 0.0,
        yarn_orig_ctx=int(m("rope.scaling.original_context_length", 4096)),
        yarn_mscale=log_mul / 0.1 if log_mul else 1.0, yarn_mscale_all_dim=log_mul / 0.1 if log_mul else 0.0,
        norm_eps=float(m("attention.layer_norm_rms_epsilon", 1e-6)),
        tie_embeddings="output.weight" not in g.tensors)


def load_deepseek_weights(path: str, device="cuda"):
    """GGUF (llama.cpp ``deepseek2`` tensor names) -> (DeepSeekConfig, DeepSeekWeights)."""
    from ..models.deepseek import DeepSeekWeights

    g = GGUFFile(path)
    cfg = deepseek_config_from_gguf(g)
    dev = torch.device(device)
    t = lambda n: g.tensor(n).to(dev)  # noqa: E731
    w = DeepSeekWeights.__new__(DeepSeekWeights)
    w.cfg, w.device = cfg, dev
    H, qh, nope = cfg.n_heads, cfg.qk_head, cfg.qk_nope
    perm = _rope_rows_to_halves(cfg.qk_rope).to(dev)

    def fix_q(wq):  # rows [H, qh]: reorder each head's RoPE rows
        v = wq.view(H, qh, -1)
        return torch.cat([v[:, :nope], v[:, nope:][:, perm]], 1).reshape(H * qh, -1).contiguous()

    w.embed = t("token_embd.weight")
    w.lm_head = w.embed if cfg.tie_embeddings else t("output.weight")
    w.final_norm = t("output_norm.weight")
    names = ("attn_norm", "mlp_norm", "wq", "wq_a", "q_a_norm", "wq_b", "wkv_a", "kv_norm", "w_uk", "w_uv", "wo",
             "dense_gu", "dense_d", "router", "exp_gu", "exp_d", "sh_gu", "sh_d")
    for n in names:
        setattr(w, n, [])
    for i in range(cfg.n_layers):
        p = f"blk.{i}."
        w.attn_norm.append(t(p + "attn_norm.weight"))
        w.mlp_norm.append(t(p + "ffn_norm.weight"))
        if cfg.q_lora_rank:
            w.wq.append(None)
            w.wq_a.append(t(p + "attn_q_a.weight"))
            w.q_a_norm.append(t(p + "attn_q_a_norm.weight"))
            w.wq_b.append(fix_q(t(p + "attn_q_b.weight")))
        else:
            w.wq.append(fix_q(t(p + "attn_q.weight")))
            for lst in (w.wq_a, w.q_a_norm, w.wq_b):
                lst.append(None)
        kva = t(p + "attn_kv_a_mqa.weight")
        w.wkv_a.append(torch.cat([kva[: cfg.kv_lora_rank], kva[cfg.kv_lora_rank :][perm]]).contiguous())
        w.kv_norm.append(g.tensor(p + "attn_kv_a_norm.weight", torch.float32).to(dev))
        kvb = t(p + "attn_kv_b.weight").view(H, nope + cfg.v_head, cfg.kv_lora_rank)
        w.w_uk.append(kvb[:, :nope].contiguous())
        w.w_uv.append(kvb[:, nope:].contiguous())
        w.wo.append(t(p + "attn_output.weight"))
        if i < cfg.first_dense:
            w.dense_gu.append(torch.cat([t(p + "ffn_gate.weight"), t(p + "ffn_up.weight")]).contiguous())
            w.dense_d.append(t(p + "ffn_down.weight"))
            for lst in (w.router, w.exp_gu, w.exp_d, w.sh_gu, w.sh_d):
                lst.append(None)
            continue
        w.dense_gu.append(None)
        w.dense_d.append(None)
        r = t(p + "ffn_gate_inp.weight")
        Ep = (cfg.n_experts + 7) // 8 * 8
        rp = torch.zeros(Ep, r.shape[1], dtype=r.dtype, device=dev)
        rp[: cfg.n_experts] = r
        w.router.append(rp)
        w.exp_gu.append(torch.cat([t(p + "ffn_gate_exps.weight"), t(p + "ffn_up_exps.weight")], 1).contiguous())
        w.exp_d.append(t(p + "ffn_down_exps.weight").contiguous())
        if cfg.n_shared:
            w.sh_gu.append(torch.cat([t(p + "ffn_gate_shexp.weight"), t(p + "ffn_up_shexp.weight")]).contiguous())
            w.sh_d.append(t(p + "ffn_down_shexp.weight"))
        else:
            w.sh_gu.append(None)
            w.sh_d.append(None)
    return cfg, w
