"""AetherLM checkpoint files, byte-compatible with the reference trainer.

``<stem>.weights`` = the 9 bytes ``AETHER01\\n`` + u64 little-endian parameter
count + that many little-endian fp32 values (the flat parameter arena in
layout order); ``<stem>.meta`` = one line of JSON
``{"vocab","d_model","n_layers","n_heads","d_ff","seq_len","params"}``.
Reference: save_checkpoint (trainer/src/main.rs:166-191) and the loader in
trainer/src/bin/infer.rs:67-90. The native AetherLM trainer in
``csrc/rt/nano.cpp`` writes the same files; this module reads and writes them
from Python.
"""
from __future__ import annotations

import json
import os
import struct

import numpy as np

MAGIC = b"AETHER01\n"


def save(stem: str, params: np.ndarray, meta: dict) -> None:
    p = np.ascontiguousarray(params, dtype="<f4").reshape(-1)
    tmp = stem + ".weights.tmp"
    with open(tmp, "wb") as f:
        f.write(MAGIC)
        f.write(struct.pack("<Q", p.size))
        f.write(p.tobytes())
    os.replace(tmp, stem + ".weights")
    keys = ("vocab", "d_model", "n_layers", "n_heads", "d_ff", "seq_len")
    line = {k: int(meta[k]) for k in keys}
    line["params"] = int(p.size)
    with open(stem + ".meta", "w") as f:
        f.write(json.dumps(line, separators=(",", ":")) + "\n")


def load(stem_or_path: str) -> tuple:
    """-> (params fp32 ndarray, meta dict or None)."""
    path = stem_or_path if stem_or_path.endswith(".weights") else stem_or_path + ".weights"
    with open(path, "rb") as f:
        if f.read(9) != MAGIC:
            raise ValueError(f"{path}: bad magic")
        n = struct.unpack("<Q", f.read(8))[0]
        p = np.frombuffer(f.read(4 * n), dtype="<f4")
    if p.size != n:
        raise ValueError(f"{path}: truncated ({p.size} of {n} values)")
    meta_path = path[: -len(".weights")] + ".meta"
    meta = json.load(open(meta_path)) if os.path.exists(meta_path) else None
    return p.copy(), meta
