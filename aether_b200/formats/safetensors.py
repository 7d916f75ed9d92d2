"""safetensors reader / writer (no external dependency).

Format: u64 little-endian header length N, N bytes of JSON
{name: {"dtype", "shape", "data_offsets": [begin, end]}, "__metadata__": {...}},
then the raw little-endian tensor bytes. Reference: safetensors_* in
runtime/src/lib.rs:1220-1232, 1814-1886, 9063-9153 (parse / save / load /
multi-file) with an atomic write (temp file + rename).
"""
from __future__ import annotations

import json
import mmap
import os
import struct

import numpy as np
import torch

_DT = {
    "F32": torch.float32, "F16": torch.float16, "BF16": torch.bfloat16, "F64": torch.float64,
    "I64": torch.int64, "I32": torch.int32, "I16": torch.int16, "I8": torch.int8, "U8": torch.uint8,
    "BOOL": torch.bool,
}
_NAME = {v: k for k, v in _DT.items()}


def save_file(tensors: dict, path: str, metadata: dict | None = None) -> None:
    header = {}
    off = 0
    blobs = []
    for name, t in tensors.items():
        t = t.detach().contiguous().cpu()
        raw = t.view(torch.uint8).numpy().tobytes() if t.dtype != torch.bool else t.numpy().tobytes()
        header[name] = {"dtype": _NAME[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    if metadata:
        header["__metadata__"] = {k: str(v) for k, v in metadata.items()}
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for b in blobs:
            f.write(b)
    os.replace(tmp, path)


def read_header(path: str) -> tuple:
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
    return header, 8 + n


def load_file(path: str, device="cpu", names=None) -> dict:
    header, base = read_header(path)
    out = {}
    with open(path, "rb") as f:
        mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
        try:
            for name, info in header.items():
                if name == "__metadata__" or (names is not None and name not in names):
                    continue
                b, e = info["data_offsets"]
                dt = _DT[info["dtype"]]
                buf = np.frombuffer(mm, dtype=np.uint8, count=e - b, offset=base + b).copy()
                t = torch.from_numpy(buf).view(dt).reshape(info["shape"])
                out[name] = t.to(device)
        finally:
            mm.close()
    return out


def metadata(path: str) -> dict:
    return read_header(path)[0].get("__metadata__", {})
