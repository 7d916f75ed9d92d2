"""Sharded training checkpoints with exact resume.

Each data-parallel rank writes ``rank{r:05d}.safetensors`` holding its ZeRO-1
shard: the fp32 master weights ``master`` [start, end), the AdamW moments
``m``/``v`` of that range, and metadata (step, optimiser step count, shard
bounds, arena size, CPU and CUDA RNG states). Rank 0 also writes
``meta.json`` (world size, arena size, slot table, user metadata). Every file
goes through a temp-file + rename, so a crash mid-save leaves the previous
checkpoint readable.

Loading concatenates all ranks' shards into the full master / moment vectors
and slices the caller's own shard out of them, so a checkpoint written at one
DP degree resumes at another. The bf16 compute copy is rebuilt from the fp32
master (bf16 = round(master), which is how every optimiser step writes it), so
the continuation is bit-identical to an uninterrupted run.

Reference: the AetherLM ``.weights``/``.meta`` checkpoint
(trainer/src/main.rs:166-211, params only) and the safetensors optimiser
round trip (runtime/src/lib.rs:1814-1886,
tests/runtime/checkpoint_resume.aether). Those formats are kept by
``formats/aether_weights.py``; this module adds the optimiser state, step and
RNG that a DP resume needs.
"""
from __future__ import annotations

import json
import os

import torch

from .formats import safetensors as st


def _opt_state(opt):
    """(m, v, get_step, set_step, start, end) of FlatAdamW, DataParallel or
    FusedDataParallel."""
    inner = getattr(opt, "opt", opt)
    start = getattr(inner, "start", 0)
    end = getattr(inner, "end", None)

    def get():
        return inner.step_count

    def put(s):
        inner.step_count = s

    return inner.m, inner.v, get, put, start, end


def save(path: str, arena, opt, step: int, rank: int = 0, world: int = 1, extra: dict | None = None) -> None:
    os.makedirs(path, exist_ok=True)
    m, v, get_step, _, start, end = _opt_state(opt)
    end = arena.numel if end is None else end
    meta = {"step": step, "opt_step": get_step(), "start": start, "end": end, "numel": arena.numel,
            "rank": rank, "world": world, "cpu_rng": torch.get_rng_state().tolist()}
    if arena.device.type == "cuda":
        meta["cuda_rng"] = torch.cuda.get_rng_state(arena.device).tolist()
    st.save_file({"master": arena.master[start:end], "m": m, "v": v}, os.path.join(path, f"rank{rank:05d}.safetensors"),
                 metadata={"aether": json.dumps(meta)})
    if rank == 0:
        info = {"world": world, "numel": arena.numel, "step": step,
                "slots": {n: [list(s.shape), s.offset, s.numel, s.decay] for n, s in arena.slots.items()},
                "extra": extra or {}}
        tmp = os.path.join(path, "meta.json.tmp")
        with open(tmp, "w") as f:
            json.dump(info, f)
        os.replace(tmp, os.path.join(path, "meta.json"))


def load(path: str, arena, opt, restore_rng: bool = True) -> int:
    """Restore ``arena`` (master + bf16) and ``opt`` (moments, step count) from
    a checkpoint directory; returns the saved training step."""
    info = json.load(open(os.path.join(path, "meta.json")))
    if info["numel"] != arena.numel:
        # a different DP degree pads the arena differently; the slots must agree
        for n, s in arena.slots.items():
            shape, off, numel, _ = info["slots"][n]
            if off != s.offset or numel != s.numel:
                raise ValueError(f"checkpoint slot {n} does not match the model")
    full = {k: torch.zeros(max(info["numel"], arena.numel), dtype=torch.float32) for k in ("master", "m", "v")}
    my_rank_meta = None
    m, v, _, put_step, start, end = _opt_state(opt)
    end = arena.numel if end is None else end
    for r in range(info["world"]):
        f = os.path.join(path, f"rank{r:05d}.safetensors")
        meta = json.loads(st.metadata(f)["aether"])
        t = st.load_file(f)
        s, e = meta["start"], meta["end"]
        for k in full:
            full[k][s:e] = t[k]
        if my_rank_meta is None or s <= start < e:  # the shard that holds ours (rank 0's as a fallback)
            my_rank_meta = meta
    with torch.no_grad():
        arena.master.copy_(full["master"][: arena.numel].to(arena.master.device))
        arena.sync_bf16_from_master()
        m.copy_(full["m"][start:end].to(m.device))
        v.copy_(full["v"][start:end].to(v.device))
    put_step(int(my_rank_meta["opt_step"]))
    if restore_rng:
        torch.set_rng_state(torch.tensor(my_rank_meta["cpu_rng"], dtype=torch.uint8))
        if "cuda_rng" in my_rank_meta and arena.device.type == "cuda":
            torch.cuda.set_rng_state(torch.tensor(my_rank_meta["cuda_rng"], dtype=torch.uint8), arena.device)
    return int(info["step"])
