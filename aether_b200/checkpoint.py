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
DP degree resumes at another. The bucketed DP engine
(``OverlappedDataParallel``) owns one chunk of every layer instead of one
range; its ranks save the list of (arena begin, end) chunks and their
concatenated master / moments, which load into any engine the same way.
ZeRO-2 / ZeRO-3 arenas (``parallel.fsdp``)
save their per-layer-unit shards with the unit layout; loading rebuilds every
parameter's full master and moments by name, so either kind of checkpoint
resumes into either kind of arena at any world size. The bf16 compute copy is rebuilt from the fp32
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


def _sharded(arena) -> bool:
    return hasattr(arena, "units") and hasattr(arena, "scatter_full")


def _slices(opt):
    """[(arena begin, arena end, state offset)] of an engine that owns several
    chunks (OverlappedDataParallel), else None."""
    return getattr(getattr(opt, "opt", opt), "slices", None)


def save(path: str, arena, opt, step: int, rank: int = 0, world: int = 1, extra: dict | None = None) -> None:
    os.makedirs(path, exist_ok=True)
    m, v, get_step, _, start, end = _opt_state(opt)
    end = arena.numel if end is None else end
    meta = {"step": step, "opt_step": get_step(), "start": start, "end": end, "numel": arena.numel,
            "rank": rank, "world": world, "cpu_rng": torch.get_rng_state().tolist()}
    slices = _slices(opt)
    if _sharded(arena):
        meta.update(kind="sharded", layout=arena.layout(), start=0, end=arena.numel)
        start, end = 0, arena.numel
    if arena.device.type == "cuda":
        meta["cuda_rng"] = torch.cuda.get_rng_state(arena.device).tolist()
    if slices is not None:
        meta.update(slices=[[b, e] for b, e, _ in slices], start=0, end=0)
        master = torch.cat([arena.master[b:e] for b, e, _ in slices]) if slices else arena.master[:0]
        n = sum(e - b for b, e, _ in slices)
        tensors = {"master": master, "m": m[:n], "v": v[:n]}
    else:
        tensors = {"master": arena.master[start:end], "m": m, "v": v}
    st.save_file(tensors, os.path.join(path, f"rank{rank:05d}.safetensors"), metadata={"aether": json.dumps(meta)})
    if rank == 0:
        info = {"world": world, "numel": arena.numel, "step": step,
                "slots": {n: [list(s.shape), s.offset, s.numel, s.decay] for n, s in arena.slots.items()},
                "extra": extra or {}}
        if _sharded(arena):
            info.update(kind="sharded", slots={})
        tmp = os.path.join(path, "meta.json.tmp")
        with open(tmp, "w") as f:
            json.dump(info, f)
        os.replace(tmp, os.path.join(path, "meta.json"))


def named_state(path: str) -> tuple:
    """(info, {name: {"master", "m", "v": full fp32 tensors}}, [per-rank meta])
    of a checkpoint of either kind."""
    info = json.load(open(os.path.join(path, "meta.json")))
    metas, shards = [], []
    for r in range(info["world"]):
        f = os.path.join(path, f"rank{r:05d}.safetensors")
        metas.append(json.loads(st.metadata(f)["aether"]))
        shards.append(st.load_file(f))
    out = {}
    if info.get("kind") == "sharded":
        for uid, (_, _, unit_numel, slots) in metas[0]["layout"].items():
            full = {k: torch.cat([sh[k][me["layout"][uid][0] : me["layout"][uid][0] + me["layout"][uid][1]]
                                  for sh, me in zip(shards, metas)])[:unit_numel] for k in ("master", "m", "v")}
            for n, (shape, off, numel, _) in slots.items():
                out[n] = {k: full[k][off : off + numel].view(shape).clone() for k in full}
        return info, out, metas
    full = {k: torch.zeros(info["numel"], dtype=torch.float32) for k in ("master", "m", "v")}
    for me, sh in zip(metas, shards):
        _place(full, me, sh)
    for n, (shape, off, numel, _) in info["slots"].items():
        out[n] = {k: full[k][off : off + numel].view(shape).clone() for k in full}
    return info, out, metas


def _place(full: dict, meta: dict, shard: dict) -> None:
    """Writes one rank's saved state into the full vectors."""
    if "slices" in meta:
        o = 0
        for b, e in meta["slices"]:
            for k in full:
                full[k][b:e] = shard[k][o : o + e - b]
            o += e - b
        return
    for k in full:
        full[k][meta["start"] : meta["end"]] = shard[k]


def _holds(meta: dict, at: int) -> bool:
    if "slices" in meta:
        return any(b <= at < e for b, e in meta["slices"])
    return meta["start"] <= at < meta["end"]


def _restore_rng(meta, device) -> None:
    torch.set_rng_state(torch.tensor(meta["cpu_rng"], dtype=torch.uint8))
    if "cuda_rng" in meta and device.type == "cuda":
        torch.cuda.set_rng_state(torch.tensor(meta["cuda_rng"], dtype=torch.uint8), device)


def load(path: str, arena, opt, restore_rng: bool = True) -> int:
    """Restore ``arena`` (master + bf16) and ``opt`` (moments, step count) from
    a checkpoint directory; returns the saved training step."""
    info = json.load(open(os.path.join(path, "meta.json")))
    if info.get("kind") == "sharded" or _sharded(arena):
        return _load_by_name(path, arena, opt, restore_rng)
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
    slices = _slices(opt)
    first = slices[0][0] if slices else start
    for r in range(info["world"]):
        f = os.path.join(path, f"rank{r:05d}.safetensors")
        meta = json.loads(st.metadata(f)["aether"])
        _place(full, meta, st.load_file(f))
        if my_rank_meta is None or _holds(meta, first):  # the shard that holds ours (rank 0's as a fallback)
            my_rank_meta = meta
    with torch.no_grad():
        arena.master.copy_(full["master"][: arena.numel].to(arena.master.device))
        arena.sync_bf16_from_master()
        if slices is not None:
            for b, e, o in slices:
                m[o : o + e - b].copy_(full["m"][b:e].to(m.device))
                v[o : o + e - b].copy_(full["v"][b:e].to(v.device))
        else:
            m.copy_(full["m"][start:end].to(m.device))
            v.copy_(full["v"][start:end].to(v.device))
    put_step(int(my_rank_meta["opt_step"]))
    if restore_rng:
        torch.set_rng_state(torch.tensor(my_rank_meta["cpu_rng"], dtype=torch.uint8))
        if "cuda_rng" in my_rank_meta and arena.device.type == "cuda":
            torch.cuda.set_rng_state(torch.tensor(my_rank_meta["cuda_rng"], dtype=torch.uint8), arena.device)
    return int(info["step"])


def _load_by_name(path: str, arena, opt, restore_rng: bool) -> int:
    """Resume through named full tensors (a ZeRO-2/3 checkpoint, or any
    checkpoint into a ZeRO-2/3 arena)."""
    info, named, metas = named_state(path)
    missing = [n for n in arena.slots if n not in named]
    if missing:
        raise ValueError(f"checkpoint lacks parameters {missing[:4]}")
    m, v, _, put_step, start, end = _opt_state(opt)
    with torch.no_grad():
        if _sharded(arena):
            for n, t in named.items():
                if n in arena.slots:
                    arena.scatter_full(n, t["master"], arena.master)
                    arena.scatter_full(n, t["m"], m)
                    arena.scatter_full(n, t["v"], v)
        else:
            end = arena.numel if end is None else end
            fm = torch.zeros(arena.numel, dtype=torch.float32)
            fv = torch.zeros(arena.numel, dtype=torch.float32)
            for n, t in named.items():
                if n in arena.slots:
                    s = arena.slots[n]
                    arena.master_view(n).copy_(t["master"].to(arena.master.device))
                    fm[s.offset : s.offset + s.numel] = t["m"].reshape(-1)
                    fv[s.offset : s.offset + s.numel] = t["v"].reshape(-1)
            slices = _slices(opt)
            if slices is not None:
                for b, e, o in slices:
                    m[o : o + e - b].copy_(fm[b:e].to(m.device))
                    v[o : o + e - b].copy_(fv[b:e].to(v.device))
            else:
                m.copy_(fm[start:end].to(m.device))
                v.copy_(fv[start:end].to(v.device))
        arena.sync_bf16_from_master()
    rank = getattr(arena, "rank", 0)
    me = metas[rank] if rank < len(metas) else metas[0]
    put_step(int(me["opt_step"]))
    if restore_rng:
        _restore_rng(me, arena.device)
    return int(info["step"])
