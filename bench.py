#!/usr/bin/env python
"""Headline benchmark: GPT-24L (d2048, 16 heads, SwiGLU 5632, vocab 32000,
seq 2048) training tokens/s, global batch 256 sequences, bf16 compute with
fp32 master weights and AdamW, data-parallel over N GPUs (one process per GPU).

    python bench.py --gpus N --steps K --warmup W
    torchrun --nproc-per-node N bench.py --gpus N ...      (N > 1)

Rank 0 prints one JSON line. ``value`` is whole-job tokens/s from CUDA events
around exactly K steps (max over ranks) with device-resident synthetic inputs;
``e2e`` repeats the measurement through the public ``Trainer.train_step`` API
with each step's token ids copied from pinned host memory and the loss read
back to the host every step.

``--impl reference`` reports why the reference implementation cannot run here.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

REFERENCE_UNAVAILABLE = (
    "the reference (suhteevah/aether) is a Rust cargo workspace with no setup.py/pyproject "
    "(pip install of it fails) and this image has no cargo/rustc, so its NCCL+cuBLAS build "
    "cannot be built offline"
)


class ClockSampler:
    """Samples nvidia-smi clocks/throttle reasons every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices):
        self.gpus = set(gpu_indices)
        self.rows = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.rows.append(parts)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, smax, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            try:
                idx = int(r[0])
            except ValueError:
                continue
            if self.gpus and idx not in self.gpus:
                continue
            try:
                sm.append(float(r[1]))
                smax.append(float(r[2]))
                power.append(float(r[3]))
            except ValueError:
                pass
            for n, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        loaded = [s for s in sm if s > 0]
        return {
            "sm_mhz": statistics.median(loaded) if loaded else None,
            "sm_max_mhz": max(smax) if smax else None,
            "power_w_max": max(power) if power else None,
            "samples": len(sm),
            "reasons": sorted(reasons),
        }


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="aether", choices=["aether", "reference"])
    ap.add_argument("--global-batch", type=int, default=256)
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--micro-batch", type=int, default=16,
                    help="sequences per forward/backward pass (16: ~56 GB of activations on one GPU)")
    ap.add_argument("--layers", type=int, default=24, help="debug only; anything but 24 is not the benchmark config")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--dp", default="fused", choices=["fused", "nccl"],
                    help="fused: one-kernel NVLink reduce + AdamW + broadcast; nccl: NCCL reduce-scatter/all-gather")
    ap.add_argument("--tp", type=int, default=1, help="tensor-parallel degree (TP x DP mesh, e.g. --gpus 8 --tp 4)")
    ap.add_argument("--pp", type=int, default=1, help="pipeline stages (1F1B over NCCL p2p); --gpus must equal --pp")
    ap.add_argument("--sp", action="store_true",
                    help="sequence parallelism inside TP (residual stream split by token over the TP ranks)")
    ap.add_argument("--tp-comm", default="symm", choices=["symm", "nccl"],
                    help="TP all-reduce: in-kernel symmetric-memory (NVLS / peer loads) or NCCL")
    return ap.parse_args()


def main():
    args = parse()
    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) == 0:
            print(json.dumps({"impl": "reference", "unavailable": REFERENCE_UNAVAILABLE}), flush=True)
        return 0

    import torch

    from aether_b200 import _ext
    from aether_b200.models.gpt import GPT, GPTConfig
    from aether_b200.parallel import dist as D
    from aether_b200.train import Trainer

    assert args.warmup >= 3 or os.environ.get("AETHER_BENCH_DEBUG"), "at least 3 warm-up steps"
    info = D.init(timeout_s=600)
    world = info.world
    assert world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE={world}"
    _ext.require_cuda_kernels()
    dev = info.device
    torch.manual_seed(0)

    cfg = GPTConfig(n_layers=args.layers)
    S = args.seq
    if args.pp > 1:
        return run_pp(args, info, cfg)
    tp = args.tp
    assert world % tp == 0, "--gpus must be a multiple of --tp"
    dp_world = world // tp
    assert args.global_batch % dp_world == 0
    per_rank = args.global_batch // dp_world  # sequences per DP replica (shared by its TP ranks)
    dp = None
    mesh = None
    dinfo = info
    if tp > 1:
        from aether_b200.parallel.tp_train import make_mesh

        mesh = make_mesh(tp, use_symm=args.tp_comm == "symm", sequence_parallel=args.sp)
        dinfo = D.DistInfo(mesh.dp_rank, dp_world, info.local_rank, dev, info.backend)
    if dp_world > 1 and args.dp == "fused":
        from aether_b200.parallel.dp import FusedDataParallel, team_alloc
        from aether_b200.parallel.symm import SymmTeam

        team = SymmTeam(info, group=mesh.dp_group if mesh else None, timeout_s=60.0)
        model = GPT(cfg, device=dev, seed=1234, pad_multiple=dp_world, alloc=team_alloc(team),
                    tp=mesh.tp if mesh else None)
        dp = FusedDataParallel(model.arena, team, lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    else:
        model = GPT(cfg, device=dev, seed=1234, pad_multiple=dp_world, tp=mesh.tp if mesh else None)
        if mesh is not None:
            from aether_b200.parallel.dp import DataParallel

            dp = DataParallel(model.arena, dinfo, lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1,
                              group=mesh.dp_group)
    trainer = Trainer(model, dinfo, lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1,
                      micro_batch=args.micro_batch, dp=dp)

    gen = torch.Generator().manual_seed(1000 + (mesh.dp_rank if mesh else info.rank))
    host = [torch.randint(0, cfg.vocab, (per_rank, S + 1), generator=gen, dtype=torch.int64).pin_memory()
            for _ in range(2)]
    dev_batch = host[0].to(dev)

    for _ in range(args.warmup):
        trainer.train_step(dev_batch)
    torch.cuda.synchronize()
    D.barrier()

    # ---------------------------------------------------------------- device-timed region
    sampler = ClockSampler(range(torch.cuda.device_count())) if info.is_main else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    D.barrier()
    torch.cuda.synchronize()
    _ext.count_launches(True)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        trainer.train_step(dev_batch)
    e1.record()
    torch.cuda.synchronize()
    launches = _ext.count_launches(False)
    D.barrier()
    clocks = sampler.stop() if sampler else None
    ms = e0.elapsed_time(e1) / args.steps
    ms = D.all_reduce_max(ms, dev)
    tokens_per_step = args.global_batch * S
    value = tokens_per_step / (ms / 1e3)

    # ---------------------------------------------------------------- end-to-end region
    e2e = None
    if not args.no_e2e:
        k2 = max(2, args.steps // 2)
        torch.cuda.synchronize()
        D.barrier()
        t0 = time.perf_counter()
        losses = []
        for i in range(k2):
            loss = trainer.train_step(host[i % 2])  # pinned host -> device copy inside the API
            losses.append(float(loss.item()))       # device -> host read of the step's loss
        torch.cuda.synchronize()
        wall = (time.perf_counter() - t0) / k2 * 1e3
        wall = D.all_reduce_max(wall, dev)
        e2e = {
            "value": tokens_per_step / (wall / 1e3),
            "unit": "tokens/s",
            "ms_per_step": wall,
            "steps": k2,
            "h2d_bytes_per_step": per_rank * (S + 1) * 8 * world,
            "d2h_bytes_per_step": 4 * world,
            "last_loss": losses[-1],
            "timing": "host wall clock around Trainer.train_step + loss.item(), max over ranks",
        }

    flops_tok = cfg.flops_per_token(S)
    tflops_per_gpu = value * flops_tok / world / 1e12
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except (OSError, ValueError):
        pass
    peak_sus = peaks.get("bf16_tflops_sustained", 1400.0)

    if info.is_main:
        out = {
            "metric": "train_tokens_per_s",
            "value": value,
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic: uniform-random token ids, random-init N(0,0.02) weights",
            "config": {
                "model": f"GPT-{cfg.n_layers}L d{cfg.d_model} {cfg.n_heads}H SwiGLU-{cfg.d_ff} RMSNorm RoPE vocab{cfg.vocab}",
                "params": cfg.n_params(),
                "global_batch": args.global_batch,
                "seq_len": S,
                "micro_batch": args.micro_batch,
                "parallelism": (f"tp{tp}x" if tp > 1 else "") + f"dp{dp_world}"
                + ((" zero1 " + ("fused-nvlink" if args.dp == "fused" else "nccl")) if dp_world > 1 else "")
                + (f" tp-allreduce-{args.tp_comm}" if tp > 1 else "") + (" sp" if tp > 1 and args.sp else ""),
                "optimizer": "AdamW lr 3e-4 betas (0.9,0.95) wd 0.1, fp32 master",
                "l2": "no flush needed: per-step working set (2.7 GB bf16 weights + activations) >> 126 MB L2",
            },
            "model_tflops_per_gpu": tflops_per_gpu,
            "frac_of_measured_bf16_sustained": tflops_per_gpu / peak_sus,
            "clocks": clocks,
            "e2e": e2e,
            "gpu_launches": launches,
            "impl": "aether",
        }
        print(json.dumps(out), flush=True)
    D.barrier()
    D.shutdown()
    return 0


def run_pp(args, info, cfg):
    """GPT-24L as a 1F1B pipeline: one stage per GPU, the global batch split
    into micro-batches, activations and gradients over NCCL p2p."""
    import torch

    from aether_b200 import _ext
    from aether_b200.parallel import dist as D
    from aether_b200.parallel.pp import GPTPipelineStage, run_1f1b

    world, S = info.world, args.seq
    assert world == args.pp, "--gpus must equal --pp (pure pipeline)"
    st = GPTPipelineStage(cfg, info.rank, world, info.device, seed=1234, lr=3e-4, weight_decay=0.1)
    gen = torch.Generator().manual_seed(1000)  # every rank sees the same micro-batches
    toks = torch.randint(0, cfg.vocab, (args.global_batch, S + 1), generator=gen, dtype=torch.int64)
    n_mb = args.global_batch // args.micro_batch
    host = [(toks[i * args.micro_batch : (i + 1) * args.micro_batch, :-1].contiguous().pin_memory(),
             toks[i * args.micro_batch : (i + 1) * args.micro_batch, 1:].contiguous().pin_memory()) for i in range(n_mb)]
    dev = [(a.to(info.device), b.to(info.device)) for a, b in host]

    def step(batches):
        st.zero_grad()
        loss = run_1f1b(st, batches)
        st.step()
        return loss

    for _ in range(args.warmup):
        step(dev)
    torch.cuda.synchronize()
    D.barrier()
    sampler = ClockSampler(range(torch.cuda.device_count())) if info.is_main else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    D.barrier()
    torch.cuda.synchronize()
    _ext.count_launches(True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step(dev)
    e1.record()
    torch.cuda.synchronize()
    launches = _ext.count_launches(False)
    D.barrier()
    clocks = sampler.stop() if sampler else None
    ms = D.all_reduce_max(e0.elapsed_time(e1) / args.steps, info.device)
    tokens = args.global_batch * S
    value = tokens / (ms / 1e3)
    e2e = None
    if not args.no_e2e:
        torch.cuda.synchronize()
        D.barrier()
        t0 = time.perf_counter()
        k2 = max(2, args.steps // 2)
        for _ in range(k2):
            loss = step(host)  # pinned host -> device inside the schedule
            if loss is not None:
                float(loss.item())
        torch.cuda.synchronize()
        wall = D.all_reduce_max((time.perf_counter() - t0) / k2 * 1e3, info.device)
        e2e = {"value": tokens / (wall / 1e3), "unit": "tokens/s", "ms_per_step": wall, "steps": k2,
               "h2d_bytes_per_step": 2 * args.global_batch * S * 8 * world, "d2h_bytes_per_step": 4,
               "timing": "host wall clock around run_1f1b + step + loss.item(), max over ranks"}
    if info.is_main:
        tflops = value * cfg.flops_per_token(S) / world / 1e12
        print(json.dumps({
            "metric": "train_tokens_per_s", "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic: uniform-random token ids, random-init weights",
            "config": {"model": f"GPT-{cfg.n_layers}L d{cfg.d_model} {cfg.n_heads}H SwiGLU-{cfg.d_ff} vocab{cfg.vocab}",
                       "params": cfg.n_params(), "global_batch": args.global_batch, "seq_len": S,
                       "micro_batch": args.micro_batch, "parallelism": f"pp{world} 1f1b nccl-p2p",
                       "l2": "no flush needed: per-step working set >> 126 MB L2"},
            "model_tflops_per_gpu": tflops, "clocks": clocks, "e2e": e2e, "gpu_launches": launches, "impl": "aether"}),
            flush=True)
    D.barrier()
    D.shutdown()
    return 0


if __name__ == "__main__":
    sys.exit(main())
