"""Fused compute + collective paths against their NVLink roofline.

    torchrun --nproc-per-node N -m aether_b200.bench_comm

1. Data-parallel optimiser step of the GPT-24L arena (1.36 G parameters):
   the one-kernel fused path (reduce the fp32 gradient shard across ranks
   with NVLS multimem.ld_reduce or peer loads, AdamW on the fp32 master shard,
   write the bf16 parameters into every rank with multimem.st or peer stores)
   against the NCCL baseline (reduce-scatter, AdamW kernel, all-gather).
   Roofline: the bytes each GPU must push over NVLink at the measured
   770 GB/s per direction -- with NVLS, its whole fp32 gradient (the switch
   reads every element once for the rank that owns it) plus its bf16 shard
   (multicast once) on the egress side.
2. Tensor-parallel decode reduction (Qwen2.5-7B o_proj shape, batch 1 / 64):
   the decode GEMM whose epilogue reduces through multimem.red into every
   rank's accumulator and whose last CTA signals completion to the consuming
   finalize kernel, against the same GEMM followed by an NCCL all-reduce. Roofline: max(weight bytes / HBM bandwidth,
   output bytes over NVLink / link bandwidth).
3. Tensor-parallel training projections (`--only tp_train`): the fused
   all-gather -> GEMM and GEMM -> reduce-scatter kernels against NCCL around
   the plain GEMM; roofline max(FLOPs / measured GEMM peak, NVLink bytes /
   link bandwidth).
Times are CUDA-event device times, max over ranks, after warm-up.
"""
from __future__ import annotations

import json
import os

import torch
import torch.distributed as dist

LINK_GBS = 770.0  # measured peer copy per direction per GPU on this pool


def timed(fn, iters=10, warmup=3):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / iters], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


def hbm_gbs():
    try:
        with open(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")) as f:
            return json.load(f)["hbm_gbs"]
    except (OSError, KeyError, ValueError):
        return 6650.0


def dp_step(info, out):
    from .models.arena import ParamArena
    from .models.gpt import GPTConfig, gpt_param_specs
    from .parallel.dp import DataParallel, FusedDataParallel, team_alloc
    from .parallel.symm import SymmTeam

    cfg = GPTConfig.gpt_24l()
    team = SymmTeam(info, timeout_s=60.0)
    world = info.world
    fused_arena = ParamArena(gpt_param_specs(cfg), info.device, pad_multiple=world, alloc=team_alloc(team))
    fused_arena.grad.normal_()
    fused = FusedDataParallel(fused_arena, team)
    t_fused = timed(lambda: fused.step(lr=1e-4))
    n = fused_arena.numel
    del fused, fused_arena
    torch.cuda.empty_cache()
    base_arena = ParamArena(gpt_param_specs(cfg), info.device, pad_multiple=world)
    base_arena.grad.normal_()
    base = DataParallel(base_arena, info)
    t_nccl = timed(lambda: base.step(lr=1e-4))
    egress = n * 4 + (n // world) * 2  # fp32 gradient read by the switch + own bf16 shard multicast
    roof = egress / (LINK_GBS * 1e9) * 1e3
    out.append({"path": "dp_reduce_adamw_broadcast", "world": world, "params": n, "fused_ms": t_fused,
                "nccl_ms": t_nccl, "roofline_ms": roof, "fused_frac_of_roofline": roof / t_fused,
                "nvlink": "770 GB/s per direction (measured peer copy)"})


def tp_reduce(info, out):
    from .ops import functional as F
    from .parallel.tp import TensorParallel

    tp = TensorParallel(info)
    world, dev = info.world, info.device
    d = 3584
    K = 3584 // world if 3584 % world == 0 else 512
    w = (torch.randn(d, K, device=dev) * 0.02).bfloat16()
    y = torch.empty(64, d, dtype=torch.bfloat16, device=dev)
    acc_local = torch.zeros(64, d, device=dev)
    for B in (1, 64):
        x = torch.randn(B, K, device=dev).bfloat16()

        def fused():
            F.skinny_finalize(tp.reduce_gemm(x, w, 0), y[:B], wait=tp.finalize_wait())

        def nccl():
            F.skinny_gemm(x, w, acc_local[:B])
            dist.all_reduce(acc_local[:B])
            F.skinny_finalize(acc_local[:B], y[:B])

        tp.signal = True
        t_f = timed(fused, iters=200)
        tp.signal = False  # same GEMM, then a separate team-barrier launch
        t_b = timed(fused, iters=200)
        tp.signal = True
        t_n = timed(nccl, iters=200)
        roof = max(d * K * 2 / (hbm_gbs() * 1e9), B * d * 4 / (LINK_GBS * 1e9)) * 1e3
        best = min(t_f, t_b)
        out.append({"path": "tp_decode_gemm_allreduce", "world": world, "batch": B, "K": K, "N": d,
                    "fused_signal_us": t_f * 1e3, "fused_barrier_us": t_b * 1e3, "nccl_us": t_n * 1e3,
                    "roofline_us": roof * 1e3, "fused_frac_of_roofline": roof / best})
    tp.close()


def bf16_tflops():
    try:
        with open(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")) as f:
            return json.load(f)["bf16_tflops"]
    except (OSError, KeyError, ValueError):
        return 1590.0


def tp_train(info, out):
    """Fused tensor-parallel training projections (csrc/gemm_tp.cu) at the
    GPT-24L micro-batch (16 x 2048 tokens, d 2048): the qkv all-gather -> GEMM
    and the o_proj GEMM -> reduce-scatter (+ residual) of one layer, against
    NCCL all-gather / reduce-scatter around the plain tcgen05 GEMM. Roofline of
    the fused pair: the slower of its FLOPs at the measured GEMM peak and the
    bytes this GPU must send over NVLink (its rows once per peer, P2P stores;
    its partial sums of the other ranks' rows) at the measured link rate."""
    from .ops import functional as F
    from .parallel.symm import SymmTeam
    from .parallel.tp_fused import FusedTP

    tp, d, M = info.world, 2048, 16 * 2048
    Ml, nq, nin = M // tp, 3 * d // tp, d // tp
    g = torch.Generator(device="cuda").manual_seed(info.rank)
    bf = dict(dtype=torch.bfloat16, device="cuda")
    h = torch.randn(Ml, d, generator=g, **bf)
    wq = torch.randn(nq, d, generator=g, **bf) * 0.02
    o = torch.randn(M, nin, generator=g, **bf)
    wo = torch.randn(d, nin, generator=g, **bf) * 0.02
    r = torch.randn(Ml, d, generator=g, **bf)
    team = SymmTeam(info, timeout_s=60.0)
    f = FusedTP(team)

    def fused():
        f.column(h, wq)
        f.row(o, wo, r)

    hf = torch.empty(M, d, **bf)
    xs = torch.empty(Ml, d, **bf)

    def nccl():
        dist.all_gather_into_tensor(hf, h)
        F.gemm(hf, wq)
        y = F.gemm(o, wo)
        dist.reduce_scatter_tensor(xs, y)
        xs.add_(r)

    t_f = timed(fused)
    t_n = timed(nccl)
    flops = 2.0 * M * nq * d + 2.0 * M * d * nin
    ag_bytes = Ml * d * 2 * (tp - 1)
    rs_bytes = (tp - 1) * Ml * d * 2
    t_comp = flops / (bf16_tflops() * 1e12) * 1e3
    t_link = (ag_bytes + rs_bytes) / (LINK_GBS * 1e9) * 1e3
    roof = max(t_comp, t_link)
    out.append({"path": "tp_train_fused_ag_gemm_rs", "tp": tp, "tokens": M, "d_model": d,
                "fused_ms": t_f, "nccl_ms": t_n, "speedup_vs_nccl": t_n / t_f, "roofline_ms": roof,
                "roofline_compute_ms": t_comp, "roofline_nvlink_ms": t_link, "frac_of_roofline": roof / t_f})
    del team


def main():
    import sys

    from .parallel import dist as D

    only = sys.argv[sys.argv.index("--only") + 1].split(",") if "--only" in sys.argv else ["dp", "tp", "tp_train"]
    info = D.init(timeout_s=300)
    out = []
    if "dp" in only:
        dp_step(info, out)
        torch.cuda.empty_cache()
    if "tp" in only:
        tp_reduce(info, out)
        torch.cuda.empty_cache()
    if "tp_train" in only:
        tp_train(info, out)
    if info.rank == 0:
        for r in out:
            print(json.dumps(r), flush=True)
    dist.barrier()
    D.shutdown()


if __name__ == "__main__":
    main()
