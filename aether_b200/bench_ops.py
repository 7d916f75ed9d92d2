"""Runtime op sweep on one B200 (bf16 in / fp32 accumulate, N(0,1) inputs):

  matmul M=N=K in {1024, 4096, 8192} fwd + bwd (dgrad + wgrad)
  causal SDPA B=8, H=32, S in {512, 2048, 8192}, D=128 fwd + bwd
  layer_norm and softmax over [8*2048, 4096]
  cross_entropy over logits [8*2048, 152064] with uniform-random targets
  AdamW over a 1e9-element fp32 param/grad/m/v set

Each op is timed with CUDA events on the launching stream after warm-up
(median of ``--iters``), next to the torch / cuBLAS / cuDNN path for the same
op. Inputs of every case are larger than L2, except the 1024^3 GEMM, which is
also timed with an L2 flush between iterations. Prints one JSON object per op.

    python -m aether_b200.bench_ops [--only gemm,sdpa,...] [--iters 10]
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics

import torch

from . import _ext
from .ops import functional as F

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, "fallback"


_FLUSH = None


def flush_l2():
    global _FLUSH
    if _FLUSH is None:
        _FLUSH = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")
    _FLUSH.zero_()


def time_fn(fn, iters=10, warmup=3, flush=False):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        if flush:
            flush_l2()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1))
    return statistics.median(ts)


def emit(rec):
    print(json.dumps(rec), flush=True)


def bench_gemm(iters):
    hbm, tf, src = peaks()
    for n in (1024, 4096, 8192):
        a = torch.randn(n, n, device="cuda").bfloat16()
        w = torch.randn(n, n, device="cuda").bfloat16()
        dy = torch.randn(n, n, device="cuda").bfloat16()
        gw = torch.zeros(n, n, device="cuda")
        flops = 2.0 * n**3
        small = n <= 1024
        t_f = time_fn(lambda: F.gemm(a, w), iters, flush=small)
        t_dg = time_fn(lambda: F.gemm(dy, w, b_mn=True), iters, flush=small)
        t_wg = time_fn(lambda: F.gemm(dy, a, a_mn=True, b_mn=True, out=gw, accumulate=True), iters, flush=small)
        c_f = time_fn(lambda: a @ w.t(), iters, flush=small)
        c_dg = time_fn(lambda: dy @ w, iters, flush=small)
        c_wg = time_fn(lambda: gw.add_((dy.t() @ a).float()), iters, flush=small)
        for name, t, c in (("fwd", t_f, c_f), ("dgrad", t_dg, c_dg), ("wgrad_f32acc", t_wg, c_wg)):
            emit({"op": f"matmul_{name}", "shape": [n, n, n], "ms": t, "tflops": flops / t / 1e9,
                  "frac_of_peak": flops / t / 1e9 / tf, "peak": src, "torch_cublas_ms": c,
                  "speedup_vs_cublas": c / t, "l2_flush": small})


def bench_gemm_pair(iters):
    """The CTA-pair (cta_group::2, 256 x 256 tile) GEMM against the one-CTA
    kernel and torch (cuBLAS), square sizes and the GPT-24L training shapes
    (micro-batch 16 x 2048 tokens): forward x.W^T, dgrad dy.W, wgrad dy^T.x
    into fp32."""
    hbm, tf, src = peaks()
    C = _ext.C()
    T = 16 * 2048
    shapes = [(n, n, n) for n in (4096, 8192)] + [(T, 6144, 2048), (T, 2048, 2048), (T, 11264, 2048), (T, 2048, 5632)]
    for M, N, K in shapes:
        x = torch.randn(M, K, device="cuda").bfloat16()
        w = torch.randn(N, K, device="cuda").bfloat16()
        dy = torch.randn(M, N, device="cuda").bfloat16()
        gw = torch.zeros(N, K, device="cuda")
        flops = 2.0 * M * N * K
        cases = (("fwd", lambda: F.gemm(x, w), lambda: x @ w.t()),
                 ("dgrad", lambda: F.gemm(dy, w, b_mn=True), lambda: dy @ w),
                 ("wgrad_f32acc", lambda: F.gemm(dy, x, a_mn=True, b_mn=True, out=gw, accumulate=True),
                  lambda: gw.add_((dy.t() @ x).float())))
        for name, fn, tfn in cases:
            res = {}
            for mode in (0, 1):
                old = C.gemm_pair_mode(mode)
                try:
                    res[mode] = time_fn(fn, iters)
                finally:
                    C.gemm_pair_mode(old)
            c = time_fn(tfn, iters)
            emit({"op": f"matmul_{name}_pair", "shape": [M, N, K], "one_cta_ms": res[0], "pair_ms": res[1],
                  "one_cta_tflops": flops / res[0] / 1e9, "pair_tflops": flops / res[1] / 1e9,
                  "pair_frac_of_peak": flops / res[1] / 1e9 / tf, "peak": src, "torch_cublas_ms": c,
                  "pair_speedup_vs_cublas": c / res[1], "pair_speedup_vs_one_cta": res[0] / res[1]})


def bench_sdpa(iters):
    hbm, tf, src = peaks()
    B, H, D = 8, 32, 128
    for S in (512, 2048, 8192):
        q = torch.randn(B, S, H, D, device="cuda").bfloat16()
        k = torch.randn(B, S, H, D, device="cuda").bfloat16()
        v = torch.randn(B, S, H, D, device="cuda").bfloat16()
        do = torch.randn(B, S, H, D, device="cuda").bfloat16()
        sc = 1 / math.sqrt(D)
        o, lse = F.attention(q, k, v, sc, True)
        t_f = time_fn(lambda: F.attention(q, k, v, sc, True), iters)
        t_b = time_fn(lambda: F.attention_bwd(q, k, v, o, do, lse, sc, True), iters)
        flops_f = 4.0 * B * H * S * S * D / 2
        qt, kt, vt = (x.transpose(1, 2) for x in (q, k, v))
        c_f = time_fn(lambda: torch.nn.functional.scaled_dot_product_attention(qt, kt, vt, is_causal=True), iters)
        qr, kr, vr = (x.detach().clone().requires_grad_(True) for x in (qt, kt, vt))
        ot = torch.nn.functional.scaled_dot_product_attention(qr, kr, vr, is_causal=True)
        dot = do.transpose(1, 2)
        c_b = time_fn(lambda: torch.autograd.grad(ot, (qr, kr, vr), dot, retain_graph=True), iters)
        emit({"op": "sdpa_causal_fwd", "shape": [B, H, S, D], "ms": t_f, "tflops": flops_f / t_f / 1e9,
              "frac_of_peak": flops_f / t_f / 1e9 / tf, "peak": src, "torch_sdpa_ms": c_f, "speedup_vs_torch": c_f / t_f})
        emit({"op": "sdpa_causal_bwd", "shape": [B, H, S, D], "ms": t_b, "tflops": 2.5 * flops_f / t_b / 1e9,
              "frac_of_peak": 2.5 * flops_f / t_b / 1e9 / tf, "peak": src, "torch_sdpa_ms": c_b,
              "speedup_vs_torch": c_b / t_b})
        del q, k, v, do, o, lse, qr, kr, vr, ot
        torch.cuda.empty_cache()


def bench_attn_bwd(iters):
    """The flash-attention backward call at the profiled shape (B 2, H 16, S 4096,
    D 128, causal): dsum kernel + tcgen05 backward + dQ convert."""
    hbm, tf, src = peaks()
    B, H, S, D = 2, 16, 4096, 128
    q, k, v, do = (torch.randn(B, S, H, D, device="cuda").bfloat16() for _ in range(4))
    sc = D ** -0.5
    o, lse = F.attention(q, k, v, sc, True, impl="tc")
    t = time_fn(lambda: F.attention_bwd(q, k, v, o, do, lse, sc, True, impl="tc"), max(iters, 20))
    fl = 2.5 * 4 * B * H * S * S * D / 2
    emit({"op": "attention_bwd_call", "shape": [B, S, H, D], "ms": t, "tflops": fl / t / 1e9,
          "frac_of_peak": fl / t / 1e9 / tf, "peak": src})


def bench_rms_bwd(iters):
    """RMSNorm backward at the GPT-24L training rows (micro-batch 8 x 2048, d 2048)."""
    hbm, tf, src = peaks()
    R, Dm = 8 * 2048, 2048
    x = torch.randn(R, Dm, device="cuda").bfloat16()
    w = torch.randn(Dm, device="cuda").bfloat16()
    dy = torch.randn_like(x)
    _, h, rstd = F.rmsnorm(x, w)
    dw = torch.zeros(Dm, device="cuda")
    t = time_fn(lambda: F.rmsnorm_bwd(dy, h, w, rstd, dw), iters)
    nb = 3 * R * Dm * 2
    emit({"op": "rms_norm_bwd", "shape": [R, Dm], "ms": t, "gbs": nb / t / 1e6, "frac_of_hbm": nb / t / 1e6 / hbm,
          "peak": src})
    # LayerNorm backward at the encoder width (BERT-large / ViT-L, d 1024)
    R2, D2 = 16384, 1024
    x2 = torch.randn(R2, D2, device="cuda").bfloat16()
    w2, b2 = torch.randn(D2, device="cuda").bfloat16(), torch.randn(D2, device="cuda").bfloat16()
    _, _, mean2, rstd2 = F.layernorm(x2, w2, b2)
    dy2 = torch.randn_like(x2)
    dw2, db2 = torch.zeros(D2, device="cuda"), torch.zeros(D2, device="cuda")
    t = time_fn(lambda: F.layernorm_bwd(dy2, x2, w2, mean2, rstd2, dw2, db2), iters)
    nb = 3 * R2 * D2 * 2
    emit({"op": "layer_norm_bwd", "shape": [R2, D2], "ms": t, "gbs": nb / t / 1e6, "frac_of_hbm": nb / t / 1e6 / hbm,
          "peak": src})


def bench_rows(iters):
    hbm, tf, src = peaks()
    R, Dm = 8 * 2048, 4096
    x = torch.randn(R, Dm, device="cuda").bfloat16()
    w = torch.randn(Dm, device="cuda").bfloat16()
    b = torch.randn(Dm, device="cuda").bfloat16()
    nbytes = 2 * R * Dm * 2
    t = time_fn(lambda: F.layernorm(x, w, b), iters)
    c = time_fn(lambda: torch.nn.functional.layer_norm(x, (Dm,), w, b), iters)
    emit({"op": "layer_norm_fwd", "shape": [R, Dm], "ms": t, "gbs": nbytes / t / 1e6, "frac_of_hbm": nbytes / t / 1e6 / hbm,
          "peak": src, "torch_ms": c, "speedup_vs_torch": c / t})
    y, h, mean, rstd = F.layernorm(x, w, b)
    dy = torch.randn_like(x)
    dw, db = torch.zeros(Dm, device="cuda"), torch.zeros(Dm, device="cuda")
    t = time_fn(lambda: F.layernorm_bwd(dy, x, w, mean, rstd, dw, db), iters)
    emit({"op": "layer_norm_bwd", "shape": [R, Dm], "ms": t, "gbs": 3 * R * Dm * 2 / t / 1e6,
          "frac_of_hbm": 3 * R * Dm * 2 / t / 1e6 / hbm, "peak": src})
    t = time_fn(lambda: F.rmsnorm(x, w), iters)
    emit({"op": "rms_norm_fwd", "shape": [R, Dm], "ms": t, "gbs": nbytes / t / 1e6, "frac_of_hbm": nbytes / t / 1e6 / hbm, "peak": src})
    t = time_fn(lambda: F.softmax(x), iters)
    c = time_fn(lambda: torch.softmax(x, -1), iters)
    emit({"op": "softmax_fwd", "shape": [R, Dm], "ms": t, "gbs": nbytes / t / 1e6, "frac_of_hbm": nbytes / t / 1e6 / hbm,
          "peak": src, "torch_ms": c, "speedup_vs_torch": c / t})
    sy = F.softmax(x)
    t = time_fn(lambda: F.softmax_bwd(sy, dy), iters)
    emit({"op": "softmax_bwd", "shape": [R, Dm], "ms": t, "gbs": 3 * R * Dm * 2 / t / 1e6,
          "frac_of_hbm": 3 * R * Dm * 2 / t / 1e6 / hbm, "peak": src})


def bench_ce(iters):
    hbm, tf, src = peaks()
    T, V = 8 * 2048, 152064
    logits = torch.randn(T, V, device="cuda").bfloat16()
    tgt = torch.randint(0, V, (T,), device="cuda")
    buf = logits.clone()
    # fused loss + gradient: reads the row twice (second pass mostly from L2) and writes the gradient
    t = time_fn(lambda: F.cross_entropy_fused(buf, tgt, grad_scale=1.0 / T), iters)
    nbytes = 2 * T * V * 2
    t_loss = time_fn(lambda: F.cross_entropy_fused(logits, tgt, write_grad=False), iters)
    lr = logits.detach().requires_grad_(True)

    def torch_ce():
        loss = torch.nn.functional.cross_entropy(lr.float(), tgt)
        torch.autograd.grad(loss, lr)

    c = time_fn(torch_ce, max(3, iters // 2))
    emit({"op": "cross_entropy_fwd_bwd", "shape": [T, V], "ms": t, "gbs": nbytes / t / 1e6,
          "frac_of_hbm": nbytes / t / 1e6 / hbm, "peak": src, "torch_ms": c, "speedup_vs_torch": c / t})
    emit({"op": "cross_entropy_fwd", "shape": [T, V], "ms": t_loss, "gbs": T * V * 2 / t_loss / 1e6,
          "frac_of_hbm": T * V * 2 / t_loss / 1e6 / hbm, "peak": src})


def bench_adamw(iters):
    hbm, tf, src = peaks()
    n = 1_000_000_000
    p = torch.randn(n, device="cuda")
    g = torch.randn(n, device="cuda")
    m = torch.zeros(n, device="cuda")
    v = torch.zeros(n, device="cuda")
    pb = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    step = [0]

    def run():
        step[0] += 1
        F.adamw_(p, g, m, v, pb, lr=1e-4, wd=0.1, step=step[0])

    t = time_fn(run, max(3, iters // 2))
    nbytes = n * (16 + 12 + 2)  # read p,g,m,v; write p,m,v; write the bf16 copy
    emit({"op": "adamw_1e9", "shape": [n], "ms": t, "gbs": nbytes / t / 1e6, "frac_of_hbm": nbytes / t / 1e6 / hbm,
          "peak": src})
    del pb
    torch.cuda.empty_cache()
    opt = torch.optim.AdamW([p], lr=1e-4, weight_decay=0.1, fused=True)
    p.grad = g

    c = time_fn(opt.step, max(3, iters // 2))
    emit({"op": "adamw_1e9_torch_fused", "shape": [n], "ms": c, "note": "torch fused AdamW (no bf16 copy)"})


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default="gemm,sdpa,attn_bwd,rows,rms_bwd,ce,adamw")
    ap.add_argument("--iters", type=int, default=10)
    args = ap.parse_args()
    _ext.C()
    sel = set(args.only.split(","))
    for name, fn in (("gemm", bench_gemm), ("gemm_pair", bench_gemm_pair), ("sdpa", bench_sdpa), ("attn_bwd", bench_attn_bwd), ("rows", bench_rows),
                     ("rms_bwd", bench_rms_bwd), ("ce", bench_ce), ("adamw", bench_adamw)):
        if name in sel:
            fn(args.iters)
            torch.cuda.empty_cache()
    assert _ext.check_status() == 0


if __name__ == "__main__":
    main()
