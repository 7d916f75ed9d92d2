"""Small, self-terminating cases of the hot kernels for Nsight Compute.

Each case builds inputs larger than the 126 MB L2 (so DRAM counters mean
something) but only a few hundred MB in total, runs the kernel a few times and
exits. Meant to be run under ``ncu -k regex:<kernel> -c 1`` after it has run
once on its own:

    python -m aether_b200.profile_cases gemm        # tcgen05 GEMM 8192x8192x4096
    python -m aether_b200.profile_cases attn_fwd    # tcgen05 flash attention fwd, B2 H16 S4096 D128 causal
    python -m aether_b200.profile_cases attn_bwd    # tcgen05 flash attention bwd, same shape
    python -m aether_b200.profile_cases skinny      # decode GEMM 1 x 3584 -> 37888 (Qwen-7B gate/up)
    python -m aether_b200.profile_cases decode_attn # split-K decode attention B8 Hq28 Hkv4 S8192
    python -m aether_b200.profile_cases decode_attn_b1  # the same at batch 1, 2048 keys, 32 splits
    python -m aether_b200.profile_cases adamw       # fused AdamW over 64M fp32 params
    python -m aether_b200.profile_cases decode7b    # eager Qwen2.5-7B-shape decode steps (batch 1, 2048 cached)
                                                    # inside NVTX range "decode": for the launch list only
                                                    # (ncu --nvtx --nvtx-include "decode/" --metrics gpu__time_duration.sum)
    python -m aether_b200.profile_cases decode7b_tp8 # the same for one TP=8 rank's shards, emulated on one GPU
    python -m aether_b200.profile_cases rows 1      # one launch of each row / elementwise / loss / MoE / MLA / quant kernel
    python -m aether_b200.profile_cases gemm_tp     # fused TP-training GEMMs, two ranks emulated on one GPU
"""
from __future__ import annotations

import sys

import torch

from .ops import functional as F


def gemm(reps):
    a = torch.randn(8192, 4096, device="cuda").bfloat16()
    b = torch.randn(8192, 4096, device="cuda").bfloat16()
    for _ in range(reps):
        F.gemm(a, b)


def _qkv():
    B, S, H, D = 2, 4096, 16, 128
    q = torch.randn(B, S, H, D, device="cuda").bfloat16()
    return q, torch.randn_like(q), torch.randn_like(q), D ** -0.5


def attn_fwd(reps):
    q, k, v, s = _qkv()
    for _ in range(reps):
        F.attention(q, k, v, s, True, impl="tc")


def attn_bwd(reps):
    q, k, v, s = _qkv()
    o, lse = F.attention(q, k, v, s, True, impl="tc")
    do = torch.randn_like(q)
    for _ in range(reps):
        F.attention_bwd(q, k, v, o, do, lse, s, True, impl="tc")


def skinny(reps):
    x = torch.randn(1, 3584, device="cuda").bfloat16()
    w = torch.randn(37888, 3584, device="cuda").bfloat16()
    acc = torch.zeros(1, 37888, device="cuda")
    for _ in range(reps):
        F.skinny_gemm(x, w, acc)
        acc.zero_()


def decode_attn(reps):
    B, Hq, Hkv, D, S = 8, 28, 4, 128, 8192
    kc = torch.randn(B, S, Hkv, D, device="cuda").bfloat16()
    vc = torch.randn_like(kc)
    q = torch.randn(B, Hq * D, device="cuda").bfloat16()
    slot = torch.arange(B, dtype=torch.int32, device="cuda")
    seqlen = torch.full((B,), S, dtype=torch.int32, device="cuda")
    out = torch.empty(B, Hq * D, dtype=torch.bfloat16, device="cuda")
    counters = torch.zeros(B * Hkv, dtype=torch.int32, device="cuda")
    for _ in range(reps):
        F.decode_attention(q, kc, vc, slot, seqlen, out, Hq, D ** -0.5, splits=8, counters=counters)


def decode_attn_b1(reps):
    """The decode attention of one Qwen2.5-7B-shape layer at batch 1 with 2048
    cached keys and the serving path's 32 splits."""
    Hq, Hkv, D, S = 28, 4, 128, 2048
    kc = torch.randn(2, 4096, Hkv, D, device="cuda").bfloat16()
    vc = torch.randn_like(kc)
    q = torch.randn(1, (Hq + 2 * Hkv) * D, device="cuda").bfloat16()
    slot = torch.zeros(1, dtype=torch.int32, device="cuda")
    seqlen = torch.full((1,), S, dtype=torch.int32, device="cuda")
    out = torch.empty(1, Hq * D, dtype=torch.bfloat16, device="cuda")
    counters = torch.zeros(Hkv, dtype=torch.int32, device="cuda")
    for _ in range(reps):
        F.decode_attention(q, kc, vc, slot, seqlen, out, Hq, D ** -0.5, splits=32, counters=counters)


def adamw(reps):
    n = 64 * 1024 * 1024
    p, g = torch.randn(n, device="cuda"), torch.randn(n, device="cuda")
    m, v = torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
    pb = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    for i in range(reps):
        F.adamw_(p, g, m, v, pb, lr=1e-4, beta1=0.9, beta2=0.95, eps=1e-8, wd=0.1, step=i + 1)


def decode7b(reps, tp=None):
    from .models.qwen import QwenConfig, QwenModel

    cfg = QwenConfig.qwen25_7b()
    m = QwenModel(cfg, device="cuda", seed=1, max_batch=1, max_seq=4096, tp=tp)
    prompt = torch.randint(0, cfg.vocab, (1, 2048), device="cuda")
    tok = m.prefill(prompt)
    pos = torch.full((1,), 2048, dtype=torch.int32, device="cuda")
    slots = torch.zeros(1, dtype=torch.int32, device="cuda")
    m.decode_step(tok, pos, slots, use_graph=False)
    torch.cuda.synchronize()
    for _ in range(reps):
        torch.cuda.nvtx.range_push("decode")
        tok = m.decode_step(tok, pos, slots, use_graph=False)
        torch.cuda.nvtx.range_pop()


def rows(reps):
    """One launch each of the row / elementwise / loss / MoE / MLA / quant
    kernels at training or serving sizes (inputs > L2 where the op streams):
    rmsnorm fwd + bwd and layernorm fwd + bwd [16384, 2048], softmax
    [16384, 4096], swiglu fwd + bwd [16384, 11264], RoPE on a [16384, 6144]
    qkv, embedding fwd + bwd (vocab 32000), fused cross-entropy [4096, 152064],
    the grouped MoE GEMM (8 experts, 8192 token rows x 1408 -> 2048), absorbed
    MLA decode attention (16 heads, 4 sequences x 4096 latent rows), Q8_0
    quantise + dequantise of 64M values."""
    from .ops import reference as ref

    T, d = 16384, 2048
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(T, d, device="cuda", generator=g).bfloat16()
    w = torch.ones(d, device="cuda", dtype=torch.bfloat16)
    dw = torch.zeros(d, device="cuda")
    for _ in range(reps):
        y, h, rstd = F.rmsnorm(x, w)
        F.rmsnorm_bwd(y, h, w, rstd, dw)
    out = F.layernorm(x, w, w)
    F.layernorm_bwd(out[0], x, w, out[-2], out[-1], dw, dw.clone())
    F.softmax(torch.randn(T, 4096, device="cuda", generator=g).bfloat16())
    hgu = torch.randn(T, 2 * 5632, device="cuda", generator=g).bfloat16()
    act = F.swiglu(hgu)
    F.swiglu_bwd(hgu, act)
    qkv = torch.randn(T, 3 * d, device="cuda", generator=g).bfloat16()
    cos, sin = ref.rope_tables(2048, 128, 10000.0, device="cuda")
    pos = torch.arange(2048, device="cuda", dtype=torch.int32).repeat(T // 2048)
    F.rope_(qkv, pos, cos.contiguous(), sin.contiguous(), 32, 128)
    table = torch.randn(32000, d, device="cuda", generator=g).bfloat16()
    ids = torch.randint(0, 32000, (T,), device="cuda", generator=g)
    e = F.embedding(table, ids)
    F.embedding_bwd(e, ids, torch.zeros(32000, d, device="cuda"))
    logits = torch.randn(4096, 152064, device="cuda", generator=g).bfloat16()
    F.cross_entropy_fused(logits, torch.randint(0, 152064, (4096,), device="cuda", generator=g), grad_scale=1 / 4096)
    del logits
    E, Tm, K, N = 8, 8192, 2048, 1408
    idx = torch.randint(0, E, (Tm, 1), device="cuda", generator=g, dtype=torch.int32)
    row_of, src_row, tile_group = F.moe_permute(idx, E)
    X = F.moe_gather(torch.randn(Tm, K, device="cuda", generator=g).bfloat16(), src_row)
    F.gemm_grouped(X, torch.randn(E, N, K, device="cuda", generator=g).bfloat16() * 0.02, tile_group)
    cache = torch.randn(4, 4096, 576, device="cuda", generator=g).bfloat16()
    q_abs = torch.randn(4, 16, 576, device="cuda", generator=g).bfloat16()
    F.mla_attention(q_abs, cache, torch.arange(4, device="cuda", dtype=torch.int32),
                    torch.full((4,), 4096, device="cuda", dtype=torch.int32),
                    torch.empty(4, 16, 512, device="cuda", dtype=torch.bfloat16), 576 ** -0.5, splits=8)
    big = torch.randn(1 << 26, device="cuda", generator=g).bfloat16()
    q = F.quantize_blocks(big)
    F.dequantize_blocks(q, big.shape)


def decode7b_tp8(reps):
    """decode7b for one TP=8 rank's shards, emulated on one GPU (no exchanges)."""
    from .bench_serve import EmulatedTP

    decode7b(reps, tp=EmulatedTP(0, 8))


def gemm_tp(reps):
    """The fused TP-training GEMM with two TP ranks emulated on one GPU (one
    cooperative launch, 74 SMs per rank): all-gather -> qkv GEMM (8192 x 3072 x
    2048) and o_proj GEMM -> reduce-scatter (8192 x 2048 x 1024), against the
    plain tcgen05 GEMM doing the same math on the whole GPU. Prints CUDA-event
    times (the emulated ranks share the GPU, so the fused launch does both
    ranks' work)."""
    tp, Ml, d, nq, nin = 2, 4096, 2048, 3072, 1024
    M = tp * Ml
    bf = dict(dtype=torch.bfloat16, device="cuda")
    h = [torch.randn(Ml, d, **bf) for _ in range(tp)]
    wq = [torch.randn(nq, d, **bf) * 0.02 for _ in range(tp)]
    o = [torch.randn(M, nin, **bf) for _ in range(tp)]
    wo = [torch.randn(d, nin, **bf) * 0.02 for _ in range(tp)]
    ag = [[torch.zeros(M, d, **bf) for _ in range(tp)] for _ in range(2)]
    agf = [[torch.zeros(tp * (Ml // 128), dtype=torch.int32, device="cuda") for _ in range(tp)] for _ in range(2)]
    rs = [[torch.zeros(tp * Ml * d, **bf) for _ in range(tp)] for _ in range(2)]
    rsf = [[torch.zeros((Ml // 128) * (d // 256) * 4, dtype=torch.int32, device="cuda") for _ in range(tp)]
           for _ in range(2)]
    y = [torch.empty(M, nq, **bf) for _ in range(tp)]
    x = [torch.empty(Ml, d, **bf) for _ in range(tp)]
    ptr = lambda ts: [t.data_ptr() for t in ts]
    n = [0]

    def fused():
        k, e = n[0] & 1, (n[0] >> 1) + 1
        n[0] += 1
        F.gemm_tp(h, ag[k], wq, y, [], h, list(range(tp)), tp, Ml, False, 1, False, False, ptr(ag[k]), ptr(agf[k]),
                    0, [], [], e, 0, 5.0)
        F.gemm_tp(o, [], wo, x, [], [], list(range(tp)), tp, Ml, False, 0, True, False, [], [], 0, ptr(rs[k]),
                    ptr(rsf[k]), 0, e, 5.0)

    hf = torch.cat(h)

    def plain():
        for r in range(tp):
            F.gemm(hf, wq[r])
            F.gemm(o[r], wo[r])

    for fn, tag in ((fused, "fused (2 emulated ranks)"), (plain, "plain gemm_bf16 x2")):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        flops = 2 * tp * (M * nq * d + M * d * nin)
        ms = e0.elapsed_time(e1) / reps
        print(f"gemm_tp {tag}: {ms * 1e3:.1f} us per AG-GEMM + GEMM-RS pair, {flops / ms / 1e9:.0f} TFLOP/s")


CASES = {f.__name__: f for f in (gemm, attn_fwd, attn_bwd, skinny, decode_attn, decode_attn_b1, adamw, decode7b,
                                 decode7b_tp8, rows, gemm_tp)}


def main():
    name = sys.argv[1] if len(sys.argv) > 1 else ""
    if name not in CASES:
        raise SystemExit(f"usage: python -m aether_b200.profile_cases {{{','.join(CASES)}}} [reps]")
    reps = int(sys.argv[2]) if len(sys.argv) > 2 else 3
    CASES[name](reps)
    torch.cuda.synchronize()
    print(f"{name}: ok")


if __name__ == "__main__":
    main()
