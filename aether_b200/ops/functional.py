"""Functional ops. CUDA tensors run the sm_100a kernels of ``aether_b200._C``;
CPU tensors run the fp32 statements in ``reference`` (and return the same
dtypes). Outputs are allocated here unless an ``out`` tensor is passed.
"""
from __future__ import annotations

import os

import torch

from .._ext import C
from . import reference as ref

BF16 = torch.bfloat16


def _cuda(t: torch.Tensor) -> bool:
    return t.is_cuda


# ------------------------------------------------------------------ GEMM
def gemm(a, b, *, a_mn=False, b_mn=False, out=None, out_dtype=BF16, bias=None, residual=None, alpha=1.0,
         accumulate=False, alpha_t=None):
    """out (+)= alpha * opA(a) @ opB(b)^T (+ bias) (+ residual).

    a: [M, K] (a_mn=False) or [K, M] (a_mn=True); b: [N, K] (b_mn=False) or [K, N] (b_mn=True).
    alpha_t: optional fp32 device scalar multiplied into alpha without a host sync.
    """
    M = a.shape[1] if a_mn else a.shape[0]
    N = b.shape[1] if b_mn else b.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=out_dtype, device=a.device)
    if _cuda(a):
        C().gemm_bf16(a, b, out, a_mn, b_mn, bias, residual, float(alpha), bool(accumulate), alpha_t)
        return out
    if alpha_t is not None:
        alpha = alpha * float(alpha_t.reshape(-1)[0])
    r = ref.gemm(a, b, a_mn, b_mn, bias, residual, alpha)
    if accumulate:
        out.add_(r.to(out.dtype))
    else:
        out.copy_(r.to(out.dtype))
    return out


def gemm_tp(*args):
    """The tensor-parallel training GEMM with its collective inside
    (csrc/gemm_tp.cu; arguments as the extension's gemm_tp). A refused
    argument set comes back as a message and is raised here."""
    msg = C().gemm_tp(*args)
    if msg:
        raise RuntimeError(msg)


def gemm_param_gather(*args):
    """The GEMM whose weight unit (ZeRO-3) is all-gathered inside the same
    kernel (csrc/gemm_tp.cu); raises a refused argument set."""
    msg = C().gemm_param_gather(*args)
    if msg:
        raise RuntimeError(msg)


def linear(x, w, bias=None, residual=None, out=None):
    """y = x @ w^T (+ bias) (+ residual); x [..., K], w [N, K]."""
    shp = x.shape
    x2 = x.reshape(-1, shp[-1])
    r2 = residual.reshape(-1, w.shape[0]) if residual is not None else None
    y = gemm(x2, w, bias=bias, residual=r2, out=out)
    return y.view(*shp[:-1], w.shape[0])


# ------------------------------------------------------------------ norms
def rmsnorm(x, w, eps=1e-6, res=None, want_h=False):
    """Returns (y, h, rstd): h = x + res (the residual stream) or x."""
    if _cuda(x):
        y = torch.empty_like(x)
        rstd = torch.empty(x.numel() // x.shape[-1], dtype=torch.float32, device=x.device)
        h = torch.empty_like(x) if res is not None else x
        C().rmsnorm_fwd(x, res, w, y, h if res is not None else None, rstd, float(eps))
        return y, h, rstd
    y, h, rstd = ref.rmsnorm(x, w, eps, res)
    return y.to(x.dtype), h.to(x.dtype), rstd


def rmsnorm_bwd(dy, h, w, rstd, dw_f32, dres=None, accumulate=True):
    if _cuda(dy):
        dx = torch.empty_like(dy)
        C().rmsnorm_bwd(dy, h, w, rstd, dres, dx, dw_f32, bool(accumulate))
        return dx
    hf = h.float()
    xhat = hf * rstd.view(*rstd.shape, 1)
    g = dy.float() * w.float()
    d = h.shape[-1]
    dx = rstd.view(*rstd.shape, 1) * (g - xhat * (g * xhat).sum(-1, keepdim=True) / d)
    if dres is not None:
        dx = dx + dres.float()
    dwp = (dy.float() * xhat).reshape(-1, d).sum(0)
    if accumulate:
        dw_f32.add_(dwp.detach())
    else:
        dw_f32.copy_(dwp.detach())
    return dx.detach().to(dy.dtype)


def layernorm(x, w, b=None, eps=1e-5, res=None):
    if _cuda(x):
        y = torch.empty_like(x)
        rows = x.numel() // x.shape[-1]
        mean = torch.empty(rows, dtype=torch.float32, device=x.device)
        rstd = torch.empty_like(mean)
        h = torch.empty_like(x) if res is not None else x
        C().layernorm_fwd(x, res, w, b, y, h if res is not None else None, mean, rstd, float(eps))
        return y, h, mean, rstd
    y, h = ref.layernorm(x, w, b, eps, res)
    hf = h.float()
    mean = hf.mean(-1).reshape(-1)
    rstd = torch.rsqrt(hf.var(-1, unbiased=False) + eps).reshape(-1)
    return y.to(x.dtype), h.to(x.dtype), mean, rstd


def layernorm_bwd(dy, h, w, mean, rstd, dw_f32, db_f32, dres=None, accumulate=True):
    if _cuda(dy):
        dx = torch.empty_like(dy)
        C().layernorm_bwd(dy, h, w, mean, rstd, dres, dx, dw_f32, db_f32, bool(accumulate))
        return dx
    d = h.shape[-1]
    hf = h.float().reshape(-1, d)
    g = dy.float().reshape(-1, d)
    xh = (hf - mean[:, None]) * rstd[:, None]
    gw = g * w.float()
    dx = rstd[:, None] * (gw - gw.mean(-1, keepdim=True) - xh * (gw * xh).mean(-1, keepdim=True))
    if dres is not None:
        dx = dx + dres.float().reshape(-1, d)
    if accumulate:
        dw_f32.add_((g * xh).sum(0))
        db_f32.add_(g.sum(0))
    else:
        dw_f32.copy_((g * xh).sum(0))
        db_f32.copy_(g.sum(0))
    return dx.view_as(dy).to(dy.dtype)


def softmax(x, scale=1.0):
    if _cuda(x):
        y = torch.empty_like(x)
        C().softmax_fwd(x, y, float(scale))
        return y
    return ref.softmax(x, scale).to(x.dtype)


def softmax_bwd(y, dy, scale=1.0):
    if _cuda(y):
        dx = torch.empty_like(dy)
        C().softmax_bwd(y, dy, dx, float(scale))
        return dx
    yf, g = y.float(), dy.float()
    return (scale * yf * (g - (yf * g).sum(-1, keepdim=True))).to(dy.dtype)


# ------------------------------------------------------------------ activations
def swiglu(h):
    F_ = h.shape[-1] // 2
    if _cuda(h):
        act = torch.empty(*h.shape[:-1], F_, dtype=h.dtype, device=h.device)
        C().swiglu_fwd(h, act)
        return act
    return ref.swiglu(h).to(h.dtype)


def swiglu_bwd(h, dact):
    if _cuda(h):
        dh = torch.empty(*dact.shape[:-1], 2 * dact.shape[-1], dtype=h.dtype, device=h.device)
        C().swiglu_bwd(h, dact, dh)
        return dh
    g, u = h.float().chunk(2, dim=-1)
    s = torch.sigmoid(g)
    da = dact.float()
    dg = da * u * s * (1 + g * (1 - s))
    du = da * g * s
    return torch.cat([dg, du], dim=-1).to(h.dtype)


def gelu(x):
    if _cuda(x):
        y = torch.empty_like(x)
        C().gelu_fwd(x, y)
        return y
    return ref.gelu_tanh(x).to(x.dtype)


def gelu_bwd(x, dy):
    if _cuda(x):
        dx = torch.empty_like(x)
        C().gelu_bwd(x, dy, dx)
        return dx
    with torch.enable_grad():
        xf = x.detach().float().requires_grad_(True)
        y = ref.gelu_tanh(xf)
        (g,) = torch.autograd.grad(y, xf, dy.float())
    return g.to(x.dtype)


# ------------------------------------------------------------------ RoPE
def rope_(x2d, pos, cos_t, sin_t, n_heads, head_dim, inverse=False):
    """In-place half-split RoPE on heads [0, n_heads) of each row of x2d [T, row]."""
    if _cuda(x2d):
        C().rope_apply(x2d, pos, cos_t, sin_t, int(n_heads), int(head_dim), bool(inverse))
        return x2d
    y = ref.rope(x2d, pos, cos_t, sin_t, n_heads, head_dim, inverse)
    x2d.copy_(y.to(x2d.dtype))
    return x2d


# ------------------------------------------------------------------ embedding
def embedding(table, ids):
    if _cuda(table):
        out = torch.empty(*ids.shape, table.shape[1], dtype=table.dtype, device=table.device)
        C().embedding_fwd(table, ids.long(), out.view(-1, table.shape[1]))
        return out
    return table[ids.long().clamp(0, table.shape[0] - 1)]


def embedding_bwd(dy, ids, dtable_f32):
    if _cuda(dy):
        C().embedding_bwd(dy.reshape(-1, dy.shape[-1]).contiguous(), ids.long().reshape(-1), dtable_f32)
        return
    dtable_f32.index_add_(0, ids.long().reshape(-1), dy.reshape(-1, dy.shape[-1]).float())


# ------------------------------------------------------------------ loss
def cross_entropy_fused(logits, targets, *, grad_scale=None, scale_tensor=None, ignore_index=-100,
                        write_grad=True, grad_out=None):
    """Loss per row [T] fp32; when write_grad, the logits buffer is overwritten
    in place with (softmax - onehot) * grad_scale (or written to grad_out)."""
    T = logits.shape[0]
    if _cuda(logits):
        loss = torch.empty(T, dtype=torch.float32, device=logits.device)
        lse = torch.empty(T, dtype=torch.float32, device=logits.device)
        d = None
        if write_grad:
            d = logits if grad_out is None else grad_out
        C().cross_entropy_fused(logits, targets.long().contiguous(), loss, lse, d, scale_tensor,
                                float(grad_scale if grad_scale is not None else 1.0), int(ignore_index))
        return loss, lse
    loss, lse = ref.cross_entropy(logits, targets.long(), ignore_index)
    if write_grad:
        s = float(grad_scale if grad_scale is not None else 1.0)
        if scale_tensor is not None:
            s = s * float(scale_tensor.reshape(-1)[0])
        g = ref.cross_entropy_grad(logits, targets.long(), s, ignore_index)
        (logits if grad_out is None else grad_out).copy_(g.to(logits.dtype))
    return loss, lse


def argmax(x):
    if _cuda(x):
        out = torch.empty(x.shape[0], dtype=torch.long, device=x.device)
        C().argmax_rows(x, out)
        return out
    return x.float().argmax(-1)


# ------------------------------------------------------------------ attention
_FA2_ONLY = os.environ.get("AETHER_FA2", "0") == "1"


def _tc_ok(q, k, v):
    """The tcgen05 forward handles head_dim 128 with [B, S, H, D] views whose
    batch stride is S * row stride (e.g. slices of one packed qkv buffer)."""
    if _FA2_ONLY or q.shape[-1] != 128:
        return False
    for t in (q, k, v):
        if t.stride(0) != t.shape[1] * t.stride(1) or t.stride(3) != 1 or t.stride(2) != 128:
            return False
    return True


def attention(q, k, v, scale, causal=True, causal_offset=0, out=None, want_lse=True, impl="auto", window=0,
              softcap=0.0):
    """q [B,Sq,Hq,D], k/v [B,Sk,Hkv,D] (strided views ok) -> (o [B,Sq,Hq,D], lse [B,Hq,Sq]).

    impl: "auto" (tcgen05 kernel when it applies, else the mma.sync kernel),
    "tc" or "fa2". Flex attention: ``window`` > 0 (sliding window: query i
    sees keys (i + offset - window, i + offset]) and ``softcap`` > 0 (logits
    soft-capped by softcap * tanh(s / softcap)); ``attention_bwd`` takes the same."""
    B, Sq, Hq, D = q.shape
    if _cuda(q):
        o = out if out is not None else torch.empty(B, Sq, Hq, D, dtype=q.dtype, device=q.device)
        lse = torch.empty(B, Hq, Sq, dtype=torch.float32, device=q.device) if want_lse else None
        if impl == "tc" or (impl == "auto" and _tc_ok(q, k, v)):
            C().attention_fwd_tc(q, k, v, o, lse, float(scale), bool(causal), int(causal_offset), int(window),
                                 float(softcap))
        else:
            C().attention_fwd(q, k, v, o, lse, float(scale), bool(causal), int(causal_offset), int(window),
                              float(softcap))
        return o, lse
    o, lse = ref.attention(q, k, v, scale, causal, causal_offset, window, softcap)
    o = o.to(q.dtype).contiguous()
    if out is not None:
        out.copy_(o)
        o = out
    return o, lse


def attention_bwd(q, k, v, o, do, lse, scale, causal=True, causal_offset=0, dq=None, dk=None, dv=None,
                  impl="auto", window=0, softcap=0.0):
    """Gradients of ``attention`` (same window / softcap; those forms run on
    the mma.sync kernel)."""
    if _cuda(q):
        dq = dq if dq is not None else torch.empty_like(q)
        dk = dk if dk is not None else torch.empty(k.shape, dtype=k.dtype, device=k.device)
        dv = dv if dv is not None else torch.empty(v.shape, dtype=v.dtype, device=v.device)
        use_tc = impl == "tc" or (impl == "auto" and _tc_ok(q, k, v) and _tc_ok(do, dk, dv))
        C().attention_bwd(q, k, v, o, do, lse, dq, dk, dv, float(scale), bool(causal), int(causal_offset), use_tc,
                          int(window), float(softcap))
        return dq, dk, dv
    with torch.enable_grad():
        qf = q.detach().float().requires_grad_(True)
        kf = k.detach().float().requires_grad_(True)
        vf = v.detach().float().requires_grad_(True)
        of, _ = ref.attention(qf, kf, vf, scale, causal, causal_offset, window, softcap)
        gq, gk, gv = torch.autograd.grad(of, (qf, kf, vf), do.float())
    res = []
    for g, buf, like in ((gq, dq, q), (gk, dk, k), (gv, dv, v)):
        if buf is not None:
            buf.copy_(g.to(buf.dtype))
            res.append(buf)
        else:
            res.append(g.to(like.dtype))
    return tuple(res)


# ------------------------------------------------------------------ optimiser
def adamw_(p, g, m, v, p_bf16=None, *, lr, beta1=0.9, beta2=0.95, eps=1e-8, wd=0.0, step=1, gscale=1.0,
           gscale_tensor=None):
    if _cuda(p):
        C().adamw_step(p, g, m, v, p_bf16, float(lr), float(beta1), float(beta2), float(eps), float(wd), int(step),
                       float(gscale), gscale_tensor)
        return p
    s = gscale * (float(gscale_tensor.reshape(-1)[0]) if gscale_tensor is not None else 1.0)
    ref.adamw(p, g, m, v, lr, beta1, beta2, eps, wd, step, s)
    if p_bf16 is not None:
        p_bf16.copy_(p.to(p_bf16.dtype))
    return p


def grad_norm(g, pre_scale=1.0, max_norm=0.0):
    """Returns (norm[1], clip_coef[1]) as device tensors (no host sync)."""
    norm = torch.empty(1, dtype=torch.float32, device=g.device)
    clip = torch.empty(1, dtype=torch.float32, device=g.device)
    if _cuda(g):
        C().grad_norm(g, norm, clip, float(pre_scale), float(max_norm))
        return norm, clip
    n = g.float().norm() * pre_scale
    norm.fill_(float(n))
    clip.fill_(min(1.0, max_norm / (float(n) + 1e-6)) if max_norm > 0 else 1.0)
    return norm, clip


# ------------------------------------------------------------------ decode path
def skinny_gemm(x, w, acc, splits=0, acc_mc=0, signal=None):
    """acc[M, N] += x[M, K] @ w[N, K]^T in fp32 (acc starts zeroed), M <= 64.
    acc_mc: NVLS multicast address of a symmetric acc (reduce into all ranks).
    signal: (peer slot pointers, epoch, done counter, rank, world) -- the
    kernel's last CTA announces to every rank that its reductions landed."""
    if _cuda(x):
        if signal is None:
            C().skinny_gemm(x, w, acc, int(splits), int(acc_mc))
        else:
            peers, epoch, done, rank, world = signal
            C().skinny_gemm(x, w, acc, int(splits), int(acc_mc), peers, epoch, done, int(rank), int(world))
        return acc
    acc[:, : w.shape[0]] += x.float() @ w.float().t()
    return acc


def skinny_finalize(acc, y, bias=None, res=None, swiglu=False, wait=None):
    """y = bf16(acc + bias + res) or swiglu(acc halves); zeroes acc.
    wait: (signal slots, epoch, rank, world, timeout_s) -- first wait until
    every rank has announced its reductions into acc (see skinny_gemm)."""
    if _cuda(acc):
        if wait is None:
            C().skinny_finalize(acc, y, bias, res, bool(swiglu))
        else:
            C().skinny_finalize(acc, y, bias, res, bool(swiglu), *wait)
        return y
    M, N = y.shape
    if swiglu:
        a = acc[:M, : 2 * N].clone()
        if bias is not None:
            a = a + bias.float()
        g, u = a[:, :N], a[:, N:]
        y.copy_((torch.nn.functional.silu(g) * u).to(y.dtype))
        acc[:M, : 2 * N] = 0
    else:
        a = acc[:M, :N].clone()
        if bias is not None:
            a = a + bias.float()
        if res is not None:
            a = a + res.float()
        y.copy_(a.to(y.dtype))
        acc[:M, :N] = 0
    return y


def _kv_index(slot, pos, k_cache, page_table):
    """(dim-0 index, dim-1 index) of (sequence row, position) in a cache: the
    slot and position, or with a page table the physical page and its row."""
    if page_table is None:
        return slot.long(), pos.long()
    P = k_cache.shape[1]
    pos = pos.long()
    return page_table[slot.long(), pos // P].long(), pos % P


def rope_kv_append(qkv, pos, slot, cos_t, sin_t, k_cache, v_cache, Hq, Hkv, D, page_table=None):
    """Rotates q/k of qkv [T, row] in place and writes k, v into the caches
    [slots, max_seq, Hkv, D] at (slot[t], pos[t]) -- or, with ``page_table``
    [rows, max_pages] int32, into page pools [pages, page_size, Hkv, D]."""
    if _cuda(qkv):
        C().rope_kv_append(qkv, pos, slot, cos_t, sin_t, k_cache, v_cache, int(Hq), int(Hkv), int(D), page_table)
        return qkv
    rope_(qkv, pos, cos_t, sin_t, Hq + Hkv, D)
    T = qkv.shape[0]
    k = qkv[:, Hq * D : (Hq + Hkv) * D].view(T, Hkv, D)
    v = qkv[:, (Hq + Hkv) * D : (Hq + 2 * Hkv) * D].view(T, Hkv, D)
    i0, i1 = _kv_index(slot, pos, k_cache, page_table)
    k_cache[i0, i1] = k
    v_cache[i0, i1] = v
    return qkv


def gather_kv(cache, slot: int, L: int, page_table=None):
    """Keys (or values) [L, Hkv, D] of one sequence row as a contiguous tensor."""
    if page_table is None:
        return cache[slot, :L]
    P = cache.shape[1]
    pages = page_table[slot, : (L + P - 1) // P].long()
    return cache[pages].reshape(-1, cache.shape[2], cache.shape[3])[:L]


def decode_attention(q, k_cache, v_cache, slot, seqlen, out, Hq, scale, splits=8, part_o=None, part_lse=None,
                     counters=None, page_table=None, window=0, softcap=0.0):
    """q [B, >=Hq*D] (one new token per sequence), caches [slots, max_seq, Hkv, D]
    (or page pools with ``page_table``), seqlen [B] = valid keys. Writes out [B, Hq*D].
    window > 0: only the last ``window`` keys; softcap > 0: soft-capped logits."""
    B = q.shape[0]
    D = k_cache.shape[3]
    if _cuda(q):
        if part_o is None:
            part_o = torch.empty(B * Hq * splits * D, dtype=torch.float32, device=q.device)
            part_lse = torch.empty(B * Hq * splits, dtype=torch.float32, device=q.device)
        C().decode_attention(q, k_cache, v_cache, slot, seqlen, out, part_o, part_lse, int(Hq), int(splits),
                             float(scale), counters, page_table, int(window), float(softcap))
        return out
    Hkv = k_cache.shape[2]
    for b in range(B):
        L = int(seqlen[b])
        s = int(slot[b])
        qb = q[b, : Hq * D].view(1, 1, Hq, D)
        kb = gather_kv(k_cache, s, L, page_table).unsqueeze(0)
        vb = gather_kv(v_cache, s, L, page_table).unsqueeze(0)
        o, _ = ref.attention(qb, kb, vb, scale, True, L - 1, window, softcap)
        out[b, : Hq * D] = o.reshape(-1).to(out.dtype)
    return out


def rmsnorm_into(x, w, out, eps=1e-6):
    """out = rmsnorm(x) * w into a preallocated tensor (no statistics saved)."""
    if _cuda(x):
        C().rmsnorm_fwd(x, None, w, out, None, None, float(eps))
        return out
    y, _, _ = ref.rmsnorm(x, w, eps)
    out.copy_(y.to(out.dtype))
    return out


def qkv_finalize_rope(acc, bias, qkv, pos, slot, cos_t, sin_t, k_cache, v_cache, Hq, Hkv, D, page_table=None):
    """Decode QKV epilogue: qkv = rope(bf16(acc + bias)); k/v appended to the
    caches at (slot, pos); acc zeroed."""
    if _cuda(acc):
        C().qkv_finalize_rope(acc, bias, qkv, pos, slot, cos_t, sin_t, k_cache, v_cache, int(Hq), int(Hkv), int(D),
                              page_table)
        return qkv
    B, W = qkv.shape[0], (Hq + 2 * Hkv) * D
    a = acc[:B, :W].clone()
    if bias is not None:
        a = a + bias.float()
    qkv[:, :W].copy_(a.to(qkv.dtype))
    acc[:B, :W] = 0
    return rope_kv_append(qkv, pos, slot, cos_t, sin_t, k_cache, v_cache, Hq, Hkv, D, page_table)


def skinny_gemm_swiglu(x, w, acc, act, tile_cnt, splits=0):
    """act[M, F] = silu(x w_gate^T) * (x w_up^T), w = [gate; up] [2F, K], as one
    decode GEMM whose tile finisher applies the SwiGLU (acc: zeroed fp32
    scratch, left zeroed; tile_cnt: int32 counters, left zeroed)."""
    if _cuda(x):
        C().skinny_gemm_swiglu(x, w, acc, act, tile_cnt, int(splits))
        return act
    F_ = w.shape[0] // 2
    z = x.float() @ w.float().t()
    act[: x.shape[0], :F_].copy_((torch.nn.functional.silu(z[:, :F_]) * z[:, F_:]).to(act.dtype))
    return act


def decode_mega(m, embed, final_norm, head, vocab_rows, vocab_col0, d, hq, hkv, f, eps, scale, tok, pos, slot,
                seqlen, next_tok, logits, cache0, page_table, rank, world, timeout_s):
    """The whole greedy decode step in one persistent kernel (csrc/decode_mega.cu);
    ``m`` holds the layer table, scratch, state and exchange buffers built by
    QwenModel._mega_setup. CUDA only (the kernel chain is the portable path)."""
    if not _cuda(embed):
        raise RuntimeError("decode_mega runs on CUDA devices only")
    C().decode_mega(m["table"], embed, final_norm, head, int(vocab_rows), int(vocab_col0), int(d), int(hq), int(hkv),
                    int(f), float(eps), float(scale), tok, pos, slot, seqlen, next_tok, logits, cache0, page_table,
                    m["x"], m["x2"], m["q"], m["o"], m["act"], m["part"], m["pair_ctr"], m["red0"], m["red1"],
                    int(m["red0_mc"]), int(m["red1_mc"]), m["flags"], m["flag_peers"], m["keys"], m["key_peers"],
                    int(rank), int(world), m["state"], float(timeout_s), m.get("trace"), int(m.get("debug", 0)))


def skinny_gemm_qkv(x, w, acc, tile_cnt, bias, qkv, pos, slot, cos_t, sin_t, k_cache, v_cache, Hq, Hkv,
                    page_table=None, splits=0):
    """The decode QKV projection and its epilogue in one GEMM (head_dim 128):
    qkv = rope(bf16(x wqkv^T + bias)) with k / v appended to the caches."""
    if _cuda(x):
        C().skinny_gemm_qkv(x, w, acc, tile_cnt, bias, qkv, pos, slot, cos_t, sin_t, k_cache, v_cache, int(Hq),
                            int(Hkv), page_table, int(splits))
        return qkv
    skinny_gemm(x, w, acc)
    return qkv_finalize_rope(acc, bias, qkv, pos, slot, cos_t, sin_t, k_cache, v_cache, Hq, Hkv, 128, page_table)


def finalize_residual_norm(acc, y, w, h, bias=None, res=None, eps=1e-6, wait=None):
    """y = bf16(acc + bias + res) (residual stream); h = rmsnorm(y) * w; acc zeroed.
    wait: as in skinny_finalize."""
    if _cuda(acc):
        if wait is None:
            C().finalize_residual_norm(acc, bias, res, y, w, h, float(eps))
        else:
            C().finalize_residual_norm(acc, bias, res, y, w, h, float(eps), *wait)
        return y, h
    B, N = y.shape
    a = acc[:B, :N].clone()
    if bias is not None:
        a = a + bias.float()
    if res is not None:
        a = a + res.float()
    y.copy_(a.to(y.dtype))
    acc[:B, :N] = 0
    rmsnorm_into(y, w, h, eps)
    return y, h


# ------------------------------------------------------------------ block quantisation (QLoRA base weights)
Q8_0, Q4_0 = 8, 2  # GGUF type ids
_QBYTES = {Q8_0: 34, Q4_0: 18}


def quantize_blocks(x, fmt=Q8_0):
    """bf16 tensor (numel % 32 == 0) -> uint8 GGUF blocks (Q8_0 or Q4_0)."""
    n = x.numel()
    assert n % 32 == 0
    if _cuda(x):
        out = torch.empty(n // 32 * _QBYTES[fmt], dtype=torch.uint8, device=x.device)
        C().quantize_blocks(x.contiguous(), out, int(fmt))
        return out
    from ..formats import gguf

    q = gguf._quant_q8_0 if fmt == Q8_0 else gguf._quant_q4_0
    return torch.frombuffer(bytearray(q(x.float().numpy().reshape(-1))), dtype=torch.uint8)


GGUF_DEVICE_TYPES = frozenset({0, 1, 2, 6, 8, 12, 13, 14, 30})  # F32 F16 Q4_0 Q5_0 Q8_0 Q4_K Q5_K Q6_K BF16


def gguf_dequant(blocks, typ, rows, K, out):
    """``rows`` rows of K elements stored back to back as GGUF type ``typ``
    (uint8 blocks) -> out[:rows, :K] (bf16). CUDA: one kernel for every type
    in GGUF_DEVICE_TYPES; CPU: the host dequantiser."""
    if _cuda(blocks):
        C().gguf_dequant(blocks, int(typ), int(rows), int(K), out)
        return out
    from ..formats import gguf

    x = gguf.dequantize(blocks.numpy(), int(typ), int(rows) * int(K)).reshape(int(rows), int(K))
    out[:rows, :K].copy_(torch.from_numpy(x).to(out.dtype))
    return out


def dequantize_blocks(q, shape, fmt=Q8_0, out=None):
    """uint8 GGUF blocks -> bf16 tensor of ``shape``."""
    n = 1
    for s_ in shape:
        n *= int(s_)
    if _cuda(q):
        out = out if out is not None else torch.empty(shape, dtype=torch.bfloat16, device=q.device)
        C().dequantize_blocks(q, out, int(fmt))
        return out
    from ..formats import gguf

    x = torch.from_numpy(gguf.dequantize(q.numpy(), fmt, n)).reshape(shape).to(torch.bfloat16)
    if out is not None:
        out.copy_(x)
        return out
    return x


# ------------------------------------------------------------------ mixture of experts
MOE_TILE = 128


def moe_route(logits, k, softmax_all=True, renorm=False, sigmoid=False, scale=1.0):
    """fp32 router logits [T, E] -> (expert ids int32 [T, k], weights fp32 [T, k]).
    softmax_all: softmax over all experts then top-k (renorm: weights / their sum);
    sigmoid: per-expert sigmoid scores then top-k (renorm likewise); otherwise
    softmax over the k selected logits. Weights are multiplied by ``scale``."""
    T, E = logits.shape
    if _cuda(logits):
        idx = torch.empty(T, k, dtype=torch.int32, device=logits.device)
        wt = torch.empty(T, k, dtype=torch.float32, device=logits.device)
        lg = logits if logits.dtype == torch.float32 and logits.stride(1) == 1 else logits.float().contiguous()
        C().moe_route(lg, idx, wt, int(k), bool(softmax_all), bool(renorm), bool(sigmoid), float(scale))
        return idx, wt
    idx, wt = _moe_route_cpu(logits, k, softmax_all, renorm, sigmoid)
    return idx, wt * scale


def _moe_route_cpu(logits, k, softmax_all, renorm, sigmoid):
    lf = logits.float()
    if sigmoid:
        wt, idx = torch.topk(torch.sigmoid(lf), k, dim=-1)
        if renorm:
            wt = wt / wt.sum(-1, keepdim=True)
        return idx.to(torch.int32), wt
    if softmax_all:
        pr = torch.softmax(lf, -1)
        wt, idx = torch.topk(pr, k, dim=-1)
        if renorm:
            wt = wt / wt.sum(-1, keepdim=True)
    else:
        top, idx = torch.topk(lf, k, dim=-1)
        wt = torch.softmax(top, -1)
    return idx.to(torch.int32), wt


# ------------------------------------------------------------------ multi-head latent attention
MLA_LAT, MLA_ROPE = 512, 64


def mla_attention(q_abs, cache, slot, seqlen, out, scale, splits=1, part_o=None, part_lse=None):
    """Absorbed MLA: q_abs [N, H, 576], latent cache [slots, max_seq, 576],
    query n sees cache rows [0, seqlen[n]) of slot[n]; out [N, H, 512] =
    softmax(scale q_abs . cache) cache[:, :512]."""
    N, H, _ = q_abs.shape
    if _cuda(q_abs):
        if part_o is None:
            part_o = torch.empty(N * H * splits * MLA_LAT, dtype=torch.float32, device=q_abs.device)
            part_lse = torch.empty(N * H * splits, dtype=torch.float32, device=q_abs.device)
        C().mla_attention(q_abs, cache, slot, seqlen, out, part_o, part_lse, int(splits), float(scale))
        return out
    for n in range(N):
        L = int(seqlen[n])
        kv = cache[int(slot[n]), :L].float()
        pr = torch.softmax(q_abs[n].float() @ kv.t() * scale, -1)
        out[n] = (pr @ kv[:, :MLA_LAT]).to(out.dtype)
    return out


def mla_prep(kv_a, norm_w, eps, q, H, q_hd, nope, pos, slot, cos_t, sin_t, cache, q_abs):
    """Per token: cache[slot, pos] = [RMSNorm(kv_a[:512]) * w, rope(kv_a[512:576])]
    and q_abs[:, h, 512:] = rope(q[:, h, nope:nope + 64])."""
    if _cuda(kv_a):
        C().mla_prep(kv_a, norm_w, float(eps), q, int(H), int(q_hd), int(nope), pos, slot, cos_t, sin_t, cache,
                     q_abs)
        return
    T = kv_a.shape[0]
    c = kv_a[:, :MLA_LAT].float()
    c = c * torch.rsqrt(c.pow(2).mean(-1, keepdim=True) + eps) * norm_w.float()
    kpe = ref.rope(kv_a[:, MLA_LAT : MLA_LAT + MLA_ROPE].float().contiguous(), pos, cos_t, sin_t, 1, MLA_ROPE)
    qpe = q.view(T, H, q_hd)[:, :, nope : nope + MLA_ROPE].float().reshape(T, H * MLA_ROPE)
    qpe = ref.rope(qpe, pos, cos_t, sin_t, H, MLA_ROPE).view(T, H, MLA_ROPE)
    for t in range(T):
        cache[int(slot[t]), int(pos[t]), :MLA_LAT] = c[t].to(cache.dtype)
        cache[int(slot[t]), int(pos[t]), MLA_LAT:] = kpe[t].to(cache.dtype)
    q_abs[:, :, MLA_LAT:] = qpe.to(q_abs.dtype)


def moe_rows(T, k, E):
    """Rows of the permuted buffer: every expert segment padded to 128 rows."""
    n = T * k + E * (MOE_TILE - 1)
    return (n + MOE_TILE - 1) // MOE_TILE * MOE_TILE


def moe_permute(idx, E, e0=0):
    """-> (row_of int32 [T*k], src_row int32 [Mpad], tile_group int32 [Mpad/128]).
    Experts [e0, e0 + E) are local (tile groups 0..E-1); pairs routed to any
    other expert get row -1 (expert parallelism)."""
    T, k = idx.shape
    Mpad = moe_rows(T, k, E)
    dev = idx.device
    if _cuda(idx):
        row_of = torch.empty(T * k, dtype=torch.int32, device=dev)
        src_row = torch.empty(Mpad, dtype=torch.int32, device=dev)
        tile_group = torch.empty(Mpad // MOE_TILE, dtype=torch.int32, device=dev)
        C().moe_permute(idx.contiguous(), int(E), row_of, src_row, tile_group, int(e0))
        return row_of, src_row, tile_group
    flat = idx.reshape(-1).long() - e0
    local = (flat >= 0) & (flat < E)
    counts = torch.bincount(flat[local], minlength=E)
    seg = (counts + MOE_TILE - 1) // MOE_TILE * MOE_TILE
    off = torch.zeros(E + 1, dtype=torch.long)
    off[1:] = torch.cumsum(seg, 0)
    row_of = torch.empty(T * k, dtype=torch.int32)
    src_row = torch.full((Mpad,), -1, dtype=torch.int32)
    cur = off[:-1].clone()
    for i, e in enumerate(flat.tolist()):
        if e < 0 or e >= E:
            row_of[i] = -1
            continue
        row_of[i] = int(cur[e])
        src_row[int(cur[e])] = i // k
        cur[e] += 1
    tile_group = torch.full((Mpad // MOE_TILE,), -1, dtype=torch.int32)
    for e in range(E):
        tile_group[int(off[e]) // MOE_TILE : int(off[e + 1]) // MOE_TILE] = e
    return row_of, src_row, tile_group


def moe_gather(x, src_row):
    Mpad = src_row.numel()
    if _cuda(x):
        X = torch.empty(Mpad, x.shape[1], dtype=x.dtype, device=x.device)
        C().moe_gather(x, src_row, X)
        return X
    X = torch.zeros(Mpad, x.shape[1], dtype=x.dtype)
    ok = src_row >= 0
    X[ok] = x[src_row[ok].long()]
    return X


def gemm_grouped(X, w, tile_group):
    """X [Mpad, K] bf16 (expert segments on 128-row boundaries), w [E, N, K] ->
    [Mpad, N]; rows of unused tiles are left undefined."""
    E, N, K = w.shape
    if _cuda(X):
        out = torch.empty(X.shape[0], N, dtype=torch.bfloat16, device=X.device)
        C().gemm_grouped(X, w, out, tile_group)
        return out
    out = torch.zeros(X.shape[0], N, dtype=torch.bfloat16)
    for t, e in enumerate(tile_group.tolist()):
        if e >= 0:
            rows = slice(t * MOE_TILE, (t + 1) * MOE_TILE)
            out[rows] = (X[rows].float() @ w[e].float().t()).to(torch.bfloat16)
    return out


def moe_combine(Y, row_of, wt, res=None, extra=None):
    """out[t] = sum_j wt[t, j] * Y[row_of[t, j]] (+ res) (+ extra), bf16 [T, d]."""
    T, k = wt.shape
    if _cuda(Y):
        out = torch.empty(T, Y.shape[1], dtype=torch.bfloat16, device=Y.device)
        C().moe_combine(Y, row_of, wt, int(k), res, extra, out)
        return out
    r = row_of.long()
    w = torch.where(r >= 0, wt.reshape(-1), torch.zeros(())).view(T, k, 1)
    acc = (Y[r.clamp(min=0)].float().view(T, k, -1) * w).sum(1)
    for a in (res, extra):
        if a is not None:
            acc = acc + a.float()
    return acc.to(torch.bfloat16)


def head_rmsnorm_(x, h0, nh, D, w, eps=1e-6):
    """In place: RMSNorm (weight [D]) of heads [h0, h0+nh) of every row of x [T, row]."""
    if _cuda(x):
        C().head_rmsnorm(x, int(h0), int(nh), int(D), w, float(eps))
        return x
    v = x[:, h0 * D : (h0 + nh) * D].float().view(x.shape[0], nh, D)
    v = v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + eps) * w.float()
    x[:, h0 * D : (h0 + nh) * D] = v.reshape(x.shape[0], -1).to(x.dtype)
    return x
