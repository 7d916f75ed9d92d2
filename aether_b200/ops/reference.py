"""Plain-PyTorch fp32 statements of every op: the numerics oracle for the CUDA
kernels and the implementation used for CPU tensors.

Semantics follow the reference runtime's CPU ops (runtime/src/ops.rs) and CUDA
kernels (runtime/src/cuda.rs): tanh-GELU with 0.044715, half-split RoPE with
theta_i = base^(-2i/d), cross-entropy with the 1e-12 probability floor, and
the decoupled AdamW update p -= lr * (m_hat / (sqrt(v_hat) + eps) + wd * p).
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def gemm(a, b, a_mn=False, b_mn=False, bias=None, residual=None, alpha=1.0):
    A = a.float().t() if a_mn else a.float()
    B = b.float() if b_mn else b.float().t()
    out = alpha * (A @ B)
    if bias is not None:
        out = out + bias.float()
    if residual is not None:
        out = out + residual.float()
    return out


def rmsnorm(x, w, eps=1e-6, res=None):
    h = x.float()
    if res is not None:
        h = (h + res.float()).to(x.dtype).float()
    rstd = torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps)
    return h * rstd * w.float(), h, rstd.squeeze(-1)


def layernorm(x, w, b=None, eps=1e-5, res=None):
    h = x.float()
    if res is not None:
        h = (h + res.float()).to(x.dtype).float()
    return F.layer_norm(h, (h.shape[-1],), w.float(), None if b is None else b.float(), eps), h


def softmax(x, scale=1.0):
    return torch.softmax(x.float() * scale, dim=-1)


def swiglu(h):
    g, u = h.float().chunk(2, dim=-1)
    return F.silu(g) * u


def gelu_tanh(x):
    x = x.float()
    return 0.5 * x * (1.0 + torch.tanh(math.sqrt(2.0 / math.pi) * (x + 0.044715 * x.pow(3))))


def rope_tables(max_pos: int, head_dim: int, base: float = 10000.0, device=None):
    inv = base ** (-torch.arange(0, head_dim // 2, dtype=torch.float64) * 2.0 / head_dim)
    ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None, :]
    return ang.cos().float().to(device), ang.sin().float().to(device)


def rope(x, pos, cos_t, sin_t, n_heads, head_dim, inverse=False):
    """x: [T, row] with heads [0, n_heads) rotated (half-split pairs)."""
    T = x.shape[0]
    xs = x[:, : n_heads * head_dim].float().view(T, n_heads, head_dim)
    c = cos_t[pos.long()][:, None, :]
    s = sin_t[pos.long()][:, None, :]
    if inverse:
        s = -s
    a, b = xs[..., : head_dim // 2], xs[..., head_dim // 2 :]
    out = torch.cat([a * c - b * s, b * c + a * s], dim=-1)
    y = x.float().clone()
    y[:, : n_heads * head_dim] = out.reshape(T, n_heads * head_dim)
    return y


def attention(q, k, v, scale, causal=True, causal_offset=0, window=0, softcap=0.0):
    """q [B,Sq,Hq,D], k/v [B,Sk,Hkv,D] -> (out [B,Sq,Hq,D], lse [B,Hq,Sq]).
    window > 0: query i sees keys (i + offset - window, i + offset];
    softcap > 0: logits -> softcap * tanh(logits / softcap)."""
    B, Sq, Hq, D = q.shape
    Sk, Hkv = k.shape[1], k.shape[2]
    g = Hq // Hkv
    qf = q.float().permute(0, 2, 1, 3)
    kf = k.float().permute(0, 2, 1, 3).repeat_interleave(g, dim=1)
    vf = v.float().permute(0, 2, 1, 3).repeat_interleave(g, dim=1)
    s = (qf @ kf.transpose(-1, -2)) * scale
    if softcap > 0:
        s = softcap * torch.tanh(s / softcap)
    i = torch.arange(Sq, device=q.device)[:, None]
    j = torch.arange(Sk, device=q.device)[None, :]
    if causal:
        s = s.masked_fill(j > i + causal_offset, float("-inf"))
    if window > 0:
        s = s.masked_fill(j < i + causal_offset - window + 1, float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    p = torch.softmax(s, dim=-1)
    o = p @ vf
    return o.permute(0, 2, 1, 3), lse


def cross_entropy(logits, targets, ignore_index=-100):
    """Per-row loss with the reference's probability floor."""
    lf = logits.float()
    lse = torch.logsumexp(lf, dim=-1)
    t = targets.clamp(min=0)
    xt = lf.gather(-1, t[:, None]).squeeze(-1)
    p = torch.exp(xt - lse).clamp(min=1e-12)
    loss = -torch.log(p)
    return torch.where(targets == ignore_index, torch.zeros_like(loss), loss), lse


def cross_entropy_grad(logits, targets, scale, ignore_index=-100):
    lf = logits.float()
    p = torch.softmax(lf, dim=-1)
    valid = targets != ignore_index
    oh = torch.zeros_like(p)
    oh[valid, targets[valid]] = 1.0
    g = (p - oh) * scale
    g[~valid] = 0
    return g


def adamw(p, g, m, v, lr, beta1, beta2, eps, wd, step, gscale=1.0):
    g = g * gscale
    m.mul_(beta1).add_(g, alpha=1 - beta1)
    v.mul_(beta2).addcmul_(g, g, value=1 - beta2)
    mh = m / (1 - beta1**step)
    vh = v / (1 - beta2**step)
    p.sub_(lr * (mh / (vh.sqrt() + eps) + wd * p))
    return p
