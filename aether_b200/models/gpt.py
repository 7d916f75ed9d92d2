"""GPT-style decoder (pre-RMSNorm, RoPE, SwiGLU, untied LM head) for training.

This is the model family of the training benchmark: 24 layers, d_model 2048,
16 heads, SwiGLU intermediate 5632, vocab 32000, seq 2048, random init
N(0, 0.02), bf16 compute with fp32 master weights. The reference's trainer
model (trainer/src/model.rs:200-670: pre-LN, GELU MLP, learned positions,
tied head) and its GPU Qwen block stage (trainer/src/qwen_stage.rs:48-446:
RMSNorm, QKV, RoPE, causal SDPA, O, SwiGLU) are the two shapes this class
covers; ``AetherLMNano`` in ``nano.py`` is the exact CPU trainer model.

One layer, as executed (T = B*S token rows, everything bf16 [T, *]):
    h   = rmsnorm(x)                       (norm.cu)
    qkv = h @ Wqkv^T ; rope(q, k)          (tcgen05 GEMM, in-place RoPE)
    o   = attention(qkv)                   (flash attention, causal)
    x   = x + o @ Wo^T                     (residual fused in GEMM epilogue)
    h   = rmsnorm(x)
    a   = swiglu(h @ Wgu^T)
    x   = x + a @ Wd^T                     (residual fused)
and finally loss = CE(rmsnorm(x) @ Wlm^T) with the logits gradient produced in
the same pass.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from ..ops import autograd as A
from ..ops import reference as ref
from .arena import ParamArena


@dataclass
class GPTConfig:
    vocab: int = 32000
    d_model: int = 2048
    n_layers: int = 24
    n_heads: int = 16
    n_kv_heads: int = 16
    d_ff: int = 5632
    max_seq: int = 2048
    rope_theta: float = 10000.0
    norm_eps: float = 1e-5
    init_std: float = 0.02
    tie_embeddings: bool = False
    qk_norm: bool = False  # Qwen3: per-head RMSNorm of q and k before RoPE
    qkv_bias: bool = False  # Qwen2: bias on the q / k / v projections
    head_dim_: int = 0  # explicit head dimension (0: d_model / n_heads)
    attn_window: int = 0  # > 0: sliding-window attention (query i sees keys (i - window, i])
    attn_softcap: float = 0.0  # > 0: attention logits soft-capped by softcap * tanh(s / softcap)

    @property
    def head_dim(self) -> int:
        return self.head_dim_ or self.d_model // self.n_heads

    @staticmethod
    def gpt_24l() -> "GPTConfig":
        return GPTConfig()

    def n_params(self) -> int:
        d, f, v, L = self.d_model, self.d_ff, self.vocab, self.n_layers
        qkv = (self.n_heads + 2 * self.n_kv_heads) * self.head_dim * d
        per = qkv + d * d + 2 * f * d + f * d + 2 * d
        return L * per + v * d * (1 if self.tie_embeddings else 2) + d

    def flops_per_token(self, seq: int) -> float:
        """Training FLOPs per token (fwd + bwd = 3x fwd), causal attention counted at half."""
        d, L = self.d_model, self.n_layers
        mm = self.n_params() - self.vocab * d * (0 if self.tie_embeddings else 1)  # embedding gather is free
        attn = 2 * 2 * seq * d * L / 2
        return 6.0 * mm + 3.0 * attn


def gpt_param_specs(cfg: GPTConfig, layers=None, first: bool = True, last: bool = True, tp_size: int = 1):
    """Parameter specs (name, shape, weight_decay). ``layers`` / ``first`` /
    ``last`` select one pipeline stage's share of the model, ``tp_size`` one
    tensor-parallel rank's shard shapes."""
    d, f, v = cfg.d_model, cfg.d_ff, cfg.vocab
    qkv = (cfg.n_heads + 2 * cfg.n_kv_heads) * cfg.head_dim
    layers = range(cfg.n_layers) if layers is None else layers
    specs = [("tok_emb", (v, d), True)] if (first or (last and cfg.tie_embeddings)) else []
    for i in layers:
        specs += [
            (f"l{i}.attn_norm", (d,), False),
            (f"l{i}.wqkv", (qkv, d), True),
        ]
        if cfg.qkv_bias:
            specs.append((f"l{i}.bqkv", (qkv,), False))
        if cfg.qk_norm:
            specs += [(f"l{i}.q_norm", (cfg.head_dim,), False), (f"l{i}.k_norm", (cfg.head_dim,), False)]
        specs += [
            (f"l{i}.wo", (d, cfg.n_heads * cfg.head_dim), True),
            (f"l{i}.mlp_norm", (d,), False),
            (f"l{i}.wgu", (2 * f, d), True),
            (f"l{i}.wd", (d, f), True),
        ]
    if last:
        specs.append(("final_norm", (d,), False))
        if not cfg.tie_embeddings:
            specs.append(("lm_head", (v, d), True))
    if tp_size > 1:
        from ..parallel.tp_train import shard_shape

        assert not cfg.qkv_bias, "tensor-parallel training shards no qkv bias"
        specs = [(n, shard_shape(cfg, n, shp, tp_size), dec) for n, shp, dec in specs]
    return specs


class _ReadyHook:
    """Gradient hook on a layer's input: tells the data-parallel engine that the
    named parameter bucket's gradients are final (returns None: the gradient
    passes through unchanged)."""

    def __init__(self, fn, key: str):
        self.fn, self.key = fn, key

    def __call__(self, grad):
        self.fn(self.key)


class GPT:
    """The whole model, or one pipeline stage of it (``layers``, ``first``,
    ``last``): a first stage embeds token ids, a last stage ends in the final
    norm, LM head and loss, other stages map hidden states to hidden states."""

    def __init__(self, cfg: GPTConfig, device="cuda", seed: int = 0, pad_multiple: int = 1, alloc=None,
                 layers=None, first: bool = True, last: bool = True, tp=None, cp=None, shard=None,
                 external: frozenset = frozenset(), loss_chunk: int = 0):
        """tp: a ``parallel.tp_train.TPGroup`` -- this rank then holds its
        Megatron shard of every layer (and the same values as the matching
        slice of the unsharded model with the same seed).
        shard: a ``parallel.fsdp.ShardSpec`` -- ZeRO-2 / ZeRO-3 (FSDP) storage:
        the arena holds only this rank's slice of every layer.
        external: projection names ("wqkv", "wo", "wgu", "wd") whose weights
        live outside the arena (a frozen quantised base: adapters replace
        ``_linear`` and supply them); their shapes are in ``external_shapes``.
        loss_chunk > 0: the LM head + cross-entropy runs over that many tokens
        at a time (peak memory [loss_chunk, vocab] instead of [tokens, vocab])."""
        self.cfg = cfg
        self.loss_chunk = loss_chunk
        self.tp = tp if tp is not None and tp.world > 1 else None
        # context parallel (parallel.cp.CPGroup): this rank holds one contiguous
        # chunk of every sequence; attention all-gathers K/V over the group
        self.cp = cp if cp is not None and cp.world > 1 else None
        tp_size = self.tp.world if self.tp else 1
        if self.tp is not None and self.tp.sp:
            assert first and last and self.cp is None and shard is None, \
                "sequence parallelism needs the whole model on a flat arena, without CP"
        assert cfg.n_heads % tp_size == 0 and cfg.n_kv_heads % tp_size == 0 and cfg.d_ff % tp_size == 0
        self.device = torch.device(device)
        self.layers = list(range(cfg.n_layers) if layers is None else layers)
        self.first, self.last = first, last
        specs = gpt_param_specs(cfg, self.layers, first, last, tp_size)
        self.external_shapes = {n: shp for n, shp, _ in specs if n.split(".")[-1] in external}
        specs = [sp for sp in specs if sp[0] not in self.external_shapes]
        if shard is not None:
            from ..parallel.fsdp import ShardedArena

            self.arena = ShardedArena(specs, self.device, shard)
        else:
            self.arena = ParamArena(specs, self.device, pad_multiple=pad_multiple, alloc=alloc)
        self.init_weights(seed)
        cos, sin = ref.rope_tables(cfg.max_seq, cfg.head_dim, cfg.rope_theta, device=self.device)
        self.rope_cos, self.rope_sin = cos.contiguous(), sin.contiguous()
        self._pos_cache: dict[tuple, torch.Tensor] = {}

    def init_weights(self, seed: int) -> None:
        """N(0, init_std) weights, unit norms. Every tensor has its own CPU
        generator keyed by its index in the full model, so any pipeline split
        (and any device) produces the same values as the unsplit model."""
        full = gpt_param_specs(self.cfg)
        index = {name: i for i, (name, _, _) in enumerate(full)}
        full_shape = {name: shp for name, shp, _ in full}
        a = self.arena
        with torch.no_grad():
            for name in a.names():
                if name.endswith("norm"):
                    t = torch.ones(full_shape[name], dtype=torch.float32)
                elif name.endswith("bqkv"):
                    t = torch.zeros(full_shape[name], dtype=torch.float32)
                else:
                    g = torch.Generator(device="cpu").manual_seed(seed * 1000003 + index[name])
                    t = torch.empty(full_shape[name], dtype=torch.float32)
                    t.normal_(0.0, self.cfg.init_std, generator=g)
                if self.tp is not None:
                    from ..parallel.tp_train import shard_tensor

                    t = shard_tensor(self.cfg, name, t, self.tp.rank, self.tp.world)
                a.set_full(name, t)
        a.sync_bf16_from_master()

    def _linear(self, i: int, name: str, x: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        """The projection ``name`` of layer i (adapters replace this hook).
        Under TP: column-parallel projections see the input through
        ``tp_copy``; row-parallel ones all-reduce their partial sums, with the
        residual added once (by TP rank 0's GEMM epilogue)."""
        w = self.arena[f"l{i}.{name}"]
        if self.tp is None:
            return A.linear(x, w, residual=residual)
        from ..parallel import tp_train as T

        if self.tp.sp:  # x and the residual are this rank's token rows
            if name in T.COLUMN:
                return T.sp_column_linear(x, w, self.tp)
            return T.sp_row_linear(x, w, residual, self.tp)
        if name in T.COLUMN:
            return A.linear(T.tp_copy(x, self.tp), w)
        y = A.linear(x, w, residual=residual.detach() if (residual is not None and self.tp.rank == 0) else None)
        return T.tp_reduce_residual(y, residual, self.tp)

    def _qk_norm(self, i: int, qkv: torch.Tensor, Hq: int, Hkv: int, D: int) -> torch.Tensor:
        """Qwen3's per-head RMSNorm of the q and k heads (one shared weight of
        head_dim per layer each): the heads become the rows of the row-norm
        kernels, and the normalised q, k and the untouched v are reassembled."""
        T, a = qkv.shape[0], self.arena
        eps = self.cfg.norm_eps
        # contiguous head rows (with one head a reshape would keep the qkv row stride)
        q = A.rmsnorm(qkv[:, : Hq * D].contiguous().view(T * Hq, D), a[f"l{i}.q_norm"], eps).view(T, Hq * D)
        k = A.rmsnorm(qkv[:, Hq * D : (Hq + Hkv) * D].contiguous().view(T * Hkv, D), a[f"l{i}.k_norm"],
                      eps).view(T, Hkv * D)
        return torch.cat([q, k, qkv[:, (Hq + Hkv) * D :]], 1)

    def freeze(self) -> None:
        """Stops gradients to every base parameter (adapter fine-tuning): the
        weight-gradient GEMMs are skipped and the flat gradient stays unused."""
        for name in self.arena.names():
            v = self.arena[name]
            v.requires_grad_(False)
            if hasattr(v, "main_grad"):
                del v.main_grad

    def positions(self, B: int, S: int) -> torch.Tensor:
        """Global positions of this rank's tokens (offset by the CP chunk)."""
        key = (B, S)
        if key not in self._pos_cache:
            off = self.cp.rank * S if self.cp is not None else 0
            self._pos_cache[key] = (torch.arange(S, dtype=torch.int32, device=self.device) + off).repeat(B)
        return self._pos_cache[key]

    def forward_hidden(self, ids: torch.Tensor, x: torch.Tensor | None = None, B: int | None = None,
                       S: int | None = None) -> torch.Tensor:
        """First stage: ids [B, S] -> hidden; later stages: x [B*S, d] -> hidden.
        The last stage applies the final RMSNorm."""
        cfg, a = self.cfg, self.arena
        if ids is not None:
            B, S = ids.shape
        tpw = self.tp.world if self.tp else 1
        Hq, Hkv, D = cfg.n_heads // tpw, cfg.n_kv_heads // tpw, cfg.head_dim
        scale = 1.0 / math.sqrt(D)
        pos = self.positions(B, S)
        sp = self.tp is not None and self.tp.sp
        if self.first:
            x = A.embedding(a["tok_emb"], ids.reshape(-1))  # [T, d]
        if sp:
            from ..parallel import tp_train as T

            assert x.shape[0] % self.tp.world == 0, "sequence parallelism needs B*S divisible by the TP degree"
            x = T.sp_split(x, self.tp)
        lin = self._linear
        ready = getattr(self, "grad_ready_hook", None) if torch.is_grad_enabled() else None
        for i in self.layers:
            if ready is not None and x.requires_grad:
                # x's gradient is complete only after every op of layer i has run
                # backward, so layer i's parameter gradients are final then
                x.register_hook(_ReadyHook(ready, f"l{i}"))
            h, res = A.rmsnorm_residual(x, a[f"l{i}.attn_norm"], cfg.norm_eps)
            qkv = lin(i, "wqkv", h)
            if cfg.qkv_bias:
                qkv = A.add_bias(qkv, a[f"l{i}.bqkv"])
            if cfg.qk_norm:
                qkv = self._qk_norm(i, qkv, Hq, Hkv, D)
            qkv = A.rope_(qkv, pos, self.rope_cos, self.rope_sin, Hq + Hkv, D)
            if self.cp is None:
                o = A.attention_packed(qkv, B, S, Hq, Hkv, D, scale, causal=True, window=cfg.attn_window,
                                       softcap=cfg.attn_softcap)
            else:
                from ..parallel.cp import cp_attention

                o = cp_attention(qkv, B, S, Hq, Hkv, D, scale, self.cp)
            x = lin(i, "wo", o, residual=res)
            h, res = A.rmsnorm_residual(x, a[f"l{i}.mlp_norm"], cfg.norm_eps)
            gu = lin(i, "wgu", h)
            act = A.swiglu(gu)
            x = lin(i, "wd", act, residual=res)
        if sp:
            x = T.sp_gather(x, self.tp)
        if ready is not None and self.last and x.requires_grad:
            x.register_hook(_ReadyHook(ready, "head"))  # after the LM head and final norm backward
        return A.rmsnorm(x, a["final_norm"], cfg.norm_eps) if self.last else x

    def finish_grads(self) -> None:
        """After the last backward of a step, sum over the TP group the
        gradients that each rank holds only in part: the per-layer norms under
        sequence parallelism (each rank saw its own tokens) and the shared q/k
        norm weights under any TP (each rank normalised its own heads). One
        all-reduce; everything else already holds the full gradient."""
        if self.tp is None:
            return
        names = [n for n in ("attn_norm", "mlp_norm") if self.tp.sp]
        names += [n for n in ("q_norm", "k_norm") if self.cfg.qk_norm]
        gs = [getattr(self.arena[f"l{i}.{n}"], "main_grad", None) for i in self.layers for n in names]
        gs = [g for g in gs if g is not None]  # frozen base weights (adapters) have none
        if not gs:
            return
        flat = torch.cat([g.reshape(-1) for g in gs])
        self.tp.all_reduce_(flat)
        off = 0
        for g in gs:
            g.view(-1).copy_(flat[off : off + g.numel()])
            off += g.numel()

    def _loss(self, ids, targets, loss_scale, x):
        assert self.last, "loss needs the last stage"
        B, S = targets.shape
        h = self.forward_hidden(ids, x=x, B=B, S=S)
        w = self.arena["tok_emb"] if self.cfg.tie_embeddings else self.arena["lm_head"]
        if loss_scale is None:
            loss_scale = 1.0 / targets.numel()
        if self.loss_chunk and h.shape[0] > self.loss_chunk:
            return A.lm_head_cross_entropy_chunked(h, w, targets.reshape(-1), loss_scale, self.loss_chunk)
        return A.lm_head_cross_entropy(h, w, targets.reshape(-1), loss_scale)

    def loss(self, ids: torch.Tensor, targets: torch.Tensor, loss_scale: float | None = None,
             x: torch.Tensor | None = None) -> torch.Tensor:
        """Sum of per-token CE times loss_scale (default 1/num_tokens = mean).
        A last pipeline stage passes its input hidden states as ``x``."""
        hooks = getattr(self.arena, "autograd_hooks", None)
        if hooks is None:
            return self._loss(ids, targets, loss_scale, x)
        with hooks():
            return self._loss(ids, targets, loss_scale, x)

    @torch.no_grad()
    def logits(self, ids: torch.Tensor) -> torch.Tensor:
        from ..ops import functional as F

        h = self.forward_hidden(ids)
        w = self.arena["tok_emb"] if self.cfg.tie_embeddings else self.arena["lm_head"]
        return F.gemm(h, w)
