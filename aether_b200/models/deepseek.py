"""DeepSeek-V2 family (DeepSeek-V2 / V2-Lite, GLM-4.7-flash): multi-head
latent attention with the weight-absorbed cache, YaRN RoPE, and DeepSeek MoE
(routed experts with softmax or sigmoid scores and a routed scaling factor,
plus always-on shared experts), for serving.

Attention of one layer (H heads, latent rank 512, RoPE dims 64):
    q      = h Wq^T                      (or Wq_b RMSNorm(h Wq_a^T) with a q LoRA)
    kv_a   = h Wkv_a^T = [c_kv (512), k_pe (64)]
    cache[slot, pos] = [RMSNorm(c_kv) * w, rope(k_pe)]            (mla_prep)
    q_abs[h] = [q_nope[h] W_uk[h], rope(q_pe[h])]                  (576 dims)
    o_lat[h] = softmax(scale q_abs[h] . cache) cache[:, :512]     (mla_attention)
    o[h]   = o_lat[h] W_uv[h]^T ;  x += o Wo^T
where W_uk[h] / W_uv[h] are head h's key / value blocks of Wkv_b. Only the
576-dim latent is cached per token (all heads share it), and prefill and
decode run the same per-token path: a prefill token is a query whose length
is its position + 1.

Tensor parallelism (``tp``: ``rank``, ``world``, ``all_reduce_``): the heads
are split over the ranks (their q rows, W_uk / W_uv blocks and W_o columns),
the shared latent is computed and cached on every rank, the routed experts are
partitioned over the same ranks and the dense / shared-expert FFNs are split
by columns / rows; each block ends in one all-reduce of its partial output.

FFN: the first ``first_dense`` layers are dense SwiGLU; the others route
each token to ``top_k`` of ``n_experts`` (grouped tcgen05 GEMMs over tokens
sorted by expert, as in ``models/moe.py``) and add the shared experts (one
SwiGLU of width n_shared * d_expert). DeepSeek-V3's selection bias and
group-limited routing are not modelled.

Reference: the MLA fields of ModelConfig (runtime/src/serving.rs:459-900,
is_mla_absorbed :769), the MLA forward (serving.rs:1747-2100) and its
kernels (cuda.rs:1718-2670), and the DeepSeek / GLM MoE routing
(serving.rs:2269-2400).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from ..ops import functional as F
from ..ops import reference as ref


@dataclass
class DeepSeekConfig:
    vocab: int = 102400
    d_model: int = 2048
    n_layers: int = 27
    n_heads: int = 16
    q_lora_rank: int = 0
    kv_lora_rank: int = 512
    qk_nope: int = 128
    qk_rope: int = 64
    v_head: int = 128
    d_ff: int = 10944          # dense layers
    first_dense: int = 1
    n_experts: int = 64
    top_k: int = 6
    d_expert: int = 1408
    n_shared: int = 2
    router: str = "softmax"    # or "sigmoid"
    norm_topk: bool = False
    routed_scale: float = 1.0
    rope_theta: float = 10000.0
    yarn_factor: float = 0.0   # 0: plain RoPE
    yarn_orig_ctx: int = 4096
    yarn_beta_fast: float = 32.0
    yarn_beta_slow: float = 1.0
    yarn_mscale: float = 1.0
    yarn_mscale_all_dim: float = 0.0
    norm_eps: float = 1e-6
    max_seq: int = 4096
    init_std: float = 0.02
    tie_embeddings: bool = False

    @staticmethod
    def deepseek_v2_lite(**kw) -> "DeepSeekConfig":
        base = dict(yarn_factor=40.0, yarn_mscale=0.707, yarn_mscale_all_dim=0.707, max_seq=4096)
        base.update(kw)
        return DeepSeekConfig(**base)

    @property
    def qk_head(self) -> int:
        return self.qk_nope + self.qk_rope

    def softmax_scale(self) -> float:
        s = 1.0 / math.sqrt(self.qk_head)
        if self.yarn_factor > 1.0 and self.yarn_mscale_all_dim:
            m = yarn_mscale(self.yarn_factor, self.yarn_mscale_all_dim)
            s *= m * m
        return s


def yarn_mscale(scale: float, mscale: float = 1.0) -> float:
    return 1.0 if scale <= 1.0 else 0.1 * mscale * math.log(scale) + 1.0


def yarn_rope_tables(cfg: DeepSeekConfig, max_pos: int, device=None):
    """RoPE tables [max_pos, 32] for the 64 RoPE dims. With yarn_factor > 1:
    YaRN (Peng et al., "YaRN: Efficient Context Window Extension of Large
    Language Models", 2023) -- per-frequency interpolation between the
    original and the factor-scaled frequencies by a linear ramp over the
    dims whose wavelength falls between beta_fast and beta_slow rotations of
    the original context, and cos / sin scaled by the attention temperature
    ratio."""
    dim, base = cfg.qk_rope, cfg.rope_theta
    expo = torch.arange(0, dim, 2, dtype=torch.float64) / dim
    extra = 1.0 / base**expo
    if cfg.yarn_factor <= 1.0:
        inv, msc = extra, 1.0
    else:
        s = cfg.yarn_factor

        def corr_dim(rot):
            return dim * math.log(cfg.yarn_orig_ctx / (rot * 2 * math.pi)) / (2 * math.log(base))

        lo = max(math.floor(corr_dim(cfg.yarn_beta_fast)), 0)
        hi = min(math.ceil(corr_dim(cfg.yarn_beta_slow)), dim - 1)
        if lo == hi:
            hi += 0.001
        ramp = ((torch.arange(dim // 2, dtype=torch.float64) - lo) / (hi - lo)).clamp(0, 1)
        keep = 1.0 - ramp  # 1: original frequency (high-frequency dims), 0: interpolated
        inv = (extra / s) * (1 - keep) + extra * keep
        msc = yarn_mscale(s, cfg.yarn_mscale) / yarn_mscale(s, cfg.yarn_mscale_all_dim or 1.0)
    ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None, :]
    return (ang.cos() * msc).float().to(device).contiguous(), (ang.sin() * msc).float().to(device).contiguous()


class DeepSeekWeights:
    def __init__(self, cfg: DeepSeekConfig, device, seed: int = 0, tp_rank: int = 0, tp_size: int = 1):
        """tp_rank / tp_size: keep this rank's heads, experts and FFN slices
        (the same values as the matching slices of the unsplit weights)."""
        assert cfg.kv_lora_rank == F.MLA_LAT and cfg.qk_rope == F.MLA_ROPE, "MLA kernels: latent 512, rope 64"
        assert cfg.n_heads % tp_size == 0 and cfg.d_ff % tp_size == 0, "heads and d_ff must split over TP"
        assert (cfg.n_shared * cfg.d_expert) % tp_size == 0, "the shared experts must split over TP"
        dev = torch.device(device)
        self.cfg, self.device = cfg, dev
        self.tp_rank, self.tp_size = tp_rank, tp_size
        d, H = cfg.d_model, cfg.n_heads
        idx = [0]

        def rnd(*shape, std=cfg.init_std):
            idx[0] += 1
            g = torch.Generator(device=dev).manual_seed(seed * 7919 + 31 * idx[0])
            return (torch.randn(*shape, generator=g, device=dev) * std).to(torch.bfloat16)

        r, w = tp_rank, tp_size
        Hl = H // w
        h0 = r * Hl

        def rows(t, n):  # this rank's n-row block
            return t[r * n : (r + 1) * n].contiguous()

        def cols(t, n):
            return t[:, r * n : (r + 1) * n].contiguous()

        def gu_rows(t, f):  # gate and up halves each split into w blocks
            g_, u_ = t[:f], t[f:]
            return torch.cat([rows(g_, f // w), rows(u_, f // w)]).contiguous()

        from .moe import expert_range

        e0, e1 = expert_range(cfg.n_experts, r, w)
        self.e0, self.e1 = e0, e1

        ones = lambda n: torch.ones(n, dtype=torch.bfloat16, device=dev)  # noqa: E731
        self.embed = rnd(cfg.vocab, d)
        self.lm_head = self.embed if cfg.tie_embeddings else rnd(cfg.vocab, d)
        self.final_norm = ones(d)
        L = cfg.n_layers
        self.attn_norm, self.mlp_norm = [ones(d) for _ in range(L)], [ones(d) for _ in range(L)]
        self.wq, self.wq_a, self.q_a_norm, self.wq_b = [], [], [], []
        self.wkv_a, self.kv_norm, self.w_uk, self.w_uv, self.wo = [], [], [], [], []
        self.dense_gu, self.dense_d = [], []
        self.router, self.exp_gu, self.exp_d, self.sh_gu, self.sh_d = [], [], [], [], []
        qh, Ep = cfg.qk_head, (cfg.n_experts + 7) // 8 * 8
        for i in range(L):
            if cfg.q_lora_rank:
                self.wq.append(None)
                self.wq_a.append(rnd(cfg.q_lora_rank, d))
                self.q_a_norm.append(ones(cfg.q_lora_rank))
                self.wq_b.append(rows(rnd(H * qh, cfg.q_lora_rank), Hl * qh))
            else:
                self.wq.append(rows(rnd(H * qh, d), Hl * qh))
            self.wkv_a.append(rnd(F.MLA_LAT + F.MLA_ROPE, d))  # the shared latent: every rank
            self.kv_norm.append(torch.ones(F.MLA_LAT, dtype=torch.float32, device=dev))
            wkv_b = rnd(H * (cfg.qk_nope + cfg.v_head), F.MLA_LAT).view(H, cfg.qk_nope + cfg.v_head, F.MLA_LAT)
            self.w_uk.append(wkv_b[h0 : h0 + Hl, : cfg.qk_nope].contiguous())   # [Hl, 128, 512]
            self.w_uv.append(wkv_b[h0 : h0 + Hl, cfg.qk_nope :].contiguous())   # [Hl, v_head, 512]
            self.wo.append(cols(rnd(d, H * cfg.v_head), Hl * cfg.v_head))
            if i < cfg.first_dense:
                self.dense_gu.append(gu_rows(rnd(2 * cfg.d_ff, d), cfg.d_ff))
                self.dense_d.append(cols(rnd(d, cfg.d_ff), cfg.d_ff // w))
                for lst in (self.router, self.exp_gu, self.exp_d, self.sh_gu, self.sh_d):
                    lst.append(None)
            else:
                self.dense_gu.append(None)
                self.dense_d.append(None)
                rt = torch.zeros(Ep, d, dtype=torch.bfloat16, device=dev)
                rt[: cfg.n_experts] = rnd(cfg.n_experts, d)
                self.router.append(rt)
                self.exp_gu.append(rnd(cfg.n_experts, 2 * cfg.d_expert, d)[e0:e1].contiguous())
                self.exp_d.append(rnd(cfg.n_experts, d, cfg.d_expert)[e0:e1].contiguous())
                fs = cfg.n_shared * cfg.d_expert
                self.sh_gu.append(gu_rows(rnd(2 * fs, d), fs) if fs else None)
                self.sh_d.append(cols(rnd(d, fs), fs // w) if fs else None)


class DeepSeekModel:
    def __init__(self, cfg: DeepSeekConfig, device="cuda", seed: int = 0, max_batch: int = 16,
                 max_seq: int | None = None, weights: DeepSeekWeights | None = None, tp=None):
        self.cfg = cfg
        self.device = torch.device(device)
        self.tp = tp if tp is not None and tp.world > 1 else None
        r, w = (tp.rank, tp.world) if self.tp is not None else (0, 1)
        self.w = weights or DeepSeekWeights(cfg, device, seed, r, w)
        self.heads = cfg.n_heads // w  # this rank's heads
        self.max_batch = max_batch
        self.max_seq = max_seq or cfg.max_seq
        self.scratch_slot = max_batch
        self.paged = False  # per-slot contiguous latent caches
        # the latent cache: one 576-wide row per token for all heads
        self.cache = [torch.zeros(max_batch + 1, self.max_seq, F.MLA_LAT + F.MLA_ROPE, dtype=torch.bfloat16,
                                  device=self.device) for _ in range(cfg.n_layers)]
        self.cos, self.sin = yarn_rope_tables(cfg, self.max_seq, self.device)
        self.scale = cfg.softmax_scale()
        self.hgroups = (self.heads + 15) // 16
        self._graphs: dict[tuple, torch.cuda.CUDAGraph] = {}
        B = max_batch
        self.buf = {"tok": torch.zeros(B, dtype=torch.long, device=self.device),
                    "pos": torch.zeros(B, dtype=torch.int32, device=self.device),
                    "slot": torch.arange(B, dtype=torch.int32, device=self.device),
                    "next": torch.zeros(B, dtype=torch.long, device=self.device),
                    "logits": torch.zeros(B, cfg.vocab, dtype=torch.float32, device=self.device)}
        self._want_logits = False

    # ------------------------------------------------------------------ blocks
    def _attention(self, i: int, h: torch.Tensor, x: torch.Tensor, pos, slot, splits: int) -> torch.Tensor:
        cfg, w = self.cfg, self.w
        T, H = h.shape[0], self.heads
        if cfg.q_lora_rank:
            qa = F.gemm(h, w.wq_a[i])
            qa, _, _ = F.rmsnorm(qa, w.q_a_norm[i], cfg.norm_eps)
            q = F.gemm(qa, w.wq_b[i])
        else:
            q = F.gemm(h, w.wq[i])  # [T, H * 192]
        kv_a = F.gemm(h, w.wkv_a[i])  # [T, 576]
        q_abs = torch.empty(T, H, F.MLA_LAT + F.MLA_ROPE, dtype=torch.bfloat16, device=h.device)
        q_nope = q.view(T, H, cfg.qk_head)[:, :, : cfg.qk_nope]
        q_abs[:, :, : F.MLA_LAT] = torch.bmm(q_nope.transpose(0, 1), w.w_uk[i]).transpose(0, 1)
        F.mla_prep(kv_a, w.kv_norm[i], cfg.norm_eps, q, H, cfg.qk_head, cfg.qk_nope, pos, slot, self.cos, self.sin,
                   self.cache[i], q_abs)
        o_lat = torch.empty(T, H, F.MLA_LAT, dtype=torch.bfloat16, device=h.device)
        F.mla_attention(q_abs, self.cache[i], slot, pos + 1, o_lat, self.scale, splits)
        o = torch.bmm(o_lat.transpose(0, 1), w.w_uv[i].transpose(1, 2)).transpose(0, 1).reshape(T, H * cfg.v_head)
        if self.tp is None:
            return F.gemm(o.contiguous(), w.wo[i], residual=x)
        y = F.gemm(o.contiguous(), w.wo[i])  # this rank's heads' share
        self.tp.all_reduce_(y)
        return x + y

    def _ffn(self, i: int, h: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
        cfg, w = self.cfg, self.w
        if w.dense_gu[i] is not None:
            if self.tp is None:
                return F.gemm(F.swiglu(F.gemm(h, w.dense_gu[i])), w.dense_d[i], residual=x)
            y = F.gemm(F.swiglu(F.gemm(h, w.dense_gu[i])), w.dense_d[i])
            self.tp.all_reduce_(y)
            return x + y
        logits = F.gemm(h, w.router[i], out_dtype=torch.float32)[:, : cfg.n_experts]
        idx, wt = F.moe_route(logits, cfg.top_k, softmax_all=cfg.router == "softmax", renorm=cfg.norm_topk,
                              sigmoid=cfg.router == "sigmoid", scale=cfg.routed_scale)
        e0, e1 = getattr(w, "e0", 0), getattr(w, "e1", cfg.n_experts)
        row_of, src_row, tile_group = F.moe_permute(idx, e1 - e0, e0)
        X = F.moe_gather(h, src_row)
        Y = F.gemm_grouped(F.swiglu(F.gemm_grouped(X, w.exp_gu[i], tile_group)), w.exp_d[i], tile_group)
        extra = F.gemm(F.swiglu(F.gemm(h, w.sh_gu[i])), w.sh_d[i]) if w.sh_gu[i] is not None else None
        if self.tp is None:
            return F.moe_combine(Y, row_of, wt, res=x, extra=extra)
        y = F.moe_combine(Y, row_of, wt, extra=extra)  # this rank's experts + shared-expert slice
        self.tp.all_reduce_(y)
        return x + y

    def _forward(self, tok: torch.Tensor, pos: torch.Tensor, slot: torch.Tensor, splits: int) -> torch.Tensor:
        """Token rows (any mix of sequences and positions) -> final hidden [T, d];
        every row's K/V latent is appended to its slot's cache first."""
        cfg, w = self.cfg, self.w
        x = F.embedding(w.embed, tok)
        for i in range(cfg.n_layers):
            h, _, _ = F.rmsnorm(x, w.attn_norm[i], cfg.norm_eps)
            x = self._attention(i, h, x, pos, slot, splits)
            h, _, _ = F.rmsnorm(x, w.mlp_norm[i], cfg.norm_eps)
            x = self._ffn(i, h, x)
        h, _, _ = F.rmsnorm(x, w.final_norm, cfg.norm_eps)
        return h

    def _splits(self, rows: int) -> int:
        return max(1, min(16, -(-296 // max(1, rows * self.hgroups))))

    # ------------------------------------------------------------------ serving API
    @torch.no_grad()
    def prefill(self, tokens: torch.Tensor, slots: torch.Tensor | None = None, start_pos: int = 0,
                return_logits: bool = False):
        """tokens [B, S] at positions start_pos.. (the cache of each slot already
        holds the earlier ones) -> greedy next token [B] (and fp32 logits)."""
        B, S = tokens.shape
        dev = self.device
        slots = torch.arange(B, dtype=torch.int32, device=dev) if slots is None else slots.to(dev, torch.int32)
        pos = (torch.arange(S, dtype=torch.int32, device=dev) + start_pos).repeat(B)
        h = self._forward(tokens.to(dev).reshape(-1), pos, slots.repeat_interleave(S), 1)
        last = h.view(B, S, -1)[:, -1].contiguous()
        logits = F.gemm(last, self.w.lm_head, out_dtype=torch.float32)
        nxt = logits.argmax(-1)
        return (nxt, logits) if return_logits else nxt

    def _decode_body(self, B: int) -> None:
        b = self.buf
        h = self._forward(b["tok"][:B], b["pos"][:B], b["slot"][:B], self._splits(B))
        logits = F.gemm(h, self.w.lm_head, out_dtype=torch.float32)
        if self._want_logits:
            b["logits"][:B].copy_(logits)
        b["next"][:B].copy_(logits.argmax(-1))

    def _bucket(self, B: int) -> int:
        for s in (1, 2, 4, 8, 16, 32, 64):
            if B <= s <= self.max_batch:
                return s
        return self.max_batch

    @torch.no_grad()
    def decode_step(self, tokens: torch.Tensor, pos: torch.Tensor, slots: torch.Tensor | None = None,
                    use_graph: bool = True, want_logits: bool = False) -> torch.Tensor:
        """tokens [B] at positions pos [B] -> greedy next tokens [B]; with
        want_logits the fp32 logits are left in ``buf["logits"][:B]``."""
        B = tokens.shape[0]
        Bb = self._bucket(B)
        b = self.buf
        b["tok"][:B].copy_(tokens)
        b["pos"][:B].copy_(pos)
        if slots is not None:
            b["slot"][:B].copy_(slots)
        if Bb > B:
            b["tok"][B:Bb].zero_()
            b["pos"][B:Bb].zero_()
            b["slot"][B:Bb].fill_(self.scratch_slot)
        self._want_logits = want_logits
        if use_graph and self.device.type == "cuda":
            key = (Bb, want_logits)
            if key not in self._graphs:
                s = torch.cuda.Stream(self.device)
                s.wait_stream(torch.cuda.current_stream(self.device))
                with torch.cuda.stream(s):
                    for _ in range(2):
                        self._decode_body(Bb)
                torch.cuda.current_stream(self.device).wait_stream(s)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, capture_error_mode="thread_local"):
                    self._decode_body(Bb)
                self._graphs[key] = g
            self._graphs[key].replay()
        else:
            self._decode_body(Bb)
        self._want_logits = False
        return b["next"][:B]

    @torch.no_grad()
    def generate(self, prompts: torch.Tensor, max_new_tokens: int, use_graph: bool = True) -> torch.Tensor:
        B, S = prompts.shape
        assert B <= self.max_batch and S + max_new_tokens <= self.max_seq
        out = torch.empty(B, max_new_tokens, dtype=torch.long, device=self.device)
        tok = self.prefill(prompts)
        out[:, 0] = tok
        pos = torch.full((B,), S, dtype=torch.int32, device=self.device)
        slots = torch.arange(B, dtype=torch.int32, device=self.device)
        for t in range(1, max_new_tokens):
            tok = self.decode_step(tok, pos, slots, use_graph=use_graph).clone()
            out[:, t] = tok
            pos += 1
        return out

    # ------------------------------------------------------------------ oracle
    @torch.no_grad()
    def reference_logits(self, tokens: torch.Tensor) -> torch.Tensor:
        """fp32 forward of [B, S] tokens in the standard (non-absorbed) MLA form:
        per-head keys / values decompressed from the latent, causal attention
        over 192-dim queries / keys, 128-dim values (one rank)."""
        assert self.tp is None, "the oracle needs the unsplit weights"
        cfg, w = self.cfg, self.w
        B, S = tokens.shape
        H, nope, rope_d, vh = cfg.n_heads, cfg.qk_nope, cfg.qk_rope, cfg.v_head
        rms = lambda t, g, eps=cfg.norm_eps: t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + eps) * g.float()  # noqa: E731
        x = w.embed.float()[tokens.to(self.device)]
        pos = torch.arange(S, device=self.device).repeat(B)
        for i in range(cfg.n_layers):
            h = rms(x, w.attn_norm[i])
            if cfg.q_lora_rank:
                q = rms(h @ w.wq_a[i].float().t(), w.q_a_norm[i]) @ w.wq_b[i].float().t()
            else:
                q = h @ w.wq[i].float().t()
            q = q.view(B, S, H, nope + rope_d)
            kv_a = h @ w.wkv_a[i].float().t()
            c = rms(kv_a[..., : F.MLA_LAT], w.kv_norm[i])
            k_pe = ref.rope(kv_a[..., F.MLA_LAT :].reshape(B * S, rope_d), pos, self.cos, self.sin, 1, rope_d)
            q_pe = ref.rope(q[..., nope:].reshape(B * S, H * rope_d), pos, self.cos, self.sin, H, rope_d)
            k_nope = torch.einsum("bsl,hnl->bshn", c, w.w_uk[i].float())
            v = torch.einsum("bsl,hvl->bshv", c, w.w_uv[i].float())
            qf = torch.cat([q[..., :nope], q_pe.view(B, S, H, rope_d)], -1)
            kf = torch.cat([k_nope, k_pe.view(B, S, 1, rope_d).expand(B, S, H, rope_d)], -1)
            s = torch.einsum("bqhd,bkhd->bhqk", qf, kf) * self.scale
            s = s.masked_fill(torch.ones(S, S, dtype=torch.bool, device=self.device).triu(1), float("-inf"))
            o = torch.einsum("bhqk,bkhv->bqhv", torch.softmax(s, -1), v).reshape(B, S, H * vh)
            x = x + o @ w.wo[i].float().t()
            h = rms(x, w.mlp_norm[i])
            x = x + self._reference_ffn(i, h)
        return rms(x, w.final_norm) @ w.lm_head.float().t()

    def _reference_ffn(self, i: int, h: torch.Tensor) -> torch.Tensor:
        cfg, w = self.cfg, self.w

        def swiglu(t, wgu, wd):
            g, u = (t @ wgu.float().t()).chunk(2, -1)
            return (torch.nn.functional.silu(g) * u) @ wd.float().t()

        if w.dense_gu[i] is not None:
            return swiglu(h, w.dense_gu[i], w.dense_d[i])
        shp = h.shape
        h2 = h.reshape(-1, shp[-1])
        lg = h2 @ w.router[i][: cfg.n_experts].float().t()
        if cfg.router == "sigmoid":
            wt, idx = torch.topk(torch.sigmoid(lg), cfg.top_k, dim=-1)
        else:
            wt, idx = torch.topk(torch.softmax(lg, -1), cfg.top_k, dim=-1)
        if cfg.norm_topk:
            wt = wt / wt.sum(-1, keepdim=True)
        wt = wt * cfg.routed_scale
        out = torch.zeros_like(h2)
        for t in range(h2.shape[0]):
            for j in range(cfg.top_k):
                e = int(idx[t, j])
                out[t] += wt[t, j] * swiglu(h2[t], w.exp_gu[i][e], w.exp_d[i][e])
        if w.sh_gu[i] is not None:
            out += swiglu(h2, w.sh_gu[i], w.sh_d[i])
        return out.view(shp)
