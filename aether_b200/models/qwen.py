"""Qwen2 / Qwen2.5 decoder for serving (also Llama/Mistral-shaped when
``qkv_bias=False``): batched prefill into a preallocated KV cache and a
CUDA-graph-captured greedy decode step.

Reference: QwenSession (runtime/src/serving.rs:2528-4835) and its block
forward (serving.rs:1334-1500). Differences by design:
  * prefill runs the whole prompt through the tensor-core GEMM and flash
    attention at once (the reference loops the decode path token by token,
    serving.rs:3285-3299, so its TTFT is O(prompt) decode launches);
  * decode GEMMs are split-K swap-AB tcgen05 GEMMs over all SMs with fused
    bias / residual / SwiGLU finalisation; decode attention is split-K over the
    cache with one CTA per (sequence, KV head, split);
  * positions, slots and lengths live in device buffers, so one captured CUDA
    graph per batch bucket replays every step (the reference captures one
    global graph, cuda.rs:8295-8380);
  * greedy sampling runs on the device (the reference copies [vocab] fp32
    logits to the host every step, serving.rs:3418).

Weights are random-init bf16 (N(0, 0.02)) unless loaded from a
safetensors/GGUF checkpoint through ``aether_b200.formats``.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from ..ops import functional as F
from ..ops import reference as ref


@dataclass
class QwenConfig:
    vocab: int = 151936
    d_model: int = 1536
    n_layers: int = 28
    n_heads: int = 12
    n_kv_heads: int = 2
    d_ff: int = 8960
    rope_theta: float = 1e6
    norm_eps: float = 1e-6
    tie_embeddings: bool = True
    qkv_bias: bool = True
    max_seq: int = 4096
    init_std: float = 0.02
    qk_norm: bool = False  # Qwen3: per-head RMSNorm of q and k before RoPE
    head_dim_: int = 0     # 0: d_model / n_heads
    # flex attention: a sliding window of `sliding_window` keys (0: full); with
    # `sliding_window_pattern` p > 0 only layers i % p != p - 1 are windowed
    # (the others attend globally) and windowed layers use rope_theta_swa when
    # set; attn_softcap > 0 soft-caps the logits (softcap * tanh(s / softcap))
    sliding_window: int = 0
    sliding_window_pattern: int = 0
    rope_theta_swa: float = 0.0
    attn_softcap: float = 0.0

    def layer_window(self, i: int) -> tuple[int, float]:
        """(sliding window, RoPE base) of layer i (reference: ModelConfig::attn_layer_params)."""
        if self.sliding_window_pattern > 0:
            p = self.sliding_window_pattern
            if i % p != p - 1:
                return self.sliding_window, self.rope_theta_swa or self.rope_theta
            return 0, self.rope_theta
        return self.sliding_window, self.rope_theta

    @property
    def head_dim(self) -> int:
        return self.head_dim_ or self.d_model // self.n_heads

    @staticmethod
    def qwen25_1_5b(**kw) -> "QwenConfig":
        return QwenConfig(**kw)

    @staticmethod
    def qwen25_7b(**kw) -> "QwenConfig":
        base = dict(vocab=152064, d_model=3584, n_layers=28, n_heads=28, n_kv_heads=4, d_ff=18944,
                    tie_embeddings=False)
        base.update(kw)
        return QwenConfig(**base)

    @staticmethod
    def qwen3_8b(**kw) -> "QwenConfig":
        base = dict(vocab=151936, d_model=4096, n_layers=36, n_heads=32, n_kv_heads=8, d_ff=12288, qkv_bias=False,
                    qk_norm=True, tie_embeddings=False)
        base.update(kw)
        return QwenConfig(**base)

    @staticmethod
    def llama3_8b(**kw) -> "QwenConfig":
        base = dict(vocab=128256, d_model=4096, n_layers=32, n_heads=32, n_kv_heads=8, d_ff=14336, qkv_bias=False,
                    tie_embeddings=False, rope_theta=500000.0, norm_eps=1e-5)
        base.update(kw)
        return QwenConfig(**base)

    @staticmethod
    def mistral_7b(**kw) -> "QwenConfig":
        base = dict(vocab=32000, d_model=4096, n_layers=32, n_heads=32, n_kv_heads=8, d_ff=14336, qkv_bias=False,
                    tie_embeddings=False, rope_theta=1e6, norm_eps=1e-5)
        base.update(kw)
        return QwenConfig(**base)

    @staticmethod
    def mistral_7b_v01(**kw) -> "QwenConfig":
        """Mistral-7B v0.1: every layer attends over a 4096-key sliding window."""
        base = dict(vocab=32000, d_model=4096, n_layers=32, n_heads=32, n_kv_heads=8, d_ff=14336, qkv_bias=False,
                    tie_embeddings=False, rope_theta=1e4, norm_eps=1e-5, sliding_window=4096)
        base.update(kw)
        return QwenConfig(**base)

    def n_params(self) -> int:
        d, f, D = self.d_model, self.d_ff, self.head_dim
        qkv = (self.n_heads + 2 * self.n_kv_heads) * D
        per = qkv * d + (qkv if self.qkv_bias else 0) + self.n_heads * D * d + 3 * d * f + 2 * d
        return self.n_layers * per + self.vocab * d * (1 if self.tie_embeddings else 2) + d


def tp_heads(Hq: int, Hkv: int, rank: int, tp: int) -> tuple:
    """(query heads, KV heads) of one TP rank. With at least as many KV heads as
    ranks every rank takes whole GQA groups; with fewer, each KV head is
    replicated on tp / Hkv ranks, which split its group's query heads as evenly
    as they go -- so Qwen2.5-7B (28 q / 4 KV heads) runs at TP = 8 with 4 or 3
    query heads per rank."""
    if tp <= Hkv:
        assert Hkv % tp == 0 and Hq % tp == 0, "heads must split evenly over TP"
        hq, hkv = Hq // tp, Hkv // tp
        return list(range(rank * hq, (rank + 1) * hq)), list(range(rank * hkv, (rank + 1) * hkv))
    assert tp % Hkv == 0, "KV heads must replicate evenly over TP"
    per_kv, G = tp // Hkv, Hq // Hkv
    j, sub = divmod(rank, per_kv)
    sizes = [G // per_kv + (1 if s < G % per_kv else 0) for s in range(per_kv)]
    assert min(sizes) > 0, "more ranks than query heads per KV head"
    start = j * G + sum(sizes[:sub])
    return list(range(start, start + sizes[sub])), [j]


class QwenWeights:
    """bf16 weights, optionally one tensor-parallel rank's shard.

    Every full tensor is drawn from its own seeded generator on the target
    device and then sliced, so all TP degrees shard the same random model:
    q/k/v heads and the gate/up rows are split column-parallel, o_proj and
    down_proj row-parallel (Megatron layout, reference
    runtime/src/tensor_parallel.rs:8-29); KV heads are replicated when there
    are fewer KV heads than ranks. Embedding, LM head and norms are replicated.
    """

    def __init__(self, cfg: QwenConfig, device, seed: int = 0, tp_rank: int = 0, tp_size: int = 1):
        self.cfg = cfg
        self.device = torch.device(device)
        self.tp_rank, self.tp_size = tp_rank, tp_size
        d, F_, D, L = cfg.d_model, cfg.d_ff, cfg.head_dim, cfg.n_layers
        Hq, Hkv = cfg.n_heads, cfg.n_kv_heads
        assert F_ % tp_size == 0, "d_ff must split over TP"
        q_heads, kv_heads = tp_heads(Hq, Hkv, tp_rank, tp_size)
        self.hq = len(q_heads)
        self.hkv = len(kv_heads)
        self.f = F_ // tp_size
        r = tp_rank
        idx = [0]

        def rnd(*shape):
            idx[0] += 1
            g = torch.Generator(device=self.device).manual_seed(seed * 1000003 + idx[0])
            t = torch.randn(*shape, generator=g, device=self.device, dtype=torch.float32) * cfg.init_std
            return t.to(torch.bfloat16)

        def heads(t, hs, base):  # rows of the given heads from a [(H...)*D, ...] tensor
            return torch.cat([t[(base + h) * D : (base + h + 1) * D] for h in hs], 0)

        self.embed = rnd(cfg.vocab, d)
        self.lm_head = self.embed if cfg.tie_embeddings else rnd(cfg.vocab, d)
        self._set_vocab_shard()
        self.final_norm = torch.ones(d, dtype=torch.bfloat16, device=self.device)
        self.attn_norm = [torch.ones(d, dtype=torch.bfloat16, device=self.device) for _ in range(L)]
        self.q_norm = [torch.ones(D, dtype=torch.bfloat16, device=self.device) for _ in range(L)] if cfg.qk_norm else None
        self.k_norm = [torch.ones(D, dtype=torch.bfloat16, device=self.device) for _ in range(L)] if cfg.qk_norm else None
        self.mlp_norm = [torch.ones(d, dtype=torch.bfloat16, device=self.device) for _ in range(L)]
        self.wqkv, self.bqkv, self.wo, self.wgu, self.wd = [], [], [], [], []
        for _ in range(L):
            wqkv = rnd((Hq + 2 * Hkv) * D, d)
            bqkv = rnd((Hq + 2 * Hkv) * D) if cfg.qkv_bias else None
            wo = rnd(d, Hq * D)
            wgu = rnd(2 * F_, d)
            wd = rnd(d, F_)
            if tp_size == 1:
                self.wqkv.append(wqkv)
                self.bqkv.append(bqkv)
                self.wo.append(wo)
                self.wgu.append(wgu)
                self.wd.append(wd)
                continue
            parts = [heads(wqkv, q_heads, 0), heads(wqkv, kv_heads, Hq), heads(wqkv, kv_heads, Hq + Hkv)]
            self.wqkv.append(torch.cat(parts, 0).contiguous())
            if bqkv is not None:
                bp = [heads(bqkv, q_heads, 0), heads(bqkv, kv_heads, Hq), heads(bqkv, kv_heads, Hq + Hkv)]
                self.bqkv.append(torch.cat(bp, 0).contiguous())
            else:
                self.bqkv.append(None)
            self.wo.append(wo[:, q_heads[0] * D : (q_heads[-1] + 1) * D].contiguous())
            f0, f1 = r * self.f, (r + 1) * self.f
            self.wgu.append(torch.cat([wgu[f0:f1], wgu[F_ + f0 : F_ + f1]], 0).contiguous())
            self.wd.append(wd[:, f0:f1].contiguous())
            del wqkv, bqkv, wo, wgu, wd

    def _set_vocab_shard(self) -> None:
        """Vocabulary-parallel LM head under TP: rank r keeps rows
        [r * per, r * per + n) of the head (zero-padded to ``per`` rows, a
        multiple of 8), and an untied full head is dropped from the device."""
        cfg, tp = self.cfg, self.tp_size
        self.lm_head_shard = None
        if tp == 1:
            return
        V, d = cfg.vocab, cfg.d_model
        per = (-(-V // tp) + 7) // 8 * 8
        col0 = self.tp_rank * per
        n = max(0, min(per, V - col0))
        assert n > 0, "more TP ranks than vocabulary slices"
        shard = torch.zeros(per, d, dtype=torch.bfloat16, device=self.device)
        shard[:n].copy_(self.lm_head[col0 : col0 + n])
        self.lm_head_shard, self.vocab_col0, self.vocab_n, self.vocab_per = shard, col0, n, per
        if not cfg.tie_embeddings:
            self.lm_head = None  # each rank streams only its slice

    @staticmethod
    def shard(full: "QwenWeights", tp_rank: int, tp_size: int, device) -> "QwenWeights":
        """One rank's shard of full (e.g. GGUF- or HF-loaded) weights, in the
        same layout as the random-init shards, moved to ``device``."""
        cfg = full.cfg
        dev = torch.device(device)
        D, Hq, Hkv, F_ = cfg.head_dim, cfg.n_heads, cfg.n_kv_heads, cfg.d_ff
        q_heads, kv_heads = tp_heads(Hq, Hkv, tp_rank, tp_size)
        w = QwenWeights.__new__(QwenWeights)
        w.cfg, w.device, w.tp_rank, w.tp_size = cfg, dev, tp_rank, tp_size
        w.hq, w.hkv, w.f = len(q_heads), len(kv_heads), F_ // tp_size
        f0, f1 = tp_rank * w.f, (tp_rank + 1) * w.f

        def heads(t, hs, base):
            return torch.cat([t[(base + h) * D : (base + h + 1) * D] for h in hs], 0)

        def qkv(t):
            return torch.cat([heads(t, q_heads, 0), heads(t, kv_heads, Hq), heads(t, kv_heads, Hq + Hkv)],
                             0).contiguous().to(dev)

        to = lambda t: None if t is None else t.to(dev)  # noqa: E731
        w.embed = to(full.embed)
        w.lm_head = w.embed if cfg.tie_embeddings else full.lm_head
        w._set_vocab_shard()
        w.final_norm = to(full.final_norm)
        w.attn_norm = [to(t) for t in full.attn_norm]
        w.mlp_norm = [to(t) for t in full.mlp_norm]
        w.q_norm = [to(t) for t in full.q_norm] if full.q_norm is not None else None
        w.k_norm = [to(t) for t in full.k_norm] if full.k_norm is not None else None
        w.wqkv = [qkv(t) for t in full.wqkv]
        w.bqkv = [None if t is None else qkv(t) for t in full.bqkv]
        w.wo = [t[:, q_heads[0] * D : (q_heads[-1] + 1) * D].contiguous().to(dev) for t in full.wo]
        w.wgu = [torch.cat([t[f0:f1], t[F_ + f0 : F_ + f1]], 0).contiguous().to(dev) for t in full.wgu]
        w.wd = [t[:, f0:f1].contiguous().to(dev) for t in full.wd]
        return w


class KVCache:
    def __init__(self, cfg: QwenConfig, n_kv_heads: int, slots: int, max_seq: int, device):
        shape = (slots, max_seq, n_kv_heads, cfg.head_dim)
        self.k = [torch.zeros(shape, dtype=torch.bfloat16, device=device) for _ in range(cfg.n_layers)]
        self.v = [torch.zeros(shape, dtype=torch.bfloat16, device=device) for _ in range(cfg.n_layers)]
        self.slots, self.max_seq = slots, max_seq

    def bytes(self) -> int:
        return sum(t.numel() * 2 for t in self.k + self.v)


class QwenModel:
    """Single-GPU (or one TP rank's) Qwen2 forward for serving.

    ``tp`` (optional) is an object with ``all_reduce_(t)`` used after the
    row-parallel o_proj and down_proj (see ``parallel/tp.py``)."""

    def __init__(self, cfg: QwenConfig, device="cuda", seed: int = 0, max_batch: int = 64, max_seq: int | None = None,
                 weights: QwenWeights | None = None, tp=None, decode_splits: int = 0, kv_pages: int = 0,
                 page_size: int = 64):
        """kv_pages > 0 selects the paged KV cache (``serving.kv.PagedKVCache``)
        with that many pages of ``page_size`` tokens shared by all sequences;
        otherwise every batch slot owns a contiguous max_seq cache."""
        self.cfg = cfg
        self.device = torch.device(device)
        self.tp = tp
        tp_rank = tp.rank if tp is not None else 0
        tp_size = tp.world if tp is not None else 1
        self.w = weights or QwenWeights(cfg, device, seed, tp_rank, tp_size)
        self.hq, self.hkv, self.f = self.w.hq, self.w.hkv, self.w.f
        # vocabulary-parallel head: needs the TP object's merge / gather and a sharded head
        self.vp = (tp is not None and hasattr(tp, "vocab_argmax")
                   and getattr(self.w, "lm_head_shard", None) is not None)
        # one-shot push reduction of the decode row-parallel GEMMs (CUDA TP only)
        self.push = tp is not None and getattr(tp, "mode", None) == "push"
        self.max_batch = max_batch
        self.max_seq = max_seq or cfg.max_seq
        # one extra slot absorbs the K/V writes of padded batch rows
        if kv_pages > 0:
            from ..serving.kv import PagedKVCache

            self.cache = PagedKVCache(cfg.n_layers, self.hkv, cfg.head_dim, kv_pages, page_size, max_batch + 1,
                                      self.max_seq, self.device)
            self.page_table = self.cache.table
        else:
            self.cache = KVCache(cfg, self.hkv, max_batch + 1, self.max_seq, self.device)
            self.page_table = None
        self.paged = self.page_table is not None
        self.scratch_slot = max_batch
        cos, sin = ref.rope_tables(self.max_seq, cfg.head_dim, cfg.rope_theta, device=self.device)
        self.cos, self.sin = cos.contiguous(), sin.contiguous()
        # per-layer flex attention parameters: window and RoPE tables
        self.win, self.rope_cs = [], []
        tables = {cfg.rope_theta: (self.cos, self.sin)}
        for i in range(cfg.n_layers):
            wnd, base = cfg.layer_window(i)
            if base not in tables:
                c2, s2 = ref.rope_tables(self.max_seq, cfg.head_dim, base, device=self.device)
                tables[base] = (c2.contiguous(), s2.contiguous())
            self.win.append(wnd)
            self.rope_cs.append(tables[base])
        self.softcap = cfg.attn_softcap
        self.scale = 1.0 / math.sqrt(cfg.head_dim)
        self._fixed_splits = decode_splits
        self.decode_splits = decode_splits or self._auto_splits(1)  # the most any batch size uses
        import os as _os
        # the fused decode epilogue has no slot for Qwen3's q/k norm
        self.fused_decode = _os.environ.get("AETHER_UNFUSED_DECODE", "0") != "1" and not cfg.qk_norm
        # QKV (bias + RoPE + KV append) and SwiGLU finished inside their decode GEMMs (opt-in:
        # measured on a B200 the tile finisher serialises in the GEMM tail -- Qwen2.5-7B TP1
        # batch 64: 7.43 ms per step against 5.72 with the separate finalize kernels; batch 1
        # within noise of the separate kernels)
        self.fused_epilogues = (self.fused_decode and cfg.head_dim == 128 and self.f % 64 == 0
                                and _os.environ.get("AETHER_GEMM_EPILOGUES", "0") == "1")
        self._graphs: dict[int, tuple] = {}
        self._alloc_decode_buffers()
        if tp is not None and hasattr(tp, "prepare_decode"):
            V = cfg.vocab
            cols = tp.world * self.w.vocab_per if self.vp else V
            tp.prepare_decode(max_batch + 1, cfg.d_model, cols)
        # the whole decode step as one persistent kernel for batch buckets 1 / 2 / 4
        self.mega = self._mega_supported()
        self._mega = None
        if self.mega:
            self._mega_setup()
        # batch buckets that take the one-kernel step: none unless
        # AETHER_DECODE_MEGA=force. Measured on B200s at batch 1: one GPU
        # holding one TP=8 rank's Qwen2.5-7B shards 1.245 ms per step against
        # 1.367 for the kernel chain (TP=4 shards: +2 %), but Qwen2.5-7B whole
        # 3.57 against 3.36, Qwen2.5-1.5B 1.72 against 1.53, real TP=8 2.21
        # against 1.76 (its in-kernel cross-rank barriers cost more than the
        # chain's push reductions), and batch 2 / 4 slower throughout.
        import os as _os
        forced = _os.environ.get("AETHER_DECODE_MEGA") == "force"
        self.mega_batches = {1, 2, 4} if forced else set()

    # ------------------------------------------------------------------ buffers
    def _mat(self, t):
        """A projection as a bf16 [N, K] tensor: GGUF-quantised weights kept on
        the device (``load_qwen_weights(..., keep_quant=True)``) are expanded
        into the weights' shared scratch right before their GEMM."""
        return t if isinstance(t, torch.Tensor) else t.bf16()

    def _auto_splits(self, B: int) -> int:
        """Key splits of the decode attention for batch size B: enough
        (sequence, KV head, split) CTAs for about two per SM, and no more --
        fewer splits mean longer pipelined runs per CTA and a cheaper merge."""
        if self._fixed_splits:
            return self._fixed_splits
        sms = torch.cuda.get_device_properties(self.device).multi_processor_count if self.device.type == "cuda" else 148
        return max(1, min(32, -(-2 * sms // max(1, B * self.hkv))))

    def _alloc_decode_buffers(self):
        cfg, B, dev = self.cfg, self.max_batch, self.device
        D = cfg.head_dim
        qkv_w = (self.hq + 2 * self.hkv) * D
        widest = max(qkv_w, 2 * self.f, cfg.d_model, self.w.vocab_per if self.vp else cfg.vocab)
        bf = torch.bfloat16
        self.buf = {
            "tok": torch.zeros(B, dtype=torch.long, device=dev),
            "pos": torch.zeros(B, dtype=torch.int32, device=dev),
            "slot": torch.arange(B, dtype=torch.int32, device=dev),
            "seqlen": torch.ones(B, dtype=torch.int32, device=dev),
            "x": torch.zeros(B, cfg.d_model, dtype=bf, device=dev),
            "x2": torch.zeros(B, cfg.d_model, dtype=bf, device=dev),
            "h": torch.zeros(B, cfg.d_model, dtype=bf, device=dev),
            "qkv": torch.zeros(B, qkv_w, dtype=bf, device=dev),
            "o": torch.zeros(B, self.hq * D, dtype=bf, device=dev),
            "act": torch.zeros(B, self.f, dtype=bf, device=dev),
            "acc": torch.zeros(B, widest, dtype=torch.float32, device=dev),
            "part_o": torch.empty(B * self.hq * self.decode_splits * D, dtype=torch.float32, device=dev),
            "part_lse": torch.empty(B * self.hq * self.decode_splits, dtype=torch.float32, device=dev),
            "next": torch.zeros(B, dtype=torch.long, device=dev),
            "counters": torch.zeros(B * self.hkv, dtype=torch.int32, device=dev),
            "logits": torch.zeros(B, cfg.vocab, dtype=torch.float32, device=dev),
            # per-tile K-block counters of the fused-epilogue GEMMs (they return to zero)
            "tiles": torch.zeros(max(qkv_w // 128, self.f // 64) + 1, dtype=torch.int32, device=dev),
        }
        self._want_logits = False

    # ------------------------------------------------------------------ prefill
    @torch.no_grad()
    def prefill(self, tokens: torch.Tensor, slots: torch.Tensor | None = None, start_pos: int = 0,
                return_logits: bool = False):
        """tokens [B, S] (one prompt per cache slot, equal lengths) -> greedy next
        token [B] (and the fp32 last-position logits with return_logits).
        Writes K/V for positions [start_pos, start_pos + S)."""
        cfg, w = self.cfg, self.w
        B, S = tokens.shape
        D = cfg.head_dim
        dev = self.device
        if slots is None:
            slots = torch.arange(B, dtype=torch.int32, device=dev)
        T = B * S
        pos = (torch.arange(S, dtype=torch.int32, device=dev) + start_pos).repeat(B)
        slot_t = slots.to(dev, torch.int32).repeat_interleave(S)
        x = F.embedding(w.embed, tokens.to(dev).reshape(-1))
        row = (self.hq + 2 * self.hkv) * D
        for i in range(cfg.n_layers):
            h, _, _ = F.rmsnorm(x, w.attn_norm[i], cfg.norm_eps)
            qkv = F.gemm(h, self._mat(w.wqkv[i]), bias=w.bqkv[i])
            self._qk_norm(i, qkv)
            F.rope_kv_append(qkv, pos, slot_t, *self.rope_cs[i], self.cache.k[i], self.cache.v[i], self.hq,
                             self.hkv, D, page_table=self.page_table)
            q = qkv.view(B, S, row)[:, :, : self.hq * D].view(B, S, self.hq, D)
            if start_pos == 0:
                k = qkv.view(B, S, row)[:, :, self.hq * D : (self.hq + self.hkv) * D].view(B, S, self.hkv, D)
                v = qkv.view(B, S, row)[:, :, (self.hq + self.hkv) * D :].view(B, S, self.hkv, D)
                o, _ = F.attention(q, k, v, self.scale, True, 0, want_lse=False, window=self.win[i],
                                   softcap=self.softcap)
            else:
                Lk = start_pos + S
                if self.paged:
                    rows = [int(r) for r in slots.tolist()]
                    k = torch.stack([F.gather_kv(self.cache.k[i], r, Lk, self.page_table) for r in rows])
                    v = torch.stack([F.gather_kv(self.cache.v[i], r, Lk, self.page_table) for r in rows])
                else:
                    assert bool((slots == torch.arange(B, device=slots.device)).all()), "chunked prefill needs slots 0..B-1"
                    k = self.cache.k[i][:B, :Lk]
                    v = self.cache.v[i][:B, :Lk]
                o, _ = F.attention(q, k, v, self.scale, True, start_pos, want_lse=False, window=self.win[i],
                                   softcap=self.softcap)
            o2 = o.view(T, self.hq * D)
            if self.tp is None:
                x = F.gemm(o2, self._mat(w.wo[i]), residual=x)
            else:
                y = F.gemm(o2, self._mat(w.wo[i]))
                self.tp.all_reduce_(y)
                x = x + y
            h, _, _ = F.rmsnorm(x, w.mlp_norm[i], cfg.norm_eps)
            x = self._ffn(i, h, x)
        last = x.view(B, S, cfg.d_model)[:, -1].contiguous()
        hl, _, _ = F.rmsnorm(last, w.final_norm, cfg.norm_eps)
        if self.vp:
            loc = F.gemm(hl, w.lm_head_shard, out_dtype=torch.float32)
            nxt = self.tp.vocab_argmax(loc, w.vocab_n, w.vocab_col0)
            if return_logits:
                return nxt, self.tp.gather_vocab(loc, w.vocab_n, w.vocab_col0, cfg.vocab)
            return nxt
        head = self._prefill_head()
        logits = F.gemm(hl, head, out_dtype=torch.float32)
        if head.shape[0] != cfg.vocab:
            logits = logits[:, : cfg.vocab].contiguous()
        nxt = F.argmax(logits)
        return (nxt, logits) if return_logits else nxt

    def _qk_norm(self, i: int, qkv: torch.Tensor) -> None:
        if self.cfg.qk_norm:
            D, eps = self.cfg.head_dim, self.cfg.norm_eps
            F.head_rmsnorm_(qkv, 0, self.hq, D, self.w.q_norm[i], eps)
            F.head_rmsnorm_(qkv, self.hq, self.hkv, D, self.w.k_norm[i], eps)

    def _ffn(self, i: int, h: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
        """x + FFN(h) for token rows (prefill); subclasses swap the FFN."""
        w = self.w
        act = F.swiglu(F.gemm(h, self._mat(w.wgu[i])))
        if self.tp is None:
            return F.gemm(act, self._mat(w.wd[i]), residual=x)
        y = F.gemm(act, self._mat(w.wd[i]))
        self.tp.all_reduce_(y)
        return x + y

    def _prefill_head(self) -> torch.Tensor:
        """LM head for the tensor-core GEMM, whose N must be a multiple of 8:
        vocabularies that are not get a zero-padded copy (made once)."""
        V = self.cfg.vocab
        if V % 8 == 0 or self.device.type != "cuda":
            return self.w.lm_head
        if getattr(self, "_head_p", None) is None:
            hp = torch.zeros((V + 7) // 8 * 8, self.cfg.d_model, dtype=torch.bfloat16, device=self.device)
            hp[:V].copy_(self.w.lm_head)
            self._head_p = hp
        return self._head_p

    # ------------------------------------------------------------------ decode
    def _decode_body(self, B: int) -> None:
        """One greedy decode step for the first B rows of the static buffers.

        Per layer (9 kernels): qkv GEMM -> fused bias+RoPE+KV-append ->
        split-K attention with in-kernel combine -> o_proj GEMM (TP: with the
        all-reduce fused in its epilogue) -> fused residual+RMSNorm -> gate/up
        GEMM -> SwiGLU finalise -> down GEMM (TP: reduce fused) -> fused
        residual+RMSNorm of the next layer. The GEMMs use programmatic
        dependent launch, so their weight stream starts while the preceding
        small kernel still runs."""
        cfg, w, b = self.cfg, self.w, self.buf
        D = cfg.head_dim
        x, x2, h = b["x"][:B], b["x2"][:B], b["h"][:B]
        qkv, o, act, acc = b["qkv"][:B], b["o"][:B], b["act"][:B], b["acc"][:B]
        pos, slot, seqlen = b["pos"][:B], b["slot"][:B], b["seqlen"][:B]
        x.copy_(F.embedding(w.embed, b["tok"][:B]))
        F.rmsnorm_into(x, w.attn_norm[0], h, cfg.norm_eps)
        L = cfg.n_layers
        fused_ep = self.fused_epilogues
        push = self._push_for(B)
        for i in range(L):
            if fused_ep:  # bias + RoPE + KV append finished inside the GEMM
                F.skinny_gemm_qkv(h, self._mat(w.wqkv[i]), acc, b["tiles"], w.bqkv[i], qkv, pos, slot, *self.rope_cs[i],
                                  self.cache.k[i], self.cache.v[i], self.hq, self.hkv, page_table=self.page_table)
            else:
                F.skinny_gemm(h, self._mat(w.wqkv[i]), acc)
                F.qkv_finalize_rope(acc, w.bqkv[i], qkv, pos, slot, *self.rope_cs[i], self.cache.k[i],
                                    self.cache.v[i], self.hq, self.hkv, D, page_table=self.page_table)
            F.decode_attention(qkv, self.cache.k[i], self.cache.v[i], slot, seqlen, o, self.hq, self.scale,
                               self._auto_splits(B), b["part_o"], b["part_lse"], b["counters"], page_table=self.page_table,
                               window=self.win[i], softcap=self.softcap)
            if push:  # local GEMM, then one push-reduce + residual + RMSNorm kernel
                F.skinny_gemm(o, self._mat(w.wo[i]), acc)
                self.tp.push_reduce(acc, x2, res=x, w=w.mlp_norm[i], h=h, eps=cfg.norm_eps)
            else:
                if self.tp is None:
                    F.skinny_gemm(o, self._mat(w.wo[i]), acc)
                    racc = acc
                else:
                    racc = self.tp.reduce_gemm(o, self._mat(w.wo[i]), 2 * i)  # GEMM + all-reduce in one kernel
                F.finalize_residual_norm(racc, x2, w.mlp_norm[i], h, res=x, eps=cfg.norm_eps, wait=self._tp_wait())
            if fused_ep:  # SwiGLU finished inside the gate/up GEMM
                F.skinny_gemm_swiglu(h, self._mat(w.wgu[i]), acc, act, b["tiles"])
            else:
                F.skinny_gemm(h, self._mat(w.wgu[i]), acc)
                F.skinny_finalize(acc, act, swiglu=True)
            nw = w.attn_norm[i + 1] if i + 1 < L else w.final_norm
            if push:
                F.skinny_gemm(act, self._mat(w.wd[i]), acc)
                self.tp.push_reduce(acc, x, res=x2, w=nw, h=h, eps=cfg.norm_eps)
                continue
            if self.tp is None:
                F.skinny_gemm(act, self._mat(w.wd[i]), acc)
                racc = acc
            else:
                racc = self.tp.reduce_gemm(act, self._mat(w.wd[i]), 2 * i + 1)
            F.finalize_residual_norm(racc, x, nw, h, res=x2, eps=cfg.norm_eps, wait=self._tp_wait())
        self._decode_head(B, h, acc)

    def _decode_head(self, B: int, h, acc) -> None:
        """LM head GEMM and greedy pick (TP: this rank's vocabulary slice and
        the cross-rank merge); fp32 logits copied out when asked for."""
        cfg, w, b = self.cfg, self.w, self.buf
        if self.vp:
            F.skinny_gemm(h, w.lm_head_shard, acc)
            if self._want_logits:
                self.tp.gather_vocab(acc, w.vocab_n, w.vocab_col0, cfg.vocab, out=b["logits"][:B])
            self.tp.vocab_argmax(acc, w.vocab_n, w.vocab_col0, out=b["next"][:B])
        else:
            F.skinny_gemm(h, w.lm_head, acc)
            if self._want_logits:
                b["logits"][:B].copy_(acc[:, : cfg.vocab])
            b["next"][:B].copy_(F.argmax(acc[:, : cfg.vocab]))
        acc.zero_()

    def _step_body(self, B: int) -> None:
        if self._mega_for(B):
            self._decode_mega(B, self.buf["logits"][:B] if self._want_logits else None)
            return
        (self._decode_body if self.fused_decode else self._decode_body_unfused)(B)

    # ------------------------------------------------------------------ one-kernel decode step
    def _mega_world(self) -> int:
        """Ranks the kernel exchanges with: a real tensor-parallel team, else 1
        (one GPU, or a single-GPU emulation of one rank's shards)."""
        team = getattr(self.tp, "team", None)
        return self.tp.world if team is not None else 1

    def _mega_supported(self) -> bool:
        """Whether the model fits the one-kernel decode step (csrc/decode_mega.cu):
        head_dim 128, no q/k norm, sliding window or softcap, at most 8 query
        heads per KV head, and -- under real tensor parallelism -- multicast
        reduction buffers (the batch bucket must also fit its activation rows in
        40 KB of shared memory, see _mega_for). AETHER_DECODE_MEGA=0 skips even
        its buffers; =force makes decode use it for every bucket it supports."""
        import os as _os

        cfg = self.cfg
        if _os.environ.get("AETHER_DECODE_MEGA", "1") == "0" or self.device.type != "cuda":
            return False
        if not self.fused_decode or cfg.head_dim != 128 or self.softcap or any(self.win):
            return False
        if not isinstance(self.w.wqkv[0], torch.Tensor):
            return False  # quantised weights are expanded per projection; the one-kernel step streams bf16
        d, f, hq, hkv = cfg.d_model, self.f, self.hq, self.hkv
        if d % 8 or f % 8 or hq % hkv or hq // hkv > 8:
            return False
        if self._mega_world() > 1:
            team = self.tp.team
            if not getattr(team, "use_multicast", False) or self.tp.world > 8:
                return False
        return True

    def _mega_for(self, B: int) -> bool:
        if not self.mega or B not in (1, 2, 4) or B not in self.mega_batches:
            return False
        if self._want_logits and self._mega_world() > 1:
            return False  # full logits need the cross-rank gather of the kernel chain
        return (B * max(self.cfg.d_model, self.hq * 128, self.f) * 2 <= 40 * 1024
                and B * self.hq * 1024 <= 40 * 1024)

    def _mega_setup(self) -> None:
        """Scratch, state and (tensor parallel: symmetric, collectively
        allocated) exchange buffers of the one-kernel decode step, and the
        device table of per-layer weight / cache / RoPE pointers."""
        cfg, w, dev = self.cfg, self.w, self.device
        L, d = cfg.n_layers, cfg.d_model
        G = self.hq // self.hkv
        nsm = torch.cuda.get_device_properties(dev).multi_processor_count
        bf = torch.bfloat16
        rows = []
        for i in range(L):
            cos, sin = self.rope_cs[i]
            ptrs = [w.wqkv[i], w.bqkv[i], w.wo[i], w.wgu[i], w.wd[i], w.attn_norm[i], w.mlp_norm[i],
                    self.cache.k[i], self.cache.v[i], cos, sin]
            rows.append([0 if t is None else t.data_ptr() for t in ptrs])
        m = {
            "table": torch.tensor(rows, dtype=torch.int64, device=dev),
            "x": torch.zeros(4, d, dtype=bf, device=dev),
            "x2": torch.zeros(4, d, dtype=bf, device=dev),
            "q": torch.zeros(4, self.hq * 128, dtype=bf, device=dev),
            "o": torch.zeros(4, self.hq * 128, dtype=bf, device=dev),
            "act": torch.zeros(4, self.f, dtype=bf, device=dev),
            "part": torch.zeros(4 * self.hkv * nsm * G * 130, dtype=torch.float32, device=dev),
            "pair_ctr": torch.zeros(4 * self.hkv, dtype=torch.int32, device=dev),
            "state": torch.zeros(64, dtype=torch.int32, device=dev),
        }
        world = self._mega_world()
        if world > 1:
            team = self.tp.team
            r0, r1 = team.alloc(4 * d, torch.float32), team.alloc(4 * d, torch.float32)
            fl, ky = team.alloc(8, torch.int32), team.alloc(8 * 4, torch.int64)
            for buf in (r0, r1, fl, ky):
                buf.tensor.zero_()
            if not (r0.mc_ptr and r1.mc_ptr):  # no NVLS multicast on this system: keep the kernel chain
                self.mega = False
            m.update(red0=r0.tensor, red1=r1.tensor, red0_mc=r0.mc_ptr, red1_mc=r1.mc_ptr, flags=fl.tensor,
                     flag_peers=torch.tensor(fl.peers_host, dtype=torch.int64), keys=ky.tensor,
                     key_peers=torch.tensor(ky.peers_host, dtype=torch.int64), _bufs=(r0, r1, fl, ky))
            torch.cuda.synchronize(dev)
            import torch.distributed as _dist

            _dist.barrier()
        else:
            m.update(red0=torch.zeros(4, d, dtype=torch.float32, device=dev),
                     red1=torch.zeros(4, d, dtype=torch.float32, device=dev), red0_mc=0, red1_mc=0,
                     flags=torch.zeros(8, dtype=torch.int32, device=dev), flag_peers=torch.zeros(8, dtype=torch.int64),
                     keys=torch.zeros(32, dtype=torch.int64, device=dev), key_peers=torch.zeros(8, dtype=torch.int64))
        self._mega = m

    def _decode_mega(self, B: int, logits=None) -> None:
        """One greedy decode step of B rows in one kernel launch; with logits
        (fp32 [B, >= head rows]) this rank's head rows' logits are written too."""
        cfg, w, b, m = self.cfg, self.w, self.buf, self._mega
        if self.vp:
            head, rows, col0 = w.lm_head_shard, w.vocab_n, w.vocab_col0
        else:
            head, rows, col0 = w.lm_head, cfg.vocab, 0
        tp = self.tp
        world = self._mega_world()
        rank = tp.rank if world > 1 else 0
        timeout = float(tp.team.timeout_s) if world > 1 else 2.0
        F.decode_mega(m, w.embed, w.final_norm, head, rows, col0, cfg.d_model, self.hq, self.hkv, self.f,
                      cfg.norm_eps, self.scale, b["tok"][:B], b["pos"][:B], b["slot"][:B], b["seqlen"][:B],
                      b["next"][:B], logits, self.cache.k[0], self.page_table, rank, world, timeout)

    def _decode_body_unfused(self, B: int) -> None:
        """Decode step with separate norm / RoPE / combine kernels (13 per layer)."""
        cfg, w, b = self.cfg, self.w, self.buf
        D = cfg.head_dim
        x, x2, h = b["x"][:B], b["x2"][:B], b["h"][:B]
        qkv, o, act, acc = b["qkv"][:B], b["o"][:B], b["act"][:B], b["acc"][:B]
        pos, slot, seqlen = b["pos"][:B], b["slot"][:B], b["seqlen"][:B]
        x.copy_(F.embedding(w.embed, b["tok"][:B]))
        for i in range(cfg.n_layers):
            F.rmsnorm_into(x, w.attn_norm[i], h, cfg.norm_eps)
            F.skinny_gemm(h, self._mat(w.wqkv[i]), acc)
            F.skinny_finalize(acc, qkv, bias=w.bqkv[i])
            self._qk_norm(i, qkv)
            F.rope_kv_append(qkv, pos, slot, *self.rope_cs[i], self.cache.k[i], self.cache.v[i], self.hq, self.hkv, D,
                             page_table=self.page_table)
            F.decode_attention(qkv, self.cache.k[i], self.cache.v[i], slot, seqlen, o, self.hq, self.scale,
                               self._auto_splits(B), b["part_o"], b["part_lse"], page_table=self.page_table,
                               window=self.win[i], softcap=self.softcap)
            if self._push_for(B):
                F.skinny_gemm(o, self._mat(w.wo[i]), acc)
                self.tp.push_reduce(acc, x2, res=x)
            elif self.tp is None:
                F.skinny_gemm(o, self._mat(w.wo[i]), acc)
                F.skinny_finalize(acc, x2, res=x)
            else:
                racc = self.tp.reduce_gemm(o, self._mat(w.wo[i]), 2 * i)
                F.skinny_finalize(racc, x2, res=x, wait=self._tp_wait())
            F.rmsnorm_into(x2, w.mlp_norm[i], h, cfg.norm_eps)
            self._decode_ffn(i, h, x2, x, act, acc)
        F.rmsnorm_into(x, w.final_norm, h, cfg.norm_eps)
        self._decode_head(B, h, acc)

    def _tp_wait(self):
        return self.tp.finalize_wait() if self.tp is not None else None

    def _push_for(self, B: int) -> bool:
        """Push reduction for this batch bucket: measured on B200s (Qwen2.5-7B
        shape) the multicast-reduce GEMM is faster for one or a few rows (TP8
        batch 1: 1.76 vs 1.87 ms per step) and the push faster from 16 rows on
        (TP8 batch 64: 3.46 vs 5.01 ms); AETHER_TP_REDUCE pins one mode."""
        if not self.push:
            return False
        import os as _os

        if _os.environ.get("AETHER_TP_REDUCE") == "push":
            return True
        return B > 4

    def _decode_ffn(self, i, h, x2, x, act, acc) -> None:
        """x = x2 + FFN(h) on the decode rows (static buffers)."""
        w = self.w
        F.skinny_gemm(h, self._mat(w.wgu[i]), acc)
        F.skinny_finalize(acc, act, swiglu=True)
        if self._push_for(h.shape[0]):
            F.skinny_gemm(act, self._mat(w.wd[i]), acc)
            self.tp.push_reduce(acc, x, res=x2)
        elif self.tp is None:
            F.skinny_gemm(act, self._mat(w.wd[i]), acc)
            F.skinny_finalize(acc, x, res=x2)
        else:
            racc = self.tp.reduce_gemm(act, self._mat(w.wd[i]), 2 * i + 1)
            F.skinny_finalize(racc, x, res=x2, wait=self._tp_wait())

    def _bucket(self, B: int) -> int:
        for s in (1, 2, 4, 8, 16, 32, 64):
            if B <= s and s <= self.max_batch:
                return s
        return self.max_batch

    @torch.no_grad()
    def capture(self, B: int, want_logits: bool = False) -> None:
        """Captures the decode step for batch bucket B as a CUDA graph (the
        variant with want_logits also copies the fp32 logits out)."""
        key = (B, want_logits)
        if self.device.type != "cuda" or key in self._graphs:
            return
        self._want_logits = want_logits
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(2):  # warm up allocations and tensor maps outside the graph
                self._step_body(B)
        torch.cuda.current_stream(self.device).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        # thread_local: the serving engine captures on its worker thread while
        # other threads may still issue CUDA calls
        with torch.cuda.graph(g, capture_error_mode="thread_local"):
            self._step_body(B)
        self._graphs[key] = g
        self._want_logits = False

    @torch.no_grad()
    def decode_step(self, tokens: torch.Tensor, pos: torch.Tensor, slots: torch.Tensor | None = None,
                    use_graph: bool = True, want_logits: bool = False) -> torch.Tensor:
        """tokens [B] at positions pos [B] (0-based) -> greedy next tokens [B]
        (device tensor, valid until the next call). With want_logits the fp32
        logits of the step are left in ``self.buf["logits"][:B]``."""
        B = tokens.shape[0]
        Bb = self._bucket(B)
        b = self.buf
        b["tok"][:B].copy_(tokens, non_blocking=True)
        b["pos"][:B].copy_(pos, non_blocking=True)
        b["seqlen"][:B].copy_(pos + 1, non_blocking=True)
        if slots is not None:
            b["slot"][:B].copy_(slots, non_blocking=True)
        if Bb > B:  # padded rows decode into spare slots and are ignored
            b["tok"][B:Bb].zero_()
            b["pos"][B:Bb].zero_()
            b["seqlen"][B:Bb].fill_(1)
            b["slot"][B:Bb].fill_(self.scratch_slot)
        if use_graph and self.device.type == "cuda":
            if (Bb, want_logits) not in self._graphs:
                self.capture(Bb, want_logits)
            self._graphs[(Bb, want_logits)].replay()
        else:
            self._want_logits = want_logits
            self._step_body(Bb)
            self._want_logits = False
        return b["next"][:B]

    @torch.no_grad()
    def generate(self, prompts: torch.Tensor, max_new_tokens: int, use_graph: bool = True) -> torch.Tensor:
        """Greedy generation for B equal-length prompts [B, S] -> [B, max_new_tokens]."""
        B, S = prompts.shape
        assert B <= self.max_batch and S + max_new_tokens <= self.max_seq
        out = torch.empty(B, max_new_tokens, dtype=torch.long, device=self.device)
        if self.paged:
            for r in range(B):
                self.cache.release(r)
                self.cache.ensure(r, S + max_new_tokens)
        nxt = self.prefill(prompts)
        out[:, 0] = nxt
        pos = torch.full((B,), S, dtype=torch.int32, device=self.device)
        slots = torch.arange(B, dtype=torch.int32, device=self.device)
        tok = nxt
        for t in range(1, max_new_tokens):
            tok = self.decode_step(tok, pos, slots, use_graph=use_graph).clone()
            out[:, t] = tok
            pos += 1
        return out

    @torch.no_grad()
    def reference_logits(self, tokens: torch.Tensor) -> torch.Tensor:
        """fp32 eager forward of [B, S] tokens (no cache) for numerics checks."""
        cfg, w = self.cfg, self.w
        B, S = tokens.shape
        D = cfg.head_dim
        x = w.embed.float()[tokens.to(self.device)]
        pos = torch.arange(S, device=self.device)
        for i in range(cfg.n_layers):
            h = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + cfg.norm_eps) * w.attn_norm[i].float()
            qkv = h @ self._mat(w.wqkv[i]).float().t()
            if w.bqkv[i] is not None:
                qkv = qkv + w.bqkv[i].float()
            if cfg.qk_norm:
                qkv = qkv.clone()
                for (h0, nh, wn) in ((0, self.hq, w.q_norm[i]), (self.hq, self.hkv, w.k_norm[i])):
                    v = qkv[..., h0 * D : (h0 + nh) * D].reshape(B, S, nh, D)
                    v = v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + cfg.norm_eps) * wn.float()
                    qkv[..., h0 * D : (h0 + nh) * D] = v.reshape(B, S, nh * D)
            qkv2 = qkv.reshape(B * S, -1)
            qkv2 = ref.rope(qkv2, pos.repeat(B), *self.rope_cs[i], self.hq + self.hkv, D)
            qkv = qkv2.view(B, S, -1)
            q = qkv[..., : self.hq * D].view(B, S, self.hq, D)
            k = qkv[..., self.hq * D : (self.hq + self.hkv) * D].view(B, S, self.hkv, D)
            v = qkv[..., (self.hq + self.hkv) * D :].view(B, S, self.hkv, D)
            o, _ = ref.attention(q, k, v, self.scale, True, 0, self.win[i], self.softcap)
            x = x + o.reshape(B, S, -1) @ self._mat(w.wo[i]).float().t()
            h = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + cfg.norm_eps) * w.mlp_norm[i].float()
            x = x + self._reference_ffn(i, h)
        h = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + cfg.norm_eps) * w.final_norm.float()
        assert w.lm_head is not None, "reference_logits needs the full LM head (a TP rank keeps only its slice)"
        return h @ w.lm_head.float().t()

    def _reference_ffn(self, i: int, h: torch.Tensor) -> torch.Tensor:
        w = self.w
        g, u = (h @ self._mat(w.wgu[i]).float().t()).chunk(2, -1)
        return (torch.nn.functional.silu(g) * u) @ self._mat(w.wd[i]).float().t()
