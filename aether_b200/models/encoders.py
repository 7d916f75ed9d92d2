"""Encoder models for the embedding routes: BERT/BGE sentence embeddings and a
DINOv3-style ViT-L/16 image backbone (inference).

Reference: BertSession (runtime/src/bert.rs -- post-LN BERT encoder, GELU,
CLS pooling, L2-normalised output, synthetic-weights constructor) and the
DINOv3 ViT-L/16 session (runtime/src/vit.rs -- tokens [CLS, 4 registers,
patches], pre-LN blocks with LayerScale, no q/k/v bias, 2-D axial RoPE on patch
tokens only, final LayerNorm, L2-normalised CLS).

Every dense op runs on this library's kernels (tcgen05 GEMM with fused bias /
residual epilogues, LayerNorm with fused residual, GELU, flash attention).
LayerScale is folded into the output projections at construction
(W' = diag(ls) W, b' = ls * b), which is the same function with one op less.
Weights are random-init (N(0, 0.02)) or provided as tensors by the caller.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from ..ops import functional as F


def _rnd(gen, *shape, std=0.02, device="cpu"):
    return (torch.randn(*shape, generator=gen) * std).to(device=device, dtype=torch.bfloat16)


# ---------------------------------------------------------------------------- BERT
@dataclass
class BertConfig:
    vocab: int = 30522
    d_model: int = 1024
    n_layers: int = 24
    n_heads: int = 16
    d_ff: int = 4096
    max_pos: int = 512
    type_vocab: int = 2
    eps: float = 1e-12

    @staticmethod
    def bge_large() -> "BertConfig":
        return BertConfig()

    @staticmethod
    def bge_small() -> "BertConfig":
        return BertConfig(d_model=384, n_layers=12, n_heads=12, d_ff=1536)


class BertEncoder:
    def __init__(self, cfg: BertConfig, device="cuda", seed: int = 0, name: str = "bge-large-synthetic"):
        self.cfg, self.device, self.name = cfg, torch.device(device), name
        g = torch.Generator().manual_seed(seed)
        d, f = cfg.d_model, cfg.d_ff
        dev = self.device
        self.word = _rnd(g, cfg.vocab, d, device=dev)
        self.pos = _rnd(g, cfg.max_pos, d, device=dev)
        self.typ = _rnd(g, cfg.type_vocab, d, device=dev)
        ones = lambda: torch.ones(d, dtype=torch.bfloat16, device=dev)  # noqa: E731
        zeros = lambda n=d: torch.zeros(n, dtype=torch.bfloat16, device=dev)  # noqa: E731
        self.emb_g, self.emb_b = ones(), zeros()
        self.layers = []
        for _ in range(cfg.n_layers):
            self.layers.append(dict(
                wqkv=_rnd(g, 3 * d, d, device=dev), bqkv=zeros(3 * d), wo=_rnd(g, d, d, device=dev), bo=zeros(),
                ln1_g=ones(), ln1_b=zeros(), w1=_rnd(g, f, d, device=dev), b1=zeros(f), w2=_rnd(g, d, f, device=dev),
                b2=zeros(), ln2_g=ones(), ln2_b=zeros()))

    @torch.no_grad()
    def hidden(self, ids: torch.Tensor, types: torch.Tensor | None = None) -> torch.Tensor:
        """ids [S] (one sequence) -> final hidden states [S, d] (bf16)."""
        cfg = self.cfg
        S = ids.shape[0]
        d, H = cfg.d_model, cfg.n_heads
        D = d // H
        ids = ids.to(self.device)
        types = torch.zeros_like(ids) if types is None else types.to(self.device)
        x = F.embedding(self.word, ids) + self.pos[:S] + F.embedding(self.typ, types)
        x, _, _, _ = F.layernorm(x.contiguous(), self.emb_g, self.emb_b, cfg.eps)
        for L in self.layers:
            qkv = F.gemm(x, L["wqkv"], bias=L["bqkv"])
            q = qkv.view(1, S, 3 * d)[:, :, :d].view(1, S, H, D)
            k = qkv.view(1, S, 3 * d)[:, :, d : 2 * d].view(1, S, H, D)
            v = qkv.view(1, S, 3 * d)[:, :, 2 * d :].view(1, S, H, D)
            o, _ = F.attention(q, k, v, 1.0 / math.sqrt(D), causal=False, want_lse=False)
            y = F.gemm(o.view(S, d), L["wo"], bias=L["bo"])
            x, _, _, _ = F.layernorm(y, L["ln1_g"], L["ln1_b"], cfg.eps, res=x)  # post-LN: LN(x + attn)
            h = F.gelu(F.gemm(x, L["w1"], bias=L["b1"]))
            y = F.gemm(h, L["w2"], bias=L["b2"])
            x, _, _, _ = F.layernorm(y, L["ln2_g"], L["ln2_b"], cfg.eps, res=x)
        return x

    @torch.no_grad()
    def embed(self, ids: torch.Tensor) -> torch.Tensor:
        """CLS pooling + L2 normalisation -> fp32 [d]."""
        cls = self.hidden(ids)[0].float()
        return cls / cls.norm().clamp(min=1e-12)


class TextEmbedder:
    """Tokenise -> [CLS] ids [SEP] -> BertEncoder.embed, for /v1/embeddings."""

    def __init__(self, encoder: BertEncoder, tokenizer, cls_id: int = 101, sep_id: int = 102):
        self.enc, self.tok, self.cls_id, self.sep_id = encoder, tokenizer, cls_id, sep_id
        self.name = encoder.name

    def embed_texts(self, texts: list) -> list:
        out = []
        for t in texts:
            ids = [self.cls_id] + [i % self.enc.cfg.vocab for i in self.tok.encode(t)][: self.enc.cfg.max_pos - 2]
            ids.append(self.sep_id)
            out.append(self.enc.embed(torch.tensor(ids, dtype=torch.long)).tolist())
        return out


# ---------------------------------------------------------------------------- ViT
@dataclass
class VitConfig:
    d: int = 1024
    n_layers: int = 24
    n_heads: int = 16
    d_ff: int = 4096
    patch: int = 16
    img: int = 224
    n_reg: int = 4
    eps: float = 1e-5
    rope_theta: float = 100.0

    @property
    def grid(self) -> int:
        return self.img // self.patch

    @property
    def n_patches(self) -> int:
        return self.grid * self.grid

    @property
    def seq(self) -> int:
        return 1 + self.n_reg + self.n_patches

    @staticmethod
    def vitl16() -> "VitConfig":
        return VitConfig()


def axial_rope_tables(cfg: VitConfig, device) -> tuple:
    """cos/sin [n_patches, head_dim/2] for the half-split rotation: the first
    quarter of each head's dims turns with the patch row, the second with the
    column (coordinates centred on the grid and scaled to [-1, 1])."""
    D = cfg.d // cfg.n_heads
    q = D // 4
    freqs = cfg.rope_theta ** (-torch.arange(q, dtype=torch.float64) / q)
    coords = (torch.arange(cfg.grid, dtype=torch.float64) + 0.5) / cfg.grid * 2 - 1
    yy, xx = torch.meshgrid(coords, coords, indexing="ij")
    ang = torch.cat([yy.reshape(-1, 1) * freqs * math.pi, xx.reshape(-1, 1) * freqs * math.pi], dim=1)  # [P, D/2]
    return ang.cos().float().to(device).contiguous(), ang.sin().float().to(device).contiguous()


class VitEncoder:
    def __init__(self, cfg: VitConfig, device="cuda", seed: int = 0, name: str = "dinov3-vitl16-synthetic"):
        self.cfg, self.device, self.name = cfg, torch.device(device), name
        g = torch.Generator().manual_seed(seed)
        d, f = cfg.d, cfg.d_ff
        dev = self.device
        pin = 3 * cfg.patch * cfg.patch
        self.patch_w = _rnd(g, d, pin, device=dev)
        self.patch_b = torch.zeros(d, dtype=torch.bfloat16, device=dev)
        self.cls = _rnd(g, 1, d, device=dev)
        self.reg = _rnd(g, cfg.n_reg, d, device=dev)
        ones = lambda: torch.ones(d, dtype=torch.bfloat16, device=dev)  # noqa: E731
        zeros = lambda n=d: torch.zeros(n, dtype=torch.bfloat16, device=dev)  # noqa: E731
        self.layers = []
        for _ in range(cfg.n_layers):
            ls1 = torch.full((d,), 1e-1)
            ls2 = torch.full((d,), 1e-1)
            wo = (torch.randn(d, d, generator=g) * 0.02) * ls1[:, None]
            w2 = (torch.randn(d, f, generator=g) * 0.02) * ls2[:, None]
            self.layers.append(dict(
                n1_g=ones(), n1_b=zeros(), wqkv=_rnd(g, 3 * d, d, device=dev),
                wo=wo.to(dev, torch.bfloat16), bo=zeros(),  # LayerScale folded in
                n2_g=ones(), n2_b=zeros(), w1=_rnd(g, f, d, device=dev), b1=zeros(f),
                w2=w2.to(dev, torch.bfloat16), b2=zeros()))
        self.norm_g, self.norm_b = ones(), zeros()
        self.cos, self.sin = axial_rope_tables(cfg, dev)
        self.patch_pos = torch.arange(cfg.n_patches, dtype=torch.int32, device=dev)

    def patchify(self, img: torch.Tensor) -> torch.Tensor:
        """img [3, H, W] float -> [n_patches, 3*p*p] bf16 (channel-major per patch)."""
        p = self.cfg.patch
        x = img.to(self.device, torch.float32).unfold(1, p, p).unfold(2, p, p)  # [3, gh, gw, p, p]
        return x.permute(1, 2, 0, 3, 4).reshape(-1, 3 * p * p).to(torch.bfloat16).contiguous()

    @torch.no_grad()
    def forward(self, img: torch.Tensor) -> torch.Tensor:
        """img [3, img, img] -> final tokens [seq, d] (bf16)."""
        cfg = self.cfg
        d, H = cfg.d, cfg.n_heads
        D = d // H
        S = cfg.seq
        P = cfg.n_patches
        patches = F.gemm(self.patchify(img), self.patch_w, bias=self.patch_b)
        x = torch.cat([self.cls, self.reg, patches], dim=0).contiguous()
        npre = 1 + cfg.n_reg
        for L in self.layers:
            h, _, _, _ = F.layernorm(x, L["n1_g"], L["n1_b"], cfg.eps)
            qkv = F.gemm(h, L["wqkv"])
            F.rope_(qkv[npre:], self.patch_pos, self.cos, self.sin, 2 * H, D)  # q and k heads of patch tokens
            q = qkv.view(1, S, 3 * d)[:, :, :d].view(1, S, H, D)
            k = qkv.view(1, S, 3 * d)[:, :, d : 2 * d].view(1, S, H, D)
            v = qkv.view(1, S, 3 * d)[:, :, 2 * d :].view(1, S, H, D)
            o, _ = F.attention(q, k, v, 1.0 / math.sqrt(D), causal=False, want_lse=False)
            x = F.gemm(o.view(S, d), L["wo"], bias=L["bo"], residual=x)
            h, _, _, _ = F.layernorm(x, L["n2_g"], L["n2_b"], cfg.eps)
            a = F.gelu(F.gemm(h, L["w1"], bias=L["b1"]))
            x = F.gemm(a, L["w2"], bias=L["b2"], residual=x)
        x, _, _, _ = F.layernorm(x, self.norm_g, self.norm_b, cfg.eps)
        assert x.shape[0] == S and P == S - npre
        return x

    @torch.no_grad()
    def embed(self, img: torch.Tensor) -> torch.Tensor:
        cls = self.forward(img)[0].float()
        return cls / cls.norm().clamp(min=1e-12)
