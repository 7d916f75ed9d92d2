"""QLoRA over a GGUF-quantised Qwen / Llama base.

The base model comes straight from a llama.cpp GGUF file (architectures
qwen2, qwen3, llama, mistral). Its four projection groups per layer -- q/k/v
(fused rows), o, gate/up (fused rows), down -- stay on the device in the
file's own blocks (Q4_0, Q5_0, Q8_0, Q4_K, Q5_K, Q6_K, F16, BF16, F32; each
part keeps its own type, so a Q4_K_M file with Q6_K v / down rows works) and
are expanded to bf16 into one shared scratch buffer right before each GEMM,
forward and backward (csrc/gguf_dequant.cu). Embeddings, norms, q/k biases,
q/k norms and the LM head are small and held in bf16. LoRA adapters (rank r,
fp32 master in their own arena) train on top; the LM-head loss can run in
token chunks so no [tokens, vocab] logits tensor exists (Qwen's 152K vocab).
Any layer range / first / last selection builds one pipeline stage.

    m = qlora_from_gguf("qwen2.5-7b-q4_k_m.gguf", device="cuda", lora=LoRAConfig(rank=16))
    loss = m.loss(ids, targets); loss.backward(); FlatAdamW(m.arena).step()

Reference: the QLoRA stage over a GGUF base (trainer/src/qwen_qlora_stage.rs:
233-712: ``build(gguf_path, range, ...)`` with frozen quantised projections,
seven adapters per layer and a chunked LM-head loss). Here q/k/v and gate/up
are fused projections, so a layer has four adapted GEMMs covering the same
seven matrices.
"""
from __future__ import annotations

import numpy as np
import torch

from ..formats import gguf as G
from ..ops import functional as F
from .gpt import GPT, GPTConfig
from .lora import LoRAConfig, LoRAGPT

PROJ = ("wqkv", "wo", "wgu", "wd")


class GGUFPart:
    """Rows [r0, r0 + rows) of a fused projection: the file's blocks on the
    device (types the device decoder handles) or, for other types, the rows
    already expanded to bf16."""

    def __init__(self, g: G.GGUFFile, name: str, device):
        buf, dims, typ = g.raw(name)
        self.K, self.rows = int(dims[0]), int(np.prod(dims[1:])) if len(dims) > 1 else 1
        self.typ = typ
        dev = torch.device(device)
        if typ in F.GGUF_DEVICE_TYPES and (dev.type != "cuda" or self.K % 256 == 0 or typ not in (12, 13, 14)):
            self.blocks = torch.from_numpy(np.array(buf, dtype=np.uint8)).to(dev)
            self.dense = None
        else:
            self.blocks = None
            self.dense = g.tensor(name).to(dev)

    def expand_into(self, out: torch.Tensor) -> None:
        if self.blocks is not None:
            F.gguf_dequant(self.blocks, self.typ, self.rows, self.K, out)
        else:
            out.copy_(self.dense)

    @property
    def nbytes(self) -> int:
        return (self.blocks.numel() if self.blocks is not None else 2 * self.dense.numel())


class GGUFWeight:
    """A frozen [rows, K] projection made of row parts; ``bf16()`` expands all
    parts into the owner's shared scratch buffer (``scratch(n)``)."""

    def __init__(self, parts: list, scratch=None):
        self.parts = parts
        self.shape = (sum(p.rows for p in parts), parts[0].K)
        self.scratch = scratch

    def bf16(self) -> torch.Tensor:
        rows, K = self.shape
        out = self.scratch(rows * K).view(rows, K)
        r0 = 0
        for p in self.parts:
            p.expand_into(out[r0 : r0 + p.rows])
            r0 += p.rows
        return out

    @property
    def nbytes(self) -> int:
        return sum(p.nbytes for p in self.parts)


def config_from_gguf(g: G.GGUFFile, max_seq: int = 4096) -> GPTConfig:
    q = G.qwen_config_from_gguf(g)
    return GPTConfig(vocab=q.vocab, d_model=q.d_model, n_layers=q.n_layers, n_heads=q.n_heads,
                     n_kv_heads=q.n_kv_heads, d_ff=q.d_ff, max_seq=max_seq, rope_theta=q.rope_theta,
                     norm_eps=q.norm_eps, tie_embeddings=q.tie_embeddings, qk_norm=q.qk_norm,
                     qkv_bias=q.qkv_bias, head_dim_=q.head_dim if q.head_dim != q.d_model // q.n_heads else 0)


def qlora_from_gguf(path: str, device="cuda", lora: LoRAConfig = LoRAConfig(), seed: int = 0, layers=None,
                    first: bool = True, last: bool = True, max_seq: int = 4096, loss_chunk: int = 1024,
                    pad_multiple: int = 1, alloc=None) -> LoRAGPT:
    """LoRA adapters over the GGUF base at ``path`` (optionally one pipeline
    stage: ``layers``, ``first``, ``last``)."""
    g = G.GGUFFile(path)
    cfg = config_from_gguf(g, max_seq)
    base = GPT(cfg, device=device, seed=seed, layers=layers, first=first, last=last, external=frozenset(PROJ),
               loss_chunk=loss_chunk, pad_multiple=pad_multiple)
    a = base.arena
    names = set(a.names())

    def put(arena_name: str, *gguf_names: str) -> None:
        if arena_name in names:
            t = torch.cat([g.tensor(n, dtype=torch.float32).reshape(-1) for n in gguf_names])
            a.set_full(arena_name, t.view(a.slots[arena_name].shape))

    with torch.no_grad():
        put("tok_emb", "token_embd.weight")
        put("final_norm", "output_norm.weight")
        if not cfg.tie_embeddings:
            put("lm_head", "output.weight")
        for i in base.layers:
            p = f"blk.{i}."
            put(f"l{i}.attn_norm", p + "attn_norm.weight")
            put(f"l{i}.mlp_norm", p + "ffn_norm.weight")
            if cfg.qkv_bias:
                put(f"l{i}.bqkv", p + "attn_q.bias", p + "attn_k.bias", p + "attn_v.bias")
            if cfg.qk_norm:
                put(f"l{i}.q_norm", p + "attn_q_norm.weight")
                put(f"l{i}.k_norm", p + "attn_k_norm.weight")
        a.sync_bf16_from_master()
    dev = base.device
    weights = {}
    for i in base.layers:
        p = f"blk.{i}."
        parts = {
            "wqkv": [p + "attn_q.weight", p + "attn_k.weight", p + "attn_v.weight"],
            "wo": [p + "attn_output.weight"],
            "wgu": [p + "ffn_gate.weight", p + "ffn_up.weight"],
            "wd": [p + "ffn_down.weight"],
        }
        for t, ns in parts.items():
            weights[(i, t)] = GGUFWeight([GGUFPart(g, n, dev) for n in ns])
            assert weights[(i, t)].shape == tuple(base.external_shapes[f"l{i}.{t}"]), (i, t)
    m = LoRAGPT(base, lora, seed=seed + 1, weights=weights, pad_multiple=pad_multiple, alloc=alloc)
    m.gguf_path = path
    m.base_bytes = sum(w.nbytes for w in weights.values())
    return m
