"""Hugging Face checkpoint directory (config.json + *.safetensors, optionally
sharded with model.safetensors.index.json) -> QwenWeights.

Reference: the multi-file safetensors loader and HF-name mapping
(runtime/src/lib.rs:9063-9153; runtime/src/serving.rs:459-560, config from
config.json). Tensors are read with this package's own safetensors reader and
fused on load into the layouts the kernels use: q/k/v stacked into one
[(Hq+2Hkv)*D, d] matrix (one GEMM), gate/up stacked into [2F, d].
"""
from __future__ import annotations

import json
import os

import torch

from . import safetensors as st


def qwen_config_from_hf(cfg_json: dict):
    from ..models.qwen import QwenConfig

    d, H = cfg_json["hidden_size"], cfg_json["num_attention_heads"]
    hd = int(cfg_json.get("head_dim") or d // H)
    return QwenConfig(vocab=cfg_json["vocab_size"], d_model=d, n_layers=cfg_json["num_hidden_layers"], n_heads=H,
                      n_kv_heads=cfg_json.get("num_key_value_heads", H), d_ff=cfg_json["intermediate_size"],
                      rope_theta=float(cfg_json.get("rope_theta", 1e6)),
                      norm_eps=float(cfg_json.get("rms_norm_eps", 1e-6)),
                      tie_embeddings=bool(cfg_json.get("tie_word_embeddings", False)),
                      qkv_bias=True, max_seq=int(cfg_json.get("max_position_embeddings", 4096)),
                      head_dim_=hd if hd != d // H else 0)


def _all_tensors(path: str) -> dict:
    idx = os.path.join(path, "model.safetensors.index.json")
    if os.path.exists(idx):
        files = sorted(set(json.load(open(idx))["weight_map"].values()))
    else:
        files = sorted(f for f in os.listdir(path) if f.endswith(".safetensors"))
    out = {}
    for f in files:
        out.update(st.load_file(os.path.join(path, f)))
    return out


def load_qwen_hf(path: str, device="cuda"):
    from ..models.qwen import QwenWeights

    cfg = qwen_config_from_hf(json.load(open(os.path.join(path, "config.json"))))
    t = _all_tensors(path)
    cfg.qkv_bias = "model.layers.0.self_attn.q_proj.bias" in t
    cfg.qk_norm = "model.layers.0.self_attn.q_norm.weight" in t
    g = lambda n: t[n].to(device=device, dtype=torch.bfloat16).contiguous()  # noqa: E731
    w = QwenWeights.__new__(QwenWeights)
    w.cfg, w.device, w.tp_rank, w.tp_size = cfg, torch.device(device), 0, 1
    w.hq, w.hkv, w.f = cfg.n_heads, cfg.n_kv_heads, cfg.d_ff
    w.embed = g("model.embed_tokens.weight")
    w.lm_head = w.embed if cfg.tie_embeddings or "lm_head.weight" not in t else g("lm_head.weight")
    w.final_norm = g("model.norm.weight")
    w.attn_norm, w.mlp_norm, w.wqkv, w.bqkv, w.wo, w.wgu, w.wd = [], [], [], [], [], [], []
    w.q_norm = [] if cfg.qk_norm else None
    w.k_norm = [] if cfg.qk_norm else None
    for i in range(cfg.n_layers):
        p = f"model.layers.{i}."
        a = p + "self_attn."
        if cfg.qk_norm:
            w.q_norm.append(g(a + "q_norm.weight"))
            w.k_norm.append(g(a + "k_norm.weight"))
        w.attn_norm.append(g(p + "input_layernorm.weight"))
        w.mlp_norm.append(g(p + "post_attention_layernorm.weight"))
        w.wqkv.append(torch.cat([g(a + "q_proj.weight"), g(a + "k_proj.weight"), g(a + "v_proj.weight")]).contiguous())
        w.bqkv.append(torch.cat([g(a + "q_proj.bias"), g(a + "k_proj.bias"), g(a + "v_proj.bias")]).contiguous()
                      if cfg.qkv_bias else None)
        w.wo.append(g(a + "o_proj.weight"))
        m = p + "mlp."
        w.wgu.append(torch.cat([g(m + "gate_proj.weight"), g(m + "up_proj.weight")]).contiguous())
        w.wd.append(g(m + "down_proj.weight"))
    return cfg, w


def save_qwen_hf(cfg, w, path: str) -> None:
    """Inverse of ``load_qwen_hf`` for a TP=1 QwenWeights (exports and tests)."""
    os.makedirs(path, exist_ok=True)
    D = cfg.head_dim
    q, kv = cfg.n_heads * D, cfg.n_kv_heads * D
    t = {"model.embed_tokens.weight": w.embed, "model.norm.weight": w.final_norm}
    if not cfg.tie_embeddings:
        t["lm_head.weight"] = w.lm_head
    for i in range(cfg.n_layers):
        p = f"model.layers.{i}."
        a = p + "self_attn."
        t[p + "input_layernorm.weight"] = w.attn_norm[i]
        t[p + "post_attention_layernorm.weight"] = w.mlp_norm[i]
        t[a + "q_proj.weight"], t[a + "k_proj.weight"], t[a + "v_proj.weight"] = w.wqkv[i].split([q, kv, kv])
        if w.bqkv[i] is not None:
            t[a + "q_proj.bias"], t[a + "k_proj.bias"], t[a + "v_proj.bias"] = w.bqkv[i].split([q, kv, kv])
        t[a + "o_proj.weight"] = w.wo[i]
        t[p + "mlp.gate_proj.weight"], t[p + "mlp.up_proj.weight"] = w.wgu[i].split([cfg.d_ff, cfg.d_ff])
        t[p + "mlp.down_proj.weight"] = w.wd[i]
        if cfg.qk_norm:
            t[a + "q_norm.weight"], t[a + "k_norm.weight"] = w.q_norm[i], w.k_norm[i]
    st.save_file(t, os.path.join(path, "model.safetensors"), metadata={"format": "pt"})
    json.dump({"vocab_size": cfg.vocab, "hidden_size": cfg.d_model, "num_hidden_layers": cfg.n_layers,
               "num_attention_heads": cfg.n_heads, "num_key_value_heads": cfg.n_kv_heads,
               "intermediate_size": cfg.d_ff, "rope_theta": cfg.rope_theta, "rms_norm_eps": cfg.norm_eps,
               "tie_word_embeddings": cfg.tie_embeddings, "max_position_embeddings": cfg.max_seq,
               "head_dim": cfg.head_dim,
               "architectures": ["Qwen2ForCausalLM"]}, open(os.path.join(path, "config.json"), "w"))
