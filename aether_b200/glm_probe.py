"""GGUF model probe: open a GGUF file, print the model configuration it maps
to, check that this package's kernels support its geometry, and exit without
loading any tensor to the device.

    python -m aether_b200.glm_probe <model.gguf>

For the ``deepseek2`` family (DeepSeek-V2, GLM-4.7-flash: multi-head latent
attention) the check is the absorbed-MLA kernel's geometry: a 512 + 64 =
576-wide latent row (kv_lora_rank + qk_rope) and value heads of at most 128;
for Qwen / Llama / Mistral it is the attention kernels' head_dim 128 (64 on
the mma.sync path) and a GQA group of at most 8. Exit 0 when supported, 1 when
the geometry is not, 2 for a usage error, 3 when the file cannot be read.

Reference: trainer/src/bin/glm_probe.rs (open, dump ModelConfig, apply the
session's head_dim guard, exit before any upload).
"""
from __future__ import annotations

import dataclasses
import sys


def probe(path: str) -> int:
    from .formats import gguf as G

    try:
        g = G.GGUFFile(path)
    except Exception as e:  # noqa: BLE001 - any unreadable file is reported the same way
        print(f"[glm-probe] cannot open {path}: {e}", file=sys.stderr)
        return 3
    arch = g.meta.get("general.architecture", "?")
    print(f"[glm-probe] opened: {path}")
    print(f"[glm-probe] arch              = {arch}")
    print(f"[glm-probe] tensors           = {len(g.tensors)}")
    problems = []
    if arch in ("deepseek2", "glm4moe", "deepseek"):
        cfg = G.deepseek_config_from_gguf(g)
        for f in dataclasses.fields(cfg):
            print(f"[glm-probe] {f.name:<18}= {getattr(cfg, f.name)}")
        latent = cfg.kv_lora_rank + cfg.qk_rope
        print(f"[glm-probe] mla latent width  = {latent} (absorbed kernel: 576)")
        if latent != 576:
            problems.append(f"latent row {latent} != 576 (kv_lora_rank 512 + rope 64)")
        if cfg.v_head > 128:
            problems.append(f"value head {cfg.v_head} > 128")
    else:
        cfg = G.qwen_config_from_gguf(g)
        for f in dataclasses.fields(cfg):
            print(f"[glm-probe] {f.name:<18}= {getattr(cfg, f.name)}")
        D = cfg.head_dim
        if D not in (64, 128):
            problems.append(f"head_dim {D} (attention kernels take 64 or 128)")
        if cfg.n_heads % cfg.n_kv_heads or cfg.n_heads // cfg.n_kv_heads > 8:
            problems.append(f"GQA group {cfg.n_heads}/{cfg.n_kv_heads} (at most 8 query heads per KV head)")
    if problems:
        for p in problems:
            print(f"[glm-probe] UNSUPPORTED: {p}")
        return 1
    print("[glm-probe] geometry supported; no tensors were loaded")
    return 0


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    if len(argv) != 1:
        print("usage: python -m aether_b200.glm_probe <model.gguf>", file=sys.stderr)
        return 2
    return probe(argv[0])


if __name__ == "__main__":
    sys.exit(main())
