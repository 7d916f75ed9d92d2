"""The GGUF probe command line: metadata-only inspection of a deepseek2 (MLA)
and a qwen2 GGUF, the kernel-geometry verdict in the exit code, and the
usage / unreadable-file codes."""
import os
import subprocess
import sys

import torch

from aether_b200.formats import gguf as G

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _probe(*args):
    env = dict(os.environ, PYTHONPATH=ROOT)
    return subprocess.run([sys.executable, "-m", "aether_b200.glm_probe", *args], capture_output=True, text=True,
                          env=env, timeout=120)


def test_probe_reports_mla_geometry(tmp_path):
    a = "deepseek2."
    meta = {"general.architecture": "deepseek2", a + "block_count": 2, a + "embedding_length": 128,
            a + "feed_forward_length": 256, a + "attention.head_count": 4, a + "attention.kv_lora_rank": 512,
            a + "attention.key_length": 192, a + "attention.value_length": 128, a + "rope.dimension_count": 64,
            a + "expert_count": 8, a + "expert_used_count": 2, a + "expert_feed_forward_length": 64,
            "tokenizer.ggml.tokens": [f"t{i}" for i in range(64)]}
    p = str(tmp_path / "glm.gguf")
    G.write_gguf(p, meta, {"token_embd.weight": (torch.zeros(64, 128), G.F32)})
    r = _probe(p)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "kv_lora_rank      = 512" in r.stdout and "mla latent width  = 576" in r.stdout
    meta[a + "attention.kv_lora_rank"] = 256  # a latent row the absorbed kernel does not take
    G.write_gguf(p, meta, {"token_embd.weight": (torch.zeros(64, 128), G.F32)})
    r = _probe(p)
    assert r.returncode == 1 and "UNSUPPORTED" in r.stdout


def test_probe_qwen_and_errors(tmp_path):
    meta = {"general.architecture": "qwen2", "qwen2.embedding_length": 256, "qwen2.block_count": 2,
            "qwen2.attention.head_count": 2, "qwen2.attention.head_count_kv": 1, "qwen2.feed_forward_length": 512,
            "tokenizer.ggml.tokens": [f"t{i}" for i in range(64)]}
    p = str(tmp_path / "q.gguf")
    G.write_gguf(p, meta, {"token_embd.weight": (torch.zeros(64, 256), G.F32)})
    r = _probe(p)
    assert r.returncode == 0 and "head_dim" in r.stdout, r.stdout + r.stderr
    assert _probe().returncode == 2
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"not a gguf file")
    assert _probe(str(bad)).returncode == 3
