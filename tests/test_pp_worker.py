"""The pipeline-parallel worker command line (one rank per process, the
reference's pp-qwen-worker / pp-qlora-worker): two gloo ranks on the CPU end
with the same per-epoch losses as the one-process run, and their parameter
checksums add up to the one-process checksum; the QLoRA form trains only its
adapters over a Q8_0 base, or over a GGUF model file's quantised layers."""
import os
import re
import socket
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(rank, world, port, extra=()):
    env = dict(os.environ, PYTHONPATH=ROOT)
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MASTER_ADDR", "MASTER_PORT"):
        env.pop(k, None)
    cmd = [sys.executable, "-m", "aether_b200.pp_worker", "--rank", str(rank), "--world-size", str(world), "--layers",
           "4", "--epochs", "3", "--device", "cpu", "--base-port", str(port), *extra]
    return subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True, env=env, cwd=ROOT)


def _parse(out):
    epochs = [float(x) for x in re.findall(r"^EPOCH \d+ (\S+)$", out, re.M)]
    sums = [float(x) for x in re.findall(r"^CHECKSUM .* value=(\S+)$", out, re.M)]
    return epochs, sums


def _tiny_gguf(path):
    """A 4-layer Qwen2-architecture GGUF with mixed Q8_0 / Q4_0 / F16 projections."""
    import torch

    from aether_b200.formats import gguf as G

    V, D, H, HKV, FF = 512, 128, 2, 1, 256
    g = torch.Generator().manual_seed(7)
    rnd = lambda *sh: torch.randn(*sh, generator=g) * 0.05  # noqa: E731
    hd = D // H
    t = {"token_embd.weight": (rnd(V, D), G.F16), "output_norm.weight": (1 + 0.1 * rnd(D), G.F32)}
    for i in range(4):
        p = f"blk.{i}."
        t.update({p + "attn_norm.weight": (1 + 0.1 * rnd(D), G.F32), p + "ffn_norm.weight": (1 + 0.1 * rnd(D), G.F32),
                  p + "attn_q.weight": (rnd(H * hd, D), G.Q8_0), p + "attn_k.weight": (rnd(HKV * hd, D), G.Q4_0),
                  p + "attn_v.weight": (rnd(HKV * hd, D), G.F16), p + "attn_q.bias": (rnd(H * hd), G.F32),
                  p + "attn_k.bias": (rnd(HKV * hd), G.F32), p + "attn_v.bias": (rnd(HKV * hd), G.F32),
                  p + "attn_output.weight": (rnd(D, H * hd), G.Q8_0), p + "ffn_gate.weight": (rnd(FF, D), G.Q4_0),
                  p + "ffn_up.weight": (rnd(FF, D), G.Q8_0), p + "ffn_down.weight": (rnd(D, FF), G.F16)})
    meta = {"general.architecture": "qwen2", "qwen2.embedding_length": D, "qwen2.block_count": 4,
            "qwen2.attention.head_count": H, "qwen2.attention.head_count_kv": HKV, "qwen2.feed_forward_length": FF,
            "qwen2.rope.freq_base": 1e6, "qwen2.attention.layer_norm_rms_epsilon": 1e-6,
            "tokenizer.ggml.tokens": [f"t{i}" for i in range(V)]}
    G.write_gguf(path, meta, t)
    return path


@pytest.mark.parametrize("extra", [(), ("--qlora", "q8_0"), ("--gguf", "GGUF")])
def test_two_ranks_reproduce_one_process(extra, tmp_path):
    if "GGUF" in extra:
        extra = ("--gguf", _tiny_gguf(str(tmp_path / "tiny.gguf")))
    one = _run(0, 1, _free_port(), extra)
    o1, e1 = one.communicate(timeout=600)
    assert one.returncode == 0, e1[-3000:]
    ep1, sum1 = _parse(o1)
    port = _free_port()
    ps = [_run(r, 2, port, extra) for r in range(2)]
    outs = [p.communicate(timeout=600) for p in ps]
    for p, (o, e) in zip(ps, outs):
        assert p.returncode == 0, e[-3000:]
    ep2, _ = _parse(outs[1][0])
    s2 = sum(_parse(o)[1][0] for o, _ in outs)
    assert len(ep1) == 3 and ep2 == ep1, (ep1, ep2)
    assert abs(s2 - sum1[0]) <= 1e-9 * abs(sum1[0]), (s2, sum1)
    assert "RESULT rank=1 world=2" in outs[1][0]
