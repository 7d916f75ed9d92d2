"""The pipeline-parallel worker command line (one rank per process, the
reference's pp-qwen-worker / pp-qlora-worker): two gloo ranks on the CPU end
with the same per-epoch losses as the one-process run, and their parameter
checksums add up to the one-process checksum; the QLoRA form trains only its
adapters over a Q8_0 base."""
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


@pytest.mark.parametrize("extra", [(), ("--qlora", "q8_0")])
def test_two_ranks_reproduce_one_process(extra):
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
