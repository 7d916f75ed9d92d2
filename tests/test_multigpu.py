"""Multi-GPU paths (NVLink symmetric memory): run as child processes via
torchrun on 2+ GPUs; skipped with fewer. Host-side DP logic is also tested on
CPU gloo ranks (world 2)."""
import os
import socket
import subprocess
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.gpu
def test_multigpu_nvlink_paths():
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 GPUs")
    n = min(n, 8)
    env = dict(os.environ)
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nproc-per-node", str(n),
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(ROOT, "tests", "multigpu_worker.py")]
    out = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT)
    assert out.returncode == 0, out.stdout[-4000:] + out.stderr[-4000:]
    assert out.stdout.count("OK ") >= 10 * n


def _gloo_dp_worker(rank, world, port, q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    sys.path.insert(0, ROOT)
    from aether_b200.models.gpt import GPT, GPTConfig
    from aether_b200.parallel import dist as D
    from aether_b200.train import Trainer

    info = D.init(device="cpu", timeout_s=60)
    cfg = GPTConfig(vocab=128, d_model=64, n_layers=1, n_heads=2, n_kv_heads=2, d_ff=128, max_seq=16)
    m = GPT(cfg, device="cpu", seed=0, pad_multiple=world)
    tr = Trainer(m, info, lr=1e-2, weight_decay=0.0, micro_batch=2)
    toks = torch.randint(0, 128, (2, 17), generator=torch.Generator().manual_seed(rank))
    for _ in range(3):
        tr.train_step(toks)
    q.put((rank, m.arena.bf16.float().sum().item(), m.arena.master.sum().item()))
    D.shutdown()


def test_gloo_dp_ranks_stay_in_sync():
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_gloo_dp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=120)
    res = sorted(q.get(timeout=10) for _ in range(2))
    assert all(p.exitcode == 0 for p in ps)
    assert abs(res[0][1] - res[1][1]) < 1e-3, res  # identical bf16 compute copies after all-gather
