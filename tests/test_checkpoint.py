"""Checkpoint / resume: training N steps straight and training k steps, saving,
rebuilding everything from scratch, loading and training N-k more give
bit-identical parameters and optimiser state (single process, and two gloo DP
ranks resumed on one)."""
import os
import socket
import sys

import torch

from aether_b200 import checkpoint
from aether_b200.models.gpt import GPT, GPTConfig
from aether_b200.parallel import dist as D
from aether_b200.train import Trainer

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TINY = dict(vocab=128, d_model=64, n_layers=2, n_heads=2, n_kv_heads=2, d_ff=128, max_seq=32)


def _tokens(step, rank=0):
    return torch.randint(0, 128, (2, 17), generator=torch.Generator().manual_seed(1000 * rank + step))


def _trainer(info=None, pad=1):
    m = GPT(GPTConfig(**TINY), device="cpu", seed=2, pad_multiple=pad)
    return Trainer(m, info or D.DistInfo(), lr=3e-3, weight_decay=0.1, micro_batch=2, warmup_steps=2, total_steps=6)


def test_resume_is_bitwise(tmp_path):
    a = _trainer()
    for s in range(5):
        a.train_step(_tokens(s))
    b = _trainer()
    for s in range(2):
        b.train_step(_tokens(s))
    checkpoint.save(str(tmp_path), b.model.arena, b.dp, step=b.step_idx)
    c = _trainer()
    c.step_idx = checkpoint.load(str(tmp_path), c.model.arena, c.dp)
    assert c.step_idx == 2
    for s in range(2, 5):
        c.train_step(_tokens(s))
    assert torch.equal(a.model.arena.master, c.model.arena.master)
    assert torch.equal(a.model.arena.bf16, c.model.arena.bf16)
    assert torch.equal(a.dp.opt.m, c.dp.opt.m) and torch.equal(a.dp.opt.v, c.dp.opt.v)
    assert a.dp.opt.step_count == c.dp.opt.step_count == 5


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _dp_worker(rank, world, port, path, q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    sys.path.insert(0, ROOT)
    from aether_b200 import checkpoint as ck
    from aether_b200.parallel import dist as Dd

    info = Dd.init(device="cpu", timeout_s=60)
    t = _trainer(info, pad=world)
    for s in range(2):
        t.train_step(_tokens(s, rank))
    ck.save(path, t.model.arena, t.dp, step=t.step_idx, rank=rank, world=world)
    Dd.barrier()
    q.put((rank, t.model.arena.master.numpy().copy()))
    Dd.shutdown()


def test_dp_checkpoint_reshards_to_one_rank(tmp_path):
    """Two gloo ranks save their ZeRO-1 shards; one process loads both and
    holds the full master / moments the two ranks held together."""
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    path = str(tmp_path / "ck")
    ps = [ctx.Process(target=_dp_worker, args=(r, 2, port, path, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    one = _trainer(pad=2)
    assert checkpoint.load(path, one.model.arena, one.dp) == 2
    n = one.model.arena.numel // 2
    # rank r's master is authoritative on its own shard
    assert torch.equal(one.model.arena.master[:n], torch.from_numpy(got[0][:n]))
    assert torch.equal(one.model.arena.master[n:], torch.from_numpy(got[1][n:]))
    assert one.dp.opt.step_count == 2 and float(one.dp.opt.v.abs().sum()) > 0
