"""ZeRO-2 and ZeRO-3 (FSDP) on gloo ranks (CPU): two optimiser steps give the
same losses and parameters as the ZeRO-1 data-parallel engine."""
import os
import socket
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CFG = dict(vocab=128, d_model=64, n_layers=3, n_heads=2, n_kv_heads=2, d_ff=128, max_seq=16)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, stage, micro, q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    sys.path.insert(0, ROOT)
    from aether_b200.models.gpt import GPT, GPTConfig
    from aether_b200.parallel import dist as D
    from aether_b200.parallel.dp import DataParallel
    from aether_b200.parallel.fsdp import ShardedDataParallel, ShardSpec
    from aether_b200.train import Trainer

    info = D.init(device="cpu", timeout_s=60)
    g = torch.Generator().manual_seed(100 + rank)
    batches = [torch.randint(0, 128, (4, 17), generator=g) for _ in range(int(os.environ.get("NSTEPS", "2")))]
    if stage == 1:
        m = GPT(GPTConfig(**CFG), device="cpu", seed=3, pad_multiple=world)
        eng = DataParallel(m.arena, info, lr=1e-2)
    else:
        m = GPT(GPTConfig(**CFG), device="cpu", seed=3, shard=ShardSpec(rank, world, stage))
        eng = ShardedDataParallel(m.arena, lr=1e-2)
    tr = Trainer(m, info, micro_batch=micro, dp=eng, lr=1e-2)
    losses = [float(tr.train_step(b)) for b in batches]
    if stage == 1:  # ZeRO-1 refreshes only its own master shard; the bf16 copy is all-gathered
        params = {n: m.arena[n].detach().float().clone() for n in m.arena.names()}
    else:
        params = {n: t.bfloat16().float() for n, t in m.arena.full_state().items()}
    q.put((rank, losses, {k: v.numpy() for k, v in params.items()}))
    D.shutdown()


def _run(stage, micro):
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, stage, micro, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = dict((r, (l, prm)) for r, l, prm in (q.get(timeout=300) for _ in ps))
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    return out


@pytest.mark.parametrize("micro", [4, 2])
def test_zero2_zero3_match_zero1(micro):
    """One micro-batch per step: the same sums in the same order, so the
    parameters agree to a bf16 rounding. Two micro-batches: ZeRO-2/3 reduce
    each micro-batch separately (a different fp32 summation order), so
    compare the direction of the whole update."""
    from aether_b200.models.gpt import GPT, GPTConfig

    init = GPT(GPTConfig(**CFG), device="cpu", seed=3)
    p0 = {n: init.arena[n].detach().float() for n in init.arena.names()}
    base = _run(1, micro)
    for stage in (2, 3):
        got = _run(stage, micro)
        for r in (0, 1):
            lb, pb = base[r]
            lg, pg = got[r]
            assert all(abs(a - b) < 1e-4 for a, b in zip(lb, lg)), (stage, lb, lg)
            ub = torch.cat([(torch.from_numpy(pb[n]) - p0[n]).flatten() for n in pb])
            ug = torch.cat([(torch.from_numpy(pg[n]) - p0[n]).flatten() for n in pb])
            if micro == 4:
                assert float((ub - ug).abs().max()) < 1e-4, stage
            cos = float(torch.dot(ub, ug) / (ub.norm() * ug.norm()))
            assert cos > 0.999, (stage, cos)


def test_stage_bytes():
    from aether_b200.parallel.fsdp import stage_bytes

    n, w = 1_000_000, 8
    assert stage_bytes(n, w, 3) < stage_bytes(n, w, 2) < stage_bytes(n, w, 1)
    assert stage_bytes(n, 1, 3) == stage_bytes(n, 1, 1) == 18 * n


def _one_rank(n_layers, stage, device, tie=False):
    from aether_b200.models.gpt import GPT, GPTConfig
    from aether_b200.parallel.fsdp import ShardSpec

    cfg = dict(CFG, n_layers=n_layers, tie_embeddings=tie)
    if device == "cuda":  # the attention kernels take head_dim 64 or 128
        cfg.update(d_model=128, d_ff=256)
    g = torch.Generator().manual_seed(5)
    ts = [torch.randint(0, 128, (2, 17), generator=g).to(device) for _ in range(2)]
    m1 = GPT(GPTConfig(**cfg), device=device, seed=3)
    m2 = GPT(GPTConfig(**cfg), device=device, seed=3, shard=ShardSpec(0, 1, stage))
    for m in (m1, m2):
        for t in ts:
            m.loss(t[:, :-1].contiguous(), t[:, 1:].contiguous()).backward()
    m2.arena._finish_grads()
    a = m2.arena
    for n, s in a.slots.items():
        unit = a.units[a.unit_of[n]]
        g2 = a.grad[unit.offset + s.offset : unit.offset + s.offset + s.numel]
        o1 = m1.arena.slots[n].offset
        g1 = m1.arena.grad[o1 : o1 + s.numel]
        assert float((g1 - g2).abs().max()) <= 1e-6 * max(1.0, float(g1.abs().max())), n


@pytest.mark.parametrize("n_layers", [1, 2, 3])
@pytest.mark.parametrize("stage", [2, 3])
def test_sharded_grads_accumulate_one_rank(n_layers, stage):
    """World 1: two backward passes accumulate the same gradients as the flat
    arena (exercises the rotating unit buffers and their recycling)."""
    _one_rank(n_layers, stage, "cpu")


@pytest.mark.parametrize("stage", [2, 3])
def test_sharded_tied_embeddings_one_rank(stage):
    """The tied embedding / LM head weight lives in the root unit and gets
    both its gradients."""
    _one_rank(2, stage, "cpu", tie=True)


@pytest.mark.gpu
@pytest.mark.parametrize("stage", [2, 3])
def test_sharded_grads_accumulate_one_rank_gpu(stage):
    """The same on the GPU kernels: the weight-gradient GEMMs reduce into the
    rotating unit buffers found through the autograd gradient-buffer table."""
    _one_rank(3, stage, "cuda")


def _ckpt_worker(rank, world, port, path, q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    sys.path.insert(0, ROOT)
    from aether_b200 import checkpoint
    from aether_b200.models.gpt import GPT, GPTConfig
    from aether_b200.parallel import dist as D
    from aether_b200.parallel.fsdp import ShardedDataParallel, ShardSpec
    from aether_b200.train import Trainer

    info = D.init(device="cpu", timeout_s=60)
    g = torch.Generator().manual_seed(200 + rank)
    batches = [torch.randint(0, 128, (4, 17), generator=g) for _ in range(3)]

    def build():
        m = GPT(GPTConfig(**CFG), device="cpu", seed=3, shard=ShardSpec(rank, world, 3))
        eng = ShardedDataParallel(m.arena, lr=1e-2)
        return m, eng, Trainer(m, info, micro_batch=4, dp=eng, lr=1e-2)

    m, eng, tr = build()
    for b in batches[:2]:
        tr.train_step(b)
    checkpoint.save(path, m.arena, eng, step=2, rank=rank, world=world)
    straight = float(tr.train_step(batches[2]))
    want = m.arena.full_state()
    m2, eng2, tr2 = build()
    step = checkpoint.load(path, m2.arena, eng2)
    tr2.step_idx = step
    resumed = float(tr2.train_step(batches[2]))
    got = m2.arena.full_state()
    same = all(torch.equal(want[n], got[n]) for n in want)
    q.put((rank, step, straight, resumed, same))
    D.shutdown()


def test_zero3_checkpoint_resume_bitwise_and_into_plain_arena(tmp_path):
    import multiprocessing as mp

    from aether_b200 import checkpoint
    from aether_b200.models.gpt import GPT, GPTConfig
    from aether_b200.optim import FlatAdamW

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    path = str(tmp_path / "ck")
    ps = [ctx.Process(target=_ckpt_worker, args=(r, 2, port, path, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = [q.get(timeout=300) for _ in ps]
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, step, straight, resumed, same in out:
        assert step == 2 and straight == resumed and same, (rank, straight, resumed, same)
    # the world-2 ZeRO-3 checkpoint resumes into a one-process flat arena
    info, named, _ = checkpoint.named_state(path)
    m = GPT(GPTConfig(**CFG), device="cpu", seed=99)
    opt = FlatAdamW(m.arena, lr=1e-2)
    assert checkpoint.load(path, m.arena, opt) == 2
    for n in m.arena.names():
        assert torch.equal(m.arena.master_view(n), named[n]["master"]), n
    assert opt.step_count == 2 and float(opt.m.abs().sum()) > 0
