"""Tensor-parallel training on gloo ranks (CPU): a TP=2 GPT gives the loss and
(sharded) gradients of the unsharded model, and a TP=2 x DP=2 mesh trains to
the same parameters as one process over the same global batch -- with the
residual stream replicated over the TP ranks and with it split by token
(sequence parallelism)."""
import os
import socket
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CFG = dict(vocab=128, d_model=64, n_layers=2, n_heads=4, n_kv_heads=2, d_ff=128, max_seq=16)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _tokens(step, n=4):
    return torch.randint(0, 128, (n, 17), generator=torch.Generator().manual_seed(50 + step))


def _worker(rank, world, tp, port, q, sp=False, extra=None):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    sys.path.insert(0, ROOT)
    from aether_b200.models.gpt import GPT, GPTConfig
    from aether_b200.parallel import dist as D
    from aether_b200.parallel.dp import DataParallel
    from aether_b200.parallel.tp_train import make_mesh
    from aether_b200.train import Trainer

    D.init(device="cpu", timeout_s=60)
    mesh = make_mesh(tp, sequence_parallel=sp)
    assert mesh.tp.sp == sp
    m = GPT(GPTConfig(**CFG, **(extra or {})), device="cpu", seed=9, tp=mesh.tp, pad_multiple=mesh.dp_world)
    # one gradient for the checks against the unsharded model
    toks = _tokens(0)
    loss = m.loss(toks[:, :-1].contiguous(), toks[:, 1:].contiguous())
    loss.backward()
    m.finish_grads()
    grads = {n: m.arena.grad[s.offset : s.offset + s.numel].view(s.shape).clone().numpy() for n, s in m.arena.slots.items()}
    m.arena.zero_grad()
    # then a few training steps over the mesh: each DP rank takes its half of the global batch
    dinfo = D.DistInfo(mesh.dp_rank, mesh.dp_world, 0, torch.device("cpu"), "gloo")
    dp = DataParallel(m.arena, dinfo, lr=1e-2, weight_decay=0.0, group=mesh.dp_group)
    tr = Trainer(m, dinfo, lr=1e-2, micro_batch=2, dp=dp)
    for step in range(3):
        t = _tokens(1 + step, 4)
        half = t.shape[0] // mesh.dp_world
        tr.train_step(t[mesh.dp_rank * half : (mesh.dp_rank + 1) * half])
    # ZeRO-1: only this DP rank's shard of the fp32 master is current; the bf16
    # compute copy is all-gathered, so compare that
    master = {n: m.arena[n].detach().float().clone().numpy() for n in m.arena.names()}
    q.put((rank, float(loss.detach()), grads, master))
    D.shutdown()


def _run(world, tp, sp=False, extra=None):
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, tp, port, q, sp, extra)) for r in range(world)]
    for p in ps:
        p.start()
    got = {}
    for _ in ps:
        r, loss, grads, master = q.get(timeout=300)
        got[r] = (loss, grads, master)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    return got


def _reference(extra=None):
    from aether_b200.models.gpt import GPT, GPTConfig
    from aether_b200.parallel import dist as D
    from aether_b200.train import Trainer

    m = GPT(GPTConfig(**CFG, **(extra or {})), device="cpu", seed=9)
    toks = _tokens(0)
    loss = m.loss(toks[:, :-1].contiguous(), toks[:, 1:].contiguous())
    loss.backward()
    grads = {n: m.arena.grad[s.offset : s.offset + s.numel].view(s.shape).clone() for n, s in m.arena.slots.items()}
    m.arena.zero_grad()
    tr = Trainer(m, D.DistInfo(), lr=1e-2, weight_decay=0.0, micro_batch=2)
    for step in range(3):
        tr.train_step(_tokens(1 + step, 4))
    return m, float(loss.detach()), grads


def _init_master(extra=None):
    from aether_b200.models.gpt import GPT, GPTConfig

    m = GPT(GPTConfig(**CFG, **(extra or {})), device="cpu", seed=9)
    return {n: m.arena.master_view(n).clone() for n in m.arena.names()}


def _check(got, tp, extra=None):
    from aether_b200.models.gpt import GPTConfig
    from aether_b200.parallel.tp_train import shard_tensor

    cfg = GPTConfig(**CFG, **(extra or {}))
    ref, lref, gref = _reference(extra)
    for rank, (loss, grads, master) in got.items():
        assert abs(loss - lref) < 1e-4 * abs(lref), (loss, lref)
        tr = rank % tp
        # bf16 activations: TP rounds each partial sum before the all-reduce
        for n, g in grads.items():
            want = shard_tensor(cfg, n, gref[n], tr, tp)
            err = float((torch.from_numpy(g) - want).norm() / want.norm().clamp(min=1e-12))
            assert err < 3e-2, (n, err)
        # Adam turns tiny, rounding-level gradient differences into full-size
        # steps, so compare the direction of each tensor's total update
        init = _init_master(extra)
        for n, w in master.items():
            want = shard_tensor(cfg, n, ref.arena.master_view(n), tr, tp) - shard_tensor(cfg, n, init[n], tr, tp)
            got = torch.from_numpy(w) - shard_tensor(cfg, n, init[n], tr, tp)
            cos = float((got * want).sum() / (got.norm() * want.norm()).clamp(min=1e-20))
            assert cos > 0.95, (n, cos)


def test_tp2_matches_single_process():
    _check(_run(2, 2), 2)


def test_tp2_dp2_mesh_matches_single_process():
    _check(_run(4, 2), 2)


def test_tp2_sequence_parallel_matches_single_process():
    _check(_run(2, 2, sp=True), 2)


def test_tp2_dp2_sequence_parallel_mesh_matches_single_process():
    _check(_run(4, 2, sp=True), 2)


def test_tp2_qk_norm_matches_single_process():
    """Qwen3-style q/k norms: each rank normalises its own heads, so the shared
    norm weights' gradients are summed over the TP group."""
    qk = {"qk_norm": True}
    _check(_run(2, 2, extra=qk), 2, qk)
    _check(_run(2, 2, sp=True, extra=qk), 2, qk)


def test_fused_tp_gemm_refusals():
    """The fused TP / ZeRO-3 GEMM entry points refuse what they cannot tile
    with a message (raised by the Python wrappers), before touching a device."""
    import pytest as _pytest

    from aether_b200.ops import functional as F

    a = [torch.zeros(100, 256, dtype=torch.bfloat16)] * 2
    with _pytest.raises(RuntimeError, match="multiple of 128"):
        F.gemm_tp(a, [], a, a, [], [], [0, 1], 2, 100, False, 0, True, False, [], [], 0, [16, 16], [16, 16], 0, 1, 1.0)
    with _pytest.raises(RuntimeError, match="nothing to fuse"):
        F.gemm_tp(a, [], a, a, [], [], [0, 1], 2, 128, False, 0, False, False, [], [], 0, [], [], 0, 0, 1.0)
    sq = [torch.zeros(256, 256, dtype=torch.bfloat16)] * 2
    with _pytest.raises(RuntimeError, match="CUDA tensors"):
        F.gemm_tp(sq, sq, sq, sq, [], sq, [0, 1], 2, 128, False, 1, False, False, [16, 32], [16, 32], 0, [], [], 1, 0,
                  1.0)
    with _pytest.raises(RuntimeError, match="world unit buffers"):
        F.gemm_param_gather(a, a, a, a, a, [0, 1], 2, 2048, False, [16], [16], [16], 0, 1, 1.0)
