"""PowerSGD gradient compression on gloo ranks (CPU)."""
import os
import socket
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class _Arena:
    def __init__(self, shapes):
        from aether_b200.models.arena import ParamArena

        self.a = ParamArena([(f"p{i}", s, True) for i, s in enumerate(shapes)], "cpu")


def _worker(rank, world, port, q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    sys.path.insert(0, ROOT)
    import torch.distributed as dist

    from aether_b200.parallel.compress import PowerSGD

    dist.init_process_group("gloo", rank=rank, world_size=world)
    out = {}
    # 1) rank >= the matrix rank: the estimate is the exact mean
    a = _Arena([(64, 48), (48,)]).a
    g = torch.Generator().manual_seed(10 + rank)
    low = torch.randn(64, 3, generator=torch.Generator().manual_seed(1))
    a.grad[:64 * 48].copy_((low @ torch.randn(3, 48, generator=g)).flatten())
    a.grad[a.slots["p1"].offset : a.slots["p1"].offset + 48].copy_(torch.randn(48, generator=g))
    local = a.grad.clone()
    comp = PowerSGD(a, world, rank=8, seed=0)
    assert len(comp.mats) == 1 and len(comp.plain) == 1
    comp.all_reduce_()
    mean = local.clone()
    dist.all_reduce(mean)
    mean /= world
    out["exact_err"] = float((a.grad - mean).norm() / mean.norm())
    out["err_feedback"] = float((comp.err[0] - (local[:64 * 48].view(64, 48) - a.grad[:64 * 48].view(64, 48))).norm())
    # 2) full-rank gradients at rank 2: error feedback makes the running sum of
    #    estimates equal the running sum of true means less the outstanding errors
    b = _Arena([(96, 80)]).a
    comp2 = PowerSGD(b, world, rank=2, seed=0)
    est, true = torch.zeros(96 * 80), torch.zeros(96 * 80)
    for step in range(30):
        gg = torch.randn(96 * 80, generator=torch.Generator().manual_seed(1000 * step + rank))
        b.grad[: 96 * 80].copy_(gg)
        m = gg.clone()
        dist.all_reduce(m)
        true += m / world
        comp2.all_reduce_()
        est += b.grad[: 96 * 80]
    # error feedback: sum of estimates + mean over ranks of the final errors = sum of true means
    e = comp2.err[0].flatten().clone()
    dist.all_reduce(e)
    out["track"] = float((est + e / world - true).norm() / true.norm())
    out["ratio"] = comp2.bytes_sent / comp2.bytes_dense
    out["grad"] = b.grad.clone()
    q.put((rank, out))
    dist.destroy_process_group()


def test_powersgd_two_ranks():
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=300) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in (0, 1):
        o = got[r]
        assert o["exact_err"] < 1e-4, o["exact_err"]
        assert o["err_feedback"] < 1e-4
        assert o["track"] < 1e-4, o["track"]
        assert o["ratio"] < 0.05
    assert torch.equal(got[0]["grad"], got[1]["grad"])  # every rank applies the same update
