"""Context parallelism on gloo ranks (CPU): two ranks, each holding half of
every sequence, give the loss and (averaged) gradients of one process over
the whole sequence."""
import os
import socket
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CFG = dict(vocab=128, d_model=64, n_layers=2, n_heads=2, n_kv_heads=2, d_ff=128, max_seq=32)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _tokens():
    return torch.randint(0, 128, (2, 33), generator=torch.Generator().manual_seed(11))


def _worker(rank, world, port, q, mode="allgather"):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    sys.path.insert(0, ROOT)
    import torch.distributed as dist

    from aether_b200.models.gpt import GPT, GPTConfig
    from aether_b200.parallel import dist as D
    from aether_b200.parallel.cp import CPGroup, shard_sequence

    D.init(device="cpu", timeout_s=60)
    cp = CPGroup(rank, world, None, mode)
    m = GPT(GPTConfig(**CFG), device="cpu", seed=4, cp=cp)
    ids, tgt = shard_sequence(_tokens(), cp)
    loss = m.loss(ids, tgt)
    loss.backward()
    g = m.arena.grad.clone()
    dist.all_reduce(g)  # the data-parallel average over the CP group
    g /= world
    lt = loss.detach().clone()
    dist.all_reduce(lt)
    q.put((rank, float(lt) / world, g.numpy()))
    D.shutdown()


@pytest.mark.parametrize("mode", ["allgather", "ring", "ulysses"])
def test_cp2_matches_full_sequence(mode):
    """All three attention schemes (K/V all-gather, ring attention with
    log-sum-exp merging, Ulysses all-to-all over heads) reproduce the
    one-process loss and gradients."""
    import multiprocessing as mp

    from aether_b200.models.gpt import GPT, GPTConfig

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q, mode)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict((r, (l, g)) for r, l, g in (q.get(timeout=300) for _ in ps))
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    ref = GPT(GPTConfig(**CFG), device="cpu", seed=4)
    t = _tokens()
    lr = ref.loss(t[:, :-1].contiguous(), t[:, 1:].contiguous())
    lr.backward()
    for r, (l, g) in got.items():
        assert abs(l - float(lr.detach())) < 1e-3 * float(lr.detach()), (l, float(lr))
        err = float((torch.from_numpy(g) - ref.arena.grad).norm() / ref.arena.grad.norm())
        assert err < 2e-2, err
