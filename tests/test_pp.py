"""Pipeline parallel 1F1B: two gloo ranks on CPU reproduce the single-process
run (loss trajectory and updated parameters), the reference's PP witness
(scripts/pp_2rank_witness.sh) in miniature."""
import os
import socket
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CFG = dict(vocab=128, d_model=64, n_layers=4, n_heads=2, n_kv_heads=2, d_ff=128, max_seq=16)


def _batches(step):
    g = torch.Generator().manual_seed(100 + step)
    toks = torch.randint(0, 128, (4, 2, 17), generator=g)
    return [(t[:, :-1].contiguous(), t[:, 1:].contiguous()) for t in toks]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    sys.path.insert(0, ROOT)
    from aether_b200.models.gpt import GPTConfig
    from aether_b200.parallel import dist as D
    from aether_b200.parallel.pp import GPTPipelineStage, run_1f1b

    D.init(device="cpu", timeout_s=60)
    st = GPTPipelineStage(GPTConfig(**CFG), rank, world, "cpu", seed=7, lr=1e-2, weight_decay=0.0)
    losses = []
    for step in range(3):
        st.zero_grad()
        loss = run_1f1b(st, _batches(step))
        st.step()
        if loss is not None:
            losses.append(float(loss))
    q.put((rank, losses, {n: st.model.arena.master_view(n).numpy().copy() for n in st.model.arena.names()}))
    D.shutdown()


def test_pp_matches_single_process():
    import multiprocessing as mp

    from aether_b200.models.gpt import GPT, GPTConfig
    from aether_b200.optim import FlatAdamW

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = {}
    for _ in range(2):
        r, losses, params = q.get(timeout=180)
        res[r] = (losses, params)
    for p in ps:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in ps)

    ref = GPT(GPTConfig(**CFG), device="cpu", seed=7)
    opt = FlatAdamW(ref.arena, lr=1e-2, weight_decay=0.0)
    ref_losses = []
    for step in range(3):
        ref.arena.zero_grad()
        bs = _batches(step)
        n_tok = sum(t.numel() for _, t in bs)
        tot = 0.0
        for ids, tgt in bs:
            loss = ref.loss(ids, tgt, 1.0 / n_tok)
            loss.backward()
            tot += float(loss)
        opt.step()
        ref_losses.append(tot)
    for a, b in zip(res[1][0], ref_losses):
        assert abs(a - b) < 1e-3 * abs(b), (res[1][0], ref_losses)
    for r in (0, 1):
        for name, v in res[r][1].items():
            assert torch.allclose(torch.from_numpy(v), ref.arena.master_view(name), atol=1e-4), name
