"""Failure detection without faulting a GPU.

Host side (gloo ranks on CPU): a rank that dies between steps is reported by
the heartbeat watchdog of the survivors; a rank that never joins a collective
makes the others' collective end with an error after the short process-group
timeout instead of hanging; a crash inside a training step leaves a
``crash_<pid>_<step>.dump`` breadcrumb.
Device side: the in-kernel team barrier waiting on a peer flag that nothing
sets gives up after its limit, records the timeout status and leaves the
context usable.
"""
import datetime
import json
import os
import socket
import sys
import time

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _put_and_exit(q, item):
    q.put(item)
    q.close()
    q.join_thread()  # flush the queue's feeder thread before the hard exit
    os._exit(0)


def _hb_worker(rank, world, port, q):
    sys.path.insert(0, ROOT)
    import torch.distributed as dist

    from aether_b200.utils.health import Heartbeat, RankFailure, Watchdog

    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=30))
    dist.init_process_group("gloo", store=store, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    hb = Heartbeat(store, rank, world, period=0.1, timeout=1.5).start()
    wd = Watchdog(hb)
    t = torch.ones(4)
    for step in range(3):  # healthy steps
        wd.between_steps()
        dist.all_reduce(t)
    if rank == world - 1:
        _put_and_exit(q, (rank, "left"))  # dies between steps, without a clean stop
    deadline = time.time() + 15
    try:
        while time.time() < deadline:
            wd.between_steps()
            time.sleep(0.1)
        _put_and_exit(q, (rank, "not detected"))
    except RankFailure as e:
        _put_and_exit(q, (rank, e.ranks))


def test_heartbeat_detects_dead_rank():
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    world = 3
    ps = [ctx.Process(target=_hb_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=90) for _ in ps)
    for p in ps:
        p.join(timeout=30)
    assert got[2] == "left"
    assert got[0] == [2] and got[1] == [2], got


def _timeout_worker(rank, world, port, q):
    sys.path.insert(0, ROOT)
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=3))
    t = torch.ones(4)
    dist.all_reduce(t)  # everyone joins this one
    if rank == 1:
        time.sleep(12)  # never joins the next collective in time
        _put_and_exit(q, (rank, "slept"))
    t0 = time.time()
    try:
        dist.all_reduce(t)
        _put_and_exit(q, (rank, "completed"))
    except Exception as e:  # noqa: BLE001
        _put_and_exit(q, (rank, ("error", round(time.time() - t0, 1), type(e).__name__)))


def test_collective_times_out_instead_of_hanging():
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_timeout_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=90) for _ in ps)
    for p in ps:
        p.join(timeout=30)
    assert got[0][0] == "error" and got[0][1] < 11, got


def test_crash_dump_written(tmp_path):
    from aether_b200.models.gpt import GPT, GPTConfig
    from aether_b200.parallel import dist as D
    from aether_b200.train import Trainer

    m = GPT(GPTConfig(vocab=64, d_model=32, n_layers=1, n_heads=2, n_kv_heads=2, d_ff=64, max_seq=16), device="cpu")
    tr = Trainer(m, D.DistInfo(), lr=1e-3, crash_dir=str(tmp_path))
    tr.train_step(torch.randint(0, 64, (2, 9)))
    with pytest.raises(Exception) as ei:
        tr.train_step(torch.randint(64, 128, (2, 9)))  # token ids outside the vocabulary
    dumps = [f for f in os.listdir(tmp_path) if f.startswith(f"crash_{os.getpid()}_")]
    assert dumps == [f"crash_{os.getpid()}_1.dump"], dumps
    rec = json.load(open(tmp_path / dumps[0]))
    assert rec["step"] == 1 and type(ei.value).__name__ in rec["exception"] and "train_step" in rec["traceback"]


def test_tracer_sections_cpu(tmp_path):
    from aether_b200.utils.trace import Tracer

    tr = Tracer(enabled=True, nvtx=False)
    for _ in range(3):
        with tr.section("a", device=False):
            time.sleep(0.002)
    s = tr.summary()
    assert s["a"]["count"] == 3 and s["a"]["mean_ms"] >= 1.5
    tr.chrome_trace(str(tmp_path / "t.json"))
    assert len(json.load(open(tmp_path / "t.json"))["traceEvents"]) == 3


@pytest.mark.gpu
def test_device_barrier_wait_times_out_with_status():
    from aether_b200 import _ext

    C = _ext.C()
    assert _ext.check_status() == 0
    my_sig = torch.zeros(8, dtype=torch.int32, device="cuda")
    fake_peer = torch.zeros(8, dtype=torch.int32, device="cuda")  # stands in for a peer that never signals
    epoch = torch.zeros(1, dtype=torch.int32, device="cuda")
    ptrs = torch.tensor([my_sig.data_ptr(), fake_peer.data_ptr()], dtype=torch.int64)
    t0 = time.time()
    C.team_barrier(ptrs, my_sig, epoch, 0, 2, 0.3)
    torch.cuda.synchronize()
    assert time.time() - t0 < 5.0
    assert _ext.check_status() == 4  # timed out waiting for a peer
    assert int(fake_peer[0]) == 1  # our own signal was delivered
    a = torch.randn(256, 256, device="cuda").bfloat16()  # the context is still usable
    from aether_b200.ops import functional as F

    assert float((F.gemm(a, a).float() - a.float() @ a.float().t()).abs().max()) < 1.0
    assert _ext.check_status() == 0
