"""The generic collective C ABI of libaether_rt across processes: three
ranks meet at AETHER_COMM_ADDR and run broadcast, all-gather, reduce-scatter,
all-to-all, a send / recv ring, the in-place all-reduce sum and the
rendezvous the compiler emits for `#[distributed]` functions; world size 1
keeps the reference's single-rank semantics."""
import ctypes
import os
import socket

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "aether_b200", "libaether_rt.so")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _worker(rank, world, port, q):
    os.environ.update(AETHER_RANK=str(rank), AETHER_WORLD_SIZE=str(world), AETHER_COMM_ADDR=f"127.0.0.1:{port}")
    lib = ctypes.CDLL(LIB)
    lib.aether_dist_all_reduce.restype = None
    n = 5
    out = {"world": lib.aether_comm_world_size(), "rank": lib.aether_comm_rank()}
    # broadcast from rank 1
    b = np.full(n, float(rank), np.float32)
    out["bcast_rc"] = lib.aether_op_broadcast_f32(_ptr(b), n, 1)
    out["bcast"] = b.tolist()
    # all-gather: block r = rank r's vector
    src = np.arange(n, dtype=np.float32) + 10 * rank
    dst = np.zeros(n * world, np.float32)
    out["ag_rc"] = lib.aether_op_all_gather_f32(_ptr(src), _ptr(dst), n, world)
    out["ag"] = dst.tolist()
    # reduce-scatter: rank r gets sum over ranks of block r
    full = (np.arange(n * world, dtype=np.float32) + 100 * rank)
    rs = np.zeros(n, np.float32)
    out["rs_rc"] = lib.aether_op_reduce_scatter_f32(_ptr(full), _ptr(rs), n, world)
    out["rs"] = rs.tolist()
    # all-to-all: block p of my src goes to rank p
    a2a_src = np.array([1000 * rank + p for p in range(world) for _ in range(n)], np.float32)
    a2a_dst = np.zeros(n * world, np.float32)
    out["a2a_rc"] = lib.aether_op_all_to_all_f32(_ptr(a2a_src), _ptr(a2a_dst), n, world)
    out["a2a"] = a2a_dst.tolist()
    # ring: send to rank+1, receive from rank-1 (even ranks send first)
    tok = np.full(n, float(rank), np.float32)
    got = np.zeros(n, np.float32)
    nxt, prv = (rank + 1) % world, (rank - 1) % world
    if rank % 2 == 0:
        rc1 = lib.aether_op_send_f32(_ptr(tok), n, nxt)
        rc2 = lib.aether_op_recv_f32(_ptr(got), n, prv)
    else:
        rc2 = lib.aether_op_recv_f32(_ptr(got), n, prv)
        rc1 = lib.aether_op_send_f32(_ptr(tok), n, nxt)
    out["ring_rc"] = (rc1, rc2)
    out["ring"] = got.tolist()
    # in-place all-reduce sum, and a world-size mismatch
    ar = np.array([rank + 1.0, 2.0 * rank, 0.5], np.float32)
    out["ar_rc"] = lib.aether_op_all_reduce_sum_f32(_ptr(ar), world, 3)
    out["ar"] = ar.tolist()
    out["ar_bad"] = lib.aether_op_all_reduce_sum_f32(_ptr(ar), world + 1, 3)
    lib.aether_dist_all_reduce(None, world, 0)  # rendezvous; returns once every rank arrived
    q.put((rank, out))


def test_collectives_across_three_processes():
    import multiprocessing as mp

    world, n = 3, 5
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=30)
        assert p.exitcode == 0
    for r in range(world):
        o = res[r]
        assert (o["world"], o["rank"]) == (world, r)
        assert o["bcast_rc"] == 0 and o["bcast"] == [1.0] * n
        assert o["ag_rc"] == 0
        assert o["ag"] == [float(i + 10 * p) for p in range(world) for i in range(n)]
        assert o["rs_rc"] == 0
        assert o["rs"] == [float(sum(r * n + i + 100 * p for p in range(world))) for i in range(n)]
        assert o["a2a_rc"] == 0
        assert o["a2a"] == [float(1000 * p + r) for p in range(world) for _ in range(n)]
        assert o["ring_rc"] == (0, 0) and o["ring"] == [float((r - 1) % world)] * n
        assert o["ar_rc"] == 0 and o["ar"] == [6.0, 6.0, 1.5]
        assert o["ar_bad"] == -1


def test_single_rank_keeps_reference_semantics():
    import subprocess
    import sys

    code = f"""
import ctypes, numpy as np
lib = ctypes.CDLL({LIB!r})
p = lambda a: a.ctypes.data_as(ctypes.c_void_p)
src = np.arange(4, dtype=np.float32); dst = np.zeros(4, np.float32)
assert lib.aether_op_all_gather_f32(p(src), p(dst), 4, 1) == 0 and dst.tolist() == src.tolist()
dst[:] = 0
assert lib.aether_op_reduce_scatter_f32(p(src), p(dst), 4, 1) == 0 and dst.tolist() == src.tolist()
assert lib.aether_op_broadcast_f32(p(src), 4, 0) == 0
assert lib.aether_op_all_reduce_sum_f32(p(src), 1, 4) == 0 and src.tolist() == [0, 1, 2, 3]
assert lib.aether_op_all_reduce_sum_f32(p(src), 2, 4) == -1
assert lib.aether_comm_world_size() == 1
print("ok")
"""
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "AETHER_RANK", "AETHER_WORLD_SIZE")}
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=60)
    assert out.returncode == 0 and "ok" in out.stdout, out.stderr
