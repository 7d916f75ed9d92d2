"""libaether_rt developer tooling, the NCCL-shaped host communicator (one
process, and two processes meeting over TCP), the matmul tile autotuner and
the audio primitives."""
import json
import os
import socket
import time

import numpy as np

from aether_b200 import runtime as R


def _b(s):
    return s.encode()


def test_hot_reload_sbom_cov_pgo(tmp_path):
    p = str(tmp_path / "sentinel")
    open(p, "w").write("a")
    bp = _b(p)
    assert R.call("aether_hot_reload_arm", bp, len(bp)) == 0
    assert R.call("aether_hot_reload_check", bp, len(bp)) == 0
    t = time.time() + 5
    os.utime(p, (t, t))
    assert R.call("aether_hot_reload_check", bp, len(bp)) == 1
    assert R.call("aether_hot_reload_check", bp, len(bp)) == 0  # re-armed
    R.call("aether_sbom_reset")
    for n, v in (("torch", "2.11"), ('we"ird', "1.0")):
        assert R.call("aether_sbom_add", _b(n), len(n), _b(v), len(v)) == 0
    assert R.call("aether_sbom_count") == 2
    out = str(tmp_path / "sbom.json")
    assert R.call("aether_sbom_emit", _b(out), len(out)) == 0
    doc = json.load(open(out))
    assert doc["bomFormat"] == "CycloneDX" and [c["name"] for c in doc["components"]] == ["torch", 'we"ird']
    R.call("aether_cov_reset")
    for _ in range(3):
        R.call("aether_cov_record", 7, 42)
    assert R.call("aether_cov_hits", 7, 42) == 3 and R.call("aether_cov_hits", 7, 43) == 0
    R.call("aether_pgo_reset")
    for taken in (1, 1, 0, 1):
        R.call("aether_pgo_record_branch", 5, taken)
    R.call("aether_pgo_record_call", 9)
    assert abs(R.call("aether_pgo_branch_freq", 5) - 0.75) < 1e-6 and R.call("aether_pgo_call_count", 9) == 1
    buf = np.zeros(16, np.float32)
    assert R.call("aether_prefetch_t0", buf.ctypes.data) == 0


def test_autotune_and_audio():
    h = R.call("aether_autotune_matmul_tile_f32", 4096, 4096, 4096)
    tm, tn, tk = (R.call(f"aether_autotune_unpack_tile_{c}", h) for c in "mnk")
    assert 8 <= tm <= 128 and 8 <= tn <= 128 and 8 <= tk <= 64  # a candidate tile that fits half of L1
    small = R.call("aether_autotune_matmul_tile_f32", 3, 5, 7)
    assert [R.call(f"aether_autotune_unpack_tile_{c}", small) for c in "mnk"] == [3, 5, 7]
    w = np.zeros(64, np.float32)
    assert R.call("aether_audio_hann_window", R.ptr(w), 64) == 0
    assert np.allclose(w, np.hanning(64), atol=1e-6)
    x = np.sin(2 * np.pi * 5 * np.arange(64) / 64).astype(np.float32)
    mag = np.zeros(16, np.float32)
    assert R.call("aether_audio_dft_magnitude_f32", R.ptr(x), 64, R.ptr(mag), 16) == 0
    assert np.allclose(mag, np.abs(np.fft.rfft(x))[:16], atol=1e-3)


def test_nccl_surface_one_rank():
    R.call("aether_nccl_finalize")
    assert R.call("aether_nccl_init") == 0 and R.call("aether_nccl_init_count") == 1
    c = R.call("aether_nccl_comm_create", 1, 0)
    assert c >= 1 and R.call("aether_nccl_comm_world_size", c) == 1 and R.call("aether_nccl_comm_rank", c) == 0
    a = np.arange(8, dtype=np.float32)
    b = np.zeros(8, np.float32)
    assert R.call("aether_nccl_all_reduce_f32", R.ptr(a), R.ptr(b), 8, 0, c) == 0 and np.array_equal(a, b)
    assert R.call("aether_nccl_all_reduce_f32", R.ptr(a), R.ptr(b), 8, 9, c) == 2
    assert R.call("aether_nccl_comm_create", 2, 0) == -1 or "AETHER_COMM_ADDR" in os.environ
    R.call("aether_nccl_finalize")


def _comm_rank(rank, world, addr, q):
    os.environ["AETHER_COMM_ADDR"] = addr
    from aether_b200 import runtime as RR

    c = RR.call("aether_nccl_comm_create", world, rank)
    x = np.full(5, rank + 1.0, np.float32)
    outs = []
    for op in (0, 1, 2, 3):
        y = np.zeros(5, np.float32)
        rc = RR.call("aether_nccl_all_reduce_f32", RR.ptr(x), RR.ptr(y), 5, op, c)
        outs.append((rc, y.tolist()))
    RR.call("aether_nccl_comm_destroy", c)
    q.put((rank, c, outs))


def test_nccl_surface_two_processes():
    import multiprocessing as mp

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_comm_rank, args=(r, 3, f"127.0.0.1:{port}", q)) for r in range(3)]
    for p in ps:
        p.start()
    got = dict((r, (c, o)) for r, c, o in (q.get(timeout=120) for _ in ps))
    for p in ps:
        p.join(timeout=30)
        assert p.exitcode == 0
    for r in range(3):
        c, outs = got[r]
        assert c >= 1
        assert [o[0] for o in outs] == [0, 0, 0, 0]
        assert outs[0][1] == [6.0] * 5 and outs[1][1] == [3.0] * 5 and outs[2][1] == [1.0] * 5
        assert outs[3][1] == [6.0] * 5  # 1 * 2 * 3


def test_image_preprocess():
    rng = np.random.default_rng(1)
    px = rng.integers(0, 256, 48, dtype=np.uint8)
    out = np.zeros(48, np.float32)
    assert R.call("aether_img_normalize_f32", R.ptr(px), R.ptr(out), 48, 0.485, 0.229) == 0
    assert np.allclose(out, (px / 255.0 - 0.485) / 0.229, atol=1e-5)
    img = rng.standard_normal((8, 12)).astype(np.float32)
    pat = np.zeros(6 * 16, np.float32)
    assert R.call("aether_img_patchify_f32", R.ptr(img), R.ptr(pat), 8, 12, 4) == 6
    want = img.reshape(2, 4, 3, 4).transpose(0, 2, 1, 3).reshape(6, 16)
    assert np.array_equal(pat.reshape(6, 16), want)
    assert R.call("aether_img_patchify_f32", R.ptr(img), R.ptr(pat), 8, 12, 5) == -3


def test_llm_inference_bench_entry_point(capfd):
    tps = R.call("aether_llm_inference_bench_tps", 3, 64, 2, 128, 16)
    assert tps > 0
    assert R.call("aether_llm_inference_bench_tps", 0, 64, 2, 128, 16) == 0.0
    R.call("aether_print_bench", 0, 64, 64, 64, 10, 1234)
    assert "cpu  M=  64" in capfd.readouterr().out
