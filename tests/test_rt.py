"""libaether_rt C ABI through ctypes: core op bodies against numpy, the
AetherLM-Nano trainer on the BASELINE nano config (loss 5.5 -> under 1.5 in
60 steps) and its byte-exact checkpoint, the extended op / optimiser /
pooling / dtype / dequant entry points, and the serving and observability
structures."""
import ctypes
import os

import numpy as np
import torch

from aether_b200 import runtime as rt
from aether_b200.formats import aether_weights, gguf

R = np.random.default_rng(0)


def f32(*shape):
    return R.standard_normal(shape).astype(np.float32)


def test_core_ops_match_numpy():
    a, b = f32(5, 7), f32(7, 3)
    c = np.zeros((5, 3), np.float32)
    assert rt.call("aether_op_matmul_f32", rt.ptr(a), rt.ptr(b), rt.ptr(c), 5, 7, 3) == 0
    np.testing.assert_allclose(c, a @ b, rtol=1e-5, atol=1e-5)
    x = f32(4, 9)
    y = x.copy()
    rt.call("aether_op_softmax_f32", rt.ptr(y), 4, 9, -1)
    e = np.exp(x - x.max(1, keepdims=True))
    np.testing.assert_allclose(y, e / e.sum(1, keepdims=True), rtol=1e-5, atol=1e-6)
    p, g = f32(100), f32(100)
    m, v = np.zeros(100, np.float32), np.zeros(100, np.float32)
    p0 = p.copy()
    rt.call("aether_op_adamw_step_f32", rt.ptr(p), rt.ptr(g), rt.ptr(m), rt.ptr(v), 1e-2, 0.9, 0.95, 1e-8, 0.1, 1, 100)
    mh, vh = 0.1 * g / 0.1, 0.05 * g * g / 0.05
    np.testing.assert_allclose(p, p0 - 1e-2 * (mh / (np.sqrt(vh) + 1e-8) + 0.1 * p0), rtol=1e-4, atol=1e-6)
    assert rt.call("aether_rt_self_check") >= 0


def test_nano_baseline_config_trains_and_checkpoints(tmp_path):
    nano = rt.Nano(vocab=256, d_model=64, n_layers=2, n_heads=4, d_ff=128, seq_len=32, seed=42)
    assert nano.n_params == 85504  # the reference's nano parameter count (incl. positional embeddings)
    # the reference trainer's default smoke corpus: loss ~5.5 -> ~0.8 in 60 steps
    data = rt.pattern_corpus(1 << 20)
    state = np.array([42 * 7919 + 1], dtype=np.uint64)
    losses = []
    for step in range(60):
        ids, labels = rt.sample_batch(data, 8, 32, state)
        lr = float(rt.call("aether_nano_cosine_lr", step, 60, 3e-3, 10))
        losses.append(nano.train_step(ids, labels, lr, 0.0, 1.0))
    assert losses[0] > 5.0 and losses[-1] < 1.2, (losses[0], losses[-1])
    stem = str(tmp_path / "aether_lm")
    assert nano.save(stem) == 0
    params, meta = aether_weights.load(stem)
    assert np.array_equal(params, nano.params()) and meta["params"] == 85504 and meta["seq_len"] == 32
    other = rt.Nano(seed=7)
    assert other.load(stem + ".weights") == 0
    ids, labels = rt.sample_batch(data, 8, 32, state)
    assert other.loss(ids, labels) == nano.loss(ids, labels)
    # the random-word corpus (uniform words from a seeded 200-word vocabulary)
    words = rt.synthetic_corpus(1 << 16, seed=42)
    assert set(np.unique(words).tolist()) <= set(range(97, 123)) | {32}
    assert len(nano.generate([116, 104], 60)) == 60


def test_extended_ops():
    x = np.abs(f32(64)) + 0.1
    y = x.copy()
    rt.call("aether_op_pow_f32", rt.ptr(y), 1.5, 64)
    np.testing.assert_allclose(y, x ** 1.5, rtol=1e-5)
    assert abs(rt.call("aether_op_var_f32", rt.ptr(x), 64) - x.var()) < 1e-4
    assert rt.call("aether_op_argmax_f32", rt.ptr(x), 64) == int(x.argmax())
    # Lion
    p, g, m = f32(32), f32(32), f32(32)
    p0, m0 = p.copy(), m.copy()
    rt.call("aether_op_lion_step_f32", rt.ptr(p), rt.ptr(g), rt.ptr(m), 32, 0.01, 0.9, 0.99, 0.1)
    np.testing.assert_allclose(p, p0 - 0.01 * (np.sign(0.9 * m0 + 0.1 * g) + 0.1 * p0), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(m, 0.99 * m0 + 0.01 * g, rtol=1e-5)
    # pooling against torch
    img = f32(2, 3, 9, 11)
    out = np.zeros((2, 3, 4, 5), np.float32)
    rt.call("aether_op_max_pool_2d_f32", rt.ptr(img), rt.ptr(out), 2, 3, 9, 11, 3, 3, 2, 2, 0, 0)
    np.testing.assert_allclose(out, torch.nn.functional.max_pool2d(torch.from_numpy(img), 3, 2).numpy())
    img2 = f32(2, 3, 9, 12)  # divisible sizes: the ABI's floor windows equal torch's
    ad = np.zeros((2, 3, 3, 4), np.float32)
    rt.call("aether_op_adaptive_avg_pool_2d_f32", rt.ptr(img2), rt.ptr(ad), 2, 3, 9, 12, 3, 4)
    np.testing.assert_allclose(ad, torch.nn.functional.adaptive_avg_pool2d(torch.from_numpy(img2), (3, 4)).numpy(),
                               rtol=1e-5, atol=1e-6)
    # embedding bag (mean)
    w = f32(10, 4)
    idx = np.array([1, 2, 3, 9, 0], np.int32)
    off = np.array([0, 3, 5], np.int32)
    eb = np.zeros((2, 4), np.float32)
    rt.call("aether_op_embedding_bag_f32", rt.ptr(w), rt.ptr(idx), rt.ptr(off), rt.ptr(eb), 2, 10, 4, 5, 1)
    np.testing.assert_allclose(eb, np.stack([w[[1, 2, 3]].mean(0), w[[9, 0]].mean(0)]), rtol=1e-6)


def test_dtype_conversions_and_dequant():
    vals = np.array([0.0, 1.0, -2.5, 3.1415926, 1e-3, 65504.0, 1e-6], np.float32)
    for v in vals:
        bf = rt.call("aether_f32_to_bf16", float(v))
        assert rt.call("aether_bf16_to_f32", bf) == float(torch.tensor(v).bfloat16().float())
        hb = rt.call("aether_f32_to_f16", float(v))
        assert hb == int(np.array([v], np.float16).view(np.uint16)[0])
        assert rt.call("aether_f16_to_f32", hb) == float(np.float16(v))
    for typ, name, size in ((gguf.Q4_0, "aether_dequant_q4_0", 18), (gguf.Q8_0, "aether_dequant_q8_0", 34),
                            (gguf.Q4_K, "aether_dequant_q4_k_m", 144), (gguf.Q6_K, "aether_dequant_q6_k", 210)):
        nb = 3
        blocks = R.integers(0, 256, size=(nb, size), dtype=np.uint8)
        scale_at = {gguf.Q4_0: [0], gguf.Q8_0: [0], gguf.Q4_K: [0, 2], gguf.Q6_K: [208]}[typ]
        for o in scale_at:
            blocks[:, o : o + 2] = np.frombuffer(np.full(nb, 0.05, np.float16).tobytes(), np.uint8).reshape(nb, 2)
        per = {gguf.Q4_0: 32, gguf.Q8_0: 32}.get(typ, 256)
        out = np.zeros(nb * per, np.float32)
        assert rt.call(name, rt.ptr(blocks), rt.ptr(out), nb) == 0
        want = gguf.dequantize(blocks.reshape(-1), typ, nb * per)
        if typ == gguf.Q4_0:  # the ABI's Q4_0 puts each byte's low / high values side by side
            want = want.reshape(nb, 2, 16).transpose(0, 2, 1).reshape(-1)
        np.testing.assert_allclose(out, want, rtol=1e-6, atol=1e-6)


def test_serving_structures():
    pool = rt.call("aether_pkv_new", 4, 16)
    got = [rt.call("aether_pkv_allocate", pool) for _ in range(4)]
    assert got == [0, 1, 2, 3] and rt.call("aether_pkv_allocate", pool) == -1
    rt.call("aether_pkv_touch", pool, 0)  # block 1 is now the least recently used
    assert rt.call("aether_pkv_evict_lru", pool) == 1 and rt.call("aether_pkv_n_allocated", pool) == 3
    rt.call("aether_pkv_destroy", pool)
    pool = rt.call("aether_pkv_new", 8, 4)
    s = rt.call("aether_batch_sched_new", pool, 4, 2)
    assert rt.call("aether_batch_sched_admit", s, 7, 6, 3) == 0  # 6 prompt tokens -> 2 blocks
    assert rt.call("aether_pkv_n_allocated", pool) == 2
    for t in range(3):
        assert rt.call("aether_batch_sched_record_token", s, 7, 100 + t) == 0
    # the position counts tokens emitted since admission (0 after admit), as the reference ABI does;
    # positions 1..3 stay inside the prompt's first block, so no block is added
    assert rt.call("aether_batch_sched_position", s, 7) == 3 and rt.call("aether_pkv_n_allocated", pool) == 2
    pt = rt.call("aether_batch_sched_pagetable_for", s, 7)
    assert rt.call("aether_pkv_pagetable_translate", pt, 5, 4) == rt.call("aether_pkv_pagetable_get", pt, 1) * 4 + 1
    assert rt.call("aether_batch_sched_reap", s) == 1 and rt.call("aether_pkv_n_allocated", pool) == 0
    cb = rt.call("aether_cb_new", 2)
    assert [rt.call("aether_cb_admit", cb, i) for i in range(3)] == [0, 0, -1]
    assert rt.call("aether_cb_step", cb) == 2 and rt.call("aether_cb_complete", cb, 0) == 0
    assert rt.call("aether_specdec_accept", 0.2, 0.1, 0.99) == 1 and rt.call("aether_specdec_accept", 0.1, 0.4, 0.5) == 0
    mm = rt.call("aether_mm_new")
    for name, mb in ((b"qwen", 15000), (b"bge", 1300)):
        rt.call("aether_mm_register", mm, name, len(name), mb)
    assert rt.call("aether_mm_lookup", mm, b"bge", 3) == 1 and rt.call("aether_mm_total_vram_mb", mm) == 16300
    rl = rt.call("aether_rl_new", 2, 2)
    assert [rt.call("aether_rl_check", rl, b"ip", 2, 0) for _ in range(3)] == [1, 1, 0]
    assert rt.call("aether_rl_check", rl, b"ip", 2, 500_000) == 1  # one token back after 0.5 s at 2/s


def test_observability(tmp_path):
    rt.call("aether_obs_counter_inc", b"aether_obs_requests", 19, 3)
    rt.call("aether_obs_counter_inc", b"aether_obs_requests", 19, 2)
    assert rt.call("aether_obs_counter_get", b"aether_obs_requests", 19) == 5
    buf = ctypes.create_string_buffer(4096)
    n = rt.call("aether_obs_dump_prometheus", buf, 4096)
    assert b"# TYPE aether_obs_requests counter\naether_obs_requests 5\n" in buf.raw[:n]
    rt.call("aether_prof_reset")
    before = rt.call("aether_prof_alloc_live")
    p = rt.call("aether_alloc_f32", 1000)
    assert rt.call("aether_prof_alloc_live") == before + 4000 and rt.call("aether_prof_alloc_peak") >= before + 4000
    rt.call("aether_free", p)
    assert rt.call("aether_prof_alloc_live") == before
    rt.call("aether_gpu_alloc_track", 1 << 20)
    rt.call("aether_oom_signal", 1)
    cwd = os.getcwd()
    os.chdir(tmp_path)
    try:
        assert rt.call("aether_crash_dump", b"train", 5, 17) == 0
        text = open(f"crash_{os.getpid()}_17.dump").read()
    finally:
        os.chdir(cwd)
        rt.call("aether_oom_signal", 0)
        rt.call("aether_gpu_free_track", 1 << 20)
    assert "label=train" in text and "step=17" in text and "oom_flag=1" in text
    t0 = rt.call("aether_timer_start")
    assert rt.call("aether_timer_elapsed_us", t0) >= 0


def test_tcp_transport_and_tools(tmp_path):
    import subprocess
    import threading

    lib = rt.lib()
    for name, res, args in (("aether_tcp_listen", ctypes.c_int64, [ctypes.c_int64]),
                            ("aether_tcp_listener_port", ctypes.c_int64, [ctypes.c_int64]),
                            ("aether_tcp_accept_one", ctypes.c_int64, [ctypes.c_int64]),
                            ("aether_tcp_connect", ctypes.c_int64, [ctypes.c_int64]),
                            ("aether_tcp_send_all", ctypes.c_int64, [ctypes.c_int64] * 3),
                            ("aether_tcp_recv_all", ctypes.c_int64, [ctypes.c_int64] * 3),
                            ("aether_tcp_stream_close", ctypes.c_int, [ctypes.c_int64]),
                            ("aether_tcp_close", ctypes.c_int, [ctypes.c_int64])):
        getattr(lib, name).restype, getattr(lib, name).argtypes = res, args
    lst = lib.aether_tcp_listen(0)  # ephemeral port
    port = lib.aether_tcp_listener_port(lst)
    assert lst >= 0 and port > 0
    got = {}

    def server():
        s = lib.aether_tcp_accept_one(lst)
        buf = np.zeros(1000, np.float32)
        got["n"] = lib.aether_tcp_recv_all(s, buf.ctypes.data, buf.nbytes)
        got["buf"] = buf
        lib.aether_tcp_stream_close(s)

    th = threading.Thread(target=server)
    th.start()
    c = lib.aether_tcp_connect(port)
    data = np.arange(1000, dtype=np.float32)
    assert lib.aether_tcp_send_all(c, data.ctypes.data, data.nbytes) == data.nbytes
    th.join(timeout=30)
    lib.aether_tcp_stream_close(c)
    lib.aether_tcp_close(lst)
    assert got["n"] == 4000 and np.array_equal(got["buf"], data)

    # star all-reduce across three processes
    bind = os.path.join(os.path.dirname(rt.LIB_PATH), "bin")
    p = 29000 + os.getpid() % 1000
    procs = [subprocess.Popen([os.path.join(bind, "aether-allreduce"), "--role", "server" if r == 0 else "client",
                               "--port", str(p), "--world-size", "3", "--rank", str(r), "--n", "8", "--value",
                               str(1 << r)], stdout=subprocess.PIPE, text=True) for r in range(3)]
    outs = [q.communicate(timeout=60)[0] for q in procs]
    assert all(q.returncode == 0 for q in procs) and all("sum[0..4]=7,7,7,7" in o for o in outs), outs

    # corpus preparation: copies bytes, refuses paths outside the working directory
    src = tmp_path / "raw.txt"
    src.write_text("hello aether\n")
    ok = subprocess.run([os.path.join(bind, "aether-prepare"), "--in", str(src), "--out", "data/corpus.bin"],
                        cwd=tmp_path, capture_output=True)
    assert ok.returncode == 0 and (tmp_path / "data" / "corpus.bin").read_bytes() == b"hello aether\n"
    bad = subprocess.run([os.path.join(bind, "aether-prepare"), "--in", str(src), "--out", "../escape.bin"],
                         cwd=tmp_path, capture_output=True)
    assert bad.returncode != 0


def test_distributed_layout_abi():
    """The reference's single-process layout checks: column-parallel linear =
    full matmul, pipelined affine blocks = sequential, ZeRO bytes, overlap,
    rank-k projection, FSDP round trip."""
    import numpy as np

    from aether_b200 import runtime as R

    rng = np.random.default_rng(0)
    x = rng.standard_normal((3, 5)).astype(np.float32)
    w = rng.standard_normal((5, 8)).astype(np.float32)
    out = np.zeros((3, 8), np.float32)
    assert R.call("aether_tp_simulate_column_parallel_linear_f32", R.ptr(x), R.ptr(w), R.ptr(out), 3, 5, 8, 4) == 0
    assert np.allclose(out, x @ w, atol=1e-5)
    assert R.call("aether_tp_simulate_column_parallel_linear_f32", R.ptr(x), R.ptr(w), R.ptr(out), 3, 5, 8, 3) == 3
    inp = rng.standard_normal((4, 6)).astype(np.float32)
    sc = rng.standard_normal(6).astype(np.float32)
    bi = rng.standard_normal(6).astype(np.float32)
    o = np.zeros_like(inp)
    assert R.call("aether_pp_simulate_2stage_forward_f32", R.ptr(inp), R.ptr(sc), R.ptr(bi), R.ptr(o), 4, 6, 6, 2) == 0
    want = inp.copy()
    for b in range(6):
        want = want * sc[b] + bi[b]
    assert np.allclose(o, want, atol=1e-4)
    z = [R.call("aether_zero_simulate_stage_bytes_f32", 1000, 4, s) for s in (1, 2, 3)]
    assert z == [4000 + 4000 + 8000 // 4, 4000 + 12000 // 4, 16000 // 4]
    assert R.call("aether_zero_simulate_stage_bytes_f32", 1000, 4, 4) == -2
    assert R.call("aether_overlap_simulate_overlapped_us", 30, 20) == 30
    assert R.call("aether_overlap_simulate_serial_us", 30, 20) == 50
    g = rng.standard_normal((4, 6)).astype(np.float32)
    rec = np.zeros_like(g)
    assert R.call("aether_grad_compress_lowrank_f32", R.ptr(g), R.ptr(rec), 4, 6, 2) == 0
    assert np.array_equal(rec[:, :2], g[:, :2]) and not rec[:, 2:].any()
    p = rng.standard_normal(12).astype(np.float32)
    q = np.zeros_like(p)
    assert R.call("aether_fsdp_simulate_shard_alltoall_f32", R.ptr(p), R.ptr(q), 12, 4) == 0
    assert np.array_equal(p, q)


def test_chat_template_subset_and_tool_call():
    import json

    from aether_b200 import runtime as R

    tpl = ("{% for m in messages %}<|im_start|>{{ m.role }}\n{{ m.content }}<|im_end|>\n{% endfor %}"
           "{% if add_generation_prompt %}<|im_start|>assistant\n{% endif %}")
    msgs = [("system", "be brief"), ("user", "hi")]
    out = R.render_template(tpl, msgs, {"add_generation_prompt": "true"})
    assert out == "<|im_start|>system\nbe brief<|im_end|>\n<|im_start|>user\nhi<|im_end|>\n<|im_start|>assistant\n"
    assert R.render_template(tpl, msgs, {"add_generation_prompt": "false"}).endswith("hi<|im_end|>\n")
    assert R.render_template("[{{ missing }}]", []) == "[]"
    for bad in ("{% for m in messages %}x", "{% endif %}", "{% while x %}{% endwhile %}", "{{ x"):
        try:
            R.render_template(bad, msgs)
            raise AssertionError(bad)
        except ValueError:
            pass
    call = json.loads(R.render_tool_call("get_weather", '{"city": "Paris"}'))
    assert call == {"type": "function", "function": {"name": "get_weather", "arguments": '{"city": "Paris"}'}}


def test_aether_train_data_parallel_in_process_equals_multi_process(tmp_path):
    """aether-train --world-size 2: the in-process replicas and two processes
    meeting over TCP train the same model (byte-identical checkpoints)."""
    import json
    import os
    import socket
    import subprocess

    from aether_b200 import runtime as R

    R.lib()
    exe = os.path.join(os.path.dirname(R.LIB_PATH), "bin", "aether-train")
    common = ["--world-size", "2", "--steps", "12", "--batch", "4", "--log-every", "100", "--gen", "4"]
    a = subprocess.run([exe, *common, "--out", str(tmp_path / "inproc")], capture_output=True, text=True, timeout=300)
    assert a.returncode == 0, a.stderr
    assert "replicas identical" in a.stderr
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    env = dict(os.environ, AETHER_COMM_ADDR=f"127.0.0.1:{port}")
    procs = [subprocess.Popen([exe, *common, "--rank", str(r), "--out", str(tmp_path / f"mp{r}")], env=env,
                              stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True) for r in range(2)]
    outs = [p.communicate(timeout=300) for p in procs]
    assert all(p.returncode == 0 for p in procs), [o[1][-500:] for o in outs]
    assert json.loads(outs[0][0])["final_loss"] == json.loads(a.stdout)["final_loss"]
    w_in = open(str(tmp_path / "inproc") + ".weights", "rb").read()
    w_mp = open(str(tmp_path / "mp0") + ".weights", "rb").read()
    assert w_in == w_mp
    assert not os.path.exists(str(tmp_path / "mp1") + ".weights")  # rank 0 writes the checkpoint
