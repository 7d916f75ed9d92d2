"""The systems layer of libaether_rt: files, environment, processes, threads,
atomics, the poll-based executor, JIT pages and the handle containers, driven
through the C ABI as a compiled program would."""
import ctypes as C
import os
import platform

import pytest

from aether_b200 import runtime as rt

L = C.c_int64
CB = C.CFUNCTYPE(C.c_int64, C.c_int64)


def _lib():
    lb = rt.lib()
    for name in ("read_file", "file_size_last", "file_size", "path_exists", "is_dir", "copy_file", "read_dir_count",
                 "env_var_i64", "process_run", "thread_spawn", "thread_join", "atomic_load_i64",
                 "atomic_fetch_add_i64", "atomic_cas_i64", "block_on", "executor_run", "alloc_executable",
                 "call_jit_i64", "avx2_witness_arr", "vec_i64_new", "vec_i64_len", "vec_i64_get", "vec_i64_as_ptr",
                 "vec_f32_new", "vec_f32_len", "vec_f32_as_ptr", "string_new", "string_len", "string_byte_at",
                 "string_as_ptr", "hashmap_i64_new", "hashmap_i64_get", "hashmap_i64_contains", "hashmap_i64_remove",
                 "hashmap_i64_len", "rc_i64_new", "rc_i64_clone", "rc_i64_get", "rc_i64_strong_count", "box_i64_new",
                 "box_i64_get", "chan_i64_new", "chan_i64_len", "iter_vec_i64_new", "iter_vec_i64_next",
                 "iter_vec_i64_map_double", "iter_vec_i64_filter_positive", "iter_vec_i64_take",
                 "iter_vec_i64_collect", "iter_vec_i64_fold_sum", "test_f32_to_i64", "test_f64_to_i64"):
        getattr(lb, "aether_" + name).restype = L
    lb.aether_test_add_f32.restype = C.c_float
    lb.aether_test_add_f32.argtypes = [C.c_float, C.c_float]
    lb.aether_test_add_f64.restype = C.c_double
    lb.aether_test_add_f64.argtypes = [C.c_double, C.c_double]
    lb.aether_test_mix_if.restype = C.c_float
    lb.aether_test_mix_if.argtypes = [C.c_int, C.c_float, C.c_int]
    lb.aether_test_f32_to_i64.argtypes = [C.c_float]
    lb.aether_test_f64_to_i64.argtypes = [C.c_double]
    return lb


def _s(x: str):
    return C.c_char_p(x.encode())


def _addr(buf):
    return C.cast(buf, C.c_void_p).value


def test_files_env_process(tmp_path):
    lb = _lib()
    d = str(tmp_path / "a" / "b" / "c")
    assert lb.aether_create_dir_all(_s(d)) == 0 and lb.aether_is_dir(_s(d)) == 1
    f = os.path.join(d, "x.bin")
    data = os.urandom(70000)
    assert lb.aether_write_file(_s(f), C.c_char_p(data), L(len(data))) == 0
    assert lb.aether_path_exists(_s(f)) == 1 and lb.aether_file_size(_s(f)) == len(data)
    p = lb.aether_read_file(_s(f))
    assert p and lb.aether_file_size_last() == len(data) and C.string_at(p, len(data)) == data
    lb.aether_free_bytes(L(p), L(len(data)))
    g = os.path.join(d, "y.bin")
    assert lb.aether_copy_file(_s(f), _s(g)) == len(data)
    h = os.path.join(d, "z.bin")
    assert lb.aether_rename(_s(g), _s(h)) == 0 and lb.aether_path_exists(_s(g)) == 0
    assert lb.aether_read_dir_count(_s(d)) == 2
    assert lb.aether_remove_file(_s(h)) == 0 and lb.aether_read_dir_count(_s(d)) == 1
    assert lb.aether_read_file(_s(os.path.join(d, "missing"))) == 0
    assert lb.aether_file_size(_s(os.path.join(d, "missing"))) == -1

    lb.aether_env_set(_s("AETHER_T_INT"), _s(" 1234 "))
    assert lb.aether_env_var_i64(_s("AETHER_T_INT")) == 1234
    assert lb.aether_process_run(_s('test "$AETHER_T_INT" = " 1234 "')) == 0  # children inherit it
    lb.aether_env_set(_s("AETHER_T_INT"), _s("12x"))
    assert lb.aether_env_var_i64(_s("AETHER_T_INT")) == -1
    assert lb.aether_env_var_i64(_s("AETHER_T_UNSET_VAR")) == -1
    assert lb.aether_process_run(_s("exit 7")) == 7
    assert lb.aether_process_run(_s(f"test -d {d}")) == 0


def test_threads_atomics_executor():
    lb = _lib()
    counter = C.c_int64(0)

    @CB
    def work(arg):
        for _ in range(1000):
            lb.aether_atomic_fetch_add_i64(L(C.addressof(counter)), L(1))
        return arg * 3

    hs = [lb.aether_thread_spawn(L(C.cast(work, C.c_void_p).value), L(i)) for i in range(4)]
    assert all(hs)
    assert [lb.aether_thread_join(L(h)) for h in hs] == [0, 3, 6, 9]
    assert lb.aether_atomic_load_i64(L(C.addressof(counter))) == 4000
    assert lb.aether_atomic_cas_i64(L(C.addressof(counter)), L(4000), L(5)) == 4000 and counter.value == 5
    assert lb.aether_atomic_cas_i64(L(C.addressof(counter)), L(4000), L(9)) == 5 and counter.value == 5

    # a future: [poll_fn, pc, result]; ready on the third poll with result 42
    fut = (C.c_int64 * 3)()

    @CB
    def poll(addr):
        f = (C.c_int64 * 3).from_address(addr)
        f[1] += 1
        if f[1] < 3:
            return 0
        f[2] = 42
        return 1

    fut[0] = C.cast(poll, C.c_void_p).value
    assert lb.aether_block_on(L(C.addressof(fut))) == 42 and fut[1] == 3

    # two tasks needing 2 and 4 polls interleave round-robin: 2 + 4 polls in all
    order = []
    need = {1: 2, 2: 4}
    seen = {1: 0, 2: 0}

    @CB
    def task(state):
        order.append(state)
        seen[state] += 1
        return 1 if seen[state] >= need[state] else 0

    tasks = (C.c_int64 * 4)(C.cast(task, C.c_void_p).value, 1, C.cast(task, C.c_void_p).value, 2)
    assert lb.aether_executor_run(L(C.addressof(tasks)), L(2)) == 6
    assert order == [1, 2, 1, 2, 2, 2]


@pytest.mark.skipif(platform.machine() != "x86_64", reason="x86-64 machine code")
def test_jit_page_and_probes():
    lb = _lib()
    code = bytes([0x48, 0xC7, 0xC0, 0x2A, 0, 0, 0, 0xC3])  # mov rax, 42 ; ret
    p = lb.aether_alloc_executable(L(4096))
    assert p
    C.memmove(p, code, len(code))
    assert lb.aether_call_jit_i64(L(p)) == 42
    lb.aether_free_executable(L(p), L(4096))
    a = lb.aether_avx2_witness_arr(L(7), L(64))
    vals = (C.c_float * 64).from_address(a)
    assert all(0.0 <= v < 4.0 for v in vals) and len(set(vals)) > 32
    b = lb.aether_avx2_witness_arr(L(7), L(64))
    assert list((C.c_float * 64).from_address(b)) == list(vals)
    assert lb.aether_test_add_f32(1.5, 2.25) == 3.75 and lb.aether_test_add_f64(1e300, 1e300) == 2e300
    assert lb.aether_test_f32_to_i64(-3.7) == -3 and lb.aether_test_f64_to_i64(2.0**40) == 2**40
    assert lb.aether_test_mix_if(3, 0.5, 4) == 3.5  # (i + j) * f


def test_containers_and_iterators():
    lb = _lib()
    v = lb.aether_vec_i64_new()
    for x in (5, -2, 7, 0, 9, -1):
        assert lb.aether_vec_i64_push(L(v), L(x)) == 0
    assert lb.aether_vec_i64_len(L(v)) == 6 and lb.aether_vec_i64_get(L(v), L(2)) == 7
    assert lb.aether_vec_i64_get(L(v), L(99)) == 0 and lb.aether_vec_i64_set(L(v), L(99), L(1)) == -1
    assert lb.aether_vec_i64_set(L(v), L(1), L(-3)) == 0
    assert list((C.c_int64 * 6).from_address(lb.aether_vec_i64_as_ptr(L(v)))) == [5, -3, 7, 0, 9, -1]
    # filter(> 0) -> map(x2) -> take(2) -> collect
    it = lb.aether_iter_vec_i64_take(L(lb.aether_iter_vec_i64_map_double(
        L(lb.aether_iter_vec_i64_filter_positive(L(lb.aether_iter_vec_i64_new(L(v))))))), L(2))
    out = lb.aether_iter_vec_i64_collect(L(it))
    assert [lb.aether_vec_i64_get(L(out), L(i)) for i in range(lb.aether_vec_i64_len(L(out)))] == [10, 14]
    assert lb.aether_iter_vec_i64_fold_sum(L(lb.aether_iter_vec_i64_new(L(v)))) == 17
    it = lb.aether_iter_vec_i64_new(L(v))
    x = C.c_int64()
    got = []
    while lb.aether_iter_vec_i64_next(L(it), L(C.addressof(x))) == 1:
        got.append(x.value)
    assert got == [5, -3, 7, 0, 9, -1] and lb.aether_iter_vec_i64_free(L(it)) == 0
    assert lb.aether_iter_vec_i64_new(L(10**6)) == -1
    assert lb.aether_vec_i64_free(L(v)) == 0 and lb.aether_vec_i64_free(L(v)) == -1

    f = lb.aether_vec_f32_new()
    for val in (1.5, -2.0):
        bits = int.from_bytes(C.c_float(val), "little")
        assert lb.aether_vec_f32_push(L(f), L(bits)) == 0
    assert list((C.c_float * 2).from_address(lb.aether_vec_f32_as_ptr(L(f)))) == [1.5, -2.0]

    s = lb.aether_string_new()
    for ch in b"hi!":
        lb.aether_string_push_byte(L(s), L(ch))
    assert lb.aether_string_len(L(s)) == 3 and lb.aether_string_byte_at(L(s), L(1)) == ord("i")
    assert C.string_at(lb.aether_string_as_ptr(L(s))) == b"hi!"

    m = lb.aether_hashmap_i64_new()
    for k in range(100):
        lb.aether_hashmap_i64_insert(L(m), L(k), L(k * k))
    assert lb.aether_hashmap_i64_len(L(m)) == 100 and lb.aether_hashmap_i64_get(L(m), L(9)) == 81
    assert lb.aether_hashmap_i64_remove(L(m), L(9)) == 81 and lb.aether_hashmap_i64_contains(L(m), L(9)) == 0
    assert lb.aether_hashmap_i64_get(L(m), L(12345)) == 0

    r = lb.aether_rc_i64_new(L(77))
    assert lb.aether_rc_i64_clone(L(r)) == r and lb.aether_rc_i64_strong_count(L(r)) == 2
    assert lb.aether_rc_i64_drop(L(r)) == 0 and lb.aether_rc_i64_get(L(r)) == 77
    assert lb.aether_rc_i64_drop(L(r)) == 0 and lb.aether_rc_i64_strong_count(L(r)) == 0
    b = lb.aether_box_i64_new(L(3))
    assert lb.aether_box_i64_set(L(b), L(4)) == 0 and lb.aether_box_i64_get(L(b)) == 4

    ch = lb.aether_chan_i64_new()
    for k in (1, 2, 3):
        lb.aether_chan_i64_send(L(ch), L(k))
    assert lb.aether_chan_i64_len(L(ch)) == 3
    got = []
    while lb.aether_chan_i64_recv(L(ch), L(C.addressof(x))) == 1:
        got.append(x.value)
    assert got == [1, 2, 3] and lb.aether_chan_i64_free(L(ch)) == 0
