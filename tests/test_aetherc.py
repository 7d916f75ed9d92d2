"""aetherc, the Aether compiler of this package: programs lower to C, link
against libaether_rt / libaether_dev and their exit codes are checked (the
`// expect: exit=N` header of each program). Tensor methods become device-ABI
calls with shape integers from the tensor types, the matmul + in-place GELU
pair fuses into one call, and errors carry AE codes. When the reference's
runtime witnesses are on disk, the CPU ones are compiled and run as well."""
import json
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
AEC = os.path.join(ROOT, "aether_b200", "bin", "aetherc")
PROGS = os.path.join(ROOT, "tests", "aether")
REF_WITNESSES = "/root/reference/tests/runtime"

pytestmark = pytest.mark.skipif(not os.path.exists(AEC), reason="aetherc not built")


def _compile(src, out, *extra):
    return subprocess.run([AEC, src, "-o", out, *extra], capture_output=True, text=True, timeout=120)


def _expect(path):
    m = re.search(r"//\s*expect:\s*exit\s*=\s*(-?\d+)", open(path, errors="replace").read())
    return int(m.group(1)) & 255


def _run_program(path, tmp_path):
    out = str(tmp_path / os.path.basename(path)[: -len(".aether")])
    harness = re.search(r"build-mode:\s*aether-bin-test", open(path).read()) is not None
    c = _compile(path, out, *(["--test"] if harness else []))
    assert c.returncode == 0, c.stderr
    r = subprocess.run([out], capture_output=True, text=True, timeout=300, cwd=str(tmp_path))
    assert r.returncode == _expect(path), (path, r.returncode, r.stdout[-2000:], r.stderr[-2000:])
    if harness:  # one line per test, then the summary
        assert "PASS adds" in r.stdout and "FAIL fails_on_purpose" in r.stdout and "1 of 3 tests FAILED" in r.stdout


@pytest.mark.parametrize("name", sorted(f for f in os.listdir(PROGS) if f.startswith("cpu_")))
def test_cpu_programs(name, tmp_path):
    _run_program(os.path.join(PROGS, name), tmp_path)


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(f for f in os.listdir(PROGS) if f.startswith("gpu_")))
def test_gpu_training_programs(name, tmp_path):
    """Training on the device through tensor methods; the loss must fall."""
    _run_program(os.path.join(PROGS, name), tmp_path)


def test_tensor_methods_lower_to_shaped_abi_calls():
    c = subprocess.run([AEC, os.path.join(PROGS, "gpu_train_mlp.aether"), "--emit=c"], capture_output=True,
                       text=True, timeout=60)
    assert c.returncode == 0, c.stderr
    code = c.stdout
    # x: [16, 32] @ w1: [32, 64] -> act, fused with the in-place gelu that followed it
    assert re.search(r"aether_op_matmul_gelu_f32_cuda\(x_\d+, .*w1_\d+.*act_\d+.*, 16, 32, 64\)", code)
    assert "fused 1 matmul+gelu" in c.stderr
    assert re.search(r"aether_op_cross_entropy_f32_cuda\(logits_\d+, .*labels_\d+.*probs_\d+.*, 16, 5\)", code)
    assert re.search(r"aether_op_matmul_backward_lhs_f32_cuda\(dlogits_\d+, .*w2_\d+.*dact_\d+.*, 16, 64, 5\)", code)
    assert re.search(r"aether_op_adamw_step_f32_cuda\(w1_\d+, .*0\.01f.*, 2048\)", code)  # n = numel(w1)
    unfused = subprocess.run([AEC, os.path.join(PROGS, "gpu_train_mlp.aether"), "--emit=c", "--no-fuse"],
                             capture_output=True, text=True, timeout=60).stdout
    assert "aether_op_matmul_gelu_f32_cuda(x_" not in unfused and "aether_op_gelu_f32_cuda(act_" in unfused


@pytest.mark.parametrize("src,code", [
    ("fn main() -> i32 { let t: Tensor<f32, [4, 3]>; let w: Tensor<f32, [2, 5]>; "
     "let y: Tensor<f32, [4, 5]>; t.matmul(&w, &mut y); 0 }", "AE0554"),          # inner dims differ
    ("fn main() -> i32 { let t: Tensor<f32, [4]>; t.transpose(); 0 }", "AE0551"),  # unknown method
    ("fn main() -> i32 { let x: i32 = 1; x.gelu(); 0 }", "AE0550"),              # not a tensor
    ("fn main() -> i32 { undefined_fn(1) }", "AE0540"),
    ("fn main() -> i32 { let t: Tensor<f32, [0]>; 0 }", "AE0521"),
    ("fn main() -> i32 { let v = twice!(1); 0 }", "AE0500"),                    # an undefined macro
])
def test_codegen_diagnostics_carry_codes(tmp_path, src, code):
    """Errors found while lowering to C (this compiler's own AE05xx codes)."""
    f = tmp_path / "bad.aether"
    f.write_text(src)
    r = subprocess.run([AEC, str(f), "--emit=c", "-o", str(tmp_path / "bad.c"), "--json-errors"],
                       capture_output=True, text=True, timeout=60)
    assert r.returncode == 1
    d = json.loads(r.stderr.strip().splitlines()[-1])
    assert d["code"] == code and d["line"] >= 1, d


# `--check` programs and the code each must fail with (None: must check clean).
CHECK_CASES = [
    ("fn main() -> i32 { return 0; }", None),
    ("#[autodiff]\n#[distributed(world_size=4, backend=\"nccl\")]\nfn step() { let h = encode(); "
     "let l = h.mse(target); l.backward(); }", None),                              # names resolve at codegen only
    ("pub struct Pair<A, B> { a: A, b: B, }\nconst N: i64 = 64;\n"
     "extern fn mm(x: &Tensor<f32, [R, C]>, y: &mut Tensor<f32, [C, R]>) -> i32;\n"
     "fn go(x: &Tensor<f32, [R, C]>, y: &mut Tensor<f32, [C, R]>) { mm(x, y); }", None),
    ("fn k() { parallel for i in 0..32 { warp { let v = 1; } block { let w = 2; } } "
     "if 2 > 1 { let a = 1; } else { let b = 2; } }", None),
    ("fn main() -> i64 { let v: i64 = 9; let p = &v; let q = &v; let r = &v; v }", None),
    ("fn main() -> i64 { let mut v: i64 = 1; let p = &mut v; *p = 2; let q = &mut v; *q = 3; v }", None),
    ("trait Area { fn area(&self) -> i32; fn twice(&self) -> i32 { 2 } }\nstruct Sq { s: i32 }\n"
     "impl Area for Sq { fn area(&self) -> i32 { 1 } }\nfn main() -> i32 { 0 }", None),
    ("extern fn f(a: i32) -> i32 { 0 }", "AE0002"),                               # extern with a body
    ("fn g() { h(1 2); }", "AE0002"),
    ("fn main() -> i32 { 0", "AE0002"),
    ("fn main() -> i32 { let s = \"open; 0 }", "AE0001"),
    ("use no_such_module;\nfn main() -> i32 { 0 }", "AE0003"),
    ("fn main() -> i64 { let mut v: i64 = 1; let p = &mut v; let q = &mut v; *p = 2; *q = 3; v }", "AE0200"),
    ("fn main() -> i64 { let mut v: i64 = 1; let p = &mut v; let q = &v; let t = *q; *p = 2; t }", "AE0201"),
    ("fn main() -> i64 { let mut v: i64 = 1; f(&mut v, &v) }\nfn f(a: &mut i64, b: &i64) -> i64 { 0 }", "AE0201"),
    ("trait Area { fn area(&self) -> i32; }\nstruct Sq { s: i32 }\nimpl Area for Sq { }\n"
     "fn main() -> i32 { 0 }", "AE0210"),
    ("struct Sq { s: i32 }\nimpl Paint for Sq { fn paint(&self) -> i32 { 0 } }\nfn main() -> i32 { 0 }", "AE0211"),
    ("trait Base { fn b(&self) -> i32; }\ntrait Top: Base { fn t(&self) -> i32; }\nstruct C { i: i32 }\n"
     "impl Top for C { fn t(&self) -> i32 { 0 } }\nfn main() -> i32 { 0 }", "AE0212"),
    ("fn main() -> i32 { let x: i32 = 2.5; x }", "AE0220"),
    ("fn main() -> i32 { let f: f64 = 2; 0 }", "AE0220"),
    ("fn main() -> i32 { let b: bool = 1; 0 }", "AE0220"),
    ("fn half(v: i64) -> i64 { v / 2 }\nfn main() -> i32 { half(1.5) as i32 }", "AE0221"),
    ("fn r() -> i64 { 0.5 }\nfn main() -> i32 { 0 }", "AE0222"),
    ("fn r() -> i64 { return 0.5; }\nfn main() -> i32 { 0 }", "AE0222"),
    ("fn main() -> i32 { let mut n: i32 = 0; n = 0.5; n }", "AE0224"),
]


@pytest.mark.parametrize("src,code", CHECK_CASES)
def test_check_mode(tmp_path, src, code):
    """`--check` runs the reference's front-end checks: parse, `use`, traits,
    scalar type conflicts and borrows, with the reference's AE codes."""
    f = tmp_path / "p.aether"
    f.write_text(src)
    r = subprocess.run([AEC, str(f), "--check", "--json-errors"], capture_output=True, text=True, timeout=60)
    if code is None:
        assert r.returncode == 0, r.stderr
        return
    assert r.returncode == 1, (src, r.stderr)
    d = json.loads(r.stderr.strip().splitlines()[-1])
    assert d["code"] == code and d["line"] >= 1, (src, d)


REF_CONFORMANCE = "/root/reference/tests/aether"


@pytest.mark.skipif(not os.path.isdir(REF_CONFORMANCE), reason="reference conformance suite not on this machine")
def test_reference_conformance_suite():
    """The reference's conformance suite, run the way its audit tool runs it
    (tools/audit/src/conformance.rs): every file under positive/ must
    `--check` clean, every negative/expect_AE####_*.aether must fail with
    that code."""
    bad = []
    for kind in ("positive", "negative"):
        d = os.path.join(REF_CONFORMANCE, kind)
        for name in sorted(os.listdir(d)):
            if not name.endswith(".aether"):
                continue
            r = subprocess.run([AEC, os.path.join(d, name), "--check", "--json-errors"], capture_output=True,
                               text=True, timeout=60)
            if kind == "positive":
                if r.returncode != 0:
                    bad.append((name, r.stderr[-300:]))
                continue
            want = re.search(r"_(AE\d{4})_", name).group(1)
            if r.returncode == 0 or f'"code":"{want}"' not in r.stderr:
                bad.append((name, r.stderr[-300:]))
    assert not bad, bad


@pytest.mark.skipif(not os.path.isdir(REF_WITNESSES), reason="reference witnesses not on this machine")
def test_reference_runtime_witnesses(tmp_path):
    """Witnesses in the language subset compile and the CPU ones exit with
    their expected code; every `cuda_train_*` GPU training witness compiles
    (training on the device is exercised by this package's own programs)."""
    passed, cuda_compiled, train_missing, wrong = 0, 0, [], []
    (tmp_path / "target" / "audit-tmp").mkdir(parents=True)  # where the file-writing witnesses put their output
    for name in sorted(os.listdir(REF_WITNESSES)):
        if not name.endswith(".aether"):
            continue
        path = os.path.join(REF_WITNESSES, name)
        text = open(path, errors="replace").read()
        if not re.search(r"//\s*expect:\s*exit", text):
            continue
        cuda = "requires: cuda" in text
        out = str(tmp_path / name[:-7])
        extra = ["--test"] if re.search(r"build-mode:\s*aether-bin-test", text) else []  # the #[test] harness
        if _compile(path, out, *extra).returncode != 0:
            if name.startswith("cuda_train_"):
                train_missing.append(name)
            continue
        if cuda:
            cuda_compiled += 1
            continue
        r = subprocess.run([out], capture_output=True, text=True, timeout=60, cwd=str(tmp_path))
        if r.returncode == _expect(path):
            passed += 1
        else:
            wrong.append(name)
    assert not train_missing, train_missing
    assert cuda_compiled >= 21 and passed >= 270, (cuda_compiled, passed, wrong)
