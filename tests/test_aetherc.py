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
    c = _compile(path, out)
    assert c.returncode == 0, c.stderr
    r = subprocess.run([out], capture_output=True, text=True, timeout=300, cwd=str(tmp_path))
    assert r.returncode == _expect(path), (path, r.returncode, r.stdout[-2000:], r.stderr[-2000:])


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
     "let y: Tensor<f32, [4, 5]>; t.matmul(&w, &mut y); 0 }", "AE0254"),          # inner dims differ
    ("fn main() -> i32 { let t: Tensor<f32, [4]>; t.transpose(); 0 }", "AE0251"),  # unknown method
    ("fn main() -> i32 { let x: i32 = 1; x.gelu(); 0 }", "AE0250"),              # not a tensor
    ("fn main() -> i32 { undefined_fn(1) }", "AE0240"),
    ("fn main() -> i32 { let t: Tensor<f32, [0]>; 0 }", "AE0221"),
    ("struct S { a: i32 }\nfn main() -> i32 { 0 }", "AE0100"),
])
def test_diagnostics_carry_codes(tmp_path, src, code):
    f = tmp_path / "bad.aether"
    f.write_text(src)
    r = subprocess.run([AEC, str(f), "--check", "--json-errors"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 1
    d = json.loads(r.stderr.strip().splitlines()[-1])
    assert d["code"] == code and d["line"] >= 1, d


@pytest.mark.skipif(not os.path.isdir(REF_WITNESSES), reason="reference witnesses not on this machine")
def test_reference_runtime_witnesses(tmp_path):
    """Witnesses in the language subset compile and the CPU ones exit with
    their expected code; every `cuda_train_*` GPU training witness compiles
    (training on the device is exercised by this package's own programs)."""
    passed, cuda_compiled, train_missing, wrong = 0, 0, [], []
    for name in sorted(os.listdir(REF_WITNESSES)):
        if not name.endswith(".aether"):
            continue
        path = os.path.join(REF_WITNESSES, name)
        text = open(path, errors="replace").read()
        if not re.search(r"//\s*expect:\s*exit", text):
            continue
        cuda = "requires: cuda" in text
        out = str(tmp_path / name[:-7])
        if _compile(path, out).returncode != 0:
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
    assert cuda_compiled >= 21 and passed >= 180, (cuda_compiled, passed, wrong)
