"""The .aether developer tools (csrc/tools/aether_tools.cpp): formatter, linter,
doc index, repository audit and witness stamper, run as their command lines."""
import json
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "aether_b200", "bin")

pytestmark = pytest.mark.skipif(not os.path.exists(os.path.join(BIN, "aether-tools")), reason="tools not built")


def run(tool, *args, cwd=None, stdin=None):
    return subprocess.run([os.path.join(BIN, tool), *args], capture_output=True, text=True, cwd=cwd, input=stdin,
                          timeout=600)


MESSY = 'fn main() -> i32 {\n\tlet s: i64 = 3;   \n\n\n\nlet t = "a\tb";\n  s as i32\n}\n\n\n'


def test_fmt_normalises_and_is_idempotent(tmp_path):
    p = tmp_path / "m.aether"
    p.write_text(MESSY)
    r = run("aetherfmt", "--check", str(p))
    assert r.returncode == 1 and str(p) in r.stdout
    assert p.read_text() == MESSY  # --check writes nothing
    assert run("aetherfmt", str(p)).returncode == 0
    got = p.read_text()
    assert "\t" not in got.replace('"a\tb"', "")  # tabs outside strings replaced
    assert '"a\tb"' in got  # the tab inside the string literal kept
    assert "\n\n\n" not in got and got.endswith("}\n") and not any(l != l.rstrip() for l in got.splitlines())
    assert run("aetherfmt", "--check", str(p)).returncode == 0
    run("aetherfmt", "--reindent", str(p))
    lines = p.read_text().splitlines()
    assert lines[1].startswith("    let s") and lines[-2].startswith("    s as") and lines[-1] == "}"
    assert run("aetherfmt", "-", stdin=MESSY).stdout == got


def test_clippy_codes(tmp_path):
    src = ("const BIG: i64 = 10000;\nfn f() {}\nfn main() -> i32 {\n\tlet a: i64 = 5000;  \n"
           "    let _ = f();\n    let b = x_7000 + 0x2000;\n    let s = \"123456\";\n    // FIXME: later\n"
           "    let c = 2.50000;\n    0\n}\n" + "// " + "x" * 130 + "\n")
    p = tmp_path / "l.aether"
    p.write_text(src)
    r = run("aetherclippy", str(p))
    assert r.returncode == 1
    codes = [(int(l.split(":")[1]), l.split()[1]) for l in r.stdout.splitlines()]
    assert (2, "AC007") in codes
    assert (4, "AC001") in codes and (4, "AC002") in codes and (4, "AC004") in codes
    assert (5, "AC003") in codes
    assert (6, "AC004") in codes  # 0x2000 = 8192; x_7000 is an identifier
    assert sum(1 for ln, c in codes if ln == 6 and c == "AC004") == 1
    assert (8, "AC005") in codes and (12, "AC006") in codes
    assert not any(ln in (1, 7, 9) for ln, _ in codes)  # const decl, string literal, float
    r = run("aetherclippy", "--allow", "AC001,AC002,AC003,AC004,AC005,AC006,AC007", str(p))
    assert r.returncode == 0 and r.stdout == ""


def test_doc_index(tmp_path):
    p = tmp_path / "d.aether"
    p.write_text("/// Adds two numbers.\n/// Exactly.\npub fn add(a: i64, b: i64) -> i64 { a + b }\n\n"
                 "/// A vector.\nstruct V3 { x: i64 }\n/// floating\n\nfn nodoc() {}\n"
                 "/// Runtime entry.\nextern fn aether_print_i64(x: i64);\n")
    md = run("aetherdoc", str(p)).stdout
    assert "### `fn add` (line 3)" in md and "Adds two numbers.\nExactly." in md
    assert "### `struct V3`" in md and "nodoc" not in md and "floating" not in md
    assert "### `extern fn aether_print_i64`" in md
    html = run("aetherdoc", "--html", str(p)).stdout
    assert html.startswith("<!doctype html>") and "<code>fn add</code>" in html


def test_audit_json():
    r = run("aether-audit", "--json", "--root", ROOT, "--only", "abi")
    rep = json.loads(r.stdout)
    assert r.returncode == 0, rep["errors"]
    assert rep["abi"]["libaether_rt.so"]["missing"] == 0 and rep["abi"]["libaether_rt.so"]["defined"] > 300
    rep = json.loads(run("aether-audit", "--json", "--root", ROOT, "--only", "sloc").stdout)
    assert rep["sloc"]["csrc"]["code"] > 1000 and "aether_b200/parallel" in rep["sloc"]


def test_audit_runs_witnesses():
    r = run("aether-audit", "--json", "--root", ROOT, "--only", "witnesses")
    rep = json.loads(r.stdout)
    cpu = [w for w in rep["witnesses"] if w["name"].startswith("cpu_")]
    assert cpu and all(w["status"] == "pass" for w in cpu), rep


def test_audit_runs_conformance():
    """The package's conformance suite: positive files check clean, each
    negative file fails with the code its name carries."""
    r = run("aether-audit", "--json", "--root", ROOT, "--only", "conformance")
    rep = json.loads(r.stdout)
    assert r.returncode == 0, rep["errors"]
    names = [c["name"] for c in rep["conformance"]]
    assert len(names) >= 18 and all(c["status"] == "pass" for c in rep["conformance"]), rep
    assert sum(n.startswith("expect_AE02") for n in names) >= 9


def test_witness_stamper(tmp_path):
    d = tmp_path / "w"
    d.mkdir()
    (d / "a.aether").write_text("// expect: exit=0\nfn main() -> i32 { 0 }\n")
    (d / "b.aether").write_text("// expect: exit=42\n// roadmap: P1.1\nfn main() -> i32 { 42 }\n")
    tags = tmp_path / "tags.txt"
    tags.write_text("# file tag\na.aether P2.1\nb.aether P1.1\nb.aether P3.4\n")
    fresh = tmp_path / "fresh.txt"
    fresh.write_text("=== new_one.aether\n// expect: exit=7\nfn main() -> i32 { 7 }\n")
    assert run("witness-stamper", "--dir", str(d), "--tags", str(tags), "--fresh", str(fresh), "--check").returncode == 1
    assert not (d / "new_one.aether").exists()
    assert run("witness-stamper", "--dir", str(d), "--tags", str(tags), "--fresh", str(fresh)).returncode == 0
    assert (d / "a.aether").read_text().splitlines()[1] == "// roadmap: P2.1"
    assert (d / "b.aether").read_text().splitlines()[1] == "// roadmap: P1.1, P3.4"
    assert (d / "new_one.aether").read_text() == "// expect: exit=7\nfn main() -> i32 { 7 }\n"
    before = {f: (d / f).read_text() for f in os.listdir(d)}
    r = run("witness-stamper", "--dir", str(d), "--tags", str(tags), "--fresh", str(fresh), "--check")
    assert r.returncode == 0 and r.stdout == ""  # idempotent
    assert {f: (d / f).read_text() for f in os.listdir(d)} == before
