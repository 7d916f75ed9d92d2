"""aether-asm (csrc/asm/aether_asm.cpp) and the no-libc runtime
(csrc/asm/runtime_nolibc.s): encodings checked byte for byte against GNU as
where it is installed, ELF objects linked by the system linker and by C code,
static executables built with no linker at all, and line-numbered errors."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ASM = os.path.join(ROOT, "aether_b200", "bin", "aether-asm")
RUNTIME = os.path.join(ROOT, "csrc", "asm", "runtime_nolibc.s")
LINREG = os.path.join(ROOT, "tests", "asm", "linreg.s")

pytestmark = pytest.mark.skipif(not os.path.exists(ASM), reason="aether-asm not built")
HAVE_GAS = shutil.which("as") is not None and shutil.which("objcopy") is not None
HAVE_LD = shutil.which("ld") is not None

FORMS = """movq %rax, %rbx
movq %r8, %r15
movl %eax, %r9d
movq 8(%rsp), %rax
movq %rax, -16(%rbp)
movq 0(%rbp), %rcx
movq (%r12), %r13
movq (%r13), %rax
movq 1024(%rax,%rbx,8), %rdx
movq (%rax,%r9,4), %r10
movq $5, %rax
movq $-1, %rcx
movl $123456, %eax
movq $3, 16(%rsp)
movl $7, (%rdi)
movabsq $0x123456789abc, %r9
movb %sil, 3(%rsp)
movb (%rsi), %r9b
movb $10, (%rax)
movb $1, %r10b
leaq (%rax,%rcx,2), %rdx
addq $1, %rax
addq $1000, %rax
addq $1000, %rbx
subl $4096, %r12d
orq 8(%rbp), %rcx
xorl %eax, %eax
cmpl $100000, 4(%rsp)
cmpb $0, (%rax)
cmpb $0, %dil
testq $255, %rax
testl $7, %ecx
imulq 8(%rsp), %rcx
imulq $10, %rax, %rdx
imulq $1000, %rsi, %rdi
negq %rax
notq %r9
decl %edx
idivq %rcx
shlq $3, %rax
shrq $1, %rdx
sarq %cl, %r10
pushq %r12
popq %r15
pushq $100000
cqto
cltq
leave
syscall
setl %r11b
setne %sil
cmovgeq 8(%rsp), %rdx
movzbq %sil, %rax
movsbq (%rdi), %rcx
movslq 4(%rsp), %r8
call *%rax
jmp *%r11
movsd %xmm1, -8(%rbp)
movss (%rdi), %xmm9
subsd 16(%rsp), %xmm2
mulsd %xmm8, %xmm15
sqrtsd %xmm0, %xmm0
ucomisd %xmm1, %xmm0
xorps %xmm2, %xmm2
cvtsi2sdq %rax, %xmm0
cvtsi2ssq %rax, %xmm1
cvttsd2siq %xmm1, %rcx
cvtss2sd %xmm0, %xmm0
movq %rax, %xmm0
movq %xmm7, %r12""".splitlines()


def _text_bytes(obj, tmp):
    out = os.path.join(tmp, "t.bin")
    subprocess.run(["objcopy", "-O", "binary", "-j", ".text", obj, out], check=True)
    return open(out, "rb").read()


@pytest.mark.skipif(not HAVE_GAS, reason="GNU as / objcopy not installed")
def test_encodings_match_gnu_as(tmp_path):
    bad = []
    for ins in FORMS:
        src = tmp_path / "x.s"
        src.write_text(".text\n" + ins + "\n")
        subprocess.run(["as", "--64", "-o", str(tmp_path / "g.o"), str(src)], check=True)
        r = subprocess.run([ASM, "-c", "-o", str(tmp_path / "m.o"), str(src)], capture_output=True, text=True)
        assert r.returncode == 0, (ins, r.stderr)
        g = _text_bytes(str(tmp_path / "g.o"), str(tmp_path))
        m = _text_bytes(str(tmp_path / "m.o"), str(tmp_path))
        if g != m:
            bad.append((ins, g.hex(), m.hex()))
    assert not bad, bad


def test_static_executable_without_linker(tmp_path):
    exe = str(tmp_path / "linreg")
    r = subprocess.run([ASM, "-o", exe, RUNTIME, LINREG], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    out = subprocess.run([exe], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0, out.stdout
    first, last = [int(x) for x in out.stdout.split()]
    assert first > 1_000_000 and last * 10_000 < first  # loss (micro-units) fell by > 1e4
    assert open(exe, "rb").read(4) == b"\x7fELF"
    if shutil.which("ldd"):  # a static image: no dynamic section, no interpreter
        d = subprocess.run(["ldd", exe], capture_output=True, text=True)
        assert "not a dynamic executable" in (d.stdout + d.stderr)


@pytest.mark.skipif(not (HAVE_GAS and HAVE_LD), reason="GNU as / ld not installed")
def test_objects_link_with_system_linker(tmp_path):
    """Objects from aether-asm, linked by ld, behave like the same sources
    assembled by GNU as (same output bytes)."""
    outs = []
    for tool in ("mine", "gas"):
        objs = []
        for src in (RUNTIME, LINREG):
            o = str(tmp_path / f"{tool}_{os.path.basename(src)}.o")
            cmd = [ASM, "-c", "-o", o, src] if tool == "mine" else ["as", "--64", "-o", o, src]
            subprocess.run(cmd, check=True)
            objs.append(o)
        exe = str(tmp_path / f"{tool}_exe")
        subprocess.run(["ld", "-static", "-o", exe, *objs], check=True)
        r = subprocess.run([exe], capture_output=True, text=True, timeout=60)
        assert r.returncode == 0
        outs.append(r.stdout)
    assert outs[0] == outs[1]


@pytest.mark.skipif(shutil.which("gcc") is None, reason="no C compiler")
def test_object_called_from_c_with_data_relocations(tmp_path):
    """A function and a pointer table (.quad SYMBOL -> R_X86_64_64) assembled
    here, called from C through the system toolchain."""
    (tmp_path / "f.s").write_text("""
.text
.globl triple_sum
triple_sum:                 # (i64 a, i64 b, i64 c) -> 3 * (a + b + c)
    leaq (%rdi,%rsi), %rax
    addq %rdx, %rax
    imulq $3, %rax, %rax
    ret
.globl pick
pick:                       # (i) -> table[i]()
    leaq table(%rip), %rax
    movq (%rax,%rdi,8), %rax
    jmp *%rax
seven:
    movl $7, %eax
    ret
nine:
    movl $9, %eax
    ret
.section .data
.p2align 3
.globl table
table:
    .quad seven, nine
.globl greeting
greeting:
    .asciz "hi\\n"
""")
    (tmp_path / "m.c").write_text("""
#include <string.h>
long triple_sum(long, long, long); long pick(long); extern char greeting[];
int main(void) { return (triple_sum(1, 2, 4) == 21 && pick(0) == 7 && pick(1) == 9
                        && strcmp(greeting, "hi\\n") == 0) ? 0 : 1; }
""")
    subprocess.run([ASM, "-c", "-o", str(tmp_path / "f.o"), str(tmp_path / "f.s")], check=True)
    subprocess.run(["gcc", "-no-pie", "-o", str(tmp_path / "m"), str(tmp_path / "m.c"), str(tmp_path / "f.o")],
                   check=True)
    assert subprocess.run([str(tmp_path / "m")]).returncode == 0


@pytest.mark.parametrize("src,msg", [
    ("movq %rax\n", "takes 2 operand"),
    ("frobq %rax, %rbx\n", "unknown instruction frobq"),
    ("movq %rax, %ebx\n", "operand size mismatch"),
    ("movq (%eax), %rbx\n", "bad base"),
    ("x: x:\n", "defined twice"),
    (".bogus 1\n", "unknown directive"),
    ("jne\n", "takes 1 operand"),
])
def test_errors_carry_line_numbers(tmp_path, src, msg):
    p = tmp_path / "bad.s"
    p.write_text(".text\nnop\n" + src)
    r = subprocess.run([ASM, "-c", "-o", str(tmp_path / "bad.o"), str(p)], capture_output=True, text=True)
    assert r.returncode == 1 and "line 3" in r.stderr and msg in r.stderr, r.stderr


def test_executable_needs_entry_and_symbols(tmp_path):
    p = tmp_path / "p.s"
    p.write_text(".text\n.globl main\nmain:\n    call missing\n    ret\n")
    r = subprocess.run([ASM, "-o", str(tmp_path / "e"), str(p)], capture_output=True, text=True)
    assert r.returncode == 1 and "undefined symbol missing" in r.stderr
    r = subprocess.run([ASM, "-o", str(tmp_path / "e"), RUNTIME], capture_output=True, text=True)
    assert r.returncode == 1 and "undefined symbol main" in r.stderr
