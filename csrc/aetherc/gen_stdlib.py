"""Writes the `use runtime;` module of the aetherc compiler: one `extern fn`
declaration per function the C-ABI libraries export (libaether_rt.so and
libaether_dev.so), with the Aether types of their C parameter and return
types. Run by the runtime Makefile after the libraries are linked:

    python csrc/aetherc/gen_stdlib.py <out.aether> <lib.so>... -- <source>...

Only functions that a library really exports (its dynamic symbol table) are
declared, so a program that compiles against this module also links.
"""
import re
import subprocess
import sys

C2AE = {
    "int64_t": "i64", "long long": "i64", "long": "i64", "intptr_t": "i64", "ssize_t": "i64", "size_t": "i64",
    "uint64_t": "u64", "unsigned long long": "u64", "int": "i32", "int32_t": "i32", "uint32_t": "u32",
    "unsigned": "u32", "unsigned int": "u32", "int16_t": "i16", "uint16_t": "u16", "int8_t": "i8", "uint8_t": "u8",
    "char": "i8", "bool": "bool", "float": "f32", "double": "f64",
}
DEF = re.compile(r"^(?:AE_API\s+|extern\s+\"C\"\s+|static\s+)*([A-Za-z_][\w\s]*?[\w*]\s*\**)\s*\b([A-Za-z_]\w*)\s*\(([^;{}]*?)\)\s*(?:noexcept\s*)?\{",
                 re.M | re.S)


def ae_type(c: str):
    c = re.sub(r"\b(const|volatile|struct|__restrict__|restrict)\b", " ", c).strip()
    if "*" in c or "[" in c:
        return "i64"  # pointers travel as 64-bit integers
    c = " ".join(c.split())
    return C2AE.get(c)


def exported(libs):
    names = set()
    for lib in libs:
        out = subprocess.run(["nm", "-D", "--defined-only", lib], capture_output=True, text=True).stdout
        names |= {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    return names


def main():
    argv = sys.argv[1:]
    out, rest = argv[0], argv[1:]
    cut = rest.index("--")
    libs, srcs = rest[:cut], rest[cut + 1:]
    names = exported(libs)
    decls = {}
    for path in srcs:
        text = open(path, encoding="utf-8", errors="replace").read()
        text = re.sub(r"//[^\n]*", "", text)
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in DEF.finditer(text):
            ret, name, params = m.group(1).strip(), m.group(2), m.group(3).strip()
            if name not in names or name in decls:
                continue
            rt = None if ret == "void" else ae_type(ret)
            if ret != "void" and rt is None:
                continue
            ps, ok = [], True
            if params and params != "void":
                for i, p in enumerate(params.split(",")):
                    p = re.sub(r"/\*.*?\*/", "", p).strip()
                    p = p.split("=")[0].strip()
                    mm = re.match(r"(.*?)([A-Za-z_]\w*)?\s*$", p, re.S)
                    ctype, pname = mm.group(1).strip(), mm.group(2)
                    if not ctype:  # a parameter written without a name
                        ctype, pname = p, None
                    if pname in C2AE or pname in ("const",):
                        ctype, pname = p, None
                    t = ae_type(ctype)
                    if t is None:
                        ok = False
                        break
                    ps.append(f"{pname or 'a' + str(i)}: {t}")
            if ok:
                decls[name] = f"extern fn {name}({', '.join(ps)})" + (f" -> {rt}" if rt else "") + ";"
    with open(out, "w") as f:
        f.write("// `use runtime;`: every C function exported by libaether_rt.so and libaether_dev.so,\n"
                "// generated from their sources by csrc/aetherc/gen_stdlib.py. Pointers are i64.\n")
        for name in sorted(decls):
            f.write(decls[name] + "\n")
    print(f"{out}: {len(decls)} extern declarations ({len(names)} exported symbols)")


if __name__ == "__main__":
    main()
