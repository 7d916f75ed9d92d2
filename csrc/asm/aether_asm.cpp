// aether-asm: an x86-64 assembler for the GAS (AT&T) subset a compiler
// back end emits, writing ELF64 -- a relocatable object (-c) that the system
// linker accepts, or a static executable directly (no linker, no libc).
//
// Reference: aether_asm/src/{encode,parse,coff,pe}.rs, which encodes a
// similar subset into Windows COFF objects and PE images. On this platform the
// object format is ELF, so the writers here are ELF ones; the executable form
// plays the part of the PE writer (one image, entry `_start`, every symbol
// resolved at assembly time).
//
// Accepted source:
//   directives  .text .data .rodata .section NAME  .globl/.global  .extern
//               .byte .short/.word .long/.int .quad (number or symbol)
//               .ascii .asciz/.string  .zero/.skip N  .align/.p2align
//               .set/.equ NAME, VALUE
//   labels      NAME:
//   operands    %reg (64 / 32 / 8-bit GPRs, %xmm0-15), $imm or $SYMBOL,
//               disp(base[,index[,scale]]), SYMBOL[+/-off](%rip)
//   integer     mov movabs lea add or adc sbb and sub xor cmp test imul
//               neg not inc dec mul div idiv shl sal shr sar push pop
//               movzb movsb movslq cqto cltq setCC cmovCC
//   control     call jmp jCC (labels or *%reg), ret leave nop syscall ud2
//   SSE         movsd movss movq addsd subsd mulsd divsd sqrtsd (and ss
//               forms) ucomisd ucomiss xorpd cvtsi2sdq cvttsd2siq
// Branches to labels are always encoded with 32-bit displacements.
#include <sys/stat.h>

#include <array>
#include <algorithm>
#include <cctype>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <map>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

namespace {

struct AsmError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

[[noreturn]] void fail(int line, const std::string& msg) {
  throw AsmError("line " + std::to_string(line) + ": " + msg);
}

// ------------------------------------------------------------------ registers
struct Reg {
  int num = -1;  // 0..15
  int bits = 0;  // 64, 32, 8; 128 = xmm
  bool rex8 = false;  // spl / bpl / sil / dil: needs a REX prefix
};

bool parse_reg(const std::string& s, Reg& r) {
  static const char* r64[] = {"rax", "rcx", "rdx", "rbx", "rsp", "rbp", "rsi", "rdi",
                              "r8",  "r9",  "r10", "r11", "r12", "r13", "r14", "r15"};
  static const char* r32[] = {"eax", "ecx", "edx", "ebx", "esp", "ebp", "esi", "edi",
                              "r8d", "r9d", "r10d", "r11d", "r12d", "r13d", "r14d", "r15d"};
  static const char* r8[] = {"al",  "cl",  "dl",   "bl",   "spl",  "bpl",  "sil",  "dil",
                             "r8b", "r9b", "r10b", "r11b", "r12b", "r13b", "r14b", "r15b"};
  for (int i = 0; i < 16; ++i) {
    if (s == r64[i]) {
      r = {i, 64, false};
      return true;
    }
    if (s == r32[i]) {
      r = {i, 32, false};
      return true;
    }
    if (s == r8[i]) {
      r = {i, 8, i >= 4 && i < 8};
      return true;
    }
  }
  if (s.rfind("xmm", 0) == 0 && s.size() <= 5) {
    const int n = std::atoi(s.c_str() + 3);
    if (n >= 0 && n < 16 && std::isdigit((unsigned char)s[3])) {
      r = {n, 128, false};
      return true;
    }
  }
  return false;
}

// ------------------------------------------------------------------ operands
struct Operand {
  enum Kind { NONE, REG, IMM, MEM } kind = NONE;
  Reg reg;
  int64_t imm = 0;
  std::string sym;     // IMM: $SYMBOL (absolute); MEM: symbol displacement
  bool indirect = false;  // *%reg / *mem for call / jmp
  // MEM
  int base = -1, index = -1, scale = 1;
  bool rip = false;
  int64_t disp = 0;
};

enum Section { TEXT = 0, DATA = 1, RODATA = 2, NSEC = 3 };
const char* kSecName[NSEC] = {".text", ".data", ".rodata"};

struct RelocSite {
  Section sec;
  uint64_t off;
  std::string sym;
  int64_t addend;
  int type;  // R_X86_64_64 = 1, PC32 = 2, PLT32 = 4
  int line;
};

struct Label {
  Section sec;
  uint64_t off;
  bool defined = false;
};

struct Unit {
  std::vector<uint8_t> bytes[NSEC];
  std::map<std::string, Label> labels;
  std::map<std::string, int64_t> equs;
  std::vector<std::string> globals;
  std::vector<RelocSite> relocs;
};

std::string trim(const std::string& s) {
  size_t b = 0, e = s.size();
  while (b < e && std::isspace((unsigned char)s[b])) ++b;
  while (e > b && std::isspace((unsigned char)s[e - 1])) --e;
  return s.substr(b, e - b);
}

bool is_ident_start(char c) { return std::isalpha((unsigned char)c) || c == '_' || c == '.'; }
bool is_ident(char c) { return std::isalnum((unsigned char)c) || c == '_' || c == '.' || c == '$'; }

// Integer expressions: numbers (decimal, 0x hex), 'c', .set / .equ names,
// unary minus, parentheses, * binding tighter than + and -. At most one
// symbol, added at the top level, may stand in the expression (when sym_out
// is given): its value is left to a relocation.
struct ExprParser {
  const std::string& s;
  const Unit& u;
  std::string* sym_out;
  size_t i = 0;
  bool ok = true;

  void ws() {
    while (i < s.size() && std::isspace((unsigned char)s[i])) ++i;
  }
  int64_t factor(bool top_plus) {
    ws();
    if (i >= s.size()) return ok = false, 0;
    if (s[i] == '-') {
      ++i;
      return -factor(false);
    }
    if (s[i] == '+') {
      ++i;
      return factor(top_plus);
    }
    if (s[i] == '(') {
      ++i;
      const int64_t v = expr(false);
      ws();
      if (i >= s.size() || s[i] != ')') return ok = false, 0;
      ++i;
      return v;
    }
    if (std::isdigit((unsigned char)s[i])) {
      size_t j = i;
      int base = 10;
      if (s[i] == '0' && i + 1 < s.size() && (s[i + 1] == 'x' || s[i + 1] == 'X')) {
        base = 16;
        j = i + 2;
      }
      const size_t st = j;
      while (j < s.size() && (base == 16 ? std::isxdigit((unsigned char)s[j]) : std::isdigit((unsigned char)s[j]))) ++j;
      if (j == st) return ok = false, 0;
      const int64_t v = (int64_t)std::strtoull(s.substr(st, j - st).c_str(), nullptr, base);
      i = j;
      return v;
    }
    if (s[i] == '\'' && i + 2 < s.size() && s[i + 2] == '\'') {
      const int64_t v = (unsigned char)s[i + 1];
      i += 3;
      return v;
    }
    if (is_ident_start(s[i])) {
      size_t j = i;
      while (j < s.size() && is_ident(s[j])) ++j;
      const std::string name = s.substr(i, j - i);
      i = j;
      auto it = u.equs.find(name);
      if (it != u.equs.end()) return it->second;
      if (sym_out != nullptr && sym_out->empty() && top_plus) {
        *sym_out = name;
        return 0;
      }
      return ok = false, 0;
    }
    return ok = false, 0;
  }
  int64_t term(bool top_plus) {
    int64_t v = factor(top_plus);
    while (true) {
      ws();
      if (i < s.size() && s[i] == '*') {
        ++i;
        v *= factor(false);
      } else {
        return v;
      }
    }
  }
  int64_t expr(bool top) {
    int64_t v = term(top);
    while (true) {
      ws();
      if (i < s.size() && (s[i] == '+' || s[i] == '-')) {
        const bool plus = s[i] == '+';
        ++i;
        const int64_t t = term(top && plus);
        v = plus ? v + t : v - t;
      } else {
        return v;
      }
    }
  }
};

bool eval_int(const std::string& s0, const Unit& u, int64_t& v, std::string* sym_out = nullptr) {
  const std::string s = trim(s0);
  if (s.empty()) return false;
  ExprParser p{s, u, sym_out};
  v = p.expr(true);
  p.ws();
  return p.ok && p.i == s.size();
}

Operand parse_operand(const std::string& s0, const Unit& u, int line) {
  Operand op;
  std::string s = trim(s0);
  if (s.empty()) fail(line, "empty operand");
  if (s[0] == '*') {
    op.indirect = true;
    s = trim(s.substr(1));
  }
  if (s[0] == '%') {
    op.kind = Operand::REG;
    if (!parse_reg(s.substr(1), op.reg)) fail(line, "unknown register " + s);
    return op;
  }
  if (s[0] == '$') {
    op.kind = Operand::IMM;
    if (!eval_int(s.substr(1), u, op.imm, &op.sym)) fail(line, "bad immediate " + s);
    return op;
  }
  // memory: [disp-expr](base, index, scale)
  op.kind = Operand::MEM;
  const size_t lp = s.find('(');
  const std::string dexpr = trim(lp == std::string::npos ? s : s.substr(0, lp));
  if (!dexpr.empty() && !eval_int(dexpr, u, op.disp, &op.sym)) fail(line, "bad displacement " + dexpr);
  if (lp == std::string::npos) {
    // bare symbol / absolute address: only as a branch target
    return op;
  }
  const size_t rp = s.find(')', lp);
  if (rp == std::string::npos || trim(s.substr(rp + 1)) != "") fail(line, "bad memory operand " + s);
  std::vector<std::string> parts;
  std::stringstream ss(s.substr(lp + 1, rp - lp - 1));
  std::string p;
  while (std::getline(ss, p, ',')) parts.push_back(trim(p));
  if (parts.empty() || parts.size() > 3) fail(line, "bad memory operand " + s);
  if (!parts[0].empty()) {
    if (parts[0] == "%rip") {
      op.rip = true;
    } else {
      Reg b;
      if (parts[0][0] != '%' || !parse_reg(parts[0].substr(1), b) || b.bits != 64) fail(line, "bad base " + parts[0]);
      op.base = b.num;
    }
  }
  if (parts.size() >= 2 && !parts[1].empty()) {
    Reg x;
    if (parts[1][0] != '%' || !parse_reg(parts[1].substr(1), x) || x.bits != 64 || x.num == 4)
      fail(line, "bad index " + parts[1]);
    op.index = x.num;
  }
  if (parts.size() == 3) {
    op.scale = std::atoi(parts[2].c_str());
    if (op.scale != 1 && op.scale != 2 && op.scale != 4 && op.scale != 8) fail(line, "bad scale " + parts[2]);
  }
  if (op.rip && op.index >= 0) fail(line, "%rip cannot take an index");
  if (op.base < 0 && !op.rip) fail(line, "memory operands need a base register or %rip");
  return op;
}

std::vector<std::string> split_operands(const std::string& s) {
  std::vector<std::string> out;
  int depth = 0;
  std::string cur;
  bool in_str = false;
  for (char c : s) {
    if (c == '"') in_str = !in_str;
    if (!in_str && c == '(') ++depth;
    if (!in_str && c == ')') --depth;
    if (!in_str && c == ',' && depth == 0) {
      out.push_back(trim(cur));
      cur.clear();
    } else {
      cur.push_back(c);
    }
  }
  if (!trim(cur).empty()) out.push_back(trim(cur));
  return out;
}

// ------------------------------------------------------------------ encoder
struct Enc {
  Unit& u;
  Section sec;
  int line;
  std::vector<uint8_t>& out() { return u.bytes[sec]; }
  void b(uint8_t x) { out().push_back(x); }
  void le(uint64_t v, int n) {
    for (int i = 0; i < n; ++i) b((uint8_t)(v >> (8 * i)));
  }

  // prefix (0x66 / 0xF2 / 0xF3 or 0), REX, opcode bytes, ModRM (+SIB, disp), immediate
  void modrm(int prefix, bool w, const std::vector<uint8_t>& opc, int regf, const Operand& rm, int imm_bytes,
             int64_t imm, bool force_rex = false) {
    int rex = 0x40 | (w ? 8 : 0) | ((regf & 8) ? 4 : 0);
    if (rm.kind == Operand::REG) {
      rex |= (rm.reg.num & 8) ? 1 : 0;
      if (rm.reg.rex8) force_rex = true;
    } else {
      if (rm.index >= 0 && (rm.index & 8)) rex |= 2;
      if (rm.base >= 0 && (rm.base & 8)) rex |= 1;
    }
    if (prefix) b((uint8_t)prefix);
    if (rex != 0x40 || force_rex) b((uint8_t)rex);
    for (uint8_t o : opc) b(o);
    const int r3 = regf & 7;
    if (rm.kind == Operand::REG) {
      b((uint8_t)(0xC0 | (r3 << 3) | (rm.reg.num & 7)));
    } else if (rm.rip) {
      b((uint8_t)((r3 << 3) | 5));
      const uint64_t at = out().size();
      le(0, 4);
      if (!rm.sym.empty()) {
        // the displacement is relative to the end of the instruction
        u.relocs.push_back({sec, at, rm.sym, rm.disp - 4 - imm_bytes, 2, line});
      } else {
        int32_t d = (int32_t)rm.disp;
        std::memcpy(&out()[at], &d, 4);
      }
    } else {
      if (!rm.sym.empty()) fail(line, "symbolic displacement needs %rip");
      const int base = rm.base;
      const bool need_sib = rm.index >= 0 || (base & 7) == 4;
      int mod;
      if (rm.disp == 0 && (base & 7) != 5) mod = 0;
      else if (rm.disp >= -128 && rm.disp <= 127) mod = 1;
      else mod = 2;
      if (rm.disp < INT32_MIN || rm.disp > INT32_MAX) fail(line, "displacement out of range");
      b((uint8_t)((mod << 6) | (r3 << 3) | (need_sib ? 4 : (base & 7))));
      if (need_sib) {
        const int ss = rm.scale == 1 ? 0 : rm.scale == 2 ? 1 : rm.scale == 4 ? 2 : 3;
        const int idx = rm.index >= 0 ? (rm.index & 7) : 4;
        b((uint8_t)((ss << 6) | (idx << 3) | (base & 7)));
      }
      if (mod == 1) le((uint64_t)(int8_t)rm.disp, 1);
      if (mod == 2) le((uint64_t)(int32_t)rm.disp, 4);
    }
    if (imm_bytes) le((uint64_t)imm, imm_bytes);
  }

  void rel32_branch(const std::vector<uint8_t>& opc, const std::string& sym) {
    for (uint8_t o : opc) b(o);
    const uint64_t at = out().size();
    le(0, 4);
    u.relocs.push_back({sec, at, sym, -4, 4, line});  // PLT32 form; resolved locally when defined here
  }
};

bool fits8(int64_t v) { return v >= -128 && v <= 127; }
bool fits32(int64_t v) { return v >= INT32_MIN && v <= INT32_MAX; }

struct Cc {
  const char* name;
  int code;
};
const Cc kCc[] = {{"o", 0},  {"no", 1}, {"b", 2},   {"c", 2},   {"nae", 2}, {"ae", 3}, {"nb", 3},  {"nc", 3},
                  {"e", 4},  {"z", 4},  {"ne", 5},  {"nz", 5},  {"be", 6},  {"na", 6}, {"a", 7},   {"nbe", 7},
                  {"s", 8},  {"ns", 9}, {"p", 10},  {"pe", 10}, {"np", 11}, {"po", 11}, {"l", 12}, {"nge", 12},
                  {"ge", 13}, {"nl", 13}, {"le", 14}, {"ng", 14}, {"g", 15},  {"nle", 15}};

int cc_of(const std::string& s) {
  for (const Cc& c : kCc)
    if (s == c.name) return c.code;
  return -1;
}

// operand width from the suffix (q / l / b) or the register operands
int width_of(const std::string& mn, const std::string& base, const std::vector<Operand>& ops, int line) {
  int w = 0;
  if (mn.size() == base.size() + 1) {
    const char s = mn.back();
    w = s == 'q' ? 64 : s == 'l' ? 32 : s == 'b' ? 8 : s == 'w' ? 16 : 0;
  }
  for (const Operand& o : ops)
    if (o.kind == Operand::REG && o.reg.bits != 128) {
      if (w && o.reg.bits != w) fail(line, "operand size mismatch in " + mn);
      w = o.reg.bits;
    }
  if (!w) fail(line, "cannot tell the operand size of " + mn + " (add a q / l suffix)");
  if (w == 16) fail(line, "16-bit operands are not supported");
  return w;
}

bool strip_suffix(const std::string& mn, const std::string& base) {
  if (mn == base) return true;
  return mn.size() == base.size() + 1 && mn.compare(0, base.size(), base) == 0 && std::strchr("qlb", mn.back());
}

void encode(Unit& u, Section sec, const std::string& mn, const std::vector<std::string>& args, int line) {
  Enc e{u, sec, line};
  std::vector<Operand> ops;
  for (const std::string& a : args) ops.push_back(parse_operand(a, u, line));
  auto nops = [&](size_t n) {
    if (ops.size() != n) fail(line, mn + " takes " + std::to_string(n) + " operand(s)");
  };
  auto is = [&](size_t i, Operand::Kind k) { return ops.size() > i && ops[i].kind == k; };

  // ---- no-operand forms
  if (mn == "ret" || mn == "retq") return nops(0), e.b(0xC3);
  if (mn == "leave" || mn == "leaveq") return nops(0), e.b(0xC9);
  if (mn == "nop") return nops(0), e.b(0x90);
  if (mn == "syscall") return nops(0), e.b(0x0F), e.b(0x05);
  if (mn == "ud2") return nops(0), e.b(0x0F), e.b(0x0B);
  if (mn == "cqto" || mn == "cqo") return nops(0), e.b(0x48), e.b(0x99);
  if (mn == "cltq" || mn == "cdqe") return nops(0), e.b(0x48), e.b(0x98);
  if (mn == "cltd" || mn == "cdq") return nops(0), e.b(0x99);

  // ---- control flow
  if (mn == "call" || mn == "callq" || mn == "jmp" || mn == "jmpq") {
    nops(1);
    const bool call = mn[0] == 'c';
    if (ops[0].indirect) {
      if (ops[0].kind == Operand::MEM && ops[0].sym.empty() && ops[0].base < 0 && !ops[0].rip)
        fail(line, "bad indirect target");
      Operand rm = ops[0];
      if (rm.kind == Operand::REG && rm.reg.bits != 64) fail(line, "indirect branch needs a 64-bit register");
      return e.modrm(0, false, {0xFF}, call ? 2 : 4, rm, 0, 0);
    }
    if (ops[0].kind != Operand::MEM || ops[0].sym.empty() || ops[0].base >= 0 || ops[0].rip)
      fail(line, mn + " needs a label or *%reg");
    e.rel32_branch(call ? std::vector<uint8_t>{0xE8} : std::vector<uint8_t>{0xE9}, ops[0].sym);
    if (ops[0].disp) u.relocs.back().addend += ops[0].disp;
    return;
  }
  if (mn.size() >= 2 && mn[0] == 'j') {
    const int cc = cc_of(mn.substr(1));
    if (cc < 0) fail(line, "unknown instruction " + mn);
    nops(1);
    if (ops[0].kind != Operand::MEM || ops[0].sym.empty() || ops[0].base >= 0) fail(line, mn + " needs a label");
    e.rel32_branch({0x0F, (uint8_t)(0x80 | cc)}, ops[0].sym);
    return;
  }
  if (mn.rfind("set", 0) == 0 && cc_of(mn.substr(3)) >= 0) {
    nops(1);
    if (!is(0, Operand::REG) || ops[0].reg.bits != 8) fail(line, mn + " needs an 8-bit register");
    return e.modrm(0, false, {0x0F, (uint8_t)(0x90 | cc_of(mn.substr(3)))}, 0, ops[0], 0, 0);
  }
  if (mn.rfind("cmov", 0) == 0) {
    std::string c = mn.substr(4);
    if (!c.empty() && (c.back() == 'q' || c.back() == 'l') && cc_of(c) < 0) c.pop_back();
    const int cc = cc_of(c);
    if (cc < 0) fail(line, "unknown instruction " + mn);
    nops(2);
    if (!is(1, Operand::REG) || is(0, Operand::IMM)) fail(line, mn + " needs reg/mem, reg");
    const int w = width_of(mn, "cmov" + c, ops, line);
    return e.modrm(0, w == 64, {0x0F, (uint8_t)(0x40 | cc)}, ops[1].reg.num, ops[0], 0, 0);
  }

  // ---- push / pop
  if (strip_suffix(mn, "push") || strip_suffix(mn, "pop")) {
    nops(1);
    const bool push = mn[1] == 'u';
    if (is(0, Operand::REG)) {
      if (ops[0].reg.bits != 64) fail(line, mn + " needs a 64-bit register");
      if (ops[0].reg.num & 8) e.b(0x41);
      return e.b((uint8_t)((push ? 0x50 : 0x58) + (ops[0].reg.num & 7)));
    }
    if (push && is(0, Operand::IMM) && ops[0].sym.empty()) {
      if (fits8(ops[0].imm)) return e.b(0x6A), e.le((uint64_t)ops[0].imm, 1);
      if (!fits32(ops[0].imm)) fail(line, "push immediate out of range");
      return e.b(0x68), e.le((uint64_t)ops[0].imm, 4);
    }
    if (is(0, Operand::MEM)) return e.modrm(0, false, {push ? (uint8_t)0xFF : (uint8_t)0x8F}, push ? 6 : 0, ops[0], 0, 0);
    fail(line, "bad operand for " + mn);
  }

  // ---- SSE
  struct Sse {
    const char* name;
    int prefix;
    uint8_t op;
  };
  static const Sse kSse[] = {{"addsd", 0xF2, 0x58}, {"subsd", 0xF2, 0x5C}, {"mulsd", 0xF2, 0x59},
                             {"divsd", 0xF2, 0x5E}, {"sqrtsd", 0xF2, 0x51}, {"addss", 0xF3, 0x58},
                             {"subss", 0xF3, 0x5C}, {"mulss", 0xF3, 0x59}, {"divss", 0xF3, 0x5E},
                             {"sqrtss", 0xF3, 0x51}, {"ucomisd", 0x66, 0x2E}, {"ucomiss", 0, 0x2E},
                             {"xorpd", 0x66, 0x57}, {"xorps", 0, 0x57}, {"cvtsd2ss", 0xF2, 0x5A},
                             {"cvtss2sd", 0xF3, 0x5A}};
  for (const Sse& s : kSse) {
    if (mn != s.name) continue;
    nops(2);
    if (!is(1, Operand::REG) || ops[1].reg.bits != 128 || is(0, Operand::IMM) ||
        (is(0, Operand::REG) && ops[0].reg.bits != 128))
      fail(line, mn + " needs xmm/mem, xmm");
    return e.modrm(s.prefix, false, {0x0F, s.op}, ops[1].reg.num, ops[0], 0, 0);
  }
  if (mn == "movsd" || mn == "movss") {
    nops(2);
    const int pf = mn == "movsd" ? 0xF2 : 0xF3;
    if (is(1, Operand::REG) && ops[1].reg.bits == 128 && !is(0, Operand::IMM) &&
        !(is(0, Operand::REG) && ops[0].reg.bits != 128))
      return e.modrm(pf, false, {0x0F, 0x10}, ops[1].reg.num, ops[0], 0, 0);
    if (is(0, Operand::REG) && ops[0].reg.bits == 128 && is(1, Operand::MEM))
      return e.modrm(pf, false, {0x0F, 0x11}, ops[0].reg.num, ops[1], 0, 0);
    fail(line, mn + " needs xmm/mem, xmm or xmm, mem");
  }
  if (mn == "cvtsi2sdq" || mn == "cvtsi2sdl" || mn == "cvtsi2ssq" || mn == "cvtsi2ssl") {
    nops(2);
    if (!is(1, Operand::REG) || ops[1].reg.bits != 128) fail(line, mn + " needs an xmm destination");
    return e.modrm(mn.compare(6, 2, "sd") == 0 ? 0xF2 : 0xF3, mn.back() == 'q', {0x0F, 0x2A}, ops[1].reg.num, ops[0], 0, 0);
  }
  if (mn == "cvttsd2siq" || mn == "cvttsd2sil" || mn == "cvttss2siq" || mn == "cvttss2sil") {
    nops(2);
    if (!is(1, Operand::REG) || ops[1].reg.bits == 128) fail(line, mn + " needs a general-register destination");
    return e.modrm(mn[5] == 'd' ? 0xF2 : 0xF3, mn.back() == 'q', {0x0F, 0x2C}, ops[1].reg.num, ops[0], 0, 0);
  }
  if (mn == "movq" && ops.size() == 2 && ((is(0, Operand::REG) && ops[0].reg.bits == 128) ||
                                          (is(1, Operand::REG) && ops[1].reg.bits == 128))) {
    if (is(1, Operand::REG) && ops[1].reg.bits == 128 && is(0, Operand::REG) && ops[0].reg.bits == 64)
      return e.modrm(0x66, true, {0x0F, 0x6E}, ops[1].reg.num, ops[0], 0, 0);
    if (is(0, Operand::REG) && ops[0].reg.bits == 128 && is(1, Operand::REG) && ops[1].reg.bits == 64)
      return e.modrm(0x66, true, {0x0F, 0x7E}, ops[0].reg.num, ops[1], 0, 0);
    fail(line, "movq between xmm and a 64-bit register only");
  }

  // ---- moves with extension
  if (mn == "movzbl" || mn == "movzbq" || mn == "movsbl" || mn == "movsbq") {
    nops(2);
    if (!is(1, Operand::REG) || is(0, Operand::IMM) || (is(0, Operand::REG) && ops[0].reg.bits != 8))
      fail(line, mn + " needs r8/mem8, reg");
    return e.modrm(0, mn.back() == 'q', {0x0F, (uint8_t)(mn[3] == 'z' ? 0xB6 : 0xBE)}, ops[1].reg.num, ops[0], 0, 0,
                   is(0, Operand::REG) && ops[0].reg.rex8);
  }
  if (mn == "movslq" || mn == "movsxd") {
    nops(2);
    if (!is(1, Operand::REG) || ops[1].reg.bits != 64 || is(0, Operand::IMM) ||
        (is(0, Operand::REG) && ops[0].reg.bits != 32))
      fail(line, mn + " needs r32/mem32, r64");
    return e.modrm(0, true, {0x63}, ops[1].reg.num, ops[0], 0, 0);
  }

  // ---- mov / movabs / lea
  if (mn == "movabs" || mn == "movabsq") {
    nops(2);
    if (!is(0, Operand::IMM) || !is(1, Operand::REG) || ops[1].reg.bits != 64) fail(line, "movabs needs $imm64, r64");
    e.b((uint8_t)(0x48 | ((ops[1].reg.num & 8) ? 1 : 0)));
    e.b((uint8_t)(0xB8 + (ops[1].reg.num & 7)));
    const uint64_t at = e.out().size();
    e.le((uint64_t)ops[0].imm, 8);
    if (!ops[0].sym.empty()) u.relocs.push_back({sec, at, ops[0].sym, ops[0].imm, 1, line});
    return;
  }
  if (strip_suffix(mn, "lea")) {
    nops(2);
    if (!is(0, Operand::MEM) || !is(1, Operand::REG)) fail(line, "lea needs mem, reg");
    const int w = width_of(mn, "lea", {ops[1]}, line);
    return e.modrm(0, w == 64, {0x8D}, ops[1].reg.num, ops[0], 0, 0);
  }
  if (strip_suffix(mn, "mov")) {
    nops(2);
    const int w = width_of(mn, "mov", ops, line);
    const bool W = w == 64;
    if (w == 8) {
      const bool rex8 = (is(0, Operand::REG) && ops[0].reg.rex8) || (is(1, Operand::REG) && ops[1].reg.rex8);
      if (is(0, Operand::IMM)) {
        if (!ops[0].sym.empty() || ops[0].imm < -128 || ops[0].imm > 255) fail(line, "8-bit immediate out of range");
        if (is(1, Operand::REG)) {
          if ((ops[1].reg.num & 8) || rex8) e.b((uint8_t)(0x40 | ((ops[1].reg.num & 8) ? 1 : 0)));
          e.b((uint8_t)(0xB0 + (ops[1].reg.num & 7)));
          return e.le((uint64_t)ops[0].imm, 1);
        }
        return e.modrm(0, false, {0xC6}, 0, ops[1], 1, ops[0].imm);
      }
      if (is(0, Operand::REG)) return e.modrm(0, false, {0x88}, ops[0].reg.num, ops[1], 0, 0, rex8);
      if (is(1, Operand::REG) && is(0, Operand::MEM)) return e.modrm(0, false, {0x8A}, ops[1].reg.num, ops[0], 0, 0, rex8);
      fail(line, "bad operands for " + mn);
    }
    if (is(0, Operand::IMM)) {
      if (!ops[0].sym.empty()) fail(line, "use movabs or lea for symbol addresses");
      if (is(1, Operand::REG)) {
        if (!W || (ops[0].imm >= 0 && ops[0].imm <= 0xFFFFFFFFll && !W)) {
          if (ops[1].reg.num & 8) e.b(0x41);
          e.b((uint8_t)(0xB8 + (ops[1].reg.num & 7)));
          return e.le((uint64_t)ops[0].imm, 4);
        }
        if (fits32(ops[0].imm)) return e.modrm(0, true, {0xC7}, 0, ops[1], 4, ops[0].imm);
        e.b((uint8_t)(0x48 | ((ops[1].reg.num & 8) ? 1 : 0)));
        e.b((uint8_t)(0xB8 + (ops[1].reg.num & 7)));
        return e.le((uint64_t)ops[0].imm, 8);
      }
      if (!fits32(ops[0].imm)) fail(line, "immediate out of range");
      return e.modrm(0, W, {0xC7}, 0, ops[1], 4, ops[0].imm);
    }
    if (is(0, Operand::REG) && ops[0].reg.bits != 128) return e.modrm(0, W, {0x89}, ops[0].reg.num, ops[1], 0, 0);
    if (is(1, Operand::REG) && is(0, Operand::MEM)) return e.modrm(0, W, {0x8B}, ops[1].reg.num, ops[0], 0, 0);
    fail(line, "bad operands for " + mn);
  }

  // ---- two-operand ALU
  static const char* kAlu[] = {"add", "or", "adc", "sbb", "and", "sub", "xor", "cmp"};
  for (int n = 0; n < 8; ++n) {
    if (!strip_suffix(mn, kAlu[n])) continue;
    nops(2);
    const int w = width_of(mn, kAlu[n], ops, line);
    const bool W = w == 64;
    if (w == 8) {
      const bool rex8 = (is(0, Operand::REG) && ops[0].reg.rex8) || (is(1, Operand::REG) && ops[1].reg.rex8);
      if (is(0, Operand::IMM)) {
        if (!ops[0].sym.empty() || ops[0].imm < -128 || ops[0].imm > 255) fail(line, "8-bit immediate out of range");
        if (is(1, Operand::REG) && ops[1].reg.num == 0) return e.b((uint8_t)(8 * n + 4)), e.le((uint64_t)ops[0].imm, 1);
        return e.modrm(0, false, {0x80}, n, ops[1], 1, ops[0].imm, rex8);
      }
      if (is(0, Operand::REG)) return e.modrm(0, false, {(uint8_t)(8 * n)}, ops[0].reg.num, ops[1], 0, 0, rex8);
      if (is(0, Operand::MEM) && is(1, Operand::REG)) return e.modrm(0, false, {(uint8_t)(8 * n + 2)}, ops[1].reg.num, ops[0], 0, 0, rex8);
      fail(line, "bad operands for " + mn);
    }
    if (is(0, Operand::IMM)) {
      if (!ops[0].sym.empty()) fail(line, "symbolic immediate in arithmetic");
      if (is(1, Operand::MEM) || is(1, Operand::REG)) {
        if (fits8(ops[0].imm)) return e.modrm(0, W, {0x83}, n, ops[1], 1, ops[0].imm);
        if (!fits32(ops[0].imm) && !(w == 32 && ops[0].imm <= 0xFFFFFFFFll)) fail(line, "immediate out of range");
        if (is(1, Operand::REG) && ops[1].reg.num == 0) {  // accumulator short form
          if (W) e.b(0x48);
          e.b((uint8_t)(8 * n + 5));
          return e.le((uint64_t)ops[0].imm, 4);
        }
        return e.modrm(0, W, {0x81}, n, ops[1], 4, ops[0].imm);
      }
    }
    if (is(0, Operand::REG)) return e.modrm(0, W, {(uint8_t)(8 * n + 1)}, ops[0].reg.num, ops[1], 0, 0);
    if (is(0, Operand::MEM) && is(1, Operand::REG)) return e.modrm(0, W, {(uint8_t)(8 * n + 3)}, ops[1].reg.num, ops[0], 0, 0);
    fail(line, "bad operands for " + mn);
  }
  if (strip_suffix(mn, "test")) {
    nops(2);
    const int w = width_of(mn, "test", ops, line);
    const bool W = w == 64;
    if (w == 8) fail(line, "8-bit test is not supported");
    if (is(0, Operand::IMM)) {
      if (is(1, Operand::REG) && ops[1].reg.num == 0) {
        if (W) e.b(0x48);
        e.b(0xA9);
        return e.le((uint64_t)ops[0].imm, 4);
      }
      return e.modrm(0, W, {0xF7}, 0, ops[1], 4, ops[0].imm);
    }
    if (is(0, Operand::REG)) return e.modrm(0, W, {0x85}, ops[0].reg.num, ops[1], 0, 0);
    fail(line, "bad operands for test");
  }
  if (strip_suffix(mn, "imul") && ops.size() >= 2) {
    const int w = width_of(mn, "imul", ops, line);
    const bool W = w == 64;
    if (ops.size() == 2) {
      if (!is(1, Operand::REG) || is(0, Operand::IMM)) fail(line, "imul needs reg/mem, reg");
      return e.modrm(0, W, {0x0F, 0xAF}, ops[1].reg.num, ops[0], 0, 0);
    }
    nops(3);
    if (!is(0, Operand::IMM) || !is(2, Operand::REG)) fail(line, "imul needs $imm, reg/mem, reg");
    if (fits8(ops[0].imm)) return e.modrm(0, W, {0x6B}, ops[2].reg.num, ops[1], 1, ops[0].imm);
    return e.modrm(0, W, {0x69}, ops[2].reg.num, ops[1], 4, ops[0].imm);
  }

  // ---- one-operand group 3 / 5
  struct One {
    const char* name;
    uint8_t op;
    int ext;
  };
  static const One kOne[] = {{"not", 0xF7, 2}, {"neg", 0xF7, 3}, {"mul", 0xF7, 4}, {"imul", 0xF7, 5},
                             {"div", 0xF7, 6}, {"idiv", 0xF7, 7}, {"inc", 0xFF, 0}, {"dec", 0xFF, 1}};
  for (const One& o : kOne) {
    if (!strip_suffix(mn, o.name)) continue;
    nops(1);
    const int w = width_of(mn, o.name, ops, line);
    if (w == 8 || is(0, Operand::IMM)) fail(line, "bad operand for " + mn);
    return e.modrm(0, w == 64, {o.op}, o.ext, ops[0], 0, 0);
  }

  // ---- shifts
  struct Sh {
    const char* name;
    int ext;
  };
  static const Sh kSh[] = {{"rol", 0}, {"ror", 1}, {"shl", 4}, {"sal", 4}, {"shr", 5}, {"sar", 7}};
  for (const Sh& s : kSh) {
    if (!strip_suffix(mn, s.name)) continue;
    if (ops.size() == 1) ops.insert(ops.begin(), Operand{Operand::IMM, {}, 1});
    if (ops.size() != 2) fail(line, mn + " takes a count and a destination");
    std::vector<Operand> dst = {ops[1]};
    const int w = width_of(mn, s.name, dst, line);
    const bool W = w == 64;
    if (is(0, Operand::REG)) {
      if (ops[0].reg.num != 1 || ops[0].reg.bits != 8) fail(line, "shift count register must be %cl");
      return e.modrm(0, W, {0xD3}, s.ext, ops[1], 0, 0);
    }
    if (!is(0, Operand::IMM)) fail(line, "bad shift count");
    if (ops[0].imm == 1) return e.modrm(0, W, {0xD1}, s.ext, ops[1], 0, 0);
    return e.modrm(0, W, {0xC1}, s.ext, ops[1], 1, ops[0].imm);
  }
  fail(line, "unknown instruction " + mn);
}

// ------------------------------------------------------------------ parser
std::string parse_string_lit(const std::string& s, int line) {
  const std::string t = trim(s);
  if (t.size() < 2 || t.front() != '"' || t.back() != '"') fail(line, "expected a string literal");
  std::string out;
  for (size_t i = 1; i + 1 < t.size(); ++i) {
    char c = t[i];
    if (c == '\\' && i + 2 < t.size()) {
      const char n = t[++i];
      if (n == 'n') c = '\n';
      else if (n == 't') c = '\t';
      else if (n == 'r') c = '\r';
      else if (n == '0') c = '\0';
      else if (n == '\\') c = '\\';
      else if (n == '"') c = '"';
      else if (n == 'x' && i + 2 < t.size()) {
        c = (char)std::strtol(t.substr(i + 1, 2).c_str(), nullptr, 16);
        i += 2;
      } else
        fail(line, std::string("unknown escape \\") + n);
    }
    out.push_back(c);
  }
  return out;
}

void assemble(const std::string& src, Unit& u) {
  Section sec = TEXT;
  std::vector<std::string> lines;
  {
    std::stringstream ss(src);
    std::string l;
    while (std::getline(ss, l)) lines.push_back(l);
  }
  for (size_t n = 0; n < lines.size(); ++n) {
    const int line = (int)n + 1;
    // strip comments outside strings: '#' and '//'
    std::string l;
    bool in_str = false;
    const std::string& raw = lines[n];
    for (size_t i = 0; i < raw.size(); ++i) {
      const char c = raw[i];
      if (c == '"' && (i == 0 || raw[i - 1] != '\\')) in_str = !in_str;
      if (!in_str && (c == '#' || (c == '/' && i + 1 < raw.size() && raw[i + 1] == '/'))) break;
      l.push_back(c);
    }
    l = trim(l);
    // labels (possibly several, then a statement)
    while (true) {
      size_t k = 0;
      while (k < l.size() && is_ident(l[k])) ++k;
      if (k > 0 && k < l.size() && l[k] == ':' && is_ident_start(l[0])) {
        const std::string name = l.substr(0, k);
        Label& lab = u.labels[name];
        if (lab.defined) fail(line, "label " + name + " defined twice");
        lab = {sec, (uint64_t)u.bytes[sec].size(), true};
        l = trim(l.substr(k + 1));
        continue;
      }
      break;
    }
    if (l.empty()) continue;
    size_t sp = 0;
    while (sp < l.size() && !std::isspace((unsigned char)l[sp])) ++sp;
    const std::string head = l.substr(0, sp);
    const std::string rest = trim(l.substr(sp));
    if (head[0] == '.') {
      const std::vector<std::string> args = split_operands(rest);
      if (head == ".text") sec = TEXT;
      else if (head == ".data") sec = DATA;
      else if (head == ".rodata") sec = RODATA;
      else if (head == ".section") {
        const std::string nm = trim(args.empty() ? "" : args[0]);
        if (nm == ".text" || nm.rfind(".text.", 0) == 0) sec = TEXT;
        else if (nm == ".data" || nm.rfind(".data.", 0) == 0) sec = DATA;
        else if (nm == ".rodata" || nm == ".rdata" || nm.rfind(".rodata.", 0) == 0) sec = RODATA;
        else fail(line, "unknown section " + nm);
      } else if (head == ".globl" || head == ".global") {
        for (const std::string& a : args) u.globals.push_back(a);
      } else if (head == ".extern" || head == ".type" || head == ".size" || head == ".file" || head == ".ident") {
        // accepted and ignored: undefined symbols are external already
      } else if (head == ".set" || head == ".equ") {
        int64_t v;
        if (args.size() != 2 || !eval_int(args[1], u, v)) fail(line, head + " NAME, VALUE");
        u.equs[args[0]] = v;
      } else if (head == ".byte" || head == ".short" || head == ".word" || head == ".long" || head == ".int" ||
                 head == ".quad") {
        const int size = head == ".byte" ? 1 : (head == ".short" || head == ".word") ? 2 : head == ".quad" ? 8 : 4;
        for (const std::string& a : args) {
          int64_t v;
          std::string sym;
          if (!eval_int(a, u, v, size == 8 ? &sym : nullptr)) fail(line, "bad value " + a);
          const uint64_t at = u.bytes[sec].size();
          for (int i = 0; i < size; ++i) u.bytes[sec].push_back((uint8_t)((uint64_t)v >> (8 * i)));
          if (!sym.empty()) u.relocs.push_back({sec, at, sym, v, 1, line});
        }
      } else if (head == ".ascii" || head == ".asciz" || head == ".string") {
        for (const std::string& a : args) {
          const std::string s = parse_string_lit(a, line);
          u.bytes[sec].insert(u.bytes[sec].end(), s.begin(), s.end());
          if (head != ".ascii") u.bytes[sec].push_back(0);
        }
      } else if (head == ".zero" || head == ".skip" || head == ".space") {
        int64_t v;
        if (args.empty() || !eval_int(args[0], u, v) || v < 0) fail(line, "bad size");
        u.bytes[sec].insert(u.bytes[sec].end(), (size_t)v, 0);
      } else if (head == ".align" || head == ".balign" || head == ".p2align") {
        int64_t v;
        if (args.empty() || !eval_int(args[0], u, v) || v < 0) fail(line, "bad alignment");
        const uint64_t a = head == ".p2align" ? (1ull << v) : (uint64_t)v;
        if (a == 0 || (a & (a - 1))) fail(line, "alignment must be a power of two");
        while (u.bytes[sec].size() % a) u.bytes[sec].push_back(sec == TEXT ? 0x90 : 0);
      } else {
        fail(line, "unknown directive " + head);
      }
      continue;
    }
    std::string mn = head;
    for (char& c : mn) c = (char)std::tolower((unsigned char)c);
    encode(u, sec, mn, rest.empty() ? std::vector<std::string>{} : split_operands(rest), line);
  }
  // labels referenced in relocations but never defined are external
}

// ------------------------------------------------------------------ ELF writer
struct Buf {
  std::vector<uint8_t> d;
  void u8(uint8_t v) { d.push_back(v); }
  void u16(uint16_t v) { le(v, 2); }
  void u32(uint32_t v) { le(v, 4); }
  void u64(uint64_t v) { le(v, 8); }
  void le(uint64_t v, int n) {
    for (int i = 0; i < n; ++i) d.push_back((uint8_t)(v >> (8 * i)));
  }
  void pad(size_t a) {
    while (d.size() % a) d.push_back(0);
  }
  void put(const std::vector<uint8_t>& x) { d.insert(d.end(), x.begin(), x.end()); }
};

void elf_header(Buf& b, uint16_t type, uint64_t entry, uint64_t phoff, uint16_t phnum, uint64_t shoff, uint16_t shnum,
                uint16_t shstrndx) {
  const uint8_t ident[16] = {0x7F, 'E', 'L', 'F', 2, 1, 1, 0, 0, 0, 0, 0, 0, 0, 0, 0};
  b.d.insert(b.d.end(), ident, ident + 16);
  b.u16(type);
  b.u16(62);  // EM_X86_64
  b.u32(1);
  b.u64(entry);
  b.u64(phoff);
  b.u64(shoff);
  b.u32(0);
  b.u16(64);
  b.u16(56);
  b.u16(phnum);
  b.u16(64);
  b.u16(shnum);
  b.u16(shstrndx);
}

std::vector<uint8_t> write_object(const Unit& u) {
  // sections: 0 null, 1 .text, 2 .data, 3 .rodata, then .rela.* for the ones with relocations,
  // .symtab, .strtab, .shstrtab
  std::string strtab(1, '\0'), shstr(1, '\0');
  auto add_str = [](std::string& t, const std::string& s) {
    const uint32_t off = (uint32_t)t.size();
    t += s;
    t.push_back('\0');
    return off;
  };
  std::map<std::string, bool> global_set;
  for (const std::string& g : u.globals) global_set[g] = true;
  struct Sym {
    std::string name;
    uint8_t info;
    uint16_t shndx;
    uint64_t value;
  };
  std::vector<Sym> syms = {{"", 0, 0, 0}};
  for (int s = 0; s < NSEC; ++s) syms.push_back({"", (uint8_t)((0 << 4) | 3), (uint16_t)(s + 1), 0});  // STT_SECTION
  std::map<std::string, int> index;
  for (const auto& kv : u.labels)
    if (!global_set.count(kv.first)) syms.push_back({kv.first, (uint8_t)((0 << 4) | 0), (uint16_t)(kv.second.sec + 1), kv.second.off});
  const size_t first_global = syms.size();
  std::vector<std::string> externs;
  for (const RelocSite& r : u.relocs)
    if (!u.labels.count(r.sym) && !global_set.count(r.sym)) global_set[r.sym] = true;
  for (const auto& kv : global_set) {
    auto it = u.labels.find(kv.first);
    if (it != u.labels.end())
      syms.push_back({kv.first, (uint8_t)((1 << 4) | 0), (uint16_t)(it->second.sec + 1), it->second.off});
    else
      syms.push_back({kv.first, (uint8_t)((1 << 4) | 0), 0, 0});  // undefined
  }
  for (size_t i = 0; i < syms.size(); ++i)
    if (!syms[i].name.empty()) index[syms[i].name] = (int)i;

  // relocations per section; locals against their section symbol
  std::vector<uint8_t> sdata[NSEC];
  for (int s = 0; s < NSEC; ++s) sdata[s] = u.bytes[s];
  Buf rela[NSEC];
  for (const RelocSite& r : u.relocs) {
    auto it = u.labels.find(r.sym);
    const bool local = it != u.labels.end() && !std::count(u.globals.begin(), u.globals.end(), r.sym);
    if (local && it->second.sec == r.sec && (r.type == 2 || r.type == 4)) {
      // same-section PC-relative: resolve now
      const int64_t v = (int64_t)it->second.off + r.addend - (int64_t)r.off;
      if (!fits32(v)) fail(r.line, "branch out of range");
      int32_t d = (int32_t)v;
      std::memcpy(&sdata[r.sec][r.off], &d, 4);
      continue;
    }
    uint32_t symi;
    int64_t add = r.addend;
    if (local) {
      symi = 1 + it->second.sec;
      add += (int64_t)it->second.off;
    } else {
      symi = (uint32_t)index.at(r.sym);
    }
    const uint32_t type = r.type == 4 && local ? 2 : r.type;
    rela[r.sec].u64(r.off);
    rela[r.sec].u64(((uint64_t)symi << 32) | type);
    rela[r.sec].u64((uint64_t)add);
  }
  Buf symtab;
  for (const Sym& s : syms) {
    symtab.u32(s.name.empty() ? 0 : add_str(strtab, s.name));
    symtab.u8(s.info);
    symtab.u8(0);
    symtab.u16(s.shndx);
    symtab.u64(s.value);
    symtab.u64(0);
  }
  struct Sh {
    uint32_t name, type;
    uint64_t flags, off = 0, size = 0;
    uint32_t link = 0, info = 0;
    uint64_t align = 1, entsize = 0;
    const std::vector<uint8_t>* data = nullptr;
  };
  std::vector<Sh> sh(1);
  const uint64_t flags[NSEC] = {0x6 /*AX*/, 0x3 /*WA*/, 0x2 /*A*/};
  for (int s = 0; s < NSEC; ++s) {
    Sh h{add_str(shstr, kSecName[s]), 1 /*PROGBITS*/, flags[s]};
    h.size = sdata[s].size();
    h.align = s == TEXT ? 16 : 8;
    h.data = &sdata[s];
    sh.push_back(h);
  }
  const uint32_t symtab_idx = (uint32_t)(sh.size() + [&] {
    int n = 0;
    for (int s = 0; s < NSEC; ++s) n += rela[s].d.empty() ? 0 : 1;
    return n;
  }());
  for (int s = 0; s < NSEC; ++s) {
    if (rela[s].d.empty()) continue;
    Sh h{add_str(shstr, std::string(".rela") + kSecName[s]), 4 /*RELA*/, 0x40 /*INFO_LINK*/};
    h.size = rela[s].d.size();
    h.link = symtab_idx;
    h.info = (uint32_t)(s + 1);
    h.align = 8;
    h.entsize = 24;
    h.data = &rela[s].d;
    sh.push_back(h);
  }
  Sh hs{add_str(shstr, ".symtab"), 2 /*SYMTAB*/, 0};
  hs.size = symtab.d.size();
  hs.link = symtab_idx + 1;
  hs.info = (uint32_t)first_global;
  hs.align = 8;
  hs.entsize = 24;
  hs.data = &symtab.d;
  sh.push_back(hs);
  std::vector<uint8_t> strv(strtab.begin(), strtab.end());
  Sh hstr{add_str(shstr, ".strtab"), 3 /*STRTAB*/, 0};
  hstr.size = strv.size();
  hstr.data = &strv;
  sh.push_back(hstr);
  Sh hsh{add_str(shstr, ".shstrtab"), 3, 0};
  std::vector<uint8_t> shv(shstr.begin(), shstr.end());
  hsh.size = shv.size();
  hsh.data = &shv;
  sh.push_back(hsh);

  Buf out;
  out.d.resize(64);
  for (size_t i = 1; i < sh.size(); ++i) {
    out.pad(sh[i].align);
    sh[i].off = out.d.size();
    out.put(*sh[i].data);
  }
  out.pad(8);
  const uint64_t shoff = out.d.size();
  for (const Sh& h : sh) {
    out.u32(h.name);
    out.u32(h.type);
    out.u64(h.flags);
    out.u64(0);
    out.u64(h.off);
    out.u64(h.size);
    out.u32(h.link);
    out.u32(h.info);
    out.u64(h.align);
    out.u64(h.entsize);
  }
  Buf hdr;
  elf_header(hdr, 1 /*ET_REL*/, 0, 0, 0, shoff, (uint16_t)sh.size(), (uint16_t)(sh.size() - 1));
  std::memcpy(out.d.data(), hdr.d.data(), 64);
  return out.d;
}

// Static executable: every input's sections concatenated, symbols resolved,
// two PT_LOAD segments (text + rodata read / execute, data read / write).
std::vector<uint8_t> write_executable(std::vector<Unit>& units) {
  const uint64_t base = 0x400000, page = 0x1000;
  // per-unit section offsets inside the merged sections
  std::vector<uint8_t> merged[NSEC];
  std::vector<std::array<uint64_t, NSEC>> at(units.size());
  for (size_t i = 0; i < units.size(); ++i)
    for (int s = 0; s < NSEC; ++s) {
      while (merged[s].size() % 16) merged[s].push_back(s == TEXT ? 0x90 : 0);
      at[i][s] = merged[s].size();
      merged[s].insert(merged[s].end(), units[i].bytes[s].begin(), units[i].bytes[s].end());
    }
  const uint64_t text_off = page;
  const uint64_t text_va = base + text_off;
  uint64_t ro_rel = (merged[TEXT].size() + 15) & ~15ull;
  const uint64_t ro_va = text_va + ro_rel;
  const uint64_t rx_size = ro_rel + merged[RODATA].size();
  const uint64_t data_off = (text_off + rx_size + page - 1) & ~(page - 1);
  const uint64_t data_va = base + data_off;
  const uint64_t sec_va[NSEC] = {text_va, data_va, ro_va};
  // global symbol table
  std::map<std::string, uint64_t> globals;
  for (size_t i = 0; i < units.size(); ++i)
    for (const std::string& g : units[i].globals) {
      auto it = units[i].labels.find(g);
      if (it == units[i].labels.end()) continue;
      if (globals.count(g)) throw AsmError("symbol " + g + " defined in two inputs");
      globals[g] = sec_va[it->second.sec] + at[i][it->second.sec] + it->second.off;
    }
  for (size_t i = 0; i < units.size(); ++i)
    for (const RelocSite& r : units[i].relocs) {
      uint64_t S;
      auto it = units[i].labels.find(r.sym);
      if (it != units[i].labels.end()) S = sec_va[it->second.sec] + at[i][it->second.sec] + it->second.off;
      else if (globals.count(r.sym)) S = globals[r.sym];
      else fail(r.line, "undefined symbol " + r.sym);
      const uint64_t P = sec_va[r.sec] + at[i][r.sec] + r.off;
      uint8_t* dst = &merged[r.sec][at[i][r.sec] + r.off];
      if (r.type == 1) {
        const uint64_t v = S + (uint64_t)r.addend;
        std::memcpy(dst, &v, 8);
      } else {
        const int64_t v = (int64_t)(S + (uint64_t)r.addend - P);
        if (!fits32(v)) fail(r.line, "relocation out of range");
        const int32_t d = (int32_t)v;
        std::memcpy(dst, &d, 4);
      }
    }
  if (!globals.count("_start")) throw AsmError("no global _start: the executable needs an entry point");
  Buf out;
  elf_header(out, 2 /*ET_EXEC*/, globals["_start"], 64, 2, 0, 0, 0);
  auto phdr = [&](uint32_t flags, uint64_t off, uint64_t va, uint64_t fsz, uint64_t msz) {
    out.u32(1);  // PT_LOAD
    out.u32(flags);
    out.u64(off);
    out.u64(va);
    out.u64(va);
    out.u64(fsz);
    out.u64(msz);
    out.u64(page);
  };
  phdr(5 /*R X*/, text_off, text_va, rx_size, rx_size);
  const uint64_t dsz = std::max<uint64_t>(merged[DATA].size(), 1);
  phdr(6 /*R W*/, data_off, data_va, merged[DATA].size(), dsz);
  out.d.resize(text_off, 0);
  out.put(merged[TEXT]);
  out.d.resize(text_off + ro_rel, 0);
  out.put(merged[RODATA]);
  out.d.resize(data_off, 0);
  out.put(merged[DATA]);
  return out.d;
}

bool read_all(const std::string& p, std::string& s) {
  std::ifstream f(p, std::ios::binary);
  if (!f) return false;
  std::stringstream ss;
  ss << f.rdbuf();
  s = ss.str();
  return true;
}

}  // namespace



int main(int argc, char** argv) {
  std::vector<std::string> inputs;
  std::string out;
  bool obj = false;
  for (int i = 1; i < argc; ++i) {
    const std::string a = argv[i];
    if (a == "-o" && i + 1 < argc) out = argv[++i];
    else if (a == "-c") obj = true;
    else if (a == "-h" || a == "--help") {
      std::printf("usage: aether-asm [-c] -o OUT input.s...\n  -c  write an ELF64 relocatable object (one input)\n"
                  "      otherwise a static executable (entry _start) from all inputs\n");
      return 0;
    } else inputs.push_back(a);
  }
  if (inputs.empty() || out.empty()) {
    std::fprintf(stderr, "usage: aether-asm [-c] -o OUT input.s...\n");
    return 2;
  }
  if (obj && inputs.size() != 1) {
    std::fprintf(stderr, "aether-asm: -c takes one input\n");
    return 2;
  }
  std::vector<Unit> units(inputs.size());
  for (size_t i = 0; i < inputs.size(); ++i) {
    std::string src;
    if (!read_all(inputs[i], src)) {
      std::fprintf(stderr, "aether-asm: cannot read %s\n", inputs[i].c_str());
      return 2;
    }
    try {
      assemble(src, units[i]);
    } catch (const AsmError& e) {
      std::fprintf(stderr, "aether-asm: %s: %s\n", inputs[i].c_str(), e.what());
      return 1;
    }
  }
  std::vector<uint8_t> bytes;
  try {
    bytes = obj ? write_object(units[0]) : write_executable(units);
  } catch (const AsmError& e) {
    std::fprintf(stderr, "aether-asm: %s\n", e.what());
    return 1;
  }
  std::ofstream f(out, std::ios::binary | std::ios::trunc);
  f.write(reinterpret_cast<const char*>(bytes.data()), (std::streamsize)bytes.size());
  if (!f) {
    std::fprintf(stderr, "aether-asm: cannot write %s\n", out.c_str());
    return 2;
  }
  f.close();
  if (!obj) chmod(out.c_str(), 0755);
  return 0;
}
