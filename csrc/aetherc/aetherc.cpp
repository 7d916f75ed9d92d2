// aetherc: a compiler for the Aether language subset that the runtime
// witnesses and training programs are written in, lowering to C and linking
// against this package's C-ABI libraries (libaether_rt / libaether_dev).
//
// Reference: the aetherc CLI (compiler/src/main.rs:60-140: --emit kinds,
// --check, --json-errors, -o), the `Tensor` method lowering of its asm
// backend (compiler/src/codegen/asm/mod.rs:4195-4380: a method on a
// shape-typed device tensor becomes one aether_op_*_cuda call with the shape
// integers appended), its matmul -> gelu fusion peephole (compiler/src/mir/
// fuse.rs:1-30) and the `--emit=c` backend (compiler/src/codegen/c/mod.rs).
// The reference emits x86-64 assembly or C; this one always goes through C
// (gcc / cc) and links the shared runtime libraries.
//
// Language covered: `use <module>;` (stdlib modules of extern declarations),
// `const`, `extern fn`, `fn` with typed parameters and return type, `let` /
// `let mut` with optional type, scalar types (bool, i8..i64, u8..u64, f32,
// f64, &str), fixed arrays `[T; N]` (literal and repeat forms, indexing),
// `Tensor<f32|i32, [dims]>` device tensors (allocated at `let`, freed when
// the scope ends), `while`, `loop`, `for i in a..b` / `a..=b`, `break`,
// `continue`, `return`, `if` / `else if` / `else` as statements and
// expressions, block tail expressions, arithmetic / comparison / logical /
// bitwise operators, compound assignment, `as` casts and the cast builtins
// f32() f64() i32() i64(), println / print, float math builtins, method
// calls on tensors, structs (C structs by value: literals, nested and array
// fields), impl and trait methods (`Type__method`, `&self` by pointer, trait
// default bodies copied into each impl, `Type::f()`, `Self`), enums (no
// payload: integers; with payloads: tagged structs), `match` with literal,
// wildcard, binding, path and tuple-variant patterns, `|` and guards,
// `if let` / `while let`, references to scalars and structs as pointers
// (an address passed where an i64 is declared is the address as an integer),
// tuples and tuple structs, functions as values, and closures: one without
// captures is a static function (its address an i64), one with captures a
// heap object [function, captured values...] of type `Closure`, called with
// the object as its first argument. Generic functions, structs and impls are
// specialised per use (`id__int64_t`, `Pair__float`): type parameters bind
// from argument types, then from the expected type, and a generic impl's
// methods are generated for each instance that calls them. `macro_rules!`
// macros expand at parse time (captures, one level of repetition, rules in
// order) and `println!` / `print!` take `{}` holes. Slices `&[T]` are
// (pointer, length) structs: `slice_from_raw`, `&s[a..b]` of a slice, a
// fixed array or a runtime vector / string handle, `len()`, indexing and
// `for x in s`. Generic enums are specialised like generic structs, and
// `e?` yields the `Ok` / `Some` value or returns the enum from the enclosing
// function. `async fn` is compiled as a plain function that runs to
// completion where it is awaited (`.await` yields its value, `yield_now()`
// does nothing): with a single task this gives the result polling would.
// Shape generics
// (`Tensor<f32, [M, K]>` with M a parameter) are diagnostics, not
// miscompiles.
#include <sys/stat.h>
#include <unistd.h>

#include <cctype>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <functional>
#include <map>
#include <memory>
#include <set>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

namespace ae {

// ============================================================================ diagnostics
struct Diag : std::runtime_error {
  std::string code;
  int line, col;
  Diag(std::string c, int l, int k, const std::string& m) : std::runtime_error(m), code(std::move(c)), line(l), col(k) {}
};
[[noreturn]] void fail(const char* code, int line, int col, const std::string& msg) { throw Diag(code, line, col, msg); }

// ============================================================================ lexer
enum class T { Id, Int, Float, Str, Char, Op, Eof };
struct Tok {
  T t;
  std::string s;
  int line, col;
};

std::vector<Tok> lex(const std::string& src) {
  std::vector<Tok> out;
  size_t i = 0;
  int line = 1, col = 1;
  auto adv = [&](size_t n) {
    for (size_t k = 0; k < n && i < src.size(); ++k, ++i) {
      if (src[i] == '\n') {
        ++line;
        col = 1;
      } else {
        ++col;
      }
    }
  };
  static const char* ops3[] = {"..=", "<<=", ">>=", nullptr};
  static const char* ops2[] = {"->", "=>", "==", "!=", "<=", ">=", "&&", "||", "+=", "-=", "*=", "/=", "%=",
                               "&=", "|=", "^=", "<<", ">>", "::", "..", nullptr};
  while (i < src.size()) {
    const char c = src[i];
    if (c == ' ' || c == '\t' || c == '\r' || c == '\n') {
      adv(1);
      continue;
    }
    if (c == '/' && i + 1 < src.size() && src[i + 1] == '/') {  // comments are dropped at lex time
      while (i < src.size() && src[i] != '\n') adv(1);
      continue;
    }
    if (c == '/' && i + 1 < src.size() && src[i + 1] == '*') {
      int depth = 0;
      do {
        if (src.compare(i, 2, "/*") == 0) {
          ++depth;
          adv(2);
        } else if (src.compare(i, 2, "*/") == 0) {
          --depth;
          adv(2);
        } else {
          adv(1);
        }
      } while (depth > 0 && i < src.size());
      continue;
    }
    const int l0 = line, c0 = col;
    if (isalpha((unsigned char)c) || c == '_') {
      size_t j = i;
      while (j < src.size() && (isalnum((unsigned char)src[j]) || src[j] == '_')) ++j;
      out.push_back({T::Id, src.substr(i, j - i), l0, c0});
      adv(j - i);
      continue;
    }
    if (isdigit((unsigned char)c)) {
      size_t j = i;
      bool flt = false;
      std::string text;
      if (c == '0' && j + 1 < src.size() && (src[j + 1] == 'x' || src[j + 1] == 'X')) {
        j += 2;
        while (j < src.size() && (isxdigit((unsigned char)src[j]) || src[j] == '_')) {
          if (src[j] != '_') text += src[j];
          ++j;
        }
        text = std::to_string((long long)std::stoull(text, nullptr, 16));
      } else if (c == '0' && j + 1 < src.size() && (src[j + 1] == 'o' || src[j + 1] == 'O')) {
        j += 2;
        while (j < src.size() && ((src[j] >= '0' && src[j] <= '7') || src[j] == '_')) {
          if (src[j] != '_') text += src[j];
          ++j;
        }
        text = std::to_string((long long)std::stoull(text, nullptr, 8));
      } else if (c == '0' && j + 1 < src.size() && (src[j + 1] == 'b' || src[j + 1] == 'B')) {
        j += 2;
        while (j < src.size() && (src[j] == '0' || src[j] == '1' || src[j] == '_')) {
          if (src[j] != '_') text += src[j];
          ++j;
        }
        text = std::to_string((long long)std::stoull(text, nullptr, 2));
      } else {
        while (j < src.size() && (isdigit((unsigned char)src[j]) || src[j] == '_')) {
          if (src[j] != '_') text += src[j];
          ++j;
        }
        // a '.' starts a fraction unless it begins a range (`0..n`) or a method call (`1.max`)
        if (j + 1 < src.size() && src[j] == '.' && isdigit((unsigned char)src[j + 1])) {
          flt = true;
          text += src[j++];
          while (j < src.size() && (isdigit((unsigned char)src[j]) || src[j] == '_')) {
            if (src[j] != '_') text += src[j];
            ++j;
          }
        } else if (j < src.size() && src[j] == '.' && (j + 1 >= src.size() || (src[j + 1] != '.' &&
                                                                                 !isalpha((unsigned char)src[j + 1]) &&
                                                                                 src[j + 1] != '_'))) {
          flt = true;  // `1.` literal
          text += src[j++];
        }
        if (j < src.size() && (src[j] == 'e' || src[j] == 'E') && j + 1 < src.size() &&
            (isdigit((unsigned char)src[j + 1]) || ((src[j + 1] == '-' || src[j + 1] == '+') && j + 2 < src.size() &&
                                                    isdigit((unsigned char)src[j + 2])))) {
          flt = true;
          text += src[j++];
          if (src[j] == '-' || src[j] == '+') text += src[j++];
          while (j < src.size() && isdigit((unsigned char)src[j])) text += src[j++];
        }
      }
      // type suffixes (1i32, 2.0f32, 3u8): kept as the literal's text after '#'
      size_t k = j;
      while (k < src.size() && (isalnum((unsigned char)src[k]) || src[k] == '_')) ++k;
      std::string suffix = src.substr(j, k - j);
      if (!suffix.empty()) {
        if (suffix[0] == '_') suffix = suffix.substr(1);
        if (suffix == "f32" || suffix == "f64") flt = true;
        text += "#" + suffix;
        j = k;
      }
      out.push_back({flt ? T::Float : T::Int, text, l0, c0});
      adv(j - i);
      continue;
    }
    if (c == '"') {
      std::string s;
      size_t j = i + 1;
      while (j < src.size() && src[j] != '"') {
        if (src[j] == '\\' && j + 1 < src.size()) {
          const char e = src[j + 1];
          s += e == 'n' ? '\n' : e == 't' ? '\t' : e == 'r' ? '\r' : e == '0' ? '\0' : e;
          j += 2;
        } else {
          s += src[j++];
        }
      }
      if (j >= src.size()) fail("AE0001", l0, c0, "unterminated string literal");
      out.push_back({T::Str, s, l0, c0});
      adv(j + 1 - i);
      continue;
    }
    if (c == '\'' && i + 1 < src.size() && (std::isalpha((unsigned char)src[i + 1]) || src[i + 1] == '_') &&
        !(i + 2 < src.size() && src[i + 2] == '\'')) {  // a lifetime (`'a`): no meaning here, dropped
      adv(1);
      while (i < src.size() && (std::isalnum((unsigned char)src[i]) || src[i] == '_')) adv(1);
      continue;
    }
    if (c == '\'' && i + 2 < src.size() && (src[i + 2] == '\'' || (src[i + 1] == '\\' && i + 3 < src.size()))) {
      int v;
      size_t len;
      if (src[i + 1] == '\\') {
        const char e = src[i + 2];
        v = e == 'n' ? '\n' : e == 't' ? '\t' : e == 'r' ? '\r' : e == '0' ? 0 : e;
        len = 4;
      } else {
        v = (unsigned char)src[i + 1];
        len = 3;
      }
      out.push_back({T::Char, std::to_string(v), l0, c0});
      adv(len);
      continue;
    }
    std::string op;
    for (int k = 0; ops3[k]; ++k)
      if (src.compare(i, 3, ops3[k]) == 0) op = ops3[k];
    if (op.empty())
      for (int k = 0; ops2[k]; ++k)
        if (src.compare(i, 2, ops2[k]) == 0) op = ops2[k];
    if (op.empty()) op = std::string(1, c);
    if (std::string("(){}[],;:.+-*/%<>=!&|^~#?@$").find(op[0]) == std::string::npos)
      fail("AE0001", l0, c0, std::string("unexpected character '") + c + "'");
    out.push_back({T::Op, op, l0, c0});
    adv(op.size());
  }
  out.push_back({T::Eof, "", line, col});
  return out;
}

// ============================================================================ types
enum class B { Void, Bool, I8, I16, I32, I64, U8, U16, U32, U64, F32, F64, Str, Tensor, Array, Struct, Unknown };

struct Ty {
  B b = B::Unknown;
  B elem = B::Unknown;           // tensor element (F32 / I32)
  std::vector<int64_t> dims;     // tensor shape
  std::shared_ptr<Ty> inner;     // array element
  int64_t len = 0;               // array length
  std::string sname;             // struct name
  bool ref = false;              // a reference (`&T` of a scalar or struct): a C pointer
  bool is_int() const { return b >= B::I8 && b <= B::U64; }
  bool is_float() const { return b == B::F32 || b == B::F64; }
  bool is_num() const { return is_int() || is_float(); }
  int64_t numel() const {
    int64_t n = 1;
    for (int64_t d : dims) n *= d;
    return n;
  }
};
Ty prim(B b) {
  Ty t;
  t.b = b;
  return t;
}

const std::map<std::string, B>& prim_names() {
  static const std::map<std::string, B> m = {
      {"bool", B::Bool}, {"i8", B::I8},   {"i16", B::I16}, {"i32", B::I32}, {"i64", B::I64}, {"isize", B::I64},
      {"u8", B::U8},     {"u16", B::U16}, {"u32", B::U32}, {"u64", B::U64}, {"usize", B::U64}, {"f32", B::F32},
      {"f64", B::F64},   {"str", B::Str}};
  return m;
}

std::string ctype(const Ty& t) {
  if (t.ref) {
    Ty base = t;
    base.ref = false;
    return ctype(base) + "*";
  }
  if (t.b == B::Struct) return "aes_" + t.sname;
  switch (t.b) {
    case B::Void: return "void";
    case B::Bool: return "int";
    case B::I8: return "int8_t";
    case B::I16: return "int16_t";
    case B::I32: return "int32_t";
    case B::I64: return "int64_t";
    case B::U8: return "uint8_t";
    case B::U16: return "uint16_t";
    case B::U32: return "uint32_t";
    case B::U64: return "uint64_t";
    case B::F32: return "float";
    case B::F64: return "double";
    case B::Str: return "const char*";
    case B::Tensor: return "int64_t";  // a device buffer handle
    default: return "int64_t";
  }
}

std::string tyname(const Ty& t) {
  if (t.ref) {
    Ty base = t;
    base.ref = false;
    return "&" + tyname(base);
  }
  for (auto& kv : prim_names())
    if (kv.second == t.b && kv.first != "isize" && kv.first != "usize") return t.b == B::Str ? "&str" : kv.first;
  if (t.b == B::Void) return "()";
  if (t.b == B::Tensor) {
    std::string s = std::string("Tensor<") + (t.elem == B::I32 ? "i32" : "f32") + ", [";
    for (size_t i = 0; i < t.dims.size(); ++i) s += (i ? ", " : "") + std::to_string(t.dims[i]);
    return s + "]>";
  }
  if (t.b == B::Array) return "[" + tyname(*t.inner) + "; " + std::to_string(t.len) + "]";
  if (t.b == B::Struct) return t.sname;
  return "?";
}

// ============================================================================ AST
struct Expr;
struct Stmt;
struct Block;
using EP = std::shared_ptr<Expr>;
using SP = std::shared_ptr<Stmt>;
using BP = std::shared_ptr<Block>;

struct TyExpr {  // a type as written; tensor dims / array lengths may name constants
  std::string name;              // primitive / "Tensor" / "[]" / "&str" / a struct name
  bool generic = false;          // written with generic arguments (Vec<T>, ...)
  bool ref = false;              // written `&T` / `&mut T`
  std::vector<std::shared_ptr<TyExpr>> elems;  // a tuple type's element types
  std::vector<std::shared_ptr<TyExpr>> targs;  // generic arguments: `W<i64>`
  std::string elem;              // tensor element
  std::vector<EP> dims;          // tensor dims or {array length}
  std::shared_ptr<TyExpr> inner; // array element
  int line = 0, col = 0;
};

struct Fn;

// A `match` / `if let` / `while let` pattern.
struct Pat {
  enum K { Wild, Lit, Bind, Path, Tuple, Or } k = Wild;
  std::string s;  // literal text, binding name or path
  bool neg = false;  // a negative literal
  std::vector<std::shared_ptr<Pat>> subs;  // Tuple: the payload patterns; Or: the alternatives
  int line = 0, col = 0;
};
using PP = std::shared_ptr<Pat>;

struct Expr {
  enum K { Int, Float, BoolL, Str, Char, Var, Unary, Binary, Call, Method, Cast, Ref, If, BlockE, Index, ArrayLit,
           ArrayRep, LoopE, Field, Deref, StructLit, Match, TupleLit, Closure, Try } k;
  std::string s;  // literal / name / operator / method / struct
  std::vector<EP> a;
  std::vector<std::string> fields;  // struct literal: the field each of `a` initialises
  std::vector<PP> pats;             // match: one pattern per arm (a[0] the scrutinee, a[i + 1] arm i)
  std::vector<EP> guards;           // match: the arm's `if` guard or null
  std::shared_ptr<Fn> closure;      // closure: parameters, optional return type, body (its tail)
  BP blk, blk2;   // if: then / else block (else may be an `if` wrapped in a block)
  std::shared_ptr<TyExpr> cast;
  bool mut = false;
  int line = 0, col = 0;
};

struct Block {
  std::vector<SP> stmts;
  EP tail;
  int line = 0, col = 0;
};

struct Stmt {
  enum K { Let, ExprS, Assign, While, Loop, For, Return, Break, Continue } k;
  PP pat;  // `while let pat = e`
  std::vector<std::string> names;  // `let (a, b, _) = e`
  std::string name, op;
  bool mut = false, inclusive = false;
  std::shared_ptr<TyExpr> ty;
  EP e, e2, e3;
  BP body;
  int line = 0, col = 0;
};

struct Param {
  std::string name;
  std::shared_ptr<TyExpr> ty;
  bool self_ref = false;  // `&self` / `&mut self`
};
struct Fn {
  std::string name;
  std::vector<Param> params;  // a method's receiver is the parameter `self` (no type)
  std::shared_ptr<TyExpr> ret;
  BP body;                    // null: extern, or a trait method without a default body
  std::vector<std::string> generics;  // type parameters: specialised per use
  bool is_extern = false;
  bool is_test = false;  // #[test]: run by the `--test` harness
  int line = 0, col = 0;
};
struct StructDef {
  std::string name;
  std::vector<std::string> generics;
  std::vector<Param> fields;
  int line = 0, col = 0;
};
struct TraitDef {
  std::string name;
  std::vector<std::string> supers;  // `trait Pet: Animal + Named`
  std::vector<Fn> methods;
  int line = 0, col = 0;
};
struct EnumDef {
  std::string name;
  std::vector<std::string> generics;
  std::vector<std::pair<std::string, std::vector<std::shared_ptr<TyExpr>>>> variants;  // name, payload types
  int line = 0, col = 0;
};
struct ImplDef {
  std::string trait;  // empty: an inherent impl
  std::string type;
  std::vector<Fn> methods;
  int line = 0, col = 0;
};
struct Const {
  std::string name;
  std::shared_ptr<TyExpr> ty;
  EP e;
  int line = 0, col = 0;
};
struct Program {
  std::vector<Fn> fns;
  std::vector<Const> consts;
  std::vector<std::string> uses;
  std::vector<StructDef> structs;
  std::vector<TraitDef> traits;
  std::vector<ImplDef> impls;
  std::vector<EnumDef> enums;
};

// ============================================================================ parser
class Parser {
 public:
  explicit Parser(std::vector<Tok> t) : t_(std::move(t)) {}

  Program program() {
    Program p;
    while (!at(T::Eof)) {
      if (eat_id("pub") && is_op("(")) group();  // pub(crate) / pub(super) / pub(in path): all public here
      if (eat_id("use")) {
        std::string path = ident();
        while (eat_op("::")) path += "::" + ident();
        expect_op(";");
        p.uses.push_back(path);
      } else if (eat_id("const") || eat_id("static")) {
        Const c;
        c.line = cur().line;
        c.col = cur().col;
        eat_id("mut");
        c.name = ident();
        expect_op(":");
        c.ty = type();
        expect_op("=");
        c.e = expr();
        expect_op(";");
        p.consts.push_back(c);
      } else if (is_id("macro_rules") && peek().t == T::Op && peek().s == "!") {
        macro_def();
      } else if (is_id("unsafe") && peek().t == T::Id && peek().s == "impl") {
        next();
        p.impls.push_back(impl_def());
      } else if (is_id("extern") || is_id("fn") || is_id("unsafe") || is_id("async")) {
        p.fns.push_back(fn());
        p.fns.back().is_test = pending_test_;
        pending_test_ = false;
      } else if (is_op("#")) {
        if (attribute() == "test") pending_test_ = true;
      } else if (is_id("struct")) {
        p.structs.push_back(struct_def());
      } else if (is_id("trait")) {
        p.traits.push_back(trait_def());
      } else if (is_id("impl")) {
        p.impls.push_back(impl_def());
      } else if (is_id("enum")) {
        p.enums.push_back(enum_def());
      } else {
        fail("AE0002", cur().line, cur().col, "expected an item (fn, extern fn, const, static, struct, trait, impl, "
                                              "use), found '" + cur().s + "'");
      }
    }
    return p;
  }

 private:
  std::vector<Tok> t_;
  size_t i_ = 0;
  const Tok& cur() const { return t_[i_]; }
  const Tok& peek(int k = 1) const { return t_[std::min(i_ + k, t_.size() - 1)]; }
  void next() {
    if (i_ + 1 < t_.size()) ++i_;
  }
  bool at(T t) const { return cur().t == t; }
  bool is_op(const char* s) const { return cur().t == T::Op && cur().s == s; }
  bool is_id(const char* s) const { return cur().t == T::Id && cur().s == s; }
  bool eat_op(const char* s) {
    if (!is_op(s)) return false;
    next();
    return true;
  }
  bool eat_id(const char* s) {
    if (!is_id(s)) return false;
    next();
    return true;
  }
  void expect_op(const char* s) {
    if (!eat_op(s)) fail("AE0002", cur().line, cur().col, std::string("expected '") + s + "', found '" + cur().s + "'");
  }
  std::string ident() {
    if (!at(T::Id)) fail("AE0002", cur().line, cur().col, "expected an identifier, found '" + cur().s + "'");
    std::string s = cur().s;
    next();
    return s;
  }

  // `#[...]` before an item or a method: accepted and ignored.
  // `#[...]`: skipped; returns the attribute's name (`test`, `inline`, ...).
  std::string attribute() {
    expect_op("#");
    expect_op("[");
    const std::string name = at(T::Id) ? cur().s : "";
    int depth = 1;
    while (depth > 0 && !at(T::Eof)) {
      if (is_op("[")) ++depth;
      if (is_op("]")) --depth;
      next();
    }
    return name;
  }
  bool pending_test_ = false;  // the next fn carries #[test]

  // Closes a generic argument list; `>>` closes two.
  void close_angle() {
    if (is_op(">>")) {
      t_[i_].s = ">";
      return;
    }
    if (is_op(">=")) {
      t_[i_].s = "=";
      return;
    }
    expect_op(">");
  }

  // `<T, U: Bound, const N: usize>` after an item name: the parameter names.
  std::vector<std::string> generic_params() {
    std::vector<std::string> names;
    if (!eat_op("<")) return names;
    while (!is_op(">") && !is_op(">>")) {
      eat_id("const");
      names.push_back(ident());
      if (eat_op(":")) {  // bounds / const type: skip to the next top-level ',' or '>'
        int depth = 0;
        while (!at(T::Eof)) {
          if (is_op("<")) ++depth;
          if ((is_op(">") || is_op(">>")) && depth == 0) break;
          if (is_op(">")) --depth;
          if (is_op(">>")) depth -= 2;
          if (is_op(",") && depth == 0) break;
          next();
        }
      }
      if (!eat_op(",")) break;
    }
    close_angle();
    return names;
  }

  StructDef struct_def() {
    StructDef d;
    d.line = cur().line;
    d.col = cur().col;
    next();  // struct
    d.name = ident();
    d.generics = generic_params();
    if (eat_op(";")) return d;  // unit struct
    if (eat_op("(")) {          // tuple struct
      int k = 0;
      while (!is_op(")")) {
        eat_id("pub");
        Param f;
        f.name = std::to_string(k++);
        f.ty = type();
        d.fields.push_back(f);
        if (!eat_op(",")) break;
      }
      expect_op(")");
      expect_op(";");
      return d;
    }
    expect_op("{");
    while (!is_op("}")) {
      if (is_op("#")) {
        attribute();
        continue;
      }
      eat_id("pub");
      Param f;
      f.name = ident();
      expect_op(":");
      f.ty = type();
      d.fields.push_back(f);
      if (!eat_op(",")) break;
    }
    expect_op("}");
    return d;
  }

  TraitDef trait_def() {
    TraitDef d;
    d.line = cur().line;
    d.col = cur().col;
    next();  // trait
    d.name = ident();
    generic_params();
    if (eat_op(":")) {
      do {
        d.supers.push_back(ident());
      } while (eat_op("+"));
    }
    expect_op("{");
    while (!is_op("}")) {
      if (at(T::Eof)) fail("AE0002", d.line, d.col, "unclosed trait body");
      if (is_op("#")) {
        attribute();
        continue;
      }
      d.methods.push_back(fn(true));
    }
    expect_op("}");
    return d;
  }

  EnumDef enum_def() {
    EnumDef d;
    d.line = cur().line;
    d.col = cur().col;
    next();  // enum
    d.name = ident();
    d.generics = generic_params();
    expect_op("{");
    while (!is_op("}")) {
      if (is_op("#")) {
        attribute();
        continue;
      }
      std::pair<std::string, std::vector<std::shared_ptr<TyExpr>>> v;
      v.first = ident();
      if (eat_op("(")) {
        while (!is_op(")")) {
          v.second.push_back(type());
          if (!eat_op(",")) break;
        }
        expect_op(")");
      } else if (is_op("{")) {
        fail("AE0500", cur().line, cur().col, "variants with named fields are not supported");
      } else if (eat_op("=")) {
        expr();  // an explicit discriminant: variants are numbered by position here
      }
      d.variants.push_back(v);
      if (!eat_op(",")) break;
    }
    expect_op("}");
    return d;
  }

  // A pattern: `_`, a literal, a binding, a path, `Path(p, ..)`, `p | p`.
  PP pattern() {
    PP first = pattern_one();
    if (!is_op("|")) return first;
    auto o = std::make_shared<Pat>();
    o->k = Pat::Or;
    o->line = first->line;
    o->col = first->col;
    o->subs.push_back(first);
    while (eat_op("|")) o->subs.push_back(pattern_one());
    return o;
  }
  PP pattern_one() {
    auto p = std::make_shared<Pat>();
    p->line = cur().line;
    p->col = cur().col;
    if (eat_op("-")) {
      p->neg = true;
      if (!at(T::Int) && !at(T::Float)) fail("AE0002", cur().line, cur().col, "expected a number after '-'");
    }
    if (at(T::Int) || at(T::Float) || at(T::Char) || at(T::Str)) {
      p->k = Pat::Lit;
      p->s = (at(T::Char) ? "'" : "") + cur().s;
      if (at(T::Str)) p->s = "\"" + cur().s;
      next();
      return p;
    }
    if (is_id("true") || is_id("false")) {
      p->k = Pat::Lit;
      p->s = cur().s;
      next();
      return p;
    }
    std::string name = ident();
    if (name == "_") return p;
    while (eat_op("::")) name += "::" + ident();
    p->s = name;
    if (eat_op("(")) {
      p->k = Pat::Tuple;
      while (!is_op(")")) {
        p->subs.push_back(pattern());
        if (!eat_op(",")) break;
      }
      expect_op(")");
      return p;
    }
    p->k = name.find("::") != std::string::npos ? Pat::Path : Pat::Bind;
    return p;
  }

  ImplDef impl_def() {
    ImplDef d;
    d.line = cur().line;
    d.col = cur().col;
    next();  // impl
    generic_params();
    std::string first = ident();
    if (is_op("<")) type_args();
    if (eat_id("for")) {
      d.trait = first;
      d.type = ident();
      if (is_op("<")) type_args();
    } else {
      d.type = first;
    }
    expect_op("{");
    while (!is_op("}")) {
      if (at(T::Eof)) fail("AE0002", d.line, d.col, "unclosed impl body");
      if (is_op("#")) {
        attribute();
        continue;
      }
      eat_id("pub");
      d.methods.push_back(fn());
    }
    expect_op("}");
    return d;
  }

  // `<T, [M, K], 3>` after a type name: the type arguments (shapes and
  // constants are skipped).
  std::vector<std::shared_ptr<TyExpr>> type_args() {
    std::vector<std::shared_ptr<TyExpr>> out;
    expect_op("<");
    while (!is_op(">") && !is_op(">>") && !is_op(">=")) {
      if (is_op("[")) {
        next();
        while (!is_op("]")) {
          expr_prec(9);
          if (!eat_op(",")) break;
        }
        expect_op("]");
      } else if (at(T::Int)) {
        next();
      } else {
        out.push_back(type());
      }
      if (!eat_op(",")) break;
    }
    close_angle();
    return out;
  }

  std::shared_ptr<TyExpr> type() {
    auto t = std::make_shared<TyExpr>();
    t->line = cur().line;
    t->col = cur().col;
    if (eat_op("&")) {
      eat_id("mut");
      auto in = type();
      if (in->name == "str") {
        t->name = "str";
        return t;
      }
      in->ref = true;  // a pointer for scalars and structs; tensors (handles) and arrays travel as they are
      return in;
    }
    if (eat_id("impl")) {  // `impl Trait (+ Trait)`: an anonymous type parameter of the function
      ident();
      while (eat_op("+")) ident();
      t->name = "impl$" + std::to_string(++impl_params_);
      return t;
    }
    if (eat_op("[")) {
      t->name = "[]";
      t->inner = type();
      if (eat_op("]")) {  // `[T]` (written `&[T]`): a slice
        t->name = "slice";
        return t;
      }
      expect_op(";");
      t->dims.push_back(expr());
      expect_op("]");
      return t;
    }
    if (eat_op("(")) {
      if (eat_op(")")) {
        t->name = "()";
        return t;
      }
      t->name = "tuple";
      while (!is_op(")")) {
        t->elems.push_back(type());
        if (!eat_op(",")) break;
      }
      expect_op(")");
      if (t->elems.size() == 1) return t->elems[0];  // `(T)` is T
      return t;
    }
    t->name = ident();
    while (is_op("::")) {  // a path: the last segment names the type
      next();
      t->name = ident();
    }
    if (t->name == "Tensor" && is_op("<") && peek().t == T::Id && peek(2).t == T::Op && peek(2).s == ",") {
      expect_op("<");
      t->elem = ident();
      expect_op(",");
      expect_op("[");
      while (!is_op("]")) {
        t->dims.push_back(expr_prec(9));  // no comparison operators inside a shape
        if (!eat_op(",")) break;
      }
      expect_op("]");
      close_angle();
    } else if (is_op("<")) {
      t->targs = type_args();
      t->generic = true;
    }
    return t;
  }

  // A function; in a trait (`trait_method`) the body may be left out.
  Fn fn(bool trait_method = false) {
    Fn f;
    f.line = cur().line;
    f.col = cur().col;
    eat_id("unsafe");
    eat_id("async");
    if (eat_id("extern")) {
      f.is_extern = true;
      if (at(T::Str)) next();  // extern "C"
    }
    if (!eat_id("fn")) fail("AE0002", cur().line, cur().col, "expected 'fn'");
    f.name = ident();
    f.generics = generic_params();
    expect_op("(");
    while (!is_op(")")) {
      Param p;
      if (is_op("&") && (peek().s == "self" || (peek().s == "mut" && peek(2).s == "self"))) {
        next();
        eat_id("mut");
        next();  // self
        p.name = "self";
        p.self_ref = true;
      } else {
        eat_id("mut");
        p.name = ident();
        if (p.name != "self" || is_op(":")) {
          expect_op(":");
          p.ty = type();
        }
      }
      f.params.push_back(p);
      if (!eat_op(",")) break;
    }
    expect_op(")");
    if (eat_op("->")) f.ret = type();
    for (auto& prm : f.params)  // `impl Trait` parameters / result: type parameters of their own
      if (prm.ty && prm.ty->name.rfind("impl$", 0) == 0) f.generics.push_back(prm.ty->name);
    if (f.ret && f.ret->name.rfind("impl$", 0) == 0) f.generics.push_back(f.ret->name);
    if (f.is_extern || (trait_method && is_op(";"))) {
      expect_op(";");
    } else {
      f.body = block();
    }
    return f;
  }

  BP block() {
    auto b = std::make_shared<Block>();
    b->line = cur().line;
    b->col = cur().col;
    expect_op("{");
    while (!is_op("}")) {
      if (at(T::Eof)) fail("AE0002", b->line, b->col, "unclosed block");
      if (eat_op(";")) continue;
      SP s = stmt();
      if (!s) {  // a trailing expression without ';' ends the block
        b->tail = last_expr_;
        if (!is_op("}")) fail("AE0002", cur().line, cur().col, "expected ';' or '}' after an expression");
        break;
      }
      b->stmts.push_back(s);
    }
    expect_op("}");
    return b;
  }

  static bool block_like(const EP& e) {
    return e->k == Expr::If || e->k == Expr::BlockE || e->k == Expr::LoopE || e->k == Expr::Match;
  }

  EP last_expr_;

  // A statement, or nullptr when an expression ends the block (its value is last_expr_).
  SP stmt() {
    auto s = std::make_shared<Stmt>();
    s->line = cur().line;
    s->col = cur().col;
    if (eat_id("let")) {
      s->k = Stmt::Let;
      s->mut = eat_id("mut");
      if (eat_op("(")) {  // let (a, b, _) = e
        while (!is_op(")")) {
          eat_id("mut");
          s->names.push_back(ident());
          if (!eat_op(",")) break;
        }
        expect_op(")");
        if (eat_op(":")) s->ty = type();
        expect_op("=");
        s->e = expr();
        expect_op(";");
        return s;
      }
      s->name = ident();
      if (eat_op(":")) s->ty = type();
      if (eat_op("=")) s->e = expr();
      expect_op(";");
      return s;
    }
    if (eat_id("while")) {
      s->k = Stmt::While;
      if (eat_id("let")) {
        s->pat = pattern();
        expect_op("=");
      }
      s->e = expr_nostruct();
      s->body = block();
      return s;
    }
    if (is_id("parallel") && peek().t == T::Id && peek().s == "for") next();  // `parallel for`: a for loop here
    if ((is_id("warp") || is_id("block")) && peek().t == T::Op && peek().s == "{") {
      // a warp / block region: its statements, in order, as a block
      const Tok at = cur();
      next();
      s->k = Stmt::ExprS;
      s->e = mk(Expr::BlockE, at);
      s->e->blk = block();
      return s;
    }
    if (eat_id("for")) {
      s->k = Stmt::For;
      s->name = ident();
      if (!eat_id("in")) fail("AE0002", cur().line, cur().col, "expected 'in'");
      const bool saved = no_struct_;
      no_struct_ = true;
      s->e = expr_prec(9);
      no_struct_ = saved;
      if (eat_op("..=")) {
        s->inclusive = true;
      } else if (!eat_op("..")) {  // `for x in slice`
        s->body = block();
        return s;
      }
      no_struct_ = true;
      s->e2 = expr_prec(9);
      no_struct_ = saved;
      s->body = block();
      return s;
    }
    if (eat_id("return")) {
      s->k = Stmt::Return;
      if (!is_op(";") && !is_op("}")) s->e = expr();
      eat_op(";");
      return s;
    }
    if (eat_id("break")) {
      s->k = Stmt::Break;
      eat_op(";");
      return s;
    }
    if (eat_id("continue")) {
      s->k = Stmt::Continue;
      eat_op(";");
      return s;
    }
    EP e = expr();
    static const std::set<std::string> assign = {"=", "+=", "-=", "*=", "/=", "%=", "&=", "|=", "^=", "<<=", ">>="};
    if (cur().t == T::Op && assign.count(cur().s)) {
      s->k = Stmt::Assign;
      s->op = cur().s;
      next();
      s->e = e;
      s->e2 = expr();
      expect_op(";");
      return s;
    }
    if (eat_op(";")) {
      s->k = Stmt::ExprS;
      s->e = e;
      return s;
    }
    if (is_op("}")) {
      last_expr_ = e;
      return nullptr;
    }
    if (block_like(e)) {  // `if c { .. }` followed by more statements
      s->k = Stmt::ExprS;
      s->e = e;
      return s;
    }
    fail("AE0002", cur().line, cur().col, "expected ';' after expression, found '" + cur().s + "'");
  }

  EP mk(Expr::K k, const Tok& at) {
    auto e = std::make_shared<Expr>();
    e->k = k;
    e->line = at.line;
    e->col = at.col;
    return e;
  }

  EP expr() {
    const bool saved = no_struct_;
    no_struct_ = false;
    EP e = expr_prec(0);
    no_struct_ = saved;
    return e;
  }
  // A condition or range: `Name {` there opens the block, not a struct literal.
  EP expr_nostruct() {
    const bool saved = no_struct_;
    no_struct_ = true;
    EP e = expr_prec(0);
    no_struct_ = saved;
    return e;
  }
  bool no_struct_ = false;
  int impl_params_ = 0;

  // ------------------------------------------------------------- macro_rules
  // Declarative macros expanded at parse time: `$x:frag` captures (an expr
  // fragment is substituted in parentheses), one level of `$( .. ) sep *`
  // repetition, rules tried in order; the expansion is parsed as a block
  // expression by a parser that shares this one's macro table.
  struct MacroRule {
    std::vector<Tok> matcher, body;
  };
  std::shared_ptr<std::map<std::string, std::vector<MacroRule>>> macros_ =
      std::make_shared<std::map<std::string, std::vector<MacroRule>>>();

  static bool opens(const Tok& t) { return t.t == T::Op && (t.s == "(" || t.s == "[" || t.s == "{"); }
  static bool closes(const Tok& t) { return t.t == T::Op && (t.s == ")" || t.s == "]" || t.s == "}"); }

  // The tokens between an opening delimiter here and its match (consumed).
  std::vector<Tok> group() {
    if (!opens(cur())) fail("AE0002", cur().line, cur().col, "expected '(', '[' or '{', found '" + cur().s + "'");
    std::vector<Tok> out;
    const Tok start = cur();
    next();
    int depth = 1;
    while (true) {
      if (at(T::Eof)) fail("AE0002", start.line, start.col, "unclosed macro group");
      if (opens(cur())) ++depth;
      if (closes(cur()) && --depth == 0) break;
      out.push_back(cur());
      next();
    }
    next();
    return out;
  }

  void macro_def() {
    next();  // macro_rules
    next();  // !
    const std::string name = ident();
    std::vector<MacroRule> rules;
    const bool paren = is_op("(");
    if (!is_op("{") && !paren) fail("AE0002", cur().line, cur().col, "expected '{' after the macro name");
    next();
    while (!is_op("}") && !is_op(")")) {
      if (at(T::Eof)) fail("AE0002", cur().line, cur().col, "unclosed macro_rules");
      MacroRule r;
      r.matcher = group();
      expect_op("=>");
      r.body = group();
      rules.push_back(r);
      if (!eat_op(";")) break;
    }
    next();
    if (paren) eat_op(";");
    (*macros_)[name] = rules;
  }

  using Caps = std::map<std::string, std::vector<std::vector<Tok>>>;

  // Tokens of one fragment starting at in[i]: up to the next `follow`
  // token at depth 0 (or the end); `ident` / `tt` take one token or group.
  static size_t take_fragment(const std::vector<Tok>& in, size_t i, const std::string& frag, const Tok* follow) {
    if (frag == "ident" || frag == "literal" || frag == "lifetime") return i < in.size() ? i + 1 : i;
    if (frag == "tt") {
      if (i >= in.size()) return i;
      if (!opens(in[i])) return i + 1;
      int d = 0;
      for (size_t k = i; k < in.size(); ++k) {
        if (opens(in[k])) ++d;
        if (closes(in[k]) && --d == 0) return k + 1;
      }
      return in.size();
    }
    int d = 0;
    size_t k = i;
    for (; k < in.size(); ++k) {
      if (d == 0 && follow && in[k].t == follow->t && in[k].s == follow->s) break;
      if (d == 0 && in[k].t == T::Op && (in[k].s == "," || in[k].s == ";" || in[k].s == "=>")) break;  // never inside an expr
      if (opens(in[k])) ++d;
      if (closes(in[k])) --d;
    }
    return k;
  }

  // Matches matcher m against in; captures into caps. One level of repetition.
  static bool macro_match(const std::vector<Tok>& m, const std::vector<Tok>& in, Caps& caps) {
    size_t mi = 0, ii = 0;
    while (mi < m.size()) {
      if (m[mi].s == "$" && mi + 1 < m.size() && m[mi + 1].s == "(") {  // $( inner ) sep? *
        size_t close = mi + 2;
        int d = 1;
        for (; close < m.size(); ++close) {
          if (opens(m[close])) ++d;
          if (closes(m[close]) && --d == 0) break;
        }
        std::vector<Tok> inner(m.begin() + (long)mi + 2, m.begin() + (long)close);
        size_t after = close + 1;
        const Tok* sep = nullptr;
        if (after < m.size() && m[after].s != "*" && m[after].s != "+" && m[after].s != "?") sep = &m[after++];
        if (after >= m.size()) return false;
        const std::string kind = m[after].s;
        const Tok* follow = after + 1 < m.size() ? &m[after + 1] : nullptr;
        for (size_t k = 0; k + 1 < inner.size(); ++k)
          if (inner[k].s == "$") caps[inner[k + 1].s];  // repeated variables exist even when empty
        int count = 0;
        while (ii < in.size() && !(follow && in[ii].t == follow->t && in[ii].s == follow->s)) {
          size_t j = 0;
          while (j < inner.size()) {
            if (inner[j].s == "$" && j + 3 < inner.size() + 1 && inner[j + 2].s == ":") {
              const Tok* f = sep ? sep : follow;
              if (j + 4 < inner.size()) f = &inner[j + 4];
              const size_t end = take_fragment(in, ii, inner[j + 3].s, f);
              if (end == ii) return false;
              caps[inner[j + 1].s].push_back(std::vector<Tok>(in.begin() + (long)ii, in.begin() + (long)end));
              ii = end;
              j += 4;
            } else {
              if (ii >= in.size() || in[ii].s != inner[j].s) return false;
              ++ii;
              ++j;
            }
          }
          ++count;
          if (sep) {
            if (ii < in.size() && in[ii].s == sep->s) ++ii;
            else break;
          }
        }
        if (kind == "+" && count == 0) return false;
        mi = after + 1;
        continue;
      }
      if (m[mi].s == "$" && mi + 3 < m.size() + 1 && m[mi + 2].s == ":") {  // $name:frag
        const Tok* follow = mi + 4 < m.size() ? &m[mi + 4] : nullptr;
        const size_t end = take_fragment(in, ii, m[mi + 3].s, follow);
        if (end == ii) return false;
        caps[m[mi + 1].s].push_back(std::vector<Tok>(in.begin() + (long)ii, in.begin() + (long)end));
        ii = end;
        mi += 4;
        continue;
      }
      if (ii >= in.size() || in[ii].s != m[mi].s) return false;
      ++ii;
      ++mi;
    }
    return ii == in.size();
  }

  static void macro_emit(const std::vector<Tok>& body, const Caps& caps, size_t rep, bool in_rep,
                         std::vector<Tok>& out) {
    for (size_t k = 0; k < body.size(); ++k) {
      const Tok& t = body[k];
      if (t.s == "$" && k + 1 < body.size() && body[k + 1].s == "(") {
        size_t close = k + 2;
        int d = 1;
        for (; close < body.size(); ++close) {
          if (opens(body[close])) ++d;
          if (closes(body[close]) && --d == 0) break;
        }
        std::vector<Tok> inner(body.begin() + (long)k + 2, body.begin() + (long)close);
        size_t after = close + 1;
        const Tok* sep = nullptr;
        if (after < body.size() && body[after].s != "*" && body[after].s != "+" && body[after].s != "?")
          sep = &body[after++];
        size_t n = 0;
        for (size_t j = 0; j + 1 < inner.size(); ++j)
          if (inner[j].s == "$" && caps.count(inner[j + 1].s)) n = std::max(n, caps.at(inner[j + 1].s).size());
        for (size_t r = 0; r < n; ++r) {
          if (r && sep) out.push_back(*sep);
          macro_emit(inner, caps, r, true, out);
        }
        k = after;
        continue;
      }
      if (t.s == "$" && k + 1 < body.size() && caps.count(body[k + 1].s)) {
        const auto& v = caps.at(body[k + 1].s);
        const size_t idx = in_rep ? rep : 0;
        if (idx < v.size()) {
          Tok lp = t, rp = t;
          lp.t = rp.t = T::Op;
          lp.s = "(";
          rp.s = ")";
          out.push_back(lp);
          out.insert(out.end(), v[idx].begin(), v[idx].end());
          out.push_back(rp);
        }
        ++k;
        continue;
      }
      out.push_back(t);
    }
  }

  EP expand_macro(const Tok& at, const std::string& name) {
    std::vector<Tok> in = group();
    for (const MacroRule& r : (*macros_)[name]) {
      Caps caps;
      if (!macro_match(r.matcher, in, caps)) continue;
      std::vector<Tok> toks;
      Tok lb = at, rb = at;
      lb.t = rb.t = T::Op;
      lb.s = "{";
      rb.s = "}";
      toks.push_back(lb);
      macro_emit(r.body, caps, 0, false, toks);
      toks.push_back(rb);
      Tok eof = at;
      eof.t = T::Eof;
      eof.s = "";
      toks.push_back(eof);
      Parser sub(toks);
      sub.macros_ = macros_;
      return sub.expr();
    }
    fail("AE0002", at.line, at.col, "no rule of macro `" + name + "!` matches this invocation");
  }

  // println! / print!: the format string's `{}` / `{:..}` holes take the
  // arguments in order; literal text between them is printed as is.
  EP format_macro(const Tok& at, bool newline) {
    expect_op("(");
    if (cur().t != T::Str) fail("AE0002", cur().line, cur().col, "expected a format string");
    const std::string fmt = cur().s;
    next();
    std::vector<EP> args;
    while (eat_op(",")) {
      if (is_op(")")) break;
      args.push_back(expr());
    }
    expect_op(")");
    EP blk = mk(Expr::BlockE, at);
    blk->blk = std::make_shared<Block>();
    auto print = [&](EP arg) {
      auto st = std::make_shared<Stmt>();
      st->k = Stmt::ExprS;
      EP c = mk(Expr::Call, at);
      c->s = "print";
      c->a = {arg};
      st->e = c;
      blk->blk->stmts.push_back(st);
    };
    auto lit = [&](const std::string& text) {
      if (text.empty()) return;
      EP sx = mk(Expr::Str, at);
      sx->s = text;
      print(sx);
    };
    std::string text;
    size_t ai = 0;
    for (size_t i = 0; i < fmt.size(); ++i) {
      if (fmt[i] == '{' && i + 1 < fmt.size() && fmt[i + 1] == '{') {
        text += '{';
        ++i;
      } else if (fmt[i] == '}' && i + 1 < fmt.size() && fmt[i + 1] == '}') {
        text += '}';
        ++i;
      } else if (fmt[i] == '{') {
        const size_t close = fmt.find('}', i);
        if (close == std::string::npos) fail("AE0002", at.line, at.col, "unclosed '{' in a format string");
        lit(text);
        text.clear();
        if (ai >= args.size()) fail("AE0541", at.line, at.col, "format string has more holes than arguments");
        print(args[ai++]);
        i = close;
      } else {
        text += fmt[i];
      }
    }
    if (newline) text += '\n';
    lit(text);
    return blk;
  }

  static int prec(const std::string& op) {
    if (op == "||") return 1;
    if (op == "&&") return 2;
    if (op == "==" || op == "!=" || op == "<" || op == "<=" || op == ">" || op == ">=") return 3;
    if (op == "|") return 4;
    if (op == "^") return 5;
    if (op == "&") return 6;
    if (op == "<<" || op == ">>") return 7;
    if (op == "+" || op == "-") return 8;
    if (op == "*" || op == "/" || op == "%") return 9;
    return -1;
  }

  EP expr_prec(int min) {
    EP lhs = unary();
    while (cur().t == T::Op) {
      const std::string op = cur().s;
      const int p = prec(op);
      if (p < 0 || p < min) break;
      const Tok at = cur();
      next();
      EP rhs = expr_prec(p + 1);
      EP b = mk(Expr::Binary, at);
      b->s = op;
      b->a = {lhs, rhs};
      lhs = b;
    }
    return lhs;
  }

  EP unary() {
    const Tok at = cur();
    if (eat_op("-") || eat_op("!")) {
      EP e = mk(Expr::Unary, at);
      e->s = at.s;
      e->a = {unary()};
      return e;
    }
    if (eat_op("&")) {
      EP e = mk(Expr::Ref, at);
      e->mut = eat_id("mut");
      e->a = {unary()};
      return e;
    }
    if (eat_op("*")) {  // dereference (of a by-value binding: the value itself)
      EP e = mk(Expr::Deref, at);
      e->a = {unary()};
      return e;
    }
    return cast_expr(postfix(primary()));
  }

  EP cast_expr(EP e) {
    while (is_id("as")) {
      const Tok at = cur();
      next();
      EP c = mk(Expr::Cast, at);
      c->cast = type();
      c->a = {e};
      e = c;
    }
    return e;
  }

  EP postfix(EP e) {
    for (;;) {
      const Tok at = cur();
      if (eat_op(".")) {
        if (is_id("await") && !(peek().t == T::Op && peek().s == "(")) {
          next();  // `f().await`: an async fn runs to completion where it is awaited (one task)
          continue;
        }
        if (at_field_name()) {  // field access: `x.field` / `x.0`
          EP f = mk(Expr::Field, at);
          f->s = cur().s;
          next();
          f->a = {e};
          e = f;
          continue;
        }
        std::string m = ident();
        EP c = mk(Expr::Method, at);
        c->s = m;
        c->a = {e};
        expect_op("(");
        while (!is_op(")")) {
          c->a.push_back(expr());
          if (!eat_op(",")) break;
        }
        expect_op(")");
        e = c;
      } else if (is_op("?")) {  // early return unless the Ok / Some variant
        next();
        EP t = mk(Expr::Try, at);
        t->a = {e};
        e = t;
      } else if (is_op("[")) {
        next();
        EP ix = mk(Expr::Index, at);
        if (is_op("..")) {  // [..b] / [..]
          next();
          ix->s = "..";
          ix->a = {e, nullptr, is_op("]") ? nullptr : expr()};
        } else {
          EP first = expr_prec(9);
          if (eat_op("..")) {  // [a..b] / [a..]
            ix->s = "..";
            ix->a = {e, first, is_op("]") ? nullptr : expr()};
          } else {
            ix->a = {e, first};
            while (cur().t == T::Op && prec(cur().s) >= 0) {  // the rest of a full expression
              const std::string op = cur().s;
              const Tok o = cur();
              next();
              EP b = mk(Expr::Binary, o);
              b->s = op;
              b->a = {ix->a[1], expr_prec(prec(op) + 1)};
              ix->a[1] = b;
            }
          }
        }
        expect_op("]");
        e = ix;
      } else {
        return e;
      }
    }
  }

  bool at_field_name() const {
    if (cur().t == T::Int) return true;
    return cur().t == T::Id && !(peek().t == T::Op && (peek().s == "(" || peek().s == "::"));
  }

  EP primary() {
    const Tok at = cur();
    switch (at.t) {
      case T::Int: {
        next();
        EP e = mk(Expr::Int, at);
        e->s = at.s;
        return e;
      }
      case T::Float: {
        next();
        EP e = mk(Expr::Float, at);
        e->s = at.s;
        return e;
      }
      case T::Str: {
        next();
        EP e = mk(Expr::Str, at);
        e->s = at.s;
        return e;
      }
      case T::Char: {
        next();
        EP e = mk(Expr::Char, at);
        e->s = at.s;
        return e;
      }
      default: break;
    }
    if (eat_op("(")) {
      if (eat_op(")")) {
        EP e = mk(Expr::BlockE, at);  // unit
        e->blk = std::make_shared<Block>();
        return e;
      }
      EP e = expr();
      if (is_op(",")) {  // a tuple
        EP t = mk(Expr::TupleLit, at);
        t->a = {e};
        while (eat_op(",")) {
          if (is_op(")")) break;
          t->a.push_back(expr());
        }
        expect_op(")");
        return t;
      }
      expect_op(")");
      return e;
    }
    if (is_op("|") || is_op("||")) {  // a closure: |a: T, b| body  /  || body
      EP e = mk(Expr::Closure, at);
      e->closure = std::make_shared<Fn>();
      e->closure->line = at.line;
      e->closure->col = at.col;
      if (eat_op("|")) {
        while (!is_op("|")) {
          Param prm;
          prm.name = ident();
          if (eat_op(":")) prm.ty = type();
          e->closure->params.push_back(prm);
          if (!eat_op(",")) break;
        }
        expect_op("|");
      } else {
        next();  // ||
      }
      if (eat_op("->")) e->closure->ret = type();
      e->closure->body = std::make_shared<Block>();
      e->closure->body->tail = expr();
      return e;
    }
    if (is_op("[")) {
      next();
      if (eat_op("]")) fail("AE0500", at.line, at.col, "empty array literal");
      EP first = expr();
      if (eat_op(";")) {
        EP e = mk(Expr::ArrayRep, at);
        e->a = {first, expr()};
        expect_op("]");
        return e;
      }
      EP e = mk(Expr::ArrayLit, at);
      e->a = {first};
      while (eat_op(",")) {
        if (is_op("]")) break;
        e->a.push_back(expr());
      }
      expect_op("]");
      return e;
    }
    if (is_op("{")) {
      EP e = mk(Expr::BlockE, at);
      e->blk = block();
      return e;
    }
    if (eat_id("match")) {
      EP e = mk(Expr::Match, at);
      e->a = {expr_nostruct()};
      expect_op("{");
      while (!is_op("}")) {
        if (cur().t == T::Eof) fail("AE0002", at.line, at.col, "unclosed match");
        e->pats.push_back(pattern());
        e->guards.push_back(eat_id("if") ? expr() : nullptr);
        expect_op("=>");
        EP arm = expr();
        e->a.push_back(arm);
        if (!eat_op(",") && !is_op("}") && !block_like(arm))
          fail("AE0002", cur().line, cur().col, "expected ',' after a match arm, found '" + cur().s + "'");
      }
      expect_op("}");
      return e;
    }
    if (is_id("if") && peek().t == T::Id && peek().s == "let") {  // if let P = e { .. } else { .. }
      next();
      next();
      EP e = mk(Expr::Match, at);
      e->pats.push_back(pattern());
      expect_op("=");
      e->a = {expr_nostruct()};
      EP then_e = mk(Expr::BlockE, at);
      then_e->blk = block();
      e->a.push_back(then_e);
      e->guards.push_back(nullptr);
      auto wild = std::make_shared<Pat>();
      e->pats.push_back(wild);
      e->guards.push_back(nullptr);
      EP else_e = mk(Expr::BlockE, at);
      if (eat_id("else")) {
        if (is_id("if")) {
          else_e->blk = std::make_shared<Block>();
          else_e->blk->tail = primary();
        } else {
          else_e->blk = block();
        }
      } else {
        else_e->blk = std::make_shared<Block>();
      }
      e->a.push_back(else_e);
      return e;
    }
    if (eat_id("if")) {
      EP e = mk(Expr::If, at);
      e->a = {expr_nostruct()};
      e->blk = block();
      if (eat_id("else")) {
        if (is_id("if")) {
          auto b = std::make_shared<Block>();
          b->tail = primary();  // else if: the nested if is the else block's value
          e->blk2 = b;
        } else {
          e->blk2 = block();
        }
      }
      return e;
    }
    if (eat_id("unsafe")) {  // no borrow checker here: an unsafe block is a block
      EP e = mk(Expr::BlockE, at);
      e->blk = block();
      return e;
    }
    if (eat_id("loop")) {
      EP e = mk(Expr::LoopE, at);
      e->blk = block();
      return e;
    }
    if (eat_id("true") || eat_id("false")) {
      EP e = mk(Expr::BoolL, at);
      e->s = at.s;
      return e;
    }
    if (at.t == T::Id) {
      std::string name = ident();
      while (is_op("::")) {  // a path; code generation resolves `Type::item`, else the last segment
        next();
        name += "::" + ident();
      }
      if (!no_struct_ && is_op("{") &&
          (peek().s == "}" || (peek().t == T::Id && (peek(2).s == ":" || peek(2).s == "," || peek(2).s == "}")))) {
        EP e = mk(Expr::StructLit, at);  // `Name { field: value, .. }` (or the `field` shorthand)
        e->s = name;
        next();
        while (!is_op("}")) {
          const Tok f = cur();
          const std::string fname = ident();
          e->fields.push_back(fname);
          if (eat_op(":")) {
            e->a.push_back(expr());
          } else {
            EP v = mk(Expr::Var, f);
            v->s = fname;
            e->a.push_back(v);
          }
          if (!eat_op(",")) break;
        }
        expect_op("}");
        return e;
      }
      if (is_op("!") && (peek().s == "(" || peek().s == "[" || peek().s == "{")) {
        next();  // !
        if ((name == "println" || name == "print") && !macros_->count(name)) return format_macro(at, name == "println");
        if (!macros_->count(name)) fail("AE0500", at.line, at.col, "macro `" + name + "!` is not defined here");
        return expand_macro(at, name);
      }
      if (eat_op("(")) {
        EP e = mk(Expr::Call, at);
        e->s = name;
        while (!is_op(")")) {
          e->a.push_back(expr());
          if (!eat_op(",")) break;
        }
        expect_op(")");
        return e;
      }
      EP e = mk(Expr::Var, at);
      e->s = name;
      return e;
    }
    fail("AE0002", at.line, at.col, "unexpected '" + at.s + "'");
  }
};

// ============================================================================ tensor method lowering
// A method on a device tensor is one runtime call: (receiver, the call's
// arguments in order, then the integers its shape recipe derives from the
// receiver's and first argument's static shapes).
struct MethodRule {
  const char* fn;
  int recipe;
};
enum Recipe { MKN_MATMUL, MKN_NT, MKN_TN, MKN_BWD_RHS, MKN_BWD_LHS, ROWS_COLS, NUMEL, MKN_2D };

const std::map<std::string, MethodRule>& method_rules() {
  static const std::map<std::string, MethodRule> m = {
      {"matmul", {"aether_op_matmul_f32_cuda", MKN_MATMUL}},
      {"matmul_gelu", {"aether_op_matmul_gelu_f32_cuda", MKN_2D}},
      {"matmul_t", {"aether_op_matmul_nt_f32_cuda", MKN_NT}},
      {"matmul_tn", {"aether_op_matmul_tn_f32_cuda", MKN_TN}},
      {"matmul_backward_rhs", {"aether_op_matmul_backward_rhs_f32_cuda", MKN_BWD_RHS}},
      {"matmul_backward_lhs", {"aether_op_matmul_backward_lhs_f32_cuda", MKN_BWD_LHS}},
      {"cross_entropy", {"aether_op_cross_entropy_f32_cuda", ROWS_COLS}},
      {"cross_entropy_backward", {"aether_op_cross_entropy_backward_f32_cuda", ROWS_COLS}},
      {"softmax", {"aether_op_softmax_f32_cuda", ROWS_COLS}},
      {"softmax_backward", {"aether_op_softmax_backward_f32_cuda", ROWS_COLS}},
      {"softmax_backward_scaled", {"aether_op_softmax_backward_scaled_f32_cuda", ROWS_COLS}},
      {"layer_norm", {"aether_op_layer_norm_f32_cuda", ROWS_COLS}},
      {"add_layer_norm", {"aether_op_add_layer_norm_f32_cuda", ROWS_COLS}},
      {"layer_norm_backward_dx", {"aether_op_layer_norm_backward_dx_f32_cuda", ROWS_COLS}},
      {"layer_norm_backward_params", {"aether_op_layer_norm_backward_params_f32_cuda", ROWS_COLS}},
      {"adamw_step", {"aether_op_adamw_step_f32_cuda", NUMEL}},
      {"add", {"aether_op_add_f32_cuda", NUMEL}},
      {"gelu", {"aether_op_gelu_f32_cuda", NUMEL}},
      {"gelu_backward", {"aether_op_gelu_backward_f32_cuda", NUMEL}},
      {"scale", {"aether_op_scale_f32_cuda", NUMEL}},
  };
  return m;
}

// ============================================================================ fusion peephole
// `x.matmul(&w, &mut h); h.gelu(&mut h);` -> `x.matmul_gelu(&w, &mut h);`
// (the intermediate is updated in place, so no later read can see the
// unfused value). Applied to every block, nested blocks first.
int fuse_block(Block& b);
int fuse_expr(const EP& e) {
  if (!e) return 0;
  int n = 0;
  if (e->blk) n += fuse_block(*e->blk);
  if (e->blk2) n += fuse_block(*e->blk2);
  for (auto& a : e->a) n += fuse_expr(a);
  return n;
}
static std::string var_of(const EP& e) {
  if (!e) return "";
  if (e->k == Expr::Ref && !e->a.empty()) return var_of(e->a[0]);
  return e->k == Expr::Var ? e->s : "";
}
int fuse_block(Block& b) {
  int n = 0;
  for (auto& s : b.stmts) {
    if (s->body) n += fuse_block(*s->body);
    n += fuse_expr(s->e) + fuse_expr(s->e2);
  }
  n += fuse_expr(b.tail);
  for (size_t i = 0; i + 1 < b.stmts.size(); ++i) {
    Stmt &s0 = *b.stmts[i], &s1 = *b.stmts[i + 1];
    if (s0.k != Stmt::ExprS || s1.k != Stmt::ExprS || s0.e->k != Expr::Method || s1.e->k != Expr::Method) continue;
    const Expr &m0 = *s0.e, &m1 = *s1.e;
    if (m0.s != "matmul" || m1.s != "gelu" || m0.a.size() != 3 || m1.a.size() != 2) continue;
    const std::string out = var_of(m0.a[2]);
    if (out.empty() || var_of(m1.a[0]) != out || var_of(m1.a[1]) != out || m1.a[1]->k != Expr::Ref || !m1.a[1]->mut)
      continue;
    s0.e->s = "matmul_gelu";
    b.stmts.erase(b.stmts.begin() + (long)i + 1);
    ++n;
  }
  return n;
}

// ============================================================================ C code generation
struct Local {
  Ty ty;
  std::string c;
};
struct FnSig {
  std::vector<Ty> params;
  Ty ret;
  std::string c;
  bool is_extern = false;
  int self_kind = 0;  // a method's receiver: 0 none, 1 by value, 2 by pointer (`&self`)
};

class Gen {
 public:
  Gen(Program& p, std::string stdlib_dir, std::string src_dir)
      : p_(p), stdlib_(std::move(stdlib_dir)), srcdir_(std::move(src_dir)) {}

  std::string run() {
    for (auto& c : p_.consts) const_src_[c.name] = &c;
    declare_structs();
    synthesize_defaults();
    for (auto& f : p_.fns) declare(f);
    for (auto& im : p_.impls) {
      if (gstructs_.count(im.type)) {
        gimpls_[im.type].push_back(&im);
        continue;
      }
      if (!structs_.count(im.type))
        fail("AE0500", im.line, im.col, "impl for '" + im.type + "', which is not a struct of this program");
      self_type_ = im.type;
      for (auto& m : im.methods) declare_method(im.type, m);
    }
    self_type_.clear();
    std::ostringstream o;
    o << "/* generated by aetherc */\n#include <stdint.h>\n#include <stdio.h>\n#include <stdlib.h>\n#include <math.h>\n\n";
    o << "int64_t aether_dev_alloc_f32(int32_t);\nint64_t aether_dev_alloc_i32(int32_t);\n"
         "int32_t aether_dev_free_f32(int64_t);\nint32_t aether_dev_free_i32(int64_t);\n";
    o << "static void ae_drop_f32(int64_t* h) { if (*h > 0) aether_dev_free_f32(*h); }\n"
         "static void ae_drop_i32(int64_t* h) { if (*h > 0) aether_dev_free_i32(*h); }\n\n";
    std::set<std::string> pre = {"aether_dev_alloc_f32", "aether_dev_alloc_i32", "aether_dev_free_f32",
                                 "aether_dev_free_i32"};
    for (auto& kv : sigs_) {
      const FnSig& s = kv.second;
      if (!s.is_extern || pre.count(kv.first)) continue;
      o << ctype(s.ret) << " " << s.c << "(" << plist(s) << ");\n";
    }
    o << "\n";
    // Bodies first: they can add tuple types and lifted closures, whose
    // declarations the file needs ahead of every body.
    std::ostringstream defs;
    for (auto& f : p_.fns)
      if (!f.is_extern && f.generics.empty()) defs << fn_def(f, f.name);
    for (auto& im : p_.impls) {
      if (gstructs_.count(im.type)) continue;
      self_type_ = im.type;
      for (auto& m : im.methods) defs << fn_def(m, im.type + "::" + m.name);
    }
    self_type_.clear();
    o << struct_decls() << "\n";
    for (auto& c : p_.consts) {
      Ty t = resolve(*c.ty);
      o << "static const " << ctype(t) << " aec_" << c.name << " = " << lit_of(eval_const(c.e), t) << ";\n";
    }
    for (auto& f : p_.fns)
      if (!f.is_extern && f.generics.empty())
        o << "static " << ctype(sigs_[f.name].ret) << " " << sigs_[f.name].c << "(" << plist(sigs_[f.name]) << ");\n";
    for (auto& im : p_.impls)
      if (!gstructs_.count(im.type))
      for (auto& m : im.methods) {
        const FnSig& sg = sigs_[im.type + "::" + m.name];
        o << "static " << ctype(sg.ret) << " " << sg.c << "(" << plist(sg) << ");\n";
      }
    o << lifted_protos_ << "\n" << lifted_defs_ << defs.str();
    if (test_mode_) {  // --test: every #[test] fn in source order; 0 = pass
      o << "int main(void) {\n  int failed = 0, total = 0;\n";
      for (auto& f : p_.fns) {
        if (!f.is_test) continue;
        const FnSig& sg = sigs_[f.name];
        if (!sg.params.empty()) fail("AE0541", f.line, f.col, "#[test] fn '" + f.name + "' takes no arguments");
        o << "  { int r = " << (sg.ret.b == B::Void ? "(" + sg.c + "(), 0)" : "(int)" + sg.c + "()") << "; ++total; "
          << "printf(\"%s " << f.name << "\\n\", r == 0 ? \"PASS\" : \"FAIL\"); if (r) ++failed; }\n";
      }
      o << "  if (failed == 0) printf(\"ALL PASSED (%d tests)\\n\", total);\n"
           "  else printf(\"%d of %d tests FAILED\\n\", failed, total);\n  return failed != 0;\n}\n";
      return o.str();
    }
    if (!sigs_.count("main") || sigs_["main"].is_extern) fail("AE0580", 1, 1, "program has no `fn main`");
    const FnSig& m = sigs_["main"];
    o << "int main(void) {\n";
    if (m.ret.b == B::Void)
      o << "  aef_main();\n  return 0;\n}\n";
    else
      o << "  return (int)aef_main();\n}\n";
    return o.str();
  }

  // `use a::b;` loads <stdlib>/b.aether (or <source dir>/b.aether) and
  // merges its extern declarations and constants.
  static void resolve_uses(Program& p, const std::string& stdlib, const std::string& srcdir,
                           std::set<std::string>& seen);

 private:
  Program& p_;
  std::string stdlib_, srcdir_;

 public:
  bool test_mode_ = false;

 private:
  std::map<std::string, FnSig> sigs_;
  std::map<std::string, const Const*> const_src_;
  std::map<std::string, std::pair<Ty, double>> const_val_;
  std::vector<std::map<std::string, Local>> scopes_;
  Ty ret_;
  int uniq_ = 0;
  int indent_ = 1;

  static std::string plist(const FnSig& s) {
    if (s.params.empty()) return "void";
    std::string r;
    for (size_t i = 0; i < s.params.size(); ++i)
      r += (i ? ", " : "") + ctype(s.params[i]) + (i == 0 && s.self_kind == 2 ? "*" : "");
    return r;
  }

  struct V {  // a generated C expression and its type
    std::string c;
    Ty t;
  };

  // --------------------------------------------------------------- structs and impls
  struct StructInfo {
    std::vector<std::pair<std::string, Ty>> fields;
  };
  std::map<std::string, StructInfo> structs_;
  std::string self_type_;  // the impl whose methods are being declared / generated

  Ty struct_ty(const std::string& n) const {
    Ty t;
    t.b = B::Struct;
    t.sname = n;
    return t;
  }

  // Generics: functions, structs and impls are specialised per use;
  // tsubst_ maps the type parameters of the item being specialised.
  std::map<std::string, const Fn*> gfns_;
  std::map<std::string, const StructDef*> gstructs_;
  std::map<std::string, std::vector<const ImplDef*>> gimpls_;
  std::map<std::string, std::pair<std::string, std::map<std::string, Ty>>> spec_of_;  // W__i64 -> (W, {T: i64})
  std::map<std::string, Ty> tsubst_;

  static std::string mangle(const Ty& t) {
    std::string c = ctype(t);
    if (c.rfind("aes_", 0) == 0) c = c.substr(4);
    for (char& ch : c)
      if (!std::isalnum((unsigned char)ch)) ch = '_';
    return c;
  }

  std::map<std::string, const EnumDef*> genums_;

  // A generic enum's instance: a tagged struct like any enum with payloads.
  Ty specialize_enum(const std::string& base, const std::vector<Ty>& args, int line, int col) {
    const EnumDef& d = *genums_.at(base);
    if (args.size() != d.generics.size())
      fail("AE0522", line, col, "`" + base + "` takes " + std::to_string(d.generics.size()) + " type arguments");
    std::string name = base;
    std::map<std::string, Ty> sub;
    for (size_t i = 0; i < args.size(); ++i) {
      name += "__" + mangle(args[i]);
      sub[d.generics[i]] = args[i];
    }
    if (!enums_.count(name)) {
      auto saved = tsubst_;
      tsubst_ = sub;
      EnumInfo in;
      in.unit_only = false;
      for (auto& v : d.variants) {
        std::vector<Ty> ts;
        for (auto& t : v.second) ts.push_back(resolve(*t));
        in.variants.push_back({v.first, ts});
      }
      tsubst_ = saved;
      enums_[name] = in;
      tuple_names_.push_back(name);
      spec_of_[name] = {base, sub};
    }
    return struct_ty(name);
  }

  // The instance of generic enum `base` a path names: the expected type's,
  // else one bound from the payload values (unbound parameters: i64).
  std::string enum_instance(const std::string& base, const std::string& variant, const std::vector<EP>& payload,
                            const Ty& hint, int line, int col) {
    if (hint.b == B::Struct && spec_of_.count(hint.sname) && spec_of_[hint.sname].first == base) return hint.sname;
    const EnumDef& d = *genums_.at(base);
    std::map<std::string, Ty> sub;
    for (auto& v : d.variants)
      if (v.first == variant)
        for (size_t k = 0; k < v.second.size() && k < payload.size(); ++k)
          if (std::count(d.generics.begin(), d.generics.end(), v.second[k]->name) && !sub.count(v.second[k]->name))
            sub[v.second[k]->name] = gen(payload[k], prim(B::Unknown)).t;
    std::vector<Ty> args;
    for (auto& g : d.generics) args.push_back(sub.count(g) ? sub[g] : prim(B::I64));
    return specialize_enum(base, args, line, col).sname;
  }

  Ty specialize_struct(const std::string& base, const std::vector<Ty>& args, int line, int col) {
    const StructDef& d = *gstructs_.at(base);
    if (args.size() != d.generics.size())
      fail("AE0522", line, col, "`" + base + "` takes " + std::to_string(d.generics.size()) + " type arguments");
    std::string name = base;
    std::map<std::string, Ty> sub;
    for (size_t i = 0; i < args.size(); ++i) {
      name += "__" + mangle(args[i]);
      sub[d.generics[i]] = args[i];
    }
    if (!structs_.count(name)) {
      auto saved = tsubst_;
      tsubst_ = sub;
      StructInfo in;
      for (auto& f : d.fields) in.fields.push_back({f.name, resolve(*f.ty)});
      tsubst_ = saved;
      structs_[name] = in;
      tuple_names_.push_back(name);
      spec_of_[name] = {base, sub};
    }
    return struct_ty(name);
  }

  // Declares and generates `method` of a specialised generic struct.
  bool specialize_method(const std::string& sname, const std::string& method) {
    auto sp = spec_of_.find(sname);
    if (sp == spec_of_.end() || !gimpls_.count(sp->second.first)) return false;
    for (const ImplDef* im : gimpls_[sp->second.first])
      for (auto& m : im->methods) {
        if (m.name != method) continue;
        auto saved_sub = tsubst_;
        auto saved_self = self_type_;
        tsubst_ = sp->second.second;
        self_type_ = sname;
        declare_method(sname, m);
        emit_lazy(m, sname + "::" + m.name);
        tsubst_ = saved_sub;
        self_type_ = saved_self;
        return true;
      }
    return false;
  }

  // Generates a function body now, outside the one being generated.
  void emit_lazy(const Fn& f, const std::string& key) {
    auto saved_scopes = scopes_;
    const Ty saved_ret = ret_;
    const int saved_indent = indent_;
    const FnSig& sg = sigs_[key];
    lifted_protos_ += "static " + ctype(sg.ret) + " " + sg.c + "(" + plist(sg) + ");\n";
    lifted_defs_ += fn_def(f, key);
    scopes_ = saved_scopes;
    ret_ = saved_ret;
    indent_ = saved_indent;
  }

  // A call of generic function `n`: type parameters bound from the
  // arguments' types (then from the expected type), specialised once.
  V generic_call(const EP& e, const std::string& n, const Ty& hint) {
    const Fn& f = *gfns_.at(n);
    if (f.params.size() != e->a.size())
      fail("AE0541", e->line, e->col, "'" + n + "' takes " + std::to_string(f.params.size()) + " arguments, got " +
                                          std::to_string(e->a.size()));
    std::vector<V> args;
    std::map<std::string, Ty> sub;
    const std::set<std::string> gs(f.generics.begin(), f.generics.end());
    for (size_t i = 0; i < e->a.size(); ++i) {
      args.push_back(gen(e->a[i], prim(B::Unknown)));
      const auto& pt = f.params[i].ty;
      if (pt && gs.count(pt->name) && !sub.count(pt->name)) {
        Ty t = args.back().t;
        t.ref = false;
        sub[pt->name] = t;
      }
    }
    for (auto& g : f.generics)
      if (!sub.count(g)) sub[g] = (f.ret && f.ret->name == g && hint.b != B::Unknown && hint.b != B::Void) ? hint : prim(B::I64);
    std::string key = n;
    for (auto& g : f.generics) key += "__" + mangle(sub[g]);
    if (!sigs_.count(key)) {
      auto saved = tsubst_;
      tsubst_ = sub;
      FnSig s;
      for (auto& prm : f.params) s.params.push_back(resolve(*prm.ty));
      s.ret = f.ret ? resolve(*f.ret) : prim(B::Void);
      s.c = "aef_" + key;
      sigs_[key] = s;
      emit_lazy(f, key);
      tsubst_ = saved;
    }
    const FnSig& s = sigs_[key];
    std::string list;
    for (size_t i = 0; i < args.size(); ++i) list += (i ? ", " : "") + conv(args[i], s.params[i]);
    return {s.c + "(" + list + ")", s.ret};
  }

  // Slices `&[T]`: a C struct {T* ptr; int64_t len}.
  std::map<std::string, Ty> slice_elem_;
  Ty slice_ty(const Ty& elem) {
    const std::string n = "S_" + mangle(elem);
    if (!structs_.count(n)) {
      Ty pt = elem;
      pt.ref = true;
      StructInfo& in = structs_[n];
      in.fields = {{"ptr", pt}, {"len", prim(B::I64)}};
      tuple_names_.push_back(n);
      slice_elem_[n] = elem;
    }
    return struct_ty(n);
  }
  bool is_slice(const Ty& t) const { return t.b == B::Struct && !t.ref && slice_elem_.count(t.sname); }

  // `&h[a..b]`: a slice of a slice, or of a runtime vector / string handle
  // (an i64) read through the handle's pointer and length accessors.
  V slice_range(const EP& e, const Ty& hint) {
    V b = deref(gen(e->a[0], prim(B::Unknown)));
    Ty st;
    std::string ptr, len, pre;
    const std::string t = "sl_" + std::to_string(++uniq_);
    if (is_slice(b.t)) {
      st = b.t;
      pre = ctype(st) + " " + t + " = " + b.c + "; ";
      ptr = t + ".f_ptr";
      len = t + ".f_len";
    } else if (b.t.b == B::Array) {  // a fixed array: its storage and length
      st = slice_ty(*b.t.inner);
      ptr = "(" + b.c + ")";
      len = std::to_string(b.t.len);
    } else if (b.t.is_int() && is_slice(hint)) {
      st = hint;
      const Ty el = slice_elem_[hint.sname];
      std::string acc = el.b == B::U8 || el.b == B::I8 ? "aether_string" : el.b == B::F32 ? "aether_vec_f32" : "aether_vec_i64";
      pre = "int64_t " + t + " = " + b.c + "; ";
      ptr = "((" + ctype(el) + "*)(intptr_t)" + acc + "_as_ptr(" + t + "))";
      len = "((int64_t)" + acc + "_len(" + t + "))";
    } else {
      fail("AE0530", e->line, e->col, "a range index needs a slice, or a vector / string handle where a slice is expected");
    }
    const std::string lo = e->a[1] ? conv(gen(e->a[1], prim(B::I64)), prim(B::I64)) : "0";
    const std::string hi = e->a.size() > 2 && e->a[2] ? conv(gen(e->a[2], prim(B::I64)), prim(B::I64)) : len;
    return {"({ " + pre + "int64_t lo_" + t + " = " + lo + "; (" + ctype(st) + "){" + ptr + " + lo_" + t + ", (" + hi +
                ") - lo_" + t + "}; })",
            st};
  }

  // Tuples: one C struct per element-type list, fields f_0, f_1, ...
  std::vector<std::string> tuple_names_;
  Ty tuple_ty(const std::vector<Ty>& elems) {
    std::string n = "T";
    for (auto& t : elems) {
      std::string c = ctype(t);
      for (char& ch : c)
        if (!std::isalnum((unsigned char)ch)) ch = '_';
      n += "_" + c;
    }
    if (!structs_.count(n)) {
      StructInfo& in = structs_[n];
      for (size_t i = 0; i < elems.size(); ++i) in.fields.push_back({std::to_string(i), elems[i]});
      tuple_names_.push_back(n);
    }
    return struct_ty(n);
  }

  // Closures without captures become static functions; the value is the
  // function's address (as the reference passes function pointers: an i64).
  std::string lifted_protos_, lifted_defs_;

  // Names a closure body reads that are locals of the enclosing function.
  void free_vars(const EP& e, const std::set<std::string>& params, std::vector<std::string>& out) {
    if (!e) return;
    if (e->k == Expr::Var && !params.count(e->s) && lookup(e->s) &&
        std::find(out.begin(), out.end(), e->s) == out.end())
      out.push_back(e->s);
    if (e->k == Expr::Call && !params.count(e->s) && lookup(e->s) &&
        std::find(out.begin(), out.end(), e->s) == out.end())
      out.push_back(e->s);  // a captured closure called inside
    for (auto& a : e->a) free_vars(a, params, out);
    auto blk = [&](const BP& b) {
      if (!b) return;
      for (auto& st : b->stmts) {
        free_vars(st->e, params, out);
        free_vars(st->e2, params, out);
        free_vars(st->e3, params, out);
        if (st->body) {
          auto tmp = std::make_shared<Expr>();
          tmp->k = Expr::BlockE;
          tmp->blk = st->body;
          free_vars(tmp, params, out);
        }
      }
      free_vars(b->tail, params, out);
    };
    blk(e->blk);
    blk(e->blk2);
  }

  V lift_closure(const EP& e) {
    const Fn& f = *e->closure;
    std::set<std::string> pnames;
    for (auto& prm : f.params) pnames.insert(prm.name);
    std::vector<std::string> caps;
    free_vars(f.body->tail, pnames, caps);
    std::vector<Local> cap_locals;
    for (auto& c : caps) cap_locals.push_back(*lookup(c));
    auto saved_scopes = scopes_;
    const Ty saved_ret = ret_;
    const int saved_indent = indent_;
    scopes_.assign(1, {});
    const std::string name = "aecl_" + std::to_string(++uniq_);
    const std::string env_t = name + "_env";
    std::string params = caps.empty() ? "" : "int64_t env";
    std::vector<Ty> pts;
    for (size_t i = 0; i < caps.size(); ++i)  // captures: read from the environment object
      scopes_.back()[caps[i]] = {cap_locals[i].ty, "(((" + env_t + "*)(intptr_t)env)->c_" + caps[i] + ")"};
    for (auto& prm : f.params) {
      const Ty t = prm.ty ? resolve(*prm.ty) : prim(B::I64);
      pts.push_back(t);
      params += (params.empty() ? "" : ", ") + ctype(t) + " " + bind(prm.name, t);
    }
    Ty rt = f.ret ? resolve(*f.ret) : prim(B::Unknown);
    ret_ = rt;
    indent_ = 1;
    V body;
    try {
      body = gen(f.body->tail, rt);
    } catch (const Diag& d) {
      if (d.code == "AE0510")  // a name of the enclosing function: a capture
        for (auto& sc : saved_scopes)
          for (auto& kv : sc)
            if (std::string(d.what()).find("'" + kv.first + "'") != std::string::npos)
              fail("AE0500", e->line, e->col, "closures that capture `" + kv.first + "` are not compiled; pass it as a parameter");
      throw;
    }
    if (rt.b == B::Unknown) rt = body.t;
    const std::string sig = "static " + ctype(rt) + " " + name + "(" + (params.empty() ? "void" : params) + ")";
    lifted_protos_ += sig + ";\n";
    lifted_defs_ += sig + " {\n  " + (rt.b == B::Void ? body.c + ";\n" : "return " + conv(body, rt) + ";\n") + "}\n\n";
    scopes_ = saved_scopes;
    ret_ = saved_ret;
    indent_ = saved_indent;
    if (caps.empty()) {
      // a plain function; where a `Closure` is expected, a static object
      // [adapter] whose adapter drops the environment argument
      std::string ap = "int64_t env", aa;
      for (size_t i = 0; i < pts.size(); ++i) {
        ap += ", " + ctype(pts[i]) + " p" + std::to_string(i);
        aa += (i ? ", " : "") + std::string("p") + std::to_string(i);
      }
      lifted_protos_ += "static " + ctype(rt) + " " + name + "_adapt(" + ap + ") { (void)env; return " + name + "(" +
                        aa + "); }\nstatic int64_t " + name + "_obj[1] = {(int64_t)(intptr_t)&" + name + "_adapt};\n";
      Ty t = prim(B::I64);
      t.sname = "fn:" + name;
      return {"((int64_t)(intptr_t)&" + name + ")", t};
    }
    std::string decl = "typedef struct { int64_t fn;";
    for (size_t i = 0; i < caps.size(); ++i) decl += " " + ctype(cap_locals[i].ty) + " c_" + caps[i] + ";";
    lifted_protos_ = decl + " } " + env_t + ";\n" + lifted_protos_;
    std::string make = "({ " + env_t + "* ep = (" + env_t + "*)malloc(sizeof(" + env_t + ")); ep->fn = (int64_t)(intptr_t)&" +
                       name + ";";
    for (size_t i = 0; i < caps.size(); ++i) make += " ep->c_" + caps[i] + " = " + cap_locals[i].c + ";";
    make += " (int64_t)(intptr_t)ep; })";
    Ty t = prim(B::I64);
    t.sname = "Closure";
    return {make, t};
  }

  // Trait methods with a default body that an impl does not override are
  // copied into the impl, so each type gets its own `Type__method`.
  void synthesize_defaults() {
    std::map<std::string, const TraitDef*> traits;
    for (auto& t : p_.traits) traits[t.name] = &t;
    for (auto& im : p_.impls) {
      if (im.trait.empty() || !traits.count(im.trait)) continue;
      std::set<std::string> have;
      for (auto& m : im.methods) have.insert(m.name);
      for (auto& m : traits[im.trait]->methods)
        if (m.body && !have.count(m.name)) im.methods.push_back(m);
    }
  }

  // Enums: one with no payload anywhere is an integer (its variant's
  // position); one with payloads is a tagged C struct with a union of the
  // variants' payload tuples.
  struct EnumInfo {
    std::vector<std::pair<std::string, std::vector<Ty>>> variants;
    bool unit_only = true;
  };
  std::map<std::string, EnumInfo> enums_;

  int variant_index(const std::string& en, const std::string& v) const {
    const auto& vs = enums_.at(en).variants;
    for (size_t i = 0; i < vs.size(); ++i)
      if (vs[i].first == v) return (int)i;
    return -1;
  }

  void declare_structs() {
    for (auto& d : p_.structs) {
      if (structs_.count(d.name) || gstructs_.count(d.name))
        fail("AE0501", d.line, d.col, "struct '" + d.name + "' is defined twice");
      if (!d.generics.empty()) gstructs_[d.name] = &d;
      else structs_[d.name];
    }
    for (auto& d : p_.enums) {
      if (structs_.count(d.name) || enums_.count(d.name) || genums_.count(d.name))
        fail("AE0501", d.line, d.col, "type '" + d.name + "' is defined twice");
      if (!d.generics.empty()) {
        genums_[d.name] = &d;
        continue;
      }
      EnumInfo& in = enums_[d.name];
      for (auto& v : d.variants) in.unit_only &= v.second.empty();
    }
    for (auto& d : p_.structs)
      if (d.generics.empty())
        for (auto& f : d.fields) structs_[d.name].fields.push_back({f.name, resolve(*f.ty)});
    for (auto& d : p_.enums)
      if (d.generics.empty())
      for (auto& v : d.variants) {
        std::vector<Ty> ts;
        for (auto& t : v.second) ts.push_back(resolve(*t));
        enums_[d.name].variants.push_back({v.first, ts});
      }
  }

  void declare_method(const std::string& type, const Fn& m) {
    FnSig s;
    s.c = "aef_" + type + "__" + m.name;
    for (size_t i = 0; i < m.params.size(); ++i) {
      const Param& prm = m.params[i];
      if (prm.name == "self" && !prm.ty) {
        if (i != 0) fail("AE0002", m.line, m.col, "`self` must be the first parameter");
        s.self_kind = prm.self_ref ? 2 : 1;
        s.params.push_back(struct_ty(type));
      } else {
        s.params.push_back(resolve(*prm.ty));
      }
    }
    s.ret = m.ret ? resolve(*m.ret) : prim(B::Void);
    const std::string key = type + "::" + m.name;
    if (sigs_.count(key)) fail("AE0501", m.line, m.col, "method '" + key + "' is defined twice");
    sigs_[key] = s;
  }

  // C declarations of every struct, fields before the structs that hold them.
  std::string struct_decls() {
    std::ostringstream o;
    std::vector<std::string> order;
    std::set<std::string> done, visiting;
    std::function<void(const std::string&)> visit = [&](const std::string& n) {
      if (done.count(n)) return;
      if (visiting.count(n)) fail("AE0500", 1, 1, "type '" + n + "' contains itself");
      visiting.insert(n);
      std::vector<const Ty*> parts;
      if (enums_.count(n)) {
        for (auto& v : enums_[n].variants)
          for (auto& t : v.second) parts.push_back(&t);
      } else {
        for (auto& f : structs_[n].fields) parts.push_back(&f.second);
      }
      for (const Ty* t : parts) {
        while (t->b == B::Array) t = t->inner.get();
        if (t->b == B::Struct) visit(t->sname);
      }
      done.insert(n);
      order.push_back(n);
    };
    for (auto& d : p_.structs)
      if (d.generics.empty()) visit(d.name);
    for (size_t i = 0; i < tuple_names_.size(); ++i) visit(tuple_names_[i]);
    for (auto& d : p_.enums)
      if (d.generics.empty() && !enums_[d.name].unit_only) visit(d.name);
    for (auto& n : order) o << "typedef struct aes_" << n << " aes_" << n << ";\n";
    for (auto& n : order) {
      if (enums_.count(n)) {
        o << "struct aes_" << n << " { int64_t tag; union {";
        for (auto& v : enums_[n].variants) {
          if (v.second.empty()) continue;
          o << " struct {";
          for (size_t k = 0; k < v.second.size(); ++k) o << " " << ctype(v.second[k]) << " a" << k << ";";
          o << " } v_" << v.first << ";";
        }
        o << " } u; };\n";
        continue;
      }
      o << "struct aes_" << n << " {";
      if (structs_[n].fields.empty()) o << " char unused_;";
      for (auto& f : structs_[n].fields) {
        if (f.second.b == B::Array) o << " " << ctype(*f.second.inner) << " f_" << f.first << "[" << f.second.len << "];";
        else o << " " << ctype(f.second) << " f_" << f.first << ";";
      }
      o << " };\n";
    }
    return o.str();
  }

  static bool is_place(const EP& e) {
    return e->k == Expr::Var || e->k == Expr::Field || e->k == Expr::Index;
  }

  // A call of a method or associated function `key` ("Type::name"); args[0]
  // is the receiver when the method takes `self`.
  V method_call(const EP& at, const std::string& key, const std::vector<EP>& args, const V* recv) {
    const FnSig& sig = sigs_.at(key);
    const size_t given = args.size() + (recv ? 1 : 0);
    if (given != sig.params.size())
      fail("AE0541", at->line, at->col, "'" + key + "' takes " + std::to_string(sig.params.size()) + " arguments, got " +
                                            std::to_string(given));
    std::string pre, list;
    size_t pi = 0;
    auto self_arg = [&](const V& v, const EP& src) {
      if (sig.self_kind != 2) return conv(v, sig.params[0]);
      if (src && is_place(src)) return "&(" + v.c + ")";
      const std::string tmp = "tmp_" + std::to_string(++uniq_);  // an rvalue receiver: a temporary holds it
      pre += ctype(v.t) + " " + tmp + " = " + v.c + "; ";
      return "&" + tmp;
    };
    if (recv) {
      list = self_arg(*recv, args.empty() ? nullptr : nullptr);
      pi = 1;
    }
    for (size_t i = 0; i < args.size(); ++i, ++pi) {
      V v = gen(args[i], sig.params[pi]);
      std::string c = (pi == 0 && sig.self_kind) ? self_arg(v, args[i]) : conv(v, sig.params[pi]);
      list += (pi ? ", " : "") + c;
    }
    const std::string call = sig.c + "(" + list + ")";
    if (pre.empty()) return {call, sig.ret};
    return {"({ " + pre + call + "; })", sig.ret};
  }

  // The C condition under which pattern `p` matches the value `m` of type
  // `t`; the declarations of its bindings are appended to `binds`.
  std::string pat_test(const Pat& p, const std::string& m, const Ty& t, std::string& binds) {
    switch (p.k) {
      case Pat::Wild: return "1";
      case Pat::Bind:
        if (t.b == B::Array || t.b == B::Tensor)
          fail("AE0500", p.line, p.col, "bindings of arrays or tensors in patterns are not supported");
        binds += ctype(t) + " " + bind(p.s, t) + " = " + m + "; ";
        return "1";
      case Pat::Lit: {
        auto le = std::make_shared<Expr>();
        le->line = p.line;
        le->col = p.col;
        le->s = p.s;
        if (p.s == "true" || p.s == "false") le->k = Expr::BoolL;
        else if (!p.s.empty() && p.s[0] == '\'') {
          le->k = Expr::Char;
          le->s = p.s.substr(1);
        } else if (!p.s.empty() && p.s[0] == '"') {
          fail("AE0500", p.line, p.col, "string patterns are not supported");
        } else {
          le->k = p.s.find_first_of(".eE") != std::string::npos && p.s.find("0x") != 0 ? Expr::Float : Expr::Int;
        }
        V v = gen(le, t);
        return "(" + m + " == " + (p.neg ? "-" : "") + conv(v, t) + ")";
      }
      case Pat::Path:
      case Pat::Tuple: {
        const size_t cc = p.s.rfind("::");
        std::string en = cc == std::string::npos ? "" : p.s.substr(0, cc);
        if (genums_.count(en) && t.b == B::Struct && spec_of_.count(t.sname) && spec_of_[t.sname].first == en)
          en = t.sname;  // Option::Some(x) against an Option<i64> value
        if (!en.empty() && enums_.count(en)) {
          const std::string vn = p.s.substr(cc + 2);
          const int ix = variant_index(en, vn);
          if (ix < 0) fail("AE0510", p.line, p.col, "`" + en + "` has no variant '" + vn + "'");
          if (enums_[en].unit_only) {
            if (p.k == Pat::Tuple) fail("AE0541", p.line, p.col, "variant '" + p.s + "' carries no payload");
            return "(" + m + " == " + std::to_string(ix) + ")";
          }
          if (t.b != B::Struct || t.sname != en)
            fail("AE0520", p.line, p.col, "pattern '" + p.s + "' does not match a value of type " + tyname(t));
          std::string test = "(" + m + ".tag == " + std::to_string(ix);
          const auto& pay = enums_[en].variants[ix].second;
          if (p.k == Pat::Tuple) {
            if (p.subs.size() != pay.size())
              fail("AE0541", p.line, p.col, "'" + p.s + "' carries " + std::to_string(pay.size()) + " values");
            for (size_t k = 0; k < pay.size(); ++k) {
              const std::string sub = pat_test(*p.subs[k], m + ".u.v_" + vn + ".a" + std::to_string(k), pay[k], binds);
              if (sub != "1") test += " && " + sub;
            }
          }
          return test + ")";
        }
        const std::string leaf = cc == std::string::npos ? p.s : p.s.substr(cc + 2);
        if (p.k == Pat::Path && const_src_.count(leaf)) return "(" + m + " == aec_" + leaf + ")";
        fail("AE0510", p.line, p.col, "unknown pattern '" + p.s + "'");
      }
      case Pat::Or: {
        std::string r = "(";
        for (size_t k = 0; k < p.subs.size(); ++k) {
          std::string b;
          r += (k ? " || " : "") + pat_test(*p.subs[k], m, t, b);
          if (!b.empty()) fail("AE0500", p.line, p.col, "bindings inside `|` patterns are not supported");
        }
        return r + ")";
      }
    }
    return "0";
  }

  // `match` (and `if let`) as a GNU statement expression: the scrutinee is
  // evaluated once, arms are tried in order, a guard is evaluated with the
  // arm's bindings in scope.
  V match(const EP& e, const Ty& hint) {
    V sc = gen(e->a[0], prim(B::Unknown));
    const std::string id = std::to_string(++uniq_);
    const std::string m = "m_" + id, r = "r_" + id, d = "d_" + id;
    struct Arm {
      std::string test, binds, guard;
      V body;
    };
    std::vector<Arm> arms;
    Ty rt = (hint.b == B::Unknown || hint.b == B::Void) ? prim(B::Unknown) : hint;
    for (size_t i = 0; i < e->pats.size(); ++i) {
      scopes_.emplace_back();
      Arm a;
      a.test = pat_test(*e->pats[i], m, sc.t, a.binds);
      if (e->guards[i]) a.guard = gen(e->guards[i], prim(B::Bool)).c;
      a.body = gen(e->a[i + 1], rt);
      if (rt.b == B::Unknown && a.body.t.b != B::Void && a.body.t.b != B::Unknown) rt = a.body.t;
      scopes_.pop_back();
      arms.push_back(a);
    }
    const bool value = rt.b != B::Unknown && rt.b != B::Void;
    std::string o = "({ " + ctype(sc.t) + " " + m + " = " + sc.c + "; ";
    if (value) o += ctype(rt) + " " + r + " = " + zero_of(rt) + "; ";
    o += "int " + d + " = 0; ";
    for (auto& a : arms) {
      o += "if (!" + d + " && " + a.test + ") { " + a.binds;
      o += a.guard.empty() ? "{ " : "if (" + a.guard + ") { ";
      if (value && a.body.t.b != B::Void) o += r + " = " + conv(a.body, rt) + "; ";
      else o += a.body.c + "; ";
      o += d + " = 1; } } ";
    }
    if (value) o += r + "; ";
    o += "})";
    (void)m;
    return {o, value ? rt : prim(B::Void)};
  }

  V struct_method(const EP& e, const V& r) {
    const std::string key = r.t.sname + "::" + e->s;
    if (!sigs_.count(key)) specialize_method(r.t.sname, e->s);
    if (!sigs_.count(key)) fail("AE0551", e->line, e->col, "`" + r.t.sname + "` has no method '" + e->s + "'");
    if (sigs_.at(key).self_kind == 0)
      fail("AE0550", e->line, e->col, "'" + key + "' takes no `self`; call it as " + key + "(..)");
    std::vector<EP> args(e->a.begin() + 1, e->a.end());
    if (sigs_.at(key).self_kind == 2 && is_place(e->a[0])) {
      // receiver by address: the place itself
      const FnSig& sig = sigs_.at(key);
      if (args.size() + 1 != sig.params.size())
        fail("AE0541", e->line, e->col, "'" + key + "' takes " + std::to_string(sig.params.size() - 1) + " arguments");
      std::string list = "&(" + r.c + ")";
      for (size_t i = 0; i < args.size(); ++i) list += ", " + conv(gen(args[i], sig.params[i + 1]), sig.params[i + 1]);
      return {sig.c + "(" + list + ")", sig.ret};
    }
    return method_call(e, key, args, &r);
  }

  void declare(const Fn& f) {
    if (!f.generics.empty()) {
      if (gfns_.count(f.name) || sigs_.count(f.name))
        fail("AE0501", f.line, f.col, "function '" + f.name + "' is defined twice");
      gfns_[f.name] = &f;
      return;
    }
    FnSig s;
    for (auto& p : f.params) s.params.push_back(resolve(*p.ty));
    s.ret = f.ret ? resolve(*f.ret) : prim(B::Void);
    s.is_extern = f.is_extern;
    s.c = f.is_extern ? f.name : "aef_" + f.name;
    auto it = sigs_.find(f.name);
    if (it != sigs_.end()) {
      if (f.is_extern && it->second.is_extern) return;  // the same extern declared twice (program + stdlib)
      fail("AE0501", f.line, f.col, "function '" + f.name + "' is defined twice");
    }
    sigs_[f.name] = s;
  }

  // --------------------------------------------------------------- constants
  std::pair<Ty, double> eval_const(const EP& e) {
    switch (e->k) {
      case Expr::Int: return {prim(B::I64), (double)std::stoll(e->s.substr(0, e->s.find('#')))};
      case Expr::Float: return {prim(B::F32), std::stod(e->s.substr(0, e->s.find('#')))};
      case Expr::BoolL: return {prim(B::Bool), e->s == "true" ? 1.0 : 0.0};
      case Expr::Var: {
        auto it = const_val_.find(e->s);
        if (it != const_val_.end()) return it->second;
        auto src = const_src_.find(e->s);
        if (src == const_src_.end()) fail("AE0510", e->line, e->col, "'" + e->s + "' is not a constant");
        const_val_[e->s] = {prim(B::Unknown), 0};  // cycle guard
        auto v = eval_const(src->second->e);
        v.first = resolve(*src->second->ty);
        const_val_[e->s] = v;
        return v;
      }
      case Expr::Unary: {
        auto v = eval_const(e->a[0]);
        if (e->s == "-") v.second = -v.second;
        else v.second = v.second == 0;
        return v;
      }
      case Expr::Cast: {
        auto v = eval_const(e->a[0]);
        v.first = resolve(*e->cast);
        if (v.first.is_int()) v.second = (double)(int64_t)v.second;
        return v;
      }
      case Expr::Binary: {
        auto l = eval_const(e->a[0]), r = eval_const(e->a[1]);
        const bool fl = l.first.is_float() || r.first.is_float();
        const double a = l.second, b = r.second;
        double v = 0;
        const std::string& op = e->s;
        if (op == "+") v = a + b;
        else if (op == "-") v = a - b;
        else if (op == "*") v = a * b;
        else if (op == "/") {
          if (b == 0) fail("AE0511", e->line, e->col, "division by zero in a constant");
          v = fl ? a / b : (double)((int64_t)a / (int64_t)b);
        } else if (op == "%") {
          if (b == 0) fail("AE0511", e->line, e->col, "division by zero in a constant");
          v = (double)((int64_t)a % (int64_t)b);
        } else if (op == "<<") v = (double)((int64_t)a << (int64_t)b);
        else if (op == ">>") v = (double)((int64_t)a >> (int64_t)b);
        else if (op == "&") v = (double)((int64_t)a & (int64_t)b);
        else if (op == "|") v = (double)((int64_t)a | (int64_t)b);
        else if (op == "^") v = (double)((int64_t)a ^ (int64_t)b);
        else fail("AE0510", e->line, e->col, "operator '" + op + "' is not allowed in a constant");
        return {fl ? prim(B::F32) : l.first, v};
      }
      default: fail("AE0510", e->line, e->col, "not a constant expression");
    }
  }

  static std::string lit_of(const std::pair<Ty, double>& v, const Ty& t) {
    char buf[64];
    if (t.is_float()) {
      snprintf(buf, sizeof buf, "%.17g", v.second);
      std::string s = buf;
      if (s.find_first_of(".eEn") == std::string::npos) s += ".0";
      return t.b == B::F32 ? "(float)" + s : s;
    }
    snprintf(buf, sizeof buf, "%lld", (long long)v.second);
    return std::string(buf) + (t.b == B::I64 || t.b == B::U64 ? "LL" : "");
  }

  int64_t const_int(const EP& e) {
    auto v = eval_const(e);
    return (int64_t)v.second;
  }

  Ty resolve(const TyExpr& t) {
    Ty r = resolve_base(t);
    if (t.ref && r.b != B::Tensor && r.b != B::Array && r.b != B::Str && r.b != B::Void && t.name != "slice")
      r.ref = true;  // a slice is a (pointer, length) value already
    return r;
  }

  Ty resolve_base(const TyExpr& t) {
    Ty r;
    if (t.name == "()") return prim(B::Void);
    if (t.name == "slice") return slice_ty(resolve(*t.inner));
    if (t.name == "tuple") {
      std::vector<Ty> el;
      for (auto& x : t.elems) el.push_back(resolve(*x));
      return tuple_ty(el);
    }
    if (t.name == "Tensor") {
      r.b = B::Tensor;
      if (t.elem == "f32") r.elem = B::F32;
      else if (t.elem == "i32") r.elem = B::I32;
      else fail("AE0520", t.line, t.col, "tensor elements must be f32 or i32");
      for (auto& d : t.dims) {
        const int64_t v = const_int(d);
        if (v <= 0) fail("AE0521", t.line, t.col, "tensor dimensions must be positive");
        r.dims.push_back(v);
      }
      return r;
    }
    if (t.name == "[]") {
      r.b = B::Array;
      r.inner = std::make_shared<Ty>(resolve(*t.inner));
      r.len = const_int(t.dims[0]);
      return r;
    }
    if (tsubst_.count(t.name)) return tsubst_.at(t.name);
    if (t.name == "Self" && !self_type_.empty()) return struct_ty(self_type_);
    if (gstructs_.count(t.name) || genums_.count(t.name)) {
      std::vector<Ty> args;
      for (auto& a : t.targs) args.push_back(resolve(*a));
      return gstructs_.count(t.name) ? specialize_struct(t.name, args, t.line, t.col)
                                     : specialize_enum(t.name, args, t.line, t.col);
    }
    if (t.name == "Closure") {  // a closure object: the address of [function, captures...]
      Ty c = prim(B::I64);
      c.sname = "Closure";
      return c;
    }
    if (structs_.count(t.name)) return struct_ty(t.name);
    if (enums_.count(t.name)) return enums_[t.name].unit_only ? prim(B::I64) : struct_ty(t.name);
    auto it = prim_names().find(t.name);
    if (it == prim_names().end()) fail("AE0522", t.line, t.col, "unknown type '" + t.name + "'");
    return prim(it->second);
  }

  // --------------------------------------------------------------- scopes
  Local* lookup(const std::string& n) {
    for (auto it = scopes_.rbegin(); it != scopes_.rend(); ++it) {
      auto f = it->find(n);
      if (f != it->end()) return &f->second;
    }
    return nullptr;
  }
  std::string bind(const std::string& n, const Ty& t) {
    std::string c = n + "_" + std::to_string(++uniq_);
    scopes_.back()[n] = {t, c};
    return c;
  }
  std::string pad() const { return std::string(2 * indent_, ' '); }

  // --------------------------------------------------------------- expressions
  static bool is_lit(const EP& e) {
    return e->k == Expr::Int || e->k == Expr::Float || (e->k == Expr::Unary && e->s == "-" && is_lit(e->a[0]));
  }

  static V deref(const V& v) {
    if (!v.t.ref) return v;
    Ty base = v.t;
    base.ref = false;
    return {"(*" + v.c + ")", base};
  }

  static std::string conv(const V& v, const Ty& to) {
    if (to.b == B::Unknown || to.b == B::Void) return v.c;
    if (to.sname == "Closure" && v.t.sname.rfind("fn:", 0) == 0)  // a plain closure as a closure object
      return "((int64_t)(intptr_t)" + v.t.sname.substr(3) + "_obj)";
    if (v.t.ref && to.ref) return v.c;
    if (v.t.ref && !to.ref) {
      if (to.b == B::I64 || to.b == B::U64)  // an address where a 64-bit integer (a C pointer) is expected
        return "((" + ctype(to) + ")(intptr_t)(" + v.c + "))";
      return conv(deref(v), to);
    }
    if (v.t.b == to.b && to.b != B::Str) return v.c;
    if (v.t.b == B::Str && (to.is_int())) return "((" + ctype(to) + ")(intptr_t)(" + v.c + "))";
    if (v.t.b == B::Tensor && to.is_int()) return "((" + ctype(to) + ")(" + v.c + "))";
    if (v.t.b == B::Array) return v.c;
    return "((" + ctype(to) + ")(" + v.c + "))";
  }

  V gen(const EP& e, const Ty& hint) {
    switch (e->k) {
      case Expr::Int: {
        const size_t h = e->s.find('#');
        Ty t = hint.is_num() ? hint : prim(B::I64);
        if (h != std::string::npos) t = prim(prim_names().at(e->s.substr(h + 1)));
        const std::string num = e->s.substr(0, h);
        if (t.is_float()) return {"((" + ctype(t) + ")" + num + ")", t};
        return {"((" + ctype(t) + ")" + num + (t.b == B::I64 || t.b == B::U64 ? "LL" : "") + ")", t};
      }
      case Expr::Float: {
        const size_t h = e->s.find('#');
        Ty t = hint.b == B::F64 ? hint : prim(B::F32);
        if (h != std::string::npos) t = prim(prim_names().at(e->s.substr(h + 1)));
        std::string num = e->s.substr(0, h);
        if (num.back() == '.') num += "0";
        return {t.b == B::F32 ? num + "f" : num, t};
      }
      case Expr::BoolL: return {e->s == "true" ? "1" : "0", prim(B::Bool)};
      case Expr::Char: return {"((uint8_t)" + e->s + ")", hint.is_int() ? hint : prim(B::U8)};
      case Expr::Str: {
        std::string s = "\"";
        for (unsigned char c : e->s) {
          if (c == '"' || c == '\\') s += '\\', s += (char)c;
          else if (c == '\n') s += "\\n";
          else if (c == '\t') s += "\\t";
          else if (c < 32 || c >= 127) {
            char b[8];
            snprintf(b, sizeof b, "\\%03o", c);
            s += b;
          } else s += (char)c;
        }
        return {s + "\"", prim(B::Str)};
      }
      case Expr::Var: {
        if (Local* l = lookup(e->s)) return {l->c, l->ty};
        if (sigs_.count(e->s) && e->s.find("::") == std::string::npos) {  // a function as a value: its address
          fn_values_[e->s] = true;
          return {"((int64_t)(intptr_t)&" + sigs_[e->s].c + ")", prim(B::I64)};
        }
        const size_t cc = e->s.rfind("::");
        if (cc != std::string::npos && genums_.count(e->s.substr(0, cc))) {
          EP inst = std::make_shared<Expr>(*e);
          inst->s = enum_instance(e->s.substr(0, cc), e->s.substr(cc + 2), {}, hint, e->line, e->col) + "::" +
                    e->s.substr(cc + 2);
          return gen(inst, hint);
        }
        if (cc != std::string::npos && enums_.count(e->s.substr(0, cc))) {
          const std::string en = e->s.substr(0, cc);
          const int ix = variant_index(en, e->s.substr(cc + 2));
          if (ix < 0) fail("AE0510", e->line, e->col, "`" + en + "` has no variant '" + e->s.substr(cc + 2) + "'");
          if (!enums_[en].variants[ix].second.empty())
            fail("AE0541", e->line, e->col, "variant '" + e->s + "' carries a payload");
          if (enums_[en].unit_only) return {"((int64_t)" + std::to_string(ix) + ")", prim(B::I64)};
          return {"((aes_" + en + "){.tag = " + std::to_string(ix) + "})", struct_ty(en)};
        }
        if (const_src_.count(e->s)) {
          auto v = eval_const(e);
          return {"aec_" + e->s, v.first};
        }
        fail("AE0510", e->line, e->col, "unknown name '" + e->s + "'");
      }
      case Expr::Unary: {
        V a = deref(gen(e->a[0], hint));
        if (e->s == "!") return {"(!" + a.c + ")", prim(B::Bool)};  // `!` is a logical not (0 -> 1, else 0)
        return {"(-" + a.c + ")", a.t};
      }
      case Expr::Ref: {
        if (e->a[0]->k == Expr::Index && e->a[0]->s == "..") return slice_range(e->a[0], hint);
        V a = gen(e->a[0], hint);
        if (is_slice(a.t)) return a;
        if (a.t.ref || a.t.b == B::Tensor || a.t.b == B::Array || a.t.b == B::Str || a.t.b == B::Void ||
            a.t.b == B::Unknown)
          return a;  // a tensor's value is its handle; arrays and strings are pointers already
        Ty t = a.t;
        t.ref = true;
        if (is_place(e->a[0])) return {"(&(" + a.c + "))", t};
        return {"(&(" + ctype(a.t) + "){" + a.c + "})", t};  // a temporary's address
      }
      case Expr::Deref: {
        V a = gen(e->a[0], prim(B::Unknown));
        if (a.t.ref) return deref(a);
        if (a.t.b == B::I64 || a.t.b == B::U64) {  // an address held as a 64-bit integer: load through it
          const Ty t = hint.is_num() || hint.b == B::Bool ? hint : prim(B::I64);
          return {"(*(" + ctype(t) + "*)(intptr_t)(" + a.c + "))", t};
        }
        return a;  // `*x` of a by-value binding is the value itself
      }
      case Expr::Cast: {
        Ty to = resolve(*e->cast);
        V a = gen(e->a[0], to);
        return {"((" + ctype(to) + ")(" + a.c + "))", to};
      }
      case Expr::Binary: return binary(e, hint);
      case Expr::Call: return call(e, hint);
      case Expr::Method:
        if (e->s == "into" && e->a.size() == 1 && hint.b == B::Struct && !hint.ref &&
            sigs_.count(hint.sname + "::from"))  // `v.into()` where a struct is expected: Type::from(v)
          return method_call(e, hint.sname + "::from", {e->a[0]}, nullptr);
        return method(e);
      case Expr::Index: {
        if (e->s == "..") return slice_range(e, hint);
        V arr = deref(gen(e->a[0], prim(B::Unknown)));
        if (is_slice(arr.t)) {
          V ix = gen(e->a[1], prim(B::I64));
          return {"(" + arr.c + ").f_ptr[" + ix.c + "]", slice_elem_[arr.t.sname]};
        }
        if (arr.t.b != B::Array) fail("AE0530", e->line, e->col, "only arrays can be indexed");
        V ix = gen(e->a[1], prim(B::I64));
        return {arr.c + "[" + ix.c + "]", *arr.t.inner};
      }
      case Expr::If: {
        V c = gen(e->a[0], prim(B::Bool));
        std::string a = block_expr(*e->blk, hint);
        Ty t = last_block_ty_;
        if (!e->blk2) return {"({ if (" + c.c + ") " + a + "; })", prim(B::Void)};
        std::string b = block_expr(*e->blk2, t.b != B::Void ? t : hint);
        if (t.b == B::Void) t = last_block_ty_;
        if (t.b == B::Void) return {"({ if (" + c.c + ") " + a + "; else " + b + "; })", t};
        return {"((" + c.c + ") ? " + a + " : " + b + ")", t};
      }
      case Expr::BlockE: {
        std::string s = block_expr(*e->blk, hint);
        return {s, last_block_ty_};
      }
      case Expr::StructLit: {
        std::string n = e->s == "Self" && !self_type_.empty() ? self_type_ : e->s;
        if (gstructs_.count(n)) {  // the expected type's instance, else one bound from the field values
          if (hint.b == B::Struct && spec_of_.count(hint.sname) && spec_of_[hint.sname].first == n) {
            n = hint.sname;
          } else {
            const StructDef& d = *gstructs_[n];
            std::map<std::string, Ty> sub;
            for (size_t i = 0; i < e->fields.size(); ++i)
              for (auto& f : d.fields)
                if (f.name == e->fields[i] && f.ty && std::count(d.generics.begin(), d.generics.end(), f.ty->name) &&
                    !sub.count(f.ty->name))
                  sub[f.ty->name] = gen(e->a[i], prim(B::Unknown)).t;
            std::vector<Ty> args;
            for (auto& g : d.generics) args.push_back(sub.count(g) ? sub[g] : prim(B::I64));
            n = specialize_struct(n, args, e->line, e->col).sname;
          }
        }
        auto it = structs_.find(n);
        if (it == structs_.end()) fail("AE0522", e->line, e->col, "unknown struct '" + n + "'");
        std::string r = "((aes_" + n + "){";
        bool first = true;
        for (size_t i = 0; i < e->fields.size(); ++i) {
          const Ty* ft = nullptr;
          for (auto& f : it->second.fields)
            if (f.first == e->fields[i]) ft = &f.second;
          if (!ft) fail("AE0530", e->line, e->col, "`" + n + "` has no field '" + e->fields[i] + "'");
          std::string val;
          if (ft->b == B::Array) {  // an array literal or `[v; n]` fills the field in place
            const EP& x = e->a[i];
            std::vector<std::string> items;
            if (x->k == Expr::ArrayLit) {
              for (auto& el : x->a) items.push_back(conv(gen(el, *ft->inner), *ft->inner));
            } else if (x->k == Expr::ArrayRep) {
              const int64_t n = const_int(x->a[1]);
              if (n > 65536) fail("AE0500", x->line, x->col, "array repeat longer than 65536 in a struct literal");
              const std::string one = conv(gen(x->a[0], *ft->inner), *ft->inner);
              items.assign((size_t)n, one);
            } else {
              fail("AE0500", x->line, x->col, "an array field is initialised from an array literal");
            }
            if ((int64_t)items.size() != ft->len)
              fail("AE0520", x->line, x->col, "array field '" + e->fields[i] + "' has " + std::to_string(ft->len) +
                                                  " elements, the literal " + std::to_string(items.size()));
            val = "{";
            for (size_t k = 0; k < items.size(); ++k) val += (k ? ", " : "") + items[k];
            val += "}";
          } else {
            val = conv(gen(e->a[i], *ft), *ft);
          }
          r += std::string(first ? "" : ", ") + ".f_" + e->fields[i] + " = " + val;
          first = false;
        }
        for (auto& f : it->second.fields) {
          bool given = false;
          for (auto& g : e->fields) given |= g == f.first;
          if (!given && f.second.b != B::Array)
            fail("AE0520", e->line, e->col, "`" + n + "` literal is missing the field '" + f.first + "'");
        }
        if (first) r += "0";
        return {r + "})", struct_ty(n)};
      }
      case Expr::Match: return match(e, hint);
      case Expr::Closure: return lift_closure(e);
      case Expr::TupleLit: {
        std::vector<Ty> want;
        if (hint.b == B::Struct && structs_.count(hint.sname) && !structs_[hint.sname].fields.empty() &&
            structs_[hint.sname].fields[0].first == "0" && structs_[hint.sname].fields.size() == e->a.size())
          for (auto& f : structs_[hint.sname].fields) want.push_back(f.second);
        std::vector<V> vs;
        std::vector<Ty> el;
        for (size_t i = 0; i < e->a.size(); ++i) {
          vs.push_back(gen(e->a[i], want.empty() ? prim(B::Unknown) : want[i]));
          el.push_back(want.empty() ? vs.back().t : want[i]);
        }
        const Ty t = tuple_ty(el);
        std::string r = "((" + ctype(t) + "){";
        for (size_t i = 0; i < vs.size(); ++i) r += (i ? ", " : "") + conv(vs[i], el[i]);
        return {r + "})", t};
      }
      case Expr::Try: {
        V v = gen(e->a[0], prim(B::Unknown));
        if (v.t.b != B::Struct || !enums_.count(v.t.sname))
          fail("AE0520", e->line, e->col, "`?` needs an enum value (Ok / Some and a failure variant)");
        int ok = variant_index(v.t.sname, "Ok");
        if (ok < 0) ok = variant_index(v.t.sname, "Some");
        if (ok < 0 || enums_[v.t.sname].variants[ok].second.size() != 1)
          fail("AE0520", e->line, e->col, "`?` needs an `Ok(..)` or `Some(..)` variant with one value");
        if (ret_.b != B::Struct || ret_.sname != v.t.sname)
          fail("AE0520", e->line, e->col, "`?` returns the failure itself, so the function must return " + tyname(v.t));
        const std::string t = "try_" + std::to_string(++uniq_);
        const std::string vn = enums_[v.t.sname].variants[ok].first;
        return {"({ " + ctype(v.t) + " " + t + " = " + v.c + "; if (" + t + ".tag != " + std::to_string(ok) + ") return " + t +
                    "; " + t + ".u.v_" + vn + ".a0; })",
                enums_[v.t.sname].variants[ok].second[0]};
      }
      case Expr::Field: {
        V b = deref(gen(e->a[0], prim(B::Unknown)));
        if (b.t.b != B::Struct) fail("AE0530", e->line, e->col, "field '" + e->s + "' of a value that is not a struct");
        for (auto& f : structs_[b.t.sname].fields)
          if (f.first == e->s) return {"(" + b.c + ").f_" + e->s, f.second};
        fail("AE0530", e->line, e->col, "`" + b.t.sname + "` has no field '" + e->s + "'");
      }
      case Expr::LoopE: {
        std::ostringstream o;
        o << "({ for (;;) ";
        o << block_stmt(*e->blk);
        o << " })";
        return {o.str(), prim(B::Void)};
      }
      default: fail("AE0500", e->line, e->col, "array literals are only allowed as `let` initialisers");
    }
  }

  V binary(const EP& e, const Ty& hint) {
    const std::string& op = e->s;
    const bool cmp = op == "==" || op == "!=" || op == "<" || op == "<=" || op == ">" || op == ">=";
    const bool logic = op == "&&" || op == "||";
    if (logic) {
      V a = deref(gen(e->a[0], prim(B::Bool))), b = deref(gen(e->a[1], prim(B::Bool)));
      return {"(" + a.c + " " + op + " " + b.c + ")", prim(B::Bool)};
    }
    const bool shift = op == "<<" || op == ">>";
    const Ty h = cmp ? prim(B::Unknown) : hint;
    V a, b;
    if (is_lit(e->a[0]) && !is_lit(e->a[1])) {
      b = deref(gen(e->a[1], h));
      a = deref(gen(e->a[0], shift ? h : b.t));
    } else {
      a = deref(gen(e->a[0], h));
      b = deref(gen(e->a[1], shift ? prim(B::Unknown) : a.t));
    }
    Ty t = a.t;
    if (!shift && a.t.is_num() && b.t.is_num() && a.t.b != b.t.b) {
      // mixed operands: widen to the float / wider side, as the values compare
      if (b.t.is_float() && !a.t.is_float()) t = b.t;
      else if (a.t.is_float() == b.t.is_float() && (int)b.t.b > (int)a.t.b) t = b.t;
    }
    std::string ac = conv(a, t), bc = shift ? b.c : conv(b, t);
    if (op == "%" && t.is_float())
      return {(t.b == B::F32 ? "fmodf(" : "fmod(") + ac + ", " + bc + ")", t};
    if (cmp) return {"(" + ac + " " + op + " " + bc + ")", prim(B::Bool)};
    return {"((" + ctype(t) + ")(" + ac + " " + op + " " + bc + "))", t};
  }

  V call(const EP& e, const Ty& hint) {
    const size_t colon = e->s.rfind("::");
    if (colon != std::string::npos && genums_.count(e->s.substr(0, colon))) {  // a generic enum's variant
      EP inst = std::make_shared<Expr>(*e);
      inst->s = enum_instance(e->s.substr(0, colon), e->s.substr(colon + 2), e->a, hint, e->line, e->col) + "::" +
                e->s.substr(colon + 2);
      return call(inst, hint);
    }
    if (colon != std::string::npos && enums_.count(e->s.substr(0, colon))) {  // a variant with its payload
      const std::string en = e->s.substr(0, colon);
      const int ix = variant_index(en, e->s.substr(colon + 2));
      if (ix < 0) fail("AE0540", e->line, e->col, "`" + en + "` has no variant '" + e->s.substr(colon + 2) + "'");
      const auto& pay = enums_[en].variants[ix].second;
      if (pay.size() != e->a.size())
        fail("AE0541", e->line, e->col, "'" + e->s + "' carries " + std::to_string(pay.size()) + " values, got " +
                                            std::to_string(e->a.size()));
      std::string r = "((aes_" + en + "){.tag = " + std::to_string(ix);
      if (!pay.empty()) {
        r += ", .u.v_" + e->s.substr(colon + 2) + " = {";
        for (size_t k = 0; k < pay.size(); ++k) r += (k ? ", " : "") + conv(gen(e->a[k], pay[k]), pay[k]);
        r += "}";
      }
      return {r + "})", struct_ty(en)};
    }
    if (colon != std::string::npos) {
      std::string type = e->s.substr(0, colon);
      if (type == "Self" && !self_type_.empty()) type = self_type_;
      const std::string key = type + "::" + e->s.substr(colon + 2);
      if (sigs_.count(key)) return method_call(e, key, e->a, nullptr);
    }
    const std::string n = colon == std::string::npos ? e->s : e->s.substr(colon + 2);
    if (structs_.count(n) && !structs_[n].fields.empty() && structs_[n].fields[0].first == "0") {  // Name(a, b)
      const auto& fs = structs_[n].fields;
      if (fs.size() != e->a.size())
        fail("AE0541", e->line, e->col, "'" + n + "' has " + std::to_string(fs.size()) + " fields, got " +
                                            std::to_string(e->a.size()));
      std::string r = "((aes_" + n + "){";
      for (size_t i = 0; i < fs.size(); ++i) r += (i ? ", " : "") + conv(gen(e->a[i], fs[i].second), fs[i].second);
      return {r + "})", struct_ty(n)};
    }
    const size_t us = n.find("__");
    if (us != std::string::npos && us > 0 && !sigs_.count(n)) {  // a flattened `Type__method` name
      const std::string key = n.substr(0, us) + "::" + n.substr(us + 2);
      if (sigs_.count(key)) return method_call(e, key, e->a, nullptr);
    }
    if (Local* fp = lookup(n)) {  // a local or parameter holding a function's address: an indirect call
      if (!fp->ty.is_int()) fail("AE0540", e->line, e->col, "'" + n + "' is not a function");
      std::vector<V> args;
      std::string types, list;
      for (size_t i = 0; i < e->a.size(); ++i) {
        V v = deref(gen(e->a[i], prim(B::Unknown)));
        types += (i ? ", " : "") + ctype(v.t);
        list += (i ? ", " : "") + v.c;
      }
      const Ty rt = hint.is_num() ? hint : prim(B::I64);
      if (fp->ty.sname == "Closure")  // [function, captures...]: the object itself is the first argument
        return {"((" + ctype(rt) + " (*)(int64_t" + (types.empty() ? "" : ", " + types) + "))(intptr_t)(((int64_t*)(intptr_t)(" +
                    fp->c + "))[0]))(" + fp->c + (list.empty() ? "" : ", " + list) + ")",
                rt};
      return {"((" + ctype(rt) + " (*)(" + (types.empty() ? "void" : types) + "))(intptr_t)(" + fp->c + "))(" + list + ")",
              rt};
    }
    auto one_arg = [&](const Ty& t) {
      if (e->a.size() != 1) fail("AE0540", e->line, e->col, n + "() takes one argument");
      return gen(e->a[0], t);
    };
    // casts written as calls
    static const std::map<std::string, B> casts = {{"f32", B::F32}, {"f64", B::F64}, {"i32", B::I32},
                                                   {"i64", B::I64}, {"u8", B::U8},   {"u32", B::U32},
                                                   {"u64", B::U64}, {"i8", B::I8},   {"i16", B::I16}};
    if (!sigs_.count(n) && casts.count(n)) {
      Ty to = prim(casts.at(n));
      V a = one_arg(to);
      return {"((" + ctype(to) + ")(" + a.c + "))", to};
    }
    if (!sigs_.count(n) && (n == "println" || n == "print")) {
      std::string fmt = n == "println" ? "\\n" : "";
      if (e->a.empty()) return {"printf(\"" + fmt + "\")", prim(B::Void)};
      V a = gen(e->a[0], prim(B::Unknown));
      std::string f = a.t.b == B::Str ? "%s" : a.t.is_float() ? "%g" : "%lld";
      std::string val = a.t.b == B::Str ? a.c : a.t.is_float() ? "(double)(" + a.c + ")" : "(long long)(" + a.c + ")";
      return {"(printf(\"" + f + fmt + "\", " + val + "), fflush(stdout))", prim(B::Void)};
    }
    static const std::set<std::string> math = {"sqrt", "sin", "cos", "tan", "exp", "log", "abs", "floor", "ceil",
                                               "tanh", "powf", "pow"};
    if (!sigs_.count(n) && math.count(n)) {
      if (n == "pow" || n == "powf") {
        if (e->a.size() != 2) fail("AE0540", e->line, e->col, n + "() takes two arguments");
        V a = gen(e->a[0], hint.is_float() ? hint : prim(B::F32));
        V b = gen(e->a[1], a.t);
        return {(a.t.b == B::F64 ? "pow(" : "powf(") + a.c + ", " + conv(b, a.t) + ")", a.t};
      }
      V a = one_arg(hint.is_float() ? hint : prim(B::F32));
      if (a.t.is_int()) {
        if (n == "abs") return {"((" + a.c + ") < 0 ? -(" + a.c + ") : (" + a.c + "))", a.t};
        a = {"((float)(" + a.c + "))", prim(B::F32)};
      }
      const std::string cn = n == "abs" ? "fabs" : n;
      return {(a.t.b == B::F32 ? cn + "f(" : cn + "(") + a.c + ")", a.t};
    }
    if (gfns_.count(n)) return generic_call(e, n, hint);
    if (n == "yield_now" && !sigs_.count(n) && e->a.empty()) return {"((void)0)", prim(B::Void)};  // one task: nothing to yield to
    if (n == "slice_from_raw" && !sigs_.count(n)) {  // (pointer as i64, length) -> the expected slice type
      if (!is_slice(hint)) fail("AE0520", e->line, e->col, "slice_from_raw needs an expected `&[T]` type");
      if (e->a.size() != 2) fail("AE0541", e->line, e->col, "slice_from_raw takes a pointer and a length");
      const Ty el = slice_elem_[hint.sname];
      return {"((" + ctype(hint) + "){(" + ctype(el) + "*)(intptr_t)(" + conv(gen(e->a[0], prim(B::I64)), prim(B::I64)) +
                  "), " + conv(gen(e->a[1], prim(B::I64)), prim(B::I64)) + "})",
              hint};
    }
    auto it = sigs_.find(n);
    if (it == sigs_.end()) fail("AE0540", e->line, e->col, "unknown function '" + n + "'");
    const FnSig& s = it->second;
    if (s.params.size() != e->a.size())
      fail("AE0541", e->line, e->col, "'" + n + "' takes " + std::to_string(s.params.size()) + " arguments, got " +
                                           std::to_string(e->a.size()));
    std::string args;
    for (size_t i = 0; i < e->a.size(); ++i) {
      V v = gen(e->a[i], s.params[i]);
      if (s.params[i].ref && !v.t.ref) {
        Ty base = s.params[i];
        base.ref = false;
        if (v.t.b == B::I64 || v.t.b == B::U64)  // an address held as an integer: the pointer itself
          v = V{"((" + ctype(s.params[i]) + ")(intptr_t)(" + v.c + "))", s.params[i]};
        else  // a value where a reference is declared: its address
          v = is_place(e->a[i]) ? V{"(&(" + v.c + "))", s.params[i]}
                                : V{"(&(" + ctype(base) + "){" + conv(v, base) + "})", s.params[i]};
      }
      if (v.t.b == B::Tensor && !s.params[i].is_int() && s.params[i].b != B::Tensor)
        fail("AE0520", e->a[i]->line, e->a[i]->col, "a tensor passed where " + tyname(s.params[i]) + " is expected");
      args += (i ? ", " : "") + conv(v, s.params[i]);
    }
    return {s.c + "(" + args + ")", s.ret};
  }

  V method(const EP& e) {
    V r = gen(e->a[0], prim(B::Unknown));
    if (is_slice(deref(r).t) && e->s == "len" && e->a.size() == 1) return {"(" + deref(r).c + ").f_len", prim(B::I64)};
    if (r.t.b == B::Struct && r.t.ref) {  // through a reference: `&self` methods take the pointer itself
      const std::string key = r.t.sname + "::" + e->s;
      if (sigs_.count(key) && sigs_.at(key).self_kind == 2) {
        const FnSig& sig = sigs_.at(key);
        if (e->a.size() != sig.params.size())
          fail("AE0541", e->line, e->col, "'" + key + "' takes " + std::to_string(sig.params.size() - 1) + " arguments");
        std::string list = r.c;
        for (size_t i = 1; i < e->a.size(); ++i) list += ", " + conv(gen(e->a[i], sig.params[i]), sig.params[i]);
        return {sig.c + "(" + list + ")", sig.ret};
      }
      r = deref(r);
    }
    if (r.t.b == B::Struct) return struct_method(e, r);
    if (r.t.b != B::Tensor)
      fail("AE0550", e->line, e->col, "method '" + e->s + "' needs a Tensor receiver, not " + tyname(r.t));
    auto it = method_rules().find(e->s);
    if (it == method_rules().end()) fail("AE0551", e->line, e->col, "unknown tensor method '" + e->s + "'");
    const MethodRule& rule = it->second;
    std::vector<V> args;
    std::vector<Ty> shapes;
    for (size_t i = 1; i < e->a.size(); ++i) {
      V v = gen(e->a[i], prim(B::Unknown));
      args.push_back(v);
      shapes.push_back(v.t);
    }
    const std::vector<int64_t>& s = r.t.dims;
    auto arg_dims = [&](size_t k) -> const std::vector<int64_t>& {
      if (k >= shapes.size() || shapes[k].b != B::Tensor)
        fail("AE0552", e->line, e->col, e->s + ": argument " + std::to_string(k + 1) + " must be a Tensor");
      return shapes[k].dims;
    };
    auto need2 = [&](const std::vector<int64_t>& d, const char* what) {
      if (d.size() != 2) fail("AE0553", e->line, e->col, e->s + ": " + what + " must be 2-dimensional");
    };
    std::vector<int64_t> extra;
    switch (rule.recipe) {
      case MKN_MATMUL: {
        const auto& w = arg_dims(0);
        need2(w, "the weight");
        if (s.size() == 2) extra = {s[0], s[1], w[1]};
        else if (s.size() == 3) extra = {s[0] * s[1], s[2], w[1]};
        else fail("AE0553", e->line, e->col, "matmul: the receiver must be 2- or 3-dimensional");
        if (extra[1] != w[0]) fail("AE0554", e->line, e->col, "matmul: inner dimensions differ");
        break;
      }
      case MKN_2D: {
        const auto& w = arg_dims(0);
        need2(s, "the receiver");
        need2(w, "the weight");
        extra = {s[0], s[1], w[1]};
        break;
      }
      case MKN_NT: {
        const auto& k = arg_dims(0);
        need2(s, "the receiver");
        need2(k, "the right operand");
        extra = {s[0], s[1], k[0]};
        break;
      }
      case MKN_TN: {
        const auto& b = arg_dims(0);
        need2(s, "the receiver");
        need2(b, "the right operand");
        extra = {s[1], s[0], b[1]};
        break;
      }
      case MKN_BWD_RHS: {
        const auto& dy = arg_dims(0);
        need2(s, "the receiver");
        need2(dy, "dy");
        extra = {s[0], s[1], dy[1]};
        break;
      }
      case MKN_BWD_LHS: {
        const auto& w = arg_dims(0);
        need2(s, "the receiver");
        need2(w, "the weight");
        extra = {s[0], w[0], s[1]};
        break;
      }
      case ROWS_COLS:
        need2(s, "the receiver");
        extra = {s[0], s[1]};
        break;
      case NUMEL: extra = {r.t.numel()}; break;
    }
    // the runtime signature types the user's arguments and the appended shape ints
    auto sit = sigs_.find(rule.fn);
    std::string call = std::string(rule.fn) + "(" + r.c;
    Ty ret = prim(B::I32);
    if (sit != sigs_.end()) {
      const FnSig& fs = sit->second;
      ret = fs.ret;
      if (fs.params.size() != 1 + args.size() + extra.size())
        fail("AE0541", e->line, e->col, "tensor method '" + e->s + "' lowers to " + rule.fn + ", which takes " +
                                            std::to_string(fs.params.size()) + " arguments; the call supplies " +
                                            std::to_string(1 + args.size() + extra.size()));
      for (size_t i = 0; i < args.size(); ++i) {
        V v = args[i];
        if (is_lit(e->a[i + 1])) v = gen(e->a[i + 1], fs.params[i + 1]);
        call += ", " + conv(v, fs.params[i + 1]);
      }
    } else {
      used_undeclared_.insert(rule.fn);
      for (auto& v : args) call += ", " + v.c;
    }
    for (int64_t x : extra) call += ", " + std::to_string(x);
    return {call + ")", ret};
  }

  std::set<std::string> used_undeclared_;
  std::map<std::string, bool> fn_values_;  // functions whose address was taken
  Ty last_block_ty_;

  // A block as a GNU statement expression; its type lands in last_block_ty_.
  std::string block_expr(const Block& b, const Ty& hint) {
    scopes_.emplace_back();
    std::ostringstream o;
    o << "({ ";
    ++indent_;
    for (auto& s : b.stmts) o << stmt(*s) << " ";
    Ty t = prim(B::Void);
    if (b.tail) {
      V v = gen(b.tail, hint);
      t = v.t;
      o << v.c << "; ";
    }
    --indent_;
    o << "})";
    scopes_.pop_back();
    last_block_ty_ = t;
    return o.str();
  }

  std::string block_stmt(const Block& b) {
    scopes_.emplace_back();
    std::ostringstream o;
    o << "{\n";
    ++indent_;
    for (auto& s : b.stmts) o << pad() << stmt(*s) << "\n";
    if (b.tail) {
      V v = gen(b.tail, prim(B::Unknown));
      o << pad() << v.c << ";\n";
    }
    --indent_;
    o << pad() << "}";
    scopes_.pop_back();
    return o.str();
  }

  // --------------------------------------------------------------- statements
  std::string stmt(const Stmt& s) {
    switch (s.k) {
      case Stmt::Let: return let(s);
      case Stmt::ExprS: {
        V v = gen(s.e, prim(B::Unknown));
        return v.c + ";";
      }
      case Stmt::Assign: {
        V lhs = gen(s.e, prim(B::Unknown));
        if (s.e->k != Expr::Var && s.e->k != Expr::Index && s.e->k != Expr::Field && s.e->k != Expr::Deref)
          fail("AE0560", s.line, s.col, "can only assign to a variable, a field or an array element");
        if (lhs.t.b == B::Tensor) fail("AE0561", s.line, s.col, "tensor bindings cannot be reassigned");
        V rhs = gen(s.e2, lhs.t);
        if (s.op == "%=" && lhs.t.is_float())
          return lhs.c + " = " + (lhs.t.b == B::F32 ? "fmodf(" : "fmod(") + lhs.c + ", " + conv(rhs, lhs.t) + ");";
        return lhs.c + " " + s.op + " " + conv(rhs, lhs.t) + ";";
      }
      case Stmt::While: {
        if (s.pat) {  // while let: match once per iteration, leave on the first miss
          V sc = gen(s.e, prim(B::Unknown));
          const std::string m = "m_" + std::to_string(++uniq_);
          scopes_.emplace_back();
          std::string binds;
          const std::string test = pat_test(*s.pat, m, sc.t, binds);
          const std::string body = block_stmt(*s.body);
          scopes_.pop_back();
          return "for (;;) { " + ctype(sc.t) + " " + m + " = " + sc.c + "; if (!" + test + ") break; " + binds + body +
                 " }";
        }
        V c = gen(s.e, prim(B::Bool));
        return "while (" + c.c + ") " + block_stmt(*s.body);
      }
      case Stmt::Loop: return "for (;;) " + block_stmt(*s.body);
      case Stmt::For: {
        if (!s.e2) {  // for x in slice
          V c = deref(gen(s.e, prim(B::Unknown)));
          if (!is_slice(c.t)) fail("AE0500", s.line, s.col, "for loops iterate over ranges a..b, a..=b or slices");
          const Ty el = slice_elem_[c.t.sname];
          const std::string sv = "it_" + std::to_string(++uniq_), k = "k_" + std::to_string(uniq_);
          scopes_.emplace_back();
          const std::string x = bind(s.name, el);
          std::string r = "{ " + ctype(c.t) + " " + sv + " = " + c.c + "; for (int64_t " + k + " = 0; " + k + " < " + sv +
                          ".f_len; ++" + k + ") { " + ctype(el) + " " + x + " = " + sv + ".f_ptr[" + k + "]; " +
                          block_stmt(*s.body) + " } }";
          scopes_.pop_back();
          return r;
        }
        V a = gen(s.e, prim(B::Unknown));
        V b = gen(s.e2, a.t);
        Ty t = a.t.is_int() ? a.t : prim(B::I64);
        scopes_.emplace_back();
        const std::string iv = bind(s.name, t), lim = "lim_" + std::to_string(++uniq_);
        std::string r = "for (" + ctype(t) + " " + iv + " = " + conv(a, t) + ", " + lim + " = " + conv(b, t) + "; " + iv +
                        (s.inclusive ? " <= " : " < ") + lim + "; ++" + iv + ") " + block_stmt(*s.body);
        scopes_.pop_back();
        return r;
      }
      case Stmt::Return: {
        if (!s.e) return ret_.b == B::Void ? "return;" : "return " + zero_of(ret_) + ";";
        V v = gen(s.e, ret_);
        return "return " + conv(v, ret_) + ";";
      }
      case Stmt::Break: return "break;";
      case Stmt::Continue: return "continue;";
    }
    return "";
  }

  std::string let(const Stmt& s) {
    if (!s.names.empty()) {  // let (a, b, _) = e: a temporary, then one binding per element
      V v = gen(s.e, s.ty ? resolve(*s.ty) : prim(B::Unknown));
      if (v.t.b != B::Struct || structs_[v.t.sname].fields.size() != s.names.size() ||
          structs_[v.t.sname].fields[0].first != "0")
        fail("AE0520", s.line, s.col, "destructuring needs a tuple of " + std::to_string(s.names.size()) + " elements");
      const std::string tmp = "tup_" + std::to_string(++uniq_);
      std::string r = ctype(v.t) + " " + tmp + " = " + v.c + ";";
      const auto fs = structs_[v.t.sname].fields;
      for (size_t i = 0; i < s.names.size(); ++i) {
        if (s.names[i] == "_") continue;
        const std::string c = bind(s.names[i], fs[i].second);
        r += " " + ctype(fs[i].second) + " " + c + " = " + tmp + ".f_" + std::to_string(i) + ";";
      }
      return r;
    }
    if (s.name == "_" && s.e && !s.ty) {  // `let _ = e;` evaluates e and drops the value
      V v = gen(s.e, prim(B::Unknown));
      return "(void)(" + v.c + ");";
    }
    if (s.ty && s.ty->name == "Tensor") {
      if (s.e) fail("AE0570", s.line, s.col, "a Tensor binding is allocated by its declaration and takes no initialiser");
      Ty t = resolve(*s.ty);
      const std::string c = bind(s.name, t);
      const bool f = t.elem == B::F32;
      return std::string("int64_t ") + c + " __attribute__((cleanup(" + (f ? "ae_drop_f32" : "ae_drop_i32") + "))) = " +
             (f ? "aether_dev_alloc_f32(" : "aether_dev_alloc_i32(") + std::to_string(t.numel()) + ");";
    }
    Ty t = s.ty ? resolve(*s.ty) : prim(B::Unknown);
    if (t.b == B::Array && !s.e) {  // zero-filled
      const std::string c = bind(s.name, t);
      return ctype(*t.inner) + " " + c + "[" + std::to_string(t.len) + "] = {0};";
    }
    if (t.b == B::Array || (s.e && (s.e->k == Expr::ArrayLit || s.e->k == Expr::ArrayRep))) {
      Ty el = t.b == B::Array ? *t.inner : prim(B::Unknown);
      std::vector<std::string> vals;
      std::string rep_val, rep_len;
      int64_t len = 0;
      if (s.e->k == Expr::ArrayLit) {
        for (auto& x : s.e->a) {
          V v = gen(x, el);
          if (el.b == B::Unknown) el = v.t;
          vals.push_back(conv(v, el));
        }
        len = (int64_t)vals.size();
      } else if (s.e->k == Expr::ArrayRep) {
        V v = gen(s.e->a[0], el);
        if (el.b == B::Unknown) el = v.t;
        rep_val = conv(v, el);
        len = const_int(s.e->a[1]);
      } else {
        fail("AE0571", s.line, s.col, "arrays are initialised from an array literal");
      }
      if (t.b == B::Array && t.len != len) fail("AE0520", s.line, s.col, "array length does not match its type");
      Ty at;
      at.b = B::Array;
      at.inner = std::make_shared<Ty>(el);
      at.len = len;
      const std::string c = bind(s.name, at);
      std::string r = ctype(el) + " " + c + "[" + std::to_string(len) + "]";
      if (!vals.empty()) {
        r += " = {";
        for (size_t i = 0; i < vals.size(); ++i) r += (i ? ", " : "") + vals[i];
        return r + "};";
      }
      const std::string k = "i_" + std::to_string(++uniq_);
      return r + "; for (int64_t " + k + " = 0; " + k + " < " + std::to_string(len) + "; ++" + k + ") " + c + "[" + k +
             "] = " + rep_val + ";";
    }
    std::string init;
    if (s.e) {
      V v = gen(s.e, t);
      if (t.b == B::Unknown) t = v.t;
      if (v.t.b == B::Tensor && t.b == B::Tensor)
        fail("AE0572", s.line, s.col, "a Tensor binding cannot be copied (use the original binding)");
      if (t.b == B::Void) fail("AE0573", s.line, s.col, "binding has no value");
      init = conv(v, t);
    } else {
      if (t.b == B::Unknown) fail("AE0574", s.line, s.col, "a binding without initialiser needs a type");
      init = t.b == B::Struct ? "{0}" : "0";
    }
    const std::string c = bind(s.name, t);
    return ctype(t) + " " + c + " = " + init + ";";
  }

  static std::string zero_of(const Ty& t) { return t.b == B::Struct ? "(" + ctype(t) + "){0}" : "0"; }

  std::string fn_def(const Fn& f, const std::string& key) {
    const FnSig& sig = sigs_[key];
    ret_ = sig.ret;
    scopes_.clear();
    scopes_.emplace_back();
    std::string params;
    for (size_t i = 0; i < f.params.size(); ++i) {
      if (i == 0 && sig.self_kind == 2) {  // `&self`: a pointer; `self` names what it points at
        const std::string c = "self_" + std::to_string(++uniq_);
        scopes_.back()["self"] = {sig.params[0], "(*" + c + ")"};
        params += ctype(sig.params[0]) + "* " + c;
        continue;
      }
      const std::string c = bind(f.params[i].name, sig.params[i]);
      params += (i ? ", " : "") + ctype(sig.params[i]) + " " + c;
    }
    if (params.empty()) params = "void";
    std::ostringstream o;
    o << "static " << ctype(sig.ret) << " " << sig.c << "(" << params << ") {\n";
    indent_ = 1;
    const Block& b = *f.body;
    for (auto& s : b.stmts) o << pad() << stmt(*s) << "\n";
    if (b.tail) {
      V v = gen(b.tail, ret_);
      if (ret_.b == B::Void) o << pad() << v.c << ";\n";
      else o << pad() << "return " << conv(v, ret_) << ";\n";
    } else if (ret_.b != B::Void) {
      o << pad() << "return " << zero_of(ret_) << ";\n";
    }
    o << "}\n\n";
    return o.str();
  }
};

bool read_file(const std::string& path, std::string& out) {
  std::ifstream f(path, std::ios::binary);
  if (!f) return false;
  std::ostringstream s;
  s << f.rdbuf();
  out = s.str();
  return true;
}

void Gen::resolve_uses(Program& p, const std::string& stdlib, const std::string& srcdir,
                       std::set<std::string>& seen) {
  std::vector<std::string> uses = p.uses;
  for (const std::string& u : uses) {
    const std::string leaf = u.substr(u.rfind(':') == std::string::npos ? 0 : u.rfind(':') + 1);
    if (seen.count(leaf)) continue;
    seen.insert(leaf);
    std::string text;
    if (!read_file(stdlib + "/" + leaf + ".aether", text) && !read_file(srcdir + "/" + leaf + ".aether", text) &&
        !read_file(srcdir + "/_" + leaf + ".aether", text))
      fail("AE0003", 1, 1, "cannot find module '" + u + "'");
    Parser ps(lex(text));
    Program m = ps.program();
    resolve_uses(m, stdlib, srcdir, seen);
    for (auto& f : m.fns) p.fns.push_back(f);
    for (auto& d : m.structs) p.structs.push_back(d);
    for (auto& d : m.traits) p.traits.push_back(d);
    for (auto& d : m.impls) p.impls.push_back(d);
    for (auto& c : m.consts) {
      bool dup = false;
      for (auto& e : p.consts) dup |= e.name == c.name;
      if (!dup) p.consts.push_back(c);
    }
  }
}

// ============================================================================ front-end checks
// The checks the reference's `aetherc --check` runs before code generation
// (compiler/src/main.rs:330-540): trait completeness (mir/traits_drive.rs:
// AE0210 a required method missing from an impl, AE0211 an impl of an
// undeclared trait, AE0212 a supertrait not implemented for the type), scalar
// type conflicts (mir/infer.rs: AE0220 a `let` annotation, AE0221 a call
// argument, AE0222 a returned value, AE0224 a reassignment -- only where both
// sides are concrete scalars of different classes: integer, float, bool) and
// borrows (mir/lifetimes.rs: AE0200 a `&mut` while the place is borrowed,
// AE0201 a `&` while it is mutably borrowed). The codes and what they flag are
// the reference's; the passes are written here over this compiler's AST. A
// `let`-bound borrow lives from its `let` to the last statement that names
// its binding; a borrow inside an expression lives for its statement.

// Traits of the language's standard prelude: an impl of one needs no declaration here.
bool prelude_trait(const std::string& n) {
  static const std::set<std::string> names = {"From", "Into", "Clone", "Copy", "Debug", "Default", "Display",
                                              "PartialEq", "Eq", "PartialOrd", "Ord", "Hash", "Send", "Sync",
                                              "Drop", "Iterator", "Add", "Sub", "Mul", "Div", "Neg", "Deref",
                                              "AsRef", "ToString"};
  return names.count(n) != 0;
}

void check_traits(const Program& p) {
  std::map<std::string, const TraitDef*> traits;
  for (auto& t : p.traits) traits[t.name] = &t;
  std::set<std::pair<std::string, std::string>> impls;  // (trait, type)
  for (auto& im : p.impls)
    if (!im.trait.empty()) impls.insert({im.trait, im.type});
  for (auto& im : p.impls) {
    if (im.trait.empty()) continue;
    auto it = traits.find(im.trait);
    if (it == traits.end() && prelude_trait(im.trait)) continue;
    if (it == traits.end())
      fail("AE0211", im.line, im.col, "`impl " + im.trait + " for " + im.type + "`: no trait `" + im.trait + "` is declared");
    std::set<std::string> have;
    for (auto& m : im.methods) have.insert(m.name);
    for (auto& m : it->second->methods)
      if (!m.body && !have.count(m.name))
        fail("AE0210", im.line, im.col, "`impl " + im.trait + " for " + im.type + "` is missing the required method `" +
                                            m.name + "`");
    for (auto& sup : it->second->supers)
      if (!impls.count({sup, im.type}))
        fail("AE0212", im.line, im.col, "`" + im.type + "` implements `" + im.trait + "` but not its supertrait `" +
                                            sup + "`");
  }
}

// ---------------------------------------------------------------- scalar classes
enum class SC { Unknown, Int, Float, Bool, Str, Unit };

const char* sc_name(SC c) {
  switch (c) {
    case SC::Int: return "an integer";
    case SC::Float: return "a float";
    case SC::Bool: return "a bool";
    case SC::Str: return "a string";
    case SC::Unit: return "()";
    default: return "unknown";
  }
}
bool sc_scalar(SC c) { return c == SC::Int || c == SC::Float || c == SC::Bool; }
bool sc_clash(SC a, SC b) { return sc_scalar(a) && sc_scalar(b) && a != b; }

SC sc_of(const std::shared_ptr<TyExpr>& t) {
  if (!t) return SC::Unknown;
  static const std::set<std::string> ints = {"i8", "i16", "i32", "i64", "i128", "isize",
                                             "u8", "u16", "u32", "u64", "u128", "usize"};
  if (ints.count(t->name)) return SC::Int;
  if (t->name == "f32" || t->name == "f64") return SC::Float;
  if (t->name == "bool") return SC::Bool;
  if (t->name == "str") return SC::Str;
  if (t->name == "()") return SC::Unit;
  return SC::Unknown;
}

class TypeCheck {
 public:
  explicit TypeCheck(const Program& p) : p_(p) {
    for (auto& f : p.fns) sigs_[f.name] = &f;
  }
  void run() {
    for (auto& f : p_.fns) {
      if (!f.body) continue;
      check_fn(f);
    }
    for (auto& im : p_.impls)
      for (auto& f : im.methods)
        if (f.body) check_fn(f);
  }

 private:
  const Program& p_;
  std::map<std::string, const Fn*> sigs_;
  std::vector<std::map<std::string, SC>> env_;
  const Fn* fn_ = nullptr;

  void check_fn(const Fn& f) {
    fn_ = &f;
    env_.assign(1, {});
    for (auto& prm : f.params) env_.back()[prm.name] = sc_of(prm.ty);
    const SC body = block(*f.body);
    const SC want = f.ret ? sc_of(f.ret) : SC::Unit;
    if (f.body->tail && sc_clash(body, want))
      fail("AE0222", f.body->tail->line, f.body->tail->col,
           "`" + f.name + "` returns " + sc_name(want) + ", but its body yields " + sc_name(body));
  }
  SC lookup(const std::string& n) const {
    for (auto it = env_.rbegin(); it != env_.rend(); ++it) {
      auto f = it->find(n);
      if (f != it->end()) return f->second;
    }
    return SC::Unknown;
  }
  SC block(const Block& b) {
    env_.emplace_back();
    for (auto& st : b.stmts) stmt(*st);
    const SC t = b.tail ? expr(b.tail) : SC::Unit;
    env_.pop_back();
    return t;
  }
  void stmt(const Stmt& st) {
    switch (st.k) {
      case Stmt::Let: {
        const SC v = st.e ? expr(st.e) : SC::Unknown;
        const SC ann = sc_of(st.ty);
        if (st.ty && st.e && sc_clash(ann, v))
          fail("AE0220", st.line, st.col, "type mismatch in `let " + st.name + "`: annotation is " + sc_name(ann) +
                                              ", but the value is " + sc_name(v));
        env_.back()[st.name] = st.ty ? ann : v;
        break;
      }
      case Stmt::Assign: {
        const SC v = expr(st.e2);
        if (st.op == "=" && st.e->k == Expr::Var) {
          const SC have = lookup(st.e->s);
          if (sc_clash(have, v))
            fail("AE0224", st.line, st.col, "cannot assign " + std::string(sc_name(v)) + " to `" + st.e->s +
                                                "`, which is " + sc_name(have));
        } else {
          expr(st.e);
        }
        break;
      }
      case Stmt::Return:
        if (st.e) {
          const SC v = expr(st.e);
          const SC want = fn_->ret ? sc_of(fn_->ret) : SC::Unit;
          if (sc_clash(v, want))
            fail("AE0222", st.line, st.col, "returned value is " + std::string(sc_name(v)) + ", but `" + fn_->name +
                                                "` returns " + sc_name(want));
        }
        break;
      case Stmt::For:
        expr(st.e);
        expr(st.e2);
        env_.emplace_back();
        env_.back()[st.name] = SC::Int;
        block(*st.body);
        env_.pop_back();
        break;
      case Stmt::While:
        expr(st.e);
        block(*st.body);
        break;
      case Stmt::Loop:
        if (st.body) block(*st.body);
        break;
      case Stmt::ExprS:
        expr(st.e);
        break;
      default: break;
    }
  }
  SC expr(const EP& e) {
    if (!e) return SC::Unknown;
    switch (e->k) {
      case Expr::Int: return SC::Int;
      case Expr::Float: return SC::Float;
      case Expr::BoolL: return SC::Bool;
      case Expr::Str: return SC::Str;
      case Expr::Char: return SC::Unknown;
      case Expr::Var: return lookup(e->s);
      case Expr::Unary: {
        const SC t = expr(e->a[0]);
        return e->s == "!" ? (t == SC::Int ? SC::Int : SC::Bool) : t;
      }
      case Expr::Binary: {
        const SC l = expr(e->a[0]);
        const SC r = expr(e->a[1]);
        static const std::set<std::string> rel = {"==", "!=", "<", "<=", ">", ">=", "&&", "||"};
        if (rel.count(e->s)) return SC::Bool;
        return sc_scalar(l) ? l : r;
      }
      case Expr::Call: {
        std::vector<SC> args;
        for (auto& a : e->a) args.push_back(expr(a));
        auto it = sigs_.find(e->s);
        if (it == sigs_.end()) return SC::Unknown;
        const Fn& f = *it->second;
        for (size_t i = 0; i < args.size() && i < f.params.size(); ++i) {
          const SC want = sc_of(f.params[i].ty);
          if (sc_clash(args[i], want))
            fail("AE0221", e->a[i]->line, e->a[i]->col,
                 "argument " + std::to_string(i + 1) + " to `" + f.name + "` is " + sc_name(args[i]) +
                     ", but the parameter is " + sc_name(want));
        }
        return f.ret ? sc_of(f.ret) : SC::Unit;
      }
      case Expr::Cast:
        expr(e->a[0]);
        return sc_of(e->cast);
      case Expr::If: {
        expr(e->a[0]);
        const SC a = block(*e->blk);
        const SC b = e->blk2 ? block(*e->blk2) : SC::Unit;
        return a == b ? a : SC::Unknown;
      }
      case Expr::BlockE: return e->blk ? block(*e->blk) : SC::Unit;
      case Expr::LoopE:
        block(*e->blk);
        return SC::Unknown;
      default:
        for (auto& a : e->a) expr(a);
        if (e->blk) block(*e->blk);
        return SC::Unknown;
    }
  }
};

// ---------------------------------------------------------------- borrows
class BorrowCheck {
 public:
  void run(const Program& p) {
    for (auto& f : p.fns)
      if (f.body) fn(*f.body);
    for (auto& im : p.impls)
      for (auto& f : im.methods)
        if (f.body) fn(*f.body);
  }

 private:
  struct Borrow {
    std::string place, binding;  // binding empty: lives for its statement only
    bool mut;
    int from, until;
  };
  std::vector<Borrow> live_;
  std::map<std::string, int> last_use_;
  int pos_ = 0;

  // Pass 1: the statement index of each name's last mention.
  void uses_block(const Block& b) {
    for (auto& s : b.stmts) uses_stmt(*s);
    if (b.tail) {
      ++pos_;
      uses_expr(b.tail);
    }
  }
  void uses_stmt(const Stmt& s) {
    ++pos_;
    uses_expr(s.e);
    uses_expr(s.e2);
    uses_expr(s.e3);
    if (s.body) uses_block(*s.body);
  }
  void uses_expr(const EP& e) {
    if (!e) return;
    if (e->k == Expr::Var) last_use_[e->s] = pos_;
    for (auto& a : e->a) uses_expr(a);
    if (e->blk) uses_block(*e->blk);
    if (e->blk2) uses_block(*e->blk2);
  }

  // Pass 2: borrows in statement order.
  void fn(const Block& body) {
    last_use_.clear();
    pos_ = 0;
    uses_block(body);
    live_.clear();
    pos_ = 0;
    walk_block(body);
  }
  void walk_block(const Block& b) {
    for (auto& s : b.stmts) walk_stmt(*s);
    if (b.tail) {
      ++pos_;
      drop_dead();
      walk_expr(b.tail, "");
    }
  }
  void drop_dead() {
    std::vector<Borrow> keep;
    for (auto& b : live_)
      if (b.until >= pos_) keep.push_back(b);
    live_.swap(keep);
  }
  void walk_stmt(const Stmt& s) {
    ++pos_;
    drop_dead();
    if (s.k == Stmt::Let && s.e && s.e->k == Expr::Ref) {
      walk_expr(s.e, s.name);
    } else {
      walk_expr(s.e, "");
      walk_expr(s.e2, "");
      walk_expr(s.e3, "");
    }
    if (s.body) walk_block(*s.body);
  }
  void walk_expr(const EP& e, const std::string& binding) {
    if (!e) return;
    if (e->k == Expr::Ref && !e->a.empty() && e->a[0]->k == Expr::Var) {
      const std::string& place = e->a[0]->s;
      for (auto& b : live_) {
        if (b.place != place) continue;
        if (e->mut)
          fail("AE0200", e->line, e->col, "cannot borrow `" + place + "` as mutable: already borrowed");
        if (b.mut)
          fail("AE0201", e->line, e->col, "cannot borrow `" + place + "` as shared: already mutably borrowed");
      }
      int until = pos_;
      if (!binding.empty()) {
        auto it = last_use_.find(binding);
        until = it == last_use_.end() ? pos_ : std::max(pos_, it->second);
      }
      live_.push_back({place, binding, e->mut, pos_, until});
      return;
    }
    for (auto& a : e->a) walk_expr(a, "");
    if (e->blk) walk_block(*e->blk);
    if (e->blk2) walk_block(*e->blk2);
  }
};

// The code generator takes no structs, traits, impls or field accesses, and
// reads `*x` of a by-value binding as `x`.
void strip_deref(EP& e) {
  if (!e) return;
  for (auto& a : e->a) strip_deref(a);
  auto blk = [](const BP& b) {
    if (!b) return;
    for (auto& st : b->stmts) {
      strip_deref(st->e);
      strip_deref(st->e2);
      strip_deref(st->e3);
      if (st->body) {
        EP tmp = std::make_shared<Expr>();
        tmp->k = Expr::BlockE;
        tmp->blk = st->body;
        strip_deref(tmp);
      }
    }
    strip_deref(b->tail);
  };
  blk(e->blk);
  blk(e->blk2);
}
void prepare_codegen(Program& p) {
  auto strip = [](const BP& body) {
    if (!body) return;
    EP tmp = std::make_shared<Expr>();
    tmp->k = Expr::BlockE;
    tmp->blk = body;
    strip_deref(tmp);
  };
  for (auto& f : p.fns) strip(f.body);
  for (auto& im : p.impls)
    for (auto& m : im.methods) strip(m.body);
  for (auto& t : p.traits)
    for (auto& m : t.methods) strip(m.body);
}

// ============================================================================ AST dump
void dump_expr(std::ostream& o, const EP& e);
void dump_block(std::ostream& o, const Block& b) {
  o << "(block";
  for (auto& s : b.stmts) {
    o << " (" << (s->k == Stmt::Let ? "let " + s->name : s->k == Stmt::Assign ? "assign" + s->op
                : s->k == Stmt::While ? "while" : s->k == Stmt::For ? "for " + s->name
                : s->k == Stmt::Return ? "return" : s->k == Stmt::Break ? "break" : s->k == Stmt::Continue ? "continue"
                : "expr");
    if (s->e) o << " ", dump_expr(o, s->e);
    if (s->e2) o << " ", dump_expr(o, s->e2);
    if (s->body) o << " ", dump_block(o, *s->body);
    o << ")";
  }
  if (b.tail) o << " (tail ", dump_expr(o, b.tail), o << ")";
  o << ")";
}
void dump_expr(std::ostream& o, const EP& e) {
  static const char* names[] = {"int", "float", "bool", "str", "char", "var", "unary", "binary", "call", "method",
                                "cast", "ref", "if", "block", "index", "array", "array-repeat", "loop"};
  o << "(" << names[e->k];
  if (!e->s.empty()) o << " " << e->s;
  for (auto& a : e->a) o << " ", dump_expr(o, a);
  if (e->blk) o << " ", dump_block(o, *e->blk);
  if (e->blk2) o << " ", dump_block(o, *e->blk2);
  o << ")";
}

}  // namespace ae

// ============================================================================ driver
namespace {
std::string dirname_of(const std::string& p) {
  const size_t s = p.rfind('/');
  return s == std::string::npos ? "." : p.substr(0, s);
}
std::string self_dir() {
  char buf[4096];
  const ssize_t n = readlink("/proc/self/exe", buf, sizeof buf - 1);
  if (n <= 0) return ".";
  buf[n] = 0;
  return dirname_of(buf);
}
std::string json_escape(const std::string& s) {
  std::string r;
  for (char c : s) {
    if (c == '"' || c == '\\') r += '\\', r += c;
    else if (c == '\n') r += "\\n";
    else r += c;
  }
  return r;
}
void usage() {
  std::puts(
      "aetherc - compiler for Aether programs against the aether_b200 C-ABI runtime\n\n"
      "USAGE:\n"
      "  aetherc <input.aether> [-o <out>] [--emit=bin|c|ast|tokens] [--check] [--json-errors]\n"
      "          [--no-fuse] [--O0|--O1|--O2] [--stdlib <dir>] [--libdir <dir>] [--cc <compiler>]\n\n"
      "--emit=bin     lower to C, compile with the C compiler and link libaether_rt / libaether_dev (default)\n"
      "--emit=c       write the generated C\n"
      "--emit=ast     write the parsed program as an S-expression\n"
      "--check        parse, resolve `use`, check traits, scalar types and borrows; no code\n"
      "--no-fuse      keep `matmul` + in-place `gelu` as two runtime calls\n"
      "--test         main runs every #[test] fn (0 = pass), prints PASS / FAIL and a summary\n"
      "The reference's other emit kinds (mir, llvm-ir, asm, asm-bin, aether-bin, pe-bin) are not produced.");
}
}  // namespace

int main(int argc, char** argv) {
  std::string input, output, emit = "bin", stdlib, libdir, cc = "cc", opt = "-O2";
  bool check = false, json = false, fuse = true, test_mode = false;
  for (int i = 1; i < argc; ++i) {
    const std::string a = argv[i];
    if (a == "-o" && i + 1 < argc) output = argv[++i];
    else if (a.rfind("--emit=", 0) == 0) emit = a.substr(7);
    else if (a == "--check") check = true;
    else if (a == "--json-errors") json = true;
    else if (a == "--no-fuse") fuse = false;
    else if (a == "--test") test_mode = true;
    else if (a == "--O0") opt = "-O0";
    else if (a == "--O1") opt = "-O1";
    else if (a == "--O2") opt = "-O2";
    else if (a == "--stdlib" && i + 1 < argc) stdlib = argv[++i];
    else if (a == "--libdir" && i + 1 < argc) libdir = argv[++i];
    else if (a == "--cc" && i + 1 < argc) cc = argv[++i];
    else if (a == "-h" || a == "--help") {
      usage();
      return 0;
    } else if (a == "--version") {
      std::puts("aetherc (aether_b200) 0.2");
      return 0;
    } else if (!a.empty() && a[0] != '-') input = a;
    else {
      std::fprintf(stderr, "aetherc: unknown argument %s\n", a.c_str());
      return 2;
    }
  }
  if (input.empty()) {
    usage();
    return 2;
  }
  const std::string here = self_dir();
  if (stdlib.empty()) stdlib = here + "/../aetherc_stdlib";
  if (libdir.empty()) libdir = here + "/..";
  static const std::set<std::string> kinds = {"bin", "c", "ast", "tokens"};
  if (!kinds.count(emit)) {
    std::fprintf(stderr, "aetherc: --emit=%s is not produced by this compiler (bin, c, ast, tokens)\n", emit.c_str());
    return 2;
  }
  std::string src;
  if (!ae::read_file(input, src)) {
    if (json)
      std::fprintf(stderr, "{\"code\":\"AE0100\",\"file\":\"%s\",\"line\":0,\"col\":0,\"message\":\"cannot read input\"}\n",
                   json_escape(input).c_str());
    else
      std::fprintf(stderr, "%s: error[AE0100]: cannot read input\n", input.c_str());
    return 2;
  }
  try {
    std::vector<ae::Tok> toks = ae::lex(src);
    if (emit == "tokens") {
      for (auto& t : toks) std::printf("%d:%d %s\n", t.line, t.col, t.s.c_str());
      return 0;
    }
    ae::Parser ps(toks);
    ae::Program prog = ps.program();
    if (emit == "ast") {
      std::ostringstream o;
      for (auto& f : prog.fns) {
        o << "(fn " << f.name;
        if (f.body) o << " ", ae::dump_block(o, *f.body);
        o << ")\n";
      }
      if (output.empty()) std::fputs(o.str().c_str(), stdout);
      else std::ofstream(output) << o.str();
      return 0;
    }
    std::set<std::string> seen;
    ae::Gen::resolve_uses(prog, stdlib, dirname_of(input), seen);
    // The reference's order: traits always; scalar types under --check; borrows on both paths.
    ae::check_traits(prog);
    if (check) {
      ae::TypeCheck(prog).run();
      ae::BorrowCheck().run(prog);
      return 0;
    }
    ae::BorrowCheck().run(prog);
    ae::prepare_codegen(prog);
    int fused = 0;
    if (fuse)
      for (auto& f : prog.fns)
        if (f.body) fused += ae::fuse_block(*f.body);
    ae::Gen g(prog, stdlib, dirname_of(input));
    g.test_mode_ = test_mode;
    const std::string c = g.run();
    if (emit == "c") {
      if (output.empty()) std::fputs(c.c_str(), stdout);
      else std::ofstream(output) << c;
      if (fused) std::fprintf(stderr, "aetherc: fused %d matmul+gelu pair(s)\n", fused);
      return 0;
    }
    if (output.empty()) {
      output = input;
      const size_t dot = output.rfind(".aether");
      if (dot != std::string::npos) output = output.substr(0, dot);
    }
    const std::string tmp = output + ".aetherc.c";
    std::ofstream(tmp) << c;
    const std::string cmd = cc + " " + opt + " -w -o '" + output + "' '" + tmp + "' -L'" + libdir +
                            "' -Wl,--no-as-needed -laether_rt -Wl,--as-needed -laether_dev -Wl,--no-as-needed -lm "
                            "-Wl,-rpath,'" + libdir + "'";
    const int rc = std::system(cmd.c_str());
    std::remove(tmp.c_str());
    if (rc != 0) {
      std::fprintf(stderr, "aetherc: C compiler failed (%s)\n", cmd.c_str());
      return 1;
    }
    return 0;
  } catch (const ae::Diag& d) {
    if (json)
      std::fprintf(stderr, "{\"code\":\"%s\",\"file\":\"%s\",\"line\":%d,\"col\":%d,\"message\":\"%s\"}\n",
                   d.code.c_str(), json_escape(input).c_str(), d.line, d.col, json_escape(d.what()).c_str());
    else
      std::fprintf(stderr, "%s:%d:%d: error[%s]: %s\n", input.c_str(), d.line, d.col, d.code.c_str(), d.what());
    return 1;
  }
}
