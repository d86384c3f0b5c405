// .prk verified-IR container: reader, verifier, writer and structural matcher.
//
// The container layout is the reference's format 1 (compiler/ir/artifact.cpp:10-20,
// :248-313): magic "PARALYN\0", u32 format 1, u32 numerical policy 1, then kernels
// of (name, parameters, statement tree), all integers little-endian u32 and strings
// length-prefixed. The layout and limits must be identical for the bytes to be
// interchangeable; the code here is written for this engine. The verifier applies
// the rules of the reference IR (compiler/ir/ir.cpp:45-267).
//
// There is no run-time compiler in this backend. A loaded kernel must be
// structurally identical (up to commuting the operands of + and *) to a kernel
// this library implements natively for sm_100a; anything else is PR_UNSUPPORTED.
#include "module.hpp"
#include <algorithm>
#include <cctype>
#include <cerrno>
#include <cmath>
#include <cstdlib>
#include <functional>
#include <map>
#include <set>

namespace pb {
namespace {

constexpr unsigned char prk_magic[8] = {'P', 'A', 'R', 'A', 'L', 'Y', 'N', 0};
constexpr uint32_t prk_format = 1, prk_policy = 1;
constexpr uint32_t max_kernels = 64, max_parameters = 256, max_nodes = 100000, max_depth = 64,
                   max_string = 4096, max_statements = 65536;

[[noreturn]] void bad(const std::string &why) {
  throw std::runtime_error("invalid module artifact: " + why);
}
[[noreturn]] void invalid(const std::string &why) { throw std::runtime_error("invalid IR: " + why); }

IrType ir_type(uint32_t code) {
  if (code > 3)
    bad("unknown scalar type");
  return static_cast<IrType>(code);
}
ExprKind expr_kind(uint32_t code) {
  if (code > 5)
    bad("unknown expression kind");
  return static_cast<ExprKind>(code);
}

class Reader {
  const unsigned char *p_;
  size_t size_, at_ = 0;
  uint32_t nodes_ = 0;

public:
  Reader(const void *data, size_t size) : p_(static_cast<const unsigned char *>(data)), size_(size) {
    if (!data || size > prk_max_bytes)
      bad("null input or artifact exceeds byte limit");
  }
  size_t position() const { return at_; }
  size_t size() const { return size_; }
  void node(unsigned depth) {
    if (depth > max_depth)
      bad("nesting depth exceeds limit");
    if (++nodes_ > max_nodes)
      bad("node count exceeds limit");
  }
  void need(size_t n) const {
    if (n > size_ - at_)
      bad("truncated input");
  }
  unsigned char byte() {
    need(1);
    return p_[at_++];
  }
  uint32_t u32() {
    need(4);
    uint32_t v = uint32_t(p_[at_]) | uint32_t(p_[at_ + 1]) << 8 | uint32_t(p_[at_ + 2]) << 16 |
                 uint32_t(p_[at_ + 3]) << 24;
    at_ += 4;
    return v;
  }
  uint32_t count(uint32_t limit, size_t minimum_bytes) {
    const uint32_t v = u32();
    if (v > limit)
      bad("collection count exceeds limit");
    if (minimum_bytes && v > (size_ - at_) / minimum_bytes)
      bad("truncated collection");
    return v;
  }
  std::string string() {
    const uint32_t n = count(max_string, 1);
    std::string s(reinterpret_cast<const char *>(p_ + at_), n);
    at_ += n;
    if (s.find('\0') != std::string::npos)
      bad("embedded NUL in string");
    return s;
  }
  Expr expression(unsigned depth) {
    node(depth);
    Expr e;
    e.kind = expr_kind(u32());
    e.type = ir_type(u32());
    e.text = string();
    e.line = u32();
    e.column = u32();
    const uint32_t n = count(2, 24);
    for (uint32_t i = 0; i < n; ++i)
      e.operands.push_back(expression(depth + 1));
    return e;
  }
  std::vector<Stmt> body(unsigned depth) {
    const uint32_t n = count(max_statements, 4);
    std::vector<Stmt> out;
    for (uint32_t i = 0; i < n; ++i) {
      node(depth);
      Stmt s;
      switch (u32()) {
      case 0:
        s.kind = StmtKind::Let;
        s.name = string();
        s.type = ir_type(u32());
        s.expression = expression(depth + 1);
        break;
      case 1:
        s.kind = StmtKind::Store;
        s.type = ir_type(u32());
        s.expression = expression(depth + 1);
        s.target = expression(depth + 1);
        break;
      case 2:
        s.kind = StmtKind::If;
        s.expression = expression(depth + 1);
        s.body = body(depth + 1);
        break;
      default:
        bad("unknown statement kind");
      }
      out.push_back(std::move(s));
    }
    return out;
  }
};

class Writer {
public:
  std::vector<unsigned char> bytes;
  void u32(uint32_t v) {
    for (int shift = 0; shift < 32; shift += 8)
      bytes.push_back(static_cast<unsigned char>(v >> shift));
  }
  void string(const std::string &s) {
    if (s.size() > max_string || s.find('\0') != std::string::npos)
      bad("string exceeds limit or contains NUL");
    u32(uint32_t(s.size()));
    bytes.insert(bytes.end(), s.begin(), s.end());
  }
  void expression(const Expr &e) {
    u32(uint32_t(e.kind));
    u32(uint32_t(e.type));
    string(e.text);
    u32(e.line);
    u32(e.column);
    u32(uint32_t(e.operands.size()));
    for (const auto &o : e.operands)
      expression(o);
  }
  void body(const std::vector<Stmt> &statements) {
    u32(uint32_t(statements.size()));
    for (const auto &s : statements) {
      u32(uint32_t(s.kind));
      if (s.kind == StmtKind::Let) {
        string(s.name);
        u32(uint32_t(s.type));
        expression(s.expression);
      } else if (s.kind == StmtKind::Store) {
        u32(uint32_t(s.type));
        expression(s.expression);
        expression(s.target);
      } else {
        expression(s.expression);
        body(s.body);
      }
    }
  }
};

// ---- verifier ----
bool is_identifier(const std::string &n) {
  if (n.empty() || !(std::isalpha(static_cast<unsigned char>(n[0])) || n[0] == '_'))
    return false;
  return std::all_of(n.begin(), n.end(),
                     [](unsigned char c) { return std::isalnum(c) || c == '_'; });
}
bool integral(IrType t) { return t == IrType::I32 || t == IrType::U32; }

struct Symbol {
  IrType type;
  bool buffer, read_only;
};
using Symbols = std::map<std::string, Symbol>;

void check_literal(const Expr &e) {
  if (e.text.empty())
    invalid("empty literal");
  for (unsigned char c : e.text)
    if (std::isspace(c) || std::iscntrl(c))
      invalid("whitespace/control character in literal");
  if (e.type == IrType::Bool) {
    if (e.text != "0" && e.text != "1")
      invalid("invalid predicate literal");
    return;
  }
  char *end = nullptr;
  errno = 0;
  if (e.type == IrType::F32) {
    const float v = std::strtof(e.text.c_str(), &end);
    if (!std::isfinite(v) || errno == ERANGE)
      invalid("non-finite or out-of-range float literal");
  } else if (e.type == IrType::I32) {
    const long long v = std::strtoll(e.text.c_str(), &end, 10);
    if (errno || v < INT32_MIN || v > INT32_MAX)
      invalid("out-of-range i32 literal");
  } else {
    const unsigned long long v = std::strtoull(e.text.c_str(), &end, 10);
    if (errno || e.text[0] == '-' || v > UINT32_MAX)
      invalid("out-of-range u32 literal");
  }
  if (!end || *end)
    invalid("invalid literal spelling");
}

void check_expr(const Expr &e, const Symbols &symbols, bool as_buffer = false) {
  auto arity = [&](size_t n) {
    if (e.operands.size() != n)
      invalid("incorrect expression arity");
  };
  switch (e.kind) {
  case ExprKind::Literal:
    arity(0);
    check_literal(e);
    return;
  case ExprKind::Ref: {
    arity(0);
    const auto it = symbols.find(e.text);
    if (it == symbols.end())
      invalid("undefined symbol " + e.text);
    if (it->second.type != e.type)
      invalid("reference type mismatch for " + e.text);
    if (it->second.buffer != as_buffer)
      invalid(as_buffer ? "load/store requires buffer" : "buffer used as scalar " + e.text);
    return;
  }
  case ExprKind::Builtin: {
    arity(0);
    const auto dot = e.text.find('.');
    if (e.type != IrType::U32 || dot == std::string::npos)
      invalid("builtin type/name");
    const auto base = e.text.substr(0, dot), dim = e.text.substr(dot + 1);
    if ((base != "threadIdx" && base != "blockIdx" && base != "blockDim" && base != "gridDim") ||
        (dim != "x" && dim != "y" && dim != "z"))
      invalid("unknown index builtin");
    return;
  }
  case ExprKind::Cast:
    arity(1);
    check_expr(e.operands[0], symbols);
    if (e.type != e.operands[0].type && !(integral(e.type) && integral(e.operands[0].type)))
      invalid("unsupported scalar conversion");
    return;
  case ExprKind::Binary: {
    arity(2);
    for (const auto &o : e.operands)
      check_expr(o, symbols);
    const IrType t = e.operands[0].type;
    if (t != e.operands[1].type || t == IrType::Bool)
      invalid("binary operand type mismatch");
    if (e.text == "<") {
      if (e.type != IrType::Bool)
        invalid("comparison result must be predicate");
    } else if (e.text == "+" || e.text == "*") {
      if (e.type != t)
        invalid("arithmetic result type mismatch");
    } else
      invalid("unsupported operator " + e.text);
    return;
  }
  case ExprKind::Load:
    arity(2);
    if (e.operands[0].kind != ExprKind::Ref)
      invalid("buffer base must be parameter reference");
    check_expr(e.operands[0], symbols, true);
    check_expr(e.operands[1], symbols);
    if (!integral(e.operands[1].type) || e.type != e.operands[0].type)
      invalid("invalid load type");
    return;
  }
  invalid("unknown expression kind");
}

void check_body(const std::vector<Stmt> &body, Symbols symbols) {
  for (const auto &s : body) {
    switch (s.kind) {
    case StmtKind::Let:
      if (!s.body.empty())
        invalid("local declaration cannot contain statements");
      if (!is_identifier(s.name) || symbols.count(s.name))
        invalid("duplicate/invalid local " + s.name);
      check_expr(s.expression, symbols);
      if (s.type != s.expression.type || s.type == IrType::Bool)
        invalid("invalid local type");
      symbols.emplace(s.name, Symbol{s.type, false, false});
      break;
    case StmtKind::Store:
      if (!s.body.empty())
        invalid("store cannot contain statements");
      if (s.target.kind != ExprKind::Load)
        invalid("store target is not indexed buffer");
      check_expr(s.target, symbols);
      check_expr(s.expression, symbols);
      if (s.target.type != s.expression.type || s.type != s.target.type)
        invalid("store type mismatch");
      if (symbols.at(s.target.operands[0].text).read_only)
        invalid("store to read-only buffer");
      break;
    case StmtKind::If:
      check_expr(s.expression, symbols);
      if (s.expression.type != IrType::Bool)
        invalid("if condition must be predicate");
      check_body(s.body, symbols);
      break;
    default:
      invalid("unknown statement kind");
    }
  }
}

// ---- canonical form for structural matching ----
const char *type_tag(IrType t) {
  switch (t) {
  case IrType::I32: return "i32";
  case IrType::U32: return "u32";
  case IrType::F32: return "f32";
  case IrType::Bool: return "bool";
  }
  return "?";
}

struct Canon {
  std::map<std::string, std::string> names; // parameter/local name -> positional tag
  unsigned locals = 0;
  std::string expr(const Expr &e) {
    switch (e.kind) {
    case ExprKind::Literal:
      return std::string("lit:") + type_tag(e.type) + ":" + e.text;
    case ExprKind::Ref:
      return names.at(e.text);
    case ExprKind::Builtin:
      return e.text;
    case ExprKind::Cast:
      return std::string("cast<") + type_tag(e.type) + ">(" + expr(e.operands[0]) + ")";
    case ExprKind::Binary: {
      std::string a = expr(e.operands[0]), b = expr(e.operands[1]);
      if (e.text != "<" && b < a)
        std::swap(a, b); // + and * commute exactly in IEEE and integer arithmetic
      return "(" + a + e.text + b + "):" + type_tag(e.type);
    }
    case ExprKind::Load:
      return names.at(e.operands[0].text) + "[" + expr(e.operands[1]) + "]";
    }
    return "?";
  }
  std::string body(const std::vector<Stmt> &statements) {
    std::string out;
    for (const auto &s : statements) {
      if (s.kind == StmtKind::Let) {
        const std::string tag = "l" + std::to_string(locals++);
        out += "let " + tag + ":" + type_tag(s.type) + "=" + expr(s.expression) + ";";
        names[s.name] = tag;
      } else if (s.kind == StmtKind::Store) {
        out += "store " + expr(s.target) + "=" + expr(s.expression) + ";";
      } else {
        auto saved = names;
        out += "if(" + expr(s.expression) + "){" + body(s.body) + "}";
        names = saved;
      }
    }
    return out;
  }
};

std::string canonical(const IrKernel &k) {
  Canon c;
  std::string sig;
  for (size_t i = 0; i < k.params.size(); ++i) {
    const auto &p = k.params[i];
    c.names[p.name] = "p" + std::to_string(i);
    sig += std::string(p.buffer ? "buf<" : "") + type_tag(p.type) + (p.buffer ? ">" : "") + ",";
  }
  return "(" + sig + ")" + c.body(k.body);
}

// ---- the IR of the kernels implemented natively ----
Expr ref(const std::string &n, IrType t) { return Expr{ExprKind::Ref, t, n, {}, 0, 0}; }
Expr builtin(const std::string &n) { return Expr{ExprKind::Builtin, IrType::U32, n, {}, 0, 0}; }
Expr bin(const std::string &op, IrType t, Expr a, Expr b) {
  return Expr{ExprKind::Binary, t, op, {std::move(a), std::move(b)}, 0, 0};
}
Expr load(const std::string &buffer, const Expr &index) {
  return Expr{ExprKind::Load, IrType::F32, "", {ref(buffer, IrType::F32), index}, 0, 0};
}

// out[i] = value(i) guarded by i < n, with i = blockIdx.x * blockDim.x + threadIdx.x.
IrKernel elementwise(const std::string &name, IrType index, std::vector<IrParam> params,
                     const std::string &out, const std::function<Expr(const Expr &)> &value) {
  Expr global = bin("+", IrType::U32, bin("*", IrType::U32, builtin("blockIdx.x"), builtin("blockDim.x")),
                    builtin("threadIdx.x"));
  if (index == IrType::I32)
    global = Expr{ExprKind::Cast, IrType::I32, "", {global}, 0, 0};
  Stmt let;
  let.kind = StmtKind::Let;
  let.name = "i";
  let.type = index;
  let.expression = global;
  const Expr i = ref("i", index);
  Stmt store;
  store.kind = StmtKind::Store;
  store.type = IrType::F32;
  store.expression = value(i);
  store.target = load(out, i);
  Stmt guard;
  guard.kind = StmtKind::If;
  guard.type = IrType::Bool;
  guard.expression = bin("<", IrType::Bool, i, ref("n", index));
  guard.body = {store};
  return IrKernel{name, std::move(params), {let, guard}};
}

struct Known {
  std::string builtin;
  IrKernel kernel;
};

const std::vector<Known> &known_kernels() {
  static const std::vector<Known> value = [] {
    std::vector<Known> v;
    for (IrType index : {IrType::U32, IrType::I32}) {
      const std::string suffix = index == IrType::U32 ? "u32" : "i32";
      std::vector<IrParam> ab = {{"a", IrType::F32, true, true},
                                 {"b", IrType::F32, true, true},
                                 {"out", IrType::F32, true, false},
                                 {"n", index, false, false}};
      v.push_back({"ir.add." + suffix, elementwise("add", index, ab, "out", [](const Expr &i) {
                     return bin("+", IrType::F32, load("a", i), load("b", i));
                   })});
      auto affine = ab;
      affine.push_back({"scale", IrType::F32, false, false});
      v.push_back({"ir.affine." + suffix, elementwise("affine", index, affine, "out", [](const Expr &i) {
                     return bin("+", IrType::F32,
                                bin("*", IrType::F32, load("a", i), ref("scale", IrType::F32)),
                                load("b", i));
                   })});
    }
    // out[i] = a[i] * scale + bias: the affine map with a scalar addend.
    std::vector<IrParam> scalar = {{"a", IrType::F32, true, true},
                                   {"out", IrType::F32, true, false},
                                   {"n", IrType::U32, false, false},
                                   {"scale", IrType::F32, false, false},
                                   {"bias", IrType::F32, false, false}};
    v.push_back({"ir.affine_scalar.u32",
                 elementwise("affine_scalar", IrType::U32, scalar, "out", [](const Expr &i) {
                   return bin("+", IrType::F32,
                              bin("*", IrType::F32, load("a", i), ref("scale", IrType::F32)),
                              ref("bias", IrType::F32));
                 })});
    return v;
  }();
  return value;
}

void collect_reads(const Expr &e, std::set<std::string> &names) {
  if (e.kind == ExprKind::Load)
    names.insert(e.operands[0].text);
  for (const auto &o : e.operands)
    collect_reads(o, names);
}
void collect(const std::vector<Stmt> &body, std::set<std::string> &read, std::set<std::string> &write) {
  for (const auto &s : body) {
    collect_reads(s.expression, read);
    if (s.kind == StmtKind::Store) {
      write.insert(s.target.operands[0].text);
      collect_reads(s.target.operands[1], read);
    }
    collect(s.body, read, write);
  }
}

} // namespace

void verify_ir(const IrKernel &k) {
  if (!is_identifier(k.name))
    invalid("invalid kernel name");
  Symbols symbols;
  for (const auto &p : k.params) {
    if (!is_identifier(p.name) || symbols.count(p.name))
      invalid("duplicate/invalid parameter");
    if (p.type == IrType::Bool)
      invalid("predicate kernel arguments unsupported");
    symbols.emplace(p.name, Symbol{p.type, p.buffer, p.read_only});
  }
  check_body(k.body, symbols);
}

std::vector<IrKernel> parse_prk(const void *data, size_t size) {
  Reader r(data, size);
  for (unsigned char c : prk_magic)
    if (r.byte() != c)
      bad("incorrect magic");
  if (r.u32() != prk_format)
    bad("unsupported format version");
  if (r.u32() != prk_policy)
    bad("unsupported numerical policy");
  const uint32_t count = r.count(max_kernels, 12);
  if (!count)
    bad("module contains no kernels");
  std::vector<IrKernel> kernels;
  std::set<std::string> names;
  for (uint32_t i = 0; i < count; ++i) {
    IrKernel k;
    k.name = r.string();
    if (!names.insert(k.name).second)
      bad("duplicate entrypoint " + k.name);
    const uint32_t params = r.count(max_parameters, 12);
    for (uint32_t p = 0; p < params; ++p) {
      IrParam param;
      param.name = r.string();
      param.type = ir_type(r.u32());
      const uint32_t flags = r.u32();
      if (flags > 3)
        bad("unknown parameter flags");
      param.buffer = flags & 1;
      param.read_only = flags & 2;
      k.params.push_back(param);
    }
    k.body = r.body(0);
    verify_ir(k);
    kernels.push_back(std::move(k));
  }
  if (r.position() != r.size())
    bad("trailing data");
  return kernels;
}

std::vector<unsigned char> write_prk(const std::vector<IrKernel> &kernels) {
  if (kernels.empty())
    bad("module contains no kernels");
  Writer w;
  w.bytes.assign(std::begin(prk_magic), std::end(prk_magic));
  w.u32(prk_format);
  w.u32(prk_policy);
  w.u32(uint32_t(kernels.size()));
  for (const auto &k : kernels) {
    verify_ir(k);
    w.string(k.name);
    w.u32(uint32_t(k.params.size()));
    for (const auto &p : k.params) {
      w.string(p.name);
      w.u32(uint32_t(p.type));
      w.u32((p.buffer ? 1u : 0u) | (p.read_only ? 2u : 0u));
    }
    w.body(k.body);
  }
  return w.bytes;
}

std::string match_ir(const IrKernel &kernel) {
  const std::string form = canonical(kernel);
  for (const auto &known : known_kernels())
    if (canonical(known.kernel) == form)
      return known.builtin;
  return "";
}

pr_access ir_access(const IrKernel &kernel, size_t index) {
  std::set<std::string> read, write;
  collect(kernel.body, read, write);
  const auto &p = kernel.params[index];
  const unsigned bits = (read.count(p.name) ? PR_READ : 0) | (write.count(p.name) ? PR_WRITE : 0);
  return static_cast<pr_access>(bits ? bits : unsigned(PR_READ));
}

// ---- provider artifact ----
const std::vector<unsigned char> &provider_artifact() {
  static const std::vector<unsigned char> bytes = [] {
    Writer w;
    const char magic[8] = {'P', 'A', 'R', 'A', 'L', 'Y', 'N', 'B'};
    w.bytes.assign(magic, magic + 8);
    w.u32(1);
    w.string("paralyn.b200.tensor");
    w.string("0.1.0");
    w.string("sm_100a");
    const auto &entries = provider_builtins();
    w.u32(uint32_t(entries.size()));
    for (const auto &e : entries) {
      w.string(e.name);
      for (int d = 0; d < 3; ++d)
        w.u32(e.required_block[d]);
      w.u32(uint32_t(e.params.size()));
      for (const auto &p : e.params) {
        w.string(p.name);
        w.u32(uint32_t(p.type));
        w.u32(p.buffer ? 1 : 0);
        w.u32(uint32_t(p.access));
      }
    }
    return w.bytes;
  }();
  return bytes;
}

bool is_provider_artifact(const void *data, size_t size) {
  const auto &a = provider_artifact();
  return data && size == a.size() && std::equal(a.begin(), a.end(), static_cast<const unsigned char *>(data));
}

} // namespace pb
