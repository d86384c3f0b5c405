// Kernel modules: verified-IR .prk modules and the built-in tensor provider.
#pragma once
#include "builtin.hpp"
#include <memory>

namespace pb {

// ---- Verified scalar IR (the data model of the .prk container) ----
enum class IrType : uint32_t { I32 = 0, U32 = 1, F32 = 2, Bool = 3 };
enum class ExprKind : uint32_t { Literal = 0, Ref = 1, Builtin = 2, Binary = 3, Cast = 4, Load = 5 };
struct Expr {
  ExprKind kind = ExprKind::Literal;
  IrType type = IrType::I32;
  std::string text;
  std::vector<Expr> operands;
  uint32_t line = 0, column = 0;
};
enum class StmtKind : uint32_t { Let = 0, Store = 1, If = 2 };
struct Stmt {
  StmtKind kind = StmtKind::Let;
  std::string name;
  IrType type = IrType::I32;
  Expr expression, target;
  std::vector<Stmt> body;
};
struct IrParam {
  std::string name;
  IrType type = IrType::I32;
  bool buffer = false, read_only = false;
};
struct IrKernel {
  std::string name;
  std::vector<IrParam> params;
  std::vector<Stmt> body;
};

constexpr size_t prk_max_bytes = 16u << 20;

// Parses a .prk (magic "PARALYN\0", format 1, numerical policy 1) and verifies
// every kernel; throws std::runtime_error on malformed or invalid input.
std::vector<IrKernel> parse_prk(const void *data, size_t size);
void verify_ir(const IrKernel &kernel);
// Serializes kernels in the same container format (used by tests and the
// operators.prk generator through pr_b200_* helpers).
std::vector<unsigned char> write_prk(const std::vector<IrKernel> &kernels);
// Name of the built-in kernel implementing exactly this IR, or "" if none.
std::string match_ir(const IrKernel &kernel);
// Parameter access inferred from loads and stores (reference runtime/native.cpp:241-264).
pr_access ir_access(const IrKernel &kernel, size_t index);

// ---- Provider artifact ----
// The tensor provider's artifact: magic "PARALYNB", version 1, then its entry
// table. The entries (names, parameter names, types, buffer flags, access) are the
// reference's provider schema (runtime/tensor.cpp:322-371), so the reference's
// schema check (runtime/tensor.cpp:595-614) accepts them unchanged.
const std::vector<unsigned char> &provider_artifact();
bool is_provider_artifact(const void *data, size_t size);

struct JitKernel;
// One entry of a loaded module, as pr_module_kernel/pr_kernel_parameter see it.
struct Entry {
  std::string name;
  std::vector<Param> params;
  const Builtin *builtin = nullptr;
  std::shared_ptr<JitKernel> jit; // set for IR compiled at run time
};

} // namespace pb
