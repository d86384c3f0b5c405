// Built-in kernel table. The provider entries keep the reference provider's
// entry names, parameter names, types, buffer flags, access and required block
// (runtime/tensor.cpp:322-371), because clients check that schema before use
// (runtime/tensor.cpp:595-614).
#include "builtin.hpp"

namespace pb {
namespace {
Param buf(const char *name, pr_access access = PR_READ) {
  return Param{name, Scalar::F32, true, access};
}
Param u32(const char *name) { return Param{name, Scalar::U32, false, PR_READ}; }
Param f32(const char *name) { return Param{name, Scalar::F32, false, PR_READ}; }
constexpr pr_access RW = PR_READ_WRITE;
} // namespace

const std::vector<Builtin> &provider_builtins() {
  static const std::vector<Builtin> table = {
      {"paralyn_matmul_f32", {16, 16, 1},
       {buf("a"), buf("b"), buf("c", RW), u32("m"), u32("n"), u32("k"), u32("transpose_a"),
        u32("transpose_b")},
       launch_provider_matmul},
      {"paralyn_bias_activation_f32", {256, 1, 1},
       {buf("x"), buf("bias"), buf("out", RW), u32("count"), u32("columns"), u32("activation")},
       launch_provider_bias_activation},
      {"paralyn_activation_f32", {256, 1, 1},
       {buf("x"), buf("out", RW), u32("count"), u32("activation")}, launch_provider_activation},
      {"paralyn_fill_f32", {256, 1, 1}, {buf("out", RW), u32("count"), f32("value")},
       launch_provider_fill},
      {"paralyn_batched_matmul_f32", {16, 16, 1},
       {buf("a"), buf("b"), buf("c", RW), u32("m"), u32("n"), u32("k"), u32("a_batch"),
        u32("a_row"), u32("a_col"), u32("b_batch"), u32("b_row"), u32("b_col"), u32("c_batch"),
        u32("c_row"), u32("c_col")},
       launch_provider_batched_matmul},
      {"paralyn_batched_fill_f32", {16, 16, 1},
       {buf("c", RW), u32("m"), u32("n"), u32("c_batch"), u32("c_row"), u32("c_col"),
        f32("value")},
       launch_provider_batched_fill},
      {"paralyn_reduce_rows_f32", {256, 1, 1},
       {buf("x"), buf("out", RW), u32("columns"), u32("op")}, launch_provider_reduce_rows},
      {"paralyn_softmax_rows_f32", {256, 1, 1},
       {buf("x"), buf("out", RW), u32("columns"), u32("rows"), u32("causal"), f32("scale")},
       launch_provider_softmax_rows},
      {"paralyn_layer_norm_f32", {256, 1, 1},
       {buf("x"), buf("gamma"), buf("beta"), buf("out", RW), u32("columns"), f32("epsilon")},
       launch_provider_layer_norm},
      {"paralyn_add_f32", {256, 1, 1}, {buf("x"), buf("y"), buf("out", RW), u32("count")},
       launch_provider_add},
  };
  return table;
}

// Verified-IR kernels recognised by match_ir (module.cpp); their parameter
// names and access come from the loaded IR, so only the launcher matters here.
static const std::vector<Builtin> &ir_builtins() {
  static const std::vector<Builtin> table = {
      {"ir.add.u32", {0, 0, 0}, {}, launch_ir_add_u32},
      {"ir.add.i32", {0, 0, 0}, {}, launch_ir_add_i32},
      {"ir.affine.u32", {0, 0, 0}, {}, launch_ir_affine_u32},
      {"ir.affine.i32", {0, 0, 0}, {}, launch_ir_affine_i32},
      {"ir.affine_scalar.u32", {0, 0, 0}, {}, launch_ir_affine_scalar_u32},
  };
  return table;
}

const Builtin *find_builtin(const std::string &name) {
  for (const auto *table : {&provider_builtins(), &ir_builtins()})
    for (const auto &b : *table)
      if (name == b.name)
        return &b;
  return nullptr;
}

} // namespace pb
