// Thin C entry points over the reference's OWN sources, compiled in place from
// the reference checkout by oracle/Makefile (target `ref`) into oracle/_ref/.
// Test infrastructure only: used to pin the oracle and the .prk writer against
// the reference itself; nothing in the product links or loads it.
//
//   ref_prk_emit_cuda   deserialize_module (compiler/ir/artifact.cpp:275-313) +
//                       emit_cuda (compiler/codegen/cuda.cpp:84-107) for every
//                       kernel of a .prk; returns the generated CUDA text
//   ref_tree_sum_f32    tree_sum_f32 (examples/native/transformer_reference.hpp:172-181)
//   ref_layer_norm_row  layer_norm_row float64 bound (same header :133-147)
//   ref_tree_max_f32    tree_max_f32 (same header :182-191)
//   ref_softmax_row     softmax_row float64 bound (same header :122-132)
//   ref_dot             dot float64 bound (same header :101-111)
//   ref_gelu            gelu float64 bound (same header :113-121)
#include "paralyn/artifact.hpp"
#include "paralyn/cuda_codegen.hpp"
#include "transformer_reference.hpp"
#include <cstring>
#include <string>
#include <vector>

extern "C" {
// Returns 0 and writes the concatenated CUDA sources (NUL-terminated) on success;
// returns 1 and writes the exception text when the reference rejects the bytes.
int ref_prk_emit_cuda(const void *data, size_t size, char *out, size_t capacity) {
  std::string text;
  int status = 0;
  try {
    for (const auto &kernel : paralyn::deserialize_module(data, size))
      text += paralyn::emit_cuda(kernel);
  } catch (const std::exception &e) {
    text = e.what();
    status = 1;
  }
  if (capacity) {
    const size_t n = text.size() < capacity - 1 ? text.size() : capacity - 1;
    std::memcpy(out, text.data(), n);
    out[n] = 0;
  }
  return status;
}
float ref_tree_sum_f32(const float *x, size_t n) { return paralyn_reference::tree_sum_f32(x, n); }
void ref_layer_norm_row(const float *x, const float *gamma, const float *beta, size_t columns,
                        double epsilon, double *value, double *error) {
  namespace r = paralyn_reference;
  std::vector<float> xs(x, x + columns), gs(gamma, gamma + columns), bs(beta, beta + columns);
  const auto y = r::layer_norm_row(r::exact_values(xs), r::exact_values(gs), r::exact_values(bs),
                                   epsilon);
  for (size_t j = 0; j < columns; ++j) {
    value[j] = y[j].v;
    error[j] = y[j].e;
  }
}
float ref_tree_max_f32(const float *x, size_t n) { return paralyn_reference::tree_max_f32(x, n); }
void ref_softmax_row(const float *x, size_t columns, double scale, size_t visible, double *value,
                     double *error) {
  namespace r = paralyn_reference;
  const auto y = r::softmax_row(r::exact_values(std::vector<float>(x, x + columns)), scale, visible);
  for (size_t j = 0; j < columns; ++j) {
    value[j] = y[j].v;
    error[j] = y[j].e;
  }
}
void ref_dot(const float *a, const float *b, size_t k, double *value, double *error) {
  namespace r = paralyn_reference;
  const auto d = r::dot(r::exact_values(std::vector<float>(a, a + k)), r::exact_values(std::vector<float>(b, b + k)));
  *value = d.v;
  *error = d.e;
}
void ref_gelu(const float *x, size_t n, double *value, double *error) {
  namespace r = paralyn_reference;
  for (size_t i = 0; i < n; ++i) {
    const auto y = r::gelu(r::exact(double(x[i])));
    value[i] = y.v;
    error[i] = y.e;
  }
}
}
