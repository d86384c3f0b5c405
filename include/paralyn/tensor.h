/* FP32 tensor descriptors and the native tensor-operator provider — B200 build.
 *
 * Same records, constants and functions as the reference tensor ABI
 * (reference: include/paralyn/tensor.h:1-192); layouts are pinned with
 * static_asserts in paralyn_b200/csrc/runtime/abi.cpp. The provider returned by
 * pr_tensor_operators_load runs hand-written sm_100a CUDA kernels; the reference's
 * provider is Metal-only.
 *
 * Contract kept from the reference (runtime/tensor.cpp:448-1038):
 *  - descriptors are (buffer, byte offset, dtype, rank, shape, strides); operators
 *    accept contiguous row-major FP32 only and reject other layouts with
 *    PR_UNSUPPORTED; at most INT32_MAX elements per descriptor;
 *  - queue, provider module and every tensor buffer must share one context, checked
 *    before the zero-work decision; zero work returns *out = 0 and launches nothing;
 *  - an output overlapping an input is PR_INVALID_ARGUMENT, an output sharing an
 *    input's allocation at disjoint bytes is PR_UNSUPPORTED; inputs may alias;
 *  - only module handles returned by pr_tensor_operators_load are providers.
 * Numerics: add is exact (one rounding). LayerNorm follows the reference's fixed
 * 256-lane order bit for bit. Matmul accumulates in FP32; its summation mode is a
 * per-context setting (see paralyn/b200.h): the reference order (bit-exact with
 * the sequential FP32 checker), FFMA, or 3xTF32 on the tensor cores. */
#ifndef PARALYN_TENSOR_H
#define PARALYN_TENSOR_H
#include "paralyn/native.h"
#ifdef __cplusplus
extern "C" {
#endif

#define PR_TENSOR_VERSION_1 1u
#define PR_TENSOR_MAX_RANK 8u

typedef struct pr_tensor_desc_v1 {
  uint32_t struct_size, version;
  pr_buffer buffer;
  uint64_t byte_offset; /* multiple of 4 */
  pr_type dtype;        /* PR_F32 */
  uint32_t rank;        /* 0..8; unused dimensions are zero */
  uint64_t shape[PR_TENSOR_MAX_RANK];
  int64_t strides[PR_TENSOR_MAX_RANK]; /* elements, relative to byte_offset */
} pr_tensor_desc_v1;

typedef enum pr_activation {
  PR_ACTIVATION_NONE = 0,
  PR_ACTIVATION_RELU = 1,
  PR_ACTIVATION_GELU_TANH = 2
} pr_activation;

/* C[m,n] = op(A)[m,k] op(B)[k,n]; A stored [m,k] or [k,m] (transpose_a),
 * B stored [k,n] or [n,k] (transpose_b). k == 0 writes +0.0. */
typedef struct pr_matmul_v1 {
  uint32_t struct_size, version;
  uint64_t m, n, k;
  uint32_t transpose_a, transpose_b;
  const pr_tensor_desc_v1 *a, *b, *c;
} pr_matmul_v1;

/* out[i,j] = act(x[i,j] + bias[j]); bias may be NULL. */
typedef struct pr_bias_activation_v1 {
  uint32_t struct_size, version;
  pr_activation activation;
  uint32_t reserved;
  const pr_tensor_desc_v1 *x, *bias, *out;
} pr_bias_activation_v1;

pr_status pr_tensor_desc_contiguous(pr_buffer buffer, uint64_t byte_offset, pr_type dtype,
                                    uint32_t rank, const uint64_t *shape,
                                    pr_tensor_desc_v1 *out);
pr_status pr_tensor_desc_validate(const pr_tensor_desc_v1 *desc, uint64_t *required_bytes);
/* Provider artifact bytes; data == NULL queries the size only. */
pr_status pr_tensor_operators_artifact(void *data, uint64_t capacity, uint64_t *bytes);
pr_status pr_tensor_operators_load(pr_context context, pr_module *out);
pr_status pr_matmul_f32(pr_queue queue, pr_module operators, const pr_matmul_v1 *op,
                        pr_event *out);
pr_status pr_bias_activation_f32(pr_queue queue, pr_module operators,
                                 const pr_bias_activation_v1 *op, pr_event *out);

typedef struct pr_batched_matmul_v1 {
  uint32_t struct_size, version;
  uint64_t batch, m, n, k;
  const pr_tensor_desc_v1 *a, *b, *c;
} pr_batched_matmul_v1;
typedef enum pr_reduce_op { PR_REDUCE_SUM = 0, PR_REDUCE_MAX = 1 } pr_reduce_op;
typedef struct pr_reduce_rows_v1 {
  uint32_t struct_size, version;
  pr_reduce_op op;
  uint32_t reserved;
  const pr_tensor_desc_v1 *x, *out;
} pr_reduce_rows_v1;
/* Row operators keep the reference's row limit floor((2^32-1)/256). */
#define PR_TENSOR_ROW_OPERATOR_MAX_ROWS 16777215u
typedef struct pr_softmax_rows_v1 {
  uint32_t struct_size, version;
  uint32_t causal;
  float scale;
  const pr_tensor_desc_v1 *x, *out;
} pr_softmax_rows_v1;
/* out = ((x - mean) * rstd) * gamma + beta per row; rstd = 1/sqrt(var + epsilon),
 * population variance by two passes; columns <= 2^24; epsilon finite and > 0. */
typedef struct pr_layer_norm_v1 {
  uint32_t struct_size, version;
  float epsilon;
  uint32_t reserved;
  const pr_tensor_desc_v1 *x, *gamma, *beta, *out;
} pr_layer_norm_v1;
typedef struct pr_add_v1 {
  uint32_t struct_size, version;
  const pr_tensor_desc_v1 *x, *y, *out;
} pr_add_v1;
pr_status pr_batched_matmul_f32(pr_queue queue, pr_module operators,
                                const pr_batched_matmul_v1 *op, pr_event *out);
pr_status pr_reduce_rows_f32(pr_queue queue, pr_module operators, const pr_reduce_rows_v1 *op,
                             pr_event *out);
pr_status pr_softmax_rows_f32(pr_queue queue, pr_module operators, const pr_softmax_rows_v1 *op,
                              pr_event *out);
pr_status pr_layer_norm_f32(pr_queue queue, pr_module operators, const pr_layer_norm_v1 *op,
                            pr_event *out);
pr_status pr_add_f32(pr_queue queue, pr_module operators, const pr_add_v1 *op, pr_event *out);

#define PR_TENSOR_OP_MATMUL (1ull << 0)
#define PR_TENSOR_OP_BIAS_ACTIVATION (1ull << 1)
#define PR_TENSOR_OP_BATCHED_MATMUL (1ull << 2)
#define PR_TENSOR_OP_REDUCE_ROWS (1ull << 3)
#define PR_TENSOR_OP_SOFTMAX_ROWS (1ull << 4)
#define PR_TENSOR_OP_LAYER_NORM (1ull << 5)
#define PR_TENSOR_OP_ADD (1ull << 6)
#define PR_TENSOR_ACTIVATION_BIT(activation) (1ull << (unsigned)(activation))
#define PR_TENSOR_REDUCE_BIT(reduce) (1ull << (unsigned)(reduce))
/* Reports the operations this library's provider implements (a library
 * property, not device availability). */
typedef struct pr_tensor_operators_capabilities_v1 {
  uint32_t struct_size, version;
  uint64_t operations;
  uint64_t activations;
  uint64_t reductions;
  uint64_t max_tensor_elements;
  uint64_t max_row_operator_rows;
  uint64_t max_layer_norm_columns;
} pr_tensor_operators_capabilities_v1;
pr_status pr_tensor_operators_capabilities(pr_tensor_operators_capabilities_v1 *out);

#ifdef __cplusplus
}
#endif
#endif
