/*
 * CPU oracle for the FP32 operator path: TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load
 * this library, and only as the parity oracle or the timed CPU baseline. The product
 * (libparalyn_native.so) never calls it and has no CPU fallback.
 *
 * Every function restates the arithmetic the reference specifies, in the
 * reference's evaluation order, compiled with -O2 -fno-fast-math
 * -ffp-contract=off so that every FP32 + and * rounds separately:
 *
 *   orc_add_f32            bindings/python/operators.cu:3-8 (array_add),
 *                          runtime/tensor.cpp:302-308 (paralyn_add_f32)
 *   orc_affine_f32         bindings/python/operators.cu:10-16; the verifier in
 *                          scripts/qualify_cuda.py:93 is f32(f32(a*s)+b)
 *   orc_layer_norm_f32     runtime/tensor.cpp:276-299 with the 256-lane tree of
 *                          runtime/tensor.cpp:200-212; the tree emulation follows
 *                          examples/native/transformer_reference.hpp:172-181
 *   orc_layer_norm_bound   float64 running bound of
 *                          examples/native/transformer_reference.hpp:40-147
 *   orc_matmul_f32         runtime/tensor.cpp:44-77 (one accumulator, strictly
 *                          increasing k, product and sum rounded separately);
 *                          sequential checker tests/native/tensor_tests.cpp:62-85
 *   orc_matmul_exact       float64 exact sum and sum|a*b| of the same checker
 *   orc_bias_activation_f32 runtime/tensor.cpp:82-124 (NONE and RELU only)
 *   orc_reduce_rows_f32    runtime/tensor.cpp:214-246 (lane-sequential sum from
 *                          +0.0 / max from -inf, then the 256-lane tree; the max
 *                          rule of :184-191); emulation as in
 *                          examples/native/transformer_reference.hpp:165-191
 *   orc_softmax_rows_f32   runtime/tensor.cpp:248-272 in FP32 with the C library's
 *                          expf (a timing baseline; checks use the bound below)
 *   orc_softmax_bound      float64 running bound of softmax_row,
 *                          examples/native/transformer_reference.hpp:70-73, :122-132
 *                          (exp budgeted at 4 ulp, division at 2.5 ulp)
 *   orc_batched_matmul_f32 runtime/tensor.cpp:130-166: per output one accumulator,
 *                          increasing k, FP32 product then FP32 sum, arbitrary
 *                          non-negative element strides; checker
 *                          tests/native/transformer_ops_tests.cpp:129-169
 *   orc_batched_dot_bound  float64 dot bound of the same checker (gamma_k,
 *                          examples/native/transformer_reference.hpp:100-111)
 *   orc_gelu_bound         float64 bound of the tanh-form GELU with the FP32
 *                          constants, same header :74-80 (tanh at 5 ulp), :113-121
 *
 * Threaded (_mt) variants split rows or ranges across OpenMP threads; each
 * output element is still computed in the reference order, so they are
 * bit-identical to the scalar versions.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_LANES 256u

int orc_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void orc_add_f32(const float *a, const float *b, float *out, size_t n) {
  for (size_t i = 0; i < n; ++i)
    out[i] = a[i] + b[i];
}

void orc_affine_f32(const float *a, const float *b, float *out, size_t n, float scale) {
  for (size_t i = 0; i < n; ++i) {
    const float product = a[i] * scale;
    out[i] = product + b[i];
  }
}

/* out = fl(fl(a*scale) + bias): the affine kernel with a broadcast addend. */
void orc_affine_scalar_f32(const float *a, float *out, size_t n, float scale, float bias) {
  for (size_t i = 0; i < n; ++i) {
    const float product = a[i] * scale;
    out[i] = product + bias;
  }
}

void orc_add_f32_mt(const float *a, const float *b, float *out, size_t n) {
  long long count = (long long)n;
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < count; ++i)
    out[i] = a[i] + b[i];
}

void orc_affine_f32_mt(const float *a, const float *b, float *out, size_t n, float scale) {
  long long count = (long long)n;
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < count; ++i) {
    const float product = a[i] * scale;
    out[i] = product + b[i];
  }
}

void orc_affine_scalar_f32_mt(const float *a, float *out, size_t n, float scale, float bias) {
  long long count = (long long)n;
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < count; ++i) {
    const float product = a[i] * scale;
    out[i] = product + bias;
  }
}

/* Lane t owns columns t, t+256, ... and adds them in increasing order from +0.0;
 * then the pairwise tree p[t] = p[t] + p[t + w] for w = 128, 64, ..., 1. */
static float tree_sum_256(float *p) {
  for (unsigned w = ORC_LANES / 2; w > 0; w >>= 1)
    for (unsigned t = 0; t < w; ++t)
      p[t] = p[t] + p[t + w];
  return p[0];
}

float orc_tree_sum_f32(const float *x, size_t n) {
  float p[ORC_LANES];
  for (unsigned t = 0; t < ORC_LANES; ++t) {
    float s = 0.0f;
    for (size_t j = t; j < n; j += ORC_LANES)
      s = s + x[j];
    p[t] = s;
  }
  return tree_sum_256(p);
}

static void layer_norm_row(const float *x, const float *gamma, const float *beta, float *out,
                           size_t columns, float epsilon) {
  float p[ORC_LANES];
  const float n = (float)columns; /* exact: columns <= 2^24 */
  for (unsigned t = 0; t < ORC_LANES; ++t) {
    float s = 0.0f;
    for (size_t j = t; j < columns; j += ORC_LANES)
      s = s + x[j];
    p[t] = s;
  }
  const float mean = tree_sum_256(p) / n;
  for (unsigned t = 0; t < ORC_LANES; ++t) {
    float q = 0.0f;
    for (size_t j = t; j < columns; j += ORC_LANES) {
      const float d = x[j] - mean;
      const float dd = d * d;
      q = q + dd;
    }
    p[t] = q;
  }
  const float variance = tree_sum_256(p) / n;
  const float root = sqrtf(variance + epsilon);
  const float rstd = 1.0f / root;
  for (size_t j = 0; j < columns; ++j) {
    const float centered = x[j] - mean;
    const float scaled = centered * rstd;
    const float weighted = scaled * gamma[j];
    out[j] = weighted + beta[j];
  }
}

void orc_layer_norm_f32(const float *x, const float *gamma, const float *beta, float *out,
                        size_t rows, size_t columns, float epsilon) {
  for (size_t r = 0; r < rows; ++r)
    layer_norm_row(x + r * columns, gamma, beta, out + r * columns, columns, epsilon);
}

void orc_layer_norm_f32_mt(const float *x, const float *gamma, const float *beta, float *out,
                           size_t rows, size_t columns, float epsilon) {
  long long count = (long long)rows;
#pragma omp parallel for schedule(dynamic, 4)
  for (long long r = 0; r < count; ++r)
    layer_norm_row(x + (size_t)r * columns, gamma, beta, out + (size_t)r * columns, columns,
                   epsilon);
}

/* ---- float64 running error bound (value, error) pairs ----
 * Assumptions as in the reference's bound: FP32 +, -, *, sqrt round to nearest
 * (u = 2^-24), division budgeted at 2.5 ulp, a subnormal result may flush (adds
 * 2^-126 per rounding), no overflow. */
typedef struct {
  double v, e;
} orc_b;
static const double ORC_U = 1.0 / 16777216.0;
static const double ORC_TINY = 1.1754943508222875e-38;
static double gamma_n(double n) { return n * ORC_U / (1.0 - n * ORC_U); }
static double rounded(double magnitude, double eps) { return eps * magnitude + ORC_TINY; }
static orc_b b_sub(orc_b a, orc_b b) {
  orc_b r;
  r.v = a.v - b.v;
  const double e0 = a.e + b.e;
  r.e = e0 + rounded(fabs(r.v) + e0, ORC_U);
  return r;
}
static orc_b b_add(orc_b a, orc_b b) {
  orc_b r;
  r.v = a.v + b.v;
  const double e0 = a.e + b.e;
  r.e = e0 + rounded(fabs(r.v) + e0, ORC_U);
  return r;
}
static orc_b b_mul(orc_b a, orc_b b) {
  orc_b r;
  r.v = a.v * b.v;
  const double e0 = fabs(a.v) * b.e + fabs(b.v) * a.e + a.e * b.e;
  r.e = e0 + rounded(fabs(r.v) + e0, ORC_U);
  return r;
}
static orc_b b_div(orc_b a, orc_b b) {
  orc_b r;
  const double d = fabs(b.v);
  r.v = a.v / b.v;
  if (!(d > b.e)) {
    r.e = INFINITY;
    return r;
  }
  const double e0 = (fabs(a.v) * b.e + d * a.e) / (d * (d - b.e));
  r.e = e0 + rounded(fabs(r.v) + e0, 2.5 * 2.0 * ORC_U);
  return r;
}
static orc_b b_sqrt(orc_b a) {
  orc_b r;
  r.v = sqrt(a.v);
  const double lower = a.v - a.e > 0.0 ? a.v - a.e : 0.0;
  const double e0 = a.e / (r.v + sqrt(lower));
  r.e = e0 + rounded(r.v + e0, ORC_U);
  return r;
}
/* Sum whose deepest addition path has ceil(n/256) + 8 roundings (Higham 4.2). */
static orc_b b_tree_sum(const orc_b *x, size_t n) {
  double v = 0, e0 = 0, magnitude = 0;
  for (size_t i = 0; i < n; ++i) {
    v += x[i].v;
    e0 += x[i].e;
    magnitude += fabs(x[i].v) + x[i].e;
  }
  const double depth = (double)((n + ORC_LANES - 1) / ORC_LANES + 8);
  orc_b r = {v, e0 + gamma_n(depth) * magnitude + depth * ORC_TINY};
  return r;
}

/* value/error arrays of rows*columns entries; scratch needs 2*columns orc_b. */
void orc_layer_norm_bound(const float *x, const float *gamma, const float *beta, size_t rows,
                          size_t columns, double epsilon, double *value, double *error,
                          void *scratch) {
  orc_b *c = (orc_b *)scratch, *q = c + columns;
  for (size_t r = 0; r < rows; ++r) {
    const float *xr = x + r * columns;
    orc_b n = {(double)columns, 0.0};
    for (size_t j = 0; j < columns; ++j) {
      c[j].v = (double)xr[j];
      c[j].e = 0.0;
    }
    const orc_b mean = b_div(b_tree_sum(c, columns), n);
    for (size_t j = 0; j < columns; ++j) {
      orc_b xj = {(double)xr[j], 0.0};
      c[j] = b_sub(xj, mean);
      q[j] = b_mul(c[j], c[j]);
    }
    const orc_b variance = b_div(b_tree_sum(q, columns), n);
    const orc_b one = {1.0, 0.0}, eps = {epsilon, 0.0};
    const orc_b rstd = b_div(one, b_sqrt(b_add(variance, eps)));
    for (size_t j = 0; j < columns; ++j) {
      orc_b g = {(double)gamma[j], 0.0}, b = {(double)beta[j], 0.0};
      orc_b y = b_add(b_mul(b_mul(c[j], rstd), g), b);
      value[r * columns + j] = y.v;
      error[r * columns + j] = y.e;
    }
  }
}

static inline float load_a(const float *a, int ta, size_t m, size_t k, size_t i, size_t p) {
  return ta ? a[p * m + i] : a[i * k + p];
}
static inline float load_b(const float *b, int tb, size_t n, size_t k, size_t p, size_t j) {
  return tb ? b[j * k + p] : b[p * n + j];
}

static void matmul_row(const float *a, const float *b, float *c, size_t m, size_t n, size_t k,
                       int ta, int tb, size_t i) {
  for (size_t j = 0; j < n; ++j) {
    float sum = 0.0f;
    for (size_t p = 0; p < k; ++p) {
      const float product = load_a(a, ta, m, k, i, p) * load_b(b, tb, n, k, p, j);
      sum = sum + product;
    }
    c[i * n + j] = sum;
  }
}

/* C[m,n] = op(A)op(B); rows [row_begin, row_end) only (for sampled baselines). */
void orc_matmul_f32_rows(const float *a, const float *b, float *c, size_t m, size_t n, size_t k,
                         int ta, int tb, size_t row_begin, size_t row_end) {
  for (size_t i = row_begin; i < row_end && i < m; ++i)
    matmul_row(a, b, c, m, n, k, ta, tb, i);
}

void orc_matmul_f32(const float *a, const float *b, float *c, size_t m, size_t n, size_t k, int ta,
                    int tb) {
  orc_matmul_f32_rows(a, b, c, m, n, k, ta, tb, 0, m);
}

void orc_matmul_f32_rows_mt(const float *a, const float *b, float *c, size_t m, size_t n,
                            size_t k, int ta, int tb, size_t row_begin, size_t row_end) {
  long long begin = (long long)row_begin, end = (long long)(row_end < m ? row_end : m);
#pragma omp parallel for schedule(dynamic, 1)
  for (long long i = begin; i < end; ++i)
    matmul_row(a, b, c, m, n, k, ta, tb, (size_t)i);
}

/* float64 exact sum of products and sum of |products| (tests/native/tensor_tests.cpp:69-82). */
void orc_matmul_exact(const float *a, const float *b, double *exact, double *magnitude, size_t m,
                      size_t n, size_t k, int ta, int tb) {
  long long rows = (long long)m;
#pragma omp parallel for schedule(dynamic, 1)
  for (long long ii = 0; ii < rows; ++ii) {
    const size_t i = (size_t)ii;
    for (size_t j = 0; j < n; ++j) {
      double s = 0.0, mag = 0.0;
      for (size_t p = 0; p < k; ++p) {
        const double x = (double)load_a(a, ta, m, k, i, p), y = (double)load_b(b, tb, n, k, p, j);
        s += x * y;
        mag += fabs(x * y);
      }
      exact[i * n + j] = s;
      magnitude[i * n + j] = mag;
    }
  }
}

/* out[i,j] = act(x[i,j] + bias[j]); bias may be NULL. activation 0 = none, 1 = ReLU
 * (values that compare less than zero become +0.0; NaN and -0.0 pass through). */
void orc_bias_activation_f32(const float *x, const float *bias, float *out, size_t rows,
                             size_t columns, int activation) {
  for (size_t i = 0; i < rows; ++i)
    for (size_t j = 0; j < columns; ++j) {
      float v = x[i * columns + j];
      if (bias)
        v = v + bias[j];
      if (activation == 1 && v < 0.0f)
        v = 0.0f;
      out[i * columns + j] = v;
    }
}

/* Sets the OpenMP team size of the _mt variants (launchers such as torchrun export
 * OMP_NUM_THREADS=1 into every process). */
void orc_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0)
    omp_set_num_threads(n);
#else
  (void)n;
#endif
}

/* ---- transformer-block row operators ---- */

/* NaN if either is NaN (the first one), +0.0 preferred over -0.0, else the larger. */
static float max2(float a, float b) {
  if (isnan(a))
    return a;
  if (isnan(b))
    return b;
  if (b > a)
    return b;
  if (b == a && signbit(a) && !signbit(b))
    return b;
  return a;
}

static float tree_max_f32(const float *x, size_t n) {
  float p[ORC_LANES];
  for (unsigned t = 0; t < ORC_LANES; ++t) {
    float m = -INFINITY;
    for (size_t j = t; j < n; j += ORC_LANES)
      m = max2(m, x[j]);
    p[t] = m;
  }
  for (unsigned w = ORC_LANES / 2; w > 0; w >>= 1)
    for (unsigned t = 0; t < w; ++t)
      p[t] = max2(p[t], p[t + w]);
  return p[0];
}

/* op 0 = sum, 1 = max; empty rows give +0.0 / -inf. */
void orc_reduce_rows_f32(const float *x, float *out, size_t rows, size_t columns, int op) {
  for (size_t r = 0; r < rows; ++r)
    out[r] = op == 1 ? tree_max_f32(x + r * columns, columns) : orc_tree_sum_f32(x + r * columns, columns);
}

static orc_b b_exp(orc_b a) {
  orc_b r;
  r.v = exp(a.v);
  const double e0 = r.v * expm1(a.e);
  r.e = e0 + rounded(r.v + e0, 4.0 * 2.0 * ORC_U);
  return r;
}

/* Rows of `columns` entries, `all_rows` of them; row i of a batch of `rows` rows has
 * visible = causal ? i + (columns - rows) + 1 : columns leading entries; the rest are
 * exact zeros (value 0, error 0). scratch needs 2*columns orc_b. */
void orc_softmax_bound(const float *x, size_t all_rows, size_t rows, size_t columns, int causal,
                       float scale, double *value, double *error, void *scratch) {
  orc_b *v = (orc_b *)scratch, *e = v + columns;
  const orc_b s_scale = {(double)scale, 0.0};
  for (size_t r = 0; r < all_rows; ++r) {
    const float *xr = x + r * columns;
    const size_t visible = causal ? (r % rows) + (columns - rows) + 1 : columns;
    orc_b m = {-INFINITY, 0.0};
    for (size_t j = 0; j < visible; ++j) {
      const orc_b xj = {(double)xr[j], 0.0};
      v[j] = b_mul(s_scale, xj);
      m.v = v[j].v > m.v ? v[j].v : m.v;
      m.e = v[j].e > m.e ? v[j].e : m.e;
    }
    for (size_t j = 0; j < visible; ++j)
      e[j] = b_exp(b_sub(v[j], m));
    const orc_b sum = b_tree_sum(e, visible);
    for (size_t j = 0; j < columns; ++j) {
      orc_b y = {0.0, 0.0};
      if (j < visible)
        y = b_div(e[j], sum);
      value[r * columns + j] = y.v;
      error[r * columns + j] = y.e;
    }
  }
}

/* Element (z, i, j) of a strided 3-D operand: base[off + z*s0 + i*s1 + j*s2]. */
typedef struct {
  int64_t offset, s0, s1, s2;
} orc_view;

void orc_batched_matmul_f32(const float *a, orc_view av, const float *b, orc_view bv, float *c,
                            orc_view cv, size_t batch, size_t m, size_t n, size_t k) {
  for (size_t z = 0; z < batch; ++z)
    for (size_t i = 0; i < m; ++i)
      for (size_t j = 0; j < n; ++j) {
        float sum = 0.0f;
        for (size_t p = 0; p < k; ++p) {
          const float x = a[av.offset + z * av.s0 + i * av.s1 + p * av.s2];
          const float y = b[bv.offset + z * bv.s0 + p * bv.s1 + j * bv.s2];
          const float product = x * y;
          sum = sum + product;
        }
        c[cv.offset + z * cv.s0 + i * cv.s1 + j * cv.s2] = sum;
      }
}

/* value/error per output, in [batch][m][n] order; magnitude (sum |a*b|) when not NULL. */
void orc_batched_dot_bound(const float *a, orc_view av, const float *b, orc_view bv, size_t batch,
                           size_t m, size_t n, size_t k, double *value, double *error, double *magnitude_out) {
  for (size_t z = 0; z < batch; ++z)
    for (size_t i = 0; i < m; ++i)
      for (size_t j = 0; j < n; ++j) {
        double v = 0, magnitude = 0;
        for (size_t p = 0; p < k; ++p) {
          const double x = a[av.offset + z * av.s0 + i * av.s1 + p * av.s2];
          const double y = b[bv.offset + z * bv.s0 + p * bv.s1 + j * bv.s2];
          v += x * y;
          magnitude += fabs(x * y);
        }
        const size_t o = (z * m + i) * n + j;
        value[o] = v;
        error[o] = gamma_n((double)k) * magnitude + (double)k * ORC_TINY;
        if (magnitude_out)
          magnitude_out[o] = magnitude;
      }
}

static orc_b b_tanh(orc_b a) {
  orc_b r;
  r.v = tanh(a.v);
  const double lower = fabs(a.v) - a.e > 0.0 ? fabs(a.v) - a.e : 0.0;
  const double t = tanh(lower);
  const double e0 = (1.0 - t * t) * a.e; /* sech^2 decreases in |x| */
  r.e = e0 + rounded(fabs(r.v) + e0, 5.0 * 2.0 * ORC_U);
  return r;
}

/* gelu(x) = (0.5 x)(1 + tanh(c0 (x + c1 ((x x) x)))) with c0, c1 the FP32 constants. */
void orc_gelu_bound(const float *x, size_t n, double *value, double *error) {
  const orc_b c0 = {(double)0.7978845608028654f, 0.0}, c1 = {(double)0.044715f, 0.0};
  const orc_b half = {0.5, 0.0}, one = {1.0, 0.0};
  for (size_t i = 0; i < n; ++i) {
    const orc_b v = {(double)x[i], 0.0};
    const orc_b cube = b_mul(b_mul(v, v), v);
    const orc_b inner = b_add(v, b_mul(c1, cube));
    const orc_b t = b_tanh(b_mul(c0, inner));
    const orc_b y = b_mul(b_mul(half, v), b_add(one, t));
    value[i] = y.v;
    error[i] = y.e;
  }
}

static float tree_sum_of(float *p) { return tree_sum_256(p); }

static void softmax_row(const float *x, float *out, size_t columns, size_t visible, float scale) {
  float p[ORC_LANES];
  for (unsigned t = 0; t < ORC_LANES; ++t) {
    float m = -INFINITY;
    for (size_t j = t; j < visible; j += ORC_LANES)
      m = max2(m, scale * x[j]);
    p[t] = m;
  }
  for (unsigned w = ORC_LANES / 2; w > 0; w >>= 1)
    for (unsigned t = 0; t < w; ++t)
      p[t] = max2(p[t], p[t + w]);
  const float m = p[0];
  for (unsigned t = 0; t < ORC_LANES; ++t) {
    float s = 0.0f;
    for (size_t j = t; j < visible; j += ORC_LANES)
      s = s + expf(scale * x[j] - m);
    p[t] = s;
  }
  const float s = tree_sum_of(p);
  for (size_t j = 0; j < columns; ++j)
    out[j] = j < visible ? expf(scale * x[j] - m) / s : 0.0f;
}

void orc_softmax_rows_f32_mt(const float *x, float *out, size_t all_rows, size_t rows, size_t columns,
                             int causal, float scale) {
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < (long long)all_rows; ++r) {
    const size_t visible = causal ? ((size_t)r % rows) + (columns - rows) + 1 : columns;
    softmax_row(x + (size_t)r * columns, out + (size_t)r * columns, columns, visible, scale);
  }
}

void orc_reduce_rows_f32_mt(const float *x, float *out, size_t rows, size_t columns, int op) {
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < (long long)rows; ++r)
    out[r] = op == 1 ? tree_max_f32(x + (size_t)r * columns, columns)
                     : orc_tree_sum_f32(x + (size_t)r * columns, columns);
}

void orc_batched_matmul_f32_mt(const float *a, orc_view av, const float *b, orc_view bv, float *c, orc_view cv,
                               size_t batch, size_t m, size_t n, size_t k) {
#pragma omp parallel for collapse(2) schedule(static)
  for (long long z = 0; z < (long long)batch; ++z)
    for (long long i = 0; i < (long long)m; ++i)
      for (size_t j = 0; j < n; ++j) {
        float sum = 0.0f;
        for (size_t p = 0; p < k; ++p) {
          const float product = a[av.offset + z * av.s0 + i * av.s1 + p * av.s2] *
                                b[bv.offset + z * bv.s0 + p * bv.s1 + j * bv.s2];
          sum = sum + product;
        }
        c[cv.offset + z * cv.s0 + i * cv.s1 + j * cv.s2] = sum;
      }
}
