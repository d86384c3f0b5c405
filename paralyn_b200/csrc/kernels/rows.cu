// Row reductions and row softmax for sm_100a, in the reference's fixed order.
//
// Reference (runtime/tensor.cpp:184-272): one 256-lane group per row; lane t first
// combines columns t, t+256, ... in increasing order (sums from +0.0, maxima from
// -inf), then the pairwise tree p[t] = op(p[t], p[t+w]) for w = 128..1. The
// maximum is total and order-independent except for NaN payloads: NaN if either
// operand is NaN (the first one), +0.0 over -0.0, else the larger value.
// Softmax: v = fl(scale * x); m = tree max of v over the visible columns; e =
// exp(v - m); s = tree sum of e; out = e / s; masked (causal) columns are +0.0 and
// enter neither m nor s. Row r of a batch of `rows` rows sees
// r % rows + (columns - rows) + 1 leading columns when causal.
//
// Sums and maxima round exactly as the reference's (__fadd_rn, __fmul_rn,
// __fsub_rn), so reductions are bit-identical to the reference order. exp is
// CUDA's expf (full-range error within 2 ulp), inside the reference's 4-ulp budget
// for exp; e / s is e times the correctly rounded reciprocal of s (two roundings,
// within about 1 ulp), inside its 2.5-ulp budget for the division.
//
// Fast paths (16-byte aligned rows, columns % 4 == 0) use the lane mapping of the
// LayerNorm kernels: one warp per row, thread L holds the reference lanes
// 4L..4L+3 and 128+4L..128+4L+3, i.e. the float4 at 256i + 4L and at
// 256i + 128 + 4L of chunk i. The tree then runs w = 128 inside the thread,
// w = 64..4 as shuffles with thread L + 16..1 and w = 2, 1 inside the thread.
//   reduce_warp_rows     streams chunks (any column count), 8 rows per block
//   softmax_warp_rows<R> keeps the row in registers (columns <= 256 R, R <= 2),
//                        skips masked columns and takes the row maximum with
//                        max.NaN (same softmax values; see max_nan)
//   softmax_stream_rows  longer rows: the same arithmetic over three passes, e
//                        parked in the output row between the second and third
//                        (at 1024 causal columns 0.92 of HBM against 0.79 for the
//                        row held in registers)
// Other rows take one 256-thread block per row with thread t = lane t.
#include "../runtime/builtin.hpp"
#include <algorithm>

namespace pb {
namespace {

constexpr unsigned full_mask = 0xffffffffu;

struct Sum {
  static __device__ __forceinline__ float identity() { return 0.0f; }
  static __device__ __forceinline__ float apply(float a, float b) { return __fadd_rn(a, b); }
};
struct Max {
  static __device__ __forceinline__ float identity() { return -__int_as_float(0x7f800000); }
  static __device__ __forceinline__ float apply(float a, float b) {
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
};

// Tree over the 8 chains of each thread of a warp (mapping above); every lane
// receives the reference's p[0].
template <class Op> __device__ __forceinline__ float warp_tree(float (&s)[8]) {
#pragma unroll
  for (int c = 0; c < 4; ++c)
    s[c] = Op::apply(s[c], s[c + 4]); // w = 128
#pragma unroll
  for (int offset = 16; offset >= 1; offset >>= 1) // w = 64 .. 4
#pragma unroll
    for (int c = 0; c < 4; ++c)
      s[c] = Op::apply(s[c], __shfl_down_sync(full_mask, s[c], offset));
  s[0] = Op::apply(s[0], s[2]); // w = 2
  s[1] = Op::apply(s[1], s[3]);
  s[0] = Op::apply(s[0], s[1]); // w = 1
  return __shfl_sync(full_mask, s[0], 0);
}

// Tree over 256 threads (thread t = lane t): w = 128, 64, 32 through shared memory,
// w = 16..1 as shuffles in warp 0; every thread receives p[0].
template <class Op> __device__ __forceinline__ float block_tree(float value, float *scratch) {
  const uint32_t t = threadIdx.x;
  scratch[t] = value;
  __syncthreads();
#pragma unroll
  for (uint32_t w = 128; w >= 32; w >>= 1) {
    if (t < w)
      scratch[t] = Op::apply(scratch[t], scratch[t + w]);
    __syncthreads();
  }
  if (t < 32) {
    float v = scratch[t];
#pragma unroll
    for (int offset = 16; offset >= 1; offset >>= 1)
      v = Op::apply(v, __shfl_down_sync(full_mask, v, offset));
    if (t == 0)
      scratch[0] = v;
  }
  __syncthreads();
  const float result = scratch[0];
  __syncthreads(); // scratch is reused by the next tree
  return result;
}

__device__ __forceinline__ void unpack(const float4 &q, float *v) {
  v[0] = q.x, v[1] = q.y, v[2] = q.z, v[3] = q.w;
}

// ---- row reductions ----
template <class Op>
__global__ void __launch_bounds__(256) reduce_warp_rows(const float *__restrict__ x, float *__restrict__ out,
                                                        uint32_t rows, uint32_t columns) {
  const uint32_t lane = threadIdx.x & 31u;
  const uint64_t row = uint64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= rows)
    return;
  const float *xr = x + row * columns;
  float s[8];
#pragma unroll
  for (int c = 0; c < 8; ++c)
    s[c] = Op::identity();
  const uint32_t chunks = (columns + 255) / 256;
  uint32_t i = 0;
  for (; i + 2 <= chunks; i += 2) { // two chunks of loads in flight, combined in order
    float4 q[2][2];
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t col = 256u * (i + u) + 128u * h + 4u * lane;
        q[u][h] = col < columns ? __ldcs(reinterpret_cast<const float4 *>(xr + col))
                                : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
      for (int h = 0; h < 2; ++h)
        if (256u * (i + u) + 128u * h + 4u * lane < columns) {
          float v[4];
          unpack(q[u][h], v);
#pragma unroll
          for (int c = 0; c < 4; ++c)
            s[4 * h + c] = Op::apply(s[4 * h + c], v[c]);
        }
  }
  for (; i < chunks; ++i)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t col = 256u * i + 128u * h + 4u * lane;
      if (col < columns) {
        float v[4];
        unpack(__ldcs(reinterpret_cast<const float4 *>(xr + col)), v);
#pragma unroll
        for (int c = 0; c < 4; ++c)
          s[4 * h + c] = Op::apply(s[4 * h + c], v[c]);
      }
    }
  const float result = warp_tree<Op>(s);
  if (lane == 0)
    out[row] = result;
}

template <class Op>
__global__ void __launch_bounds__(256) reduce_block_rows(const float *x, float *out, uint32_t columns) {
  __shared__ float scratch[256];
  const uint64_t row = blockIdx.x;
  const float *xr = x + row * columns;
  float s = Op::identity();
  for (uint32_t j = threadIdx.x; j < columns; j += 256)
    s = Op::apply(s, xr[j]);
  const float result = block_tree<Op>(s, scratch);
  if (threadIdx.x == 0)
    out[row] = result;
}

// ---- row softmax ----
__device__ __forceinline__ uint32_t visible_columns(uint64_t row, uint32_t rows, uint32_t columns, bool causal) {
  return causal ? uint32_t(row % rows) + (columns - rows) + 1u : columns;
}

// NaN-propagating maximum (max.NaN). For softmax only the value of the row
// maximum matters: exp(v - m) is the same for m = +0.0 and m = -0.0, and any NaN
// makes the whole row NaN, so this one instruction gives the reference's results
// where Max::apply (its exact total order) takes several.
__device__ __forceinline__ float max_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
struct MaxValue {
  static __device__ __forceinline__ float identity() { return -__int_as_float(0x7f800000); }
  static __device__ __forceinline__ float apply(float a, float b) { return max_nan(a, b); }
};

// Row in registers. Columns past `visible` (causal mask) are neither read nor
// computed: whole float4 groups are skipped, only the group holding the mask edge
// checks each element.
template <int R>
__global__ void __launch_bounds__(256, R <= 4 ? 3 : 1) softmax_warp_rows(const float *__restrict__ x, float *__restrict__ out,
                                                         uint32_t all_rows, uint32_t rows, uint32_t columns,
                                                         uint32_t causal, float scale) {
  const uint32_t lane = threadIdx.x & 31u;
  const uint64_t row = uint64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= all_rows)
    return;
  const float *xr = x + row * columns;
  float *yr = out + row * columns;
  const uint32_t visible = visible_columns(row, rows, columns, causal != 0);
  float v[R][2][4];
  float s[8];
#pragma unroll
  for (int c = 0; c < 8; ++c)
    s[c] = MaxValue::identity();
#pragma unroll
  for (int i = 0; i < R; ++i)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t col = 256u * i + 128u * h + 4u * lane;
      if (col < visible) { // masked groups are not read
        unpack(__ldcs(reinterpret_cast<const float4 *>(xr + col)), v[i][h]);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          v[i][h][c] = __fmul_rn(scale, v[i][h][c]);
          if (col + 4 <= visible || col + c < visible)
            s[4 * h + c] = MaxValue::apply(s[4 * h + c], v[i][h][c]);
        }
      }
    }
  const float m = warp_tree<MaxValue>(s);
#pragma unroll
  for (int c = 0; c < 8; ++c)
    s[c] = 0.0f;
#pragma unroll
  for (int i = 0; i < R; ++i)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t col = 256u * i + 128u * h + 4u * lane;
      if (col + 4 <= visible) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          v[i][h][c] = expf(__fsub_rn(v[i][h][c], m));
          s[4 * h + c] = __fadd_rn(s[4 * h + c], v[i][h][c]);
        }
      } else if (col < visible) { // the group holding the mask edge
#pragma unroll
        for (int c = 0; c < 4; ++c)
          if (col + c < visible) {
            v[i][h][c] = expf(__fsub_rn(v[i][h][c], m));
            s[4 * h + c] = __fadd_rn(s[4 * h + c], v[i][h][c]);
          }
      }
    }
  const float rinv = __frcp_rn(warp_tree<Sum>(s));
#pragma unroll
  for (int i = 0; i < R; ++i)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t col = 256u * i + 128u * h + 4u * lane;
      if (col < columns) {
        float y[4];
#pragma unroll
        for (int c = 0; c < 4; ++c)
          y[c] = col + c < visible ? __fmul_rn(v[i][h][c], rinv) : 0.0f;
        __stcs(reinterpret_cast<float4 *>(yr + col), make_float4(y[0], y[1], y[2], y[3]));
      }
    }
}

// Rows over 512 columns in three passes, 8 rows per block and two chunks of loads in
// flight per pass: the maximum over x; e = exp(v - m) summed and stored into the
// output row (write-back, so it stays in L2); e read back and scaled by 1/s. exp is
// evaluated once per element (the kernel is issue-bound), 40 registers keep 48 warps
// on an SM, and the second read of x and the read of e mostly hit L2. Same operations
// in the same order as softmax_warp_rows, so the same bits.
__device__ __forceinline__ float4 load_group(const float *p, bool last_use) {
  const float4 *q = reinterpret_cast<const float4 *>(p);
  return last_use ? __ldcs(q) : __ldcg(q);
}

__global__ void __launch_bounds__(256, 6) softmax_stream_rows(const float *__restrict__ x, float *__restrict__ out,
                                                              uint32_t all_rows, uint32_t rows, uint32_t columns,
                                                              uint32_t causal, float scale) {
  const uint32_t lane = threadIdx.x & 31u;
  const uint64_t row = uint64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= all_rows)
    return;
  const float *xr = x + row * columns;
  float *yr = out + row * columns;
  const uint32_t visible = visible_columns(row, rows, columns, causal != 0);
  const uint32_t chunks = (visible + 255) / 256; // chunks holding a visible column
  float s[8];
#pragma unroll
  for (int c = 0; c < 8; ++c)
    s[c] = MaxValue::identity();
  for (uint32_t i = 0; i < chunks; i += 2) {
    float4 q[2][2];
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t col = 256u * (i + u) + 128u * h + 4u * lane;
        q[u][h] = col < visible ? load_group(xr + col, false) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t col = 256u * (i + u) + 128u * h + 4u * lane;
        float v[4];
        unpack(q[u][h], v);
#pragma unroll
        for (int c = 0; c < 4; ++c)
          if (col + c < visible)
            s[4 * h + c] = MaxValue::apply(s[4 * h + c], __fmul_rn(scale, v[c]));
      }
  }
  const float m = warp_tree<MaxValue>(s);
#pragma unroll
  for (int c = 0; c < 8; ++c)
    s[c] = 0.0f;
  for (uint32_t i = 0; i < chunks; i += 2) {
    float4 q[2][2];
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t col = 256u * (i + u) + 128u * h + 4u * lane;
        q[u][h] = col < visible ? load_group(xr + col, true) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t col = 256u * (i + u) + 128u * h + 4u * lane;
        if (col < visible) {
          float v[4];
          unpack(q[u][h], v);
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            v[c] = col + c < visible ? expf(__fsub_rn(__fmul_rn(scale, v[c]), m)) : 0.0f;
            if (col + c < visible)
              s[4 * h + c] = __fadd_rn(s[4 * h + c], v[c]);
          }
          // e is kept in the output row (write-back, stays in L2) for the last pass
          *reinterpret_cast<float4 *>(yr + col) = make_float4(v[0], v[1], v[2], v[3]);
        }
      }
  }
  const float rinv = __frcp_rn(warp_tree<Sum>(s));
  for (uint32_t i = 0; 256u * i < columns; i += 2) {
    float4 q[2][2];
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t col = 256u * (i + u) + 128u * h + 4u * lane;
        q[u][h] = col < visible ? __ldcg(reinterpret_cast<const float4 *>(yr + col)) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t col = 256u * (i + u) + 128u * h + 4u * lane;
        if (col < columns) {
          float e[4], y[4];
          unpack(q[u][h], e);
#pragma unroll
          for (int c = 0; c < 4; ++c)
            y[c] = col + c < visible ? __fmul_rn(e[c], rinv) : 0.0f;
          __stcs(reinterpret_cast<float4 *>(yr + col), make_float4(y[0], y[1], y[2], y[3]));
        }
      }
  }
}

__global__ void __launch_bounds__(256) softmax_block_rows(const float *x, float *out, uint32_t rows,
                                                          uint32_t columns, uint32_t causal, float scale) {
  __shared__ float scratch[256];
  const uint64_t row = blockIdx.x;
  const float *xr = x + row * columns;
  float *yr = out + row * columns;
  const uint32_t visible = visible_columns(row, rows, columns, causal != 0);
  float m = Max::identity();
  for (uint32_t j = threadIdx.x; j < visible; j += 256)
    m = Max::apply(m, __fmul_rn(scale, xr[j]));
  m = block_tree<Max>(m, scratch);
  float s = 0.0f;
  for (uint32_t j = threadIdx.x; j < visible; j += 256)
    s = __fadd_rn(s, expf(__fsub_rn(__fmul_rn(scale, xr[j]), m)));
  const float rinv = __frcp_rn(block_tree<Sum>(s, scratch));
  for (uint32_t j = threadIdx.x; j < columns; j += 256)
    yr[j] = j < visible ? __fmul_rn(expf(__fsub_rn(__fmul_rn(scale, xr[j]), m)), rinv) : 0.0f;
}

bool aligned16(const void *p) { return (uintptr_t(p) & 15u) == 0; }

template <int R>
void launch_softmax_warp(Launch &L, const float *x, float *y, uint32_t all_rows, uint32_t rows, uint32_t columns,
                         uint32_t causal, float scale) {
  softmax_warp_rows<R><<<(all_rows + 7) / 8, 256, 0, L.stream>>>(x, y, all_rows, rows, columns, causal, scale);
  L.variant = "softmax_warp_rows";
}

} // namespace

// (x, out, columns, op) with one 256-lane group per row: grid.x = rows.
void launch_provider_reduce_rows(Launch &L) {
  const uint32_t rows = L.grid.x, columns = L.args[2].u32(), op = L.args[3].u32();
  if (op > 1)
    throw Failure(PR_INVALID_ARGUMENT, "Unknown reduction");
  if (!rows) {
    L.variant = "empty";
    return;
  }
  need_elements(L.args[0], uint64_t(rows) * columns, "x");
  need_elements(L.args[1], rows, "out");
  if (L.dry_run)
    return;
  const auto *x = static_cast<const float *>(L.args[0].ptr);
  auto *out = static_cast<float *>(L.args[1].ptr);
  L.kernels = 1;
  if (aligned16(x) && columns % 4 == 0) { // also columns == 0: every row gets the identity
    if (op == 1)
      reduce_warp_rows<Max><<<(rows + 7) / 8, 256, 0, L.stream>>>(x, out, rows, columns);
    else
      reduce_warp_rows<Sum><<<(rows + 7) / 8, 256, 0, L.stream>>>(x, out, rows, columns);
    L.variant = "reduce_warp_rows";
    return;
  }
  if (op == 1)
    reduce_block_rows<Max><<<rows, 256, 0, L.stream>>>(x, out, columns);
  else
    reduce_block_rows<Sum><<<rows, 256, 0, L.stream>>>(x, out, columns);
  L.variant = "reduce_block_rows";
}

// (x, out, columns, rows, causal, scale) with one 256-lane group per row:
// grid.x = batch * rows.
void launch_provider_softmax_rows(Launch &L) {
  const uint32_t all_rows = L.grid.x, columns = L.args[2].u32(), rows = L.args[3].u32();
  const uint32_t causal = L.args[4].u32();
  const float scale = L.args[5].f32();
  if (causal > 1)
    throw Failure(PR_INVALID_ARGUMENT, "causal must be 0 or 1");
  if (!all_rows || !columns) { // no element to write
    L.variant = "empty";
    return;
  }
  if (causal && (!rows || columns < rows))
    throw Failure(PR_INVALID_ARGUMENT, "causal softmax requires 0 < rows <= columns");
  need_elements(L.args[0], uint64_t(all_rows) * columns, "x");
  need_elements(L.args[1], uint64_t(all_rows) * columns, "out");
  if (L.dry_run)
    return;
  const auto *x = static_cast<const float *>(L.args[0].ptr);
  auto *y = static_cast<float *>(L.args[1].ptr);
  L.kernels = 1;
  if (aligned16(x) && aligned16(y) && columns % 4 == 0) {
    const uint32_t chunks = (columns + 255) / 256;
    if (chunks <= 1)
      launch_softmax_warp<1>(L, x, y, all_rows, rows, columns, causal, scale);
    else if (chunks <= 2)
      launch_softmax_warp<2>(L, x, y, all_rows, rows, columns, causal, scale);
    else {
      softmax_stream_rows<<<(all_rows + 7) / 8, 256, 0, L.stream>>>(x, y, all_rows, rows, columns, causal, scale);
      L.variant = "softmax_stream_rows";
    }
    return;
  }
  softmax_block_rows<<<all_rows, 256, 0, L.stream>>>(x, y, rows, columns, causal, scale);
  L.variant = "softmax_block_rows";
}

} // namespace pb
