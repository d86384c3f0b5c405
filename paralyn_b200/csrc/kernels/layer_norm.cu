// Row LayerNorm for sm_100a, bit-exact with the reference's evaluation order.
//
// Reference (runtime/tensor.cpp:200-212, :276-299): 256 lanes per row; lane t sums
// columns t, t+256, ... in increasing order from +0.0; a pairwise tree
// p[t] = p[t] + p[t+w] for w = 128..1 combines the lanes; mean = S / n;
// var = tree((x - mean)^2) / n with separate roundings; rstd = 1 / sqrt(var + eps);
// out = ((x - mean) * rstd) * gamma + beta. Every step here uses the same
// round-to-nearest operations (__fadd_rn, __fmul_rn, __fdiv_rn, __fsqrt_rn) in the
// same order, so outputs equal the reference order bit for bit.
//
// Fast path (columns % 4 == 0, 16-byte aligned rows, columns <= 4096): one warp per
// row. Thread L owns the reference lanes 8L..8L+7 and loads them as two 128-bit
// vectors per 256-column chunk, so HBM sees one read and one write of the row. The
// tree maps onto the warp: w = 128, 64, 32, 16, 8 pair thread L with L + 16, 8, 4,
// 2, 1 (shuffles), and w = 4, 2, 1 stay inside the thread.
//
// General path: one 256-thread block per row with the reference's lane mapping,
// three passes over the row (the second and third hit L2 for moderate widths).
#include "../runtime/builtin.hpp"
#include <algorithm>

namespace pb {
namespace {

constexpr unsigned full_mask = 0xffffffffu;

template <int R>
__global__ void __launch_bounds__(128) layer_norm_warp_rows(const float *__restrict__ x,
                                                            const float *__restrict__ gamma,
                                                            const float *__restrict__ beta,
                                                            float *__restrict__ out, uint32_t rows,
                                                            uint32_t columns, float epsilon) {
  const uint32_t lane = threadIdx.x & 31u;
  const uint64_t row = uint64_t(blockIdx.x) * 4 + (threadIdx.x >> 5);
  if (row >= rows)
    return;
  const float *xr = x + row * columns;
  float *yr = out + row * columns;
  float v[R][8];
#pragma unroll
  for (int i = 0; i < R; ++i) {
    const uint32_t col = 256u * i + 8u * lane;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
      if (col + 4u * h < columns)
        q = *reinterpret_cast<const float4 *>(xr + col + 4 * h);
      v[i][4 * h + 0] = q.x;
      v[i][4 * h + 1] = q.y;
      v[i][4 * h + 2] = q.z;
      v[i][4 * h + 3] = q.w;
    }
  }
  const float n = __uint2float_rn(columns);
  float s[8];
  auto tree = [&]() {
#pragma unroll
    for (int offset = 16; offset >= 1; offset >>= 1)
#pragma unroll
      for (int c = 0; c < 8; ++c)
        s[c] = __fadd_rn(s[c], __shfl_down_sync(full_mask, s[c], offset));
#pragma unroll
    for (int c = 0; c < 4; ++c)
      s[c] = __fadd_rn(s[c], s[c + 4]);
    s[0] = __fadd_rn(s[0], s[2]);
    s[1] = __fadd_rn(s[1], s[3]);
    s[0] = __fadd_rn(s[0], s[1]);
    return __shfl_sync(full_mask, s[0], 0);
  };
#pragma unroll
  for (int c = 0; c < 8; ++c)
    s[c] = 0.0f;
#pragma unroll
  for (int i = 0; i < R; ++i) {
    const uint32_t col = 256u * i + 8u * lane;
#pragma unroll
    for (int c = 0; c < 8; ++c)
      if (col + 4u * (c / 4) < columns)
        s[c] = __fadd_rn(s[c], v[i][c]);
  }
  const float mean = __fdiv_rn(tree(), n);
#pragma unroll
  for (int c = 0; c < 8; ++c)
    s[c] = 0.0f;
#pragma unroll
  for (int i = 0; i < R; ++i) {
    const uint32_t col = 256u * i + 8u * lane;
#pragma unroll
    for (int c = 0; c < 8; ++c)
      if (col + 4u * (c / 4) < columns) {
        const float d = __fsub_rn(v[i][c], mean);
        s[c] = __fadd_rn(s[c], __fmul_rn(d, d));
      }
  }
  const float variance = __fdiv_rn(tree(), n);
  const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(variance, epsilon)));
#pragma unroll
  for (int i = 0; i < R; ++i) {
    const uint32_t col = 256u * i + 8u * lane;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t j = col + 4u * h;
      if (j < columns) {
        const float4 g = *reinterpret_cast<const float4 *>(gamma + j);
        const float4 b = *reinterpret_cast<const float4 *>(beta + j);
        const float *p = &v[i][4 * h];
        float4 y;
        y.x = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(p[0], mean), rstd), g.x), b.x);
        y.y = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(p[1], mean), rstd), g.y), b.y);
        y.z = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(p[2], mean), rstd), g.z), b.z);
        y.w = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(p[3], mean), rstd), g.w), b.w);
        *reinterpret_cast<float4 *>(yr + j) = y;
      }
    }
  }
}

// 256-lane block tree with lane t = 32*warp + l: w = 128, 64, 32 combine warps
// (w+4, w+2, w+1), w = 16..1 are shuffles inside a warp. Every warp evaluates the
// same expression, so all threads hold the result without a second barrier.
__device__ __forceinline__ float block_tree(float value, float (*scratch)[32]) {
  const uint32_t l = threadIdx.x & 31u, w = threadIdx.x >> 5;
  scratch[w][l] = value;
  __syncthreads();
  const float a = __fadd_rn(__fadd_rn(scratch[0][l], scratch[4][l]), __fadd_rn(scratch[2][l], scratch[6][l]));
  const float b = __fadd_rn(__fadd_rn(scratch[1][l], scratch[5][l]), __fadd_rn(scratch[3][l], scratch[7][l]));
  float s = __fadd_rn(a, b);
#pragma unroll
  for (int offset = 16; offset >= 1; offset >>= 1)
    s = __fadd_rn(s, __shfl_down_sync(full_mask, s, offset));
  return __shfl_sync(full_mask, s, 0);
}

__global__ void __launch_bounds__(256) layer_norm_block_rows(const float *x, const float *gamma,
                                                             const float *beta, float *out,
                                                             uint32_t columns, float epsilon) {
  __shared__ float scratch[2][8][32];
  const uint32_t t = threadIdx.x;
  const uint64_t row = blockIdx.x;
  const float *xr = x + row * columns;
  float *yr = out + row * columns;
  const float n = __uint2float_rn(columns);
  float s = 0.0f;
  for (uint32_t j = t; j < columns; j += 256)
    s = __fadd_rn(s, xr[j]);
  const float mean = __fdiv_rn(block_tree(s, scratch[0]), n);
  float q = 0.0f;
  for (uint32_t j = t; j < columns; j += 256) {
    const float d = __fsub_rn(xr[j], mean);
    q = __fadd_rn(q, __fmul_rn(d, d));
  }
  const float variance = __fdiv_rn(block_tree(q, scratch[1]), n);
  const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(variance, epsilon)));
  for (uint32_t j = t; j < columns; j += 256)
    yr[j] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xr[j], mean), rstd), gamma[j]), beta[j]);
}

template <int R>
void launch_warp_rows(Launch &L, const float *x, const float *g, const float *b, float *y,
                      uint32_t rows, uint32_t columns, float eps) {
  layer_norm_warp_rows<R><<<(rows + 3) / 4, 128, 0, L.stream>>>(x, g, b, y, rows, columns, eps);
  L.variant = "warp_rows_r" + std::to_string(R);
}

} // namespace

// (x, gamma, beta, out, columns, epsilon); one row per 256-lane group of the grid.
void launch_provider_layer_norm(Launch &L) {
  const uint32_t rows = L.grid.x, columns = L.args[4].u32();
  const float eps = L.args[5].f32();
  if (!columns || !rows) { // no element is written for an empty row
    L.variant = "empty";
    return;
  }
  const uint64_t elements = uint64_t(rows) * columns;
  need_elements(L.args[0], elements, "x");
  need_elements(L.args[1], columns, "gamma");
  need_elements(L.args[2], columns, "beta");
  need_elements(L.args[3], elements, "out");
  if (L.dry_run)
    return;
  const auto *x = static_cast<const float *>(L.args[0].ptr);
  const auto *g = static_cast<const float *>(L.args[1].ptr);
  const auto *b = static_cast<const float *>(L.args[2].ptr);
  auto *y = static_cast<float *>(L.args[3].ptr);
  const bool aligned = ((uintptr_t(x) | uintptr_t(g) | uintptr_t(b) | uintptr_t(y)) & 15u) == 0;
  L.kernels = 1;
  if (aligned && columns % 4 == 0 && columns <= 4096) {
    const uint32_t chunks = (columns + 255) / 256;
    if (chunks <= 1)
      launch_warp_rows<1>(L, x, g, b, y, rows, columns, eps);
    else if (chunks <= 2)
      launch_warp_rows<2>(L, x, g, b, y, rows, columns, eps);
    else if (chunks <= 4)
      launch_warp_rows<4>(L, x, g, b, y, rows, columns, eps);
    else if (chunks <= 8)
      launch_warp_rows<8>(L, x, g, b, y, rows, columns, eps);
    else
      launch_warp_rows<16>(L, x, g, b, y, rows, columns, eps);
    return;
  }
  layer_norm_block_rows<<<rows, 256, 0, L.stream>>>(x, g, b, y, columns, eps);
  L.variant = "block_rows";
}

} // namespace pb
