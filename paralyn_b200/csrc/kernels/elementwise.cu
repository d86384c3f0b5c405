// Elementwise FP32 kernels for sm_100a: array add/affine (verified-IR entries),
// the provider's add and fill, and bias + activation.
//
// Numerics are those of the reference kernels: add is one round-to-nearest add
// (bindings/python/operators.cu:3-8, emitted as __fadd_rn in
// tests/cuda/golden/array_add.cu), affine is fl(fl(a*scale) + b) with contraction
// off (operators.cu:10-16, golden array_affine.cu), so every result is bit-exact.
//
// Layout: HBM-bound streams. When all pointers share the same offset modulo 16
// bytes, a scalar head brings them to 16-byte alignment and the body moves
// 128-bit vectors; otherwise 32-bit loads are used (still fully coalesced). The
// grid is a multiple of the SM count, each thread keeps four independent 128-bit
// loads per operand in flight.
#include "../runtime/builtin.hpp"
#include "activation.cuh"
#include <algorithm>

namespace pb {
namespace {

enum Op : int { op_add = 0, op_affine = 1, op_affine_scalar = 2, op_fill = 3 };

template <int OP> __device__ __forceinline__ float apply(float a, float b, float scale, float c) {
  if constexpr (OP == op_add)
    return __fadd_rn(a, b);
  else if constexpr (OP == op_affine)
    return __fadd_rn(__fmul_rn(a, scale), b);
  else if constexpr (OP == op_affine_scalar)
    return __fadd_rn(__fmul_rn(a, scale), c);
  else
    return c;
}

template <int OP> __device__ __forceinline__ float4 apply4(float4 a, float4 b, float s, float c) {
  return make_float4(apply<OP>(a.x, b.x, s, c), apply<OP>(a.y, b.y, s, c),
                     apply<OP>(a.z, b.z, s, c), apply<OP>(a.w, b.w, s, c));
}

constexpr bool reads_a(int op) { return op != op_fill; }
constexpr bool reads_b(int op) { return op == op_add || op == op_affine; }

// out[i] = op(a[i], b[i]) for i < n. Elements [0, head) and the tail after the
// last full vector are scalar; [head, head + 4*n4) moves as float4.
template <int OP>
__global__ void __launch_bounds__(256) elementwise_vec(const float *a, const float *b, float *out,
                                                       uint64_t n, uint32_t head, float scale,
                                                       float c) {
  const uint64_t n4 = (n - head) / 4;
  const uint64_t tail = head + n4 * 4;
  const uint64_t tid = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
  if (tid < head)
    out[tid] = apply<OP>(reads_a(OP) ? a[tid] : 0.f, reads_b(OP) ? b[tid] : 0.f, scale, c);
  if (tid < n - tail) {
    const uint64_t i = tail + tid;
    out[i] = apply<OP>(reads_a(OP) ? a[i] : 0.f, reads_b(OP) ? b[i] : 0.f, scale, c);
  }
  const float4 *a4 = reinterpret_cast<const float4 *>(a + head);
  const float4 *b4 = reinterpret_cast<const float4 *>(b + head);
  float4 *o4 = reinterpret_cast<float4 *>(out + head);
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  uint64_t i = tid;
  for (; i + 3 * stride < n4; i += 4 * stride) {
    float4 va[4], vb[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      va[u] = reads_a(OP) ? __ldcs(a4 + i + u * stride) : zero; // streamed: read once
      vb[u] = reads_b(OP) ? __ldcs(b4 + i + u * stride) : zero;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
      __stcs(o4 + i + u * stride, apply4<OP>(va[u], vb[u], scale, c));
  }
  for (; i < n4; i += stride)
    o4[i] = apply4<OP>(reads_a(OP) ? a4[i] : zero, reads_b(OP) ? b4[i] : zero, scale, c);
}

template <int OP>
__global__ void __launch_bounds__(256) elementwise_scalar(const float *a, const float *b, float *out,
                                                          uint64_t n, float scale, float c) {
  const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
  for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    out[i] = apply<OP>(reads_a(OP) ? a[i] : 0.f, reads_b(OP) ? b[i] : 0.f, scale, c);
}

uint32_t blocks_for(uint64_t work_items, int sm_count) {
  const uint64_t wanted = (work_items + 255) / 256;
  const uint64_t cap = uint64_t(sm_count) * 8; // 8 x 256 threads fill an SM
  return uint32_t(std::max<uint64_t>(1, std::min(wanted, cap)));
}

template <int OP>
void enqueue(Launch &L, const float *a, const float *b, float *out, uint64_t n, float scale, float c) {
  L.kernels = 0;
  if (!n)
    return;
  const auto mis = [](const void *p) { return uintptr_t(p) & 15u; };
  bool aligned = true;
  if (reads_a(OP))
    aligned = aligned && mis(a) == mis(out);
  if (reads_b(OP))
    aligned = aligned && mis(b) == mis(out);
  if (aligned) {
    const uint32_t head = uint32_t(std::min<uint64_t>(((16 - mis(out)) & 15) / 4, n));
    const uint64_t vectors = (n - head) / 4;
    elementwise_vec<OP><<<blocks_for(std::max<uint64_t>(vectors / 4, 4), L.sm_count), 256, 0, L.stream>>>(
        a, b, out, n, head, scale, c);
    L.variant = "vec4";
  } else {
    elementwise_scalar<OP><<<blocks_for(n / 4, L.sm_count), 256, 0, L.stream>>>(a, b, out, n, scale, c);
    L.variant = "scalar";
  }
  L.kernels = 1;
}

// Elements a verified-IR elementwise kernel writes: indices i < n among
// blockIdx.x * blockDim.x + threadIdx.x (u32 index; y/z only repeat the same i).
uint64_t ir_count_u32(const Launch &L, uint32_t n) {
  const uint64_t covered = uint64_t(L.grid.x) * L.block.x;
  return std::min<uint64_t>(n, covered);
}
// i32 index: i = int(blockIdx.x * blockDim.x + threadIdx.x). Indices at or above
// 2^31 would turn negative and pass `i < n`; such launches are refused.
uint64_t ir_count_i32(const Launch &L, int32_t n) {
  const uint64_t covered = uint64_t(L.grid.x) * L.block.x;
  if (covered > (uint64_t(1) << 31) && n > INT32_MIN)
    throw Failure(PR_OUT_OF_BOUNDS, "Launch geometry produces negative i32 indices (more than 2^31 "
                                    "threads along x); the access would leave the views");
  if (n <= 0)
    return 0;
  return std::min<uint64_t>(uint64_t(n), covered);
}

template <int OP> void ir_elementwise(Launch &L, uint64_t count) {
  const auto &v = L.args;
  if (OP == op_affine_scalar) { // (a, out, n, scale, bias)
    need_elements(v[0], count, "a");
    need_elements(v[1], count, "out");
    if (L.dry_run)
      return;
    enqueue<OP>(L, static_cast<const float *>(v[0].ptr), nullptr, static_cast<float *>(v[1].ptr),
                count, v[3].f32(), v[4].f32());
    return;
  }
  need_elements(v[0], count, "a"); // (a, b, out, n[, scale])
  need_elements(v[1], count, "b");
  need_elements(v[2], count, "out");
  if (L.dry_run)
    return;
  enqueue<OP>(L, static_cast<const float *>(v[0].ptr), static_cast<const float *>(v[1].ptr),
              static_cast<float *>(v[2].ptr), count, OP == op_affine ? v[4].f32() : 0.f, 0.f);
}

// ---- bias + activation (reference runtime/tensor.cpp:79-115; activation.cuh) ----
__global__ void __launch_bounds__(256) bias_activation(const float *x, const float *bias, float *out,
                                                       uint64_t count, uint32_t columns,
                                                       uint32_t activation) {
  const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
  for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += stride) {
    float v = x[i];
    if (bias)
      v = __fadd_rn(v, bias[i % columns]);
    out[i] = activate(v, activation);
  }
}

} // namespace

void launch_ir_add_u32(Launch &L) { ir_elementwise<op_add>(L, ir_count_u32(L, L.args[3].u32())); }
void launch_ir_add_i32(Launch &L) { ir_elementwise<op_add>(L, ir_count_i32(L, L.args[3].i32())); }
void launch_ir_affine_u32(Launch &L) { ir_elementwise<op_affine>(L, ir_count_u32(L, L.args[3].u32())); }
void launch_ir_affine_i32(Launch &L) { ir_elementwise<op_affine>(L, ir_count_i32(L, L.args[3].i32())); }
void launch_ir_affine_scalar_u32(Launch &L) {
  ir_elementwise<op_affine_scalar>(L, ir_count_u32(L, L.args[2].u32()));
}

// Provider entries use thread_position_in_grid.x with a 256-lane block.
void launch_provider_add(Launch &L) {
  const uint64_t count = std::min<uint64_t>(L.args[3].u32(), uint64_t(L.grid.x) * 256);
  need_elements(L.args[0], count, "x");
  need_elements(L.args[1], count, "y");
  need_elements(L.args[2], count, "out");
  if (L.dry_run)
    return;
  enqueue<op_add>(L, static_cast<const float *>(L.args[0].ptr), static_cast<const float *>(L.args[1].ptr),
                  static_cast<float *>(L.args[2].ptr), count, 0.f, 0.f);
}

void launch_provider_fill(Launch &L) {
  const uint64_t count = std::min<uint64_t>(L.args[1].u32(), uint64_t(L.grid.x) * 256);
  need_elements(L.args[0], count, "out");
  if (L.dry_run)
    return;
  enqueue<op_fill>(L, nullptr, nullptr, static_cast<float *>(L.args[0].ptr), count, 0.f,
                   L.args[2].f32());
}

void launch_provider_bias_activation(Launch &L) { // (x, bias, out, count, columns, activation)
  const uint64_t count = std::min<uint64_t>(L.args[3].u32(), uint64_t(L.grid.x) * 256);
  const uint32_t columns = L.args[4].u32(), activation = L.args[5].u32();
  if (activation > 2)
    throw Failure(PR_INVALID_ARGUMENT, "Unknown activation");
  if (count && !columns)
    throw Failure(PR_INVALID_ARGUMENT, "bias/activation needs columns > 0");
  need_elements(L.args[0], count, "x");
  need_elements(L.args[1], std::min<uint64_t>(columns, count), "bias");
  need_elements(L.args[2], count, "out");
  if (L.dry_run || !count)
    return;
  bias_activation<<<blocks_for(count, L.sm_count), 256, 0, L.stream>>>(
      static_cast<const float *>(L.args[0].ptr), static_cast<const float *>(L.args[1].ptr),
      static_cast<float *>(L.args[2].ptr), count, columns, activation);
  L.kernels = 1;
  L.variant = "bias_activation";
}

void launch_provider_activation(Launch &L) { // (x, out, count, activation)
  const uint64_t count = std::min<uint64_t>(L.args[2].u32(), uint64_t(L.grid.x) * 256);
  const uint32_t activation = L.args[3].u32();
  if (activation > 2)
    throw Failure(PR_INVALID_ARGUMENT, "Unknown activation");
  need_elements(L.args[0], count, "x");
  need_elements(L.args[1], count, "out");
  if (L.dry_run || !count)
    return;
  bias_activation<<<blocks_for(count, L.sm_count), 256, 0, L.stream>>>(
      static_cast<const float *>(L.args[0].ptr), nullptr, static_cast<float *>(L.args[1].ptr), count,
      1, activation);
  L.kernels = 1;
  L.variant = "activation";
}

} // namespace pb
