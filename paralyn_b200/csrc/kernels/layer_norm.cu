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
// Lane mapping (fast paths, columns % 4 == 0, 16-byte aligned rows): one warp per
// row; thread L keeps the 8 reference lanes 4L..4L+3 and 128+4L..128+4L+3, i.e.
// the float4 at column 256i + 4L and the float4 at 256i + 128 + 4L of every
// 256-column chunk i. Each 128-bit access of a warp is 512 contiguous bytes
// (coalesced in HBM, conflict-free in shared memory). The reference tree maps as:
// w = 128 inside the thread (lane c with lane c + 4), w = 64, 32, 16, 8, 4 are
// shuffles with thread L + 16, 8, 4, 2, 1, and w = 2, 1 are inside the thread.
//
//  layer_norm_bulk<R>      (1024 < columns <= 4096) persistent, 6 warps per SM; each
//                          warp streams its rows through two shared-memory slots
//                          filled by TMA bulk copies (cp.async.bulk, one per row,
//                          completion on an mbarrier), so the next row is in flight
//                          while the current one is reduced; gamma and beta are
//                          staged once per block. HBM sees one read and one write.
//  layer_norm_warp_rows<R> (columns <= 1024) the row in registers, one warp per row.
//  layer_norm_block_rows   any other width: one 256-thread block per row with the
//                          reference lane mapping, three passes over the row.
#include "../runtime/builtin.hpp"
#include <algorithm>

namespace pb {
namespace {

constexpr unsigned full_mask = 0xffffffffu;

// Extra destinations of every output row: row r of this launch also lands at row
// row_offset + r of each dest (tensors of this or peer GPUs, [*, columns]).
struct Gather {
  float *dest[8];
  uint32_t count;
  uint64_t row_offset;
};

template <bool GATHER>
__device__ __forceinline__ void store4(float *yr, const Gather &g, uint64_t row, uint32_t columns, uint32_t col,
                                       const float4 &y) {
  __stcs(reinterpret_cast<float4 *>(yr + col), y); // streamed: written once
  if constexpr (GATHER)
    for (uint32_t d = 0; d < g.count; ++d)
      *reinterpret_cast<float4 *>(g.dest[d] + (g.row_offset + row) * columns + col) = y;
}

// Tree over the 8 chains of every thread of the warp (mapping above); returns the
// reference's p[0] in every lane.
__device__ __forceinline__ float warp_tree(float (&s)[8]) {
#pragma unroll
  for (int c = 0; c < 4; ++c)
    s[c] = __fadd_rn(s[c], s[c + 4]); // w = 128
#pragma unroll
  for (int offset = 16; offset >= 1; offset >>= 1) // w = 64 .. 4
#pragma unroll
    for (int c = 0; c < 4; ++c)
      s[c] = __fadd_rn(s[c], __shfl_down_sync(full_mask, s[c], offset));
  s[0] = __fadd_rn(s[0], s[2]); // w = 2
  s[1] = __fadd_rn(s[1], s[3]);
  s[0] = __fadd_rn(s[0], s[1]); // w = 1
  return __shfl_sync(full_mask, s[0], 0);
}

__device__ __forceinline__ void unpack(const float4 &q, float *v) {
  v[0] = q.x, v[1] = q.y, v[2] = q.z, v[3] = q.w;
}

// Sum and squared-deviation passes over chunks held by `fetch(i, h)` (h = 0: the
// float4 at 256i + 4L, h = 1: at 256i + 128 + 4L), returning mean and rstd.
template <int R, class Fetch>
__device__ __forceinline__ void row_statistics(Fetch fetch, uint32_t lane, uint32_t columns, float epsilon,
                                               float &mean, float &rstd) {
  const float n = __uint2float_rn(columns);
  float s[8];
#pragma unroll
  for (int c = 0; c < 8; ++c)
    s[c] = 0.0f;
#pragma unroll
  for (int i = 0; i < R; ++i)
#pragma unroll
    for (int h = 0; h < 2; ++h)
      if (256u * i + 128u * h + 4u * lane < columns) {
        float v[4];
        unpack(fetch(i, h), v);
#pragma unroll
        for (int c = 0; c < 4; ++c)
          s[4 * h + c] = __fadd_rn(s[4 * h + c], v[c]);
      }
  mean = __fdiv_rn(warp_tree(s), n);
#pragma unroll
  for (int c = 0; c < 8; ++c)
    s[c] = 0.0f;
#pragma unroll
  for (int i = 0; i < R; ++i)
#pragma unroll
    for (int h = 0; h < 2; ++h)
      if (256u * i + 128u * h + 4u * lane < columns) {
        float v[4];
        unpack(fetch(i, h), v);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float d = __fsub_rn(v[c], mean);
          s[4 * h + c] = __fadd_rn(s[4 * h + c], __fmul_rn(d, d));
        }
      }
  const float variance = __fdiv_rn(warp_tree(s), n);
  rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(variance, epsilon)));
}

__device__ __forceinline__ float4 normalize4(const float4 &x, const float4 &g, const float4 &b, float mean,
                                             float rstd) {
  float4 y;
  y.x = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(x.x, mean), rstd), g.x), b.x);
  y.y = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(x.y, mean), rstd), g.y), b.y);
  y.z = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(x.z, mean), rstd), g.z), b.z);
  y.w = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(x.w, mean), rstd), g.w), b.w);
  return y;
}

// ---- the row in registers (narrow rows) ----
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
  float4 v[R][2];
#pragma unroll
  for (int i = 0; i < R; ++i)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t col = 256u * i + 128u * h + 4u * lane;
      v[i][h] = col < columns ? *reinterpret_cast<const float4 *>(xr + col) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  float mean, rstd;
  row_statistics<R>([&](int i, int h) { return v[i][h]; }, lane, columns, epsilon, mean, rstd);
#pragma unroll
  for (int i = 0; i < R; ++i)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t col = 256u * i + 128u * h + 4u * lane;
      if (col < columns)
        *reinterpret_cast<float4 *>(yr + col) =
            normalize4(v[i][h], *reinterpret_cast<const float4 *>(gamma + col),
                       *reinterpret_cast<const float4 *>(beta + col), mean, rstd);
    }
}

// ---- rows streamed through shared memory by TMA bulk copies ----
constexpr int BULK_WARPS = 6, BULK_SLOTS = 2;
constexpr long long BULK_WAIT_CYCLES = 4000000000ll; // ~2 s
constexpr int STATUS_LAYER_NORM_TIMEOUT = 0x7f3301;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity))
    return true;
  const long long start = clock64();
  while (!mbar_try_wait(bar, parity))
    if (clock64() - start > BULK_WAIT_CYCLES)
      return false;
  return true;
}
// Arms `bar` (count 1) for `bytes` of transactions: the phase completes when they land.
__device__ __forceinline__ void expect_bytes(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
// One bulk copy of `bytes` (multiple of 16, 16-byte aligned ends) into shared memory.
__device__ __forceinline__ void bulk_copy(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

template <int R, bool GATHER>
__global__ void __launch_bounds__(32 * BULK_WARPS, 1)
    layer_norm_bulk(const float *__restrict__ x, const float *__restrict__ gamma, const float *__restrict__ beta,
                    float *__restrict__ out, uint32_t rows, uint32_t columns, float epsilon, int *status,
                    const Gather gather) {
  extern __shared__ __align__(128) float smem[];
  constexpr int SLOT = 256 * R; // floats
  float *sg = smem, *sb = smem + SLOT;
  float *slots = smem + 2 * SLOT;
  uint64_t *bars = reinterpret_cast<uint64_t *>(slots + BULK_WARPS * BULK_SLOTS * SLOT);
  uint64_t *gbar = bars + BULK_WARPS * BULK_SLOTS;
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  const uint32_t bytes = columns * 4u;
  if (threadIdx.x == 0) {
    for (int i = 0; i < BULK_WARPS * BULK_SLOTS + 1; ++i)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bars + i)), "r"(1));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    expect_bytes(gbar, 2 * bytes); // gamma and beta complete one phase together
    bulk_copy(sg, gamma, bytes, gbar);
    bulk_copy(sb, beta, bytes, gbar);
  }
  __syncthreads();
  // Waits are bounded per thread and then agreed on, so no thread proceeds alone.
  bool ok = __syncthreads_and(mbar_wait(gbar, 0)) != 0;
  if (!ok && threadIdx.x == 0)
    atomicExch(status, STATUS_LAYER_NORM_TIMEOUT);

  float *const slot0 = slots + warp * BULK_SLOTS * SLOT;
  uint64_t *const bar0 = bars + warp * BULK_SLOTS;
  const uint64_t stride = uint64_t(gridDim.x) * BULK_WARPS;
  const uint64_t first = uint64_t(blockIdx.x) * BULK_WARPS + warp;
  uint64_t issued = 0, consumed = 0; // rows of this warp requested / read
  if (lane == 0)
    for (int s = 0; s < BULK_SLOTS; ++s) {
      const uint64_t row = first + s * stride;
      if (ok && row < rows) {
        expect_bytes(bar0 + s, bytes);
        bulk_copy(slot0 + s * SLOT, x + row * columns, bytes, bar0 + s);
        ++issued;
      }
    }
  issued = __shfl_sync(full_mask, issued, 0);
  for (uint64_t j = 0; ok; ++j) {
    const uint64_t row = first + j * stride;
    if (row >= rows)
      break;
    const int s = int(j % BULK_SLOTS);
    if (!__all_sync(full_mask, mbar_wait(bar0 + s, uint32_t((j / BULK_SLOTS) & 1)))) {
      if (lane == 0)
        atomicExch(status, STATUS_LAYER_NORM_TIMEOUT);
      ok = false;
      break;
    }
    const float *xs = slot0 + s * SLOT;
    float mean, rstd;
    row_statistics<R>(
        [&](int i, int h) { return *reinterpret_cast<const float4 *>(xs + 256 * i + 128 * h + 4 * lane); }, lane,
        columns, epsilon, mean, rstd);
    float *yr = out + row * columns;
#pragma unroll
    for (int i = 0; i < R; ++i)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t col = 256u * i + 128u * h + 4u * lane;
        if (col < columns)
          store4<GATHER>(yr, gather, row, columns, col,
                         normalize4(*reinterpret_cast<const float4 *>(xs + col),
                                    *reinterpret_cast<const float4 *>(sg + col),
                                    *reinterpret_cast<const float4 *>(sb + col), mean, rstd));
      }
    consumed = j + 1;
    // Refill this slot with the row two steps ahead once every lane is done with it.
    __syncwarp();
    const uint64_t next = row + BULK_SLOTS * stride;
    if (next < rows) {
      if (lane == 0) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        expect_bytes(bar0 + s, bytes);
        bulk_copy(slot0 + s * SLOT, x + next * columns, bytes, bar0 + s);
      }
      ++issued;
    }
  }
  // After a timeout, let copies already requested land before the block exits.
  if (!ok)
    for (uint64_t j = consumed; j < issued; ++j)
      (void)mbar_wait(bar0 + j % BULK_SLOTS, uint32_t((j / BULK_SLOTS) & 1));
  if constexpr (GATHER)
    __threadfence_system(); // peer stores are visible system-wide when the command completes
}

// ---- generic: one 256-thread block per row, the reference lane mapping ----
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

template <bool GATHER>
__global__ void __launch_bounds__(256) layer_norm_block_rows(const float *x, const float *gamma,
                                                             const float *beta, float *out,
                                                             uint32_t columns, float epsilon, const Gather gather) {
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
  for (uint32_t j = t; j < columns; j += 256) {
    const float y = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xr[j], mean), rstd), gamma[j]), beta[j]);
    yr[j] = y;
    if constexpr (GATHER)
      for (uint32_t d = 0; d < gather.count; ++d)
        gather.dest[d][(gather.row_offset + row) * columns + j] = y;
  }
  if constexpr (GATHER)
    __threadfence_system();
}

template <int R>
void launch_warp_rows(Launch &L, const float *x, const float *g, const float *b, float *y, uint32_t rows,
                      uint32_t columns, float eps) {
  layer_norm_warp_rows<R><<<(rows + 3) / 4, 128, 0, L.stream>>>(x, g, b, y, rows, columns, eps);
  L.variant = "warp_rows_r" + std::to_string(R);
}

template <int R> size_t bulk_smem() {
  return sizeof(float) * 256 * R * (2 + BULK_WARPS * BULK_SLOTS) + 8 * (BULK_WARPS * BULK_SLOTS + 1);
}

template <int R, bool GATHER = false>
bool launch_bulk(Launch &L, const float *x, const float *g, const float *b, float *y, uint32_t rows,
                 uint32_t columns, float eps, const Gather &gather = Gather{}) {
  static bool configured[64] = {};
  if (L.device < 0 || L.device >= 64)
    return false;
  if (!configured[L.device]) {
    if (cudaFuncSetAttribute(layer_norm_bulk<R, GATHER>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             int(bulk_smem<R>())) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    configured[L.device] = true;
  }
  const uint32_t blocks = uint32_t(std::min<uint64_t>(uint64_t(L.sm_count), (rows + BULK_WARPS - 1) / BULK_WARPS));
  layer_norm_bulk<R, GATHER><<<blocks, 32 * BULK_WARPS, bulk_smem<R>(), L.stream>>>(x, g, b, y, rows, columns,
                                                                                   eps, L.status, gather);
  L.variant = std::string(GATHER ? "bulk_rows_gather_r" : "bulk_rows_r") + std::to_string(R);
  return true;
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
    if (chunks > 8 && launch_bulk<16>(L, x, g, b, y, rows, columns, eps))
      return;
    if (chunks > 4 && launch_bulk<8>(L, x, g, b, y, rows, columns, eps))
      return;
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
  layer_norm_block_rows<false><<<rows, 256, 0, L.stream>>>(x, g, b, y, columns, eps, Gather{});
  L.variant = "block_rows";
}

// (x, gamma, beta, out views, columns, epsilon, rows, row_offset lo/hi, count,
//  count gathered views): LayerNorm whose output rows are also written into every
//  gathered tensor at row_offset + row (local or peer memory).
void launch_layer_norm_gather(Launch &L) {
  const auto &a = L.args;
  const uint32_t columns = a[4].u32(), rows = a[6].u32(), count = a[9].u32();
  const float eps = a[5].f32();
  const uint64_t row_offset = uint64_t(a[7].u32()) | uint64_t(a[8].u32()) << 32;
  if (count > 8 || a.size() != 10 + count)
    throw Failure(PR_INVALID_ARGUMENT, "Malformed gather launch");
  if (!columns || !rows) {
    L.variant = "empty";
    return;
  }
  const uint64_t elements = uint64_t(rows) * columns;
  need_elements(a[0], elements, "x");
  need_elements(a[1], columns, "gamma");
  need_elements(a[2], columns, "beta");
  need_elements(a[3], elements, "out");
  Gather gather{};
  gather.count = count;
  gather.row_offset = row_offset;
  bool aligned = true;
  for (uint32_t d = 0; d < count; ++d) {
    need_elements(a[10 + d], (row_offset + rows) * columns, "gathered");
    gather.dest[d] = static_cast<float *>(a[10 + d].ptr);
    aligned = aligned && (uintptr_t(gather.dest[d]) & 15u) == 0;
  }
  if (L.dry_run)
    return;
  const auto *x = static_cast<const float *>(a[0].ptr);
  const auto *g = static_cast<const float *>(a[1].ptr);
  const auto *b = static_cast<const float *>(a[2].ptr);
  auto *y = static_cast<float *>(a[3].ptr);
  aligned = aligned && ((uintptr_t(x) | uintptr_t(g) | uintptr_t(b) | uintptr_t(y)) & 15u) == 0;
  L.kernels = 1;
  if (aligned && columns % 4 == 0 && columns > 1024 && columns <= 4096) {
    const bool done = columns > 2048 ? launch_bulk<16, true>(L, x, g, b, y, rows, columns, eps, gather)
                                     : launch_bulk<8, true>(L, x, g, b, y, rows, columns, eps, gather);
    if (done)
      return;
  }
  layer_norm_block_rows<true><<<rows, 256, 0, L.stream>>>(x, g, b, y, columns, eps, gather);
  L.variant = "block_rows_gather";
}

} // namespace pb
