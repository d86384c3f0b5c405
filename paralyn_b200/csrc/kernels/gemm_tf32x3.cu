// FP32 GEMM on the sm_100a tensor cores by 3xTF32 splitting (tcgen05 + TMA + TMEM).
//
// Every FP32 operand x is split into two TF32 values, hi = rna_tf32(x) and
// lo = rna_tf32(x - hi) (x - hi is exact in FP32), so x = hi + lo + r with
// |r| <= 2^-22 |x|. Each product is a*b ~= a_hi*b_hi + a_hi*b_lo + a_lo*b_hi (the
// dropped a_lo*b_lo and the residuals are <= ~2^-20.4 |a*b|), accumulated in FP32
// in tensor memory. For k >= 16 this is far inside the FP32 contract
// |C - C_exact| <= 2*k*2^-24*sum|a||b| that the FFMA path also meets; smaller k is
// declined and runs on the SIMT kernel. Non-finite inputs can turn an
// infinite product into NaN (inf - inf in the split).
//
// Structure:
//  1. split kernels: op(A) -> A_hi, A_lo [M_pad][K_pad] and op(B)^T -> B_hi, B_lo
//     [N_pad][K_pad] in the context workspace, K contiguous, zero padded (one read,
//     two writes of each operand; 128-bit accesses, a 32x32 shared-memory transpose
//     for the transposed layouts). An operand loaded raw by the GEMM is not split.
//  2. persistent GEMM kernel (gemm_tf32x3_persistent, for the tensor provider): one
//     CTA per SM walks work units, 128 x BN output tiles (BN = 64, 128, 256) and the
//     k-ranges of the tiles of a short last round.
//     warp 0 lane 0: TMA producer. Each 16-deep k-slice is four 2-D boxes (A_hi,
//       A_lo 128x16; B_hi, B_lo BNx16; 64-byte rows, SWIZZLE_64B), or one raw FP32
//       box in place of a pair, into a 192 KB ring signalled by mbarrier transaction
//       counts.
//     warp 1: allocates 2 x BN TMEM columns; lane 0 issues per 8-deep step three
//       tcgen05.mma.kind::tf32 (128xBNx8, both operands K-major from shared memory
//       descriptors) into one of two accumulators and releases each stage with
//       tcgen05.commit.
//     warps 2-9: epilogue, two warps per TMEM lane quarter (one per column half):
//       tcgen05.ld 32 lanes x 16 columns, fused bias/ReLU, 128-bit stores staged
//       through shared memory; then the accumulator is handed back.
//     warps 10-25 (raw forms only): split the raw box of each stage into its TF32
//       pair in shared memory.
//     The transposed form of a C with at most 64 columns runs 64-row tiles (M = 64
//     MMAs, D's row r in TMEM lane (r % 16) + 32 (r / 16)).
//     A separate kernel adds the partial tiles of split tiles (split_fixup).
//  3. one-tile GEMM kernel (gemm_tf32x3, 6 warps, one 128x256 tile per CTA) for the
//     allocation-free entry point at the end of this file.
//  Every wait is bounded (about two seconds of SM clock); on expiry the kernel
//  records a status code in host-mapped memory, stops issuing, frees its TMEM and
//  returns, and the engine reports PR_EXECUTION_FAILED.
#include "../runtime/builtin.hpp"
#include "activation.cuh"
#include "prepared.hpp"
#include "tma.cuh"
#include <cuda.h>
#include <algorithm>
#include <atomic>
#include <cstdlib>

namespace pb {
namespace {

constexpr int TM = 128, TN = 256, TK = 16, STAGES = 4, THREADS = 192;
constexpr int A_BYTES = TM * TK * 4, B_BYTES = TN * TK * 4;
constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
constexpr uint32_t TMEM_COLUMNS = 256;
constexpr long long WAIT_CYCLES = tma::kWaitCycles;
constexpr int STATUS_TIMEOUT_PRODUCER = 0x7f3201, STATUS_TIMEOUT_MMA = 0x7f3202,
              STATUS_TIMEOUT_EPILOGUE = 0x7f3203;

using tma::mbar_expect_tx;
using tma::mbar_init;
using tma::mbar_try_wait;
using tma::mbar_wait;
using tma::smem_u32;
using tma::tma_load_2d;

// Shared-memory matrix descriptor: K-major, SWIZZLE_64B (64-byte rows, 8-row
// 512-byte atoms): start >> 4, leading byte offset 16 (unused for swizzled
// K-major), stride byte offset 512, descriptor version 1, layout type 4.
__device__ __forceinline__ uint64_t desc_k_sw64(uint32_t addr) {
  return uint64_t((addr & 0x3FFFFu) >> 4) | (uint64_t(16 >> 4) << 16) | (uint64_t(512 >> 4) << 32) |
         (uint64_t(1) << 46) | (uint64_t(4) << 61);
}

// Instruction descriptor: D f32, A and B tf32, both K-major, N = 256, M = 128.
constexpr uint32_t IDESC = (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(TN >> 3) << 17) |
                           (uint32_t(TM >> 4) << 24);

__device__ __forceinline__ void mma_tf32(uint32_t tmem, uint64_t a, uint64_t b, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
      "l"(a), "l"(b), "r"(IDESC), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_load_32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  // The registers are operands of the wait, so no use of them moves above it.
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i)
    v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_load_16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
               "%14, %15}, [%16];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                 "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                 "=r"(r[15])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15])
               :
               : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i)
    v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// hi/lo split of op(X) into [rows_pad][k_pad] (K contiguous), zero padded.
// Element (r, k) of op(X) is x[r*ld + k], or x[k*ld + r] when `transposed`.
// Batched (grid.z > 1): matrix z starts x_batch elements after matrix z-1 and is
// written rows_pad rows after it.
// `nonfinite` (optional) is set to `epoch` when an element's high part is infinite
// (an infinite input, or a finite one that rounds to infinity in TF32): its low part
// is then inf - inf and the 3xTF32 products would turn +-inf into NaN.
__global__ void __launch_bounds__(256) split_tf32(const float *__restrict__ x, int64_t ld, int transposed,
                                                  int64_t rows, int64_t k, float *__restrict__ hi,
                                                  float *__restrict__ lo, int64_t k_pad, int64_t x_batch,
                                                  int64_t rows_pad, unsigned long long *nonfinite,
                                                  unsigned long long epoch) {
  __shared__ float tile[32][33];
  x += int64_t(blockIdx.z) * x_batch;
  hi += int64_t(blockIdx.z) * rows_pad * k_pad;
  lo += int64_t(blockIdx.z) * rows_pad * k_pad;
  const int64_t r0 = int64_t(blockIdx.y) * 32, k0 = int64_t(blockIdx.x) * 32;
  const int tx = threadIdx.x % 32, ty = threadIdx.x / 32; // 32 x 8
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int a = ty + 8 * j;
    if (!transposed) {
      const int64_t r = r0 + a, kk = k0 + tx;
      tile[a][tx] = (r < rows && kk < k) ? x[r * ld + kk] : 0.0f;
    } else {
      const int64_t kk = k0 + a, r = r0 + tx;
      tile[tx][a] = (r < rows && kk < k) ? x[kk * ld + r] : 0.0f;
    }
  }
  __syncthreads();
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int a = ty + 8 * j;
    const float v = tile[a][tx];
    const float h = tf32_rna(v);
    const float l = tf32_rna(v - h);
    if (nonfinite && isinf(h))
      *nonfinite = epoch;
    const int64_t offset = (r0 + a) * k_pad + k0 + tx;
    hi[offset] = h;
    lo[offset] = l;
  }
}

// The same split with 128-bit accesses, for 16-byte aligned operands whose leading
// dimension is a multiple of 4 (both grids cover [rows_pad][k_pad] in 32x32 tiles,
// z = matrix). Stored [rows][k]: each thread converts four consecutive k of a row,
// no shared memory. Stored [k][rows] (transposed): a 32x32 tile is read as float4
// along the rows, transposed in shared memory and written as float4 along k.
__device__ __forceinline__ void split4(float4 v, float4 &h, float4 &l) {
  h = make_float4(tf32_rna(v.x), tf32_rna(v.y), tf32_rna(v.z), tf32_rna(v.w));
  l = make_float4(tf32_rna(v.x - h.x), tf32_rna(v.y - h.y), tf32_rna(v.z - h.z), tf32_rna(v.w - h.w));
}
__device__ __forceinline__ bool any_inf(float4 h) { return isinf(h.x) || isinf(h.y) || isinf(h.z) || isinf(h.w); }
__global__ void __launch_bounds__(256) split_tf32_vec(const float *__restrict__ x, int64_t ld, int transposed,
                                                      int64_t rows, int64_t k, float *__restrict__ hi,
                                                      float *__restrict__ lo, int64_t k_pad, int64_t x_batch,
                                                      int64_t rows_pad, unsigned long long *nonfinite,
                                                      unsigned long long epoch) {
  __shared__ float tile[32][33];
  x += int64_t(blockIdx.z) * x_batch;
  hi += int64_t(blockIdx.z) * rows_pad * k_pad;
  lo += int64_t(blockIdx.z) * rows_pad * k_pad;
  const int64_t r0 = int64_t(blockIdx.y) * 32, k0 = int64_t(blockIdx.x) * 32;
  const int q = threadIdx.x % 8, a = threadIdx.x / 8; // 8 float4 x 32 lines
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  if (!transposed) { // line a = row r0 + a, k0 + 4q .. +3
    const int64_t r = r0 + a, kk = k0 + 4 * q;
    float4 v = zero;
    if (r < rows && kk + 3 < k)
      v = *reinterpret_cast<const float4 *>(x + r * ld + kk);
    else if (r < rows)
      for (int e = 0; e < 4; ++e)
        if (kk + e < k)
          (&v.x)[e] = x[r * ld + kk + e];
    float4 h, l;
    split4(v, h, l);
    if (nonfinite && any_inf(h))
      *nonfinite = epoch;
    const int64_t offset = r * k_pad + kk;
    *reinterpret_cast<float4 *>(hi + offset) = h;
    *reinterpret_cast<float4 *>(lo + offset) = l;
    return;
  }
  { // line a = k0 + a, rows r0 + 4q .. +3
    const int64_t kk = k0 + a, r = r0 + 4 * q;
    float4 v = zero;
    if (kk < k && r + 3 < rows)
      v = *reinterpret_cast<const float4 *>(x + kk * ld + r);
    else if (kk < k)
      for (int e = 0; e < 4; ++e)
        if (r + e < rows)
          (&v.x)[e] = x[kk * ld + r + e];
    tile[4 * q + 0][a] = v.x;
    tile[4 * q + 1][a] = v.y;
    tile[4 * q + 2][a] = v.z;
    tile[4 * q + 3][a] = v.w;
  }
  __syncthreads();
  { // line a = row r0 + a, k0 + 4q .. +3
    const float4 v = make_float4(tile[a][4 * q], tile[a][4 * q + 1], tile[a][4 * q + 2], tile[a][4 * q + 3]);
    float4 h, l;
    split4(v, h, l);
    if (nonfinite && any_inf(h))
      *nonfinite = epoch;
    const int64_t offset = (r0 + a) * k_pad + k0 + 4 * q;
    *reinterpret_cast<float4 *>(hi + offset) = h;
    *reinterpret_cast<float4 *>(lo + offset) = l;
  }
}

struct TileArgs {
  float *c;
  int64_t m, n, ldc;
  int k_blocks, tiles_m, tiles_n;
  int *status;
  // Batched launches: tiles_m * tiles_n CTAs per matrix; matrix z reads the split
  // rows z*a_rows.. of A and z*b_rows.. of B (0: shared by all) and writes C at
  // c + z*c_batch. Zero tiles_per_batch means one matrix.
  int tiles_per_batch = 0, a_rows = 0, b_rows = 0;
  int64_t c_batch = 0;
  int tiles_total = 0; // persistent kernel: tiles of all matrices
  // Persistent kernel work units: units [0, full_units) are whole tiles; after them
  // every remaining tile is cut into `split` k-ranges whose partial sums go to
  // `partials` (one 128x256 tile each) and are added by split_fixup.
  int units_total = 0, full_units = 0, split = 1;
  float *partials = nullptr;
  // Fused epilogue: C = activate(fl(acc + bias[column])) (activation.cuh).
  const float *bias = nullptr;
  uint32_t activation = 0;
  // The kernel computes D = C^T (m, n above are D's): D[i][j] is stored to C[j][i].
  bool transposed = false;
  // Set to `epoch` by the converter warps when a raw operand's high part is infinite
  // (as the split kernels do for the operands they split); null: not watched.
  unsigned long long *nonfinite = nullptr;
  unsigned long long epoch = 0;
  // Tile rows per raster group (consecutive tiles walk the columns of `group` tile
  // rows, so they share B's tiles in L2); the persistent kernels and split_fixup
  // read it, the one-tile kernel uses 8.
  int group = 8;
  // CTA-pair kernel, optional: one zeroed counter per round of whole tiles. Before a
  // round's loads each pair's producer arrives and waits until the round's other
  // pairs have arrived or wave_wait_ns have passed (then it goes on: the wait only
  // keeps the pairs' k-streams of one round together, for L2 reuse).
  int *wave_count = nullptr;
  long long wave_wait_ns = 0;
  // CTA-pair kernel and its fixup: with col_group > 0 consecutive tiles walk the rows
  // of `col_group` column tiles instead (group is then unused).
  int col_group = 0;
};

__global__ void __launch_bounds__(THREADS, 1)
    gemm_tf32x3(const __grid_constant__ CUtensorMap a_hi, const __grid_constant__ CUtensorMap a_lo,
                const __grid_constant__ CUtensorMap b_hi, const __grid_constant__ CUtensorMap b_lo,
                const TileArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + STAGES * STAGE_BYTES);
  uint64_t *empty = full + STAGES;
  uint64_t *accum = empty + STAGES;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accum + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  volatile int *issued = abort_flag + 1;   // k-slices the producer has requested
  volatile int *consumed = abort_flag + 2; // k-slices whose data the MMA thread received

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int per_batch = args.tiles_per_batch ? args.tiles_per_batch : args.tiles_m * args.tiles_n;
  const int z = blockIdx.x / per_batch;
  // Grouped raster: 8 tile-rows at a time so consecutive CTAs share B tiles in L2.
  const int id = blockIdx.x % per_batch, group = 8, per_group = group * args.tiles_n;
  const int first_m = (id / per_group) * group;
  const int rows_in_group = min(group, args.tiles_m - first_m);
  const int tm = first_m + (id % per_group) % rows_in_group;
  const int tn = (id % per_group) / rows_in_group;
  const int m0 = tm * TM, n0 = tn * TN;
  const int a_y = z * args.a_rows + m0, b_y = z * args.b_rows + n0; // rows of the split operands
  float *const c_base = args.c + int64_t(z) * args.c_batch;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    *abort_flag = 0;
    *issued = 0;
    *consumed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLUMNS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  }
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) { // TMA producer
      for (int kb = 0; kb < args.k_blocks; ++kb) {
        const int s = kb % STAGES;
        const uint32_t round = kb / STAGES;
        if (kb >= STAGES && !mbar_wait(&empty[s], (round - 1) & 1)) {
          atomicExch(args.status, STATUS_TIMEOUT_PRODUCER);
          *abort_flag = 1;
          break;
        }
        if (*abort_flag)
          break;
        uint8_t *stage = smem + s * STAGE_BYTES;
        mbar_expect_tx(&full[s], STAGE_BYTES);
        tma_load_2d(stage, &a_hi, &full[s], kb * TK, a_y);
        tma_load_2d(stage + A_BYTES, &a_lo, &full[s], kb * TK, a_y);
        tma_load_2d(stage + 2 * A_BYTES, &b_hi, &full[s], kb * TK, b_y);
        tma_load_2d(stage + 2 * A_BYTES + B_BYTES, &b_lo, &full[s], kb * TK, b_y);
        *issued = kb + 1;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) { // MMA issuer
      for (int kb = 0; kb < args.k_blocks; ++kb) {
        const int s = kb % STAGES;
        if (!mbar_wait(&full[s], (kb / STAGES) & 1)) {
          atomicExch(args.status, STATUS_TIMEOUT_MMA);
          *abort_flag = 1;
          break;
        }
        *consumed = kb + 1;
        if (*abort_flag)
          break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t stage = smem_u32(smem + s * STAGE_BYTES);
#pragma unroll
        for (int kk = 0; kk < TK / 8; ++kk) {
          const uint32_t step = kk * 32; // 8 tf32 = 32 bytes along the 64-byte row
          const uint64_t ah = desc_k_sw64(stage + step), al = desc_k_sw64(stage + A_BYTES + step);
          const uint64_t bh = desc_k_sw64(stage + 2 * A_BYTES + step);
          const uint64_t bl = desc_k_sw64(stage + 2 * A_BYTES + B_BYTES + step);
          mma_tf32(tmem, ah, bh, (kb > 0 || kk > 0) ? 1u : 0u);
          mma_tf32(tmem, ah, bl, 1u);
          mma_tf32(tmem, al, bh, 1u);
        }
        mma_commit(&empty[s]);
      }
      // Always committed: it fires once every MMA this thread issued has finished,
      // so TMEM is quiet before the epilogue reads it or the block frees it.
      mma_commit(accum);
    }
  } else { // epilogue warps 2..5: TMEM lanes 32*(warp % 4) ..
    const int sub = warp % 4;
    // The accumulator is ready after the whole k loop: budget ~2 s plus 50 us per slice.
    bool ready = mbar_try_wait(accum, 0);
    const long long start = clock64(), budget = WAIT_CYCLES + 100000ll * args.k_blocks;
    while (!ready && clock64() - start < budget)
      ready = mbar_try_wait(accum, 0);
    if (!ready) {
      atomicExch(args.status, STATUS_TIMEOUT_EPILOGUE);
      *abort_flag = 1;
    } else if (!*abort_flag) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int64_t row = int64_t(m0) + 32 * sub + lane;
      float *crow = c_base + row * args.ldc;
      const bool vec = (args.ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(c_base) & 15u) == 0);
#pragma unroll 1
      for (int col = 0; col < TN; col += 32) {
        float v[32];
        tmem_load_32(tmem + (uint32_t(32 * sub) << 16) + uint32_t(col), v);
        if (row < args.m) {
          const int64_t n_first = int64_t(n0) + col;
          if (vec && n_first + 31 < args.n) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
              *reinterpret_cast<float4 *>(crow + n_first + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (n_first + j < args.n)
                crow[n_first + j] = v[j];
          }
        }
      }
    }
  }
  __syncthreads();
  if (*abort_flag && threadIdx.x == 0) {
    // Let the copies that were requested but never consumed land (bounded) before
    // the block's shared memory is released.
    for (int kb = *consumed; kb < *issued; ++kb)
      (void)mbar_wait(&full[kb % STAGES], (kb / STAGES) & 1);
  }
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLUMNS)
                 : "memory");
  }
}


// Persistent form: one CTA per SM walks the work units blockIdx.x, + gridDim.x, ...
// The shared-memory ring runs continuously across units (one k-slice counter
// for producer and MMA), and the accumulator is double-buffered in TMEM (2 x BN
// columns): the MMA thread computes unit j into buffer j % 2 while the epilogue
// warps drain unit j - 1 from the other buffer, so stores of C overlap the
// tensor-core work instead of following it.
//   tmem_full[b]  MMA -> epilogue: all MMAs of the buffer's current unit are done
//                 (tcgen05.commit); phase u = the u-th unit that used buffer b
//   tmem_empty[b] epilogue -> MMA: the eight epilogue warps have read buffer b
//                 (one elected lane per warp arrives; count 8)
// Every wait is bounded as in the one-tile kernel; before TMEM is freed the MMA
// thread's final commit guarantees no MMA is still writing it.
// Epilogue stores are coalesced: each warp passes 32 x 16 accumulator chunks
// (thread = row) through a shared-memory tile with 20-float rows (16-byte aligned;
// its writes and its reads by groups of eight lanes touch eight distinct 4-bank
// groups) and writes them back with 128-bit stores, four threads per 64-byte row
// segment, eight rows per instruction.
// ---- persistent kernel ----
// One CTA per SM walks work units (whole tiles, then k-ranges of the tiles of a
// short last round). The N tile width BN is 64, 128 or 256 (the narrow tiles keep
// the tensor cores off padding when n is small); every form uses a 192 KB ring of
// 16-deep k-slices (200 KB for the 64-row transposed form). With RAW = RAW_A (RAW_B) the producer loads raw FP32 boxes of
// the A (B) operand and sixteen converter warps split them into the hi/lo pair in
// shared memory with the same conversion as split_tf32 (so the operands, and the
// result, are bit-identical), which saves the split pass over that operand when
// few tiles re-read it. TOUT computes C^T: the kernel's M side is C's columns and
// its N side C's rows, and the epilogue stores D[i][j] to C[j][i] (a narrow C runs
// this way, since a tcgen05 MMA of N = 64 costs about as much as one of N = 256).
// Eight epilogue warps: warps 2..5 and 6..9 each cover the four TMEM lane quarters,
// the first group the left half of the tile's columns, the second the right half,
// staged 32 rows x 16 columns at a time.
constexpr int EPI_WARPS = 8, EPI_PITCH16 = 16;
constexpr int EPI_STAGE_FLOATS = 32 * EPI_PITCH16;
// An epilogue warp's staging tile, 32 rows x 16 columns, row pitch 16 floats, with the
// 4-float groups of row r stored in the order q ^ ((r / 2) % 4). Both accesses are
// free of bank conflicts: the rows written from tensor memory (lane = row, 8 lanes
// per phase) and the reads for the global stores, where each 8-lane phase takes two
// rows x 64 bytes, so that one store instruction writes 8 rows in four phases of two
// cache lines each (the unswizzled pitch-20 tile needed 8 rows per phase: 8 lines,
// and the stores kept the L1 load/store pipe 87 % busy on the batched Q K^T product).
__device__ __forceinline__ int stage_index(int r, int c) {
  return r * EPI_PITCH16 + ((((c >> 2) ^ (r >> 1)) & 3) << 2) + (c & 3);
}
constexpr int RING_BYTES = 192 * 1024, BARRIER_BYTES = 512;
constexpr int THREADS_PLAIN = 64 + 32 * EPI_WARPS;
// The one-SM kernel's converter warps, which share each k-slice (the CTA pair keeps
// four per CTA). A slice's conversion sits on the ring's critical loop (load ->
// convert -> MMA -> release), so it is spread thin: with four warps the transposed
// P V product of the encoder block took 158 us, with eight 125, with sixteen 123.
constexpr int CONVERT_WARPS = 16, CONVERT_THREADS = 32 * CONVERT_WARPS,
              THREADS_RAW_ONE = THREADS_PLAIN + CONVERT_THREADS;
constexpr int STATUS_TIMEOUT_CONVERT = 0x7f3204;
constexpr int RAW_NONE = 0, RAW_A = 1, RAW_B = 2;

// MR: rows of a tile (the MMA's M), 128, or 64 for the transposed form of a C with at
// most 64 columns: an M = 64 MMA writes D's row r to TMEM lane (r % 16) + 32 (r / 16),
// the first 16 lanes of each warp's quarter, so no MMA or TMA copy is spent on the 64
// rows of zero padding an M = 128 tile would carry, and a stage is 40 KB instead of 48.
template <int BN, int MR = TM> struct Tile {
  static_assert(BN == 64 || BN == 128 || BN == 256, "N tile");
  static_assert(MR == 128 || MR == 64, "M tile");
  static constexpr int A_BYTES = MR * TK * 4;
  static constexpr int B_BYTES = BN * TK * 4;
  static constexpr int STAGE = 2 * A_BYTES + 2 * B_BYTES;
  static constexpr int RING = MR == 64 ? 200 * 1024 : RING_BYTES;
  static constexpr int STAGES = RING / STAGE; // 4, 6 or 8; 5 for the M = 64 form
  static constexpr int SMEM = 1024 + RING + BARRIER_BYTES + EPI_WARPS * EPI_STAGE_FLOATS * 4;
  static constexpr int LANES = MR / 4;        // D rows in each warp's TMEM lane quarter
  static constexpr uint32_t COLUMNS = BN;     // TMEM columns of one accumulator
  // D f32, A and B tf32, both K-major, N = BN, M = MR.
  static constexpr uint32_t IDESC =
      (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(BN >> 3) << 17) | (uint32_t(MR >> 4) << 24);
};
static_assert(Tile<256, 64>::SMEM <= 227 * 1024, "shared memory of the M = 64 form");

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

template <int BN, int MR>
__device__ __forceinline__ void mma_tf32_n(uint32_t tmem, uint64_t a, uint64_t b, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
      "l"(a), "l"(b), "r"(Tile<BN, MR>::IDESC), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ float4 tf32_hi(float4 v) {
  return make_float4(tf32_rna(v.x), tf32_rna(v.y), tf32_rna(v.z), tf32_rna(v.w));
}

template <int BN, int RAW, bool TOUT, int MR = TM>
__global__ void __launch_bounds__(RAW ? THREADS_RAW_ONE : THREADS_PLAIN, 1)
    gemm_tf32x3_persistent(const __grid_constant__ CUtensorMap a_hi, const __grid_constant__ CUtensorMap a_lo,
                           const __grid_constant__ CUtensorMap b_hi, const __grid_constant__ CUtensorMap b_lo,
                           const TileArgs args) {
  using C = Tile<BN, MR>;
  constexpr int S = C::STAGES, A_BYTES = C::A_BYTES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::RING);
  uint64_t *empty = full + S;
  uint64_t *converted = empty + S; // RAW: the stage's raw operand is split in shared memory
  uint64_t *tmem_full = converted + S;
  uint64_t *tmem_empty = tmem_full + 2;
  uint64_t *drained = tmem_empty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drained + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  volatile int *issued = abort_flag + 1;   // k-slices the producer has requested
  volatile int *consumed = abort_flag + 2; // k-slices whose data the MMA thread received
  float *epi_tiles = reinterpret_cast<float *>(smem + C::RING + BARRIER_BYTES);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int per_batch = args.tiles_per_batch ? args.tiles_per_batch : args.tiles_m * args.tiles_n;
  auto locate = [&](int tile, int &a_y, int &b_y, int &m0, int &n0, int &z) {
    z = tile / per_batch;
    const int id = tile % per_batch, group = args.group, per_group = group * args.tiles_n;
    const int first_m = (id / per_group) * group;
    const int rows_in_group = min(group, args.tiles_m - first_m);
    m0 = (first_m + (id % per_group) % rows_in_group) * MR;
    n0 = ((id % per_group) / rows_in_group) * BN;
    a_y = z * args.a_rows + m0;
    b_y = z * args.b_rows + n0;
  };
  // Unit -> tile and k-slice range [kb0, kb1).
  auto unit = [&](int u, int &tile, int &kb0, int &kb1) {
    if (u < args.full_units) {
      tile = u;
      kb0 = 0;
      kb1 = args.k_blocks;
    } else {
      const int v = u - args.full_units, part = v % args.split;
      tile = args.full_units + v / args.split;
      kb0 = part * args.k_blocks / args.split;
      kb1 = (part + 1) * args.k_blocks / args.split;
    }
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&converted[s], CONVERT_WARPS);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tmem_full[b], 1);
      mbar_init(&tmem_empty[b], EPI_WARPS);
    }
    mbar_init(drained, 1);
    *abort_flag = 0;
    *issued = 0;
    *consumed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(2 * C::COLUMNS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  }
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) { // TMA producer
      int g = 0;
      for (int u = blockIdx.x; u < args.units_total && !*abort_flag; u += gridDim.x) {
        int tile, kb0, kb1, a_y, b_y, m0, n0, z;
        unit(u, tile, kb0, kb1);
        locate(tile, a_y, b_y, m0, n0, z);
        for (int kb = kb0; kb < kb1; ++kb, ++g) {
          const int s = g % S;
          const uint32_t round = g / S;
          if (g >= S && !mbar_wait(&empty[s], (round - 1) & 1)) {
            atomicExch(args.status, STATUS_TIMEOUT_PRODUCER);
            *abort_flag = 1;
          }
          if (*abort_flag)
            break;
          uint8_t *stage = smem + s * C::STAGE;
          mbar_expect_tx(&full[s], C::STAGE - (RAW == RAW_A ? A_BYTES : 0) - (RAW == RAW_B ? C::B_BYTES : 0));
          if (RAW == RAW_A) {
            tma_load_3d(stage, &a_hi, &full[s], kb * TK, m0, z);
          } else {
            tma_load_2d(stage, &a_hi, &full[s], kb * TK, a_y);
            tma_load_2d(stage + A_BYTES, &a_lo, &full[s], kb * TK, a_y);
          }
          if (RAW == RAW_B) {
            tma_load_3d(stage + 2 * A_BYTES, &b_hi, &full[s], kb * TK, n0, z);
          } else {
            tma_load_2d(stage + 2 * A_BYTES, &b_hi, &full[s], kb * TK, b_y);
            tma_load_2d(stage + 2 * A_BYTES + C::B_BYTES, &b_lo, &full[s], kb * TK, b_y);
          }
          *issued = g + 1;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) { // MMA issuer
      uint64_t *ready = RAW ? converted : full;
      int g = 0, j = 0;
      for (int u = blockIdx.x; u < args.units_total && !*abort_flag; u += gridDim.x, ++j) {
        int tile, kb0, kb1;
        unit(u, tile, kb0, kb1);
        const int b = j & 1;
        if (j >= 2 && !mbar_wait(&tmem_empty[b], ((j >> 1) - 1) & 1)) {
          atomicExch(args.status, STATUS_TIMEOUT_MMA);
          *abort_flag = 1;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t acc = tmem + uint32_t(b) * C::COLUMNS;
        for (int kb = kb0; kb < kb1; ++kb, ++g) {
          const int s = g % S;
          if (!mbar_wait(&ready[s], (g / S) & 1)) {
            atomicExch(args.status, STATUS_TIMEOUT_MMA);
            *abort_flag = 1;
            break;
          }
          *consumed = g + 1;
          if (*abort_flag)
            break;
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t stage = smem_u32(smem + s * C::STAGE);
#pragma unroll
          for (int kk = 0; kk < TK / 8; ++kk) {
            const uint32_t step = kk * 32;
            const uint64_t ah = desc_k_sw64(stage + step), al = desc_k_sw64(stage + A_BYTES + step);
            const uint64_t bh = desc_k_sw64(stage + 2 * A_BYTES + step);
            const uint64_t bl = desc_k_sw64(stage + 2 * A_BYTES + C::B_BYTES + step);
            // Products in the order a_hi b_hi, a_hi b_lo, a_lo b_hi of C's own operands
            // (the transposed form's A is C's B), so both forms give the same bits.
            mma_tf32_n<BN, MR>(acc, ah, bh, (kb > kb0 || kk > 0) ? 1u : 0u);
            mma_tf32_n<BN, MR>(acc, TOUT ? al : ah, TOUT ? bh : bl, 1u);
            mma_tf32_n<BN, MR>(acc, TOUT ? ah : al, TOUT ? bl : bh, 1u);
          }
          mma_commit(&empty[s]);
        }
        if (*abort_flag)
          break;
        mma_commit(&tmem_full[b]);
      }
      // Fires once every MMA issued above has finished (TMEM quiet before it is freed).
      mma_commit(drained);
    }
  } else if (warp >= 2 + EPI_WARPS) { // RAW converter warps 10..25: raw box -> hi in place, lo beside it
    const int t = threadIdx.x - THREADS_PLAIN;
    constexpr int RAW_OFFSET = RAW == RAW_B ? 2 * A_BYTES : 0, RAW_BYTES = RAW == RAW_B ? C::B_BYTES : A_BYTES;
    static_assert(RAW_BYTES % (16 * CONVERT_THREADS) == 0, "converter share");
    int g = 0;
    for (int u = blockIdx.x; u < args.units_total && !*abort_flag; u += gridDim.x) {
      int tile, kb0, kb1;
      unit(u, tile, kb0, kb1);
      for (int kb = kb0; kb < kb1; ++kb, ++g) {
        const int s = g % S;
        if (!mbar_wait(&full[s], (g / S) & 1)) {
          atomicExch(args.status, STATUS_TIMEOUT_CONVERT);
          *abort_flag = 1;
        }
        if (*abort_flag)
          break;
        float4 *hi = reinterpret_cast<float4 *>(smem + s * C::STAGE + RAW_OFFSET);
        float4 *lo = reinterpret_cast<float4 *>(smem + s * C::STAGE + RAW_OFFSET + RAW_BYTES);
        // The swizzle is the same for both boxes, so the pair is formed position by position.
#pragma unroll
        for (int i = 0; i < RAW_BYTES / 16 / CONVERT_THREADS; ++i) {
          const float4 v = hi[t + CONVERT_THREADS * i];
          const float4 h = tf32_hi(v);
          lo[t + CONVERT_THREADS * i] = tf32_hi(make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w));
          hi[t + CONVERT_THREADS * i] = h;
          if (args.nonfinite && any_inf(h))
            *args.nonfinite = args.epoch;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); // visible to the tensor cores
        __syncwarp();
        if (lane == 0)
          asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&converted[s])) : "memory");
      }
    }
  } else { // epilogue warps 2..9: TMEM lanes 32*(warp % 4) .., column half (warp - 2) / 4
    const int sub = warp % 4, half = (warp - 2) / 4;
    int j = 0;
    for (int u = blockIdx.x; u < args.units_total; u += gridDim.x, ++j) {
      int tile, kb0, kb1;
      unit(u, tile, kb0, kb1);
      const int b = j & 1;
      bool ready = mbar_try_wait(&tmem_full[b], (j >> 1) & 1);
      const long long start = clock64(), budget = WAIT_CYCLES + 100000ll * args.k_blocks;
      while (!ready && !*abort_flag && clock64() - start < budget)
        ready = mbar_try_wait(&tmem_full[b], (j >> 1) & 1);
      if (!ready || *abort_flag) {
        if (!ready && !*abort_flag)
          atomicExch(args.status, STATUS_TIMEOUT_EPILOGUE);
        *abort_flag = 1;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      int a_y, b_y, m0, n0, z;
      locate(tile, a_y, b_y, m0, n0, z);
      // Whole tiles go to C; the k-range parts of split tiles go to their own
      // 128 x BN partial tile (row stride BN), all of it written.
      const bool whole = u < args.full_units;
      float *const c_base = whole ? args.c + int64_t(z) * args.c_batch
                                  : args.partials + int64_t(u - args.full_units) * (MR * BN);
      const int64_t ldc = whole ? args.ldc : BN, m_lim = whole ? args.m : MR, n_lim = whole ? args.n : BN;
      // This warp's rows: C::LANES (32, or 16 in the M = 64 form) held by its first lanes.
      const int64_t row0 = (whole ? int64_t(m0) : 0) + C::LANES * sub;
      const int64_t col0 = whole ? int64_t(n0) : 0;
      const int64_t left = m_lim - row0;
      const int rows_here = left >= C::LANES ? C::LANES : (left > 0 ? int(left) : 0);
      float *tile_s = epi_tiles + (warp - 2) * EPI_STAGE_FLOATS;
      const uint32_t acc = tmem + uint32_t(b) * C::COLUMNS + (uint32_t(32 * sub) << 16);
      const bool vec_c = (ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(c_base) & 15u) == 0);
#pragma unroll 1
      for (int col = half * (BN / 2); col < (half + 1) * (BN / 2); col += 16) {
        float v[16];
        tmem_load_16(acc + uint32_t(col), v); // lane < C::LANES: row C::LANES*sub + lane, 16 columns
        const int64_t first = col0 + col;
        if (first >= n_lim)
          break; // the remaining columns of the tile are past n
        if (TOUT && whole) { // D row = C column (the lanes store consecutive C columns)
          const int64_t c_col = row0 + lane;
          if (lane < C::LANES && c_col < m_lim) {
            float *cptr = c_base + first * ldc + c_col;
#pragma unroll
            for (int q = 0; q < 16; ++q)
              if (first + q < n_lim)
                cptr[q * ldc] = (args.bias || args.activation)
                                    ? bias_activate(v[q], args.bias, c_col, args.activation)
                                    : v[q];
          }
          continue;
        }
        if (whole && (args.bias || args.activation)) {
#pragma unroll
          for (int q = 0; q < 16; ++q)
            if (first + q < n_lim)
              v[q] = bias_activate(v[q], args.bias, first + q, args.activation);
        }
#pragma unroll
        for (int q = 0; q < 16; q += 4)
          *reinterpret_cast<float4 *>(&tile_s[stage_index(lane, q)]) =
              make_float4(v[q], v[q + 1], v[q + 2], v[q + 3]);
        __syncwarp();
        if (vec_c && rows_here == 32 && first + 15 < n_lim) {
          // 8 rows x 64 bytes per instruction: lane = (phase, p), phase = lane / 8 takes
          // rows 2 phase and 2 phase + 1, p % 4 the 4-float group
          const int r_in = 2 * (lane >> 3) + ((lane & 7) >> 2), c4 = 4 * (lane & 3);
          float4 w[4];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            w[i] = *reinterpret_cast<const float4 *>(&tile_s[stage_index(8 * i + r_in, c4)]);
          float *cptr = c_base + (row0 + r_in) * ldc + first + c4;
#pragma unroll
          for (int i = 0; i < 4; ++i)
            *reinterpret_cast<float4 *>(cptr + int64_t(8 * i) * ldc) = w[i];
        } else { // lanes 0..15 / 16..31: one column each, even / odd rows
          const int64_t column = first + (lane & 15);
          if (column < n_lim) {
            float *cptr = c_base + row0 * ldc + column;
            for (int r = lane >> 4; r < rows_here; r += 2)
              cptr[r * ldc] = tile_s[stage_index(r, lane & 15)];
          }
        }
        __syncwarp();
      }
      // The buffer's loads are complete (tcgen05.wait::ld in tmem_load_32): hand it back.
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0)
        asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&tmem_empty[b])) : "memory");
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (*abort_flag) // copies requested but never consumed must land before shared memory is released
      for (int g = *consumed; g < *issued; ++g)
        (void)mbar_wait(&full[g % S], (g / S) & 1);
    (void)mbar_wait(drained, 0); // bounded: every MMA has finished writing TMEM
  }
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * C::COLUMNS)
                 : "memory");
  }
}

// ---- CTA-pair persistent kernel (tcgen05.mma.cta_group::2) ----
// A cluster of two CTAs on two SMs computes 256 x 256 output tiles: CTA r holds rows
// [128 r, 128 r + 128) of the tile's A pair and rows [128 r, 128 r + 128) of its B
// pair (the B^T side) in its own shared memory, and one MMA issued by CTA 0 reads
// both CTAs' operands and writes each CTA's 128 x 256 accumulator into that CTA's
// tensor memory. Each SM therefore stages and reads half of B instead of all of it:
// per 16-deep slice an SM's shared memory takes 32 KB of TMA writes and feeds 48 KB
// to the tensor cores (80 KB), against 48 KB + 72 KB for the one-SM 128 x 256 tile,
// which was bound by that traffic rather than by the MMAs.
//  warp 0 lane 0 (both CTAs): TMA producer. It waits for its own stage to be free
//    (`empty`, signalled by CTA 0's MMA commit in both CTAs), CTA 0 arms its `full`
//    barrier with both CTAs' bytes, and both CTAs' copies complete on CTA 0's
//    barrier (cta_group::2 TMA; each CTA loads its own half).
//  warp 1 (both CTAs): allocates 512 TMEM columns as a pair (two 256-column
//    accumulators); lane 0 of CTA 0 issues the MMAs and commits stages and
//    accumulators to the barriers of both CTAs.
//  warps 2 .. 1 + EW (both CTAs; EW = 8, or 16 when a bias or activation is fused):
//    drain the CTA's own accumulator as in the one-SM kernel and report to CTA 0's
//    `tmem_empty` (2 EW arrivals: the epilogue warps of both CTAs).
// Every wait is bounded. Before either CTA releases its shared and tensor memory,
// CTA 0 waits for its last MMA to finish and both CTAs meet at a cluster barrier.
// Deep products (k >= 2048) align the pairs' rounds: CTA 0's producer waits (at most
// TileArgs::wave_wait_ns) for the round's other pairs before loading its tile, so the
// tiles of one round stream the same k-slices of X and W at about the same time.
constexpr int PAIR_HALF = 128, PAIR_M = 2 * PAIR_HALF, PAIR_N = 256;
constexpr int PAIR_A_BYTES = PAIR_HALF * TK * 4, PAIR_B_BYTES = PAIR_HALF * TK * 4;
constexpr int PAIR_STAGE = 2 * PAIR_A_BYTES + 2 * PAIR_B_BYTES; // 32 KB per CTA
constexpr int PAIR_STAGES = RING_BYTES / PAIR_STAGE;            // 6
constexpr uint32_t PAIR_COLUMNS = PAIR_N;                       // TMEM columns of one accumulator
// D f32, A and B tf32, both K-major, N = 256, M = 256 (the pair's rows).
constexpr uint32_t PAIR_IDESC =
    (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(PAIR_N >> 3) << 17) | (uint32_t(PAIR_M >> 4) << 24);

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// The shared::cluster address of `p` (a shared-memory object of this CTA) in CTA `rank`.
__device__ __forceinline__ uint32_t in_cta(const void *p, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(p)), "r"(rank));
  return out;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// One arrival on the barrier at `cluster_bar` (this CTA's or the peer's). Default
// (release, CTA scope) semantics: the data a converter wrote is ordered for the
// tensor cores by its fence.proxy.async, and a cluster-scope release here would put
// a full memory barrier on every stage (measured: 2.5x slower pair kernel).
__device__ __forceinline__ void arrive_at(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}
// A 2-D tile into this CTA's shared memory whose byte count completes on the barrier
// at `cluster_bar` (CTA 0's, for both CTAs of the pair).
__device__ __forceinline__ void tma_load_2d_pair(void *dst, const CUtensorMap *map, uint32_t cluster_bar, int x,
                                                 int y) {
  asm volatile("cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
               " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(cluster_bar)
               : "memory");
}
__device__ __forceinline__ void mma_tf32_pair(uint32_t tmem, uint64_t a, uint64_t b, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
      "l"(a), "l"(b), "r"(PAIR_IDESC), "r"(accumulate)
      : "memory");
}
// Arrives (once) on the barrier at `cluster_bar` when every MMA this thread issued so
// far has completed; called once per destination CTA.
__device__ __forceinline__ void mma_commit_pair(uint32_t cluster_bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_bar)
               : "memory");
}

// RAW: A is read raw (FP32 boxes of its own rows, from the caller's matrix) and four
// converter warps per CTA form its TF32 pair in shared memory with the split pass's
// own conversion, so no split pass runs over A. The raw box of a stage completes on
// the CTA's own `raw_full` barrier; the converters of both CTAs report to CTA 0's
// `converted` barrier, which the MMA waits for besides `full` (now B's bytes only).
// The CTA pair's epilogue warps: EW / 4 per TMEM lane quarter, each taking that share
// of the tile's columns (plus four converter warps per CTA in the RAW form). Sixteen
// (EW = 16) when a bias or activation is fused: they sped up the encoder block's GELU
// up-projection from 103 to 97 us and its QKV projection from 82 to 79; without an
// epilogue computation eight, since sixteen slowed the store-bound score products
// (32 x 2048 x 2048 x 128: 141 -> 131 TFLOP/s).
template <int EW> struct PairShape {
  static_assert(EW == 8 || EW == 16, "epilogue warps");
  static constexpr int PARTS = EW / 4;
  static constexpr int THREADS_PLAIN = 64 + 32 * EW, THREADS_RAW = THREADS_PLAIN + 128;
  static constexpr int SMEM = 1024 + RING_BYTES + BARRIER_BYTES + EW * EPI_STAGE_FLOATS * 4;
  static_assert(SMEM <= 227 * 1024, "shared memory of the CTA pair");
};

template <bool RAW, int EW>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(RAW ? PairShape<EW>::THREADS_RAW : PairShape<EW>::THREADS_PLAIN, 1)
    gemm_tf32x3_pair(const __grid_constant__ CUtensorMap a_hi, const __grid_constant__ CUtensorMap a_lo,
                     const __grid_constant__ CUtensorMap b_hi, const __grid_constant__ CUtensorMap b_lo,
                     const TileArgs args) {
  constexpr int S = PAIR_STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + RING_BYTES); // used in CTA 0
  uint64_t *empty = full + S;
  uint64_t *tmem_full = empty + S;
  uint64_t *tmem_empty = tmem_full + 2; // used in CTA 0
  uint64_t *drained = tmem_empty + 2;   // used in CTA 0
  uint64_t *raw_full = drained + 1;     // RAW: this CTA's raw A box of the stage landed
  uint64_t *converted = raw_full + S;   // RAW, CTA 0: both CTAs' A pairs of the stage are formed
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(converted + S);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  volatile int *issued = abort_flag + 1;   // k-slices the producer has requested
  volatile int *consumed = abort_flag + 2; // k-slices whose data the MMA thread received (CTA 0)
  float *epi_tiles = reinterpret_cast<float *>(smem + RING_BYTES + BARRIER_BYTES);

  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int pair = blockIdx.x / 2, pairs = gridDim.x / 2;
  const int per_batch = args.tiles_per_batch ? args.tiles_per_batch : args.tiles_m * args.tiles_n;
  auto locate = [&](int tile, int &m0, int &n0, int &z) { // m0 in rows of PAIR_M tiles
    z = tile / per_batch;
    const int id = tile % per_batch;
    if (args.col_group > 0) {
      const int group = args.col_group, per_group = group * args.tiles_m;
      const int first_n = (id / per_group) * group;
      const int cols_in_group = min(group, args.tiles_n - first_n);
      n0 = (first_n + (id % per_group) % cols_in_group) * PAIR_N;
      m0 = ((id % per_group) / cols_in_group) * PAIR_M;
      return;
    }
    const int group = args.group, per_group = group * args.tiles_n;
    const int first_m = (id / per_group) * group;
    const int rows_in_group = min(group, args.tiles_m - first_m);
    m0 = (first_m + (id % per_group) % rows_in_group) * PAIR_M;
    n0 = ((id % per_group) / rows_in_group) * PAIR_N;
  };
  auto unit = [&](int u, int &tile, int &kb0, int &kb1) {
    if (u < args.full_units) {
      tile = u;
      kb0 = 0;
      kb1 = args.k_blocks;
    } else {
      const int v = u - args.full_units, part = v % args.split;
      tile = args.full_units + v / args.split;
      kb0 = part * args.k_blocks / args.split;
      kb1 = (part + 1) * args.k_blocks / args.split;
    }
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tmem_full[b], 1);
      mbar_init(&tmem_empty[b], 2 * EW);
    }
    mbar_init(drained, 1);
    for (int s = 0; s < S; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&converted[s], 2 * 4); // the four converter warps of each CTA
    }
    *abort_flag = 0;
    *issued = 0;
    *consumed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(2 * PAIR_COLUMNS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  }
  // Both CTAs' barriers are initialized and both hold the TMEM allocation before any
  // copy or MMA of the pair reaches the other CTA.
  cluster_sync_all();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  const uint32_t full0 = in_cta(full, 0), tmem_empty0 = in_cta(tmem_empty, 0);

  if (warp == 0) {
    if (lane == 0) { // TMA producer, both CTAs
      int g = 0;
      for (int u = pair; u < args.units_total && !*abort_flag; u += pairs) {
        int tile, kb0, kb1, m0, n0, z;
        unit(u, tile, kb0, kb1);
        locate(tile, m0, n0, z);
        if (leader && args.wave_count && u >= pairs && u < args.full_units) { // bounded, never fails
          const int wave = u / pairs, members = min(pairs, args.full_units - wave * pairs);
          int *count = args.wave_count + wave;
          atomicAdd(count, 1);
          const unsigned long long t0 = global_ns();
          while (*reinterpret_cast<volatile int *>(count) < members &&
                 global_ns() - t0 < static_cast<unsigned long long>(args.wave_wait_ns))
            __nanosleep(256);
        }
        const int a_y = z * args.a_rows + m0 + int(rank) * PAIR_HALF;
        const int b_y = z * args.b_rows + n0 + int(rank) * PAIR_HALF;
        for (int kb = kb0; kb < kb1; ++kb, ++g) {
          const int s = g % S;
          if (g >= S && !mbar_wait(&empty[s], ((g / S) - 1) & 1)) {
            atomicExch(args.status, STATUS_TIMEOUT_PRODUCER);
            *abort_flag = 1;
          }
          if (*abort_flag)
            break;
          uint8_t *stage = smem + s * PAIR_STAGE;
          const uint32_t bar = full0 + uint32_t(s) * 8u;
          if (RAW) { // this CTA's raw rows of A, then both CTAs' B halves on CTA 0's barrier
            mbar_expect_tx(&raw_full[s], PAIR_A_BYTES);
            tma_load_3d(stage, &a_hi, &raw_full[s], kb * TK, m0 + int(rank) * PAIR_HALF, z);
            if (leader)
              mbar_expect_tx(&full[s], 2 * 2 * PAIR_B_BYTES);
          } else {
            if (leader)
              mbar_expect_tx(&full[s], 2 * PAIR_STAGE);
            tma_load_2d_pair(stage, &a_hi, bar, kb * TK, a_y);
            tma_load_2d_pair(stage + PAIR_A_BYTES, &a_lo, bar, kb * TK, a_y);
          }
          tma_load_2d_pair(stage + 2 * PAIR_A_BYTES, &b_hi, bar, kb * TK, b_y);
          tma_load_2d_pair(stage + 2 * PAIR_A_BYTES + PAIR_B_BYTES, &b_lo, bar, kb * TK, b_y);
          *issued = g + 1;
        }
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) { // MMA issuer for the pair
      const uint32_t empty1 = in_cta(empty, 1), tmem_full1 = in_cta(tmem_full, 1);
      const uint32_t empty0 = in_cta(empty, 0), tmem_full0 = in_cta(tmem_full, 0);
      int g = 0, j = 0;
      for (int u = pair; u < args.units_total && !*abort_flag; u += pairs, ++j) {
        int tile, kb0, kb1;
        unit(u, tile, kb0, kb1);
        const int b = j & 1;
        if (j >= 2 && !mbar_wait(&tmem_empty[b], ((j >> 1) - 1) & 1)) {
          atomicExch(args.status, STATUS_TIMEOUT_MMA);
          *abort_flag = 1;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t acc = tmem + uint32_t(b) * PAIR_COLUMNS;
        for (int kb = kb0; kb < kb1; ++kb, ++g) {
          const int s = g % S;
          if (!mbar_wait(&full[s], (g / S) & 1) || (RAW && !mbar_wait(&converted[s], (g / S) & 1))) {
            atomicExch(args.status, STATUS_TIMEOUT_MMA);
            *abort_flag = 1;
            break;
          }
          *consumed = g + 1;
          if (*abort_flag)
            break;
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t stage = smem_u32(smem + s * PAIR_STAGE);
#pragma unroll
          for (int kk = 0; kk < TK / 8; ++kk) {
            const uint32_t step = kk * 32;
            const uint64_t ah = desc_k_sw64(stage + step), al = desc_k_sw64(stage + PAIR_A_BYTES + step);
            const uint64_t bh = desc_k_sw64(stage + 2 * PAIR_A_BYTES + step);
            const uint64_t bl = desc_k_sw64(stage + 2 * PAIR_A_BYTES + PAIR_B_BYTES + step);
            mma_tf32_pair(acc, ah, bh, (kb > kb0 || kk > 0) ? 1u : 0u);
            mma_tf32_pair(acc, ah, bl, 1u);
            mma_tf32_pair(acc, al, bh, 1u);
          }
          mma_commit_pair(empty0 + uint32_t(s) * 8u);
          mma_commit_pair(empty1 + uint32_t(s) * 8u);
        }
        if (*abort_flag)
          break;
        mma_commit_pair(tmem_full0 + uint32_t(b) * 8u);
        mma_commit_pair(tmem_full1 + uint32_t(b) * 8u);
      }
      // Fires once every MMA issued above has finished (both CTAs' TMEM quiet).
      mma_commit_pair(in_cta(drained, 0));
    }
  } else if (warp >= 2 + EW) { // RAW converter warps (the last four) of both CTAs
    const int t = threadIdx.x - PairShape<EW>::THREADS_PLAIN;
    const uint32_t converted0 = in_cta(converted, 0);
    int g = 0;
    for (int u = pair; u < args.units_total && !*abort_flag; u += pairs) {
      int tile, kb0, kb1;
      unit(u, tile, kb0, kb1);
      for (int kb = kb0; kb < kb1; ++kb, ++g) {
        const int s = g % S;
        if (!mbar_wait(&raw_full[s], (g / S) & 1)) {
          atomicExch(args.status, STATUS_TIMEOUT_CONVERT);
          *abort_flag = 1;
        }
        if (*abort_flag)
          break;
        float4 *hi = reinterpret_cast<float4 *>(smem + s * PAIR_STAGE);
        float4 *lo = reinterpret_cast<float4 *>(smem + s * PAIR_STAGE + PAIR_A_BYTES);
        // Same swizzle in both boxes: the pair is formed position by position.
#pragma unroll
        for (int i = 0; i < PAIR_A_BYTES / 16 / 128; ++i) {
          const float4 v = hi[t + 128 * i];
          const float4 h = tf32_hi(v);
          lo[t + 128 * i] = tf32_hi(make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w));
          hi[t + 128 * i] = h;
          if (args.nonfinite && any_inf(h))
            *args.nonfinite = args.epoch;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); // visible to the tensor cores
        __syncwarp();
        if (lane == 0)
          arrive_at(converted0 + uint32_t(s) * 8u);
      }
    }
  } else { // epilogue warps of both CTAs: TMEM lanes 32*(warp % 4) .., column part (warp - 2) / 4
    const int sub = warp % 4, part = (warp - 2) / 4;
    int j = 0;
    for (int u = pair; u < args.units_total; u += pairs, ++j) {
      int tile, kb0, kb1;
      unit(u, tile, kb0, kb1);
      const int b = j & 1;
      bool ready = mbar_try_wait(&tmem_full[b], (j >> 1) & 1);
      const long long start = clock64(), budget = WAIT_CYCLES + 100000ll * args.k_blocks;
      while (!ready && !*abort_flag && clock64() - start < budget)
        ready = mbar_try_wait(&tmem_full[b], (j >> 1) & 1);
      if (!ready || *abort_flag) {
        if (!ready && !*abort_flag)
          atomicExch(args.status, STATUS_TIMEOUT_EPILOGUE);
        *abort_flag = 1;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      int m0, n0, z;
      locate(tile, m0, n0, z);
      // Whole tiles go to C; the k-range parts of split tiles to their own 256 x 256
      // partial tile (row stride 256), all of it written.
      const bool whole = u < args.full_units;
      float *const c_base = whole ? args.c + int64_t(z) * args.c_batch
                                  : args.partials + int64_t(u - args.full_units) * (PAIR_M * PAIR_N);
      const int64_t ldc = whole ? args.ldc : PAIR_N, m_lim = whole ? args.m : PAIR_M, n_lim = whole ? args.n : PAIR_N;
      const int64_t row0 = (whole ? int64_t(m0) : 0) + int64_t(rank) * PAIR_HALF + 32 * sub; // this warp's rows
      const int64_t col0 = whole ? int64_t(n0) : 0;
      const int64_t left = m_lim - row0;
      const int rows_here = left >= 32 ? 32 : (left > 0 ? int(left) : 0);
      float *tile_s = epi_tiles + (warp - 2) * EPI_STAGE_FLOATS;
      const uint32_t acc = tmem + uint32_t(b) * PAIR_COLUMNS + (uint32_t(32 * sub) << 16);
      const bool vec_c = (ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(c_base) & 15u) == 0);
      constexpr int PART_COLUMNS = PAIR_N / PairShape<EW>::PARTS;
#pragma unroll 1
      for (int col = part * PART_COLUMNS; col < (part + 1) * PART_COLUMNS; col += 16) {
        float v[16];
        tmem_load_16(acc + uint32_t(col), v); // thread = row 32*sub + lane, 16 columns
        const int64_t first = col0 + col;
        if (first >= n_lim)
          break;
        if (whole && (args.bias || args.activation)) {
#pragma unroll
          for (int q = 0; q < 16; ++q)
            if (first + q < n_lim)
              v[q] = bias_activate(v[q], args.bias, first + q, args.activation);
        }
#pragma unroll
        for (int q = 0; q < 16; q += 4)
          *reinterpret_cast<float4 *>(&tile_s[stage_index(lane, q)]) =
              make_float4(v[q], v[q + 1], v[q + 2], v[q + 3]);
        __syncwarp();
        if (vec_c && rows_here == 32 && first + 15 < n_lim) {
          const int r_in = 2 * (lane >> 3) + ((lane & 7) >> 2), c4 = 4 * (lane & 3);
          float4 w[4];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            w[i] = *reinterpret_cast<const float4 *>(&tile_s[stage_index(8 * i + r_in, c4)]);
          float *cptr = c_base + (row0 + r_in) * ldc + first + c4;
#pragma unroll
          for (int i = 0; i < 4; ++i)
            *reinterpret_cast<float4 *>(cptr + int64_t(8 * i) * ldc) = w[i];
        } else {
          const int64_t column = first + (lane & 15);
          if (column < n_lim) {
            float *cptr = c_base + row0 * ldc + column;
            for (int r = lane >> 4; r < rows_here; r += 2)
              cptr[r * ldc] = tile_s[stage_index(r, lane & 15)];
          }
        }
        __syncwarp();
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0)
        arrive_at(tmem_empty0 + uint32_t(b) * 8u);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (*abort_flag) {
      // Copies requested but never consumed must land before shared memory is
      // released: CTA 0 waits (bounded) for those phases; CTA 1, whose copies complete
      // on CTA 0's barriers, waits a fixed ~1 ms for its own.
      if (leader) {
        for (int g = *consumed; g < *issued; ++g)
          (void)mbar_wait(&full[g % S], (g / S) & 1);
      }
      const long long start = clock64(); // copies that complete on another CTA's barrier
      while (clock64() - start < 2000000ll) {
      }
    }
    if (leader)
      (void)mbar_wait(drained, 0); // bounded: every MMA of the pair has finished
  }
  __syncthreads();
  cluster_sync_all();
  if (warp == 1) {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * PAIR_COLUMNS)
                 : "memory");
  }
}

// C of every split tile = its partial tiles added in k order: one thread per four
// columns of a tile row (128-bit loads), 1024 / BN rows per 256-thread block.
// TMR: rows of a tile (128 for the one-SM kernel, 256 for the CTA pair).
template <int BN, int TMR = TM> __global__ void __launch_bounds__(256) split_fixup(const TileArgs args) {
  constexpr int PER_ROW = BN / 4, ROWS = 256 / PER_ROW;
  const int t = blockIdx.y;                                     // remaining tile
  const int i = blockIdx.x * ROWS + threadIdx.x / PER_ROW;      // row in the tile
  const int j = 4 * (threadIdx.x % PER_ROW);                    // first of four columns
  const int tile = args.full_units + t;
  const int per_batch = args.tiles_per_batch ? args.tiles_per_batch : args.tiles_m * args.tiles_n;
  const int z = tile / per_batch, id = tile % per_batch;
  int64_t row, col;
  if (args.col_group > 0) { // the CTA pair's column-group raster
    const int group = args.col_group, per_group = group * args.tiles_m;
    const int first_n = (id / per_group) * group;
    const int cols_in_group = min(group, args.tiles_n - first_n);
    col = int64_t(first_n + (id % per_group) % cols_in_group) * BN + j;
    row = int64_t((id % per_group) / cols_in_group) * TMR + i;
  } else {
    const int group = args.group, per_group = group * args.tiles_n;
    const int first_m = (id / per_group) * group;
    const int rows_in_group = min(group, args.tiles_m - first_m);
    row = int64_t(first_m + (id % per_group) % rows_in_group) * TMR + i;
    col = int64_t((id % per_group) / rows_in_group) * BN + j;
  }
  if (row >= args.m || col >= args.n)
    return;
  const float4 *p =
      reinterpret_cast<const float4 *>(args.partials + int64_t(t) * args.split * (TMR * BN) + i * BN + j);
  float4 s4 = p[0];
  for (int q = 1; q < args.split; ++q) {
    const float4 v = p[int64_t(q) * (TMR * BN / 4)];
    s4 = make_float4(__fadd_rn(s4.x, v.x), __fadd_rn(s4.y, v.y), __fadd_rn(s4.z, v.z), __fadd_rn(s4.w, v.w));
  }
  const float sum[4] = {s4.x, s4.y, s4.z, s4.w};
  float *const c = args.c + int64_t(z) * args.c_batch;
  if (args.transposed) { // D[row][col] is C[col][row]
    for (int e = 0; e < 4 && col + e < args.n; ++e)
      c[(col + e) * args.ldc + row] = bias_activate(sum[e], args.bias, row, args.activation);
    return;
  }
  float y[4];
#pragma unroll
  for (int e = 0; e < 4; ++e)
    y[e] = bias_activate(sum[e], args.bias, col + e < args.n ? col + e : col, args.activation);
  float *dst = c + row * args.ldc + col;
  if (col + 3 < args.n && args.ldc % 4 == 0 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
    *reinterpret_cast<float4 *>(dst) = make_float4(y[0], y[1], y[2], y[3]);
  } else {
    for (int e = 0; e < 4 && col + e < args.n; ++e)
      dst[e] = y[e];
  }
}

// ---- host side ----
using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *,
                                 CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                 CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
  static EncodeTiled fn = [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      cudaGetLastError();
      return static_cast<EncodeTiled>(nullptr);
    }
    return reinterpret_cast<EncodeTiled>(p);
  }();
  return fn;
}

bool make_map(CUtensorMap *map, const float *base, int64_t rows_pad, int64_t k_pad, uint32_t box_rows) {
  const EncodeTiled encode = encoder();
  if (!encode)
    return false;
  const cuuint64_t dims[2] = {cuuint64_t(k_pad), cuuint64_t(rows_pad)};
  const cuuint64_t strides[1] = {cuuint64_t(k_pad) * 4};
  const cuuint32_t box[2] = {TK, box_rows};
  const cuuint32_t element[2] = {1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(base), dims, strides, box, element,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Raw A as a [batch][m][k] box source (k contiguous, row stride lda, matrix stride
// sa, all in elements): boxes of box_rows rows x 16 k, zero outside the matrix, so
// the k tail and the rows past m read as the zero padding of the split path.
bool make_raw_map(CUtensorMap *map, const float *a, int64_t batch, int64_t m, int64_t k, int64_t lda, int64_t sa,
                  uint32_t box_rows) {
  const EncodeTiled encode = encoder();
  if (!encode)
    return false;
  const cuuint64_t dims[3] = {cuuint64_t(k), cuuint64_t(m), cuuint64_t(batch)};
  const cuuint64_t strides[2] = {cuuint64_t(lda) * 4, cuuint64_t(sa) * 4};
  const cuuint32_t box[3] = {TK, box_rows, 1};
  const cuuint32_t element[3] = {1, 1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(a), dims, strides, box, element,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int64_t round_up(int64_t v, int64_t to) { return (v + to - 1) / to * to; }

// Shared-memory limit of one persistent-kernel form, set once per device (the
// attribute belongs to the device's context).
template <int BN, int RAW, bool TOUT, int MR = TM> bool configure_persistent(int device) {
  static bool configured[64] = {};
  if (device < 0 || device >= 64)
    return false;
  if (!configured[device]) {
    if (cudaFuncSetAttribute(gemm_tf32x3_persistent<BN, RAW, TOUT, MR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Tile<BN, MR>::SMEM) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    configured[device] = true;
  }
  return true;
}

// Work units of the persistent kernel. With G = SM count, tiles = R*G + r: when the
// last (or only) round would keep at most half of the SMs busy, its r tiles are cut
// into s = min(G / r, 4) k-ranges so that round ends about s times sooner.
struct UnitPlan {
  int ctas, full_units, split, units, remaining;
  size_t partial_bytes;
};
UnitPlan plan_units(int64_t tiles, int sm_count, int k_blocks, int bn, int tile_rows = TM) {
  UnitPlan p{};
  const int64_t g = std::max(1, sm_count);
  const int64_t r = tiles % g;
  p.split = 1;
  if (r > 0 && 2 * r <= g)
    p.split = int(std::min<int64_t>({g / r, 4, k_blocks / 2}));
  if (p.split < 2)
    p.split = 1;
  p.remaining = p.split > 1 ? int(r) : 0;
  p.full_units = int(tiles - p.remaining);
  p.units = p.full_units + p.remaining * p.split;
  p.ctas = int(std::min<int64_t>(p.units, g));
  p.partial_bytes = size_t(p.remaining) * p.split * tile_rows * bn * sizeof(float);
  return p;
}

template <int BN, int RAW, bool TOUT, int MR = TM>
void launch_persistent(Launch &L, const CUtensorMap (&maps)[4], TileArgs t, int64_t tiles, const UnitPlan &plan,
                       float *partials) {
  t.tiles_total = int(tiles);
  t.units_total = plan.units;
  t.full_units = plan.full_units;
  t.split = plan.split;
  t.partials = partials;
  gemm_tf32x3_persistent<BN, RAW, TOUT, MR><<<uint32_t(plan.ctas), RAW ? THREADS_RAW_ONE : THREADS_PLAIN,
                                              Tile<BN, MR>::SMEM, L.stream>>>(maps[0], maps[1], maps[2], maps[3], t);
  if (plan.remaining) {
    split_fixup<BN, MR><<<dim3(MR / (1024 / BN), uint32_t(plan.remaining)), 256, 0, L.stream>>>(t);
    ++L.kernels;
  }
}

// CTA pairs the device can hold at once with the pair kernel's shared memory (the
// persistent grid), set up once per device; 0 when the pair kernel cannot run.
template <bool RAW, int EW> int pair_capacity(int device) {
  static int capacity[64] = {};
  static bool known[64] = {};
  if (device < 0 || device >= 64)
    return 0;
  if (!known[device]) {
    known[device] = true;
    if (cudaFuncSetAttribute(gemm_tf32x3_pair<RAW, EW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             PairShape<EW>::SMEM) != cudaSuccess) {
      cudaGetLastError();
      return 0;
    }
    cudaLaunchConfig_t config = {};
    config.gridDim = dim3(2, 1, 1);
    config.blockDim = dim3(RAW ? PairShape<EW>::THREADS_RAW : PairShape<EW>::THREADS_PLAIN, 1, 1);
    config.dynamicSmemBytes = PairShape<EW>::SMEM;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, gemm_tf32x3_pair<RAW, EW>, &config) != cudaSuccess) {
      cudaGetLastError();
      clusters = 0;
    }
    capacity[device] = clusters;
  }
  return capacity[device];
}

// Epilogue warps per CTA of the pair: 16 when the epilogue adds a bias or applies an
// activation, else 8.
int pair_epilogue_warps(const TileArgs &t) { return t.bias || t.activation ? 16 : 8; }

void launch_pair(Launch &L, bool raw, const CUtensorMap (&maps)[4], TileArgs t, int64_t tiles, const UnitPlan &plan,
                 float *partials) {
  t.tiles_total = int(tiles);
  t.units_total = plan.units;
  t.full_units = plan.full_units;
  t.split = plan.split;
  t.partials = partials;
  const uint32_t grid = uint32_t(2 * plan.ctas);
  if (pair_epilogue_warps(t) == 16) {
    using P = PairShape<16>;
    if (raw)
      gemm_tf32x3_pair<true, 16><<<grid, P::THREADS_RAW, P::SMEM, L.stream>>>(maps[0], maps[1], maps[2], maps[3], t);
    else
      gemm_tf32x3_pair<false, 16><<<grid, P::THREADS_PLAIN, P::SMEM, L.stream>>>(maps[0], maps[1], maps[2], maps[3], t);
  } else {
    using P = PairShape<8>;
    if (raw)
      gemm_tf32x3_pair<true, 8><<<grid, P::THREADS_RAW, P::SMEM, L.stream>>>(maps[0], maps[1], maps[2], maps[3], t);
    else
      gemm_tf32x3_pair<false, 8><<<grid, P::THREADS_PLAIN, P::SMEM, L.stream>>>(maps[0], maps[1], maps[2], maps[3], t);
  }
  if (plan.remaining) {
    split_fixup<PAIR_N, PAIR_M><<<dim3(PAIR_M / (1024 / PAIR_N), uint32_t(plan.remaining)), 256, 0, L.stream>>>(t);
    ++L.kernels;
  }
}

// The CTA-pair kernel serves the wide (BN = 256) forms; PARALYN_GEMM_PAIR=0 selects
// the one-SM kernel instead. Where the one-SM kernel would convert A in shared memory
// (A stored [m][k] in 16-byte rows, at most two column tiles) the pair does too
// (PARALYN_GEMM_PAIR_RAW=0: split A first).
bool env_flag(const char *name) {
  const char *v = std::getenv(name);
  return !(v && v[0] == '0');
}
bool pair_enabled() {
  static const bool enabled = env_flag("PARALYN_GEMM_PAIR");
  return enabled;
}
bool pair_raw_enabled() {
  static const bool enabled = env_flag("PARALYN_GEMM_PAIR_RAW");
  return enabled;
}
// Deep products (k >= 2048) on CTA pairs walk the rows of groups of column tiles:
// a round of 74 pairs then covers about 9 tile-rows x 8 column tiles, against 4.6
// tile-rows x all 16 column tiles of W for two-row groups, and the chain's GEMM read
// 8.5 GB instead of 10.5 (rounds aligned) and ran 1 % faster under the power cap.
// PARALYN_GEMM_COL_GROUP (1..64) overrides the 8 column tiles; 0 keeps row groups.
int pair_col_group() {
  static const int g = [] {
    const char *v = std::getenv("PARALYN_GEMM_COL_GROUP");
    const int c = v ? std::atoi(v) : 8;
    return c >= 0 && c <= 64 ? c : 8;
  }();
  return g;
}
// Longest wait (ns) of the CTA pairs' round alignment: PARALYN_GEMM_WAVE_WAIT_US
// (microseconds, at most 10000; 0 turns the alignment off), default 50.
long long pair_wave_wait_ns() {
  static const long long ns = [] {
    const char *v = std::getenv("PARALYN_GEMM_WAVE_WAIT_US");
    const long long us = v ? std::atoll(v) : 50;
    return us > 0 && us <= 10000 ? us * 1000 : 0;
  }();
  return ns;
}
// The transposed form of a C with at most 64 columns runs 64-row tiles (M = 64 MMAs);
// PARALYN_GEMM_NARROW=0 keeps it on 128-row tiles, half of them zero padding.
bool narrow_enabled() {
  static const bool enabled = env_flag("PARALYN_GEMM_NARROW");
  return enabled;
}
// Tile rows per raster group of the pair kernel: the A rows of one group (256 rows
// each) are re-read by every column tile while B's tiles stream past them, so they
// should stay in L2 beside the B tiles in use. Two tile rows (16 MB of split A at
// k = 4096) measured best on the 65536 x 4096 x 4096 chain (1, 2, 3, 4, 8 and 16
// tried); PARALYN_GEMM_RASTER_GROUP (1..64) overrides the default.
int pair_group(bool raw) {
  static const int forced = [] {
    const char *v = std::getenv("PARALYN_GEMM_RASTER_GROUP");
    const int g = v ? std::atoi(v) : 0;
    return g >= 1 && g <= 64 ? g : 0;
  }();
  return forced ? forced : (raw ? 8 : 2);
}

// ---- prepared right-hand operands (layout in prepared.hpp)

// Header of a prepared operand, written before its split pass (which may set the
// infinity mark).
__global__ void prepared_init(prepared::Header *h, uint64_t k, uint64_t n, uint64_t k_pad, uint64_t n_pad) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    h->magic = prepared::kMagic;
    h->version = prepared::kVersion;
    h->k = k;
    h->n = n;
    h->k_pad = k_pad;
    h->n_pad = n_pad;
    h->nonfinite = 0;
  }
}

// A product given a prepared operand: its header must describe (k, n), else the
// command fails (status_prepared_mismatch) and C is undefined. The operand's
// infinity mark is copied to the command's watch word (AUTO mode), so that the
// guarded FFMA recomputation runs as it would after splitting B.
__global__ void prepared_check(const prepared::Header *h, uint64_t k, uint64_t n, int *status,
                               unsigned long long *nonfinite, unsigned long long epoch) {
  if (threadIdx.x != 0 || blockIdx.x != 0)
    return;
  if (h->magic != prepared::kMagic || h->version != prepared::kVersion || h->k != k || h->n != n) {
    if (status)
      atomicExch(status, prepared::status_mismatch);
    return;
  }
  if (nonfinite && h->nonfinite)
    *nonfinite = epoch;
}

// B stored [k][n] copied to the prepared [k][n] copy (count elements, 128-bit when
// both sides are 16-byte aligned).
__global__ void __launch_bounds__(256) prepared_copy(const float *__restrict__ b, float *__restrict__ raw,
                                                     uint64_t count, int vec) {
  const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
  const uint64_t first = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (vec) {
    for (uint64_t i = first; i < count / 4; i += stride)
      reinterpret_cast<float4 *>(raw)[i] = reinterpret_cast<const float4 *>(b)[i];
    for (uint64_t i = count / 4 * 4 + first; i < count; i += stride)
      raw[i] = b[i];
  } else {
    for (uint64_t i = first; i < count; i += stride)
      raw[i] = b[i];
  }
}

// B stored [n][k] (ldb = k) transposed into the prepared [k][n] copy: 32 x 32 tiles
// through shared memory (one padding column keeps the column reads conflict-free).
__global__ void __launch_bounds__(256) prepared_transpose(const float *__restrict__ b, float *__restrict__ raw,
                                                          int64_t k, int64_t n) {
  __shared__ float tile[32][33];
  const int64_t n0 = int64_t(blockIdx.y) * 32, k0 = int64_t(blockIdx.x) * 32;
  const int tx = threadIdx.x % 32, ty = threadIdx.x / 32; // 8 rows of 32
  for (int r = ty; r < 32; r += 8) {
    const int64_t row = n0 + r, col = k0 + tx;
    if (row < n && col < k)
      tile[r][tx] = b[row * k + col];
  }
  __syncthreads();
  for (int r = ty; r < 32; r += 8) {
    const int64_t row = k0 + r, col = n0 + tx; // raw[row][col] = B^T
    if (row < k && col < n)
      raw[row * n + col] = tile[tx][r];
  }
}

// The kernel forms: N tile width x (which operand, if any, is split in shared
// memory), plus the transposed form for narrow C (256 columns, raw B, D = C^T), with
// 64-row tiles (M = 64 MMAs) when C has at most 64 columns.
enum class Form { n64, n64_raw_a, n128, n128_raw_a, n256, n256_raw_a, transposed, transposed64 };
Form form_of(int bn, bool raw_a) {
  if (bn == 64)
    return raw_a ? Form::n64_raw_a : Form::n64;
  if (bn == 128)
    return raw_a ? Form::n128_raw_a : Form::n128;
  return raw_a ? Form::n256_raw_a : Form::n256;
}
bool configure_form(Form f, int device) {
  switch (f) {
  case Form::n64: return configure_persistent<64, RAW_NONE, false>(device);
  case Form::n64_raw_a: return configure_persistent<64, RAW_A, false>(device);
  case Form::n128: return configure_persistent<128, RAW_NONE, false>(device);
  case Form::n128_raw_a: return configure_persistent<128, RAW_A, false>(device);
  case Form::n256: return configure_persistent<256, RAW_NONE, false>(device);
  case Form::n256_raw_a: return configure_persistent<256, RAW_A, false>(device);
  case Form::transposed: return configure_persistent<256, RAW_B, true>(device);
  case Form::transposed64: return configure_persistent<256, RAW_B, true, 64>(device);
  }
  return false;
}
void launch_form(Form f, Launch &L, const CUtensorMap (&maps)[4], const TileArgs &t, int64_t tiles,
                 const UnitPlan &plan, float *partials) {
  switch (f) {
  case Form::n64: return launch_persistent<64, RAW_NONE, false>(L, maps, t, tiles, plan, partials);
  case Form::n64_raw_a: return launch_persistent<64, RAW_A, false>(L, maps, t, tiles, plan, partials);
  case Form::n128: return launch_persistent<128, RAW_NONE, false>(L, maps, t, tiles, plan, partials);
  case Form::n128_raw_a: return launch_persistent<128, RAW_A, false>(L, maps, t, tiles, plan, partials);
  case Form::n256: return launch_persistent<256, RAW_NONE, false>(L, maps, t, tiles, plan, partials);
  case Form::n256_raw_a: return launch_persistent<256, RAW_A, false>(L, maps, t, tiles, plan, partials);
  case Form::transposed: return launch_persistent<256, RAW_B, true>(L, maps, t, tiles, plan, partials);
  case Form::transposed64: return launch_persistent<256, RAW_B, true, 64>(L, maps, t, tiles, plan, partials);
  }
}

// N tile width for n columns: the narrowest of 64 / 128 / 256 that holds them, else 256.
int tile_width(int64_t n) { return n <= 64 ? 64 : (n <= 128 ? 128 : 256); }

// Raw boxes of A need A stored [m][k] (k contiguous) with 16-byte aligned rows and
// non-overlapping matrices (sa = matrix stride).
bool raw_a_layout(const float *a, bool ta, int64_t m, int64_t lda, int64_t sa) {
  return !ta && (reinterpret_cast<uintptr_t>(a) & 15u) == 0 && lda % 4 == 0 && sa % 4 == 0 && sa >= m * lda &&
         lda <= (int64_t(1) << 36) && sa <= (int64_t(1) << 36);
}

// Plans and enqueues C[z] = op(A[z]) op(B[z]) for z < batch (see the launchers below).
//  * n <= 128 and A laid out for raw boxes: the transposed form. D = C^T =
//    op(B)^T op(A)^T with op(B)^T split into 128-row tiles (n rows, zero padded)
//    and A's rows as the 256-wide side, converted in shared memory.
//  * otherwise: 128 x BN tiles of C; A converted in shared memory when at most two
//    column tiles re-read it, else split by the split pass.
//  * prep (one matrix, B stored [k][n] as far as the caller is concerned): B's TF32
//    pair comes from the prepared operand instead of a split pass over B.
bool launch_tf32x3(Launch &L, const float *a, const float *b, float *c, int64_t batch, int64_t m, int64_t n,
                   int64_t k, int64_t lda, bool ta, int64_t sa, int64_t ldb, bool tb, int64_t sb, int64_t ldc,
                   int64_t sc, const float *bias, uint32_t activation, NonFiniteFlag *watch,
                   const PreparedB *prep = nullptr) {
  if (!encoder() || !L.workspace)
    return false;
  if (prep && (batch != 1 || uint64_t(k) != prep->k || uint64_t(n) < 1 || uint64_t(n) > prep->n))
    return false;
  if (batch == 1)
    sa = m * lda;
  const bool raw_a = raw_a_layout(a, ta, m, lda, sa);
  const bool transposed = raw_a && n <= 128;
  // The kernel's D [dm, dn]: C itself, or C^T in the transposed form.
  const int64_t dm = transposed ? n : m, dn = transposed ? m : n;
  const bool narrow = transposed && dm <= 64 && narrow_enabled(); // M = 64 tiles
  const int bn = transposed ? 256 : tile_width(n);
  const int64_t k_pad = round_up(k, 32), dn_pad = round_up(dn, bn), tiles_n = dn_pad / bn;
  Form form = transposed ? (narrow ? Form::transposed64 : Form::transposed) : form_of(bn, raw_a && tiles_n <= 2);
  // Wide products run on CTA pairs (256 x 256 tiles), reading A raw when its layout
  // allows (then no split pass runs over A).
  const bool wide = (form == Form::n256 || form == Form::n256_raw_a) && dm >= PAIR_M && pair_enabled();
  // Converting A in shared memory repeats its TF32 conversions once per column tile,
  // so (as for the one-SM kernel) it pays only while few column tiles re-read A.
  const bool pair_raw = wide && form == Form::n256_raw_a && pair_raw_enabled();
  // The persistent grid: clusters the device holds at once with the launch's shared
  // memory (the epilogue's staging grows with its warps).
  const bool epilogue16 = bias || activation;
  const int pairs = !wide ? 0
                    : pair_raw ? (epilogue16 ? pair_capacity<true, 16>(L.device) : pair_capacity<true, 8>(L.device))
                               : (epilogue16 ? pair_capacity<false, 16>(L.device) : pair_capacity<false, 8>(L.device));
  if (pairs)
    form = pair_raw ? Form::n256_raw_a : Form::n256;
  const bool a_split = !transposed && (form == Form::n64 || form == Form::n128 || form == Form::n256);
  const int64_t m_tile = pairs ? PAIR_M : (narrow ? 64 : TM);
  const int64_t dm_pad = round_up(dm, m_tile), tiles_m = dm_pad / m_tile, batch_b = sb ? batch : 1;
  // Grid limits of the split passes (rows / 32 in grid.y) and 32-bit TMA row
  // coordinates of the split operands; a raw operand is addressed by its own map.
  const int64_t b_rows = transposed ? dm_pad : dn_pad;
  if (tiles_m * tiles_n * batch > INT32_MAX || k_pad / TK > INT32_MAX || b_rows / 32 > 65535 ||
      batch_b * b_rows > INT32_MAX || (a_split && (dm_pad / 32 > 65535 || batch * dm_pad > INT32_MAX)) ||
      dm > INT32_MAX || dn > INT32_MAX)
    return false;
  const UnitPlan plan = pairs ? plan_units(tiles_m * tiles_n * batch, pairs, int(k_pad / TK), bn, PAIR_M)
                              : plan_units(tiles_m * tiles_n * batch, L.sm_count, int(k_pad / TK), bn, int(m_tile));
  // Split operands in the workspace: A's pair [batch * m_pad][k_pad] unless A is
  // converted in shared memory; B's pair [batch_b * rows][k_pad], rows = n_pad
  // (or, transposed, n padded to the tile's 128 or 64 rows: the kernel's M side).
  const int64_t a_rows = a_split ? batch * dm_pad : 0;
  const int64_t b_rows_each = transposed ? dm_pad : dn_pad;
  // A prepared B holds its pair with n_pad (>= b_rows_each) rows of k_pad.
  const size_t split_bytes = size_t(8) * size_t(k_pad) * size_t(a_rows + (prep ? 0 : batch_b * b_rows_each));
  // After the split operands and the partial tiles: the non-finite flag word (8 bytes;
  // both regions are multiples of 8 bytes).
  // Then, for the CTA pairs' round alignment, one counter per round of whole tiles.
  // Deep products only (k >= 2048: a round then lasts ~70 us or more and reads its
  // operands from DRAM): on the 65536 x 4096 x 4096 chain it cut the GEMM's DRAM
  // traffic from 17.6 to 11.4 GB a launch, which under the power cap bought SM clock
  // (227 -> 237 TFLOP/s); shallow products with short rounds (k = 128, k = 1024) lost
  // 2-7 % to the waits.
  const bool deep = pairs && k_pad >= 2048;
  const bool align_waves = deep && pair_wave_wait_ns();
  const int64_t wave_slots = align_waves ? (plan.full_units + pairs - 1) / pairs + 1 : 0;
  const size_t bytes = split_bytes + plan.partial_bytes + (watch || wave_slots ? 8 : 0) + size_t(wave_slots) * 4;
  if (L.dry_run)
    return true;
  auto *scratch = static_cast<float *>(L.workspace(L.workspace_owner, bytes));
  if (!scratch)
    return false;
  float *partials = scratch + split_bytes / sizeof(float);
  unsigned long long *flag = nullptr, epoch = 0;
  if (watch) {
    static std::atomic<unsigned long long> epochs{1};
    flag = reinterpret_cast<unsigned long long *>(reinterpret_cast<char *>(scratch) + split_bytes +
                                                  plan.partial_bytes);
    epoch = epochs.fetch_add(1, std::memory_order_relaxed);
    watch->word = flag;
    watch->epoch = epoch;
  }
  float *ahi = scratch, *alo = ahi + a_rows * k_pad;
  const float *bhi = prep ? prep->hi : alo + a_rows * k_pad;
  const float *blo = prep ? prep->lo : bhi + batch_b * b_rows_each * k_pad;
  CUtensorMap maps[4];
  if (transposed) { // kernel A = op(B)^T pair, kernel B = raw rows of A
    if (!make_map(&maps[0], bhi, batch_b * dm_pad, k_pad, uint32_t(m_tile)) ||
        !make_map(&maps[1], blo, batch_b * dm_pad, k_pad, uint32_t(m_tile)) ||
        !make_raw_map(&maps[2], a, batch, m, k, lda, sa, uint32_t(bn)))
      return false;
    maps[3] = maps[2]; // unused
  } else {
    if (a_split) {
      if (!make_map(&maps[0], ahi, batch * dm_pad, k_pad, TM) || !make_map(&maps[1], alo, batch * dm_pad, k_pad, TM))
        return false;
    } else {
      if (!make_raw_map(&maps[0], a, batch, m, k, lda, sa, TM))
        return false;
      maps[1] = maps[0]; // unused
    }
    const uint32_t b_box = pairs ? PAIR_HALF : uint32_t(bn); // a CTA of a pair holds half of B's rows
    if (!make_map(&maps[2], bhi, batch_b * dn_pad, k_pad, b_box) || !make_map(&maps[3], blo, batch_b * dn_pad, k_pad, b_box))
      return false;
  }
  if (!pairs && !configure_form(form, L.device))
    return false;
  // op(A) [m, k] and op(B)^T [n, k]: B^T is B read transposed unless B is stored [n, k].
  // 128-bit split when the operand's rows (or columns) start on 16-byte boundaries.
  auto vec_ok = [](const float *x, int64_t ld, int64_t stride) {
    return (reinterpret_cast<uintptr_t>(x) & 15u) == 0 && ld % 4 == 0 && stride % 4 == 0;
  };
  if (a_split) {
    const dim3 grid(uint32_t(k_pad / 32), uint32_t(dm_pad / 32), uint32_t(batch));
    if (vec_ok(a, lda, batch > 1 ? sa : 0))
      split_tf32_vec<<<grid, 256, 0, L.stream>>>(a, lda, ta ? 1 : 0, m, k, ahi, alo, k_pad, sa, dm_pad, flag, epoch);
    else
      split_tf32<<<grid, 256, 0, L.stream>>>(a, lda, ta ? 1 : 0, m, k, ahi, alo, k_pad, sa, dm_pad, flag, epoch);
    ++L.kernels;
  }
  if (prep) {
    prepared_check<<<1, 32, 0, L.stream>>>(prep->header, prep->k, prep->n, L.status, flag, epoch);
    ++L.kernels;
  } else {
    float *bhi_w = const_cast<float *>(bhi), *blo_w = const_cast<float *>(blo);
    const dim3 grid(uint32_t(k_pad / 32), uint32_t(b_rows_each / 32), uint32_t(batch_b));
    if (vec_ok(b, ldb, sb))
      split_tf32_vec<<<grid, 256, 0, L.stream>>>(b, ldb, tb ? 0 : 1, n, k, bhi_w, blo_w, k_pad, sb, b_rows_each,
                                                 flag, epoch);
    else
      split_tf32<<<grid, 256, 0, L.stream>>>(b, ldb, tb ? 0 : 1, n, k, bhi_w, blo_w, k_pad, sb, b_rows_each, flag,
                                             epoch);
    ++L.kernels;
  }
  TileArgs t{c, dm, dn, ldc, int(k_pad / TK), int(tiles_m), int(tiles_n), L.status};
  if (batch > 1) {
    t.tiles_per_batch = int(tiles_m * tiles_n);
    if (transposed) {
      t.a_rows = sb ? int(dm_pad) : 0; // kernel A rows = op(B)^T of matrix z
    } else {
      t.a_rows = int(dm_pad);
      t.b_rows = sb ? int(dn_pad) : 0;
    }
    t.c_batch = sc;
  }
  t.bias = bias;
  t.activation = activation;
  t.transposed = transposed;
  t.nonfinite = flag;
  t.epoch = epoch;
  if (pairs) {
    t.group = pair_group(pair_raw);
    t.col_group = deep ? pair_col_group() : 0;
  }
  if (wave_slots) {
    t.wave_count = reinterpret_cast<int *>(reinterpret_cast<char *>(scratch) + split_bytes + plan.partial_bytes + 8);
    t.wave_wait_ns = pair_wave_wait_ns();
    if (cudaMemsetAsync(t.wave_count, 0, size_t(wave_slots) * 4, L.stream) != cudaSuccess)
      return false;
  }
  ++L.kernels;
  if (pairs)
    launch_pair(L, pair_raw, maps, t, tiles_m * tiles_n * batch, plan, partials);
  else
    launch_form(form, L, maps, t, tiles_m * tiles_n * batch, plan, partials);
  return true;
}

} // namespace

bool encode_map_2d(CUtensorMap *map, const void *base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                   uint32_t box_inner, uint32_t box_outer, bool swizzle_128b) {
  const EncodeTiled encode = encoder();
  if (!encode || row_bytes % 16 != 0 || (reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    return false;
  const cuuint64_t dims[2] = {cuuint64_t(inner), cuuint64_t(outer)};
  const cuuint64_t strides[1] = {cuuint64_t(row_bytes)};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t element[2] = {1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void *>(base), dims, strides, box, element,
                CU_TENSOR_MAP_INTERLEAVE_NONE,
                swizzle_128b ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Plans and enqueues the 3xTF32 GEMM; returns false (nothing enqueued) when the
// shape is outside what this kernel covers or scratch is unavailable.
bool launch_tf32x3_gemm(Launch &L, const float *a, const float *b, float *c, int64_t m, int64_t n, int64_t k,
                        int64_t lda, int64_t ldb, int64_t ldc, bool ta, bool tb, const float *bias,
                        uint32_t activation, NonFiniteFlag *watch, const PreparedB *prep) {
  if (k < 16 || m < 1 || n < 1)
    return false;
  if (L.matmul_mode == matmul_auto && (k < 64 || m * n < 128 * 256))
    return false;
  L.kernels = 0;
  // Bias and activation (ReLU or the tanh GELU) run in the GEMM epilogue.
  if (!launch_tf32x3(L, a, b, c, 1, m, n, k, lda, ta, 0, ldb, tb, 0, ldc, 0, bias, activation, watch, prep))
    return false;
  L.variant = "tcgen05_tf32x3";
  return true;
}

// Batched form: C[z] = op(A[z]) op(B[z]) for z < batch, matrix z of A at a + z*sa,
// of B at b + z*sb (sb = 0: one B shared by all), of C at c + z*sc (row stride
// ldc, column stride 1). Same split and GEMM kernels with a batch grid dimension
// (split) and batch-major tile numbering (GEMM); the split operands of all
// matrices are stacked row-wise, so no tile crosses a matrix boundary.
// The header check of a prepared operand before a SIMT product reads its [k][n] copy.
void launch_prepared_check(Launch &L, const PreparedB &prep) {
  prepared_check<<<1, 32, 0, L.stream>>>(prep.header, prep.k, prep.n, L.status, nullptr, 0);
  ++L.kernels;
}

// (b, prepared, k, n, transpose_b): B ([k][n], or [n][k] when transpose_b) into its
// prepared form (prepared.hpp): the header, B^T's TF32 pair (the split pass, which
// marks the header when a high part is infinite) and the [k][n] copy.
void launch_matmul_prepare(Launch &L) {
  const auto &A = L.args;
  const uint64_t k = A[2].u32(), n = A[3].u32();
  const uint32_t tb = A[4].u32();
  if (tb > 1)
    throw Failure(PR_INVALID_ARGUMENT, "Transpose flags must be 0 or 1");
  const uint64_t bytes = prepared::bytes(k, n);
  if (!bytes)
    throw Failure(PR_INVALID_ARGUMENT, "A prepared operand needs 1 <= k, n <= INT32_MAX");
  if (prepared::n_pad(n) / 32 > 65535)
    throw Failure(PR_UNSUPPORTED, "A prepared operand holds at most 2097152 columns");
  need_elements(A[0], k * n, "b");
  need_elements(A[1], bytes / 4, "prepared");
  if (reinterpret_cast<uintptr_t>(A[1].ptr) % prepared::kHeaderBytes)
    throw Failure(PR_INVALID_ARGUMENT, "The prepared tensor must start on a 256-byte boundary");
  L.variant = "prepare_tf32x3";
  if (L.dry_run)
    return;
  const float *b = static_cast<const float *>(A[0].ptr);
  char *base = static_cast<char *>(A[1].ptr);
  auto *header = reinterpret_cast<prepared::Header *>(base);
  float *raw = reinterpret_cast<float *>(base + prepared::raw_offset());
  float *hi = reinterpret_cast<float *>(base + prepared::hi_offset(k, n));
  float *lo = reinterpret_cast<float *>(base + prepared::lo_offset(k, n));
  const int64_t k_pad = int64_t(prepared::k_pad(k)), n_pad = int64_t(prepared::n_pad(n));
  const int64_t ldb = tb ? int64_t(k) : int64_t(n);
  L.kernels = 0;
  prepared_init<<<1, 32, 0, L.stream>>>(header, k, n, uint64_t(k_pad), uint64_t(n_pad));
  const dim3 grid(uint32_t(k_pad / 32), uint32_t(n_pad / 32), 1);
  if ((reinterpret_cast<uintptr_t>(b) & 15u) == 0 && ldb % 4 == 0)
    split_tf32_vec<<<grid, 256, 0, L.stream>>>(b, ldb, tb ? 0 : 1, int64_t(n), int64_t(k), hi, lo, k_pad, 0, n_pad,
                                               &header->nonfinite, 1);
  else
    split_tf32<<<grid, 256, 0, L.stream>>>(b, ldb, tb ? 0 : 1, int64_t(n), int64_t(k), hi, lo, k_pad, 0, n_pad,
                                           &header->nonfinite, 1);
  if (tb) {
    prepared_transpose<<<dim3(uint32_t((k + 31) / 32), uint32_t((n + 31) / 32)), 256, 0, L.stream>>>(
        b, raw, int64_t(k), int64_t(n));
  } else {
    const uint64_t count = k * n;
    const int64_t blocks = std::min<int64_t>(int64_t((count / 4 + 255) / 256) + 1, int64_t(std::max(1, L.sm_count)) * 8);
    prepared_copy<<<uint32_t(blocks), 256, 0, L.stream>>>(b, raw, count,
                                                          (reinterpret_cast<uintptr_t>(b) & 15u) == 0 ? 1 : 0);
  }
  L.kernels = 3;
}

bool launch_tf32x3_batched(Launch &L, const float *a, const float *b, float *c, int64_t batch, int64_t m,
                           int64_t n, int64_t k, int64_t lda, bool ta, int64_t sa, int64_t ldb, bool tb, int64_t sb,
                           int64_t ldc, int64_t sc, NonFiniteFlag *watch) {
  if (k < 16 || m < 1 || n < 1 || batch < 1 || batch > 65535)
    return false;
  if (L.matmul_mode == matmul_auto && (k < 64 || m * n * batch < 128 * 256 * 4))
    return false;
  L.kernels = 0;
  if (!launch_tf32x3(L, a, b, c, batch, m, n, k, lda, ta, sa, ldb, tb, sb, ldc, sc, nullptr, 0, watch))
    return false;
  L.variant = "batched_tcgen05_tf32x3";
  return true;
}

} // namespace pb

// ---- allocation-free variant (pr_b200_matmul_tf32x3_static_f32) ----
// Same split and GEMM kernels, with the split operands in one fixed device array
// instead of the context workspace, for callers that cannot allocate device memory.
#include "../runtime/abi_internal.hpp"
#include "paralyn/b200.h"
#include <mutex>

namespace pb {
namespace {

constexpr size_t STATIC_SCRATCH_BYTES = size_t(64) << 20;
static __device__ __align__(256) float static_scratch[STATIC_SCRATCH_BYTES / sizeof(float)];
static __device__ int32_t static_status; // timeout record when the caller passes no status word

constexpr int MAX_DEVICES = 64;
std::mutex static_setup_mutex;
void *static_scratch_ptr[MAX_DEVICES] = {};
int32_t *static_status_ptr[MAX_DEVICES] = {};
bool static_configured[MAX_DEVICES] = {};

// Once per device, with that device current: the device addresses of the array
// and the status word (host code cannot use the symbols' host-side names as
// device addresses), and the kernel's shared-memory limit.
pr_status static_setup(int device, const char *op) {
  std::lock_guard<std::mutex> lock(static_setup_mutex);
  if (static_configured[device])
    return PR_SUCCESS;
  void *scratch = nullptr, *status = nullptr;
  if (cudaGetSymbolAddress(&scratch, static_scratch) != cudaSuccess ||
      cudaGetSymbolAddress(&status, static_status) != cudaSuccess) {
    cudaGetLastError();
    return set_error_fixed(PR_DEVICE_UNAVAILABLE, op, "cudaGetSymbolAddress of the static workspace failed");
  }
  if (cudaFuncSetAttribute(gemm_tf32x3, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) != cudaSuccess) {
    cudaGetLastError();
    return set_error_fixed(PR_DEVICE_UNAVAILABLE, op, "cannot configure the GEMM kernel's shared memory");
  }
  static_scratch_ptr[device] = scratch;
  static_status_ptr[device] = static_cast<int32_t *>(status);
  static_configured[device] = true;
  return PR_SUCCESS;
}

} // namespace
} // namespace pb

using namespace pb;

PB_EXPORT pr_status pr_b200_matmul_tf32x3_static_f32(const float *a, const float *b, float *c, uint64_t m,
                                                     uint64_t n, uint64_t k, uint64_t lda, uint64_t ldb,
                                                     uint64_t ldc, uint32_t transpose_a, uint32_t transpose_b,
                                                     void *stream, int32_t *status) {
  static const char op[] = "b200_matmul_tf32x3_static_f32";
  if (!a || !b || !c)
    return set_error_fixed(PR_INVALID_ARGUMENT, op, "a, b and c must be device pointers");
  if (transpose_a > 1 || transpose_b > 1)
    return set_error_fixed(PR_INVALID_ARGUMENT, op, "Transpose flags must be 0 or 1");
  if (m < 1 || n < 1 || k < 16)
    return set_error_fixed(PR_UNSUPPORTED, op, "The 3xTF32 kernel needs m >= 1, n >= 1 and k >= 16");
  if (m > INT32_MAX || n > INT32_MAX || k > INT32_MAX)
    return set_error_fixed(PR_UNSUPPORTED, op, "Matmul dimensions must not exceed INT32_MAX");
  if ((transpose_a ? lda < m : lda < k) || (transpose_b ? ldb < k : ldb < n) || ldc < n)
    return set_error_fixed(PR_INVALID_ARGUMENT, op, "A row stride is smaller than its row");
  if ((uintptr_t(a) | uintptr_t(b) | uintptr_t(c)) & 3u)
    return set_error_fixed(PR_INVALID_ARGUMENT, op, "a, b and c must be 4-byte aligned");
  const int64_t k_pad = round_up(int64_t(k), 32), m_pad = round_up(int64_t(m), TM), n_pad = round_up(int64_t(n), TN);
  if (uint64_t(8) * uint64_t(k_pad) * uint64_t(m_pad + n_pad) > STATIC_SCRATCH_BYTES)
    return set_error_fixed(PR_OUT_OF_BOUNDS, op,
                           "Shape exceeds the 64 MiB static workspace: 8*round_up(k,32)*(round_up(m,128)+"
                           "round_up(n,256)) bytes must be at most 67108864");
  if (m_pad / 32 > 65535 || n_pad / 32 > 65535)
    return set_error_fixed(PR_UNSUPPORTED, op, "Shape exceeds the split kernel's grid");
  int device = -1;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= MAX_DEVICES) {
    cudaGetLastError();
    return set_error_fixed(PR_DEVICE_UNAVAILABLE, op, "No current CUDA device");
  }
  if (!encoder())
    return set_error_fixed(PR_DEVICE_UNAVAILABLE, op, "cuTensorMapEncodeTiled is unavailable");
  const pr_status setup = static_setup(device, op);
  if (setup != PR_SUCCESS)
    return setup;
  float *ahi = static_cast<float *>(static_scratch_ptr[device]);
  float *alo = ahi + m_pad * k_pad, *bhi = alo + m_pad * k_pad, *blo = bhi + n_pad * k_pad;
  CUtensorMap maps[4];
  if (!make_map(&maps[0], ahi, m_pad, k_pad, TM) || !make_map(&maps[1], alo, m_pad, k_pad, TM) ||
      !make_map(&maps[2], bhi, n_pad, k_pad, TN) || !make_map(&maps[3], blo, n_pad, k_pad, TN))
    return set_error_fixed(PR_INTERNAL_ERROR, op, "Tensor map encoding failed");
  auto s = static_cast<cudaStream_t>(stream);
  // The split writes every element of the four operand blocks the GEMM reads
  // (padding included), so the previous call's contents are never read.
  split_tf32<<<dim3(uint32_t(k_pad / 32), uint32_t(m_pad / 32)), 256, 0, s>>>(a, int64_t(lda), transpose_a ? 1 : 0,
                                                                              int64_t(m), int64_t(k), ahi, alo, k_pad,
                                                                              0, m_pad, nullptr, 0);
  split_tf32<<<dim3(uint32_t(k_pad / 32), uint32_t(n_pad / 32)), 256, 0, s>>>(b, int64_t(ldb), transpose_b ? 0 : 1,
                                                                              int64_t(n), int64_t(k), bhi, blo, k_pad,
                                                                              0, n_pad, nullptr, 0);
  TileArgs t{c, int64_t(m), int64_t(n), int64_t(ldc), int(k_pad / TK), int(m_pad / TM), int(n_pad / TN),
             status ? status : static_status_ptr[device]};
  gemm_tf32x3<<<uint32_t((m_pad / TM) * (n_pad / TN)), THREADS, SMEM_BYTES, s>>>(maps[0], maps[1], maps[2], maps[3], t);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return set_error_fixed(PR_EXECUTION_FAILED, op, cudaGetErrorString(e));
  clear_error();
  return PR_SUCCESS;
}
