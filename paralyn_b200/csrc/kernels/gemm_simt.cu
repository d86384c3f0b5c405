// FP32 SIMT GEMM for sm_100a: C[m,n] = op(A)[m,k] op(B)[k,n].
//
// Every output keeps one FP32 accumulator that takes k = 0, 1, ..., K-1 in order,
// as the reference kernel does (runtime/tensor.cpp:44-77). Two summation modes:
//   reference: sum = fl(sum + fl(a*b)) (__fmul_rn, __fadd_rn), bit-exact with the
//              sequential checker (tests/native/tensor_tests.cpp:62-85);
//   ffma:      sum = fma(a, b, sum), one rounding per step, within the
//              2*K*2^-24*sum|a||b| bound.
// Tiling: 128x128 outputs per 256-thread block, k-slices of 8 staged in shared
// memory (A stored k-major so both operands are read as 128-bit vectors), two
// shared buffers with register prefetch of the next slice, and an 8x8 register
// tile per thread laid out as 2x2 quads of 4x4 (conflict-free LDS.128).
// Blocks walk the output in groups of 8 tile-rows so consecutive blocks share B
// in L2.
#include "../runtime/builtin.hpp"
#include "activation.cuh"
#include "prepared.hpp"
#include "tma.cuh"
#include <algorithm>

namespace pb {
namespace {

constexpr int BM = 128, BN = 128, BK = 8, THREADS = 256;

struct GemmArgs {
  const float *a, *b;
  float *c;
  int64_t m, n, k;       // m, n: extent computed; k: full depth
  int64_t lda, ldb, ldc; // row strides of the stored matrices
  bool vec_a, vec_b, vec_c;
  // Batched launches (grid.z = batch): matrix z starts sa / sb / sc elements after
  // matrix z-1; C's column stride may differ from 1.
  int64_t sa = 0, sb = 0, sc = 0, c_col = 1;
  // Fused epilogue: C = activate(fl(acc + bias[column])) (activation.cuh).
  const float *bias = nullptr;
  uint32_t activation = 0;
  // Guarded launch: the kernel does nothing unless *only_if == epoch (the AUTO
  // mode's recomputation of a 3xTF32 command whose operands held an infinity).
  const unsigned long long *only_if = nullptr;
  unsigned long long epoch = 0;
};

template <int MODE> __device__ __forceinline__ float mac(float acc, float a, float b) {
  if constexpr (MODE == matmul_reference)
    return __fadd_rn(acc, __fmul_rn(a, b));
  else
    return __fmaf_rn(a, b, acc);
}

// Two accumulators at once: the sm_100 paired FP32 FMA (each component rounded as a
// scalar FMA) halves the issue slots the multiply-adds take. The reference order has
// no paired form: a paired multiply followed by a paired add, even written as PTX with
// explicit rounding, came out as fused multiply-adds (results one ulp off the
// reference's), so that order stays on scalar `__fmul_rn`/`__fadd_rn`.
__device__ __forceinline__ float2 ffma2(float2 acc, float2 a, float2 b) { return __ffma2_rn(a, b, acc); }

// Loads this thread's 4 values of the A slice [m0, m0+128) x [k0, k0+8).
//  !TA: A[m][k] at a[m*lda + k]; thread t reads row t/2, k (t%2)*4 .. +3
//   TA: A[m][k] at a[k*lda + m]; thread t reads k t/32, m (t%32)*4 .. +3
template <bool TA>
__device__ __forceinline__ void load_a(const GemmArgs &g, int64_t m0, int64_t k0, float r[4]) {
  const int t = threadIdx.x;
  if constexpr (!TA) {
    const int64_t m = m0 + t / 2, k = k0 + (t % 2) * 4;
    const float *p = g.a + m * g.lda + k;
    if (m < g.m && g.vec_a && k + 3 < g.k) {
      const float4 v = *reinterpret_cast<const float4 *>(p);
      r[0] = v.x, r[1] = v.y, r[2] = v.z, r[3] = v.w;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        r[j] = (m < g.m && k + j < g.k) ? p[j] : 0.0f;
    }
  } else {
    const int64_t k = k0 + t / 32, m = m0 + (t % 32) * 4;
    const float *p = g.a + k * g.lda + m;
    if (k < g.k && g.vec_a && m + 3 < g.m) {
      const float4 v = *reinterpret_cast<const float4 *>(p);
      r[0] = v.x, r[1] = v.y, r[2] = v.z, r[3] = v.w;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        r[j] = (k < g.k && m + j < g.m) ? p[j] : 0.0f;
    }
  }
}

//  !TB: B[k][n] at b[k*ldb + n]; thread t reads k t/32, n (t%32)*4 .. +3
//   TB: B[k][n] at b[n*ldb + k]; thread t reads n t/2, k (t%2)*4 .. +3
template <bool TB>
__device__ __forceinline__ void load_b(const GemmArgs &g, int64_t n0, int64_t k0, float r[4]) {
  const int t = threadIdx.x;
  if constexpr (!TB) {
    const int64_t k = k0 + t / 32, n = n0 + (t % 32) * 4;
    const float *p = g.b + k * g.ldb + n;
    if (k < g.k && g.vec_b && n + 3 < g.n) {
      const float4 v = *reinterpret_cast<const float4 *>(p);
      r[0] = v.x, r[1] = v.y, r[2] = v.z, r[3] = v.w;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        r[j] = (k < g.k && n + j < g.n) ? p[j] : 0.0f;
    }
  } else {
    const int64_t n = n0 + t / 2, k = k0 + (t % 2) * 4;
    const float *p = g.b + n * g.ldb + k;
    if (n < g.n && g.vec_b && k + 3 < g.k) {
      const float4 v = *reinterpret_cast<const float4 *>(p);
      r[0] = v.x, r[1] = v.y, r[2] = v.z, r[3] = v.w;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        r[j] = (n < g.n && k + j < g.k) ? p[j] : 0.0f;
    }
  }
}

// Shared slices are k-major: sa[k][m], sb[k][n].
template <bool TA> __device__ __forceinline__ void store_a(float (*sa)[BM], const float r[4]) {
  const int t = threadIdx.x;
  if constexpr (!TA) {
    const int m = t / 2, k = (t % 2) * 4;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      sa[k + j][m] = r[j];
  } else {
    *reinterpret_cast<float4 *>(&sa[t / 32][(t % 32) * 4]) = make_float4(r[0], r[1], r[2], r[3]);
  }
}
template <bool TB> __device__ __forceinline__ void store_b(float (*sb)[BN], const float r[4]) {
  const int t = threadIdx.x;
  if constexpr (!TB) {
    *reinterpret_cast<float4 *>(&sb[t / 32][(t % 32) * 4]) = make_float4(r[0], r[1], r[2], r[3]);
  } else {
    const int n = t / 2, k = (t % 2) * 4;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      sb[k + j][n] = r[j];
  }
}

template <int MODE, bool TA, bool TB>
__device__ __forceinline__ void simt_tile(const GemmArgs &g, int64_t id, int64_t tiles_m, int64_t tiles_n,
                                          float (*sa)[BK][BM], float (*sb)[BK][BN]) {
  // Grouped raster: 8 tile-rows at a time, columns fastest within the group.
  const int64_t group = 8;
  const int64_t per_group = group * tiles_n;
  const int64_t first_m = (id / per_group) * group;
  const int64_t rows_in_group = min(group, tiles_m - first_m);
  const int64_t tm = first_m + (id % per_group) % rows_in_group;
  const int64_t tn = (id % per_group) / rows_in_group;
  const int64_t m0 = tm * BM, n0 = tn * BN;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j)
      acc[i][j] = 0.0f;

  float ra[4], rb[4];
  load_a<TA>(g, m0, 0, ra);
  load_b<TB>(g, n0, 0, rb);
  store_a<TA>(sa[0], ra);
  store_b<TB>(sb[0], rb);
  __syncthreads();

  const int64_t slices = (g.k + BK - 1) / BK;
  for (int64_t s = 0; s < slices; ++s) {
    const int cur = s & 1;
    const bool more = s + 1 < slices;
    if (more) {
      load_a<TA>(g, m0, (s + 1) * BK, ra);
      load_b<TB>(g, n0, (s + 1) * BK, rb);
    }
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[8], b[8];
      const float4 a0 = *reinterpret_cast<const float4 *>(&sa[cur][kk][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4 *>(&sa[cur][kk][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4 *>(&sb[cur][kk][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4 *>(&sb[cur][kk][64 + tx * 4]);
      a[0] = a0.x, a[1] = a0.y, a[2] = a0.z, a[3] = a0.w;
      a[4] = a1.x, a[5] = a1.y, a[6] = a1.z, a[7] = a1.w;
      b[0] = b0.x, b[1] = b0.y, b[2] = b0.z, b[3] = b0.w;
      b[4] = b1.x, b[5] = b1.y, b[6] = b1.z, b[7] = b1.w;
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j)
          acc[i][j] = mac<MODE>(acc[i][j], a[i], b[j]);
    }
    if (more) {
      store_a<TA>(sa[cur ^ 1], ra);
      store_b<TB>(sb[cur ^ 1], rb);
    }
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (m >= g.m)
      continue;
    float *row = g.c + m * g.ldc;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int64_t n = n0 + h * 64 + tx * 4;
      float v[4] = {acc[i][4 * h], acc[i][4 * h + 1], acc[i][4 * h + 2], acc[i][4 * h + 3]};
      if (g.bias || g.activation) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (n + j < g.n)
            v[j] = bias_activate(v[j], g.bias, n + j, g.activation);
      }
      if (g.c_col != 1) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (n + j < g.n)
            row[(n + j) * g.c_col] = v[j];
      } else if (g.vec_c && n + 3 < g.n) {
        *reinterpret_cast<float4 *>(row + n) = make_float4(v[0], v[1], v[2], v[3]);
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (n + j < g.n)
            row[n + j] = v[j];
      }
    }
  }
}

// ---- TMA-fed form (A not transposed or transposed, B not transposed) ----
// The same 128 x 128 tiles, 8 x 8 register tiles and per-output k order, with the
// operands moved by the tensor memory accelerator instead of the threads: 32-deep
// k-slices of A and B land in a three-stage shared-memory ring (96 KB, two CTAs per
// SM), each stage tracked by a `full` barrier (TMA transaction bytes) and an `empty`
// barrier (one arrival per warp once it has read the stage). Thread 0 refills a
// stage one slice after the warps released it, so the warps only load shared
// memory and multiply: no global loads, shared stores or block barriers in the
// k loop. Layouts in shared memory:
//   A stored [m][k] (row-major): each stage holds A[m0..+128][k0..+32] as 128-byte
//     rows with the 128-byte swizzle (16-byte chunk c of row r at chunk c ^ (r % 8)).
//     Thread (tx, ty) owns rows ty + 16 i (i < 8), which share one swizzle phase, so
//     one chunk offset per k pair serves all eight; the two rows a warp reads per
//     instruction (ty and ty + 1) fall in different banks. A thread reads float2
//     along k for each of its rows and uses them for 2 k.
//   A stored [k][m] (transposed): A[k0..+32][m0..+128] as 512-byte rows; float4
//     along m, as in the register-staged kernel.
//   B stored [k][n]: B[k0..+32][n0..+128] as 512-byte rows; float4 along n.
// Rows and columns past the matrix and k past K read as zero (TMA fill), adding
// exact +0.0 products that leave every sum unchanged.
constexpr int TBK = 32, TSTAGES = 3;
constexpr int TA_BYTES = BM * TBK * 4, TB_BYTES = TBK * BN * 4, TSTAGE = TA_BYTES + TB_BYTES;
constexpr int TSMEM = 1024 + TSTAGES * TSTAGE + 256;
constexpr int STATUS_TIMEOUT_SIMT = 0x7f3205;

template <int MODE, bool TA>
__global__ void __launch_bounds__(THREADS, 2)
    gemm_simt_tma(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap, const GemmArgs g,
                  int *status) {
  static_assert(MODE == matmul_ffma, "the TMA-fed kernel accumulates with paired FMAs");
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned (the 128-byte swizzle repeats every 1024 bytes); an offset from
  // the shared array keeps the accesses in the shared state space.
  uint8_t *smem = smem_raw + ((1024u - (tma::smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + TSTAGES * TSTAGE);
  uint64_t *empty = full + TSTAGES;
  volatile int *abort_flag = reinterpret_cast<volatile int *>(empty + TSTAGES);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;

  const int64_t tiles_m = (g.m + BM - 1) / BM, tiles_n = (g.n + BN - 1) / BN;
  const int64_t id = blockIdx.x, group = 8, per_group = group * tiles_n;
  const int64_t first_m = (id / per_group) * group;
  const int64_t rows_in_group = min(group, tiles_m - first_m);
  const int m0 = int((first_m + (id % per_group) % rows_in_group) * BM);
  const int n0 = int(((id % per_group) / rows_in_group) * BN);
  const int slices = int((g.k + TBK - 1) / TBK);

  auto issue = [&](int slice) { // thread 0: slice -> stage slice % TSTAGES
    const int st = slice % TSTAGES;
    uint8_t *stage = smem + st * TSTAGE;
    tma::mbar_expect_tx(&full[st], TSTAGE);
    if (TA)
      tma::tma_load_2d(stage, &amap, &full[st], m0, slice * TBK);
    else
      tma::tma_load_2d(stage, &amap, &full[st], slice * TBK, m0);
    tma::tma_load_2d(stage + TA_BYTES, &bmap, &full[st], n0, slice * TBK);
  };
  if (threadIdx.x == 0) {
    for (int st = 0; st < TSTAGES; ++st) {
      tma::mbar_init(&full[st], 1);
      tma::mbar_init(&empty[st], THREADS / 32);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  __syncthreads();
  int issued = 0;
  if (threadIdx.x == 0)
    for (; issued < min(TSTAGES, slices); ++issued)
      issue(issued);

  // acc[i][p]: row i, columns (2p, 2p + 1) of the thread's eight (tx*4 + 0..3,
  // 64 + tx*4 + 0..3), updated with paired FP32 operations (two lanes' worth of FMA
  // per instruction, each component rounded as a scalar FMA), which halves the
  // issue slots the multiply-adds take.
  float2 acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int p = 0; p < 4; ++p)
      acc[i][p] = make_float2(0.0f, 0.0f);

  int done = 0; // slices this thread consumed
  for (int slice = 0; slice < slices; ++slice) {
    const int st = slice % TSTAGES;
    // Thread 0 refills the stage released one slice ago (all eight warps read it).
    if (threadIdx.x == 0 && slice >= 1 && issued < slices && !*abort_flag) {
      const int prev = (slice - 1) % TSTAGES;
      if (tma::mbar_wait(&empty[prev], ((slice - 1) / TSTAGES) & 1)) {
        issue(issued);
        ++issued;
      } else {
        atomicExch(status, STATUS_TIMEOUT_SIMT);
        *abort_flag = 1;
      }
    }
    if (!tma::mbar_wait(&full[st], (slice / TSTAGES) & 1)) {
      atomicExch(status, STATUS_TIMEOUT_SIMT);
      *abort_flag = 1;
    }
    if (*abort_flag)
      break;
    const float *As = reinterpret_cast<const float *>(smem + st * TSTAGE);
    const float *Bs = reinterpret_cast<const float *>(smem + st * TSTAGE + TA_BYTES);
#pragma unroll
    for (int kq = 0; kq < TBK / 2; ++kq) {
      float a4[8][2]; // this thread's 8 rows x 2 consecutive k
      if (!TA) { // rows ty + 16 i: all in swizzle phase ty % 8, one chunk offset per kq
        const int offset = ((((kq >> 1) ^ ty) & 7) << 2) + 2 * (kq & 1);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float2 v = *reinterpret_cast<const float2 *>(As + (ty + 16 * i) * TBK + offset);
          a4[i][0] = v.x, a4[i][1] = v.y;
        }
      } else {
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const float4 v0 = *reinterpret_cast<const float4 *>(As + (kq * 2 + q) * BM + ty * 4);
          const float4 v1 = *reinterpret_cast<const float4 *>(As + (kq * 2 + q) * BM + 64 + ty * 4);
          a4[0][q] = v0.x, a4[1][q] = v0.y, a4[2][q] = v0.z, a4[3][q] = v0.w;
          a4[4][q] = v1.x, a4[5][q] = v1.y, a4[6][q] = v1.z, a4[7][q] = v1.w;
        }
      }
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int kk = kq * 2 + q;
        const float4 b0 = *reinterpret_cast<const float4 *>(Bs + kk * BN + tx * 4);
        const float4 b1 = *reinterpret_cast<const float4 *>(Bs + kk * BN + 64 + tx * 4);
        const float2 b[4] = {make_float2(b0.x, b0.y), make_float2(b0.z, b0.w), make_float2(b1.x, b1.y),
                             make_float2(b1.z, b1.w)};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float2 a = make_float2(a4[i][q], a4[i][q]);
#pragma unroll
          for (int p = 0; p < 4; ++p)
            acc[i][p] = ffma2(acc[i][p], a, b[p]);
        }
      }
    }
    __syncwarp();
    if (lane == 0)
      tma::mbar_arrive(&empty[st]);
    done = slice + 1;
  }
  __syncthreads();
  if (*abort_flag) {
    if (threadIdx.x == 0) // copies requested but not consumed land before the block ends
      for (int slice = done; slice < issued; ++slice)
        (void)tma::mbar_wait(&full[slice % TSTAGES], (slice / TSTAGES) & 1);
    return; // C is left as it was; the command reports the status
  }
  (void)warp;

#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t m = m0 + (TA ? (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4)) : ty + 16 * i);
    if (m >= g.m)
      continue;
    float *row = g.c + m * g.ldc;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int64_t n = n0 + h * 64 + tx * 4;
      float v[4] = {acc[i][2 * h].x, acc[i][2 * h].y, acc[i][2 * h + 1].x, acc[i][2 * h + 1].y};
      if (g.bias || g.activation) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (n + j < g.n)
            v[j] = bias_activate(v[j], g.bias, n + j, g.activation);
      }
      if (g.vec_c && n + 3 < g.n) {
        *reinterpret_cast<float4 *>(row + n) = make_float4(v[0], v[1], v[2], v[3]);
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (n + j < g.n)
            row[n + j] = v[j];
      }
    }
  }
}

template <int MODE, bool TA> bool configure_simt_tma(int device) {
  static bool configured[64] = {};
  if (device < 0 || device >= 64)
    return false;
  if (!configured[device]) {
    if (cudaFuncSetAttribute(gemm_simt_tma<MODE, TA>, cudaFuncAttributeMaxDynamicSharedMemorySize, TSMEM) !=
        cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    configured[device] = true;
  }
  return true;
}

// The TMA-fed kernel for one (non-batched) product when its operands can be tensor
// maps: B not transposed, 16-byte aligned bases and row strides, dimensions that fit
// the maps' 32-bit coordinates. Returns false (nothing enqueued) otherwise.
template <int MODE>
bool launch_simt_tma(Launch &L, const GemmArgs &g, bool ta, bool tb) {
  if (tb || g.c_col != 1 || g.m > INT32_MAX - BM || g.n > INT32_MAX - BN || g.k > INT32_MAX - TBK)
    return false;
  if ((reinterpret_cast<uintptr_t>(g.a) & 15u) || (reinterpret_cast<uintptr_t>(g.b) & 15u) || g.lda % 4 ||
      g.ldb % 4)
    return false;
  CUtensorMap amap, bmap;
  const bool a_ok = ta ? encode_map_2d(&amap, g.a, uint64_t(g.m), uint64_t(g.k), uint64_t(g.lda) * 4, BM, TBK, false)
                       : encode_map_2d(&amap, g.a, uint64_t(g.k), uint64_t(g.m), uint64_t(g.lda) * 4, TBK, BM, true);
  if (!a_ok || !encode_map_2d(&bmap, g.b, uint64_t(g.n), uint64_t(g.k), uint64_t(g.ldb) * 4, BN, TBK, false))
    return false;
  if (!(ta ? configure_simt_tma<MODE, true>(L.device) : configure_simt_tma<MODE, false>(L.device)))
    return false;
  const int64_t tiles = ((g.m + BM - 1) / BM) * ((g.n + BN - 1) / BN);
  if (ta)
    gemm_simt_tma<MODE, true><<<uint32_t(tiles), THREADS, TSMEM, L.stream>>>(amap, bmap, g, L.status);
  else
    gemm_simt_tma<MODE, false><<<uint32_t(tiles), THREADS, TSMEM, L.stream>>>(amap, bmap, g, L.status);
  return true;
}

// One block per tile. GUARDED: the launch does nothing unless *only_if == epoch,
// and fewer blocks than tiles walk the tiles id = blockIdx.x, + gridDim.x, ...
template <int MODE, bool TA, bool TB, bool GUARDED>
__global__ void __launch_bounds__(THREADS, 2) gemm_simt(const GemmArgs batch) {
  if (GUARDED && *batch.only_if != batch.epoch)
    return;
  GemmArgs g = batch;
  g.a += int64_t(blockIdx.z) * batch.sa;
  g.b += int64_t(blockIdx.z) * batch.sb;
  g.c += int64_t(blockIdx.z) * batch.sc;
  __shared__ __align__(16) float sa[2][BK][BM];
  __shared__ __align__(16) float sb[2][BK][BN];
  const int64_t tiles_m = (g.m + BM - 1) / BM, tiles_n = (g.n + BN - 1) / BN;
  if constexpr (!GUARDED) {
    simt_tile<MODE, TA, TB>(g, blockIdx.x, tiles_m, tiles_n, sa, sb);
  } else {
    for (int64_t id = blockIdx.x; id < tiles_m * tiles_n; id += gridDim.x)
      simt_tile<MODE, TA, TB>(g, id, tiles_m, tiles_n, sa, sb);
  }
}

// One block per tile, or (guarded launches) at most max_blocks blocks per matrix.
template <int MODE, bool TA, bool TB>
void run(const GemmArgs &g, cudaStream_t stream, uint32_t batch, int64_t max_blocks) {
  const int64_t tiles = ((g.m + BM - 1) / BM) * ((g.n + BN - 1) / BN);
  if (g.only_if)
    gemm_simt<MODE, TA, TB, true><<<dim3(uint32_t(std::min(tiles, max_blocks)), 1, batch), THREADS, 0, stream>>>(g);
  else
    gemm_simt<MODE, TA, TB, false><<<dim3(uint32_t(tiles), 1, batch), THREADS, 0, stream>>>(g);
}

template <int MODE>
void dispatch(const GemmArgs &g, bool ta, bool tb, cudaStream_t stream, uint32_t batch = 1, int64_t max_blocks = 0) {
  if (!ta && !tb)
    run<MODE, false, false>(g, stream, batch, max_blocks);
  else if (!ta && tb)
    run<MODE, false, true>(g, stream, batch, max_blocks);
  else if (ta && !tb)
    run<MODE, true, false>(g, stream, batch, max_blocks);
  else
    run<MODE, true, true>(g, stream, batch, max_blocks);
}

// AUTO mode after a 3xTF32 command that watched its operands: the FFMA kernel over the
// same operands, guarded by the command's non-finite word, so it recomputes C (IEEE
// propagation of +-inf in increasing k) only when an operand held an infinity. When
// the word is clear every block returns at once; two blocks per SM walk the tiles.
void recompute_if_infinite(Launch &L, const GemmArgs &g, bool ta, bool tb, uint32_t batch,
                           const NonFiniteFlag &watch) {
  if (!watch.word)
    return;
  GemmArgs guarded = g;
  guarded.only_if = watch.word;
  guarded.epoch = watch.epoch;
  // About two blocks per SM over the whole batch: the blocks of a launch whose flag
  // is clear return at once, and for a batch of many matrices a grid of two blocks per
  // SM for every matrix would take many rounds of block launches to do nothing.
  const int64_t per_matrix = std::max<int64_t>(1, (int64_t(2) * std::max(1, L.sm_count) + batch - 1) / batch);
  dispatch<matmul_ffma>(guarded, ta, tb, L.stream, batch, per_matrix);
  ++L.kernels;
}

// Any strides: one output per thread, 16x16 threads per block, k in increasing order.
template <int MODE>
__global__ void __launch_bounds__(256) batched_generic(const float *a, const float *b, float *c, int64_t m,
                                                       int64_t n, int64_t k, int64_t a0, int64_t a1, int64_t a2,
                                                       int64_t b0, int64_t b1, int64_t b2, int64_t c0, int64_t c1,
                                                       int64_t c2) {
  const int64_t i = int64_t(blockIdx.y) * 16 + threadIdx.y, j = int64_t(blockIdx.x) * 16 + threadIdx.x;
  if (i >= m || j >= n)
    return;
  const int64_t z = blockIdx.z;
  const float *ar = a + z * a0 + i * a1, *bc = b + z * b0 + j * b2;
  float sum = 0.0f;
  for (int64_t p = 0; p < k; ++p)
    sum = mac<MODE>(sum, ar[p * a2], bc[p * b1]);
  c[z * c0 + i * c1 + j * c2] = sum;
}

__global__ void __launch_bounds__(256) batched_fill(float *c, int64_t m, int64_t n, int64_t c0, int64_t c1,
                                                    int64_t c2, float value) {
  const int64_t i = int64_t(blockIdx.y) * 16 + threadIdx.y, j = int64_t(blockIdx.x) * 16 + threadIdx.x;
  if (i < m && j < n)
    c[int64_t(blockIdx.z) * c0 + i * c1 + j * c2] = value;
}

bool aligned16(const void *p) { return (uintptr_t(p) & 15u) == 0; }

} // namespace

bool launch_tf32x3_gemm(Launch &L, const float *a, const float *b, float *c, int64_t m, int64_t n,
                        int64_t k, int64_t lda, int64_t ldb, int64_t ldc, bool ta, bool tb,
                        const float *bias, uint32_t activation, NonFiniteFlag *watch, const PreparedB *prep);
void launch_prepared_check(Launch &L, const PreparedB &prep);
bool launch_tf32x3_batched(Launch &L, const float *a, const float *b, float *c, int64_t batch, int64_t m,
                           int64_t n, int64_t k, int64_t lda, bool ta, int64_t sa, int64_t ldb, bool tb, int64_t sb,
                           int64_t ldc, int64_t sc, NonFiniteFlag *watch);

namespace {
// C = op(A) op(B) over the grid-bounded region, optionally with the bias/activation
// epilogue fused (bias: view of n values or absent; activation 0..2). With `prepared`,
// L.args[1] is B's prepared form (prepared.hpp) and transpose_b is 0: the tensor-core
// path reads its TF32 pair, the SIMT kernels its [k][n] copy.
void run_matmul(Launch &L, const BoundArg *bias_view, uint32_t activation, bool prepared = false) {
  const uint32_t m = L.args[3].u32(), n = L.args[4].u32(), k = L.args[5].u32();
  const uint32_t ta = L.args[6].u32(), tb = L.args[7].u32();
  if (ta > 1 || tb > 1)
    throw Failure(PR_INVALID_ARGUMENT, "Transpose flags must be 0 or 1");
  if (prepared && (tb || !prepared::bytes(k, n)))
    throw Failure(PR_INVALID_ARGUMENT, "A prepared operand needs transpose_b = 0 and 1 <= k, n <= INT32_MAX");
  if (activation > 2)
    throw Failure(PR_INVALID_ARGUMENT, "Unknown activation");
  const int64_t me = std::min<int64_t>(m, int64_t(L.grid.y) * 16);
  const int64_t ne = std::min<int64_t>(n, int64_t(L.grid.x) * 16);
  if (!me || !ne) {
    L.variant = "empty";
    return;
  }
  // Highest element index + 1 each operand is read or written at.
  const uint64_t a_need = ta ? uint64_t(k ? k - 1 : 0) * m + me : uint64_t(me) * k;
  const uint64_t b_need = prepared ? prepared::bytes(k, n) / 4
                                   : (tb ? uint64_t(ne) * k : uint64_t(k ? k - 1 : 0) * n + ne);
  if (k) {
    need_elements(L.args[0], a_need, "a");
    need_elements(L.args[1], b_need, prepared ? "prepared" : "b");
  }
  if (prepared && reinterpret_cast<uintptr_t>(L.args[1].ptr) % prepared::kHeaderBytes)
    throw Failure(PR_INVALID_ARGUMENT, "The prepared tensor must start on a 256-byte boundary");
  need_elements(L.args[2], uint64_t(me - 1) * n + ne, "c");
  if (bias_view)
    need_elements(*bias_view, ne, "bias");
  if (L.dry_run)
    return;
  PreparedB prep;
  if (prepared) {
    const char *base = static_cast<const char *>(L.args[1].ptr);
    prep.header = reinterpret_cast<const prepared::Header *>(base);
    prep.raw = reinterpret_cast<const float *>(base + prepared::raw_offset());
    prep.hi = reinterpret_cast<const float *>(base + prepared::hi_offset(k, n));
    prep.lo = reinterpret_cast<const float *>(base + prepared::lo_offset(k, n));
    prep.k = k;
    prep.n = n;
  }
  GemmArgs g;
  g.bias = bias_view ? static_cast<const float *>(bias_view->ptr) : nullptr;
  g.activation = activation;
  g.a = static_cast<const float *>(L.args[0].ptr);
  g.b = prepared ? prep.raw : static_cast<const float *>(L.args[1].ptr);
  g.c = static_cast<float *>(L.args[2].ptr);
  g.m = me;
  g.n = ne;
  g.k = k;
  g.lda = ta ? m : k;
  g.ldb = tb ? k : n;
  g.ldc = n;
  g.vec_a = aligned16(g.a) && g.lda % 4 == 0;
  g.vec_b = aligned16(g.b) && g.ldb % 4 == 0;
  g.vec_c = aligned16(g.c) && g.ldc % 4 == 0;
  uint32_t mode = L.matmul_mode;
  if (mode == matmul_auto || mode == matmul_tf32x3) {
    NonFiniteFlag watch;
    if (launch_tf32x3_gemm(L, g.a, g.b, g.c, me, ne, k, g.lda, g.ldb, g.ldc, ta, tb, g.bias, g.activation,
                           mode == matmul_auto ? &watch : nullptr, prepared ? &prep : nullptr)) {
      recompute_if_infinite(L, g, ta, tb, 1, watch);
      return;
    }
    mode = matmul_ffma;
  }
  L.kernels = 0;
  if (prepared)
    launch_prepared_check(L, prep);
  ++L.kernels;
  if (mode == matmul_reference) {
    // The register-staged kernel: the reference order (a rounded multiply, then a
    // rounded add, per step) takes two FP32 operations per product, so its ceiling is
    // half the FFMA peak; it measured 29.8 TFLOP/s at 4096^3 (0.80 of that ceiling)
    // against 21.7 for the TMA-fed kernel in this order.
    dispatch<matmul_reference>(g, ta, tb, L.stream);
    L.variant = "simt_reference_order";
  } else {
    if (launch_simt_tma<matmul_ffma>(L, g, ta, tb)) {
      L.variant = "simt_tma_ffma";
      return;
    }
    dispatch<matmul_ffma>(g, ta, tb, L.stream);
    L.variant = "simt_ffma";
  }
}
} // namespace

// (a, b, c, m, n, k, transpose_a, transpose_b) with a 16x16 block per 16x16 output
// tile: the grid bounds the computed region to min(m, 16*grid.y) x min(n, 16*grid.x).
void launch_provider_matmul(Launch &L) { run_matmul(L, nullptr, 0); }

// pr_b200_matmul_prepared_f32: (a, prepared, c, m, n, k, transpose_a, transpose_b =
// 0), the matmul launch with B's prepared form in place of B.
void launch_matmul_prepared(Launch &L) { run_matmul(L, nullptr, 0, true); }

// pr_b200_matmul_bias_activation_f32: (a, b, c, m, n, k, transpose_a, transpose_b,
// bias or an empty view, activation, has_bias) -- the matmul launch with the
// bias/activation epilogue fused. k == 0 runs the SIMT kernel (act(bias) everywhere).
void launch_matmul_bias_activation(Launch &L) {
  const bool has_bias = L.args[10].u32() != 0;
  run_matmul(L, has_bias ? &L.args[8] : nullptr, L.args[9].u32());
}

// pr_b200_matmul_prepared_bias_activation_f32: the fused launch's arguments with B's
// prepared form in place of B (transpose_b = 0).
void launch_matmul_prepared_bias_activation(Launch &L) {
  const bool has_bias = L.args[10].u32() != 0;
  run_matmul(L, has_bias ? &L.args[8] : nullptr, L.args[9].u32(), true);
}

namespace {
// Highest element index + 1 of a strided [d0, d1, d2] operand (all extents > 0).
uint64_t extent(uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s0, uint64_t s1, uint64_t s2) {
  return (d0 - 1) * s0 + (d1 - 1) * s1 + (d2 - 1) * s2 + 1;
}
// A strided [rows, cols] operand as a (leading dimension, transposed) pair, when one
// of its two strides is 1 (or that dimension has extent 1, so its stride is never
// used): element (r, c) at r*ld + c, or at c*ld + r when transposed.
bool as_matrix(int64_t rows, int64_t cols, int64_t row_stride, int64_t col_stride, int64_t &ld, bool &transposed) {
  if (col_stride == 1 || cols == 1) {
    ld = row_stride;
    transposed = false;
    return true;
  }
  if (row_stride == 1 || rows == 1) {
    ld = col_stride;
    transposed = true;
    return true;
  }
  return false;
}
} // namespace

// (a, b, c, m, n, k, a_batch, a_row, a_col, b_batch, b_row, b_col, c_batch, c_row,
//  c_col), grid (ceil(n/16), ceil(m/16), batch): C[z] = A[z] B[z] over element-strided
// views, each output one accumulator over increasing k (reference
// runtime/tensor.cpp:130-166). Operands whose strides make them row-major or
// transposed matrices run on the 3xTF32 tensor-core kernel (AUTO or TF32X3 mode, when
// C's columns are contiguous and the shape is large enough) or on the tiled SIMT
// kernel with a batch grid dimension; other layouts on a one-output-per-thread kernel.
void launch_provider_batched_matmul(Launch &L) {
  const auto &A = L.args;
  const int64_t m = std::min<int64_t>(A[3].u32(), int64_t(L.grid.y) * 16);
  const int64_t n = std::min<int64_t>(A[4].u32(), int64_t(L.grid.x) * 16);
  const int64_t k = A[5].u32();
  const uint64_t batch = L.grid.z;
  const int64_t s[9] = {A[6].u32(), A[7].u32(), A[8].u32(), A[9].u32(), A[10].u32(),
                        A[11].u32(), A[12].u32(), A[13].u32(), A[14].u32()};
  if (!m || !n || !batch) {
    L.variant = "empty";
    return;
  }
  if (k) {
    need_elements(A[0], extent(batch, m, k, s[0], s[1], s[2]), "a");
    need_elements(A[1], extent(batch, k, n, s[3], s[4], s[5]), "b");
  }
  need_elements(A[2], extent(batch, m, n, s[6], s[7], s[8]), "c");
  if (L.dry_run)
    return;
  const auto *a = static_cast<const float *>(A[0].ptr);
  const auto *b = static_cast<const float *>(A[1].ptr);
  auto *c = static_cast<float *>(A[2].ptr);
  const bool reference = L.matmul_mode == matmul_reference;
  L.kernels = 1;
  if (!k) {
    batched_fill<<<dim3(L.grid.x, L.grid.y, uint32_t(batch)), dim3(16, 16), 0, L.stream>>>(c, m, n, s[6], s[7], s[8],
                                                                                           0.0f);
    L.variant = "batched_fill";
    return;
  }
  if (batch > 65535)
    throw Failure(PR_UNSUPPORTED, "Batched matmul supports at most 65535 matrices per launch");
  GemmArgs g;
  bool ta = false, tb = false; // B's matrix form is [k, n]; transposed = stored [n, k]
  if (as_matrix(m, k, s[1], s[2], g.lda, ta) && as_matrix(k, n, s[4], s[5], g.ldb, tb)) {
    g.a = a;
    g.b = b;
    g.c = c;
    g.m = m;
    g.n = n;
    g.k = k;
    g.sa = s[0];
    g.sb = s[3];
    g.sc = s[6];
    g.ldc = s[7]; // element (i, j) of C[z] at i*ldc + j*c_col
    g.c_col = n == 1 ? 1 : s[8];
    g.vec_a = aligned16(a) && g.lda % 4 == 0 && g.sa % 4 == 0;
    g.vec_b = aligned16(b) && g.ldb % 4 == 0 && g.sb % 4 == 0;
    g.vec_c = aligned16(c) && g.ldc % 4 == 0 && g.sc % 4 == 0 && g.c_col == 1;
    NonFiniteFlag watch;
    if ((L.matmul_mode == matmul_auto || L.matmul_mode == matmul_tf32x3) && g.c_col == 1 &&
        launch_tf32x3_batched(L, a, b, c, int64_t(batch), m, n, k, g.lda, ta, g.sa, g.ldb, tb, g.sb, g.ldc, g.sc,
                              L.matmul_mode == matmul_auto ? &watch : nullptr)) {
      recompute_if_infinite(L, g, ta, tb, uint32_t(batch), watch);
      return;
    }
    if (reference)
      dispatch<matmul_reference>(g, ta, tb, L.stream, uint32_t(batch));
    else
      dispatch<matmul_ffma>(g, ta, tb, L.stream, uint32_t(batch));
    L.variant = reference ? "batched_simt_reference_order" : "batched_simt_ffma";
    return;
  }
  const dim3 grid(L.grid.x, L.grid.y, uint32_t(batch)), block(16, 16);
  if (reference)
    batched_generic<matmul_reference><<<grid, block, 0, L.stream>>>(a, b, c, m, n, k, s[0], s[1], s[2], s[3], s[4],
                                                                    s[5], s[6], s[7], s[8]);
  else
    batched_generic<matmul_ffma><<<grid, block, 0, L.stream>>>(a, b, c, m, n, k, s[0], s[1], s[2], s[3], s[4], s[5],
                                                               s[6], s[7], s[8]);
  L.variant = reference ? "batched_generic_reference_order" : "batched_generic_ffma";
}

// (c, m, n, c_batch, c_row, c_col, value), grid (ceil(n/16), ceil(m/16), batch).
void launch_provider_batched_fill(Launch &L) {
  const auto &A = L.args;
  const int64_t m = std::min<int64_t>(A[1].u32(), int64_t(L.grid.y) * 16);
  const int64_t n = std::min<int64_t>(A[2].u32(), int64_t(L.grid.x) * 16);
  const uint64_t batch = L.grid.z;
  if (!m || !n || !batch) {
    L.variant = "empty";
    return;
  }
  need_elements(A[0], extent(batch, m, n, A[3].u32(), A[4].u32(), A[5].u32()), "c");
  if (batch > 65535)
    throw Failure(PR_UNSUPPORTED, "Batched fill supports at most 65535 matrices per launch");
  if (L.dry_run)
    return;
  batched_fill<<<dim3(L.grid.x, L.grid.y, uint32_t(batch)), dim3(16, 16), 0, L.stream>>>(
      static_cast<float *>(A[0].ptr), m, n, A[3].u32(), A[4].u32(), A[5].u32(), A[6].f32());
  L.kernels = 1;
  L.variant = "batched_fill";
}

} // namespace pb
