// Row gather over NVLink (pr_b200_gather_rows_f32): a rank's [rows, columns] shard
// is written at rows [row_offset, row_offset + rows) of every gathered tensor, its own
// and its peers' (CUDA-IPC-mapped device memory of the other GPUs, reached with plain
// stores). This is the all-gather of a row-sharded result (a GEMM shard's C, for
// instance) as one kernel that reads the shard once and streams it to every
// destination at once; only plain stores touch peer memory (no NCCL, no TMA).
#include "../runtime/builtin.hpp"
#include <algorithm>

namespace pb {
namespace {

constexpr int kMaxTargets = 8;

struct Targets {
  float *dest[kMaxTargets];
  uint32_t count;
};

// 128-bit form: the shard and every destination row start on 16-byte boundaries
// and columns % 4 == 0, so the shard is a flat run of float4 that lands at a flat
// float4 offset in each destination.
__global__ void __launch_bounds__(256) gather_rows_vec(const float4 *__restrict__ local, uint64_t count4,
                                                       uint64_t offset4, const Targets t) {
  const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
  for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < count4; i += stride) {
    const float4 v = local[i];
#pragma unroll
    for (int d = 0; d < kMaxTargets; ++d)
      if (d < int(t.count))
        reinterpret_cast<float4 *>(t.dest[d])[offset4 + i] = v;
  }
  __threadfence_system(); // the peers' copies are complete when the command is
}

__global__ void __launch_bounds__(256) gather_rows_scalar(const float *__restrict__ local, uint64_t count,
                                                          uint64_t offset, const Targets t) {
  const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
  for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += stride) {
    const float v = local[i];
#pragma unroll
    for (int d = 0; d < kMaxTargets; ++d)
      if (d < int(t.count))
        t.dest[d][offset + i] = v;
  }
  __threadfence_system();
}

} // namespace

// (local, columns, rows, row_offset low, row_offset high, count, gathered 0..count-1)
void launch_gather_rows(Launch &L) {
  const auto &a = L.args;
  const uint32_t columns = a[1].u32(), rows = a[2].u32(), count = a[5].u32();
  const uint64_t row_offset = uint64_t(a[3].u32()) | uint64_t(a[4].u32()) << 32;
  if (count > kMaxTargets || a.size() != 6 + count)
    throw Failure(PR_INVALID_ARGUMENT, "Malformed gather launch");
  if (!columns || !rows || !count) {
    L.variant = "empty";
    return;
  }
  const uint64_t elements = uint64_t(rows) * columns;
  need_elements(a[0], elements, "local");
  Targets t{};
  t.count = count;
  bool aligned = (uintptr_t(a[0].ptr) & 15u) == 0 && columns % 4 == 0;
  for (uint32_t d = 0; d < count; ++d) {
    need_elements(a[6 + d], (row_offset + rows) * columns, "gathered");
    t.dest[d] = static_cast<float *>(a[6 + d].ptr);
    aligned = aligned && (uintptr_t(t.dest[d]) & 15u) == 0;
  }
  if (L.dry_run)
    return;
  const uint64_t offset = row_offset * columns;
  const int64_t blocks_max = int64_t(std::max(1, L.sm_count)) * 8;
  L.kernels = 1;
  if (aligned) {
    const uint64_t count4 = elements / 4;
    const int64_t blocks = std::min<int64_t>(int64_t((count4 + 255) / 256), blocks_max);
    gather_rows_vec<<<uint32_t(std::max<int64_t>(blocks, 1)), 256, 0, L.stream>>>(
        static_cast<const float4 *>(a[0].ptr), count4, offset / 4, t);
    L.variant = "vec4";
  } else {
    const int64_t blocks = std::min<int64_t>(int64_t((elements + 255) / 256), blocks_max);
    gather_rows_scalar<<<uint32_t(std::max<int64_t>(blocks, 1)), 256, 0, L.stream>>>(
        static_cast<const float *>(a[0].ptr), elements, offset, t);
    L.variant = "scalar";
  }
}

} // namespace pb
