// Shared-memory barrier and TMA helpers shared by the tensor-core and SIMT GEMMs.
//
// Every wait is bounded: mbar_wait gives up after `kWaitCycles` SM clock cycles
// (about two seconds) and returns false, so a kernel can record a status, stop
// issuing and return instead of hanging the GPU.
#pragma once
#include <cuda.h>
#include <cstdint>

namespace pb {
namespace tma {

constexpr long long kWaitCycles = 4000000000ll; // ~2 s at 1.9 GHz

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
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

// Bounded wait: false when the phase did not complete within kWaitCycles.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity))
    return true;
  const long long start = clock64();
  while (!mbar_try_wait(bar, parity))
    if (clock64() - start > kWaitCycles)
      return false;
  return true;
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// A 2-D tile of `map` at element coordinates (x, y) into this CTA's shared memory,
// completing `bar`'s transaction count.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

} // namespace tma

// Host: a 2-D FP32 tensor map over `outer` rows of `inner` elements whose rows start
// `row_bytes` apart (a multiple of 16), read in boxes of box_inner x box_outer
// elements, with the 128-byte swizzle (box_inner * 4 == 128) or none; elements
// outside the tensor read as zero. False when the driver entry point is missing or
// rejects the layout. Defined in gemm_tf32x3.cu.
bool encode_map_2d(CUtensorMap *map, const void *base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                   uint32_t box_inner, uint32_t box_outer, bool swizzle_128b);

} // namespace pb
