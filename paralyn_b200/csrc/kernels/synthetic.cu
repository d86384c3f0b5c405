// Seeded synthetic inputs, generated on the device.
//
// Stream: SplitMix64 with state seed; draw d (0-based) is mix(seed + (d+1)*G) with
// G = 0x9E3779B97F4A7C15 and the standard SplitMix64 finalizer, so any range of
// draws can be produced independently (row shards generate only their rows).
//   distribution 0, uniform: value = p0 * u with u = (int(draw >> 40) - 2^23) * 2^-23,
//                  a 24-bit dyadic value in [-1, 1) (exact in FP32);
//   distribution 1, normal:  sample i uses draws 2i and 2i+1 after first_draw:
//                  u1 = ((d0 >> 11) + 1) * 2^-53, u2 = (d1 >> 11) * 2^-53,
//                  value = float(p0 + p1 * sqrt(-2 ln u1) * cos(2 pi u2)) (Box-Muller
//                  in double, rounded once).
// paralyn_b200/synthetic.py is the host version of the same stream.
#include "../runtime/builtin.hpp"
#include <algorithm>

namespace pb {
namespace {

__device__ __forceinline__ uint64_t splitmix_draw(uint64_t seed, uint64_t draw) {
  uint64_t z = seed + (draw + 1) * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__global__ void __launch_bounds__(256) synthetic_kernel(float *out, uint64_t count, uint64_t seed,
                                                        uint64_t first, uint32_t distribution,
                                                        float p0, float p1) {
  const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
  for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += stride) {
    if (distribution == 0) {
      const uint64_t d = splitmix_draw(seed, first + i);
      const float u = float(int32_t(d >> 40) - 8388608) * 1.1920928955078125e-7f; // 2^-23
      out[i] = __fmul_rn(p0, u);
    } else {
      const uint64_t d0 = splitmix_draw(seed, first + 2 * i), d1 = splitmix_draw(seed, first + 2 * i + 1);
      const double u1 = double((d0 >> 11) + 1) * 0x1.0p-53, u2 = double(d1 >> 11) * 0x1.0p-53;
      const double v = sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
      out[i] = float(double(p0) + double(p1) * v);
    }
  }
}

} // namespace

void launch_synthetic(cudaStream_t stream, float *out, uint64_t count, uint64_t seed,
                      uint64_t first_draw, uint32_t distribution, float p0, float p1, int sm_count) {
  if (!count)
    return;
  const uint64_t blocks = std::min<uint64_t>((count + 255) / 256, uint64_t(sm_count) * 16);
  synthetic_kernel<<<uint32_t(blocks), 256, 0, stream>>>(out, count, seed, first_draw, distribution, p0, p1);
}

} // namespace pb
