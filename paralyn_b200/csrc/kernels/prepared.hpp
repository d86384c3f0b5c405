// The prepared form of a matmul's right-hand operand B (k rows, n columns): what the
// GEMM kernels read of B, made once for a B that many products reuse (a weight
// matrix), so that those products skip B's TF32 split.
//
// Layout of the caller's prepared tensor (a 1-D FP32 view starting on a 256-byte
// boundary, bytes(k, n) bytes long):
//   [0, 256)          Header (written by the prepare command)
//   [256, +raw)       B itself as [k][n] row-major FP32 (whatever B's stored
//                     orientation was), for the FFMA and reference-order kernels and
//                     the AUTO mode's recomputation of operands holding an infinity
//   hi, lo            B^T's TF32 pair, each [n_pad][k_pad] with zero padding, as the
//                     split pass writes it for the tensor-core kernels
// raw is 4*k*n rounded up to 256 bytes; n_pad = n rounded up to 256 (every tile width
// and the CTA-pair tile divide it), k_pad = k rounded up to 32.
#pragma once
#include <cstdint>

namespace pb {
namespace prepared {

constexpr uint64_t kHeaderBytes = 256;
constexpr uint32_t kMagic = 0x33425250u; // "PRB3"
constexpr uint32_t kVersion = 1;
// Status word value of a product whose prepared operand was not made for its (k, n).
constexpr int status_mismatch = 0x7f3f02;

struct Header {
  uint32_t magic, version;
  uint64_t k, n, k_pad, n_pad;
  unsigned long long nonfinite; // nonzero: some element's TF32 high part is infinite
};
static_assert(sizeof(Header) <= kHeaderBytes, "header fits its slot");

inline uint64_t round_up(uint64_t x, uint64_t m) { return (x + m - 1) / m * m; }
inline uint64_t k_pad(uint64_t k) { return round_up(k, 32); }
inline uint64_t n_pad(uint64_t n) { return round_up(n, 256); }
inline uint64_t raw_bytes(uint64_t k, uint64_t n) { return round_up(4 * k * n, 256); }
// 0 when there is no prepared form: k or n is 0 or above INT32_MAX.
inline uint64_t bytes(uint64_t k, uint64_t n) {
  if (!k || !n || k > 0x7fffffffu || n > 0x7fffffffu)
    return 0;
  return kHeaderBytes + raw_bytes(k, n) + 8 * n_pad(n) * k_pad(k);
}
inline uint64_t raw_offset() { return kHeaderBytes; }
inline uint64_t hi_offset(uint64_t k, uint64_t n) { return kHeaderBytes + raw_bytes(k, n); }
inline uint64_t lo_offset(uint64_t k, uint64_t n) { return hi_offset(k, n) + 4 * n_pad(n) * k_pad(k); }

} // namespace prepared

// Device pointers of one prepared operand (kernel-side view).
struct PreparedB {
  const prepared::Header *header = nullptr;
  const float *raw = nullptr, *hi = nullptr, *lo = nullptr;
  uint64_t k = 0, n = 0;
};

} // namespace pb
