// 3xTF32 tensor-core GEMM (tcgen05) — not yet part of this build; the launcher
// declines every shape so matmul falls back to the SIMT FFMA kernel.
#include "../runtime/builtin.hpp"

namespace pb {
bool launch_tf32x3_gemm(Launch &, const float *, const float *, float *, int64_t, int64_t, int64_t,
                        int64_t, int64_t, int64_t, bool, bool) {
  return false;
}
} // namespace pb
