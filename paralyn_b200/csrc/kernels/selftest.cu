// Probe of the bounded-wait failure path (pr_b200_selftest_bounded_wait).
//
// Every spin-wait in this library's kernels gives up after a fixed number of SM
// clock cycles, records a status code in the context's host-mapped status word and
// returns; the engine then fails the command. This kernel exercises exactly that
// path without a fault: one thread waits on a shared-memory mbarrier that nothing
// ever arrives at, gives up after the requested number of cycles and records the
// probe's status code.
#include "../runtime/builtin.hpp"

namespace pb {
namespace {

constexpr int STATUS_PROBE_TIMEOUT = 0x7f3fff;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__global__ void bounded_wait_probe(int *status, long long cycles) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&bar)));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x != 0)
    return;
  const long long start = clock64();
  for (;;) {
    uint32_t done;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n"
                 " selp.u32 %0, 1, 0, p;\n}\n"
                 : "=r"(done)
                 : "r"(smem_u32(&bar))
                 : "memory");
    if (done) // cannot happen: no thread arrives
      return;
    if (clock64() - start > cycles) {
      atomicExch(status, STATUS_PROBE_TIMEOUT);
      return;
    }
  }
}

} // namespace

// args: cycles (lo, hi u32 halves)
void launch_selftest_bounded_wait(Launch &L) {
  const long long cycles = (long long)(uint64_t(L.args[0].u32()) | uint64_t(L.args[1].u32()) << 32);
  if (cycles < 1 || cycles > 4000000000ll)
    throw Failure(PR_INVALID_ARGUMENT, "cycles must be in [1, 4e9]");
  if (L.dry_run)
    return;
  bounded_wait_probe<<<1, 32, 0, L.stream>>>(L.status, cycles);
  L.kernels = 1;
  L.variant = "bounded_wait_probe";
}

} // namespace pb
