// Queue hold (pr_b200_queue_hold): one thread that lets the device do nothing for a
// given time, read from the global nanosecond timer, and then returns. Commands
// enqueued behind it wait in the queue, so a caller can enqueue a run of short
// commands first and have them execute back to back, measuring their device time
// without the host's enqueue gaps between them (the way a GPU command buffer is
// timed). The wait ends by itself: its length is bounded by the argument (at most
// one second), and it sleeps between timer reads.
#include "../runtime/builtin.hpp"

namespace pb {
namespace {

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__global__ void queue_hold(uint64_t nanoseconds) {
  if (threadIdx.x != 0)
    return;
  const uint64_t start = global_ns();
  while (global_ns() - start < nanoseconds)
    __nanosleep(2000);
}

} // namespace

// args: nanoseconds (lo, hi u32 halves), at most 1e9
void launch_queue_hold(Launch &L) {
  const uint64_t ns = uint64_t(L.args[0].u32()) | uint64_t(L.args[1].u32()) << 32;
  if (ns > 1000000000ull)
    throw Failure(PR_INVALID_ARGUMENT, "A hold lasts at most 1e9 ns");
  if (L.dry_run)
    return;
  queue_hold<<<1, 32, 0, L.stream>>>(ns);
  L.kernels = 1;
  L.variant = "queue_hold";
}

} // namespace pb
