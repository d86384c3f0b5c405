/* Additive entry points of the B200 build (no counterpart in the reference ABI;
 * the reference symbols in native.h and tensor.h are unchanged).
 *
 * All of them follow the native.h conventions: a pr_status result, pr_last_error
 * on failure, the global API lock, and ordering on the context's one queue. */
#ifndef PARALYN_B200_H
#define PARALYN_B200_H
#include "paralyn/tensor.h"
#ifdef __cplusplus
extern "C" {
#endif

/* Summation mode of pr_matmul_f32 on one context. The initial mode comes from
 * PARALYN_MATMUL_MODE (reference | ffma | tf32x3 | auto) at context creation.
 *  AUTO:      TF32X3 where the shape qualifies (k >= 64), otherwise FFMA.
 *  REFERENCE: sum = fl(sum + fl(a*b)) in increasing k, bit-exact with the
 *             reference's sequential checker (half the FFMA rate).
 *  FFMA:      sum = fma(a, b, sum) in increasing k.
 *  TF32X3:    a = a_hi + a_lo, b = b_hi + b_lo split into TF32 on the fly;
 *             a_hi*b_hi + a_hi*b_lo + a_lo*b_hi on tcgen05 tensor cores with FP32
 *             accumulation in tensor memory; declines (falls back to FFMA) for
 *             shapes it does not cover.
 * FFMA and TF32X3 results satisfy |err| <= 2*k*2^-24*sum_p |a_ip||b_pj|. */
typedef enum pr_b200_matmul_mode {
  PR_B200_MATMUL_AUTO = 0,
  PR_B200_MATMUL_REFERENCE = 1,
  PR_B200_MATMUL_FFMA = 2,
  PR_B200_MATMUL_TF32X3 = 3
} pr_b200_matmul_mode;
pr_status pr_b200_matmul_mode_set(pr_context context, uint32_t mode);
pr_status pr_b200_matmul_mode_get(pr_context context, uint32_t *mode);

/* Fills a contiguous FP32 tensor with a seeded synthetic stream on the device
 * (SplitMix64; see paralyn_b200/csrc/kernels/synthetic.cu for the exact map).
 * distribution 0: p0 * Uniform[-1, 1); 1: Normal(mean p0, deviation p1).
 * first_draw skips that many 64-bit draws, so row shards can generate their rows
 * of one global stream independently. *out = 0 for an empty tensor. */
#define PR_B200_UNIFORM 0u
#define PR_B200_NORMAL 1u
pr_status pr_b200_fill_synthetic_f32(pr_queue queue, const pr_tensor_desc_v1 *out, uint64_t seed,
                                     uint64_t first_draw, uint32_t distribution, float p0, float p1,
                                     pr_event *event);

/* Device kernels this context has completed (every pr_launch may run several);
 * waits for the queue first. */
pr_status pr_b200_device_kernel_count(pr_context context, uint64_t *out);

/* Enqueues an empty command whose only effect is a device timestamp on the
 * context queue. pr_b200_event_elapsed returns the device time between the
 * completion of `first` and of `second` (markers or any commands of one context),
 * waiting for both. Used to time a region of queued work on the device. */
pr_status pr_b200_marker(pr_queue queue, pr_event *out);
pr_status pr_b200_event_elapsed(pr_event first, pr_event second, double *seconds);

/* Parses and verifies a module artifact without a device, as pr_module_load
 * would, and writes "kernel=implementation;" for each entry into report
 * (NUL-terminated, truncated to capacity). Same statuses as pr_module_load:
 * PR_COMPILATION_FAILED for malformed or unverifiable IR, PR_UNSUPPORTED for a
 * kernel this build has no native implementation of. */
pr_status pr_b200_module_inspect(const void *data, uint64_t bytes, char *report, uint64_t capacity);

#ifdef __cplusplus
}
#endif
#endif
