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
 *  AUTO:      TF32X3 where the shape qualifies (k >= 64), otherwise FFMA. When an
 *             operand holds +-inf (or a finite value whose TF32 high part rounds
 *             to infinity), the command recomputes C with FFMA on the GPU (a guarded
 *             kernel that does nothing otherwise; no host synchronization), so +-inf
 *             propagate as in the reference's IEEE order.
 *  REFERENCE: sum = fl(sum + fl(a*b)) in increasing k, bit-exact with the
 *             reference's sequential checker (half the FFMA rate).
 *  FFMA:      sum = fma(a, b, sum) in increasing k.
 *  TF32X3:    a = a_hi + a_lo, b = b_hi + b_lo split into TF32 on the fly;
 *             a_hi*b_hi + a_hi*b_lo + a_lo*b_hi on tcgen05 tensor cores with FP32
 *             accumulation in tensor memory; declines (falls back to FFMA) for
 *             shapes it does not cover. An infinite operand's low half is
 *             inf - inf, so outputs it reaches are NaN in this mode.
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

/* ---- Row-sharded outputs gathered over NVLink ----
 * One process drives one GPU. To gather the rows every rank computes into one
 * [rows, columns] tensor on every GPU, each rank exports its gathered buffer
 * (pr_b200_buffer_export: a CUDA IPC handle plus the size, 72 bytes, passed to the
 * other ranks by any host channel) and imports the others' (pr_b200_buffer_import:
 * a buffer handle of the importing context that refers to the peer GPU's memory).
 * pr_b200_layer_norm_gather_f32 then normalizes the local rows and writes each
 * output row both to op->out and, at row row_offset + i, into every tensor of
 * `gathered` (local and imported): a fused LayerNorm + all-gather in one kernel
 * whose stores cross NVLink directly. The gathered tensors are complete once every
 * rank's command has completed (the kernel ends with a system-scope fence); the
 * ranks synchronize on the host before reading them. */
#define PR_B200_PEER_HANDLE_BYTES 72u
#define PR_B200_MAX_GATHER 8u
pr_status pr_b200_buffer_export(pr_buffer buffer, void *handle);
pr_status pr_b200_buffer_import(pr_context context, const void *handle, pr_buffer *out);
pr_status pr_b200_layer_norm_gather_f32(pr_queue queue, pr_module operators, const pr_layer_norm_v1 *op,
                                        const pr_tensor_desc_v1 *const *gathered, uint32_t count,
                                        uint64_t row_offset, pr_event *out);
/* The same gathered output for any row-sharded result, e.g. a GEMM shard's C (the
 * reference has no multi-GPU operators; this is the optional all-gather of the
 * row-sharded path): one kernel reads `local` [rows, columns] once and writes it at
 * rows [row_offset, row_offset + rows) of every tensor of `gathered` (contiguous
 * [R_total, columns], local or imported) with plain stores, 128-bit where aligned.
 * A gathered tensor may hold `local` exactly at those rows; any other overlap of
 * `local` or between gathered tensors is rejected (PR_INVALID_ARGUMENT for
 * overlapping bytes, PR_UNSUPPORTED for a shared allocation). Completion as for the
 * gathered LayerNorm: the kernel ends with a system-scope fence and the ranks
 * synchronize on the host before reading. */
pr_status pr_b200_gather_rows_f32(pr_queue queue, const pr_tensor_desc_v1 *local,
                                  const pr_tensor_desc_v1 *const *gathered, uint32_t count, uint64_t row_offset,
                                  pr_event *out);

/* ---- Stream-ordered host copies (no counterpart in the reference) ----
 * pr_buffer_write / pr_buffer_read drain the queue and block, as the reference
 * specifies. These two enqueue the copy as a command of `queue` and return at
 * once. A copy starts after every earlier command of the queue that touches the
 * same bytes of the buffer with at least one of the two writing them, and later
 * commands that touch those bytes in that way start after it; commands on other
 * bytes run concurrently with it (copies use the GPU's copy engines, one lane per
 * direction), so uploading the next slice of an input, computing on the current
 * one and downloading the previous result overlap. The host memory must stay
 * valid (and, for a write, unchanged) until the event completes; the copy only
 * overlaps when the host memory is page-locked (pr_b200_host_register, or memory
 * from cudaHostAlloc). bytes == 0 gives *event = 0 and enqueues nothing; a range
 * past the buffer's end is PR_OUT_OF_BOUNDS. */
pr_status pr_b200_buffer_write_async(pr_queue queue, pr_buffer buffer, uint64_t offset,
                                     const void *source, uint64_t bytes, pr_event *event);
pr_status pr_b200_buffer_read_async(pr_queue queue, pr_buffer buffer, uint64_t offset,
                                    void *destination, uint64_t bytes, pr_event *event);
/* Page-locks (and unlocks) a caller-owned host range for every device
 * (cudaHostRegister, portable); registering the same range twice is
 * PR_INVALID_ARGUMENT. */
pr_status pr_b200_host_register(void *pointer, uint64_t bytes);
pr_status pr_b200_host_unregister(void *pointer);

/* C = activation(op(A) op(B) + bias[column]) as one command (no counterpart in the
 * reference, which takes two: pr_matmul_f32 then pr_bias_activation_f32). The
 * record, validation order and statuses are pr_matmul_f32's; `bias` (may be NULL) is
 * a contiguous [n] tensor not aliasing C; activation is a pr_activation value. The
 * bias add and activation run in the GEMM epilogue, so C is written once, and the
 * result equals the two-command sequence bit for bit in every matmul mode. */
pr_status pr_b200_matmul_bias_activation_f32(pr_queue queue, pr_module operators, const pr_matmul_v1 *op,
                                             const pr_tensor_desc_v1 *bias, uint32_t activation,
                                             pr_event *event);

/* Prepared right-hand operands (no counterpart in the reference, whose
 * pr_matmul_f32, runtime/tensor.cpp:755-798, reads B as given on every call). A
 * product C = op(A) B whose B is reused across many calls (a weight matrix) can give
 * B once to pr_b200_matmul_prepare_f32, which writes B's prepared form (the TF32 pair
 * the tensor-core kernels read, plus B itself as [k][n]) into a caller-owned tensor,
 * and then call pr_b200_matmul_prepared_f32 instead of pr_matmul_f32: the call then
 * skips the per-call split pass over B.
 *
 * pr_b200_matmul_prepared_bytes(k, n): the prepared form's size in bytes (a multiple
 * of 4), 0 when k or n is 0 or above INT32_MAX.
 *
 * pr_b200_matmul_prepare_f32: b is a contiguous [k, n] tensor ([n, k] with
 * transpose_b = 1); `prepared` is a contiguous 1-D tensor of exactly
 * prepared_bytes(k, n) / 4 elements whose byte offset is a multiple of 256, in an
 * allocation other than b's (PR_INVALID_ARGUMENT otherwise; PR_UNSUPPORTED for
 * non-contiguous views, as pr_matmul_f32). It enqueues one command that writes the
 * prepared form; later changes to b do not reach it.
 *
 * pr_b200_matmul_prepared_f32: pr_matmul_f32's record, validation order and statuses,
 * except that op->b is the prepared tensor (prepared for op->k and op->n) and
 * op->transpose_b must be 0. The result equals pr_matmul_f32 with the B the tensor was
 * prepared from, bit for bit, in every matmul mode (REFERENCE and FFMA read the [k][n]
 * copy; AUTO propagates infinities of B as pr_matmul_f32 does). A tensor prepared for
 * another (k, n), or not prepared at all, makes the command fail with
 * PR_EXECUTION_FAILED when it runs (C is then undefined). The prepared tensor may be
 * read by any number of products at once; writing into it while products that read
 * it are queued is ordered like any other buffer access on the queue. */
uint64_t pr_b200_matmul_prepared_bytes(uint64_t k, uint64_t n);
pr_status pr_b200_matmul_prepare_f32(pr_queue queue, pr_module operators, const pr_tensor_desc_v1 *b,
                                     uint32_t transpose_b, const pr_tensor_desc_v1 *prepared, pr_event *event);
pr_status pr_b200_matmul_prepared_f32(pr_queue queue, pr_module operators, const pr_matmul_v1 *op,
                                      pr_event *event);
/* pr_b200_matmul_prepared_f32 with pr_b200_matmul_bias_activation_f32's epilogue: C =
 * activation(op(A) B + bias[column]) with B's prepared form in op->b. Validation is
 * the prepared product's, then bias (may be NULL: a contiguous [n] tensor not
 * aliasing C) with the operands and activation with the record's scalars; the result
 * equals pr_b200_matmul_bias_activation_f32 with the B the tensor was prepared from,
 * bit for bit, in every matmul mode. */
pr_status pr_b200_matmul_prepared_bias_activation_f32(pr_queue queue, pr_module operators, const pr_matmul_v1 *op,
                                                      const pr_tensor_desc_v1 *bias, uint32_t activation,
                                                      pr_event *event);

/* Failure-path probe (no counterpart in the reference). Enqueues a one-thread
 * kernel that waits on a shared-memory barrier nothing completes and gives up after
 * `cycles` SM clock cycles (1 .. 4e9), exactly as the library's TMA and tensor-core
 * kernels give up a stalled wait: it records a status code in the context's status
 * word and returns, and the command fails with PR_EXECUTION_FAILED ("abandoned a
 * bounded wait"). The context's failure is then sticky, as after any failed command.
 * The GPU itself is left healthy. */
pr_status pr_b200_selftest_bounded_wait(pr_queue queue, uint64_t cycles, pr_event *event);

/* Enqueues a command that keeps the queue's device work waiting for `nanoseconds`
 * (at most 1e9; PR_INVALID_ARGUMENT otherwise) by the device's own timer and then
 * completes (no counterpart in the reference). Commands enqueued behind it start only
 * after it, so a caller can enqueue a run of short commands while it lasts and have
 * them run back to back: their device time (pr_b200_marker / pr_b200_event_elapsed
 * around them) then excludes the host's enqueue gaps, as the reference's GPU
 * command-buffer timing does. One thread of one block; the rest of the GPU is idle. */
pr_status pr_b200_queue_hold(pr_queue queue, uint64_t nanoseconds, pr_event *event);

/* Enqueues an empty command whose only effect is a device timestamp on the
 * context queue; it follows every earlier command, copies included.
 * pr_b200_event_elapsed returns the device time between the
 * completion of `first` and of `second` (markers or any commands of one context),
 * waiting for both. Used to time a region of queued work on the device. */
pr_status pr_b200_marker(pr_queue queue, pr_event *out);
pr_status pr_b200_event_elapsed(pr_event first, pr_event second, double *seconds);

/* C[m,n] = op(A) op(B) with the 3xTF32 tensor-core kernel, for callers that cannot
 * allocate device memory. No counterpart in the reference ABI.
 *
 * Who needs it: a host framework that owns all device memory and hands a plug-in
 * only input and output pointers, or a latency-critical loop that must not call
 * cudaMalloc (which can synchronize the device). pr_matmul_f32 needs a scratch
 * workspace for the split operands and grows it with cudaMalloc; this entry point
 * instead uses one fixed 64 MiB array compiled into the library (every GPU that
 * loads the library holds it until the process exits) and calls no allocator.
 *
 * a, b, c are device pointers of the calling thread's current device; A is stored
 * [m,k] (or [k,m] with transpose_a), B [k,n] (or [n,k] with transpose_b), C [m,n];
 * lda, ldb, ldc are the row strides in elements of the stored matrices. The work
 * is enqueued on `stream` (a cudaStream_t; NULL is the legacy default stream) and
 * the call returns without waiting. `status` (optional) is a device-accessible
 * int32 that a kernel sets non-zero if it abandoned a bounded wait (C is then only
 * partly written); the caller clears it and reads it after the stream completes.
 * With status NULL such a failure cannot be detected: the call has already
 * returned PR_SUCCESS and nothing reports the timeout later, so pass a status word
 * wherever a partly written C must not go unnoticed.
 *
 * Limits: 16 <= k, 1 <= m, n, and 8 * round_up(k,32) * (round_up(m,128) +
 * round_up(n,256)) <= 64 MiB (e.g. 1024 x 1024 x 4096 or 2048^3); larger shapes are
 * rejected with PR_OUT_OF_BOUNDS. Every call shares the one array and overwrites
 * the part it reads before reading it, so nothing carries over between calls;
 * calls that overlap on the GPU (other streams, other threads) race on it.
 * The first call on each device looks up the array's device address
 * (cudaGetSymbolAddress) with that device current; make that first call before
 * any stream capture. The address is kept for the life of the process: after
 * cudaDeviceReset (or anything else that destroys and recreates the device's
 * primary context) it is stale, so do not call this entry point on that device
 * again in the same process. Results satisfy |err| <= 2*k*2^-24*sum|a||b|, like
 * PR_B200_MATMUL_TF32X3 in pr_matmul_f32. */
pr_status pr_b200_matmul_tf32x3_static_f32(const float *a, const float *b, float *c, uint64_t m, uint64_t n,
                                           uint64_t k, uint64_t lda, uint64_t ldb, uint64_t ldc,
                                           uint32_t transpose_a, uint32_t transpose_b, void *stream,
                                           int32_t *status);

/* Parses and verifies a module artifact without a device, as pr_module_load
 * would, and writes "kernel=implementation;" for each entry into report
 * (NUL-terminated, truncated to capacity). Same statuses as pr_module_load:
 * PR_COMPILATION_FAILED for malformed or unverifiable IR, PR_UNSUPPORTED for a
 * kernel this library has no native implementation of. */
pr_status pr_b200_module_inspect(const void *data, uint64_t bytes, char *report, uint64_t capacity);

#ifdef __cplusplus
}
#endif
#endif
