// Built-in sm_100a kernels behind pr_launch.
//
// Every kernel a module can expose (the verified-IR array kernels recognised in a
// .prk, and the tensor provider's entries) is one Builtin: a parameter schema, an
// optional required block shape, and a host launcher that turns the caller's
// launch geometry and bound views into the exact element range the reference's
// kernel would touch, checks that every access stays inside its view, and enqueues
// the CUDA kernels on the context stream.
#pragma once
#include "common.hpp"
#include <cuda_runtime.h>
#include <cstring>

namespace pb {

struct BoundArg {
  bool buffer = false;
  bool writes = true;     // the kernel may write the view (false: read-only parameter)
  void *ptr = nullptr;    // device address of the view's first byte
  uint64_t bytes = 0;     // view size
  uint32_t bits = 0;      // scalar payload
  float f32() const {
    float v;
    std::memcpy(&v, &bits, 4);
    return v;
  }
  uint32_t u32() const { return bits; }
  int32_t i32() const {
    int32_t v;
    std::memcpy(&v, &bits, 4);
    return v;
  }
};

// Per-context matmul summation modes (paralyn/b200.h).
enum MatmulMode : uint32_t {
  matmul_auto = 0,
  matmul_reference = 1, // fl(fl(a*b) + sum), strictly increasing k: bit-exact with the reference's sequential checker
  matmul_ffma = 2,      // fma(a, b, sum), strictly increasing k
  matmul_tf32x3 = 3,    // 3xTF32 split products on tcgen05, FP32 accumulation in TMEM
};

// A device word that a 3xTF32 command sets to its epoch when an operand holds a value
// whose TF32 high part is infinite (an infinite input, or a finite one that rounds to
// infinity). A 3xTF32 product of such a value is NaN (its low part is inf - inf),
// where the reference's IEEE order gives +-inf; in AUTO mode the command is then
// recomputed by a guarded FFMA kernel that runs only when the word holds the epoch.
// Epochs are unique per process, so the word needs no reset between commands.
struct NonFiniteFlag {
  unsigned long long *word = nullptr;
  unsigned long long epoch = 0;
};

struct Launch {
  cudaStream_t stream = nullptr;
  int device = 0;
  int sm_count = 148;
  int *status = nullptr;       // host-mapped word kernels set on a bounded-wait timeout
  uint32_t matmul_mode = matmul_auto;
  Dim3 grid, block;            // the caller's launch geometry
  std::vector<BoundArg> args;  // in parameter order
  // Device scratch of at least `bytes`, valid for kernels enqueued on `stream` by
  // this launch (a grow-only per-context workspace); null when unavailable.
  void *(*workspace)(void *owner, size_t bytes) = nullptr;
  void *workspace_owner = nullptr;
  // A second stream of the context for work that overlaps `stream` inside one
  // launch, and four timing-free events to order the two. A launcher that uses it
  // must make `stream` wait for everything it put on `side_stream`.
  cudaStream_t side_stream = nullptr;
  cudaEvent_t side_events[4] = {};
  const void *entry_data = nullptr; // per-entry state (run-time compiled kernels)
  bool dry_run = false;        // validate and plan only; enqueue nothing
  uint32_t kernels = 0;        // device kernels enqueued (filled by the launcher)
  std::string variant;         // which implementation ran (filled by the launcher)
};

using Launcher = void (*)(Launch &);

struct Builtin {
  const char *name;
  uint32_t required_block[3]; // {0,0,0}: any block shape
  std::vector<Param> params;
  Launcher launch;
};

// Provider entries (same names and schemas as the reference's entry table,
// runtime/tensor.cpp:322-371) and the verified-IR array kernels.
const std::vector<Builtin> &provider_builtins();
const Builtin *find_builtin(const std::string &name);

// Launchers implemented in the .cu files.
void launch_ir_add_u32(Launch &);
void launch_ir_add_i32(Launch &);
void launch_ir_affine_u32(Launch &);
void launch_ir_affine_i32(Launch &);
void launch_ir_affine_scalar_u32(Launch &);
void launch_provider_add(Launch &);
void launch_provider_fill(Launch &);
void launch_provider_layer_norm(Launch &);
void launch_provider_matmul(Launch &);
void launch_provider_bias_activation(Launch &);
void launch_provider_activation(Launch &);
void launch_provider_batched_matmul(Launch &);
void launch_provider_batched_fill(Launch &);
void launch_provider_reduce_rows(Launch &);
void launch_provider_softmax_rows(Launch &);

// Synthetic input streams (paralyn/b200.h pr_b200_fill_synthetic_f32).
void launch_synthetic(cudaStream_t stream, float *out, uint64_t count, uint64_t seed,
                      uint64_t first_draw, uint32_t distribution, float p0, float p1,
                      int sm_count);

// Bounds helper for launchers: every view must cover `elements` FP32 values.
inline void need_elements(const BoundArg &view, uint64_t elements, const char *what) {
  if (elements > view.bytes / 4)
    throw Failure(PR_OUT_OF_BOUNDS,
                  std::string("Launch would access ") + std::to_string(elements) + " elements of " +
                      what + " but its view holds " + std::to_string(view.bytes / 4) +
                      "; this backend refuses out-of-view accesses");
}

void cuda_check(cudaError_t result, const char *operation);

} // namespace pb
