// Run-time compiled kernels for verified IR that no built-in kernel implements.
//
// The reference's CUDA backend turns every verified IR kernel into CUDA C++ and
// compiles it with NVRTC (backends/cuda/engine.cpp:485-580, compiler/codegen/
// cuda.cpp). Here that path serves only IR outside the native built-ins: the
// kernel is emitted with the same numerical policy (FP32 + and * as __fadd_rn and
// __fmul_rn, no contraction, no flush to zero, IEEE division and square root),
// compiled once per process straight to an sm_100a cubin, and loaded per device.
// Unlike the reference, every load and store is checked against the element count
// of its bound view: an access outside it is skipped (loads read 0) and the
// command fails with an out-of-view status instead of touching other memory.
#pragma once
#include "module.hpp"
#include <map>
#include <mutex>

namespace pb {

struct JitKernel {
  std::string name, entry, source;
  std::vector<IrParam> params;
  std::vector<char> cubin;
  double compile_seconds = 0;
  std::mutex mutex;
  std::map<int, std::pair<void *, void *>> loaded; // device -> (CUmodule, CUfunction)
  ~JitKernel();
  // The function on `device` (loaded on first use, with that device current).
  void *function(int device);
};

// CUDA C++ for `kernel` (verified IR) with bounds-checked buffer accesses.
std::string emit_ir_cuda(const IrKernel &kernel);
// Emits and compiles; Failure(PR_COMPILATION_FAILED) on a compiler error,
// Failure(PR_UNSUPPORTED) when NVRTC cannot be loaded. Identical sources share
// one compilation per process.
std::shared_ptr<JitKernel> compile_ir(const IrKernel &kernel);
// The built-in entry every run-time compiled kernel launches through.
const Builtin &jit_builtin();
// Status word value a compiled kernel writes when it skipped an out-of-view access.
constexpr int status_out_of_view = 0x7f3f01;

} // namespace pb
