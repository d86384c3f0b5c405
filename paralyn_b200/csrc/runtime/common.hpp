// Internal types shared by the C-ABI layer, the CUDA engine and the kernels.
#pragma once
#include "paralyn/native.h"
#include "paralyn/tensor.h"
#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#define PB_EXPORT extern "C" __attribute__((visibility("default")))

namespace pb {

// Backend-level error classes; the ABI layer maps them to pr_status exactly as
// the reference maps its backend codes (runtime/native.cpp:164-184).
enum class Code { invalid_value, invalid_device, invalid_handle, out_of_memory, unsupported,
                  compilation, execution, internal };

struct Error : std::runtime_error {
  Code code;
  Error(Code c, const std::string &message) : std::runtime_error(message), code(c) {}
};

// A failure that already carries its public status.
struct Failure : std::runtime_error {
  pr_status status;
  Failure(pr_status s, const std::string &message) : std::runtime_error(message), status(s) {}
};

[[noreturn]] inline void fail(pr_status status, const std::string &message) {
  throw Failure(status, message);
}
inline void require(bool ok, pr_status status, const char *message) {
  if (!ok)
    throw Failure(status, message);
}
[[noreturn]] inline void error(Code code, const std::string &message) { throw Error(code, message); }

inline pr_status status_of(Code code) {
  switch (code) {
  case Code::invalid_value: return PR_INVALID_ARGUMENT;
  case Code::invalid_device: return PR_DEVICE_UNAVAILABLE;
  case Code::invalid_handle: return PR_INVALID_HANDLE;
  case Code::out_of_memory: return PR_OUT_OF_MEMORY;
  case Code::unsupported: return PR_UNSUPPORTED;
  case Code::compilation: return PR_COMPILATION_FAILED;
  case Code::execution: return PR_EXECUTION_FAILED;
  case Code::internal: return PR_INTERNAL_ERROR;
  }
  return PR_INTERNAL_ERROR;
}

enum class Scalar : uint32_t { I32 = 0, U32 = 1, F32 = 2 };

struct Dim3 {
  uint32_t x = 1, y = 1, z = 1;
};

// One parameter of a kernel entry as reported by pr_kernel_parameter.
struct Param {
  std::string name;
  Scalar type = Scalar::F32;
  bool buffer = false;
  pr_access access = PR_READ;
};

} // namespace pb
