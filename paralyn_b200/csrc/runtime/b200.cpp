// Additive entry points declared in paralyn/b200.h.
#include "abi_internal.hpp"
#include "jit.hpp"
#include "paralyn/b200.h"
#include <cstring>
#include <limits>

namespace pb {
namespace {

uint32_t low(uint64_t v) { return uint32_t(v); }
uint32_t high(uint64_t v) { return uint32_t(v >> 32); }

// (out view, seed lo, seed hi, first lo, first hi, distribution, p0, p1)
void launch_synthetic_entry(Launch &L) {
  if (L.dry_run)
    return;
  const auto &a = L.args;
  const uint64_t seed = uint64_t(a[1].u32()) | uint64_t(a[2].u32()) << 32;
  const uint64_t first = uint64_t(a[3].u32()) | uint64_t(a[4].u32()) << 32;
  launch_synthetic(L.stream, static_cast<float *>(a[0].ptr), a[0].bytes / 4, seed, first,
                   a[5].u32(), a[6].f32(), a[7].f32(), L.sm_count);
  L.kernels = 1;
  L.variant = a[5].u32() ? "normal" : "uniform";
}

BoundArg scalar(uint32_t bits) {
  BoundArg a;
  a.bits = bits;
  return a;
}
BoundArg scalar_f32(float v) {
  BoundArg a;
  std::memcpy(&a.bits, &v, 4);
  return a;
}

} // namespace
} // namespace pb

using namespace pb;

PB_EXPORT pr_status pr_b200_matmul_mode_set(pr_context context, uint32_t mode) {
  return api("b200_matmul_mode_set", [&] {
    auto engine = context_engine(context);
    require(mode <= PR_B200_MATMUL_TF32X3, PR_INVALID_ARGUMENT, "Unknown matmul mode");
    engine->set_matmul_mode(mode);
  });
}

PB_EXPORT pr_status pr_b200_matmul_mode_get(pr_context context, uint32_t *mode) {
  return api("b200_matmul_mode_get", [&] {
    require(mode, PR_INVALID_ARGUMENT, "Missing mode output");
    *mode = context_engine(context)->matmul_mode();
  });
}

PB_EXPORT pr_status pr_b200_device_kernel_count(pr_context context, uint64_t *out) {
  return api("b200_device_kernel_count", [&] {
    require(out, PR_INVALID_ARGUMENT, "Missing count output");
    auto engine = context_engine(context);
    engine->synchronize();
    *out = engine->statistics().device_kernels;
  });
}

static_assert(sizeof(PeerHandle) == PR_B200_PEER_HANDLE_BYTES, "peer handle size");

PB_EXPORT pr_status pr_b200_buffer_export(pr_buffer buffer, void *handle) {
  return api("b200_buffer_export", [&] {
    require(handle, PR_INVALID_ARGUMENT, "Missing handle output");
    std::shared_ptr<Engine> engine;
    auto allocation = allocation_of(buffer, &engine);
    const PeerHandle h = engine->export_allocation(*allocation);
    std::memcpy(handle, &h, sizeof(h));
  });
}

PB_EXPORT pr_status pr_b200_buffer_import(pr_context context, const void *handle, pr_buffer *out) {
  return api("b200_buffer_import", [&] {
    require(out, PR_INVALID_ARGUMENT, "Missing buffer output");
    *out = 0;
    require(handle, PR_INVALID_ARGUMENT, "Missing peer handle");
    PeerHandle h;
    std::memcpy(&h, handle, sizeof(h));
    auto engine = context_engine(context);
    *out = add_buffer(context, engine->import_allocation(h));
  });
}

PB_EXPORT pr_status pr_b200_buffer_write_async(pr_queue queue, pr_buffer buffer, uint64_t offset,
                                               const void *source, uint64_t bytes, pr_event *out) {
  return api("b200_buffer_write_async", [&] {
    require(out, PR_INVALID_ARGUMENT, "Missing event output");
    *out = 0;
    *out = submit_transfer(queue, buffer, offset, const_cast<void *>(source), bytes, true);
  });
}

PB_EXPORT pr_status pr_b200_buffer_read_async(pr_queue queue, pr_buffer buffer, uint64_t offset,
                                              void *destination, uint64_t bytes, pr_event *out) {
  return api("b200_buffer_read_async", [&] {
    require(out, PR_INVALID_ARGUMENT, "Missing event output");
    *out = 0;
    *out = submit_transfer(queue, buffer, offset, destination, bytes, false);
  });
}

PB_EXPORT pr_status pr_b200_host_register(void *pointer, uint64_t bytes) {
  return api("b200_host_register", [&] {
    require(pointer && bytes, PR_INVALID_ARGUMENT, "Registering host memory needs a pointer and a size");
    const cudaError_t e = cudaHostRegister(pointer, bytes, cudaHostRegisterPortable);
    if (e != cudaSuccess) {
      cudaGetLastError();
      throw Failure(e == cudaErrorHostMemoryAlreadyRegistered ? PR_INVALID_ARGUMENT : PR_DEVICE_UNAVAILABLE,
                    std::string("cudaHostRegister failed: ") + cudaGetErrorString(e));
    }
  });
}

PB_EXPORT pr_status pr_b200_host_unregister(void *pointer) {
  return api("b200_host_unregister", [&] {
    require(pointer, PR_INVALID_ARGUMENT, "Missing host pointer");
    const cudaError_t e = cudaHostUnregister(pointer);
    if (e != cudaSuccess) {
      cudaGetLastError();
      throw Failure(PR_INVALID_ARGUMENT, std::string("cudaHostUnregister failed: ") + cudaGetErrorString(e));
    }
  });
}

namespace pb {
void launch_selftest_bounded_wait(Launch &);
}

PB_EXPORT pr_status pr_b200_selftest_bounded_wait(pr_queue queue, uint64_t cycles, pr_event *out) {
  return api("b200_selftest_bounded_wait", [&] {
    require(out, PR_INVALID_ARGUMENT, "Missing event output");
    *out = 0;
    require(cycles >= 1 && cycles <= 4000000000ull, PR_INVALID_ARGUMENT, "cycles must be in [1, 4e9]");
    std::vector<BoundArg> args(2);
    args[0].bits = uint32_t(cycles);
    args[1].bits = uint32_t(cycles >> 32);
    *out = submit_command(queue, "b200_selftest_bounded_wait", launch_selftest_bounded_wait, Dim3{}, Dim3{},
                          std::move(args), {});
  });
}

namespace pb {
void launch_queue_hold(Launch &);
}

PB_EXPORT pr_status pr_b200_queue_hold(pr_queue queue, uint64_t nanoseconds, pr_event *out) {
  return api("b200_queue_hold", [&] {
    require(out, PR_INVALID_ARGUMENT, "Missing event output");
    *out = 0;
    require(nanoseconds <= 1000000000ull, PR_INVALID_ARGUMENT, "A hold lasts at most 1e9 ns");
    std::vector<BoundArg> args(2);
    args[0].bits = uint32_t(nanoseconds);
    args[1].bits = uint32_t(nanoseconds >> 32);
    *out = submit_command(queue, "b200_queue_hold", launch_queue_hold, Dim3{}, Dim3{}, std::move(args), {});
  });
}

PB_EXPORT pr_status pr_b200_marker(pr_queue queue, pr_event *out) {
  return api("b200_marker", [&] {
    require(out, PR_INVALID_ARGUMENT, "Missing event output");
    *out = 0;
    *out = submit_marker(queue);
  });
}

PB_EXPORT pr_status pr_b200_event_elapsed(pr_event first, pr_event second, double *seconds) {
  return api("b200_event_elapsed", [&] {
    require(seconds, PR_INVALID_ARGUMENT, "Missing seconds output");
    *seconds = event_elapsed(first, second);
  });
}

PB_EXPORT pr_status pr_b200_module_inspect(const void *data, uint64_t bytes, char *report,
                                           uint64_t capacity) {
  return api("b200_module_inspect", [&] {
    require(data || !bytes, PR_INVALID_ARGUMENT, "Null module data");
    require(bytes <= prk_max_bytes, PR_COMPILATION_FAILED, "Module artifact exceeds 16 MiB limit");
    std::string text;
    static const unsigned char executable_magic[8] = {'P', 'A', 'R', 'A', 'L', 'Y', 'N', 'X'};
    if (data && bytes >= 8 && std::memcmp(data, executable_magic, 8) == 0)
      fail(PR_UNSUPPORTED, "MSL executable modules are Metal-specific; the CUDA backend accepts "
                           "verified IR modules only");
    if (is_provider_artifact(data, bytes)) {
      for (const auto &b : provider_builtins())
        text += std::string(b.name) + "=" + b.name + ";";
    } else {
      std::vector<IrKernel> kernels;
      try {
        kernels = parse_prk(data, bytes);
      } catch (const std::exception &e) {
        fail(PR_COMPILATION_FAILED, std::string("ParalynError: ") + e.what());
      }
      for (const auto &k : kernels) {
        std::string name = match_ir(k);
        if (name.empty()) { // compiled at load time; compiling here reports compiler errors
          compile_ir(k);
          name = "nvrtc_sm_100a";
        }
        text += k.name + "=" + name + ";";
      }
    }
    if (report && capacity) {
      const size_t n = std::min<size_t>(text.size(), capacity - 1);
      std::memcpy(report, text.data(), n);
      report[n] = 0;
    }
  });
}

PB_EXPORT pr_status pr_b200_fill_synthetic_f32(pr_queue queue, const pr_tensor_desc_v1 *out,
                                               uint64_t seed, uint64_t first_draw,
                                               uint32_t distribution, float p0, float p1,
                                               pr_event *event) {
  return api("b200_fill_synthetic_f32", [&] {
    require(event, PR_INVALID_ARGUMENT, "Missing event output");
    *event = 0;
    require(out, PR_INVALID_ARGUMENT, "Missing tensor descriptor");
    require(out->version == PR_TENSOR_VERSION_1 && out->struct_size == sizeof(pr_tensor_desc_v1),
            PR_INVALID_ARGUMENT, "Unsupported tensor descriptor");
    require(out->dtype == PR_F32 && out->rank <= PR_TENSOR_MAX_RANK && out->byte_offset % 4 == 0,
            PR_INVALID_ARGUMENT, "Synthetic fill needs an FP32 descriptor with aligned offset");
    require(distribution <= PR_B200_NORMAL, PR_INVALID_ARGUMENT, "Unknown distribution");
    uint64_t count = 1, expected = 1;
    for (uint32_t r = out->rank; r-- > 0;) {
      require(out->shape[r] <= uint64_t(std::numeric_limits<int32_t>::max()), PR_UNSUPPORTED,
              "Tensor too large");
      require(out->shape[r] == 1 || uint64_t(out->strides[r]) == expected, PR_UNSUPPORTED,
              "Synthetic fill needs a contiguous tensor");
      expected *= out->shape[r];
      count *= out->shape[r];
    }
    require(count <= uint64_t(std::numeric_limits<int32_t>::max()), PR_UNSUPPORTED,
            "Tensor too large");
    const QueueAccess q = queue_access(queue);
    auto allocation = buffer_allocation(out->buffer, q.context);
    require(out->byte_offset <= allocation->bytes && count * 4 <= allocation->bytes - out->byte_offset,
            PR_OUT_OF_BOUNDS, "Tensor extent exceeds its buffer");
    if (!count)
      return;
    BoundArg view;
    view.buffer = true;
    view.ptr = static_cast<char *>(allocation->ptr) + out->byte_offset;
    view.bytes = count * 4;
    std::vector<BoundArg> args = {view,
                                  scalar(low(seed)),
                                  scalar(high(seed)),
                                  scalar(low(first_draw)),
                                  scalar(high(first_draw)),
                                  scalar(distribution),
                                  scalar_f32(p0),
                                  scalar_f32(p1)};
    *event = submit_command(queue, "b200_synthetic_f32", launch_synthetic_entry, Dim3{}, Dim3{},
                            std::move(args), {allocation});
  });
}
