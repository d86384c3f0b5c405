// The native C ABI (paralyn/native.h) over the CUDA engine.
//
// Handle, ownership, error and ordering semantics are those of the reference
// runtime (runtime/native.cpp): a registry of never-reused u64 handles (:87-158),
// one global lock around every call (:36, :185-219), thread-local pr_last_error
// cleared on success, release that consumes the handle even when the completion it
// waits for failed (:451-470), and a sticky completion failure that is reported
// once and not repeated by cleanup (:332-352). An atexit handler drains every
// context and terminates with status 1 if a failure was never observed (:91-146).
#include "abi_internal.hpp"
#include "jit.hpp"
#include "paralyn/b200.h"
#include <atomic>
#include <cstdio>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <limits>
#include <mutex>
#include <new>
#include <set>
#include <unordered_map>

static_assert(sizeof(pr_error) == 4 + 64 + 1024, "pr_error layout");
static_assert(offsetof(pr_argument, view) == 8 && offsetof(pr_argument, f32) == 24 &&
                  sizeof(pr_argument) == 32,
              "pr_argument layout");
static_assert(offsetof(pr_parameter_info, type) == 4100 && sizeof(pr_parameter_info) == 4112,
              "pr_parameter_info layout");
static_assert(sizeof(pr_device_info) == 256 + 32 + 128 + 8 + 8 + 8, "pr_device_info layout");
static_assert(sizeof(pr_event_info) == 24, "pr_event_info layout");
static_assert(sizeof(pr_device_capabilities_v1) == 8 + 128 + 32 + 32 + 24, "capabilities layout");
static_assert(sizeof(pr_event_timing_v1) == 48, "pr_event_timing_v1 layout");
static_assert(sizeof(pr_backend_status_v1) == 8 + 32 + 16 + 8 + 512 + 512 + 1024,
              "pr_backend_status_v1 layout");
static_assert(offsetof(pr_tensor_desc_v1, shape) == 32 && sizeof(pr_tensor_desc_v1) == 160,
              "pr_tensor_desc_v1 layout");
static_assert(sizeof(pr_matmul_v1) == 64 && offsetof(pr_matmul_v1, a) == 40, "pr_matmul_v1 layout");
static_assert(sizeof(pr_layer_norm_v1) == 48 && offsetof(pr_layer_norm_v1, x) == 16,
              "pr_layer_norm_v1 layout");
static_assert(sizeof(pr_add_v1) == 32, "pr_add_v1 layout");
static_assert(sizeof(pr_tensor_operators_capabilities_v1) == 56, "capability record layout");

namespace pb {
namespace {

thread_local pr_error last_error{};
std::mutex api_mutex;

struct Object {
  HandleKind kind;
  explicit Object(HandleKind k) : kind(k) {}
  virtual ~Object() = default;
};
struct ContextObj : Object {
  std::shared_ptr<Engine> engine;
  bool completion_failure_observed = false;
  explicit ContextObj(std::shared_ptr<Engine> e) : Object(HandleKind::context), engine(std::move(e)) {}
};
struct BufferObj : Object {
  std::shared_ptr<ContextObj> owner;
  std::shared_ptr<Allocation> allocation;
  BufferObj(std::shared_ptr<ContextObj> c, std::shared_ptr<Allocation> a)
      : Object(HandleKind::buffer), owner(std::move(c)), allocation(std::move(a)) {}
};
struct ViewObj : Object {
  std::shared_ptr<BufferObj> buffer;
  size_t offset, size;
  uint32_t alignment;
  pr_access access;
  ViewObj(std::shared_ptr<BufferObj> b, size_t o, size_t s, uint32_t a, pr_access m)
      : Object(HandleKind::view), buffer(std::move(b)), offset(o), size(s), alignment(a), access(m) {}
};
struct ModuleObj : Object {
  std::shared_ptr<ContextObj> owner;
  std::vector<Entry> entries;
  explicit ModuleObj(std::shared_ptr<ContextObj> c) : Object(HandleKind::module), owner(std::move(c)) {}
};
struct KernelObj : Object {
  std::shared_ptr<ModuleObj> module;
  size_t index;
  KernelObj(std::shared_ptr<ModuleObj> m, size_t i) : Object(HandleKind::kernel), module(std::move(m)), index(i) {}
  const Entry &entry() const { return module->entries[index]; }
};
struct QueueObj : Object {
  std::shared_ptr<ContextObj> owner;
  explicit QueueObj(std::shared_ptr<ContextObj> c) : Object(HandleKind::queue), owner(std::move(c)) {}
};
struct EventObj : Object {
  std::shared_ptr<ContextObj> owner;
  std::shared_ptr<Work> work;
  EventObj(std::shared_ptr<ContextObj> c, std::shared_ptr<Work> w)
      : Object(HandleKind::event), owner(std::move(c)), work(std::move(w)) {}
};
// Opaque payloads of the B200 additions (collective communicators).
struct PayloadObj : Object {
  std::shared_ptr<ContextObj> owner;
  std::shared_ptr<void> payload;
  PayloadObj(HandleKind k, std::shared_ptr<ContextObj> c, std::shared_ptr<void> p)
      : Object(k), owner(std::move(c)), payload(std::move(p)) {}
};

// Never destroyed: contexts are drained by the exit handler, and destroying CUDA
// objects during static destruction would race the CUDA runtime's own teardown.
auto &objects = *new std::unordered_map<pr_handle, std::shared_ptr<Object>>();
pr_handle next_handle = 1;

void shutdown_native() {
  try {
    std::lock_guard<std::mutex> lock(api_mutex);
    std::set<std::shared_ptr<ContextObj>> contexts;
    for (const auto &entry : objects) {
      const auto &o = entry.second;
      switch (o->kind) {
      case HandleKind::context: contexts.insert(std::static_pointer_cast<ContextObj>(o)); break;
      case HandleKind::buffer: contexts.insert(std::static_pointer_cast<BufferObj>(o)->owner); break;
      case HandleKind::view: contexts.insert(std::static_pointer_cast<ViewObj>(o)->buffer->owner); break;
      case HandleKind::module: contexts.insert(std::static_pointer_cast<ModuleObj>(o)->owner); break;
      case HandleKind::kernel:
        contexts.insert(std::static_pointer_cast<KernelObj>(o)->module->owner);
        break;
      case HandleKind::queue: contexts.insert(std::static_pointer_cast<QueueObj>(o)->owner); break;
      case HandleKind::event: contexts.insert(std::static_pointer_cast<EventObj>(o)->owner); break;
      case HandleKind::collective:
        contexts.insert(std::static_pointer_cast<PayloadObj>(o)->owner);
        break;
      }
    }
    std::string failures;
    for (const auto &context : contexts) {
      try {
        context->engine->synchronize();
      } catch (const Error &e) {
        if (e.code != Code::execution || !context->completion_failure_observed)
          failures += std::string(e.what()) + "\n";
      } catch (const std::exception &e) {
        failures += std::string(e.what()) + "\n";
      }
    }
    if (!failures.empty())
      throw std::runtime_error(failures);
  } catch (const std::exception &e) {
    try {
      runtime_event("process_failure", "failed", e.what());
    } catch (...) {
    }
    std::fprintf(stderr, "Paralyn native shutdown failed: %s\n", e.what());
    std::fflush(nullptr);
    std::_Exit(EXIT_FAILURE);
  }
}

void ensure_shutdown() {
  static const bool installed = std::atexit(shutdown_native) == 0;
  require(installed, PR_INTERNAL_ERROR, "Cannot install native shutdown handler");
}

template <class T> std::shared_ptr<T> get(pr_handle h, HandleKind kind) {
  const auto it = objects.find(h);
  require(it != objects.end() && it->second->kind == kind, PR_INVALID_HANDLE,
          "Unknown, released, or wrong-kind handle");
  return std::static_pointer_cast<T>(it->second);
}

pr_handle add(std::shared_ptr<Object> object) {
  require(next_handle != 0, PR_OUT_OF_MEMORY, "Handle identity space exhausted");
  const pr_handle h = next_handle++;
  objects.emplace(h, std::move(object));
  return h;
}

template <size_t N> void text(char (&out)[N], const std::string &value) {
  const size_t n = std::min(N - 1, value.size());
  std::memcpy(out, value.data(), n);
  out[n] = 0;
}

size_t bytes(uint64_t n) {
  require(n <= std::numeric_limits<size_t>::max(), PR_OUT_OF_BOUNDS,
          "Byte count does not fit platform size_t");
  return size_t(n);
}
void range(size_t capacity, uint64_t offset, uint64_t count) {
  require(offset <= capacity && count <= capacity - offset, PR_OUT_OF_BOUNDS,
          "Byte range exceeds allocation");
}

pr_type public_type(Scalar t) {
  switch (t) {
  case Scalar::I32: return PR_I32;
  case Scalar::U32: return PR_U32;
  case Scalar::F32: return PR_F32;
  }
  return PR_F32;
}
Scalar scalar_of(IrType t) {
  switch (t) {
  case IrType::I32: return Scalar::I32;
  case IrType::U32: return Scalar::U32;
  case IrType::F32: return Scalar::F32;
  default: break;
  }
  fail(PR_UNSUPPORTED, "Predicate parameters are not supported");
}

void device_record(const DeviceRecord &d, pr_device_info *out) {
  require(out, PR_INVALID_ARGUMENT, "Missing device-info output");
  *out = {};
  text(out->name, d.name);
  text(out->backend, "CUDA");
  text(out->os, d.os);
  out->registry_id = d.registry_id;
  out->max_buffer_bytes = d.total_memory;
  out->unified_memory = d.integrated;
}

template <class T> void query_record(T *out) {
  require(out, PR_INVALID_ARGUMENT, "Missing versioned query output");
  require(out->version == PR_QUERY_VERSION_1, PR_UNSUPPORTED, "Unsupported query record version");
  require(out->struct_size == sizeof(T), PR_INVALID_ARGUMENT, "Query record size mismatch");
}

void capabilities(const DeviceRecord &d, pr_device_capabilities_v1 *out) {
  query_record(out);
  *out = {};
  out->struct_size = sizeof(*out);
  out->version = PR_QUERY_VERSION_1;
  text(out->stable_id, d.stable_id);
  text(out->backend, "CUDA");
  out->artifact_formats = PR_ARTIFACT_VERIFIED_IR;
  out->scalar_types = PR_SCALAR_I32 | PR_SCALAR_U32 | PR_SCALAR_F32;
  out->max_buffer_bytes = d.total_memory;
  out->max_threadgroup_memory_bytes = d.max_smem_block;
  out->max_block_x = d.max_block.x;
  out->max_block_y = d.max_block.y;
  out->max_block_z = d.max_block.z;
  out->max_buffer_bindings = 31;
  out->unified_memory = d.integrated;
}

std::shared_ptr<ModuleObj> load(const std::shared_ptr<ContextObj> &ctx, const void *data, size_t n) {
  require(data || !n, PR_INVALID_ARGUMENT, "Null module data");
  auto module = std::make_shared<ModuleObj>(ctx);
  static const unsigned char executable_magic[8] = {'P', 'A', 'R', 'A', 'L', 'Y', 'N', 'X'};
  if (data && n >= 8 && std::memcmp(data, executable_magic, 8) == 0)
    fail(PR_UNSUPPORTED, "MSL executable modules are Metal-specific; the CUDA backend accepts "
                         "verified IR modules only");
  if (is_provider_artifact(data, n)) {
    for (const auto &b : provider_builtins())
      module->entries.push_back(Entry{b.name, b.params, &b, nullptr});
    return module;
  }
  std::vector<IrKernel> kernels;
  try {
    kernels = parse_prk(data, n);
  } catch (const std::bad_alloc &) {
    throw;
  } catch (const std::exception &e) {
    fail(PR_COMPILATION_FAILED, std::string("ParalynError: ") + e.what());
  }
  for (const auto &k : kernels) {
    if (k.params.size() > 31)
      fail(PR_UNSUPPORTED, "Kernel exceeds the portable 31-parameter limit");
    const std::string name = match_ir(k);
    Entry entry;
    entry.name = k.name;
    if (name.empty()) { // no native kernel: compile the IR for sm_100a now
      entry.jit = compile_ir(k);
      entry.builtin = &jit_builtin();
      runtime_event("compilation", "completed", k.name, 0);
    } else {
      entry.builtin = find_builtin(name);
    }
    for (size_t i = 0; i < k.params.size(); ++i)
      entry.params.push_back(Param{k.params[i].name, scalar_of(k.params[i].type),
                                   k.params[i].buffer, ir_access(k, i)});
    module->entries.push_back(std::move(entry));
  }
  return module;
}

template <class F> auto completion(const std::shared_ptr<ContextObj> &ctx, F &&fn) -> decltype(fn()) {
  try {
    return fn();
  } catch (const Error &e) {
    if (e.code == Code::execution)
      ctx->completion_failure_observed = true;
    throw;
  }
}
template <class F> void release_completion(const std::shared_ptr<ContextObj> &ctx, F &&fn) {
  const bool observed = ctx->completion_failure_observed;
  try {
    completion(ctx, std::forward<F>(fn));
  } catch (const Error &e) {
    if (!observed || e.code != Code::execution)
      throw;
  }
}

std::shared_ptr<ContextObj> context_of(const Object &o) {
  switch (o.kind) {
  case HandleKind::context: return nullptr;
  case HandleKind::buffer: return static_cast<const BufferObj &>(o).owner;
  case HandleKind::view: return static_cast<const ViewObj &>(o).buffer->owner;
  case HandleKind::module: return static_cast<const ModuleObj &>(o).owner;
  case HandleKind::kernel: return static_cast<const KernelObj &>(o).module->owner;
  case HandleKind::queue: return static_cast<const QueueObj &>(o).owner;
  case HandleKind::event: return static_cast<const EventObj &>(o).owner;
  case HandleKind::collective: return static_cast<const PayloadObj &>(o).owner;
  }
  return nullptr;
}

pr_event submit_locked(const std::shared_ptr<QueueObj> &queue, const std::string &name,
                       Launcher launcher, Dim3 grid, Dim3 block, std::vector<BoundArg> args,
                       std::vector<std::shared_ptr<Allocation>> retained,
                       std::shared_ptr<const void> entry_data = nullptr) {
  auto event = std::make_shared<EventObj>(queue->owner, nullptr);
  const pr_handle handle = add(event);
  try {
    event->work = queue->owner->engine->submit(name, launcher, grid, block, std::move(args),
                                               std::move(retained), false, std::move(entry_data));
  } catch (...) {
    objects.erase(handle);
    throw;
  }
  return handle;
}

} // namespace

std::mutex &api_lock() noexcept { return api_mutex; }

// Called from api()'s catch block: classifies the exception in flight.
pr_status api_failure(const char *operation) noexcept {
  try {
    throw;
  } catch (const Failure &e) {
    last_error.code = e.status;
    text(last_error.message, e.what());
  } catch (const Error &e) {
    last_error.code = status_of(e.code);
    text(last_error.message, e.what());
  } catch (const std::bad_alloc &) {
    last_error.code = PR_OUT_OF_MEMORY;
    text(last_error.message, "Allocation failed");
  } catch (const std::exception &e) {
    last_error.code = PR_INTERNAL_ERROR;
    text(last_error.message, e.what());
  } catch (...) {
    last_error.code = PR_INTERNAL_ERROR;
    text(last_error.message, "Unknown native runtime failure");
  }
  text(last_error.operation, operation);
  try {
    runtime_event("api_failure", "failed", std::string(operation) + ": " + last_error.message);
  } catch (...) {
    static const char suffix[] = " [runtime event log also failed]";
    const size_t length = std::strlen(last_error.message);
    if (length + sizeof(suffix) <= sizeof(last_error.message))
      std::memcpy(last_error.message + length, suffix, sizeof(suffix));
  }
  return last_error.code;
}

pr_status report_error(pr_status code, const char *operation, const std::string &message) noexcept {
  return api(operation ? operation : "operator", [&] {
    throw Failure(code == PR_SUCCESS ? PR_INTERNAL_ERROR : code, message);
  });
}

void clear_error() noexcept { last_error = {}; }

pr_status set_error_fixed(pr_status code, const char *operation, const char *message) noexcept {
  last_error.code = code;
  std::strncpy(last_error.operation, operation ? operation : "", sizeof(last_error.operation) - 1);
  last_error.operation[sizeof(last_error.operation) - 1] = 0;
  std::strncpy(last_error.message, message ? message : "", sizeof(last_error.message) - 1);
  last_error.message[sizeof(last_error.message) - 1] = 0;
  return code;
}

pr_status handle_context(pr_handle h, HandleKind kind, const void **out) noexcept {
  return api("handle_context", [&] {
    require(out, PR_INVALID_ARGUMENT, "Missing context identity output");
    *out = nullptr;
    const auto it = objects.find(h);
    require(it != objects.end() && it->second->kind == kind, PR_INVALID_HANDLE,
            "Unknown, released, or wrong-kind handle");
    if (kind == HandleKind::context)
      *out = it->second.get();
    else
      *out = context_of(*it->second).get();
  });
}

QueueAccess queue_access(pr_queue queue) {
  auto q = get<QueueObj>(queue, HandleKind::queue);
  return QueueAccess{q->owner->engine, q->owner.get()};
}

std::shared_ptr<Engine> context_engine(pr_context context) {
  return get<ContextObj>(context, HandleKind::context)->engine;
}

pr_buffer add_buffer(pr_context context, std::shared_ptr<Allocation> allocation) {
  auto ctx = get<ContextObj>(context, HandleKind::context);
  ctx->engine->check_owner(*allocation);
  return add(std::make_shared<BufferObj>(ctx, std::move(allocation)));
}

std::shared_ptr<Allocation> allocation_of(pr_buffer buffer, std::shared_ptr<Engine> *engine) {
  auto b = get<BufferObj>(buffer, HandleKind::buffer);
  if (engine)
    *engine = b->owner->engine;
  return b->allocation;
}

std::shared_ptr<Allocation> buffer_allocation(pr_buffer buffer, const void *context) {
  auto b = get<BufferObj>(buffer, HandleKind::buffer);
  require(b->owner.get() == context, PR_CONTEXT_MISMATCH, "Buffer belongs to a different context");
  return b->allocation;
}

pr_event submit_command(pr_queue queue, const std::string &name, Launcher launcher, Dim3 grid,
                        Dim3 block, std::vector<BoundArg> args,
                        std::vector<std::shared_ptr<Allocation>> retained) {
  return submit_locked(get<QueueObj>(queue, HandleKind::queue), name, launcher, grid, block,
                       std::move(args), std::move(retained));
}

pr_event submit_transfer(pr_queue queue, pr_buffer buffer, uint64_t offset, void *host,
                         uint64_t bytes, bool to_device) {
  auto q = get<QueueObj>(queue, HandleKind::queue);
  auto b = get<BufferObj>(buffer, HandleKind::buffer);
  require(b->owner == q->owner, PR_CONTEXT_MISMATCH, "Buffer and queue belong to different contexts");
  require(host || !bytes, PR_INVALID_ARGUMENT,
          to_device ? "Nonempty write requires a host pointer" : "Nonempty read requires a host pointer");
  require(offset <= b->allocation->bytes && bytes <= b->allocation->bytes - offset, PR_OUT_OF_BOUNDS,
          "Copy range exceeds buffer");
  if (!bytes)
    return 0;
  auto event = std::make_shared<EventObj>(q->owner, nullptr);
  const pr_handle handle = add(event);
  try {
    event->work = q->owner->engine->transfer(to_device, b->allocation, offset, host, bytes);
  } catch (...) {
    objects.erase(handle);
    throw;
  }
  return handle;
}

pr_event submit_marker(pr_queue queue) {
  auto q = get<QueueObj>(queue, HandleKind::queue);
  auto event = std::make_shared<EventObj>(q->owner, nullptr);
  const pr_handle handle = add(event);
  try {
    event->work = q->owner->engine->marker();
  } catch (...) {
    objects.erase(handle);
    throw;
  }
  return handle;
}

double event_elapsed(pr_event first, pr_event second) {
  auto a = get<EventObj>(first, HandleKind::event), b = get<EventObj>(second, HandleKind::event);
  require(a->owner == b->owner, PR_CONTEXT_MISMATCH, "Events belong to different contexts");
  return completion(a->owner, [&] { return a->owner->engine->elapsed(a->work, b->work); });
}

pr_handle add_object(std::shared_ptr<void> object, HandleKind kind, const void *context) {
  for (const auto &entry : objects)
    if (entry.second.get() == context && entry.second->kind == HandleKind::context)
      return add(std::make_shared<PayloadObj>(
          kind, std::static_pointer_cast<ContextObj>(entry.second), std::move(object)));
  fail(PR_INVALID_HANDLE, "Unknown context");
}

std::shared_ptr<void> get_object(pr_handle handle, HandleKind kind, const void **context) {
  auto p = get<PayloadObj>(handle, kind);
  if (context)
    *context = p->owner.get();
  return p->payload;
}

} // namespace pb

using namespace pb;

PB_EXPORT uint32_t pr_abi_version(void) { return PR_ABI_VERSION; }

PB_EXPORT pr_status pr_last_error(pr_error *out) {
  if (!out)
    return PR_INVALID_ARGUMENT;
  *out = last_error;
  return PR_SUCCESS;
}

PB_EXPORT pr_status pr_backend_status_get(const char *backend, pr_backend_status_v1 *out) {
  return api("backend_status_get", [&] {
    query_record(out);
    require(backend, PR_INVALID_ARGUMENT, "Missing backend name");
    const std::string name = backend;
    require(name == "metal" || name == "cuda" || name == "hip", PR_INVALID_ARGUMENT,
            "Unknown backend; expected metal, cuda or hip");
    pr_backend_status_v1 result{};
    result.struct_size = sizeof(result);
    result.version = PR_QUERY_VERSION_1;
    text(result.backend, name);
    if (name == "metal") {
      text(result.reason, "Metal backend not built (macOS only)");
    } else if (name == "cuda") {
      const auto &s = backend_status();
      result.implemented = 1;
      result.available = s.available;
      result.device_count = uint32_t(s.device_count);
      result.driver_version = s.driver_version;
      result.compiler_version = s.runtime_version;
      text(result.driver_library, "libcuda.so.1");
      text(result.compiler_library, "none (kernels are compiled ahead of time for sm_100a)");
      text(result.reason, s.reason);
    } else {
      text(result.reason, "HIP/HIPRTC backend is not implemented");
    }
    *out = result;
  });
}

PB_EXPORT pr_status pr_device_count(uint32_t *out) {
  return api("device_count", [&] {
    require(out, PR_INVALID_ARGUMENT, "Missing count output");
    *out = uint32_t(devices().size());
  });
}

PB_EXPORT pr_status pr_device_get(uint32_t index, pr_device_info *out) {
  return api("device_get", [&] {
    const auto &list = devices();
    require(index < list.size(), PR_DEVICE_UNAVAILABLE, "Device index unavailable");
    device_record(list[index], out);
  });
}

PB_EXPORT pr_status pr_device_capabilities_get(uint32_t index, pr_device_capabilities_v1 *out) {
  return api("device_capabilities_get", [&] {
    query_record(out);
    const auto &list = devices();
    require(index < list.size(), PR_DEVICE_UNAVAILABLE, "Device index unavailable");
    capabilities(list[index], out);
  });
}

PB_EXPORT pr_status pr_context_create(const char *selector, pr_context *out) {
  return api("context_create", [&] {
    require(out, PR_INVALID_ARGUMENT, "Missing context output");
    *out = 0;
    ensure_shutdown();
    *out = add(std::make_shared<ContextObj>(create_engine(selector ? selector : "auto")));
  });
}

PB_EXPORT pr_status pr_context_device(pr_context h, pr_device_info *out) {
  return api("context_device", [&] {
    device_record(get<ContextObj>(h, HandleKind::context)->engine->device(), out);
  });
}

PB_EXPORT pr_status pr_context_capabilities(pr_context h, pr_device_capabilities_v1 *out) {
  return api("context_capabilities", [&] {
    capabilities(get<ContextObj>(h, HandleKind::context)->engine->device(), out);
  });
}

PB_EXPORT pr_status pr_context_synchronize(pr_context h) {
  return api("context_synchronize", [&] {
    auto ctx = get<ContextObj>(h, HandleKind::context);
    completion(ctx, [&] { ctx->engine->synchronize(); });
  });
}

PB_EXPORT pr_status pr_context_write_evidence(pr_context h, const char *directory) {
  return api("context_write_evidence", [&] {
    auto ctx = get<ContextObj>(h, HandleKind::context);
    require(directory && *directory, PR_INVALID_ARGUMENT, "Missing evidence directory");
    const std::filesystem::path path(directory);
    require(!std::filesystem::exists(path) ||
                (std::filesystem::is_directory(path) && std::filesystem::is_empty(path)),
            PR_INVALID_ARGUMENT, "Evidence directory must be new or empty");
    completion(ctx, [&] { ctx->engine->write_evidence(path.string()); });
  });
}

PB_EXPORT pr_status pr_release(pr_handle h) {
  return api("release", [&] {
    const auto it = objects.find(h);
    require(it != objects.end(), PR_INVALID_HANDLE, "Unknown or released handle");
    auto object = std::move(it->second);
    objects.erase(it); // consumed even if completion reports a failure
    if (object->kind == HandleKind::context) {
      auto ctx = std::static_pointer_cast<ContextObj>(object);
      release_completion(ctx, [&] { ctx->engine->synchronize(); });
    } else if (object->kind == HandleKind::queue) {
      auto ctx = std::static_pointer_cast<QueueObj>(object)->owner;
      release_completion(ctx, [&] { ctx->engine->synchronize(); });
    } else if (object->kind == HandleKind::event) {
      auto event = std::static_pointer_cast<EventObj>(object);
      release_completion(event->owner, [&] { event->owner->engine->wait(event->work); });
    }
  });
}

PB_EXPORT pr_status pr_buffer_create(pr_context context, uint64_t n, pr_buffer *out) {
  return api("buffer_create", [&] {
    require(out, PR_INVALID_ARGUMENT, "Missing buffer output");
    *out = 0;
    auto ctx = get<ContextObj>(context, HandleKind::context);
    *out = add(std::make_shared<BufferObj>(ctx, ctx->engine->allocate(bytes(n))));
  });
}

PB_EXPORT pr_status pr_buffer_size(pr_buffer h, uint64_t *out) {
  return api("buffer_size", [&] {
    require(out, PR_INVALID_ARGUMENT, "Missing size output");
    *out = get<BufferObj>(h, HandleKind::buffer)->allocation->bytes;
  });
}

PB_EXPORT pr_status pr_view_create(pr_buffer h, uint64_t offset, uint64_t n, uint32_t alignment,
                                   pr_access mode, pr_view *out) {
  return api("view_create", [&] {
    require(out, PR_INVALID_ARGUMENT, "Missing view output");
    *out = 0;
    auto buffer = get<BufferObj>(h, HandleKind::buffer);
    require(mode == PR_READ || mode == PR_WRITE || mode == PR_READ_WRITE, PR_INVALID_ARGUMENT,
            "Invalid view access mode");
    require(alignment == 1 || alignment == 2 || alignment == 4, PR_UNSUPPORTED,
            "Supported element alignments are 1, 2 and 4 bytes");
    range(buffer->allocation->bytes, offset, n);
    require(offset % alignment == 0 && n % alignment == 0, PR_INVALID_ARGUMENT,
            "Misaligned view offset or size");
    *out = add(std::make_shared<ViewObj>(buffer, bytes(offset), bytes(n), alignment, mode));
  });
}

PB_EXPORT pr_status pr_buffer_write(pr_buffer h, uint64_t offset, const void *source, uint64_t n) {
  return api("buffer_write", [&] {
    auto b = get<BufferObj>(h, HandleKind::buffer);
    range(b->allocation->bytes, offset, n);
    require(source || !n, PR_INVALID_ARGUMENT, "Null nonempty upload source");
    completion(b->owner, [&] { b->owner->engine->write(b->allocation, bytes(offset), source, bytes(n)); });
  });
}

PB_EXPORT pr_status pr_buffer_read(pr_buffer h, uint64_t offset, void *destination, uint64_t n) {
  return api("buffer_read", [&] {
    auto b = get<BufferObj>(h, HandleKind::buffer);
    range(b->allocation->bytes, offset, n);
    require(destination || !n, PR_INVALID_ARGUMENT, "Null nonempty download destination");
    completion(b->owner,
               [&] { b->owner->engine->read(b->allocation, bytes(offset), destination, bytes(n)); });
  });
}

PB_EXPORT pr_status pr_module_load(pr_context context, const void *data, uint64_t n, pr_module *out) {
  return api("module_load", [&] {
    require(out, PR_INVALID_ARGUMENT, "Missing module output");
    *out = 0;
    *out = add(load(get<ContextObj>(context, HandleKind::context), data, bytes(n)));
  });
}

PB_EXPORT pr_status pr_module_load_file(pr_context context, const char *path, pr_module *out) {
  return api("module_load_file", [&] {
    require(out, PR_INVALID_ARGUMENT, "Missing module output");
    *out = 0;
    auto ctx = get<ContextObj>(context, HandleKind::context);
    require(path && *path, PR_INVALID_ARGUMENT, "Missing module path");
    std::ifstream input(path, std::ios::binary | std::ios::ate);
    require(bool(input), PR_COMPILATION_FAILED, "Cannot open module artifact");
    const auto length = input.tellg();
    require(length >= 0 && uint64_t(length) <= prk_max_bytes, PR_COMPILATION_FAILED,
            "Module artifact exceeds 16 MiB limit");
    std::vector<unsigned char> data(static_cast<size_t>(length));
    input.seekg(0);
    input.read(reinterpret_cast<char *>(data.data()), std::streamsize(data.size()));
    require(bool(input), PR_COMPILATION_FAILED, "Cannot read module artifact");
    *out = add(load(ctx, data.data(), data.size()));
  });
}

PB_EXPORT pr_status pr_module_kernel(pr_module h, const char *name, pr_kernel *out) {
  return api("module_kernel", [&] {
    require(out, PR_INVALID_ARGUMENT, "Missing kernel output");
    *out = 0;
    require(name, PR_INVALID_ARGUMENT, "Missing kernel name");
    auto module = get<ModuleObj>(h, HandleKind::module);
    for (size_t i = 0; i < module->entries.size(); ++i)
      if (module->entries[i].name == name) {
        *out = add(std::make_shared<KernelObj>(module, i));
        return;
      }
    fail(PR_INVALID_ARGUMENT, "Module has no entrypoint with that name");
  });
}

PB_EXPORT pr_status pr_kernel_parameter_count(pr_kernel h, uint32_t *out) {
  return api("kernel_parameter_count", [&] {
    require(out, PR_INVALID_ARGUMENT, "Missing count output");
    *out = uint32_t(get<KernelObj>(h, HandleKind::kernel)->entry().params.size());
  });
}

PB_EXPORT pr_status pr_kernel_parameter(pr_kernel h, uint32_t index, pr_parameter_info *out) {
  return api("kernel_parameter", [&] {
    require(out, PR_INVALID_ARGUMENT, "Missing parameter output");
    auto k = get<KernelObj>(h, HandleKind::kernel);
    require(index < k->entry().params.size(), PR_OUT_OF_BOUNDS, "Parameter index out of range");
    const auto &p = k->entry().params[index];
    *out = {};
    text(out->name, p.name);
    out->type = public_type(p.type);
    out->is_buffer = p.buffer;
    out->access = p.access;
  });
}

PB_EXPORT pr_status pr_queue_get(pr_context h, pr_queue *out) {
  return api("queue_get", [&] {
    require(out, PR_INVALID_ARGUMENT, "Missing queue output");
    *out = 0;
    *out = add(std::make_shared<QueueObj>(get<ContextObj>(h, HandleKind::context)));
  });
}

PB_EXPORT pr_status pr_queue_synchronize(pr_queue h) {
  return api("queue_synchronize", [&] {
    auto ctx = get<QueueObj>(h, HandleKind::queue)->owner;
    completion(ctx, [&] { ctx->engine->synchronize(); });
  });
}

PB_EXPORT pr_status pr_launch(pr_queue q, pr_kernel h, pr_dim3 grid, pr_dim3 block,
                              const pr_argument *args, uint32_t count, pr_event *out) {
  return api("launch", [&] {
    require(out, PR_INVALID_ARGUMENT, "Missing event output");
    *out = 0;
    auto queue = get<QueueObj>(q, HandleKind::queue);
    auto kernel = get<KernelObj>(h, HandleKind::kernel);
    require(queue->owner == kernel->module->owner, PR_CONTEXT_MISMATCH,
            "Queue and kernel belong to different contexts");
    const auto &entry = kernel->entry();
    require(count == entry.params.size(), PR_INVALID_ARGUMENT, "Kernel argument count mismatch");
    require(args || !count, PR_INVALID_ARGUMENT, "Missing kernel arguments");
    std::vector<BoundArg> bound(count);
    std::vector<std::shared_ptr<Allocation>> retained;
    for (uint32_t i = 0; i < count; ++i) {
      const auto &p = entry.params[i];
      const auto &a = args[i];
      if (p.buffer) {
        require(a.type == PR_BUFFER, PR_INVALID_ARGUMENT, "Expected a buffer-view argument");
        auto view = get<ViewObj>(a.view, HandleKind::view);
        require(view->buffer->owner == queue->owner, PR_CONTEXT_MISMATCH,
                "View belongs to a different context");
        require(view->alignment == 4 && view->offset % 4 == 0 && view->size % 4 == 0,
                PR_INVALID_ARGUMENT, "Typed kernel view must have four-byte alignment and size");
        require(view->size >= 4, PR_INVALID_ARGUMENT,
                "View violates kernel minimum size or alignment");
        require((view->access & p.access) == p.access, PR_INVALID_ARGUMENT,
                "View access does not allow the kernel's reads/writes");
        bound[i].buffer = true;
        bound[i].writes = (p.access & PR_WRITE) != 0;
        bound[i].ptr = static_cast<char *>(view->buffer->allocation->ptr) + view->offset;
        bound[i].bytes = view->size;
        retained.push_back(view->buffer->allocation);
      } else {
        require(a.type == public_type(p.type), PR_INVALID_ARGUMENT, "Kernel scalar type mismatch");
        if (a.type == PR_I32)
          std::memcpy(&bound[i].bits, &a.i32, 4);
        else if (a.type == PR_U32)
          bound[i].bits = a.u32;
        else
          std::memcpy(&bound[i].bits, &a.f32, 4);
      }
    }
    const Builtin &b = *entry.builtin;
    if (b.required_block[0])
      require(block.x == b.required_block[0] && block.y == b.required_block[1] &&
                  block.z == b.required_block[2],
              PR_INVALID_ARGUMENT, "Launch block does not match the entry's required block");
    const Dim3 g{grid.x, grid.y, grid.z}, bl{block.x, block.y, block.z};
    queue->owner->engine->check_geometry(g, bl);
    *out = submit_locked(queue, entry.name, b.launch, g, bl, std::move(bound), std::move(retained),
                         entry.jit);
  });
}

namespace pb {
pr_status launch_entry(pr_queue q, pr_module m, const char *name, pr_dim3 grid, pr_dim3 block,
                       const RangeArgument *args, uint32_t count, pr_event *out) noexcept {
  return api("launch", [&] {
    require(out, PR_INVALID_ARGUMENT, "Missing event output");
    *out = 0;
    auto queue = get<QueueObj>(q, HandleKind::queue);
    auto module = get<ModuleObj>(m, HandleKind::module);
    require(queue->owner == module->owner, PR_CONTEXT_MISMATCH, "Queue and kernel belong to different contexts");
    const Entry *entry = nullptr;
    for (const auto &e : module->entries)
      if (e.name == name) {
        entry = &e;
        break;
      }
    require(entry, PR_INVALID_ARGUMENT, "Module has no entrypoint with that name");
    require(count == entry->params.size(), PR_INVALID_ARGUMENT, "Kernel argument count mismatch");
    require(args || !count, PR_INVALID_ARGUMENT, "Missing kernel arguments");
    std::vector<BoundArg> bound(count);
    std::vector<std::shared_ptr<Allocation>> retained;
    retained.reserve(count);
    for (uint32_t i = 0; i < count; ++i) {
      const auto &p = entry->params[i];
      const auto &a = args[i];
      if (p.buffer) {
        require(a.arg.type == PR_BUFFER, PR_INVALID_ARGUMENT, "Expected a buffer-view argument");
        auto buffer = get<BufferObj>(a.buffer, HandleKind::buffer);
        require(buffer->owner == queue->owner, PR_CONTEXT_MISMATCH, "View belongs to a different context");
        range(buffer->allocation->bytes, a.offset, a.bytes);
        require(a.offset % 4 == 0 && a.bytes % 4 == 0 && a.bytes >= 4, PR_INVALID_ARGUMENT,
                "Typed kernel view must have four-byte alignment and size");
        require((a.access & p.access) == p.access, PR_INVALID_ARGUMENT,
                "View access does not allow the kernel's reads/writes");
        bound[i].buffer = true;
        bound[i].writes = (p.access & PR_WRITE) != 0;
        bound[i].ptr = static_cast<char *>(buffer->allocation->ptr) + a.offset;
        bound[i].bytes = bytes(a.bytes);
        retained.push_back(buffer->allocation);
      } else {
        require(a.arg.type == public_type(p.type), PR_INVALID_ARGUMENT, "Kernel scalar type mismatch");
        if (a.arg.type == PR_I32)
          std::memcpy(&bound[i].bits, &a.arg.i32, 4);
        else if (a.arg.type == PR_U32)
          bound[i].bits = a.arg.u32;
        else
          std::memcpy(&bound[i].bits, &a.arg.f32, 4);
      }
    }
    const Builtin &b = *entry->builtin;
    if (b.required_block[0])
      require(block.x == b.required_block[0] && block.y == b.required_block[1] && block.z == b.required_block[2],
              PR_INVALID_ARGUMENT, "Launch block does not match the entry's required block");
    const Dim3 g{grid.x, grid.y, grid.z}, bl{block.x, block.y, block.z};
    queue->owner->engine->check_geometry(g, bl);
    *out = submit_locked(queue, entry->name, b.launch, g, bl, std::move(bound), std::move(retained), entry->jit);
  });
}
} // namespace pb

PB_EXPORT pr_status pr_event_wait(pr_event h, pr_event_info *out) {
  return api("event_wait", [&] {
    auto event = get<EventObj>(h, HandleKind::event);
    const auto info = completion(event->owner, [&] { return event->owner->engine->wait(event->work); });
    if (out)
      *out = {uint32_t(info.completed), 0.0, 0.0};
  });
}

PB_EXPORT pr_status pr_event_timing(pr_event h, pr_event_timing_v1 *out) {
  return api("event_timing", [&] {
    query_record(out);
    auto event = get<EventObj>(h, HandleKind::event);
    const auto info = completion(event->owner, [&] { return event->owner->engine->wait(event->work); });
    *out = {};
    out->struct_size = sizeof(*out);
    out->version = PR_QUERY_VERSION_1;
    out->completed = info.completed;
    out->duration_valid = info.duration_valid;
    out->timestamps_valid = 0;
    out->clock_domain = info.duration_valid ? PR_CLOCK_DURATION_ONLY : PR_CLOCK_UNAVAILABLE;
    out->duration_seconds = info.duration_valid ? info.duration_seconds : 0;
  });
}

PB_EXPORT pr_status pr_event_cancel(pr_event h) {
  return api("event_cancel", [&] {
    (void)get<EventObj>(h, HandleKind::event);
    fail(PR_UNSUPPORTED, "Cancellation of submitted GPU work is unsupported; wait for completion");
  });
}
