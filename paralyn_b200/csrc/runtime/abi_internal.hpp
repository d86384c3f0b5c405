// Library-internal interface between the C-ABI layer (abi.cpp) and the in-library
// clients built on it: the tensor provider (provider.cpp) and the B200 additions
// (b200.cpp). Nothing here is exported.
#pragma once
#include "engine.hpp"
#include "module.hpp"
#include <functional>
#include <memory>
#include <mutex>

namespace pb {

enum class HandleKind { context, buffer, view, module, kernel, queue, event, collective };

std::mutex &api_lock() noexcept;
void clear_error() noexcept;
// Records the exception being handled as (status, operation, message) in
// pr_last_error; only valid inside a catch block.
pr_status api_failure(const char *operation) noexcept;

// Runs `fn` under the global API lock with the reference's error boundary:
// success clears pr_last_error, a failure records (status, operation, message).
// A template, so the call costs no std::function allocation.
template <class F> pr_status api(const char *operation, F &&fn) noexcept {
  try {
    std::lock_guard<std::mutex> lock(api_lock());
    fn();
    clear_error();
    return PR_SUCCESS;
  } catch (...) {
    return api_failure(operation);
  }
}
// Records a failure for `operation` without running anything (returns `code`).
pr_status report_error(pr_status code, const char *operation, const std::string &message) noexcept;
// Records a failure from fixed strings without allocating (for entry points that
// must not allocate); does not take the API lock or write the event log.
pr_status set_error_fixed(pr_status code, const char *operation, const char *message) noexcept;
// Opaque identity of the context that owns a live handle of exactly `kind`.
pr_status handle_context(pr_handle handle, HandleKind kind, const void **out) noexcept;

// Helpers for in-library clients; call only inside api().
struct QueueAccess {
  std::shared_ptr<Engine> engine;
  const void *context = nullptr;
};
QueueAccess queue_access(pr_queue queue);
std::shared_ptr<Engine> context_engine(pr_context context);
// A buffer handle of `context` that owns `allocation` (used for imported peer memory).
pr_buffer add_buffer(pr_context context, std::shared_ptr<Allocation> allocation);
// The allocation behind a buffer handle and its owning context's engine.
std::shared_ptr<Allocation> allocation_of(pr_buffer buffer, std::shared_ptr<Engine> *engine);
std::shared_ptr<Allocation> buffer_allocation(pr_buffer buffer, const void *context);
// Publishes an event handle for a submitted command (handle allocated first, as
// pr_launch does, so a failure never leaves a command without its event).
pr_event submit_command(pr_queue queue, const std::string &name, Launcher launcher, Dim3 grid,
                        Dim3 block, std::vector<BoundArg> args,
                        std::vector<std::shared_ptr<Allocation>> retained);
pr_event submit_marker(pr_queue queue);
// A stream-ordered host copy of `queue` (0 and nothing enqueued when bytes == 0).
pr_event submit_transfer(pr_queue queue, pr_buffer buffer, uint64_t offset, void *host,
                         uint64_t bytes, bool to_device);
double event_elapsed(pr_event first, pr_event second);
// pr_launch for in-library callers without view or kernel handles: the entry is
// named in `module`, and each buffer argument is a (buffer, offset, bytes, access)
// range checked as pr_view_create would (alignment 4) and bound like a view. One
// lock for the whole submission.
struct RangeArgument {
  pr_argument arg{};      // type and, for scalars, the value
  pr_buffer buffer = 0;   // buffer arguments
  uint64_t offset = 0, bytes = 0;
  pr_access access = PR_READ;
};
pr_status launch_entry(pr_queue queue, pr_module module, const char *name, pr_dim3 grid, pr_dim3 block,
                       const RangeArgument *args, uint32_t count, pr_event *out) noexcept;
pr_handle add_object(std::shared_ptr<void> object, HandleKind kind, const void *context);
std::shared_ptr<void> get_object(pr_handle handle, HandleKind kind, const void **context);

} // namespace pb
