#include "engine.hpp"
#include "jit.hpp"
#include "../kernels/prepared.hpp"
#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <condition_variable>
#include <cstring>
#include <cstdio>
#include <cstdlib>
#include <filesystem>
#include <fstream>
#include <iomanip>
#include <limits>
#include <sstream>
#include <sys/utsname.h>
#include <thread>
#include <unistd.h>

namespace pb {

struct Accounting {
  std::atomic<uint64_t> current{0}, peak{0};
};

namespace {

std::mutex log_mutex;
uint64_t log_sequence = 0;

std::string json(const std::string &text) {
  std::ostringstream out;
  out << '"';
  for (unsigned char c : text) {
    if (c == '"' || c == '\\')
      out << '\\' << char(c);
    else if (c < 32)
      out << "\\u" << std::hex << std::setw(4) << std::setfill('0') << unsigned(c) << std::dec;
    else
      out << char(c);
  }
  out << '"';
  return out.str();
}

// CUDA runtime error classes, mirroring the driver-code classes of the reference
// engine (backends/cuda/engine.cpp:29-94).
Code code_of(cudaError_t e) {
  switch (e) {
  case cudaErrorInvalidValue:
  case cudaErrorInvalidConfiguration:
  case cudaErrorLaunchOutOfResources:
    return Code::invalid_value;
  case cudaErrorMemoryAllocation:
    return Code::out_of_memory;
  case cudaErrorNoDevice:
  case cudaErrorInvalidDevice:
  case cudaErrorInsufficientDriver:
  case cudaErrorInitializationError:
  case cudaErrorStubLibrary:
  case cudaErrorSystemNotReady:
  case cudaErrorSystemDriverMismatch:
  case cudaErrorCompatNotSupportedOnDevice:
    return Code::invalid_device;
  case cudaErrorNoKernelImageForDevice:
  case cudaErrorInvalidKernelImage:
  case cudaErrorUnsupportedPtxVersion:
    return Code::compilation;
  case cudaErrorNotPermitted:
  case cudaErrorNotSupported:
    return Code::unsupported;
  case cudaErrorInvalidResourceHandle:
  case cudaErrorContextIsDestroyed:
    return Code::internal;
  default:
    return Code::execution;
  }
}

bool is_sticky(cudaError_t e) {
  switch (e) {
  case cudaErrorECCUncorrectable:
  case cudaErrorIllegalAddress:
  case cudaErrorLaunchTimeout:
  case cudaErrorAssert:
  case cudaErrorHardwareStackError:
  case cudaErrorIllegalInstruction:
  case cudaErrorMisalignedAddress:
  case cudaErrorInvalidAddressSpace:
  case cudaErrorInvalidPc:
  case cudaErrorLaunchFailure:
  case cudaErrorUnknown:
  case cudaErrorContextIsDestroyed:
    return true;
  default:
    return false;
  }
}

std::string text_of(cudaError_t e) {
  return std::string(cudaGetErrorName(e)) + " (" + cudaGetErrorString(e) + ")";
}

std::string os_description() {
  struct utsname name {};
  if (uname(&name) == 0)
    return std::string(name.sysname) + " " + name.release;
  return "unknown";
}

// Makes `device` current for one operation and restores the caller's device.
class DeviceScope {
  int previous_ = -1, device_;

public:
  explicit DeviceScope(int device) : device_(device) {
    if (cudaGetDevice(&previous_) != cudaSuccess)
      previous_ = -1;
    if (previous_ != device_)
      cuda_check(cudaSetDevice(device_), "cudaSetDevice");
  }
  ~DeviceScope() {
    if (previous_ >= 0 && previous_ != device_)
      cudaSetDevice(previous_);
  }
};

struct Probe {
  BackendStatus status;
  std::vector<DeviceRecord> devices;
};

const Probe &probe() {
  static const Probe value = [] {
    Probe p;
    cudaRuntimeGetVersion(&p.status.runtime_version);
    if (cudaDriverGetVersion(&p.status.driver_version) != cudaSuccess)
      p.status.driver_version = 0;
    int count = 0;
    const cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess) {
      p.status.reason = "CUDA unavailable: " + text_of(e) + ". There is no CPU fallback.";
      cudaGetLastError();
      return p;
    }
    const std::string os = os_description();
    for (int i = 0; i < count; ++i) {
      cudaDeviceProp prop{};
      if (cudaGetDeviceProperties(&prop, i) != cudaSuccess)
        continue;
      DeviceRecord d;
      d.ordinal = i;
      d.name = prop.name;
      d.os = os;
      d.total_memory = prop.totalGlobalMem;
      d.max_smem_block = prop.sharedMemPerBlock;
      d.sm_count = prop.multiProcessorCount;
      d.cc_major = prop.major;
      d.cc_minor = prop.minor;
      d.max_threads = prop.maxThreadsPerBlock;
      d.max_block = {uint32_t(prop.maxThreadsDim[0]), uint32_t(prop.maxThreadsDim[1]),
                     uint32_t(prop.maxThreadsDim[2])};
      d.max_grid = {uint32_t(prop.maxGridSize[0]), uint32_t(prop.maxGridSize[1]),
                    uint32_t(prop.maxGridSize[2])};
      d.integrated = prop.integrated != 0;
      d.registry_id = 0x4355444100000000ULL | (uint64_t(i) + 1);
      std::ostringstream id;
      id << "cuda:uuid:" << std::hex << std::setfill('0');
      for (int b = 0; b < 16; ++b) {
        if (b == 4 || b == 6 || b == 8 || b == 10)
          id << '-';
        id << std::setw(2) << unsigned(static_cast<unsigned char>(prop.uuid.bytes[b]));
      }
      d.stable_id = id.str();
      p.devices.push_back(d);
    }
    p.status.device_count = int(p.devices.size());
    p.status.available = !p.devices.empty();
    if (!p.status.available)
      p.status.reason = "No CUDA device available. There is no CPU fallback.";
    return p;
  }();
  return value;
}

// Makes room for `extra` more elements so that later push_backs cannot throw. The
// capacity at least doubles: a plain reserve(size + 1) reallocates on every call,
// which made each submission cost time in proportion to every launch recorded so far.
template <class V> void reserve_more(V &v, size_t extra) {
  const size_t need = v.size() + extra;
  if (need > v.capacity())
    v.reserve(std::max(need, 2 * v.capacity()));
}

uint64_t next_trace_id() {
  static std::atomic<uint64_t> next{1};
  return (uint64_t(2) << 32) | next.fetch_add(1);
}

} // namespace

void cuda_check(cudaError_t result, const char *operation) {
  if (result != cudaSuccess)
    throw Error(code_of(result), std::string("CUDA ") + operation + " failed: " + text_of(result));
}

void progress(const std::string &message) {
  const char *path = std::getenv("PARALYN_RUNTIME_LOG");
  if (!path || !*path)
    return;
  std::lock_guard<std::mutex> lock(log_mutex);
  std::ofstream output(path, std::ios::app);
  output << message;
  output.close();
  if (!output)
    throw Error(Code::internal, "Cannot write PARALYN_RUNTIME_LOG");
}

void runtime_event(const std::string &category, const std::string &status,
                   const std::string &detail, uint64_t context_id, uint64_t operation_id,
                   uint64_t bytes) {
  const char *path = std::getenv("PARALYN_EVENT_LOG");
  if (!path || !*path)
    return;
  std::lock_guard<std::mutex> lock(log_mutex);
  const double now =
      std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
  std::ostringstream line;
  line << std::setprecision(17) << "{\"schema\":\"paralyn.runtime.event\",\"schema_version\":1,"
       << "\"sequence\":" << ++log_sequence << ",\"category\":" << json(category)
       << ",\"status\":" << json(status) << ",\"detail\":" << json(detail)
       << ",\"context_id\":" << context_id << ",\"operation_id\":" << operation_id
       << ",\"bytes\":" << bytes << ",\"host_monotonic_seconds\":" << now << "}\n";
  const std::string text = line.str();
  FILE *file = std::fopen(path, "ab");
  if (!file)
    throw Error(Code::internal, "Cannot open PARALYN_EVENT_LOG");
  bool ok = std::fwrite(text.data(), 1, text.size(), file) == text.size();
  ok = std::fflush(file) == 0 && ok;
  ok = fsync(fileno(file)) == 0 && ok;
  ok = std::fclose(file) == 0 && ok;
  if (!ok)
    throw Error(Code::internal, "Cannot durably append PARALYN_EVENT_LOG");
}

const BackendStatus &backend_status() { return probe().status; }
const std::vector<DeviceRecord> &devices() { return probe().devices; }

Allocation::~Allocation() {
  if (accounting)
    accounting->current.fetch_sub(bytes);
  if (!ptr)
    return;
  int previous = -1;
  cudaGetDevice(&previous);
  if (previous != device)
    cudaSetDevice(device);
  if (imported)
    cudaIpcCloseMemHandle(ptr);
  else
    cudaFree(ptr);
  if (previous >= 0 && previous != device)
    cudaSetDevice(previous);
}

Engine::Engine(const DeviceRecord &device)
    : device_(device), accounting_(std::make_shared<Accounting>()), trace_id_(next_trace_id()) {
  DeviceScope scope(device_.ordinal);
  cuda_check(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate");
  const cudaError_t e = cudaHostAlloc(reinterpret_cast<void **>(&status_host_), 64,
                                      cudaHostAllocMapped | cudaHostAllocPortable);
  if (e != cudaSuccess) {
    cudaStreamDestroy(stream_);
    cuda_check(e, "cudaHostAlloc(status word)");
  }
  std::memset(status_host_, 0, 64);
  cuda_check(cudaStreamCreateWithFlags(&side_stream_, cudaStreamNonBlocking),
             "cudaStreamCreate(side)");
  for (auto &copy : copy_streams_)
    cuda_check(cudaStreamCreateWithFlags(&copy, cudaStreamNonBlocking), "cudaStreamCreate(copy)");
  for (auto &event : side_events_)
    cuda_check(cudaEventCreateWithFlags(&event, cudaEventDisableTiming), "cudaEventCreate(side)");
  cuda_check(cudaHostGetDevicePointer(reinterpret_cast<void **>(&status_device_), status_host_, 0),
             "cudaHostGetDevicePointer");
  if (const char *mode = std::getenv("PARALYN_MATMUL_MODE")) {
    const std::string m = mode;
    matmul_mode_ = m == "reference" ? matmul_reference
                 : m == "ffma"      ? matmul_ffma
                 : m == "tf32x3"    ? matmul_tf32x3
                                    : matmul_auto;
  }
  runtime_event("context", "created", device_.stable_id, trace_id_);
}

Engine::~Engine() {
  try {
    synchronize();
  } catch (...) {
  }
  try {
    DeviceScope scope(device_.ordinal);
    for (auto &work : pending_)
      recycle(*work);
    for (auto e : spare_events_)
      cudaEventDestroy(e);
    if (stream_)
      cudaStreamDestroy(stream_);
    if (side_stream_)
      cudaStreamDestroy(side_stream_);
    for (int i = 0; i < staging_slots; ++i) {
      if (staging_[i])
        cudaFreeHost(staging_[i]);
      if (staging_events_[i])
        cudaEventDestroy(staging_events_[i]);
    }
    for (auto copy : copy_streams_)
      if (copy)
        cudaStreamDestroy(copy);
    for (auto event : side_events_)
      if (event)
        cudaEventDestroy(event);
    if (workspace_)
      cudaFree(workspace_);
    if (status_host_)
      cudaFreeHost(status_host_);
  } catch (...) {
  }
}

void Engine::healthy() const {
  if (!terminal_failure_.empty())
    throw Error(Code::execution, terminal_failure_);
}

void Engine::cuda_failure(cudaError_t code, const std::string &operation) {
  const std::string text = "CUDA " + operation + " failed: " + text_of(code);
  if (is_sticky(code) && terminal_failure_.empty())
    terminal_failure_ = text;
  cudaGetLastError();
  throw Error(code_of(code), text);
}

void Engine::check_owner(const Allocation &allocation) const {
  if (allocation.owner != this)
    throw Error(Code::invalid_handle, "Buffer belongs to another context");
}

std::shared_ptr<Allocation> Engine::allocate(size_t bytes) {
  std::lock_guard<std::mutex> lock(mutex_);
  healthy();
  auto result = std::make_shared<Allocation>();
  result->device = device_.ordinal;
  result->bytes = bytes;
  result->owner = this;
  if (bytes) {
    DeviceScope scope(device_.ordinal);
    const cudaError_t e = cudaMalloc(&result->ptr, bytes);
    if (e != cudaSuccess)
      cuda_failure(e, "cudaMalloc");
  }
  result->accounting = accounting_;
  const uint64_t now = accounting_->current.fetch_add(bytes) + bytes;
  uint64_t peak = accounting_->peak.load();
  while (peak < now && !accounting_->peak.compare_exchange_weak(peak, now)) {
  }
  return result;
}

PeerHandle Engine::export_allocation(const Allocation &allocation) {
  std::lock_guard<std::mutex> lock(mutex_);
  check_owner(allocation);
  if (allocation.imported || !allocation.ptr)
    throw Error(Code::invalid_value, "Only non-empty buffers allocated by this context can be exported");
  DeviceScope scope(device_.ordinal);
  PeerHandle h{};
  const cudaError_t e = cudaIpcGetMemHandle(&h.handle, allocation.ptr);
  if (e != cudaSuccess)
    cuda_failure(e, "cudaIpcGetMemHandle");
  h.bytes = allocation.bytes;
  return h;
}

std::shared_ptr<Allocation> Engine::import_allocation(const PeerHandle &handle) {
  std::lock_guard<std::mutex> lock(mutex_);
  healthy();
  if (!handle.bytes)
    throw Error(Code::invalid_value, "Peer handle describes an empty allocation");
  DeviceScope scope(device_.ordinal);
  auto result = std::make_shared<Allocation>();
  result->device = device_.ordinal;
  result->bytes = handle.bytes;
  result->owner = this;
  result->imported = true;
  const cudaError_t e = cudaIpcOpenMemHandle(&result->ptr, handle.handle, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    result->ptr = nullptr;
    cuda_failure(e, "cudaIpcOpenMemHandle");
  }
  return result;
}

static void copy_range(const Allocation &a, size_t offset, size_t bytes) {
  if (offset > a.bytes || bytes > a.bytes - offset)
    throw Error(Code::invalid_value, "Copy range exceeds allocation");
}

// Host-side copy split over a few worker threads (a pageable source or destination
// is read or written at more than one core's memory bandwidth). The pool lives for
// the process; its threads wait on a condition variable between copies.
namespace {
class CopyPool {
public:
  static CopyPool &get() {
    static CopyPool *pool = new CopyPool(); // never destroyed: workers outlive static teardown
    return *pool;
  }
  void copy(char *dst, const char *src, size_t bytes) {
    const size_t parts = workers_ + 1, piece = ((bytes + parts - 1) / parts + 63) & ~size_t(63);
    if (bytes < (size_t(1) << 20) || !workers_) {
      std::memcpy(dst, src, bytes);
      return;
    }
    {
      std::lock_guard<std::mutex> lock(mutex_);
      dst_ = dst;
      src_ = src;
      bytes_ = bytes;
      piece_ = piece;
      pending_ = workers_;
      ++generation_;
    }
    wake_.notify_all();
    const size_t mine = std::min(piece, bytes); // the caller copies part 0
    std::memcpy(dst, src, mine);
    std::unique_lock<std::mutex> lock(mutex_);
    done_.wait(lock, [&] { return pending_ == 0; });
  }

private:
  // All but three of the host's threads, at most 16 in total: on a 16-thread B200
  // host 14 threads move 1 GiB between pageable memory and the staging ring at
  // 47-55 GB/s (about PCIe speed), 6 threads at 35-44 GB/s.
  CopyPool() {
    const unsigned hw = std::thread::hardware_concurrency();
    workers_ = hw >= 8 ? std::min(hw - 3, 15u) : (hw >= 4 ? hw / 2 : 0);
    for (unsigned i = 0; i < workers_; ++i)
      std::thread([this, i] { run(i + 1); }).detach();
  }
  void run(unsigned part) {
    uint64_t seen = 0;
    for (;;) {
      char *dst;
      const char *src;
      size_t bytes, piece;
      {
        std::unique_lock<std::mutex> lock(mutex_);
        wake_.wait(lock, [&] { return generation_ != seen; });
        seen = generation_;
        dst = dst_, src = src_, bytes = bytes_, piece = piece_;
      }
      const size_t begin = std::min(bytes, part * piece), end = std::min(bytes, begin + piece);
      if (end > begin)
        std::memcpy(dst + begin, src + begin, end - begin);
      std::lock_guard<std::mutex> lock(mutex_);
      if (--pending_ == 0)
        done_.notify_one();
    }
  }
  unsigned workers_ = 0;
  std::mutex mutex_;
  std::condition_variable wake_, done_;
  char *dst_ = nullptr;
  const char *src_ = nullptr;
  size_t bytes_ = 0, piece_ = 0;
  unsigned pending_ = 0;
  uint64_t generation_ = 0;
};

bool pageable(const void *p) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false; // unknown: let the direct copy decide
  }
  return a.type == cudaMemoryTypeUnregistered;
}
} // namespace

// Slot i of the ring is reused only after the event recorded behind its last DMA.
bool Engine::staged_copy(bool to_device, char *device, void *host, size_t bytes) {
  if (bytes < (size_t(4) << 20) || !pageable(host))
    return false;
  if (!staging_[0]) {
    for (int i = 0; i < staging_slots; ++i) {
      if (cudaHostAlloc(reinterpret_cast<void **>(&staging_[i]), staging_slot_bytes, cudaHostAllocPortable) !=
              cudaSuccess ||
          cudaEventCreateWithFlags(&staging_events_[i], cudaEventDisableTiming) != cudaSuccess) {
        cudaGetLastError();
        for (int j = 0; j <= i; ++j) {
          if (staging_[j])
            cudaFreeHost(staging_[j]);
          if (staging_events_[j])
            cudaEventDestroy(staging_events_[j]);
          staging_[j] = nullptr;
          staging_events_[j] = nullptr;
        }
        return false; // no pinned memory: the direct copy still works
      }
    }
  }
  auto &pool = CopyPool::get();
  auto *h = static_cast<char *>(host);
  const size_t chunks = (bytes + staging_slot_bytes - 1) / staging_slot_bytes;
  auto check = [&](cudaError_t e, const char *what) {
    if (e != cudaSuccess)
      cuda_failure(e, what);
  };
  if (to_device) {
    for (size_t c = 0; c < chunks; ++c) {
      const int slot = int(c % staging_slots);
      const size_t off = c * staging_slot_bytes, len = std::min(staging_slot_bytes, bytes - off);
      if (c >= size_t(staging_slots))
        check(cudaEventSynchronize(staging_events_[slot]), "cudaEventSynchronize(staging)");
      pool.copy(staging_[slot], h + off, len);
      check(cudaMemcpyAsync(device + off, staging_[slot], len, cudaMemcpyHostToDevice, stream_),
            "cudaMemcpyAsync(host to device, staged)");
      check(cudaEventRecord(staging_events_[slot], stream_), "cudaEventRecord(staging)");
    }
    check(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");
    return true;
  }
  auto issue = [&](size_t c) {
    const int slot = int(c % staging_slots);
    const size_t off = c * staging_slot_bytes, len = std::min(staging_slot_bytes, bytes - off);
    check(cudaMemcpyAsync(staging_[slot], device + off, len, cudaMemcpyDeviceToHost, stream_),
          "cudaMemcpyAsync(device to host, staged)");
    check(cudaEventRecord(staging_events_[slot], stream_), "cudaEventRecord(staging)");
  };
  for (size_t c = 0; c < chunks && c < size_t(staging_slots); ++c)
    issue(c);
  for (size_t c = 0; c < chunks; ++c) {
    const int slot = int(c % staging_slots);
    const size_t off = c * staging_slot_bytes, len = std::min(staging_slot_bytes, bytes - off);
    check(cudaEventSynchronize(staging_events_[slot]), "cudaEventSynchronize(staging)");
    pool.copy(h + off, staging_[slot], len);
    if (c + staging_slots < chunks)
      issue(c + staging_slots);
  }
  return true;
}

// Host pointers may be pageable or pinned; any UVA address (including device
// memory of this process) is accepted because the copy kind is inferred.
void Engine::write(const std::shared_ptr<Allocation> &allocation, size_t offset,
                   const void *source, size_t bytes) {
  std::lock_guard<std::mutex> lock(mutex_);
  check_owner(*allocation);
  copy_range(*allocation, offset, bytes);
  if (bytes && !source)
    throw Error(Code::invalid_value, "Nonempty write requires a host pointer");
  drain_locked();
  const auto start = std::chrono::steady_clock::now();
  if (bytes) {
    DeviceScope scope(device_.ordinal);
    char *device = static_cast<char *>(allocation->ptr) + offset;
    if (staged_copy(true, device, const_cast<void *>(source), bytes)) {
      counters_.h2d_seconds += std::chrono::duration<double>(std::chrono::steady_clock::now() - start).count();
      counters_.h2d_bytes += bytes;
      runtime_event("transfer", "completed", "host_to_device", trace_id_, 0, bytes);
      return;
    }
    cudaError_t e = cudaMemcpyAsync(device, source, bytes, cudaMemcpyDefault, stream_);
    if (e == cudaSuccess)
      e = cudaStreamSynchronize(stream_);
    if (e != cudaSuccess)
      cuda_failure(e, "cudaMemcpy(host to device)");
  }
  counters_.h2d_seconds +=
      std::chrono::duration<double>(std::chrono::steady_clock::now() - start).count();
  counters_.h2d_bytes += bytes;
  runtime_event("transfer", "completed", "host_to_device", trace_id_, 0, bytes);
}

void Engine::read(const std::shared_ptr<Allocation> &allocation, size_t offset, void *destination,
                  size_t bytes) {
  std::lock_guard<std::mutex> lock(mutex_);
  check_owner(*allocation);
  copy_range(*allocation, offset, bytes);
  if (bytes && !destination)
    throw Error(Code::invalid_value, "Nonempty read requires a host pointer");
  drain_locked();
  const auto start = std::chrono::steady_clock::now();
  if (bytes) {
    DeviceScope scope(device_.ordinal);
    char *device = static_cast<char *>(allocation->ptr) + offset;
    if (staged_copy(false, device, destination, bytes)) {
      counters_.d2h_seconds += std::chrono::duration<double>(std::chrono::steady_clock::now() - start).count();
      counters_.d2h_bytes += bytes;
      runtime_event("transfer", "completed", "device_to_host", trace_id_, 0, bytes);
      return;
    }
    cudaError_t e = cudaMemcpyAsync(destination, device, bytes, cudaMemcpyDefault, stream_);
    if (e == cudaSuccess)
      e = cudaStreamSynchronize(stream_);
    if (e != cudaSuccess)
      cuda_failure(e, "cudaMemcpy(device to host)");
  }
  counters_.d2h_seconds +=
      std::chrono::duration<double>(std::chrono::steady_clock::now() - start).count();
  counters_.d2h_bytes += bytes;
  runtime_event("transfer", "completed", "device_to_host", trace_id_, 0, bytes);
}

void Engine::check_geometry(Dim3 grid, Dim3 block) const {
  if (!grid.x || !grid.y || !grid.z || !block.x || !block.y || !block.z)
    throw Error(Code::invalid_value, "Grid and block dimensions must be positive");
  const auto &limit = device_.max_block;
  if (block.x > limit.x || block.y > limit.y || block.z > limit.z)
    throw Error(Code::invalid_value, "Block dimension exceeds CUDA device limits");
  const uint64_t threads = uint64_t(block.x) * block.y * block.z;
  if (threads > uint64_t(device_.max_threads))
    throw Error(Code::invalid_value, "Block thread count exceeds CUDA device limits");
  if (grid.x > device_.max_grid.x || grid.y > device_.max_grid.y || grid.z > device_.max_grid.z)
    throw Error(Code::invalid_value, "Grid dimension exceeds CUDA device limits");
  const uint64_t x = uint64_t(grid.x) * block.x, y = uint64_t(grid.y) * block.y,
                 z = uint64_t(grid.z) * block.z;
  if (x > UINT32_MAX || y > UINT32_MAX || z > UINT32_MAX)
    throw Error(Code::invalid_value, "Logical grid dimension exceeds 32-bit indexing");
}

cudaEvent_t Engine::take_event() {
  if (!spare_events_.empty()) {
    auto e = spare_events_.back();
    spare_events_.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  const cudaError_t r = cudaEventCreate(&e);
  if (r != cudaSuccess)
    cuda_failure(r, "cudaEventCreate");
  return e;
}

void Engine::recycle(Work &work) {
  for (auto *e : {&work.start, &work.end})
    if (*e) {
      spare_events_.push_back(*e);
      *e = nullptr;
    }
}

std::shared_ptr<Work> Engine::submit(const std::string &name, Launcher launcher, Dim3 grid,
                                     Dim3 block, std::vector<BoundArg> args,
                                     std::vector<std::shared_ptr<Allocation>> retained,
                                     bool barrier, std::shared_ptr<const void> entry_data) {
  std::lock_guard<std::mutex> lock(mutex_);
  healthy();
  DeviceScope scope(device_.ordinal);
  auto work = std::make_shared<Work>();
  work->kernel = name;
  work->grid = grid;
  work->block = block;
  work->retained = std::move(retained);
  work->operation_id = next_operation_++;
  work->entry_owner = std::move(entry_data);
  Launch launch;
  launch.entry_data = work->entry_owner.get();
  launch.stream = stream_;
  launch.device = device_.ordinal;
  launch.sm_count = device_.sm_count;
  launch.status = status_device_;
  launch.matmul_mode = matmul_mode_;
  launch.grid = grid;
  launch.block = block;
  launch.args = std::move(args);
  launch.workspace = &Engine::workspace_hook;
  launch.workspace_owner = this;
  launch.side_stream = side_stream_;
  for (int i = 0; i < 4; ++i)
    launch.side_events[i] = side_events_[i];
  launch.dry_run = true;
  launcher(launch); // validation: throws before anything is enqueued
  launch.dry_run = false;
  reserve_more(pending_, 1);
  reserve_more(executions_, pending_.size() + 1);
  work->start = take_event();
  work->end = take_event();
  runtime_event("submission", "prepared", name, trace_id_, work->operation_id);
  try {
    order_after(0, launch.args, barrier);
  } catch (...) {
    recycle(*work);
    throw;
  }
  cudaError_t e = cudaEventRecord(work->start, stream_);
  if (e != cudaSuccess) {
    recycle(*work);
    cuda_failure(e, "cudaEventRecord");
  }
  try {
    launcher(launch);
  } catch (...) {
    // Part of the command may be enqueued: let it finish before its views go.
    cudaStreamSynchronize(side_stream_);
    cudaStreamSynchronize(stream_);
    recycle(*work);
    throw;
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    cudaStreamSynchronize(stream_);
    recycle(*work);
    cuda_failure(e, "kernel launch (" + name + ")");
  }
  work->kernels = launch.kernels;
  work->variant = launch.variant;
  pending_.push_back(work);
  e = cudaEventRecord(work->end, stream_);
  if (e != cudaSuccess) {
    const std::string text = "CUDA cudaEventRecord after launch failed: " + text_of(e);
    cudaStreamSynchronize(stream_);
    if (terminal_failure_.empty())
      terminal_failure_ = text;
    work->failure = text;
    throw Error(code_of(e), text);
  }
  remember(0, launch.args, work);
  progress("Kernel: " + name + " (" + launch.variant + ")\n");
  return work;
}

static bool overlaps(uintptr_t b0, uintptr_t e0, uintptr_t b1, uintptr_t e1) {
  return b0 < e1 && b1 < e0;
}

void Engine::order_after(int lane, const std::vector<BoundArg> &accesses, bool barrier) {
  const cudaStream_t stream = lane_stream(lane);
  for (int other = 0; other < lanes; ++other) {
    if (other == lane)
      continue;
    const auto &list = records_[other];
    // Newest first; a finished command means every older one of its lane finished
    // too (commands finish in submission order, and a lane runs in that order).
    for (auto it = list.rbegin(); it != list.rend() && !it->work->recorded; ++it) {
      bool conflict = barrier;
      for (size_t i = 0; i < accesses.size() && !conflict; ++i) {
        const auto &a = accesses[i];
        if (!a.buffer || !a.bytes)
          continue;
        const auto begin = reinterpret_cast<uintptr_t>(a.ptr);
        conflict = (a.writes || it->write) && overlaps(begin, begin + a.bytes, it->begin, it->end);
      }
      if (conflict) {
        const cudaError_t e = cudaStreamWaitEvent(stream, it->work->end, 0);
        if (e != cudaSuccess)
          cuda_failure(e, "cudaStreamWaitEvent");
        break;
      }
    }
  }
}

void Engine::remember(int lane, const std::vector<BoundArg> &accesses,
                      const std::shared_ptr<Work> &work) {
  auto &list = records_[lane];
  for (const auto &a : accesses)
    if (a.buffer && a.bytes) {
      const auto begin = reinterpret_cast<uintptr_t>(a.ptr);
      list.push_back({begin, begin + a.bytes, a.writes, work});
    }
  if (list.size() > 256)
    prune(lane);
}

// Drops the records of commands that the device has finished: the lane is in
// order, so a binary search finds the newest finished one.
void Engine::prune(int lane) {
  auto &list = records_[lane];
  auto finished = [](const Record &r) {
    if (r.work->recorded)
      return true;
    const cudaError_t e = cudaEventQuery(r.work->end);
    if (e == cudaErrorNotReady && cudaPeekAtLastError() == cudaErrorNotReady)
      cudaGetLastError(); // not-ready is a state, not a failure for the next launch check
    return e == cudaSuccess;
  };
  size_t lo = 0, hi = list.size(); // records [0, lo) finished; [hi, size) not
  while (lo < hi) {
    const size_t mid = lo + (hi - lo) / 2;
    if (finished(list[mid]))
      lo = mid + 1;
    else
      hi = mid;
  }
  list.erase(list.begin(), list.begin() + lo);
}

std::shared_ptr<Work> Engine::transfer(bool to_device, const std::shared_ptr<Allocation> &allocation,
                                       size_t offset, void *host, size_t bytes) {
  std::lock_guard<std::mutex> lock(mutex_);
  healthy();
  check_owner(*allocation);
  copy_range(*allocation, offset, bytes);
  if (!host || !bytes)
    throw Error(Code::invalid_value, "An asynchronous copy needs a host pointer and a nonzero size");
  DeviceScope scope(device_.ordinal);
  const int lane = to_device ? 1 : 2;
  const cudaStream_t stream = lane_stream(lane);
  auto work = std::make_shared<Work>();
  work->kernel = to_device ? "b200_buffer_write_async" : "b200_buffer_read_async";
  work->variant = "copy_engine";
  work->transfer = true;
  work->to_device = to_device;
  work->device = device_.ordinal;
  work->retained.push_back(allocation);
  work->operation_id = next_operation_++;
  std::vector<BoundArg> access(1);
  access[0].buffer = true;
  access[0].writes = to_device;
  access[0].ptr = static_cast<char *>(allocation->ptr) + offset;
  access[0].bytes = bytes;
  reserve_more(pending_, 1);
  work->start = take_event();
  work->end = take_event();
  order_after(lane, access, false);
  cudaError_t e = cudaEventRecord(work->start, stream);
  if (e == cudaSuccess)
    e = to_device ? cudaMemcpyAsync(access[0].ptr, host, bytes, cudaMemcpyDefault, stream)
                  : cudaMemcpyAsync(host, access[0].ptr, bytes, cudaMemcpyDefault, stream);
  if (e != cudaSuccess) {
    cudaStreamSynchronize(stream);
    recycle(*work);
    cuda_failure(e, to_device ? "cudaMemcpyAsync(host to device)" : "cudaMemcpyAsync(device to host)");
  }
  pending_.push_back(work);
  e = cudaEventRecord(work->end, stream);
  if (e != cudaSuccess) {
    const std::string text = "CUDA cudaEventRecord after copy failed: " + text_of(e);
    cudaStreamSynchronize(stream);
    if (terminal_failure_.empty())
      terminal_failure_ = text;
    work->failure = text;
    throw Error(code_of(e), text);
  }
  remember(lane, access, work);
  (to_device ? counters_.h2d_bytes : counters_.d2h_bytes) += bytes;
  runtime_event("transfer", "enqueued", to_device ? "host_to_device" : "device_to_host", trace_id_,
                work->operation_id, bytes);
  return work;
}

void Engine::finish(const std::shared_ptr<Work> &work) {
  if (work->recorded)
    return;
  std::string failure = work->failure;
  bool completed = false;
  double milliseconds = 0;
  if (failure.empty()) {
    cudaError_t e = cudaEventSynchronize(work->end);
    if (e != cudaSuccess) {
      failure = "CUDA command failed for " + work->kernel + ": " + text_of(e);
      if (is_sticky(e) && terminal_failure_.empty())
        terminal_failure_ = failure;
    } else {
      completed = true;
      float ms = 0;
      e = cudaEventElapsedTime(&ms, work->start, work->end);
      if (e != cudaSuccess)
        failure = "CUDA completed " + work->kernel + " without GPU duration evidence: " + text_of(e);
      else if (!std::isfinite(ms) || ms < 0)
        failure = "CUDA completed " + work->kernel + " with an invalid GPU duration";
      else
        milliseconds = ms;
      // A kernel that gave up a bounded wait reports it through the status word.
      const int status = work->transfer ? 0 : __atomic_exchange_n(status_host_, 0, __ATOMIC_ACQ_REL);
      if (status == status_out_of_view && failure.empty())
        failure = "Kernel " + work->kernel + " addressed elements outside its bound views; those "
                  "loads read 0 and those stores were skipped";
      else if (status == prepared::status_mismatch && failure.empty())
        failure = "Kernel " + work->kernel + " was given a prepared operand that was not prepared for its "
                  "k and n; its output is undefined";
      else if (status != 0 && failure.empty())
        failure = "Kernel " + work->kernel + " abandoned a bounded wait (status " +
                  std::to_string(status) + ")";
    }
  }
  if (work->keep_end && completed) {
    cudaEvent_t end = work->end;
    work->end = nullptr;
    recycle(*work);
    work->end = end; // destroyed with the Work
  } else {
    recycle(*work);
  }
  work->info = {};
  work->info.completed = completed;
  if (completed && failure.empty()) {
    work->info.duration_valid = true;
    work->info.duration_seconds = milliseconds / 1000.0;
    if (work->transfer) {
      (work->to_device ? counters_.h2d_seconds : counters_.d2h_seconds) += work->info.duration_seconds;
    } else {
      counters_.gpu_seconds += work->info.duration_seconds;
      ++counters_.completed_launches;
      counters_.device_kernels += work->kernels;
    }
  }
  if (!work->transfer)
    executions_.push_back({work->kernel, work->variant, failure, work->grid, work->block,
                           work->kernels, work->info.duration_seconds, completed});
  if (!failure.empty() && terminal_failure_.empty())
    terminal_failure_ = failure;
  work->failure = failure;
  work->recorded = true;
  work->retained.clear();
  work->entry_owner.reset();
  runtime_event("completion", failure.empty() ? "completed" : "failed",
                failure.empty() ? work->kernel : failure, trace_id_, work->operation_id);
}

void Engine::drain_locked() {
  DeviceScope scope(device_.ordinal);
  for (const auto &work : pending_)
    finish(work);
  pending_.clear();
  for (auto &list : records_)
    list.clear();
  healthy();
}

void Engine::synchronize() {
  std::lock_guard<std::mutex> lock(mutex_);
  drain_locked();
}

EventInfo Engine::wait(const std::shared_ptr<Work> &work) {
  std::lock_guard<std::mutex> lock(mutex_);
  auto end = std::find(pending_.begin(), pending_.end(), work);
  if (end != pending_.end()) {
    DeviceScope scope(device_.ordinal);
    ++end;
    for (auto it = pending_.begin(); it != end; ++it)
      finish(*it);
    pending_.erase(pending_.begin(), end);
  }
  healthy();
  if (!work->recorded)
    throw Error(Code::internal, "Event has no recorded command");
  return work->info;
}

Work::~Work() {
  if (keep_end && end && recorded) {
    int previous = -1;
    cudaGetDevice(&previous);
    if (previous != device)
      cudaSetDevice(device);
    cudaEventDestroy(end);
    if (previous >= 0 && previous != device)
      cudaSetDevice(previous);
  }
}

static void marker_launch(Launch &L) { L.variant = "marker"; }

// Called by launchers with the engine lock held. Growing waits for the stream so
// no queued kernel still reads the old block; the old block is then freed.
void *Engine::workspace_hook(void *self, size_t bytes) {
  auto *engine = static_cast<Engine *>(self);
  if (bytes <= engine->workspace_bytes_)
    return engine->workspace_;
  const size_t rounded = (bytes + (size_t(64) << 20) - 1) & ~((size_t(64) << 20) - 1);
  if (engine->workspace_) {
    if (cudaStreamSynchronize(engine->side_stream_) != cudaSuccess ||
        cudaStreamSynchronize(engine->stream_) != cudaSuccess)
      return nullptr;
    cudaFree(engine->workspace_);
    engine->workspace_ = nullptr;
    engine->workspace_bytes_ = 0;
  }
  void *p = nullptr;
  if (cudaMalloc(&p, rounded) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  engine->workspace_ = p;
  engine->workspace_bytes_ = rounded;
  return p;
}

std::shared_ptr<Work> Engine::marker() {
  auto work = submit("b200_marker", marker_launch, Dim3{}, Dim3{}, {}, {}, true);
  std::lock_guard<std::mutex> lock(mutex_);
  work->keep_end = true;
  work->device = device_.ordinal;
  return work;
}

double Engine::elapsed(const std::shared_ptr<Work> &first, const std::shared_ptr<Work> &second) {
  wait(first);
  wait(second);
  std::lock_guard<std::mutex> lock(mutex_);
  if (!first->keep_end || !second->keep_end || !first->end || !second->end)
    throw Error(Code::invalid_value, "Elapsed time is defined between two completed markers");
  DeviceScope scope(device_.ordinal);
  float ms = 0;
  const cudaError_t e = cudaEventElapsedTime(&ms, first->end, second->end);
  if (e != cudaSuccess)
    cuda_failure(e, "cudaEventElapsedTime");
  return ms / 1000.0;
}

Statistics Engine::statistics() const {
  std::lock_guard<std::mutex> lock(mutex_);
  return counters_;
}

void Engine::write_evidence(const std::string &directory) {
  std::lock_guard<std::mutex> lock(mutex_);
  std::exception_ptr failure;
  try {
    drain_locked();
  } catch (...) {
    failure = std::current_exception();
  }
  namespace fs = std::filesystem;
  fs::create_directories(directory);
  std::ostringstream out;
  out << std::setprecision(17) << "{\n  \"backend\": \"CUDA\",\n  \"device\": " << json(device_.name)
      << ",\n  \"device_ordinal\": " << device_.ordinal
      << ",\n  \"stable_device_id\": " << json(device_.stable_id)
      << ",\n  \"compute_capability\": "
      << json(std::to_string(device_.cc_major) + "." + std::to_string(device_.cc_minor))
      << ",\n  \"kernels\": \"ahead-of-time sm_100a (nvcc)\""
      << ",\n  \"cuda_runtime_version\": " << backend_status().runtime_version
      << ",\n  \"cuda_driver_version\": " << backend_status().driver_version
      << ",\n  \"os\": " << json(device_.os) << ",\n  \"cpu_fallback\": false"
      << ",\n  \"test_double\": false"
      << ",\n  \"runtime_owned_current_buffer_bytes\": " << accounting_->current.load()
      << ",\n  \"runtime_owned_peak_buffer_bytes\": " << accounting_->peak.load()
      << ",\n  \"host_to_device_bytes\": " << counters_.h2d_bytes
      << ",\n  \"device_to_host_bytes\": " << counters_.d2h_bytes << ",\n  \"launches\": [\n";
  for (size_t i = 0; i < executions_.size(); ++i) {
    const auto &e = executions_[i];
    const bool valid = e.complete && e.error.empty();
    out << "    {\"kernel\": " << json(e.kernel) << ", \"variant\": " << json(e.variant)
        << ", \"grid\": [" << e.grid.x << ',' << e.grid.y << ',' << e.grid.z << "], \"block\": ["
        << e.block.x << ',' << e.block.y << ',' << e.block.z
        << "], \"device_kernels\": " << e.kernels
        << ", \"command_status\": " << json(e.complete ? "completed" : "failed")
        << ", \"gpu_duration_seconds\": ";
    if (valid)
      out << e.duration;
    else
      out << "null";
    out << ", \"gpu_duration_valid\": " << (valid ? "true" : "false")
        << ", \"gpu_timestamps_valid\": false, \"gpu_clock_domain\": \"duration_only\""
        << ", \"error\": " << json(e.error) << '}' << (i + 1 == executions_.size() ? "\n" : ",\n");
  }
  out << "  ]\n}\n";
  std::ofstream file(fs::path(directory) / "execution.json", std::ios::binary);
  file << out.str();
  file.close();
  if (!file)
    throw Error(Code::internal, "Cannot write execution.json");
  if (failure)
    std::rethrow_exception(failure);
}

std::shared_ptr<Engine> create_engine(const std::string &selector) {
  uint32_t ordinal = 0;
  if (selector.rfind("cuda:", 0) == 0) {
    const std::string digits = selector.substr(5);
    if (digits.empty() || digits.size() > 10 ||
        digits.find_first_not_of("0123456789") != std::string::npos)
      throw Error(Code::invalid_device,
                  "CUDA selectors have the form cuda:INDEX (decimal device ordinal)");
    const auto value = std::stoull(digits);
    if (value > 0x7fffffffULL)
      throw Error(Code::invalid_device, "CUDA device ordinal is out of range for cuda:INDEX");
    ordinal = uint32_t(value);
  } else if (selector.rfind("hip:", 0) == 0 || selector.rfind("rocm:", 0) == 0) {
    throw Error(Code::invalid_device, "The HIP/ROCm backend is not implemented.");
  } else if (selector != "auto") {
    throw Error(Code::invalid_device,
                "This library has no Metal backend; select a CUDA device with cuda:INDEX or auto. "
                "There is no CPU fallback.");
  }
  const auto &status = backend_status();
  if (!status.available)
    throw Error(Code::invalid_device, "CUDA backend unavailable: " + status.reason);
  const auto &list = devices();
  if (ordinal >= list.size())
    throw Error(Code::invalid_device, "CUDA device index is out of range (" +
                                          std::to_string(list.size()) +
                                          " device(s) reported by the driver)");
  const auto &d = list[ordinal];
  if (d.cc_major != 10 || d.cc_minor != 0)
    throw Error(Code::unsupported, "This library carries sm_100a kernels only; device " + d.name +
                                       " has compute capability " + std::to_string(d.cc_major) +
                                       "." + std::to_string(d.cc_minor));
  return std::make_shared<Engine>(d);
}

} // namespace pb
