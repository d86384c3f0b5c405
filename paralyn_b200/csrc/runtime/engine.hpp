// CUDA engine: one instance per context. It owns one ordered stream on a device's
// primary context, the allocations made through it, a list of submitted work with
// per-launch start/end events (duration-only timing), a sticky terminal failure and
// the launch log written as execution.json.
//
// Behaviour follows the reference's CUDA engine (backends/cuda/engine.cpp):
// copies drain the queue first and are blocking (:435-470), each launch is
// bracketed by two events (:684-715), completion is observed in submission order
// (:719-799), the first command failure becomes sticky (:396-404, :762-773) and
// evidence lists every launch (:800-858). Unlike it, kernels are compiled ahead of
// time for sm_100a and launched through the CUDA runtime API.
#pragma once
#include "builtin.hpp"
#include <deque>
#include <memory>
#include <mutex>

namespace pb {

struct DeviceRecord {
  int ordinal = 0;
  std::string name, stable_id, os;
  uint64_t total_memory = 0, max_smem_block = 0, registry_id = 0;
  int sm_count = 0, cc_major = 0, cc_minor = 0, max_threads = 0;
  Dim3 max_block, max_grid;
  bool integrated = false;
};

struct BackendStatus {
  bool available = false;
  int device_count = 0, driver_version = 0, runtime_version = 0;
  std::string reason;
};

// Queried once per process; absence of a driver or device is a status, not a throw.
const BackendStatus &backend_status();
const std::vector<DeviceRecord> &devices();

struct Allocation {
  int device = 0;
  void *ptr = nullptr;
  size_t bytes = 0;
  const void *owner = nullptr; // identity of the creating engine
  bool imported = false;       // a peer GPU's allocation mapped into this context (CUDA IPC)
  std::shared_ptr<struct Accounting> accounting;
  ~Allocation();
};

// What pr_b200_buffer_export hands to another process: the CUDA IPC handle of
// the allocation and its size.
struct PeerHandle {
  cudaIpcMemHandle_t handle;
  uint64_t bytes;
};

struct EventInfo {
  bool completed = false, duration_valid = false;
  double duration_seconds = 0;
};

struct Work {
  cudaEvent_t start = nullptr, end = nullptr;
  std::vector<std::shared_ptr<Allocation>> retained;
  std::shared_ptr<const void> entry_owner; // keeps a run-time compiled kernel loaded
  std::string kernel, variant;
  Dim3 grid, block;
  uint32_t kernels = 0;
  uint64_t operation_id = 0;
  bool recorded = false;
  bool keep_end = false; // markers keep their end timestamp for elapsed-time queries
  bool transfer = false; // a stream-ordered host copy (not a kernel launch)
  bool to_device = false;
  int device = 0;
  EventInfo info;
  std::string failure;
  ~Work();
};

struct Statistics {
  uint64_t h2d_bytes = 0, d2h_bytes = 0, completed_launches = 0, device_kernels = 0;
  double h2d_seconds = 0, d2h_seconds = 0, gpu_seconds = 0;
};

class Engine : public std::enable_shared_from_this<Engine> {
public:
  explicit Engine(const DeviceRecord &device);
  ~Engine();
  Engine(const Engine &) = delete;
  Engine &operator=(const Engine &) = delete;

  const DeviceRecord &device() const { return device_; }
  std::shared_ptr<Allocation> allocate(size_t bytes);
  PeerHandle export_allocation(const Allocation &allocation);
  // Maps another process's exported allocation (any GPU of this node) into this
  // context; kernels of this context then read and write it over NVLink.
  std::shared_ptr<Allocation> import_allocation(const PeerHandle &handle);
  void write(const std::shared_ptr<Allocation> &, size_t offset, const void *source, size_t bytes);
  void read(const std::shared_ptr<Allocation> &, size_t offset, void *destination, size_t bytes);
  // Checks a pr_launch geometry against the device limits (reference engine.cpp:597-616).
  void check_geometry(Dim3 grid, Dim3 block) const;
  // Runs `launcher` between two events on the context stream; retains the views.
  std::shared_ptr<Work> submit(const std::string &name, Launcher launcher, Dim3 grid, Dim3 block,
                               std::vector<BoundArg> args,
                               std::vector<std::shared_ptr<Allocation>> retained,
                               bool barrier = false, std::shared_ptr<const void> entry_data = nullptr);
  EventInfo wait(const std::shared_ptr<Work> &work);
  // A host <-> device copy enqueued as a command without blocking the caller. It runs
  // on the copy lane of its direction after every earlier command that touches the
  // same bytes (read-after-write, write-after-read, write-after-write), and commands
  // submitted later order themselves after it the same way; commands on other bytes
  // overlap it. `host` must stay valid until the Work completes.
  std::shared_ptr<Work> transfer(bool to_device, const std::shared_ptr<Allocation> &allocation,
                                 size_t offset, void *host, size_t bytes);
  // An empty command that records a device timestamp (kept until the Work dies). It
  // follows every earlier command, copies included.
  std::shared_ptr<Work> marker();
  // Device seconds between the completion of two markers of this engine.
  double elapsed(const std::shared_ptr<Work> &first, const std::shared_ptr<Work> &second);
  void synchronize();
  void write_evidence(const std::string &directory);
  void check_owner(const Allocation &allocation) const;
  cudaStream_t stream() const { return stream_; }
  uint32_t matmul_mode() const { return matmul_mode_; }
  void set_matmul_mode(uint32_t mode) { matmul_mode_ = mode; }
  Statistics statistics() const;

private:
  struct Execution {
    std::string kernel, variant, error;
    Dim3 grid, block;
    uint32_t kernels;
    double duration;
    bool complete;
  };
  void healthy() const;
  [[noreturn]] void cuda_failure(cudaError_t code, const std::string &operation);
  void finish(const std::shared_ptr<Work> &work);
  void drain_locked();
  cudaEvent_t take_event();
  void recycle(Work &work);
  static void *workspace_hook(void *self, size_t bytes);
  // Cross-lane ordering. Lane 0 is the kernel stream, 1 host-to-device copies,
  // 2 device-to-host copies; each lane is one in-order CUDA stream, so a command
  // waits at most once per other lane: on the newest unfinished command there whose
  // byte range overlaps one of its own with at least one of the two writing.
  static constexpr int lanes = 3;
  struct Record {
    uintptr_t begin, end;
    bool write;
    std::shared_ptr<Work> work;
  };
  cudaStream_t lane_stream(int lane) const { return lane == 0 ? stream_ : copy_streams_[lane - 1]; }
  void order_after(int lane, const std::vector<BoundArg> &accesses, bool barrier);
  void remember(int lane, const std::vector<BoundArg> &accesses, const std::shared_ptr<Work> &work);
  void prune(int lane);
  std::deque<Record> records_[lanes];
  cudaStream_t copy_streams_[2] = {};
  // Blocking copies from or to pageable host memory go through a ring of pinned
  // staging slots (allocated on first use): host-side memcpy of one slot (several
  // threads) overlaps the DMA of the previous one.
  static constexpr int staging_slots = 4;
  static constexpr size_t staging_slot_bytes = size_t(16) << 20;
  bool staged_copy(bool to_device, char *device, void *host, size_t bytes);
  char *staging_[staging_slots] = {};
  cudaEvent_t staging_events_[staging_slots] = {};
  void *workspace_ = nullptr;
  size_t workspace_bytes_ = 0;

  DeviceRecord device_;
  cudaStream_t stream_ = nullptr;
  cudaStream_t side_stream_ = nullptr;
  cudaEvent_t side_events_[4] = {};
  int *status_host_ = nullptr, *status_device_ = nullptr;
  mutable std::mutex mutex_;
  std::vector<std::shared_ptr<Work>> pending_;
  std::vector<Execution> executions_;
  std::vector<cudaEvent_t> spare_events_;
  std::string terminal_failure_;
  Statistics counters_;
  std::shared_ptr<struct Accounting> accounting_;
  uint64_t next_operation_ = 1;
  uint64_t trace_id_ = 0;
  uint32_t matmul_mode_ = matmul_auto;
};

// "cuda:K" or "auto" (cuda:0). Metal/HIP selectors are unavailable in this library.
std::shared_ptr<Engine> create_engine(const std::string &selector);

// JSON-lines runtime events to PARALYN_EVENT_LOG, progress to PARALYN_RUNTIME_LOG
// (reference runtime/telemetry.cpp:36-86); both are no-ops when unset.
void runtime_event(const std::string &category, const std::string &status,
                   const std::string &detail, uint64_t context_id = 0, uint64_t operation_id = 0,
                   uint64_t bytes = 0);
void progress(const std::string &message);

} // namespace pb
