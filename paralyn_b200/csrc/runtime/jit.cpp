// Run-time compiled kernels for verified IR (see jit.hpp).
#include "jit.hpp"
#include <cuda.h>
#include <cuda_runtime.h>
#include <nvrtc.h>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <dlfcn.h>
#include <sstream>
#include <unordered_map>

namespace pb {
namespace {

// ---- NVRTC, loaded on first use (the library does not link it) ----
struct Nvrtc {
  nvrtcResult (*create)(nvrtcProgram *, const char *, const char *, int, const char *const *,
                        const char *const *) = nullptr;
  nvrtcResult (*compile)(nvrtcProgram, int, const char *const *) = nullptr;
  nvrtcResult (*cubin_size)(nvrtcProgram, size_t *) = nullptr;
  nvrtcResult (*cubin)(nvrtcProgram, char *) = nullptr;
  nvrtcResult (*log_size)(nvrtcProgram, size_t *) = nullptr;
  nvrtcResult (*log)(nvrtcProgram, char *) = nullptr;
  nvrtcResult (*destroy)(nvrtcProgram *) = nullptr;
  const char *(*error)(nvrtcResult) = nullptr;
  std::string failure;
};

const Nvrtc &nvrtc() {
  static const Nvrtc api = [] {
    Nvrtc n;
    std::vector<std::string> candidates;
    if (const char *path = std::getenv("PARALYN_NVRTC_LIBRARY"))
      candidates.push_back(path);
    candidates.insert(candidates.end(), {"libnvrtc.so.12", "libnvrtc.so", "/usr/local/cuda/lib64/libnvrtc.so.12"});
    void *handle = nullptr;
    for (const auto &c : candidates)
      if ((handle = dlopen(c.c_str(), RTLD_NOW | RTLD_LOCAL)))
        break;
    if (!handle) {
      n.failure = "NVRTC library not found (set PARALYN_NVRTC_LIBRARY)";
      return n;
    }
    auto sym = [&](const char *name) { return dlsym(handle, name); };
    n.create = reinterpret_cast<decltype(n.create)>(sym("nvrtcCreateProgram"));
    n.compile = reinterpret_cast<decltype(n.compile)>(sym("nvrtcCompileProgram"));
    n.cubin_size = reinterpret_cast<decltype(n.cubin_size)>(sym("nvrtcGetCUBINSize"));
    n.cubin = reinterpret_cast<decltype(n.cubin)>(sym("nvrtcGetCUBIN"));
    n.log_size = reinterpret_cast<decltype(n.log_size)>(sym("nvrtcGetProgramLogSize"));
    n.log = reinterpret_cast<decltype(n.log)>(sym("nvrtcGetProgramLog"));
    n.destroy = reinterpret_cast<decltype(n.destroy)>(sym("nvrtcDestroyProgram"));
    n.error = reinterpret_cast<decltype(n.error)>(sym("nvrtcGetErrorString"));
    if (!n.create || !n.compile || !n.cubin_size || !n.cubin || !n.log_size || !n.log || !n.destroy)
      n.failure = "NVRTC library lacks the CUBIN entry points";
    return n;
  }();
  return api;
}

// ---- driver entry points (through the runtime; no link against libcuda) ----
struct Driver {
  CUresult (*load)(CUmodule *, const void *) = nullptr;
  CUresult (*get)(CUfunction *, CUmodule, const char *) = nullptr;
  CUresult (*unload)(CUmodule) = nullptr;
  CUresult (*attribute)(int *, CUfunction_attribute, CUfunction) = nullptr;
  CUresult (*launch)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, CUstream,
                     void **, void **) = nullptr;
};

const Driver &driver() {
  static const Driver api = [] {
    Driver d;
    auto entry = [](const char *name) -> void * {
      void *p = nullptr;
      cudaDriverEntryPointQueryResult q{};
      if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess ||
          q != cudaDriverEntryPointSuccess) {
        cudaGetLastError();
        return nullptr;
      }
      return p;
    };
    d.load = reinterpret_cast<decltype(d.load)>(entry("cuModuleLoadData"));
    d.get = reinterpret_cast<decltype(d.get)>(entry("cuModuleGetFunction"));
    d.unload = reinterpret_cast<decltype(d.unload)>(entry("cuModuleUnload"));
    d.attribute = reinterpret_cast<decltype(d.attribute)>(entry("cuFuncGetAttribute"));
    d.launch = reinterpret_cast<decltype(d.launch)>(entry("cuLaunchKernel"));
    return d;
  }();
  return api;
}

struct CurrentDevice {
  int previous = -1;
  explicit CurrentDevice(int device) {
    cudaGetDevice(&previous);
    if (previous != device)
      cuda_check(cudaSetDevice(device), "cudaSetDevice");
  }
  ~CurrentDevice() {
    int now = -1;
    cudaGetDevice(&now);
    if (previous >= 0 && now != previous)
      cudaSetDevice(previous);
  }
};

// ---- CUDA C++ from verified IR ----
const char *ctype(IrType t) {
  switch (t) {
  case IrType::I32: return "int";
  case IrType::U32: return "unsigned int";
  case IrType::F32: return "float";
  case IrType::Bool: return "bool";
  }
  throw Failure(PR_INTERNAL_ERROR, "unknown IR type");
}

constexpr const char *prelude = R"(// Compiled at run time from verified Paralyn IR for sm_100a.
// FP32 + and * round separately (__fadd_rn, __fmul_rn; --fmad=false, --ftz=false);
// integer + and * wrap modulo 2^32; every buffer access is checked against the
// element count of its bound view (out-of-view loads read 0, stores are skipped,
// and the launch reports the out-of-view status).
__device__ __forceinline__ long long pb_index(int i) { return i; }
__device__ __forceinline__ long long pb_index(unsigned int i) { return (long long)i; }
template <class T>
__device__ __forceinline__ T pb_ld(const T *p, long long i, unsigned long long n, int *status) {
  if (i >= 0 && (unsigned long long)i < n)
    return p[i];
  *(volatile int *)status = 0x7f3f01;
  return T(0);
}
template <class T>
__device__ __forceinline__ void pb_st(T *p, long long i, unsigned long long n, int *status, T v) {
  if (i >= 0 && (unsigned long long)i < n)
    p[i] = v;
  else
    *(volatile int *)status = 0x7f3f01;
}
)";

struct Emitter {
  std::ostringstream out;
  std::map<std::string, std::string> names;
  std::map<std::string, size_t> buffers; // buffer parameter name -> parameter index
  unsigned locals = 0;

  std::string literal(const Expr &e) {
    switch (e.type) {
    case IrType::F32: {
      const float f = std::strtof(e.text.c_str(), nullptr);
      uint32_t bits;
      std::memcpy(&bits, &f, 4);
      return "__uint_as_float(" + std::to_string(bits) + "u)";
    }
    case IrType::U32: return std::to_string(std::strtoull(e.text.c_str(), nullptr, 10)) + "u";
    case IrType::I32: return "((int)(" + std::to_string(std::strtoll(e.text.c_str(), nullptr, 10)) + "ll))";
    case IrType::Bool: return e.text == "1" ? "true" : "false";
    }
    throw Failure(PR_INTERNAL_ERROR, "unknown literal type");
  }

  std::string expr(const Expr &e) {
    switch (e.kind) {
    case ExprKind::Literal: return literal(e);
    case ExprKind::Ref: return names.at(e.text);
    case ExprKind::Builtin: return "(" + e.text + ")";
    case ExprKind::Cast: return std::string("((") + ctype(e.type) + ")(" + expr(e.operands[0]) + "))";
    case ExprKind::Binary: {
      const std::string a = expr(e.operands[0]), b = expr(e.operands[1]);
      const IrType t = e.operands[0].type;
      if (e.text == "<")
        return "(" + a + " < " + b + ")";
      const bool add = e.text == "+";
      if (t == IrType::F32)
        return std::string(add ? "__fadd_rn(" : "__fmul_rn(") + a + ", " + b + ")";
      const std::string wrapped = "((unsigned int)(" + a + ")" + (add ? " + " : " * ") + "(unsigned int)(" + b + "))";
      return t == IrType::I32 ? "((int)" + wrapped + ")" : wrapped;
    }
    case ExprKind::Load: {
      const size_t i = buffers.at(e.operands[0].text);
      return "pb_ld(uc_arg_" + std::to_string(i) + ", pb_index(" + expr(e.operands[1]) + "), pb_n_" +
             std::to_string(i) + ", pb_status)";
    }
    }
    throw Failure(PR_INTERNAL_ERROR, "unknown IR expression");
  }

  void body(const std::vector<Stmt> &statements, unsigned indent) {
    const auto saved = names;
    for (const auto &s : statements) {
      out << std::string(indent, ' ');
      if (s.kind == StmtKind::Let) {
        const std::string value = expr(s.expression), local = "uc_local_" + std::to_string(locals++);
        names[s.name] = local;
        out << ctype(s.type) << " " << local << " = " << value << ";\n";
      } else if (s.kind == StmtKind::Store) {
        const size_t i = buffers.at(s.target.operands[0].text);
        out << "pb_st(uc_arg_" << i << ", pb_index(" << expr(s.target.operands[1]) << "), pb_n_" << i
            << ", pb_status, (" << ctype(s.type) << ")(" << expr(s.expression) << "));\n";
      } else {
        out << "if (" << expr(s.expression) << ") {\n";
        body(s.body, indent + 2);
        out << std::string(indent, ' ') << "}\n";
      }
    }
    names = saved; // locals of a block end with it
  }
};

std::string nvrtc_text(nvrtcResult r) {
  const auto &n = nvrtc();
  const char *text = n.error ? n.error(r) : nullptr;
  return std::string(text ? text : "NVRTC error") + " (" + std::to_string(int(r)) + ")";
}

} // namespace

std::string emit_ir_cuda(const IrKernel &k) {
  verify_ir(k);
  Emitter e;
  e.out << prelude << "extern \"C\" __global__ void pb_ir_kernel(";
  for (size_t i = 0; i < k.params.size(); ++i) {
    const auto &p = k.params[i];
    const std::string name = "uc_arg_" + std::to_string(i);
    e.names[p.name] = name;
    if (p.buffer)
      e.buffers[p.name] = i;
    e.out << (i ? ",\n    " : "\n    ");
    if (p.buffer)
      e.out << (p.read_only ? "const " : "") << ctype(p.type) << " *" << name;
    else
      e.out << ctype(p.type) << " " << name;
  }
  for (size_t i = 0; i < k.params.size(); ++i)
    if (k.params[i].buffer)
      e.out << ",\n    unsigned long long pb_n_" << i;
  e.out << ",\n    int *pb_status) {\n";
  e.body(k.body, 2);
  e.out << "}\n";
  return e.out.str();
}

std::shared_ptr<JitKernel> compile_ir(const IrKernel &k) {
  static std::mutex cache_mutex;
  static std::unordered_map<std::string, std::weak_ptr<JitKernel>> cache;
  std::string source = emit_ir_cuda(k);
  std::lock_guard<std::mutex> lock(cache_mutex);
  if (auto hit = cache[source].lock()) {
    auto copy = std::make_shared<JitKernel>();
    copy->name = k.name;
    copy->entry = hit->entry;
    copy->source = hit->source;
    copy->params = k.params;
    copy->cubin = hit->cubin;
    return copy;
  }
  const auto &n = nvrtc();
  if (!n.failure.empty())
    throw Failure(PR_UNSUPPORTED, "Kernel " + k.name + " needs the run-time compiler: " + n.failure);
  const auto start = std::chrono::steady_clock::now();
  nvrtcProgram program = nullptr;
  nvrtcResult r = n.create(&program, source.c_str(), "paralyn_ir.cu", 0, nullptr, nullptr);
  if (r != NVRTC_SUCCESS)
    throw Failure(PR_COMPILATION_FAILED, "NVRTC could not create a program: " + nvrtc_text(r));
  struct Destroy {
    const Nvrtc &api;
    nvrtcProgram &program;
    ~Destroy() { api.destroy(&program); }
  } destroy{n, program};
  const char *options[] = {"--gpu-architecture=sm_100a", "--fmad=false", "--ftz=false", "--prec-div=true",
                           "--prec-sqrt=true", "--std=c++17"};
  r = n.compile(program, int(sizeof(options) / sizeof(options[0])), options);
  std::string log;
  size_t log_bytes = 0;
  if (n.log_size(program, &log_bytes) == NVRTC_SUCCESS && log_bytes > 1) {
    log.resize(log_bytes);
    if (n.log(program, log.data()) == NVRTC_SUCCESS)
      log.resize(std::strlen(log.c_str()));
  }
  if (r != NVRTC_SUCCESS)
    throw Failure(PR_COMPILATION_FAILED, "NVRTC compilation of " + k.name + " failed: " + nvrtc_text(r) + "\n" + log);
  size_t bytes = 0;
  r = n.cubin_size(program, &bytes);
  if (r != NVRTC_SUCCESS || !bytes)
    throw Failure(PR_COMPILATION_FAILED, "NVRTC returned no sm_100a cubin: " + nvrtc_text(r));
  auto kernel = std::make_shared<JitKernel>();
  kernel->name = k.name;
  kernel->entry = "pb_ir_kernel";
  kernel->source = std::move(source);
  kernel->params = k.params;
  kernel->cubin.resize(bytes);
  r = n.cubin(program, kernel->cubin.data());
  if (r != NVRTC_SUCCESS)
    throw Failure(PR_COMPILATION_FAILED, "NVRTC cubin retrieval failed: " + nvrtc_text(r));
  kernel->compile_seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - start).count();
  cache[kernel->source] = kernel;
  return kernel;
}

void *JitKernel::function(int device) {
  std::lock_guard<std::mutex> lock(mutex);
  const auto found = loaded.find(device);
  if (found != loaded.end())
    return found->second.second;
  const auto &d = driver();
  if (!d.load || !d.get || !d.launch)
    throw Failure(PR_DEVICE_UNAVAILABLE, "CUDA driver entry points for module loading are unavailable");
  CurrentDevice scope(device);
  CUmodule module = nullptr;
  CUresult r = d.load(&module, cubin.data());
  if (r != CUDA_SUCCESS)
    throw Failure(PR_COMPILATION_FAILED, "cuModuleLoadData failed for " + name + " (CUresult " +
                                             std::to_string(int(r)) + ")");
  CUfunction fn = nullptr;
  r = d.get(&fn, module, entry.c_str());
  if (r != CUDA_SUCCESS) {
    d.unload(module);
    throw Failure(PR_COMPILATION_FAILED, "cuModuleGetFunction failed for " + name);
  }
  loaded[device] = {module, fn};
  return fn;
}

JitKernel::~JitKernel() {
  const auto &d = driver();
  for (const auto &entry : loaded)
    if (d.unload) {
      int previous = -1;
      cudaGetDevice(&previous);
      cudaSetDevice(entry.first);
      d.unload(static_cast<CUmodule>(entry.second.first));
      if (previous >= 0)
        cudaSetDevice(previous);
    }
}

namespace {
// Arguments in parameter order, then one element count per buffer parameter, then
// the status word; geometry is the caller's, as for the reference's generic kernels.
void launch_jit(Launch &L) {
  auto *k = static_cast<JitKernel *>(const_cast<void *>(L.entry_data));
  if (!k)
    throw Failure(PR_INTERNAL_ERROR, "Run-time compiled entry without its kernel");
  if (L.args.size() != k->params.size())
    throw Failure(PR_INVALID_ARGUMENT, "Kernel argument count mismatch");
  auto *fn = static_cast<CUfunction>(k->function(L.device));
  int max_threads = 0;
  if (driver().attribute &&
      driver().attribute(&max_threads, CU_FUNC_ATTRIBUTE_MAX_THREADS_PER_BLOCK, fn) == CUDA_SUCCESS &&
      uint64_t(L.block.x) * L.block.y * L.block.z > uint64_t(max_threads))
    throw Failure(PR_INVALID_ARGUMENT, "Block thread count exceeds this kernel's limit of " +
                                           std::to_string(max_threads));
  if (L.dry_run)
    return;
  const size_t count = k->params.size();
  std::vector<uint64_t> values(2 * count + 1);
  std::vector<void *> pointers;
  pointers.reserve(2 * count + 1);
  for (size_t i = 0; i < count; ++i) {
    if (k->params[i].buffer)
      values[i] = reinterpret_cast<uint64_t>(L.args[i].ptr);
    else
      values[i] = L.args[i].bits; // 4-byte scalar in the low bytes (little endian)
    pointers.push_back(&values[i]);
  }
  size_t extra = count;
  for (size_t i = 0; i < count; ++i)
    if (k->params[i].buffer) {
      values[extra] = L.args[i].bytes / 4;
      pointers.push_back(&values[extra++]);
    }
  values[extra] = reinterpret_cast<uint64_t>(L.status);
  pointers.push_back(&values[extra]);
  const CUresult r = driver().launch(fn, L.grid.x, L.grid.y, L.grid.z, L.block.x, L.block.y, L.block.z, 0,
                                     reinterpret_cast<CUstream>(L.stream), pointers.data(), nullptr);
  if (r != CUDA_SUCCESS)
    throw Failure(PR_INVALID_ARGUMENT, "cuLaunchKernel failed for " + k->name + " (CUresult " +
                                           std::to_string(int(r)) + ")");
  L.kernels = 1;
  L.variant = "nvrtc_sm_100a";
}
} // namespace

const Builtin &jit_builtin() {
  static const Builtin entry{"ir.nvrtc", {0, 0, 0}, {}, launch_jit};
  return entry;
}

} // namespace pb
