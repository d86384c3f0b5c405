// The tensor-operator provider (paralyn/tensor.h) and the two additive B200
// operators built on it (paralyn/b200.h: the fused GEMM epilogue and the gathered
// LayerNorm).
//
// Every operator entry point is an ordinary client of the public C ABI: it checks
// its record and tensor operands, then submits one entry of the provider module on
// the caller's queue with exact-extent buffer ranges (launch_entry), whose sm_100a
// launchers live in paralyn_b200/csrc/kernels. The checks are data-driven. Each
// operator has a Rules table: its operation name, its record's name, its operands
// (label, rank, layout rule, input or output, optional) as pointers into the record,
// and hooks for what is particular to it (record scalars, shape relations, the entry
// to run, when there is no work, the launch arguments). One runner walks every
// operator through the same sequence:
//    1. the event output (set to 0 first)      7. each output against each input:
//    2. the record header (size, version)          overlapping bytes INVALID_ARGUMENT,
//    3. the record's scalar fields                 same allocation UNSUPPORTED
//    4. presence of the required operands       8. ownership: queue, provider module
//    5. each operand's descriptor and layout       and every operand's buffer in one
//    6. shape relations and size limits            context
//                                                9. the provider entry's schema
//                                               10. no output elements: no command
//                                               11. the launch
// The statuses and this order are the reference's contract (runtime/tensor.cpp:
// 448-1038); tests/test_gpu_provider_validation.py and tests/test_abi.py pin them.
#include "abi_internal.hpp"
#include "../kernels/prepared.hpp"
#include "paralyn/b200.h"
#include <algorithm>
#include <cmath>
#include <cstring>
#include <functional>
#include <limits>
#include <mutex>
#include <string>
#include <unordered_set>
#include <vector>

namespace pb {
namespace {

constexpr uint64_t kMaxElements = uint64_t(std::numeric_limits<int32_t>::max());
constexpr uint32_t kTile = 16;   // the matmul entries' 16 x 16 launch tiles
constexpr uint32_t kLanes = 256; // one 256-lane group per row (row operators)
constexpr uint64_t kMaxRows = std::numeric_limits<uint32_t>::max() / kLanes;
constexpr uint64_t kMaxLayerNormColumns = uint64_t(1) << 24;
static_assert(kMaxRows == PR_TENSOR_ROW_OPERATOR_MAX_ROWS, "row operator limit");

[[noreturn]] void reject(pr_status status, const std::string &why) { fail(status, why); }

bool mul_ok(uint64_t a, uint64_t b, uint64_t &product) { return !__builtin_mul_overflow(a, b, &product); }

// A failed inner ABI call becomes this operator's failure, with the inner message.
void forward(pr_status status) {
  if (status == PR_SUCCESS)
    return;
  pr_error inner{};
  pr_last_error(&inner);
  reject(status, std::string(inner.operation) + ": " + inner.message);
}

// Runs an entry point's body with the ABI's error boundary.
template <class Body> pr_status guarded(const char *operation, Body &&body) noexcept {
  try {
    body();
    clear_error();
    return PR_SUCCESS;
  } catch (const Failure &f) {
    return report_error(f.status, operation, f.what());
  } catch (const Error &e) {
    return report_error(status_of(e.code), operation, e.what());
  } catch (const std::bad_alloc &) {
    return report_error(PR_OUT_OF_MEMORY, operation, "out of host memory");
  } catch (const std::exception &e) {
    return report_error(PR_INTERNAL_ERROR, operation, e.what());
  } catch (...) {
    return report_error(PR_INTERNAL_ERROR, operation, "unexpected failure");
  }
}

std::string dims_text(const uint64_t *dims, uint32_t rank) {
  std::string text = "[";
  for (uint32_t i = 0; i < rank; ++i)
    text += (i ? "," : "") + std::to_string(dims[i]);
  return text + "]";
}

// ---------------------------------------------------------------- descriptors
// What a descriptor addresses: its element count, the bytes from byte_offset to
// one past its highest element, and whether its strides are dense row-major.
struct Extent {
  uint64_t elements = 0, bytes = 0;
  bool row_major = true;
};

// pr_tensor_desc_validate's rules: the record, FP32, rank <= 8 with zeroed unused
// dimensions, a 4-byte aligned offset, non-negative strides, at most INT32_MAX
// elements, no 64-bit overflow, and the addressed bytes inside the buffer.
Extent inspect(const pr_tensor_desc_v1 *d, const std::string &who) {
  if (!d)
    reject(PR_INVALID_ARGUMENT, "Missing tensor descriptor");
  if (d->version != PR_TENSOR_VERSION_1)
    reject(PR_UNSUPPORTED, "Unsupported tensor descriptor version");
  if (d->struct_size != sizeof(pr_tensor_desc_v1))
    reject(PR_INVALID_ARGUMENT, "Tensor descriptor size mismatch");
  if (d->dtype != PR_F32)
    reject(PR_UNSUPPORTED, who + ": the element type must be PR_F32");
  if (d->rank > PR_TENSOR_MAX_RANK)
    reject(PR_INVALID_ARGUMENT, who + ": rank is above PR_TENSOR_MAX_RANK");
  if (d->byte_offset % 4 != 0)
    reject(PR_INVALID_ARGUMENT, who + ": byte_offset is not a multiple of 4");
  for (uint32_t axis = d->rank; axis < PR_TENSOR_MAX_RANK; ++axis)
    if (d->shape[axis] != 0 || d->strides[axis] != 0)
      reject(PR_INVALID_ARGUMENT, who + ": shape and strides beyond the rank must be zero");
  Extent e;
  e.elements = 1;
  for (uint32_t axis = 0; axis < d->rank; ++axis) {
    if (d->strides[axis] < 0)
      reject(PR_UNSUPPORTED, who + ": negative strides are not supported");
    if (!mul_ok(e.elements, d->shape[axis], e.elements))
      reject(PR_OUT_OF_BOUNDS, who + ": the element count overflows");
  }
  if (e.elements > kMaxElements)
    reject(PR_UNSUPPORTED, who + ": more than INT32_MAX elements");
  // Innermost axis first: the dense stride each axis would have, and the highest
  // element offset the strides reach.
  uint64_t dense = 1, highest = 0;
  for (uint32_t axis = d->rank; axis-- > 0;) {
    const uint64_t extent = d->shape[axis], stride = uint64_t(d->strides[axis]);
    e.row_major = e.row_major && (extent == 1 || stride == dense);
    dense *= extent;
    if (e.elements == 0)
      continue;
    uint64_t step = 0;
    if (!mul_ok(extent - 1, stride, step) || step > std::numeric_limits<uint64_t>::max() - highest)
      reject(PR_OUT_OF_BOUNDS, who + ": the strided extent overflows");
    highest += step;
  }
  if (e.elements == 0) {
    e.row_major = true; // an empty tensor addresses nothing
  } else {
    if (highest >= std::numeric_limits<uint64_t>::max() / 4)
      reject(PR_OUT_OF_BOUNDS, who + ": the byte extent overflows");
    e.bytes = (highest + 1) * 4;
  }
  uint64_t capacity = 0;
  forward(pr_buffer_size(d->buffer, &capacity));
  if (d->byte_offset > capacity || e.bytes > capacity - d->byte_offset)
    reject(PR_OUT_OF_BOUNDS, who + ": the tensor reaches past the end of its buffer");
  return e;
}

// A written layout must give every element its own address. Sufficient test: with
// the axes of extent > 1 in increasing stride order, each stride is larger than the
// highest offset the smaller axes reach (layouts it cannot prove are refused).
void require_injective(const pr_tensor_desc_v1 *d, const char *who) {
  std::vector<std::pair<uint64_t, uint64_t>> axes; // (stride, extent)
  for (uint32_t axis = 0; axis < d->rank; ++axis) {
    if (d->shape[axis] == 0)
      return; // writes nothing
    if (d->shape[axis] > 1)
      axes.emplace_back(uint64_t(d->strides[axis]), d->shape[axis]);
  }
  std::sort(axes.begin(), axes.end());
  uint64_t covered = 0;
  for (const auto &[stride, extent] : axes) {
    if (stride <= covered)
      reject(PR_INVALID_ARGUMENT, std::string(who) + ": the output layout writes some elements twice");
    covered += (extent - 1) * stride;
  }
}

// ---------------------------------------------------------------- operands
enum class Layout : uint8_t {
  row_major, // dense row-major (every operator but batched matmul)
  strided,   // any validated non-negative strides within 32-bit element indexing
};

struct OperandSpec {
  const char *label;
  int rank;            // required rank; kSameRank: the rank of operand 0
  Layout layout = Layout::row_major;
  bool output = false; // written by the operator
  bool optional = false;
};
constexpr int kSameRank = -1;

struct Operand {
  const pr_tensor_desc_v1 *desc = nullptr;
  Extent extent;
  const char *label = "";
  bool output = false;
  uint64_t dim(uint32_t axis) const { return desc->shape[axis]; }
};

Extent operand_extent(const pr_tensor_desc_v1 *d, const OperandSpec &spec, uint32_t rank) {
  const Extent e = inspect(d, spec.label);
  if (d->rank != rank)
    reject(PR_INVALID_ARGUMENT, std::string(spec.label) + ": expected rank " + std::to_string(rank));
  if (spec.layout == Layout::row_major && !e.row_major)
    reject(PR_UNSUPPORTED, std::string(spec.label) + ": v1 operators need a contiguous row-major layout");
  if (spec.layout == Layout::strided && e.bytes / 4 > kMaxElements)
    reject(PR_UNSUPPORTED, std::string(spec.label) + ": the strided extent exceeds INT32_MAX elements");
  return e;
}

void expect_shape(const Operand &o, std::initializer_list<uint64_t> dims, const char *what) {
  bool same = o.desc->rank == dims.size();
  uint32_t axis = 0;
  for (uint64_t d : dims)
    same = same && o.desc->shape[axis++] == d;
  if (!same) {
    std::vector<uint64_t> want(dims);
    reject(PR_INVALID_ARGUMENT, std::string(what) + " shape " + dims_text(o.desc->shape, o.desc->rank) +
                                    " does not match expected " + dims_text(want.data(), uint32_t(want.size())));
  }
}

void within_row_limit(uint64_t rows, const char *what) {
  if (rows > kMaxRows)
    reject(PR_UNSUPPORTED, std::string(what) + " handles at most " + std::to_string(kMaxRows) +
                               " rows; got " + std::to_string(rows));
}

// Buffer handles map one-to-one to allocations, so comparing handles compares
// allocations.
void separate(const Operand &out, const Operand &in) {
  if (!in.desc || out.desc->buffer != in.desc->buffer)
    return;
  const uint64_t o0 = out.desc->byte_offset, i0 = in.desc->byte_offset;
  if (out.extent.bytes && in.extent.bytes && o0 < i0 + in.extent.bytes && i0 < o0 + out.extent.bytes)
    reject(PR_INVALID_ARGUMENT, std::string("Output overlaps input ") + in.label +
                                    "; tensor operators do not run in place");
  reject(PR_UNSUPPORTED, std::string("Output shares an allocation with input ") + in.label +
                             "; outputs need an allocation of their own");
}

// ---------------------------------------------------------------- provider identity and ownership
std::mutex provider_mutex;
std::unordered_set<pr_module> &provider_modules() {
  static std::unordered_set<pr_module> modules;
  return modules;
}

const void *context_of(pr_handle handle, HandleKind kind, const char *who) {
  const void *context = nullptr;
  const pr_status status = handle_context(handle, kind, &context);
  if (status != PR_SUCCESS) {
    pr_error inner{};
    pr_last_error(&inner);
    reject(status, std::string(who) + ": " + inner.message);
  }
  return context;
}

// The queue, the provider module and every operand's buffer belong to one context,
// and the module is one that pr_tensor_operators_load returned (module handles are
// never reused, so membership cannot pass to another module).
void one_context(pr_queue queue, pr_module operators, const std::vector<Operand> &operands) {
  const void *context = context_of(queue, HandleKind::queue, "queue");
  if (context_of(operators, HandleKind::module, "operators") != context)
    reject(PR_CONTEXT_MISMATCH, "Queue and operator module belong to different contexts");
  {
    std::lock_guard<std::mutex> lock(provider_mutex);
    if (!provider_modules().count(operators))
      reject(PR_INVALID_ARGUMENT, "Module is not the tensor operator provider (load it with pr_tensor_operators_load)");
  }
  for (const Operand &o : operands)
    if (o.desc && context_of(o.desc->buffer, HandleKind::buffer, o.label) != context)
      reject(PR_CONTEXT_MISMATCH, std::string(o.label) + ": the tensor's buffer belongs to another context");
}

// The entry `name` of the provider module has the parameter schema of this
// library's built-in entry; checked once per (module, entry).
std::mutex entry_mutex;
std::vector<std::pair<pr_module, std::string>> &checked_entries() {
  static std::vector<std::pair<pr_module, std::string>> entries;
  return entries;
}
void verify_entry(pr_module operators, const char *name) {
  {
    std::lock_guard<std::mutex> lock(entry_mutex);
    for (const auto &[module, entry] : checked_entries())
      if (module == operators && entry == name)
        return;
  }
  struct KernelHandle {
    pr_kernel handle = 0;
    ~KernelHandle() {
      if (handle)
        pr_release(handle);
    }
  } kernel;
  forward(pr_module_kernel(operators, name, &kernel.handle));
  const Builtin *builtin = find_builtin(name);
  uint32_t count = 0;
  forward(pr_kernel_parameter_count(kernel.handle, &count));
  bool matches = builtin && count == builtin->params.size();
  for (uint32_t i = 0; matches && i < count; ++i) {
    pr_parameter_info info{};
    forward(pr_kernel_parameter(kernel.handle, i, &info));
    const Param &want = builtin->params[i];
    matches = want.name == info.name && info.is_buffer == uint32_t(want.buffer) &&
              info.type == (want.type == Scalar::F32 ? PR_F32 : PR_U32);
  }
  if (!matches)
    reject(PR_INVALID_ARGUMENT, "Module is not the tensor operator provider (load it with pr_tensor_operators_load)");
  std::lock_guard<std::mutex> lock(entry_mutex);
  if (checked_entries().size() >= 1024) // entries of released modules pile up: start over
    checked_entries().clear();
  checked_entries().emplace_back(operators, name);
}

// ---------------------------------------------------------------- submission
// The arguments of one provider entry, in parameter order: operands bound as
// exact byte ranges (read-only inputs, read-write outputs) and scalars.
class EntryArguments {
public:
  EntryArguments &tensor(const Operand &o) {
    RangeArgument a;
    a.arg.type = PR_BUFFER;
    a.buffer = o.desc->buffer;
    a.offset = o.desc->byte_offset;
    a.bytes = o.extent.bytes;
    a.access = o.output ? PR_READ_WRITE : PR_READ;
    args_.push_back(a);
    return *this;
  }
  EntryArguments &u32(uint64_t value) {
    RangeArgument a;
    a.arg.type = PR_U32;
    a.arg.u32 = uint32_t(value);
    args_.push_back(a);
    return *this;
  }
  EntryArguments &f32(float value) {
    RangeArgument a;
    a.arg.type = PR_F32;
    a.arg.f32 = value;
    args_.push_back(a);
    return *this;
  }
  const RangeArgument *data() const { return args_.data(); }
  uint32_t size() const { return uint32_t(args_.size()); }

private:
  std::vector<RangeArgument> args_;
};

pr_dim3 groups_of(uint64_t count) { return {uint32_t((count + kLanes - 1) / kLanes), 1, 1}; }
pr_dim3 tiles_of(uint64_t rows, uint64_t columns, uint64_t depth = 1) {
  return {uint32_t((columns + kTile - 1) / kTile), uint32_t((rows + kTile - 1) / kTile), uint32_t(depth)};
}

struct Submission {
  pr_queue queue;
  pr_module operators;
  const char *entry;
  pr_event *event;
  void operator()(pr_dim3 grid, pr_dim3 block, const EntryArguments &args) const {
    forward(launch_entry(queue, operators, entry, grid, block, args.data(), args.size(), event));
  }
};

// ---------------------------------------------------------------- the operator runner
template <class Record> struct Rules {
  const char *operation = nullptr;     // pr_last_error operation
  const char *record = nullptr;        // "<record> record" in header messages
  const char *missing = nullptr;       // message when a required operand is absent
  std::vector<OperandSpec> operands;
  std::vector<const pr_tensor_desc_v1 *const Record::*> fields; // operand i's descriptor in the record
  std::function<void(const Record &)> scalars;                  // step 3
  std::function<void(const Record &, const std::vector<Operand> &)> before_operands; // after presence
  std::function<void(const Record &, const std::vector<Operand> &)> shapes;          // step 6
  std::function<const char *(const Record &, const std::vector<Operand> &)> entry;  // step 9
  std::function<bool(const Record &, const std::vector<Operand> &)> nothing_to_do;  // step 10
  std::function<void(const Record &, const std::vector<Operand> &, const Submission &)> launch;
};

template <class Record> void check_header(const Record *r, const char *what) {
  const std::string name(what);
  if (!r)
    reject(PR_INVALID_ARGUMENT, "Missing " + name + " record");
  if (r->version != PR_TENSOR_VERSION_1)
    reject(PR_UNSUPPORTED, "Unsupported " + name + " record version");
  if (r->struct_size != sizeof(Record))
    reject(PR_INVALID_ARGUMENT, name + " record size mismatch");
}

// Steps 4-8 for operands already taken from a record (shared with the gathered
// LayerNorm, whose extra operands come from outside its record).
template <class Record>
void check_operands(const Rules<Record> &rules, const Record &r, std::vector<Operand> &operands, pr_queue queue,
                    pr_module module) {
  for (size_t i = 0; i < operands.size(); ++i)
    if (!operands[i].desc && !rules.operands[i].optional)
      reject(PR_INVALID_ARGUMENT, rules.missing);
  if (rules.before_operands)
    rules.before_operands(r, operands);
  for (size_t i = 0; i < operands.size(); ++i) {
    if (!operands[i].desc)
      continue;
    const OperandSpec &spec = rules.operands[i];
    const uint32_t rank = spec.rank == kSameRank ? operands[0].desc->rank : uint32_t(spec.rank);
    operands[i].extent = operand_extent(operands[i].desc, spec, rank);
  }
  if (rules.shapes)
    rules.shapes(r, operands);
  for (const Operand &out : operands)
    if (out.output && out.desc)
      for (const Operand &in : operands)
        if (!in.output)
          separate(out, in);
  one_context(queue, module, operands);
}

template <class Record> std::vector<Operand> operands_of(const Rules<Record> &rules, const Record &r) {
  std::vector<Operand> operands(rules.operands.size());
  for (size_t i = 0; i < operands.size(); ++i) {
    operands[i].desc = r.*(rules.fields[i]);
    operands[i].label = rules.operands[i].label;
    operands[i].output = rules.operands[i].output;
  }
  return operands;
}

template <class Record>
pr_status run_operator(const Rules<Record> &rules, pr_queue queue, pr_module module, const Record *record,
                       pr_event *event) {
  return guarded(rules.operation, [&] {
    if (!event)
      reject(PR_INVALID_ARGUMENT, "Missing event output");
    *event = 0;
    check_header(record, rules.record);
    if (rules.scalars)
      rules.scalars(*record);
    std::vector<Operand> operands = operands_of(rules, *record);
    check_operands(rules, *record, operands, queue, module);
    const char *entry = rules.entry(*record, operands);
    verify_entry(module, entry);
    if (rules.nothing_to_do(*record, operands))
      return; // no output elements: no command and no invented event
    rules.launch(*record, operands, Submission{queue, module, entry, event});
  });
}

void bounded_dims(std::initializer_list<uint64_t> dims, const char *what) {
  for (uint64_t d : dims)
    if (d > kMaxElements)
      reject(PR_UNSUPPORTED, std::string(what) + " dimensions must not exceed INT32_MAX");
}

bool known_activation(uint32_t a) {
  return a == PR_ACTIVATION_NONE || a == PR_ACTIVATION_RELU || a == PR_ACTIVATION_GELU_TANH;
}

// ---------------------------------------------------------------- the operators
const Rules<pr_matmul_v1> &matmul_rules() {
  static const Rules<pr_matmul_v1> rules = [] {
    Rules<pr_matmul_v1> r;
    r.operation = "matmul_f32";
    r.record = "matmul";
    r.missing = "Missing matmul tensor";
    r.operands = {{"A", 2}, {"B", 2}, {"C", 2, Layout::row_major, true}};
    r.fields = {&pr_matmul_v1::a, &pr_matmul_v1::b, &pr_matmul_v1::c};
    r.scalars = [](const pr_matmul_v1 &op) {
      if (op.transpose_a > 1 || op.transpose_b > 1)
        reject(PR_INVALID_ARGUMENT, "Transpose flags must be 0 or 1");
    };
    r.shapes = [](const pr_matmul_v1 &op, const std::vector<Operand> &o) {
      bounded_dims({op.m, op.n, op.k}, "Matmul");
      if (op.transpose_a)
        expect_shape(o[0], {op.k, op.m}, "A (stored transposed as [k,m])");
      else
        expect_shape(o[0], {op.m, op.k}, "A [m,k]");
      if (op.transpose_b)
        expect_shape(o[1], {op.n, op.k}, "B (stored transposed as [n,k])");
      else
        expect_shape(o[1], {op.k, op.n}, "B [k,n]");
      expect_shape(o[2], {op.m, op.n}, "C [m,n]");
    };
    r.entry = [](const pr_matmul_v1 &op, const std::vector<Operand> &) {
      return op.k ? "paralyn_matmul_f32" : "paralyn_fill_f32"; // k = 0: the empty sum, +0.0
    };
    r.nothing_to_do = [](const pr_matmul_v1 &op, const std::vector<Operand> &) { return !op.m || !op.n; };
    r.launch = [](const pr_matmul_v1 &op, const std::vector<Operand> &o, const Submission &submit) {
      EntryArguments args;
      if (!op.k) {
        args.tensor(o[2]).u32(op.m * op.n).f32(0.0f);
        submit(groups_of(op.m * op.n), {kLanes, 1, 1}, args);
        return;
      }
      args.tensor(o[0]).tensor(o[1]).tensor(o[2]).u32(op.m).u32(op.n).u32(op.k).u32(op.transpose_a)
          .u32(op.transpose_b);
      submit(tiles_of(op.m, op.n), {kTile, kTile, 1}, args);
    };
    return r;
  }();
  return rules;
}

const Rules<pr_bias_activation_v1> &bias_activation_rules() {
  static const Rules<pr_bias_activation_v1> rules = [] {
    Rules<pr_bias_activation_v1> r;
    r.operation = "bias_activation_f32";
    r.record = "bias/activation";
    r.missing = "Missing input or output tensor";
    r.operands = {{"x", 2}, {"bias", 1, Layout::row_major, false, true}, {"out", 2, Layout::row_major, true}};
    r.fields = {&pr_bias_activation_v1::x, &pr_bias_activation_v1::bias, &pr_bias_activation_v1::out};
    r.scalars = [](const pr_bias_activation_v1 &op) {
      if (!known_activation(op.activation))
        reject(PR_INVALID_ARGUMENT, "Unknown activation");
      if (op.reserved != 0)
        reject(PR_INVALID_ARGUMENT, "Reserved field must be zero");
    };
    r.shapes = [](const pr_bias_activation_v1 &, const std::vector<Operand> &o) {
      expect_shape(o[2], {o[0].dim(0), o[0].dim(1)}, "out");
      if (o[1].desc)
        expect_shape(o[1], {o[0].dim(1)}, "bias");
    };
    r.entry = [](const pr_bias_activation_v1 &op, const std::vector<Operand> &) {
      return op.bias ? "paralyn_bias_activation_f32" : "paralyn_activation_f32";
    };
    r.nothing_to_do = [](const pr_bias_activation_v1 &, const std::vector<Operand> &o) {
      return o[0].extent.elements == 0;
    };
    r.launch = [](const pr_bias_activation_v1 &op, const std::vector<Operand> &o, const Submission &submit) {
      const uint64_t count = o[0].extent.elements;
      EntryArguments args;
      if (op.bias)
        args.tensor(o[0]).tensor(o[1]).tensor(o[2]).u32(count).u32(o[0].dim(1)).u32(op.activation);
      else
        args.tensor(o[0]).tensor(o[2]).u32(count).u32(op.activation);
      submit(groups_of(count), {kLanes, 1, 1}, args);
    };
    return r;
  }();
  return rules;
}

// Transformer-block operators (reference runtime/tensor.cpp:847-970).
const Rules<pr_batched_matmul_v1> &batched_matmul_rules() {
  static const Rules<pr_batched_matmul_v1> rules = [] {
    Rules<pr_batched_matmul_v1> r;
    r.operation = "batched_matmul_f32";
    r.record = "batched matmul";
    r.missing = "Missing batched matmul tensor";
    r.operands = {{"A", 3, Layout::strided}, {"B", 3, Layout::strided}, {"C", 3, Layout::strided, true}};
    r.fields = {&pr_batched_matmul_v1::a, &pr_batched_matmul_v1::b, &pr_batched_matmul_v1::c};
    r.shapes = [](const pr_batched_matmul_v1 &op, const std::vector<Operand> &o) {
      bounded_dims({op.batch, op.m, op.n, op.k}, "Batched matmul");
      expect_shape(o[0], {op.batch, op.m, op.k}, "A [batch,m,k]");
      expect_shape(o[1], {op.batch, op.k, op.n}, "B [batch,k,n]");
      expect_shape(o[2], {op.batch, op.m, op.n}, "C [batch,m,n]");
      require_injective(o[2].desc, "C");
    };
    r.entry = [](const pr_batched_matmul_v1 &op, const std::vector<Operand> &) {
      return op.k ? "paralyn_batched_matmul_f32" : "paralyn_batched_fill_f32";
    };
    r.nothing_to_do = [](const pr_batched_matmul_v1 &op, const std::vector<Operand> &) {
      return !op.batch || !op.m || !op.n;
    };
    r.launch = [](const pr_batched_matmul_v1 &op, const std::vector<Operand> &o, const Submission &submit) {
      const pr_tensor_desc_v1 &c = *o[2].desc;
      EntryArguments args;
      if (!op.k) { // the empty sum: +0.0 at every addressed element of C
        args.tensor(o[2]).u32(op.m).u32(op.n).u32(c.strides[0]).u32(c.strides[1]).u32(c.strides[2]).f32(0.0f);
      } else {
        args.tensor(o[0]).tensor(o[1]).tensor(o[2]).u32(op.m).u32(op.n).u32(op.k);
        for (const Operand &x : o)
          for (uint32_t axis = 0; axis < 3; ++axis)
            args.u32(uint64_t(x.desc->strides[axis]));
      }
      submit(tiles_of(op.m, op.n, op.batch), {kTile, kTile, 1}, args);
    };
    return r;
  }();
  return rules;
}

const Rules<pr_reduce_rows_v1> &reduce_rows_rules() {
  static const Rules<pr_reduce_rows_v1> rules = [] {
    Rules<pr_reduce_rows_v1> r;
    r.operation = "reduce_rows_f32";
    r.record = "row reduction";
    r.missing = "Missing input or output tensor";
    r.operands = {{"x", 2}, {"out", 1, Layout::row_major, true}};
    r.fields = {&pr_reduce_rows_v1::x, &pr_reduce_rows_v1::out};
    r.scalars = [](const pr_reduce_rows_v1 &op) {
      if (op.op != PR_REDUCE_SUM && op.op != PR_REDUCE_MAX)
        reject(PR_INVALID_ARGUMENT, "Unknown reduction");
      if (op.reserved != 0)
        reject(PR_INVALID_ARGUMENT, "Reserved field must be zero");
    };
    r.shapes = [](const pr_reduce_rows_v1 &, const std::vector<Operand> &o) {
      expect_shape(o[1], {o[0].dim(0)}, "out [rows]");
      within_row_limit(o[0].dim(0), "row reduction");
    };
    r.entry = [](const pr_reduce_rows_v1 &, const std::vector<Operand> &o) {
      return o[0].dim(1) ? "paralyn_reduce_rows_f32" : "paralyn_fill_f32";
    };
    r.nothing_to_do = [](const pr_reduce_rows_v1 &, const std::vector<Operand> &o) { return o[0].dim(0) == 0; };
    r.launch = [](const pr_reduce_rows_v1 &op, const std::vector<Operand> &o, const Submission &submit) {
      const uint64_t rows = o[0].dim(0), columns = o[0].dim(1);
      EntryArguments args;
      if (!columns) { // empty rows: the sum's and the maximum's identities
        args.tensor(o[1]).u32(rows).f32(op.op == PR_REDUCE_MAX ? -std::numeric_limits<float>::infinity() : 0.0f);
        submit(groups_of(rows), {kLanes, 1, 1}, args);
        return;
      }
      args.tensor(o[0]).tensor(o[1]).u32(columns).u32(op.op);
      submit({uint32_t(rows), 1, 1}, {kLanes, 1, 1}, args);
    };
    return r;
  }();
  return rules;
}

const Rules<pr_softmax_rows_v1> &softmax_rules() {
  static const Rules<pr_softmax_rows_v1> rules = [] {
    Rules<pr_softmax_rows_v1> r;
    r.operation = "softmax_rows_f32";
    r.record = "softmax";
    r.missing = "Missing input or output tensor";
    r.operands = {{"x", kSameRank}, {"out", kSameRank, Layout::row_major, true}};
    r.fields = {&pr_softmax_rows_v1::x, &pr_softmax_rows_v1::out};
    r.scalars = [](const pr_softmax_rows_v1 &op) {
      if (op.causal > 1)
        reject(PR_INVALID_ARGUMENT, "causal must be 0 or 1");
      if (!std::isfinite(op.scale) || !(op.scale > 0.0f))
        reject(PR_INVALID_ARGUMENT, "scale must be finite and greater than zero");
    };
    r.before_operands = [](const pr_softmax_rows_v1 &, const std::vector<Operand> &o) {
      if (o[0].desc->rank != 2 && o[0].desc->rank != 3)
        reject(PR_INVALID_ARGUMENT, "x: softmax input must have rank 2 [rows,columns] or rank 3 [batch,rows,columns]");
    };
    r.shapes = [](const pr_softmax_rows_v1 &op, const std::vector<Operand> &o) {
      const uint32_t rank = o[0].desc->rank;
      if (!std::equal(o[0].desc->shape, o[0].desc->shape + rank, o[1].desc->shape))
        reject(PR_INVALID_ARGUMENT, "out shape " + dims_text(o[1].desc->shape, rank) + " does not match x shape " +
                                        dims_text(o[0].desc->shape, rank));
      const uint64_t columns = o[0].dim(rank - 1), rows = o[0].dim(rank - 2);
      if (op.causal && columns < rows)
        reject(PR_INVALID_ARGUMENT, "causal softmax needs columns >= rows (got " +
                                        dims_text(o[0].desc->shape, rank) + ")");
      uint64_t all_rows = rows; // batch * rows (the count was validated, so this cannot overflow unless 0)
      if (rank == 3 && !mul_ok(all_rows, o[0].dim(0), all_rows))
        all_rows = std::numeric_limits<uint64_t>::max();
      within_row_limit(all_rows, "softmax (batch * rows)");
    };
    r.entry = [](const pr_softmax_rows_v1 &, const std::vector<Operand> &) { return "paralyn_softmax_rows_f32"; };
    r.nothing_to_do = [](const pr_softmax_rows_v1 &, const std::vector<Operand> &o) {
      return o[0].extent.elements == 0;
    };
    r.launch = [](const pr_softmax_rows_v1 &op, const std::vector<Operand> &o, const Submission &submit) {
      const uint32_t rank = o[0].desc->rank;
      const uint64_t columns = o[0].dim(rank - 1), rows = o[0].dim(rank - 2);
      EntryArguments args;
      args.tensor(o[0]).tensor(o[1]).u32(columns).u32(rows).u32(op.causal).f32(op.scale);
      submit({uint32_t(o[0].extent.elements / columns), 1, 1}, {kLanes, 1, 1}, args);
    };
    return r;
  }();
  return rules;
}

const Rules<pr_layer_norm_v1> &layer_norm_rules() {
  static const Rules<pr_layer_norm_v1> rules = [] {
    Rules<pr_layer_norm_v1> r;
    r.operation = "layer_norm_f32";
    r.record = "layer norm";
    r.missing = "Missing layer norm tensor (x, gamma, beta and out are required)";
    r.operands = {{"x", 2}, {"gamma", 1}, {"beta", 1}, {"out", 2, Layout::row_major, true}};
    r.fields = {&pr_layer_norm_v1::x, &pr_layer_norm_v1::gamma, &pr_layer_norm_v1::beta, &pr_layer_norm_v1::out};
    r.scalars = [](const pr_layer_norm_v1 &op) {
      if (!std::isfinite(op.epsilon) || !(op.epsilon > 0.0f))
        reject(PR_INVALID_ARGUMENT, "epsilon must be finite and greater than zero");
      if (op.reserved != 0)
        reject(PR_INVALID_ARGUMENT, "Reserved field must be zero");
    };
    r.shapes = [](const pr_layer_norm_v1 &, const std::vector<Operand> &o) {
      const uint64_t rows = o[0].dim(0), columns = o[0].dim(1);
      expect_shape(o[3], {rows, columns}, "out");
      expect_shape(o[1], {columns}, "gamma");
      expect_shape(o[2], {columns}, "beta");
      if (columns > kMaxLayerNormColumns)
        reject(PR_UNSUPPORTED, "layer norm handles at most 2^24 columns (the column count must be exact in FP32)");
      within_row_limit(rows, "layer norm");
    };
    r.entry = [](const pr_layer_norm_v1 &, const std::vector<Operand> &) { return "paralyn_layer_norm_f32"; };
    r.nothing_to_do = [](const pr_layer_norm_v1 &, const std::vector<Operand> &o) {
      return o[0].extent.elements == 0;
    };
    r.launch = [](const pr_layer_norm_v1 &op, const std::vector<Operand> &o, const Submission &submit) {
      EntryArguments args;
      args.tensor(o[0]).tensor(o[1]).tensor(o[2]).tensor(o[3]).u32(o[0].dim(1)).f32(op.epsilon);
      submit({uint32_t(o[0].dim(0)), 1, 1}, {kLanes, 1, 1}, args);
    };
    return r;
  }();
  return rules;
}

const Rules<pr_add_v1> &add_rules() {
  static const Rules<pr_add_v1> rules = [] {
    Rules<pr_add_v1> r;
    r.operation = "add_f32";
    r.record = "add";
    r.missing = "Missing input or output tensor";
    r.operands = {{"x", kSameRank}, {"y", kSameRank}, {"out", kSameRank, Layout::row_major, true}};
    r.fields = {&pr_add_v1::x, &pr_add_v1::y, &pr_add_v1::out};
    r.shapes = [](const pr_add_v1 &, const std::vector<Operand> &o) {
      const uint32_t rank = o[0].desc->rank;
      if (!std::equal(o[0].desc->shape, o[0].desc->shape + rank, o[1].desc->shape) ||
          !std::equal(o[0].desc->shape, o[0].desc->shape + rank, o[2].desc->shape))
        reject(PR_INVALID_ARGUMENT, "add shapes differ: x " + dims_text(o[0].desc->shape, rank) + ", y " +
                                        dims_text(o[1].desc->shape, rank) + ", out " +
                                        dims_text(o[2].desc->shape, rank));
    };
    r.entry = [](const pr_add_v1 &, const std::vector<Operand> &) { return "paralyn_add_f32"; };
    r.nothing_to_do = [](const pr_add_v1 &, const std::vector<Operand> &o) { return o[0].extent.elements == 0; };
    r.launch = [](const pr_add_v1 &, const std::vector<Operand> &o, const Submission &submit) {
      const uint64_t count = o[0].extent.elements;
      EntryArguments args;
      args.tensor(o[0]).tensor(o[1]).tensor(o[2]).u32(count);
      submit(groups_of(count), {kLanes, 1, 1}, args);
    };
    return r;
  }();
  return rules;
}

} // namespace
} // namespace pb

using namespace pb;

// ---------------------------------------------------------------- descriptors and the provider module
PB_EXPORT pr_status pr_tensor_desc_contiguous(pr_buffer buffer, uint64_t byte_offset, pr_type dtype, uint32_t rank,
                                              const uint64_t *dims, pr_tensor_desc_v1 *out) {
  return guarded("tensor_desc_contiguous", [&] {
    if (!out)
      reject(PR_INVALID_ARGUMENT, "Missing tensor descriptor output");
    if (rank > PR_TENSOR_MAX_RANK)
      reject(PR_INVALID_ARGUMENT, "Rank exceeds PR_TENSOR_MAX_RANK");
    if (rank && !dims)
      reject(PR_INVALID_ARGUMENT, "Missing tensor shape");
    pr_tensor_desc_v1 d = {sizeof(pr_tensor_desc_v1), PR_TENSOR_VERSION_1, buffer, byte_offset, dtype, rank, {}, {}};
    uint64_t stride = 1; // dense row-major: innermost axis first
    for (uint32_t axis = rank; axis-- > 0;) {
      if (stride > uint64_t(std::numeric_limits<int64_t>::max()))
        reject(PR_OUT_OF_BOUNDS, "Contiguous stride overflows");
      d.shape[axis] = dims[axis];
      d.strides[axis] = int64_t(stride);
      if (dims[axis] && !mul_ok(stride, dims[axis], stride))
        reject(PR_OUT_OF_BOUNDS, "Contiguous stride overflows");
    }
    *out = d;
  });
}

PB_EXPORT pr_status pr_tensor_desc_validate(const pr_tensor_desc_v1 *desc, uint64_t *required_bytes) {
  return guarded("tensor_desc_validate", [&] {
    const Extent e = inspect(desc, "tensor");
    if (required_bytes)
      *required_bytes = e.bytes;
  });
}

PB_EXPORT pr_status pr_tensor_operators_artifact(void *data, uint64_t capacity, uint64_t *bytes) {
  return guarded("tensor_operators_artifact", [&] {
    if (!bytes)
      reject(PR_INVALID_ARGUMENT, "Missing artifact size output");
    const std::vector<unsigned char> &image = provider_artifact();
    *bytes = image.size();
    if (!data)
      return; // a size query
    if (capacity < image.size())
      reject(PR_OUT_OF_BOUNDS, "Artifact capacity is too small");
    std::memcpy(data, image.data(), image.size());
  });
}

PB_EXPORT pr_status pr_tensor_operators_load(pr_context context, pr_module *out) {
  return guarded("tensor_operators_load", [&] {
    if (!out)
      reject(PR_INVALID_ARGUMENT, "Missing module output");
    *out = 0;
    const std::vector<unsigned char> &image = provider_artifact();
    forward(pr_module_load(context, image.data(), image.size(), out));
    try {
      std::lock_guard<std::mutex> lock(provider_mutex);
      provider_modules().insert(*out);
    } catch (...) {
      pr_release(*out);
      *out = 0;
      throw;
    }
  });
}

PB_EXPORT pr_status pr_tensor_operators_capabilities(pr_tensor_operators_capabilities_v1 *out) {
  return guarded("tensor_operators_capabilities", [&] {
    if (!out)
      reject(PR_INVALID_ARGUMENT, "Missing capability record");
    if (out->version != PR_TENSOR_VERSION_1)
      reject(PR_UNSUPPORTED, "Unsupported tensor capability record version");
    if (out->struct_size != sizeof(*out))
      reject(PR_INVALID_ARGUMENT, "Tensor capability record size mismatch");
    pr_tensor_operators_capabilities_v1 caps{};
    caps.struct_size = sizeof(caps);
    caps.version = PR_TENSOR_VERSION_1;
    for (uint64_t bit : {PR_TENSOR_OP_MATMUL, PR_TENSOR_OP_BIAS_ACTIVATION, PR_TENSOR_OP_BATCHED_MATMUL,
                         PR_TENSOR_OP_REDUCE_ROWS, PR_TENSOR_OP_SOFTMAX_ROWS, PR_TENSOR_OP_LAYER_NORM,
                         PR_TENSOR_OP_ADD})
      caps.operations |= bit;
    for (uint32_t a : {PR_ACTIVATION_NONE, PR_ACTIVATION_RELU, PR_ACTIVATION_GELU_TANH})
      caps.activations |= PR_TENSOR_ACTIVATION_BIT(a);
    for (uint32_t r : {PR_REDUCE_SUM, PR_REDUCE_MAX})
      caps.reductions |= PR_TENSOR_REDUCE_BIT(r);
    caps.max_tensor_elements = kMaxElements;
    caps.max_row_operator_rows = kMaxRows;
    caps.max_layer_norm_columns = kMaxLayerNormColumns;
    *out = caps;
  });
}

// ---------------------------------------------------------------- the reference's operators
PB_EXPORT pr_status pr_matmul_f32(pr_queue queue, pr_module operators, const pr_matmul_v1 *op, pr_event *out) {
  return run_operator(matmul_rules(), queue, operators, op, out);
}

PB_EXPORT pr_status pr_bias_activation_f32(pr_queue queue, pr_module operators, const pr_bias_activation_v1 *op,
                                           pr_event *out) {
  return run_operator(bias_activation_rules(), queue, operators, op, out);
}

PB_EXPORT pr_status pr_batched_matmul_f32(pr_queue queue, pr_module operators, const pr_batched_matmul_v1 *op,
                                          pr_event *out) {
  return run_operator(batched_matmul_rules(), queue, operators, op, out);
}

PB_EXPORT pr_status pr_reduce_rows_f32(pr_queue queue, pr_module operators, const pr_reduce_rows_v1 *op,
                                       pr_event *out) {
  return run_operator(reduce_rows_rules(), queue, operators, op, out);
}

PB_EXPORT pr_status pr_softmax_rows_f32(pr_queue queue, pr_module operators, const pr_softmax_rows_v1 *op,
                                        pr_event *out) {
  return run_operator(softmax_rules(), queue, operators, op, out);
}

PB_EXPORT pr_status pr_layer_norm_f32(pr_queue queue, pr_module operators, const pr_layer_norm_v1 *op,
                                      pr_event *out) {
  return run_operator(layer_norm_rules(), queue, operators, op, out);
}

PB_EXPORT pr_status pr_add_f32(pr_queue queue, pr_module operators, const pr_add_v1 *op, pr_event *out) {
  return run_operator(add_rules(), queue, operators, op, out);
}

// ---------------------------------------------------------------- additive B200 operators
namespace pb {
void launch_layer_norm_gather(Launch &);
void launch_matmul_bias_activation(Launch &);
void launch_gather_rows(Launch &);
void launch_matmul_prepare(Launch &);
void launch_matmul_prepared(Launch &);
void launch_matmul_prepared_bias_activation(Launch &);

namespace {
// Binds operands as raw device ranges of one submitted command (for entries that
// run a launcher directly rather than a provider entry through launch_entry).
struct DirectArguments {
  const QueueAccess &queue;
  std::vector<BoundArg> args;
  std::vector<std::shared_ptr<Allocation>> retained;
  void tensor(const Operand &o, bool writes) {
    BoundArg a;
    a.buffer = true;
    a.writes = writes;
    if (o.desc && o.extent.bytes) {
      auto allocation = buffer_allocation(o.desc->buffer, queue.context);
      a.ptr = static_cast<char *>(allocation->ptr) + o.desc->byte_offset;
      a.bytes = o.extent.bytes;
      retained.push_back(std::move(allocation));
    }
    args.push_back(a);
  }
  void bits(uint32_t value) {
    BoundArg a;
    a.bits = value;
    args.push_back(a);
  }
};
} // namespace
} // namespace pb

// C = activation(op(A) op(B) + bias[column]) as one command: the matmul record
// under pr_matmul_f32's rules (same order and statuses) plus the optional bias [n]
// (an input, checked with the operands) and the activation (checked with the
// record's scalars). Results equal pr_matmul_f32 then pr_bias_activation_f32.
PB_EXPORT pr_status pr_b200_matmul_bias_activation_f32(pr_queue queue, pr_module operators, const pr_matmul_v1 *op,
                                                       const pr_tensor_desc_v1 *bias, uint32_t activation,
                                                       pr_event *out) {
  static const Rules<pr_matmul_v1> rules = [] {
    Rules<pr_matmul_v1> r = matmul_rules();
    r.operation = "matmul_bias_activation_f32";
    r.operands.push_back({"bias", 1, Layout::row_major, false, true});
    return r;
  }();
  return guarded(rules.operation, [&] {
    if (!out)
      reject(PR_INVALID_ARGUMENT, "Missing event output");
    *out = 0;
    check_header(op, rules.record);
    rules.scalars(*op);
    if (!known_activation(activation))
      reject(PR_INVALID_ARGUMENT, "Unknown activation");
    std::vector<Operand> operands(4);
    const pr_tensor_desc_v1 *descs[4] = {op->a, op->b, op->c, bias};
    for (int i = 0; i < 4; ++i)
      operands[i] = Operand{descs[i], {}, rules.operands[i].label, rules.operands[i].output};
    Rules<pr_matmul_v1> with_bias = rules;
    with_bias.shapes = [](const pr_matmul_v1 &m, const std::vector<Operand> &o) {
      matmul_rules().shapes(m, o);
      if (o[3].desc)
        expect_shape(o[3], {m.n}, "bias");
    };
    check_operands(with_bias, *op, operands, queue, operators);
    verify_entry(operators, "paralyn_matmul_f32");
    if (!op->m || !op->n)
      return;
    forward(api("matmul_bias_activation_f32", [&] {
      const QueueAccess q = queue_access(queue);
      DirectArguments d{q, {}, {}};
      d.tensor(operands[0], false);
      d.tensor(operands[1], false);
      d.tensor(operands[2], true);
      for (uint64_t v : {op->m, op->n, op->k, uint64_t(op->transpose_a), uint64_t(op->transpose_b)})
        d.bits(uint32_t(v));
      d.tensor(operands[3], false);
      d.bits(activation);
      d.bits(bias ? 1u : 0u);
      *out = submit_command(queue, "b200_matmul_bias_activation_f32", launch_matmul_bias_activation,
                            Dim3{uint32_t((op->n + kTile - 1) / kTile), uint32_t((op->m + kTile - 1) / kTile), 1},
                            Dim3{kTile, kTile, 1}, std::move(d.args), std::move(d.retained));
    }));
  });
}

// ---- prepared right-hand operands
PB_EXPORT uint64_t pr_b200_matmul_prepared_bytes(uint64_t k, uint64_t n) { return prepared::bytes(k, n); }

namespace pb {
namespace {
// The prepared tensor: rank 1, exactly prepared_bytes(k, n) / 4 elements, starting
// on a 256-byte boundary of its buffer.
void expect_prepared(const Operand &o, uint64_t k, uint64_t n) {
  const uint64_t bytes = prepared::bytes(k, n);
  if (!bytes)
    reject(PR_INVALID_ARGUMENT, "A prepared operand needs 1 <= k, n <= INT32_MAX");
  expect_shape(o, {bytes / 4}, "prepared");
  if (o.desc->byte_offset % prepared::kHeaderBytes)
    reject(PR_INVALID_ARGUMENT, "prepared: the view must start on a 256-byte boundary");
}
} // namespace
} // namespace pb

// B (the right-hand operand of pr_matmul_f32: [k, n], or [n, k] with transpose_b)
// into its prepared form: a command that writes `prepared` (a 1-D FP32 tensor of
// pr_b200_matmul_prepared_bytes(k, n) / 4 elements on a 256-byte boundary, in its
// own allocation). Checks, in order: event output, transpose flag, presence, ranks
// and layouts, the prepared shape, separate allocations, one context and the
// provider module.
PB_EXPORT pr_status pr_b200_matmul_prepare_f32(pr_queue queue, pr_module operators, const pr_tensor_desc_v1 *b,
                                               uint32_t transpose_b, const pr_tensor_desc_v1 *prepared_out,
                                               pr_event *out) {
  return guarded("matmul_prepare_f32", [&] {
    if (!out)
      reject(PR_INVALID_ARGUMENT, "Missing event output");
    *out = 0;
    if (transpose_b > 1)
      reject(PR_INVALID_ARGUMENT, "Transpose flags must be 0 or 1");
    if (!b || !prepared_out)
      reject(PR_INVALID_ARGUMENT, "Missing matmul tensor");
    std::vector<Operand> operands{Operand{b, operand_extent(b, {"B", 2}, 2), "B", false},
                                  Operand{prepared_out, operand_extent(prepared_out, {"prepared", 1}, 1), "prepared",
                                          true}};
    const uint64_t k = transpose_b ? b->shape[1] : b->shape[0], n = transpose_b ? b->shape[0] : b->shape[1];
    bounded_dims({k, n}, "Matmul");
    expect_prepared(operands[1], k, n);
    separate(operands[1], operands[0]);
    one_context(queue, operators, operands);
    verify_entry(operators, "paralyn_matmul_f32");
    forward(api("matmul_prepare_f32", [&] {
      const QueueAccess q = queue_access(queue);
      DirectArguments d{q, {}, {}};
      d.tensor(operands[0], false);
      d.tensor(operands[1], true);
      for (uint64_t v : {k, n, uint64_t(transpose_b)})
        d.bits(uint32_t(v));
      *out = submit_command(queue, "b200_matmul_prepare_f32", launch_matmul_prepare, Dim3{1, 1, 1},
                            Dim3{kLanes, 1, 1}, std::move(d.args), std::move(d.retained));
    }));
  });
}

// C = op(A) B with B's prepared form in op->b: pr_matmul_f32's record and rules,
// except that op->b is the prepared tensor (prepared for op->k and op->n) and
// op->transpose_b must be 0. Results equal pr_matmul_f32 with the B it was prepared
// from, in every matmul mode (bit for bit in the same mode).
PB_EXPORT pr_status pr_b200_matmul_prepared_f32(pr_queue queue, pr_module operators, const pr_matmul_v1 *op,
                                                pr_event *out) {
  static const Rules<pr_matmul_v1> rules = [] {
    Rules<pr_matmul_v1> r = matmul_rules();
    r.operation = "matmul_prepared_f32";
    r.operands[1] = {"prepared", 1};
    r.scalars = [](const pr_matmul_v1 &m) {
      matmul_rules().scalars(m);
      if (m.transpose_b)
        reject(PR_INVALID_ARGUMENT, "A prepared operand is used as prepared: transpose_b must be 0");
    };
    r.shapes = [](const pr_matmul_v1 &m, const std::vector<Operand> &o) {
      bounded_dims({m.m, m.n, m.k}, "Matmul");
      if (m.transpose_a)
        expect_shape(o[0], {m.k, m.m}, "A (stored transposed as [k,m])");
      else
        expect_shape(o[0], {m.m, m.k}, "A [m,k]");
      expect_prepared(o[1], m.k, m.n);
      expect_shape(o[2], {m.m, m.n}, "C [m,n]");
    };
    return r;
  }();
  return guarded(rules.operation, [&] {
    if (!out)
      reject(PR_INVALID_ARGUMENT, "Missing event output");
    *out = 0;
    check_header(op, rules.record);
    rules.scalars(*op);
    std::vector<Operand> operands = operands_of(rules, *op);
    check_operands(rules, *op, operands, queue, operators);
    verify_entry(operators, "paralyn_matmul_f32");
    if (!op->m)
      return;
    forward(api("matmul_prepared_f32", [&] {
      const QueueAccess q = queue_access(queue);
      DirectArguments d{q, {}, {}};
      d.tensor(operands[0], false);
      d.tensor(operands[1], false);
      d.tensor(operands[2], true);
      for (uint64_t v : {op->m, op->n, op->k, uint64_t(op->transpose_a), uint64_t(0)})
        d.bits(uint32_t(v));
      *out = submit_command(queue, "b200_matmul_prepared_f32", launch_matmul_prepared,
                            Dim3{uint32_t((op->n + kTile - 1) / kTile), uint32_t((op->m + kTile - 1) / kTile), 1},
                            Dim3{kTile, kTile, 1}, std::move(d.args), std::move(d.retained));
    }));
  });
}

// C = activation(op(A) B + bias[column]) with B's prepared form in op->b: the
// prepared product's record and rules plus the optional bias [n] (checked with the
// operands) and the activation (checked with the record's scalars), as
// pr_b200_matmul_bias_activation_f32 adds them to pr_matmul_f32's. Results equal
// pr_b200_matmul_bias_activation_f32 with the B the tensor was prepared from.
PB_EXPORT pr_status pr_b200_matmul_prepared_bias_activation_f32(pr_queue queue, pr_module operators,
                                                                const pr_matmul_v1 *op,
                                                                const pr_tensor_desc_v1 *bias, uint32_t activation,
                                                                pr_event *out) {
  static const Rules<pr_matmul_v1> rules = [] {
    Rules<pr_matmul_v1> r = matmul_rules();
    r.operation = "matmul_prepared_bias_activation_f32";
    r.operands[1] = {"prepared", 1};
    r.operands.push_back({"bias", 1, Layout::row_major, false, true});
    r.scalars = [](const pr_matmul_v1 &m) {
      matmul_rules().scalars(m);
      if (m.transpose_b)
        reject(PR_INVALID_ARGUMENT, "A prepared operand is used as prepared: transpose_b must be 0");
    };
    r.shapes = [](const pr_matmul_v1 &m, const std::vector<Operand> &o) {
      bounded_dims({m.m, m.n, m.k}, "Matmul");
      if (m.transpose_a)
        expect_shape(o[0], {m.k, m.m}, "A (stored transposed as [k,m])");
      else
        expect_shape(o[0], {m.m, m.k}, "A [m,k]");
      expect_prepared(o[1], m.k, m.n);
      expect_shape(o[2], {m.m, m.n}, "C [m,n]");
      if (o[3].desc)
        expect_shape(o[3], {m.n}, "bias");
    };
    return r;
  }();
  return guarded(rules.operation, [&] {
    if (!out)
      reject(PR_INVALID_ARGUMENT, "Missing event output");
    *out = 0;
    check_header(op, rules.record);
    rules.scalars(*op);
    if (!known_activation(activation))
      reject(PR_INVALID_ARGUMENT, "Unknown activation");
    std::vector<Operand> operands(4);
    const pr_tensor_desc_v1 *descs[4] = {op->a, op->b, op->c, bias};
    for (int i = 0; i < 4; ++i)
      operands[i] = Operand{descs[i], {}, rules.operands[i].label, rules.operands[i].output};
    check_operands(rules, *op, operands, queue, operators);
    verify_entry(operators, "paralyn_matmul_f32");
    if (!op->m)
      return;
    forward(api("matmul_prepared_bias_activation_f32", [&] {
      const QueueAccess q = queue_access(queue);
      DirectArguments d{q, {}, {}};
      d.tensor(operands[0], false);
      d.tensor(operands[1], false);
      d.tensor(operands[2], true);
      for (uint64_t v : {op->m, op->n, op->k, uint64_t(op->transpose_a), uint64_t(0)})
        d.bits(uint32_t(v));
      d.tensor(operands[3], false);
      d.bits(activation);
      d.bits(bias ? 1u : 0u);
      *out = submit_command(queue, "b200_matmul_prepared_bias_activation_f32",
                            launch_matmul_prepared_bias_activation,
                            Dim3{uint32_t((op->n + kTile - 1) / kTile), uint32_t((op->m + kTile - 1) / kTile), 1},
                            Dim3{kTile, kTile, 1}, std::move(d.args), std::move(d.retained));
    }));
  });
}

// LayerNorm whose output rows are also written into up to eight gathered tensors
// (local or imported from peer processes): pr_layer_norm_f32's rules for the record,
// then each gathered tensor [R_total, columns] must hold rows [row_offset,
// row_offset + rows) (PR_OUT_OF_BOUNDS otherwise) and may not overlap x, gamma, beta,
// another gathered tensor, or out (out may be exactly the gathered rows it mirrors).
PB_EXPORT pr_status pr_b200_layer_norm_gather_f32(pr_queue queue, pr_module operators, const pr_layer_norm_v1 *op,
                                                  const pr_tensor_desc_v1 *const *gathered, uint32_t count,
                                                  uint64_t row_offset, pr_event *out) {
  const Rules<pr_layer_norm_v1> &rules = layer_norm_rules();
  return guarded("layer_norm_gather_f32", [&] {
    if (!out)
      reject(PR_INVALID_ARGUMENT, "Missing event output");
    *out = 0;
    check_header(op, rules.record);
    rules.scalars(*op);
    if (count > PR_B200_MAX_GATHER)
      reject(PR_INVALID_ARGUMENT, "At most 8 gathered tensors");
    if (count && !gathered)
      reject(PR_INVALID_ARGUMENT, "Missing gathered tensors");
    std::vector<Operand> operands = operands_of(rules, *op);
    check_operands(rules, *op, operands, queue, operators);
    const uint64_t rows = operands[0].dim(0), columns = operands[0].dim(1);
    std::vector<Operand> targets(count);
    for (uint32_t i = 0; i < count; ++i) {
      if (!gathered[i])
        reject(PR_INVALID_ARGUMENT, "Missing gathered tensor");
      targets[i] = Operand{gathered[i], operand_extent(gathered[i], {"gathered", 2}, 2), "gathered", true};
      if (gathered[i]->shape[1] != columns)
        reject(PR_INVALID_ARGUMENT, "gathered: column count differs from x");
      if (row_offset > gathered[i]->shape[0] || rows > gathered[i]->shape[0] - row_offset)
        reject(PR_OUT_OF_BOUNDS, "gathered: rows [row_offset, row_offset + rows) exceed the tensor");
      for (int input = 0; input < 3; ++input)
        separate(targets[i], operands[input]);
      // out is either exactly the gathered rows it mirrors, or elsewhere
      const pr_tensor_desc_v1 &o = *operands[3].desc;
      const uint64_t mirror = gathered[i]->byte_offset + 4 * row_offset * columns;
      const bool exact = o.buffer == gathered[i]->buffer && o.byte_offset == mirror;
      if (!exact && o.buffer == gathered[i]->buffer) {
        const uint64_t g0 = gathered[i]->byte_offset, o0 = o.byte_offset;
        if (operands[3].extent.bytes && targets[i].extent.bytes && o0 < g0 + targets[i].extent.bytes &&
            g0 < o0 + operands[3].extent.bytes)
          reject(PR_INVALID_ARGUMENT, "gathered: overlaps out other than at the rows out mirrors");
      }
      for (uint32_t j = 0; j < i; ++j) {
        Operand earlier = targets[j];
        earlier.output = false;
        separate(targets[i], earlier);
      }
    }
    one_context(queue, operators, targets);
    verify_entry(operators, "paralyn_layer_norm_f32");
    if (!operands[0].extent.elements)
      return;
    forward(api("layer_norm_gather_f32", [&] {
      const QueueAccess q = queue_access(queue);
      DirectArguments d{q, {}, {}};
      d.tensor(operands[0], false);
      d.tensor(operands[1], false);
      d.tensor(operands[2], false);
      d.tensor(operands[3], true);
      uint32_t eps_bits;
      std::memcpy(&eps_bits, &op->epsilon, 4);
      for (uint64_t v : {columns, uint64_t(eps_bits), rows, row_offset & 0xffffffffu, row_offset >> 32,
                         uint64_t(count)})
        d.bits(uint32_t(v));
      for (const Operand &t : targets)
        d.tensor(t, true);
      *out = submit_command(queue, "b200_layer_norm_gather_f32", launch_layer_norm_gather, Dim3{uint32_t(rows), 1, 1},
                            Dim3{kLanes, 1, 1}, std::move(d.args), std::move(d.retained));
    }));
  });
}

// A rank's row shard written into every gathered tensor (its own and imported
// peers'): `local` is a contiguous [rows, columns] tensor; each gathered tensor is
// contiguous [R_total, columns] and receives rows [row_offset, row_offset + rows)
// (PR_OUT_OF_BOUNDS past R_total). A gathered tensor may contain `local` exactly at
// those rows (the rank's own rows of its own gathered tensor) but may not otherwise
// overlap it or another gathered tensor. No provider entry is involved: the queue
// and every tensor must belong to one context.
PB_EXPORT pr_status pr_b200_gather_rows_f32(pr_queue queue, const pr_tensor_desc_v1 *local,
                                            const pr_tensor_desc_v1 *const *gathered, uint32_t count,
                                            uint64_t row_offset, pr_event *out) {
  return guarded("gather_rows_f32", [&] {
    if (!out)
      reject(PR_INVALID_ARGUMENT, "Missing event output");
    *out = 0;
    if (!local)
      reject(PR_INVALID_ARGUMENT, "Missing local tensor");
    if (count > PR_B200_MAX_GATHER)
      reject(PR_INVALID_ARGUMENT, "At most 8 gathered tensors");
    if (count && !gathered)
      reject(PR_INVALID_ARGUMENT, "Missing gathered tensors");
    Operand mine{local, operand_extent(local, {"local", 2}, 2), "local", false};
    const uint64_t rows = mine.dim(0), columns = mine.dim(1);
    if (columns > kMaxElements || rows > kMaxElements)
      reject(PR_UNSUPPORTED, "local: dimensions must not exceed INT32_MAX");
    std::vector<Operand> targets(count);
    for (uint32_t i = 0; i < count; ++i) {
      if (!gathered[i])
        reject(PR_INVALID_ARGUMENT, "Missing gathered tensor");
      targets[i] = Operand{gathered[i], operand_extent(gathered[i], {"gathered", 2}, 2), "gathered", true};
      if (gathered[i]->shape[1] != columns)
        reject(PR_INVALID_ARGUMENT, "gathered: column count differs from local");
      if (row_offset > gathered[i]->shape[0] || rows > gathered[i]->shape[0] - row_offset)
        reject(PR_OUT_OF_BOUNDS, "gathered: rows [row_offset, row_offset + rows) exceed the tensor");
      const uint64_t mirror = gathered[i]->byte_offset + 4 * row_offset * columns;
      const bool exact = local->buffer == gathered[i]->buffer && local->byte_offset == mirror;
      if (!exact)
        separate(targets[i], mine);
      for (uint32_t j = 0; j < i; ++j) {
        Operand earlier = targets[j];
        earlier.output = false;
        separate(targets[i], earlier);
      }
    }
    const void *context = context_of(queue, HandleKind::queue, "queue");
    if (context_of(local->buffer, HandleKind::buffer, "local") != context)
      reject(PR_CONTEXT_MISMATCH, "local: the tensor's buffer belongs to another context");
    for (const Operand &t : targets)
      if (context_of(t.desc->buffer, HandleKind::buffer, "gathered") != context)
        reject(PR_CONTEXT_MISMATCH, "gathered: the tensor's buffer belongs to another context");
    if (!mine.extent.elements || !count)
      return;
    forward(api("gather_rows_f32", [&] {
      const QueueAccess q = queue_access(queue);
      DirectArguments d{q, {}, {}};
      d.tensor(mine, false);
      for (uint64_t v : {columns, rows, row_offset & 0xffffffffu, row_offset >> 32, uint64_t(count)})
        d.bits(uint32_t(v));
      for (const Operand &t : targets)
        d.tensor(t, true);
      *out = submit_command(queue, "b200_gather_rows_f32", launch_gather_rows, Dim3{uint32_t(rows), 1, 1},
                            Dim3{kLanes, 1, 1}, std::move(d.args), std::move(d.retained));
    }));
  });
}
