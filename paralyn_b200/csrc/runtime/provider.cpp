// The tensor-operator provider (paralyn/tensor.h).
//
// Like the reference provider (runtime/tensor.cpp:1-7) it is an ordinary client of
// the public C ABI: it validates descriptors, checks handle ownership and the
// provider's entry schema, creates exact-extent views and submits the entry with
// pr_launch on the caller's queue. The validation order and the status of every
// rejection follow runtime/tensor.cpp:448-1038, so callers see the same errors.
// The entries run the sm_100a kernels of paralyn_b200/csrc/kernels.
#include "abi_internal.hpp"
#include <algorithm>
#include <array>
#include <cmath>
#include <cstring>
#include <initializer_list>
#include <limits>
#include <mutex>
#include <unordered_set>
#include <vector>

namespace pb {
namespace {

constexpr uint64_t max_elements = uint64_t(std::numeric_limits<int32_t>::max());
constexpr uint32_t tile = 16, group = 256;
constexpr uint64_t max_rows = std::numeric_limits<uint32_t>::max() / group;
static_assert(max_rows == PR_TENSOR_ROW_OPERATOR_MAX_ROWS, "row limit");
constexpr uint64_t max_layer_norm_columns = uint64_t(1) << 24;

// Captures the inner call's structured error before cleanup can clear it.
void call(pr_status status) {
  if (status == PR_SUCCESS)
    return;
  pr_error inner{};
  pr_last_error(&inner);
  fail(status, std::string(inner.operation) + ": " + inner.message);
}

template <class F> pr_status boundary(const char *operation, F &&fn) noexcept {
  try {
    fn();
    clear_error();
    return PR_SUCCESS;
  } catch (const Failure &f) {
    return report_error(f.status, operation, f.what());
  } catch (const Error &e) {
    return report_error(status_of(e.code), operation, e.what());
  } catch (const std::bad_alloc &) {
    return report_error(PR_OUT_OF_MEMORY, operation, "Allocation failed");
  } catch (const std::exception &e) {
    return report_error(PR_INTERNAL_ERROR, operation, e.what());
  } catch (...) {
    return report_error(PR_INTERNAL_ERROR, operation, "Unknown operator failure");
  }
}

// A kernel entry of the provider module, or a buffer range bound as a kernel
// argument. Neither holds a library handle: launch_entry resolves both under one
// lock, checking each range as pr_view_create would (the launch retains the
// allocations it uses).
struct Owned {
  pr_module module = 0;
  const char *name = nullptr;
  pr_buffer buffer = 0;
  uint64_t offset = 0, bytes = 0;
  pr_access access = PR_READ;
};

struct Layout {
  uint64_t count = 0, bytes = 0;
  bool contiguous = true;
};

bool mul(uint64_t a, uint64_t b, uint64_t &out) {
  if (a && b > std::numeric_limits<uint64_t>::max() / a)
    return false;
  out = a * b;
  return true;
}

Layout validate(const pr_tensor_desc_v1 *d, const char *label) {
  const std::string name(label);
  require(d, PR_INVALID_ARGUMENT, "Missing tensor descriptor");
  require(d->version == PR_TENSOR_VERSION_1, PR_UNSUPPORTED, "Unsupported tensor descriptor version");
  require(d->struct_size == sizeof(pr_tensor_desc_v1), PR_INVALID_ARGUMENT,
          "Tensor descriptor size mismatch");
  if (d->dtype != PR_F32)
    fail(PR_UNSUPPORTED, name + ": only PR_F32 tensors are supported");
  if (d->rank > PR_TENSOR_MAX_RANK)
    fail(PR_INVALID_ARGUMENT, name + ": rank exceeds PR_TENSOR_MAX_RANK");
  if (d->byte_offset % 4)
    fail(PR_INVALID_ARGUMENT, name + ": byte offset must be four-byte aligned");
  Layout layout;
  layout.count = 1;
  for (uint32_t i = d->rank; i < PR_TENSOR_MAX_RANK; ++i)
    if (d->shape[i] || d->strides[i])
      fail(PR_INVALID_ARGUMENT, name + ": unused dimensions must be zero");
  for (uint32_t i = 0; i < d->rank; ++i) {
    if (d->strides[i] < 0)
      fail(PR_UNSUPPORTED, name + ": negative strides are unsupported");
    if (!mul(layout.count, d->shape[i], layout.count))
      fail(PR_OUT_OF_BOUNDS, name + ": element count overflows");
  }
  if (layout.count > max_elements)
    fail(PR_UNSUPPORTED, name + ": tensors support at most INT32_MAX elements");
  uint64_t expected = 1, last = 0;
  for (uint32_t r = d->rank; r-- > 0;) {
    if (d->shape[r] != 1 && uint64_t(d->strides[r]) != expected)
      layout.contiguous = false;
    expected *= d->shape[r];
    uint64_t span = 0;
    if (layout.count && (!mul(d->shape[r] - 1, uint64_t(d->strides[r]), span) ||
                         span > std::numeric_limits<uint64_t>::max() - last))
      fail(PR_OUT_OF_BOUNDS, name + ": stride extent overflows");
    if (layout.count)
      last += span;
  }
  if (!layout.count)
    layout.contiguous = true;
  if (layout.count) {
    if (last >= std::numeric_limits<uint64_t>::max() / 4)
      fail(PR_OUT_OF_BOUNDS, name + ": byte extent overflows");
    layout.bytes = (last + 1) * 4;
  }
  uint64_t size = 0;
  call(pr_buffer_size(d->buffer, &size));
  if (d->byte_offset > size || layout.bytes > size - d->byte_offset)
    fail(PR_OUT_OF_BOUNDS, name + ": tensor extent exceeds its buffer");
  return layout;
}

Layout operand(const pr_tensor_desc_v1 *d, const char *label, uint32_t rank) {
  const Layout layout = validate(d, label);
  if (d->rank != rank)
    fail(PR_INVALID_ARGUMENT, std::string(label) + ": expected rank " + std::to_string(rank));
  if (!layout.contiguous)
    fail(PR_UNSUPPORTED, std::string(label) + ": v1 operators require contiguous row-major layout");
  return layout;
}

// Strided operands (batched matmul only): any validated non-negative layout whose
// extent fits 32-bit element indexing (reference runtime/tensor.cpp:506-515).
Layout strided_operand(const pr_tensor_desc_v1 *d, const char *label, uint32_t rank) {
  const Layout layout = validate(d, label);
  if (d->rank != rank)
    fail(PR_INVALID_ARGUMENT, std::string(label) + ": expected rank " + std::to_string(rank));
  if (layout.bytes / 4 > max_elements)
    fail(PR_UNSUPPORTED, std::string(label) + ": strided extent exceeds INT32_MAX elements");
  return layout;
}

// A written layout must address each element at its own location. Sufficient test
// (reference runtime/tensor.cpp:516-535): with the dimensions of extent > 1 sorted
// by stride, each stride exceeds the largest offset the smaller ones reach.
void injective(const pr_tensor_desc_v1 *d, const char *label) {
  std::vector<std::pair<uint64_t, uint64_t>> dims; // (stride, extent)
  for (uint32_t i = 0; i < d->rank; ++i) {
    if (!d->shape[i])
      return; // an empty tensor writes nothing
    if (d->shape[i] > 1)
      dims.emplace_back(uint64_t(d->strides[i]), d->shape[i]);
  }
  std::sort(dims.begin(), dims.end());
  uint64_t reach = 0;
  for (const auto &dim : dims) {
    if (dim.first <= reach)
      fail(PR_INVALID_ARGUMENT, std::string(label) + ": output layout overlaps itself");
    reach += (dim.second - 1) * dim.first;
  }
}

std::string shape_text(const pr_tensor_desc_v1 *d) {
  std::string s = "[";
  for (uint32_t i = 0; i < d->rank; ++i)
    s += (i ? "," : "") + std::to_string(d->shape[i]);
  return s + "]";
}

void expect_dims(const pr_tensor_desc_v1 *d, const char *label, std::initializer_list<uint64_t> dims) {
  uint32_t i = 0;
  bool same = d->rank == dims.size();
  std::string wanted = "[";
  for (uint64_t v : dims) {
    same = same && d->shape[i] == v;
    wanted += (i++ ? "," : "") + std::to_string(v);
  }
  if (!same)
    fail(PR_INVALID_ARGUMENT,
         std::string(label) + " shape " + shape_text(d) + " does not match expected " + wanted + "]");
}

// Output/input allocation rule; buffer handles map one-to-one to allocations.
void no_alias(const pr_tensor_desc_v1 *out, const Layout &o, const pr_tensor_desc_v1 *in,
              const Layout &i, const char *label) {
  if (!in || out->buffer != in->buffer)
    return;
  const bool overlap = o.bytes && i.bytes && out->byte_offset < in->byte_offset + i.bytes &&
                       in->byte_offset < out->byte_offset + o.bytes;
  if (overlap)
    fail(PR_INVALID_ARGUMENT, std::string("Output overlaps input ") + label +
                                  "; in-place tensor operations are not supported");
  fail(PR_UNSUPPORTED, std::string("Output shares an allocation with input ") + label +
                           "; operators require distinct writable allocations");
}

// Provider identity: exactly the module handles returned by pr_tensor_operators_load.
std::mutex registry_mutex;
std::unordered_set<pr_module> &providers() {
  static std::unordered_set<pr_module> value;
  return value;
}
bool is_provider(pr_module module) {
  std::lock_guard<std::mutex> lock(registry_mutex);
  return providers().count(module) != 0;
}

const void *owner(pr_handle handle, HandleKind kind, const char *label) {
  const void *context = nullptr;
  const pr_status status = handle_context(handle, kind, &context);
  if (status != PR_SUCCESS) {
    pr_error inner{};
    pr_last_error(&inner);
    fail(status, std::string(label) + ": " + inner.message);
  }
  return context;
}

void same_context(pr_queue queue, pr_module operators,
                  std::initializer_list<std::pair<const pr_tensor_desc_v1 *, const char *>> tensors) {
  const void *context = owner(queue, HandleKind::queue, "queue");
  if (owner(operators, HandleKind::module, "operators") != context)
    fail(PR_CONTEXT_MISMATCH, "Queue and operator module belong to different contexts");
  if (!is_provider(operators))
    fail(PR_INVALID_ARGUMENT,
         "Module is not the tensor operator provider (load it with pr_tensor_operators_load)");
  for (const auto &t : tensors)
    if (t.first && owner(t.first->buffer, HandleKind::buffer, t.second) != context)
      fail(PR_CONTEXT_MISMATCH, std::string(t.second) + ": tensor buffer belongs to a different context");
}

// Resolves an entry and checks its schema against the provider table, once per
// (module, entry): module handles are never reused, so a checked pair stays valid
// for as long as the handle is live (launch_entry rejects it once released).
std::mutex schema_mutex;
std::vector<std::pair<pr_module, const char *>> &checked_schemas() {
  static std::vector<std::pair<pr_module, const char *>> value;
  return value;
}
void kernel(pr_module operators, const char *name, Owned &out) {
  out.module = operators;
  out.name = name;
  {
    std::lock_guard<std::mutex> lock(schema_mutex);
    for (const auto &c : checked_schemas())
      if (c.first == operators && !std::strcmp(c.second, name))
        return;
  }
  struct Handle {
    pr_kernel value = 0;
    ~Handle() {
      if (value)
        pr_release(value);
    }
  } fn;
  const Builtin *entry = find_builtin(name);
  call(pr_module_kernel(operators, name, &fn.value));
  uint32_t count = 0;
  call(pr_kernel_parameter_count(fn.value, &count));
  bool same = entry && count == entry->params.size();
  for (uint32_t i = 0; same && i < count; ++i) {
    pr_parameter_info info{};
    call(pr_kernel_parameter(fn.value, i, &info));
    const auto &p = entry->params[i];
    same = !std::strcmp(info.name, p.name.c_str()) && info.is_buffer == uint32_t(p.buffer) &&
           info.type == (p.type == Scalar::F32 ? PR_F32 : PR_U32);
  }
  require(same, PR_INVALID_ARGUMENT,
          "Module is not the tensor operator provider (load it with pr_tensor_operators_load)");
  std::lock_guard<std::mutex> lock(schema_mutex);
  auto &checked = checked_schemas();
  if (checked.size() >= 1024) // handles of released modules accumulate: start over
    checked.clear();
  checked.emplace_back(operators, entry->name);
}

void view(const pr_tensor_desc_v1 *d, const Layout &l, pr_access access, Owned &out) {
  out.buffer = d->buffer;
  out.offset = d->byte_offset;
  out.bytes = l.bytes;
  out.access = access;
}
RangeArgument buffer(const Owned &v) {
  RangeArgument a;
  a.arg.type = PR_BUFFER;
  a.buffer = v.buffer;
  a.offset = v.offset;
  a.bytes = v.bytes;
  a.access = v.access;
  return a;
}
RangeArgument u32(uint64_t value) {
  RangeArgument a;
  a.arg.type = PR_U32;
  a.arg.u32 = uint32_t(value);
  return a;
}
RangeArgument f32(float value) {
  RangeArgument a;
  a.arg.type = PR_F32;
  a.arg.f32 = value;
  return a;
}
pr_dim3 linear(uint64_t count) { return {uint32_t((count + group - 1) / group), 1, 1}; }

template <class Record> void header(const Record *op, const char *name) {
  require(op, PR_INVALID_ARGUMENT, (std::string("Missing ") + name + " record").c_str());
  require(op->version == PR_TENSOR_VERSION_1, PR_UNSUPPORTED,
          (std::string("Unsupported ") + name + " record version").c_str());
  require(op->struct_size == sizeof(Record), PR_INVALID_ARGUMENT,
          (std::string(name) + " record size mismatch").c_str());
}

void row_limit(uint64_t rows, const char *operation) {
  if (rows > max_rows)
    fail(PR_UNSUPPORTED, std::string(operation) + " supports at most " + std::to_string(max_rows) +
                             " rows (got " + std::to_string(rows) + ")");
}

} // namespace
} // namespace pb

using namespace pb;

PB_EXPORT pr_status pr_tensor_desc_contiguous(pr_buffer buffer, uint64_t byte_offset, pr_type dtype,
                                              uint32_t rank, const uint64_t *dims,
                                              pr_tensor_desc_v1 *out) {
  return boundary("tensor_desc_contiguous", [&] {
    require(out, PR_INVALID_ARGUMENT, "Missing tensor descriptor output");
    require(rank <= PR_TENSOR_MAX_RANK, PR_INVALID_ARGUMENT, "Rank exceeds PR_TENSOR_MAX_RANK");
    require(dims || !rank, PR_INVALID_ARGUMENT, "Missing tensor shape");
    pr_tensor_desc_v1 d{};
    d.struct_size = sizeof(d);
    d.version = PR_TENSOR_VERSION_1;
    d.buffer = buffer;
    d.byte_offset = byte_offset;
    d.dtype = dtype;
    d.rank = rank;
    uint64_t stride = 1;
    for (uint32_t r = rank; r-- > 0;) {
      d.shape[r] = dims[r];
      require(stride <= uint64_t(std::numeric_limits<int64_t>::max()), PR_OUT_OF_BOUNDS,
              "Contiguous stride overflows");
      d.strides[r] = int64_t(stride);
      if (dims[r] && !mul(stride, dims[r], stride))
        fail(PR_OUT_OF_BOUNDS, "Contiguous stride overflows");
    }
    *out = d;
  });
}

PB_EXPORT pr_status pr_tensor_desc_validate(const pr_tensor_desc_v1 *desc, uint64_t *required_bytes) {
  return boundary("tensor_desc_validate", [&] {
    const Layout layout = validate(desc, "tensor");
    if (required_bytes)
      *required_bytes = layout.bytes;
  });
}

PB_EXPORT pr_status pr_tensor_operators_artifact(void *data, uint64_t capacity, uint64_t *bytes) {
  return boundary("tensor_operators_artifact", [&] {
    require(bytes, PR_INVALID_ARGUMENT, "Missing artifact size output");
    const auto &value = provider_artifact();
    *bytes = value.size();
    if (data) {
      require(capacity >= value.size(), PR_OUT_OF_BOUNDS, "Artifact capacity is too small");
      std::memcpy(data, value.data(), value.size());
    }
  });
}

PB_EXPORT pr_status pr_tensor_operators_load(pr_context context, pr_module *out) {
  return boundary("tensor_operators_load", [&] {
    require(out, PR_INVALID_ARGUMENT, "Missing module output");
    *out = 0;
    const auto &value = provider_artifact();
    call(pr_module_load(context, value.data(), value.size(), out));
    try {
      std::lock_guard<std::mutex> lock(registry_mutex);
      providers().insert(*out);
    } catch (...) {
      pr_release(*out);
      *out = 0;
      throw;
    }
  });
}

PB_EXPORT pr_status pr_tensor_operators_capabilities(pr_tensor_operators_capabilities_v1 *out) {
  return boundary("tensor_operators_capabilities", [&] {
    require(out, PR_INVALID_ARGUMENT, "Missing capability record");
    require(out->version == PR_TENSOR_VERSION_1, PR_UNSUPPORTED,
            "Unsupported tensor capability record version");
    require(out->struct_size == sizeof(pr_tensor_operators_capabilities_v1), PR_INVALID_ARGUMENT,
            "Tensor capability record size mismatch");
    pr_tensor_operators_capabilities_v1 caps{};
    caps.struct_size = sizeof(caps);
    caps.version = PR_TENSOR_VERSION_1;
    caps.operations = PR_TENSOR_OP_MATMUL | PR_TENSOR_OP_BIAS_ACTIVATION | PR_TENSOR_OP_BATCHED_MATMUL |
                      PR_TENSOR_OP_REDUCE_ROWS | PR_TENSOR_OP_SOFTMAX_ROWS | PR_TENSOR_OP_LAYER_NORM |
                      PR_TENSOR_OP_ADD;
    caps.activations = PR_TENSOR_ACTIVATION_BIT(PR_ACTIVATION_NONE) |
                       PR_TENSOR_ACTIVATION_BIT(PR_ACTIVATION_RELU) |
                       PR_TENSOR_ACTIVATION_BIT(PR_ACTIVATION_GELU_TANH);
    caps.reductions = PR_TENSOR_REDUCE_BIT(PR_REDUCE_SUM) | PR_TENSOR_REDUCE_BIT(PR_REDUCE_MAX);
    caps.max_tensor_elements = max_elements;
    caps.max_row_operator_rows = max_rows;
    caps.max_layer_norm_columns = max_layer_norm_columns;
    *out = caps;
  });
}

PB_EXPORT pr_status pr_matmul_f32(pr_queue queue, pr_module operators, const pr_matmul_v1 *op,
                                  pr_event *out) {
  return boundary("matmul_f32", [&] {
    require(out, PR_INVALID_ARGUMENT, "Missing event output");
    *out = 0;
    require(op, PR_INVALID_ARGUMENT, "Missing matmul record");
    require(op->version == PR_TENSOR_VERSION_1, PR_UNSUPPORTED, "Unsupported matmul record version");
    require(op->struct_size == sizeof(pr_matmul_v1), PR_INVALID_ARGUMENT, "Matmul record size mismatch");
    require(op->transpose_a <= 1 && op->transpose_b <= 1, PR_INVALID_ARGUMENT,
            "Transpose flags must be 0 or 1");
    require(op->a && op->b && op->c, PR_INVALID_ARGUMENT, "Missing matmul tensor");
    const Layout a = operand(op->a, "A", 2), b = operand(op->b, "B", 2), c = operand(op->c, "C", 2);
    const uint64_t m = op->m, n = op->n, k = op->k;
    require(m <= max_elements && n <= max_elements && k <= max_elements, PR_UNSUPPORTED,
            "Matmul dimensions must not exceed INT32_MAX");
    if (op->transpose_a)
      expect_dims(op->a, "A (transposed storage [k,m])", {k, m});
    else
      expect_dims(op->a, "A [m,k]", {m, k});
    if (op->transpose_b)
      expect_dims(op->b, "B (transposed storage [n,k])", {n, k});
    else
      expect_dims(op->b, "B [k,n]", {k, n});
    expect_dims(op->c, "C [m,n]", {m, n});
    no_alias(op->c, c, op->a, a, "A");
    no_alias(op->c, c, op->b, b, "B");
    same_context(queue, operators, {{op->a, "A"}, {op->b, "B"}, {op->c, "C"}});
    Owned fn;
    kernel(operators, k ? "paralyn_matmul_f32" : "paralyn_fill_f32", fn);
    if (!m || !n)
      return; // no output elements: nothing is submitted and no event is invented
    Owned cv;
    view(op->c, c, PR_READ_WRITE, cv);
    if (!k) {
      const std::array<RangeArgument, 3> args{buffer(cv), u32(m * n), f32(0.0f)};
      call(launch_entry(queue, fn.module, fn.name, linear(m * n), {group, 1, 1}, args.data(), 3, out));
      return;
    }
    Owned av, bv;
    view(op->a, a, PR_READ, av);
    view(op->b, b, PR_READ, bv);
    const std::array<RangeArgument, 8> args{buffer(av), buffer(bv), buffer(cv), u32(m), u32(n), u32(k),
                                          u32(op->transpose_a), u32(op->transpose_b)};
    const pr_dim3 grid{uint32_t((n + tile - 1) / tile), uint32_t((m + tile - 1) / tile), 1};
    call(launch_entry(queue, fn.module, fn.name, grid, {tile, tile, 1}, args.data(), 8, out));
  });
}

PB_EXPORT pr_status pr_bias_activation_f32(pr_queue queue, pr_module operators,
                                           const pr_bias_activation_v1 *op, pr_event *out) {
  return boundary("bias_activation_f32", [&] {
    require(out, PR_INVALID_ARGUMENT, "Missing event output");
    *out = 0;
    require(op, PR_INVALID_ARGUMENT, "Missing bias/activation record");
    require(op->version == PR_TENSOR_VERSION_1, PR_UNSUPPORTED,
            "Unsupported bias/activation record version");
    require(op->struct_size == sizeof(pr_bias_activation_v1), PR_INVALID_ARGUMENT,
            "Bias/activation record size mismatch");
    require(op->activation == PR_ACTIVATION_NONE || op->activation == PR_ACTIVATION_RELU ||
                op->activation == PR_ACTIVATION_GELU_TANH,
            PR_INVALID_ARGUMENT, "Unknown activation");
    require(op->reserved == 0, PR_INVALID_ARGUMENT, "Reserved field must be zero");
    require(op->x && op->out, PR_INVALID_ARGUMENT, "Missing input or output tensor");
    const Layout x = operand(op->x, "x", 2), o = operand(op->out, "out", 2);
    const uint64_t rows = op->x->shape[0], columns = op->x->shape[1];
    expect_dims(op->out, "out", {rows, columns});
    Layout bias;
    if (op->bias) {
      bias = operand(op->bias, "bias", 1);
      if (op->bias->shape[0] != columns)
        fail(PR_INVALID_ARGUMENT, "bias shape " + shape_text(op->bias) + " does not match expected [" +
                                      std::to_string(columns) + "]");
    }
    no_alias(op->out, o, op->x, x, "x");
    no_alias(op->out, o, op->bias, bias, "bias");
    same_context(queue, operators, {{op->x, "x"}, {op->bias, "bias"}, {op->out, "out"}});
    Owned fn;
    kernel(operators, op->bias ? "paralyn_bias_activation_f32" : "paralyn_activation_f32", fn);
    const uint64_t count = rows * columns;
    if (!count)
      return;
    Owned xv, ov, bv;
    view(op->x, x, PR_READ, xv);
    view(op->out, o, PR_READ_WRITE, ov);
    if (op->bias) {
      view(op->bias, bias, PR_READ, bv);
      const std::array<RangeArgument, 6> args{buffer(xv), buffer(bv), buffer(ov), u32(count),
                                            u32(columns), u32(op->activation)};
      call(launch_entry(queue, fn.module, fn.name, linear(count), {group, 1, 1}, args.data(), 6, out));
    } else {
      const std::array<RangeArgument, 4> args{buffer(xv), buffer(ov), u32(count), u32(op->activation)};
      call(launch_entry(queue, fn.module, fn.name, linear(count), {group, 1, 1}, args.data(), 4, out));
    }
  });
}

// Transformer-block operators (reference runtime/tensor.cpp:847-970): the same
// record checks, validation order, zero-work rules and launch arguments.
PB_EXPORT pr_status pr_batched_matmul_f32(pr_queue queue, pr_module operators,
                                          const pr_batched_matmul_v1 *op, pr_event *out) {
  return boundary("batched_matmul_f32", [&] {
    require(out, PR_INVALID_ARGUMENT, "Missing event output");
    *out = 0;
    header(op, "batched matmul");
    require(op->a && op->b && op->c, PR_INVALID_ARGUMENT, "Missing batched matmul tensor");
    const Layout a = strided_operand(op->a, "A", 3), b = strided_operand(op->b, "B", 3),
                 c = strided_operand(op->c, "C", 3);
    const uint64_t batch = op->batch, m = op->m, n = op->n, k = op->k;
    require(batch <= max_elements && m <= max_elements && n <= max_elements && k <= max_elements,
            PR_UNSUPPORTED, "Batched matmul dimensions must not exceed INT32_MAX");
    expect_dims(op->a, "A [batch,m,k]", {batch, m, k});
    expect_dims(op->b, "B [batch,k,n]", {batch, k, n});
    expect_dims(op->c, "C [batch,m,n]", {batch, m, n});
    injective(op->c, "C");
    no_alias(op->c, c, op->a, a, "A");
    no_alias(op->c, c, op->b, b, "B");
    same_context(queue, operators, {{op->a, "A"}, {op->b, "B"}, {op->c, "C"}});
    Owned fn;
    kernel(operators, k ? "paralyn_batched_matmul_f32" : "paralyn_batched_fill_f32", fn);
    if (!batch || !m || !n)
      return; // no output elements: nothing is submitted and no event is invented
    Owned cv;
    view(op->c, c, PR_READ_WRITE, cv);
    const pr_dim3 grid{uint32_t((n + tile - 1) / tile), uint32_t((m + tile - 1) / tile), uint32_t(batch)};
    if (!k) { // the empty sum: +0.0 at every addressed output element
      const std::array<RangeArgument, 7> args{buffer(cv), u32(m), u32(n), u32(op->c->strides[0]),
                                            u32(op->c->strides[1]), u32(op->c->strides[2]), f32(0.0f)};
      call(launch_entry(queue, fn.module, fn.name, grid, {tile, tile, 1}, args.data(), 7, out));
      return;
    }
    Owned av, bv;
    view(op->a, a, PR_READ, av);
    view(op->b, b, PR_READ, bv);
    const std::array<RangeArgument, 15> args{
        buffer(av), buffer(bv), buffer(cv), u32(m), u32(n), u32(k),
        u32(op->a->strides[0]), u32(op->a->strides[1]), u32(op->a->strides[2]),
        u32(op->b->strides[0]), u32(op->b->strides[1]), u32(op->b->strides[2]),
        u32(op->c->strides[0]), u32(op->c->strides[1]), u32(op->c->strides[2])};
    call(launch_entry(queue, fn.module, fn.name, grid, {tile, tile, 1}, args.data(), 15, out));
  });
}

PB_EXPORT pr_status pr_reduce_rows_f32(pr_queue queue, pr_module operators, const pr_reduce_rows_v1 *op,
                                       pr_event *out) {
  return boundary("reduce_rows_f32", [&] {
    require(out, PR_INVALID_ARGUMENT, "Missing event output");
    *out = 0;
    header(op, "row reduction");
    require(op->op == PR_REDUCE_SUM || op->op == PR_REDUCE_MAX, PR_INVALID_ARGUMENT, "Unknown reduction");
    require(op->reserved == 0, PR_INVALID_ARGUMENT, "Reserved field must be zero");
    require(op->x && op->out, PR_INVALID_ARGUMENT, "Missing input or output tensor");
    const Layout x = operand(op->x, "x", 2), o = operand(op->out, "out", 1);
    const uint64_t rows = op->x->shape[0], columns = op->x->shape[1];
    expect_dims(op->out, "out [rows]", {rows});
    row_limit(rows, "row reduction");
    no_alias(op->out, o, op->x, x, "x");
    same_context(queue, operators, {{op->x, "x"}, {op->out, "out"}});
    Owned fn;
    kernel(operators, columns ? "paralyn_reduce_rows_f32" : "paralyn_fill_f32", fn);
    if (!rows)
      return;
    Owned ov;
    view(op->out, o, PR_READ_WRITE, ov);
    if (!columns) { // empty rows: +0.0 (sum) or -inf (max), written on the GPU
      const float identity = op->op == PR_REDUCE_MAX ? -std::numeric_limits<float>::infinity() : 0.0f;
      const std::array<RangeArgument, 3> args{buffer(ov), u32(rows), f32(identity)};
      call(launch_entry(queue, fn.module, fn.name, linear(rows), {group, 1, 1}, args.data(), 3, out));
      return;
    }
    Owned xv;
    view(op->x, x, PR_READ, xv);
    const std::array<RangeArgument, 4> args{buffer(xv), buffer(ov), u32(columns), u32(op->op)};
    call(launch_entry(queue, fn.module, fn.name, {uint32_t(rows), 1, 1}, {group, 1, 1}, args.data(), 4, out));
  });
}

PB_EXPORT pr_status pr_softmax_rows_f32(pr_queue queue, pr_module operators, const pr_softmax_rows_v1 *op,
                                        pr_event *out) {
  return boundary("softmax_rows_f32", [&] {
    require(out, PR_INVALID_ARGUMENT, "Missing event output");
    *out = 0;
    header(op, "softmax");
    require(op->causal <= 1, PR_INVALID_ARGUMENT, "causal must be 0 or 1");
    require(std::isfinite(op->scale) && op->scale > 0.0f, PR_INVALID_ARGUMENT,
            "scale must be finite and greater than zero");
    require(op->x && op->out, PR_INVALID_ARGUMENT, "Missing input or output tensor");
    const uint32_t rank = op->x->rank;
    require(rank == 2 || rank == 3, PR_INVALID_ARGUMENT,
            "x: softmax input must have rank 2 [rows,columns] or rank 3 [batch,rows,columns]");
    const Layout x = operand(op->x, "x", rank), o = operand(op->out, "out", rank);
    for (uint32_t i = 0; i < rank; ++i)
      if (op->out->shape[i] != op->x->shape[i])
        fail(PR_INVALID_ARGUMENT,
             "out shape " + shape_text(op->out) + " does not match x shape " + shape_text(op->x));
    const uint64_t columns = op->x->shape[rank - 1], rows = op->x->shape[rank - 2];
    if (op->causal && columns < rows)
      fail(PR_INVALID_ARGUMENT, "causal softmax requires columns >= rows (got " + shape_text(op->x) + ")");
    uint64_t all_rows = rows; // batch * rows for rank 3 (validate already rejected overflow)
    if (rank == 3 && !mul(all_rows, op->x->shape[0], all_rows))
      all_rows = std::numeric_limits<uint64_t>::max();
    row_limit(all_rows, "softmax (batch * rows)");
    no_alias(op->out, o, op->x, x, "x");
    same_context(queue, operators, {{op->x, "x"}, {op->out, "out"}});
    Owned fn;
    kernel(operators, "paralyn_softmax_rows_f32", fn);
    if (!x.count)
      return;
    const uint64_t total_rows = x.count / columns;
    Owned xv, ov;
    view(op->x, x, PR_READ, xv);
    view(op->out, o, PR_READ_WRITE, ov);
    const std::array<RangeArgument, 6> args{buffer(xv), buffer(ov), u32(columns), u32(rows), u32(op->causal),
                                          f32(op->scale)};
    call(launch_entry(queue, fn.module, fn.name, {uint32_t(total_rows), 1, 1}, {group, 1, 1}, args.data(), 6, out));
  });
}

PB_EXPORT pr_status pr_layer_norm_f32(pr_queue queue, pr_module operators, const pr_layer_norm_v1 *op,
                                      pr_event *out) {
  return boundary("layer_norm_f32", [&] {
    require(out, PR_INVALID_ARGUMENT, "Missing event output");
    *out = 0;
    header(op, "layer norm");
    require(std::isfinite(op->epsilon) && op->epsilon > 0.0f, PR_INVALID_ARGUMENT,
            "epsilon must be finite and greater than zero");
    require(op->reserved == 0, PR_INVALID_ARGUMENT, "Reserved field must be zero");
    require(op->x && op->gamma && op->beta && op->out, PR_INVALID_ARGUMENT,
            "Missing layer norm tensor (x, gamma, beta and out are required)");
    const Layout x = operand(op->x, "x", 2), g = operand(op->gamma, "gamma", 1),
                 b = operand(op->beta, "beta", 1), o = operand(op->out, "out", 2);
    const uint64_t rows = op->x->shape[0], columns = op->x->shape[1];
    expect_dims(op->out, "out", {rows, columns});
    expect_dims(op->gamma, "gamma", {columns});
    expect_dims(op->beta, "beta", {columns});
    require(columns <= max_layer_norm_columns, PR_UNSUPPORTED,
            "layer norm supports at most 2^24 columns (exact FP32 column count)");
    row_limit(rows, "layer norm");
    no_alias(op->out, o, op->x, x, "x");
    no_alias(op->out, o, op->gamma, g, "gamma");
    no_alias(op->out, o, op->beta, b, "beta");
    same_context(queue, operators,
                 {{op->x, "x"}, {op->gamma, "gamma"}, {op->beta, "beta"}, {op->out, "out"}});
    Owned fn;
    kernel(operators, "paralyn_layer_norm_f32", fn);
    if (!x.count)
      return;
    Owned xv, gv, bv, ov;
    view(op->x, x, PR_READ, xv);
    view(op->gamma, g, PR_READ, gv);
    view(op->beta, b, PR_READ, bv);
    view(op->out, o, PR_READ_WRITE, ov);
    const std::array<RangeArgument, 6> args{buffer(xv), buffer(gv), buffer(bv), buffer(ov),
                                          u32(columns), f32(op->epsilon)};
    call(launch_entry(queue, fn.module, fn.name, {uint32_t(rows), 1, 1}, {group, 1, 1}, args.data(), 6, out));
  });
}

PB_EXPORT pr_status pr_add_f32(pr_queue queue, pr_module operators, const pr_add_v1 *op, pr_event *out) {
  return boundary("add_f32", [&] {
    require(out, PR_INVALID_ARGUMENT, "Missing event output");
    *out = 0;
    header(op, "add");
    require(op->x && op->y && op->out, PR_INVALID_ARGUMENT, "Missing input or output tensor");
    const uint32_t rank = op->x->rank;
    const Layout x = operand(op->x, "x", rank), y = operand(op->y, "y", rank),
                 o = operand(op->out, "out", rank);
    for (uint32_t i = 0; i < rank; ++i)
      if (op->y->shape[i] != op->x->shape[i] || op->out->shape[i] != op->x->shape[i])
        fail(PR_INVALID_ARGUMENT, "add shapes differ: x " + shape_text(op->x) + ", y " +
                                      shape_text(op->y) + ", out " + shape_text(op->out));
    no_alias(op->out, o, op->x, x, "x");
    no_alias(op->out, o, op->y, y, "y");
    same_context(queue, operators, {{op->x, "x"}, {op->y, "y"}, {op->out, "out"}});
    Owned fn;
    kernel(operators, "paralyn_add_f32", fn);
    if (!x.count)
      return;
    Owned xv, yv, ov;
    view(op->x, x, PR_READ, xv);
    view(op->y, y, PR_READ, yv);
    view(op->out, o, PR_READ_WRITE, ov);
    const std::array<RangeArgument, 4> args{buffer(xv), buffer(yv), buffer(ov), u32(x.count)};
    call(launch_entry(queue, fn.module, fn.name, linear(x.count), {group, 1, 1}, args.data(), 4, out));
  });
}

// ---- LayerNorm with the output rows also gathered into peer tensors (b200.h) ----
namespace pb {
void launch_layer_norm_gather(Launch &);
}

PB_EXPORT pr_status pr_b200_layer_norm_gather_f32(pr_queue queue, pr_module operators, const pr_layer_norm_v1 *op,
                                                  const pr_tensor_desc_v1 *const *gathered, uint32_t count,
                                                  uint64_t row_offset, pr_event *out) {
  return boundary("layer_norm_gather_f32", [&] {
    require(out, PR_INVALID_ARGUMENT, "Missing event output");
    *out = 0;
    header(op, "layer norm");
    require(std::isfinite(op->epsilon) && op->epsilon > 0.0f, PR_INVALID_ARGUMENT,
            "epsilon must be finite and greater than zero");
    require(op->reserved == 0, PR_INVALID_ARGUMENT, "Reserved field must be zero");
    require(op->x && op->gamma && op->beta && op->out, PR_INVALID_ARGUMENT,
            "Missing layer norm tensor (x, gamma, beta and out are required)");
    require(count <= 8, PR_INVALID_ARGUMENT, "At most 8 gathered tensors");
    require(gathered || !count, PR_INVALID_ARGUMENT, "Missing gathered tensors");
    const Layout x = operand(op->x, "x", 2), g = operand(op->gamma, "gamma", 1),
                 b = operand(op->beta, "beta", 1), o = operand(op->out, "out", 2);
    const uint64_t rows = op->x->shape[0], columns = op->x->shape[1];
    expect_dims(op->out, "out", {rows, columns});
    expect_dims(op->gamma, "gamma", {columns});
    expect_dims(op->beta, "beta", {columns});
    require(columns <= max_layer_norm_columns, PR_UNSUPPORTED,
            "layer norm supports at most 2^24 columns (exact FP32 column count)");
    row_limit(rows, "layer norm");
    no_alias(op->out, o, op->x, x, "x");
    no_alias(op->out, o, op->gamma, g, "gamma");
    no_alias(op->out, o, op->beta, b, "beta");
    std::vector<Layout> layouts;
    for (uint32_t i = 0; i < count; ++i) {
      require(gathered[i], PR_INVALID_ARGUMENT, "Missing gathered tensor");
      layouts.push_back(operand(gathered[i], "gathered", 2));
      require(gathered[i]->shape[1] == columns, PR_INVALID_ARGUMENT, "gathered: column count differs from x");
      require(row_offset <= gathered[i]->shape[0] && rows <= gathered[i]->shape[0] - row_offset,
              PR_OUT_OF_BOUNDS, "gathered: rows [row_offset, row_offset + rows) exceed the tensor");
      no_alias(gathered[i], layouts.back(), op->x, x, "x");
      no_alias(gathered[i], layouts.back(), op->gamma, g, "gamma");
      no_alias(gathered[i], layouts.back(), op->beta, b, "beta");
    }
    same_context(queue, operators,
                 {{op->x, "x"}, {op->gamma, "gamma"}, {op->beta, "beta"}, {op->out, "out"}});
    for (uint32_t i = 0; i < count; ++i)
      same_context(queue, operators, {{gathered[i], "gathered"}});
    Owned fn;
    kernel(operators, "paralyn_layer_norm_f32", fn);
    if (!x.count)
      return;
    call(api("layer_norm_gather_f32", [&] {
      const QueueAccess q = queue_access(queue);
      std::vector<BoundArg> args;
      std::vector<std::shared_ptr<Allocation>> retained;
      auto view = [&](const pr_tensor_desc_v1 *d, const Layout &l, bool writes = true) {
        auto allocation = buffer_allocation(d->buffer, q.context);
        BoundArg a;
        a.buffer = true;
        a.writes = writes;
        a.ptr = static_cast<char *>(allocation->ptr) + d->byte_offset;
        a.bytes = l.bytes;
        args.push_back(a);
        retained.push_back(std::move(allocation));
      };
      auto scalar = [&](uint32_t bits) {
        BoundArg a;
        a.bits = bits;
        args.push_back(a);
      };
      view(op->x, x, false);
      view(op->gamma, g, false);
      view(op->beta, b, false);
      view(op->out, o);
      uint32_t eps_bits;
      std::memcpy(&eps_bits, &op->epsilon, 4);
      scalar(uint32_t(columns));
      scalar(eps_bits);
      scalar(uint32_t(rows));
      scalar(uint32_t(row_offset));
      scalar(uint32_t(row_offset >> 32));
      scalar(count);
      for (uint32_t i = 0; i < count; ++i)
        view(gathered[i], layouts[i]);
      *out = submit_command(queue, "b200_layer_norm_gather_f32", launch_layer_norm_gather,
                            Dim3{uint32_t(rows), 1, 1}, Dim3{256, 1, 1}, std::move(args), std::move(retained));
    }));
  });
}

namespace pb {
void launch_matmul_bias_activation(Launch &);
}

// C = activation(op(A) op(B) + bias[column]) in one command: the matmul record and its
// validation as pr_matmul_f32 (same order and statuses), plus an optional bias [n] and
// the activation of pr_bias_activation_f32. Results equal pr_matmul_f32 followed by
// pr_bias_activation_f32 bit for bit; C is written once.
PB_EXPORT pr_status pr_b200_matmul_bias_activation_f32(pr_queue queue, pr_module operators, const pr_matmul_v1 *op,
                                                       const pr_tensor_desc_v1 *bias, uint32_t activation,
                                                       pr_event *out) {
  return boundary("matmul_bias_activation_f32", [&] {
    require(out, PR_INVALID_ARGUMENT, "Missing event output");
    *out = 0;
    require(op, PR_INVALID_ARGUMENT, "Missing matmul record");
    require(op->version == PR_TENSOR_VERSION_1, PR_UNSUPPORTED, "Unsupported matmul record version");
    require(op->struct_size == sizeof(pr_matmul_v1), PR_INVALID_ARGUMENT, "Matmul record size mismatch");
    require(op->transpose_a <= 1 && op->transpose_b <= 1, PR_INVALID_ARGUMENT,
            "Transpose flags must be 0 or 1");
    require(activation == PR_ACTIVATION_NONE || activation == PR_ACTIVATION_RELU ||
                activation == PR_ACTIVATION_GELU_TANH,
            PR_INVALID_ARGUMENT, "Unknown activation");
    require(op->a && op->b && op->c, PR_INVALID_ARGUMENT, "Missing matmul tensor");
    const Layout a = operand(op->a, "A", 2), b = operand(op->b, "B", 2), c = operand(op->c, "C", 2);
    const uint64_t m = op->m, n = op->n, k = op->k;
    require(m <= max_elements && n <= max_elements && k <= max_elements, PR_UNSUPPORTED,
            "Matmul dimensions must not exceed INT32_MAX");
    if (op->transpose_a)
      expect_dims(op->a, "A (transposed storage [k,m])", {k, m});
    else
      expect_dims(op->a, "A [m,k]", {m, k});
    if (op->transpose_b)
      expect_dims(op->b, "B (transposed storage [n,k])", {n, k});
    else
      expect_dims(op->b, "B [k,n]", {k, n});
    expect_dims(op->c, "C [m,n]", {m, n});
    Layout bl;
    if (bias) {
      bl = operand(bias, "bias", 1);
      expect_dims(bias, "bias", {n});
    }
    no_alias(op->c, c, op->a, a, "A");
    no_alias(op->c, c, op->b, b, "B");
    no_alias(op->c, c, bias, bl, "bias");
    same_context(queue, operators, {{op->a, "A"}, {op->b, "B"}, {op->c, "C"}, {bias, "bias"}});
    Owned fn;
    kernel(operators, "paralyn_matmul_f32", fn);
    if (!m || !n)
      return; // no output elements: nothing is submitted and no event is invented
    call(api("matmul_bias_activation_f32", [&] {
      const QueueAccess q = queue_access(queue);
      std::vector<BoundArg> args;
      std::vector<std::shared_ptr<Allocation>> retained;
      auto view = [&](const pr_tensor_desc_v1 *d, const Layout &l, bool writes) {
        BoundArg arg;
        arg.buffer = true;
        arg.writes = writes;
        if (d && l.bytes) {
          auto allocation = buffer_allocation(d->buffer, q.context);
          arg.ptr = static_cast<char *>(allocation->ptr) + d->byte_offset;
          arg.bytes = l.bytes;
          retained.push_back(std::move(allocation));
        }
        args.push_back(arg);
      };
      auto scalar = [&](uint64_t bits) {
        BoundArg arg;
        arg.bits = uint32_t(bits);
        args.push_back(arg);
      };
      view(op->a, a, false);
      view(op->b, b, false);
      view(op->c, c, true);
      scalar(m);
      scalar(n);
      scalar(k);
      scalar(op->transpose_a);
      scalar(op->transpose_b);
      view(bias, bl, false);
      scalar(activation);
      scalar(bias ? 1 : 0);
      *out = submit_command(queue, "b200_matmul_bias_activation_f32", launch_matmul_bias_activation,
                            Dim3{uint32_t((n + tile - 1) / tile), uint32_t((m + tile - 1) / tile), 1},
                            Dim3{tile, tile, 1}, std::move(args), std::move(retained));
    }));
  });
}
