"""FP32 tensors and the tensor-operator provider (include/paralyn/tensor.h).

The names and meaning are the reference binding's (package `paralyn`): explicit
TensorDescriptors (buffer, byte offset, shape, strides in elements), the *_into
calls that take descriptors and return the command's Event (None when there is no
GPU work), and Tensor with tensor(), matmul(), batched_matmul(), layer_norm(),
softmax(), row_sum(), row_max(), residual_add(), bias_add(), relu(), gelu(),
bias_gelu(), which allocate a distinct output on the inputs' context.

Every operator is one row of `_OPERATORS` (entry point, record type, record
fields); `_enqueue` builds the versioned record from keyword values and submits it
with the provider module on a queue.
"""
import ctypes as _c
from contextlib import ExitStack
from dataclasses import dataclass
from enum import IntEnum

from .native import Context, Event, Module, Queue, Type, _int, _u64, layout, library
from .values import MAX_ELEMENTS, DeviceValue, common_context, float32, host_fp32, produce, upload

TENSOR_VERSION_1 = 1
MAX_RANK = 8


class Activation(IntEnum):
    NONE = 0
    RELU = 1
    GELU_TANH = 2


class Reduce(IntEnum):
    SUM = 0
    MAX = 1


# ---------------------------------------------------------------- records (tensor.h layouts)
class TensorDescRecord(_c.Structure):
    _fields_ = layout("struct_size:u32 version:u32 buffer:u64 byte_offset:u64 dtype:enum rank:u32 shape:u64[8] "
                      "strides:i64[8]")


_D = {"TensorDescRecord": TensorDescRecord}
_DESC = "ptr=TensorDescRecord"


class MatmulRecord(_c.Structure):
    _fields_ = layout(f"struct_size:u32 version:u32 m:u64 n:u64 k:u64 transpose_a:u32 transpose_b:u32 a:{_DESC} "
                      f"b:{_DESC} c:{_DESC}", **_D)


class BiasActivationRecord(_c.Structure):
    _fields_ = layout(f"struct_size:u32 version:u32 activation:enum reserved:u32 x:{_DESC} bias:{_DESC} "
                      f"out:{_DESC}", **_D)


class BatchedMatmulRecord(_c.Structure):
    _fields_ = layout(f"struct_size:u32 version:u32 batch:u64 m:u64 n:u64 k:u64 a:{_DESC} b:{_DESC} c:{_DESC}",
                      **_D)


class ReduceRowsRecord(_c.Structure):
    _fields_ = layout(f"struct_size:u32 version:u32 op:enum reserved:u32 x:{_DESC} out:{_DESC}", **_D)


class SoftmaxRowsRecord(_c.Structure):
    _fields_ = layout(f"struct_size:u32 version:u32 causal:u32 scale:f32 x:{_DESC} out:{_DESC}", **_D)


class LayerNormRecord(_c.Structure):
    _fields_ = layout(f"struct_size:u32 version:u32 epsilon:f32 reserved:u32 x:{_DESC} gamma:{_DESC} "
                      f"beta:{_DESC} out:{_DESC}", **_D)


class AddRecord(_c.Structure):
    _fields_ = layout(f"struct_size:u32 version:u32 x:{_DESC} y:{_DESC} out:{_DESC}", **_D)


class CapabilitiesRecord(_c.Structure):
    _fields_ = layout("struct_size:u32 version:u32 operations:u64 activations:u64 reductions:u64 "
                      "max_tensor_elements:u64 max_row_operator_rows:u64 max_layer_norm_columns:u64")


_TENSOR_CALLS = """
pr_tensor_desc_contiguous h u64 enum u32 *u64 *TensorDescRecord
pr_tensor_desc_validate *TensorDescRecord *u64
pr_tensor_operators_artifact ptr u64 *u64
pr_tensor_operators_load h *h
pr_tensor_operators_capabilities *CapabilitiesRecord
pr_matmul_f32 h h *MatmulRecord *h
pr_bias_activation_f32 h h *BiasActivationRecord *h
pr_batched_matmul_f32 h h *BatchedMatmulRecord *h
pr_reduce_rows_f32 h h *ReduceRowsRecord *h
pr_softmax_rows_f32 h h *SoftmaxRowsRecord *h
pr_layer_norm_f32 h h *LayerNormRecord *h
pr_add_f32 h h *AddRecord *h
"""
_RECORDS = {cls.__name__: cls for cls in (TensorDescRecord, MatmulRecord, BiasActivationRecord, BatchedMatmulRecord,
                                          ReduceRowsRecord, SoftmaxRowsRecord, LayerNormRecord, AddRecord,
                                          CapabilitiesRecord)}


def _api(lib):
    """`lib` with the tensor entry points declared."""
    if not lib.declares("pr_matmul_f32"):
        lib.declare(_TENSOR_CALLS, **_RECORDS)
    return lib


def _pointer(record):
    """A ctypes pointer to `record`, made once and kept on the record."""
    if not hasattr(record, "_self_pointer"):
        record._self_pointer = _c.pointer(record)
    return record._self_pointer


# ---------------------------------------------------------------- descriptors
def _dims(shape):
    """(shape tuple, element count) with the provider's rank and element limits."""
    if isinstance(shape, int) and not isinstance(shape, bool):
        shape = (shape,)
    if not isinstance(shape, (tuple, list)) or len(shape) > MAX_RANK:
        raise ValueError(f"a shape is a tuple of at most {MAX_RANK} extents")
    dims = tuple(_int(extent, 0, 2 ** 63 - 1, "extent") for extent in shape)
    count = 1
    for extent in dims:
        count *= extent
    if count > MAX_ELEMENTS:
        raise ValueError(f"{count} elements exceed the FP32 tensor limit of {MAX_ELEMENTS}")
    return dims, count


@dataclass(frozen=True)
class TensorDescriptor:
    """An FP32 tensor over a Buffer: shape, byte offset and strides in elements
    (None: contiguous row-major). Immutable; its native record is built on first use."""
    buffer: object
    shape: tuple
    byte_offset: int = 0
    strides: object = None

    def _native(self):
        record = self.__dict__.get("_record")
        if record is None or self.buffer.closed:  # a closed buffer reports itself as on first use
            record = self._build()
            object.__setattr__(self, "_record", record)
        return record

    def _build(self):
        lib = _api(self.buffer._lib)
        dims = tuple(self.shape)
        if len(dims) > MAX_RANK:
            raise ValueError(f"rank {len(dims)} exceeds {MAX_RANK}")
        record = TensorDescRecord()
        if self.strides is None:
            extents = (_c.c_uint64 * max(1, len(dims)))(*dims)
            lib.call("pr_tensor_desc_contiguous", self.buffer.handle, self.byte_offset, Type.F32, len(dims), extents,
                     _c.byref(record))
            return record
        if len(self.strides) != len(dims):
            raise ValueError("strides need one entry per dimension")
        # Strided views may reach beyond the contiguous extent of their shape: the
        # record is written directly and the operators check it against the buffer.
        record.struct_size, record.version = _c.sizeof(TensorDescRecord), TENSOR_VERSION_1
        record.buffer = self.buffer.handle
        record.byte_offset = _u64(self.byte_offset, "byte_offset")
        record.dtype, record.rank = Type.F32, len(dims)
        for axis, (extent, stride) in enumerate(zip(dims, self.strides)):
            record.shape[axis] = _u64(extent, "extent")
            record.strides[axis] = _int(stride, -2 ** 63, 2 ** 63 - 1, "stride")
        return record

    def required_bytes(self):
        lib = _api(self.buffer._lib)
        out = _c.c_uint64()
        lib.call("pr_tensor_desc_validate", _c.byref(self._native()), _c.byref(out))
        return out.value


# ---------------------------------------------------------------- provider module and capabilities
def tensor_operators_artifact(library_path=None):
    """The provider artifact's exact bytes."""
    lib = _api(library(library_path))
    size = _c.c_uint64()
    lib.call("pr_tensor_operators_artifact", None, 0, _c.byref(size))
    image = _c.create_string_buffer(size.value)
    lib.call("pr_tensor_operators_artifact", image, size.value, _c.byref(size))
    return image.raw[:size.value]


_OPERATION_NAMES = ("matmul", "bias_activation", "batched_matmul", "reduce_rows", "softmax_rows", "layer_norm",
                    "add")  # bit i of the capability record's operation mask


@dataclass(frozen=True)
class TensorOperatorCapabilities:
    operations: frozenset
    activations: frozenset
    reductions: frozenset
    max_tensor_elements: int
    max_row_operator_rows: int
    max_layer_norm_columns: int


def tensor_operators_capabilities(library_path=None):
    lib = _api(library(library_path))
    caps = CapabilitiesRecord(_c.sizeof(CapabilitiesRecord), TENSOR_VERSION_1)
    lib.call("pr_tensor_operators_capabilities", _c.byref(caps))

    def members(mask, names):
        return frozenset(name for bit, name in enumerate(names) if mask >> bit & 1)
    return TensorOperatorCapabilities(members(caps.operations, _OPERATION_NAMES),
                                      frozenset(a for a in Activation if caps.activations >> a & 1),
                                      frozenset(r for r in Reduce if caps.reductions >> r & 1),
                                      caps.max_tensor_elements, caps.max_row_operator_rows,
                                      caps.max_layer_norm_columns)


def load_tensor_operators(context):
    """Loads the provider module on `context`; the caller owns (and closes) it."""
    if not isinstance(context, Context):
        raise TypeError("load_tensor_operators needs a Context")
    lib = _api(context._lib)
    return Module._adopt(lib, lib.acquire("pr_tensor_operators_load", context.handle))


class _Provider:
    """A context's provider module and queue, loaded once per context."""

    def __init__(self, context):
        with ExitStack() as held:
            self.module = held.enter_context(load_tensor_operators(context))
            self.queue = held.enter_context(context.queue())
            self._held = held.pop_all()

    def close(self):
        self._held.close()


def operators_of(context):
    """The context's (module, queue) provider pair, loaded on first use."""
    return context.attached("tensor_operators", _Provider)


# ---------------------------------------------------------------- descriptor-level operators
def _flag(value, label):
    if not isinstance(value, bool):
        raise TypeError(f"{label}: expected a bool")
    return int(value)


def _real(value, label):
    if isinstance(value, bool) or not isinstance(value, (int, float)):
        raise TypeError(f"{label}: expected a real number")
    return float(value)


def _enqueue(queue, operators, entry, record_type, **fields):
    """Builds a versioned `record_type` from `fields` (descriptors become pointers to
    their records, None stays a null pointer) and submits it; the Event or None."""
    if not isinstance(queue, Queue) or not isinstance(operators, Module):
        raise TypeError(f"{entry} takes a Queue and the tensor operator Module")
    record = record_type(struct_size=_c.sizeof(record_type), version=TENSOR_VERSION_1)
    for name, value in fields.items():
        if isinstance(value, TensorDescriptor):
            value = _pointer(value._native())
        if value is not None:
            setattr(record, name, value)
    lib = _api(queue._lib)
    handle = lib.acquire(entry, queue.handle, operators.handle, _c.byref(record))
    return Event._adopt(lib, handle) if handle else None


def matmul_into(queue, operators, a, b, c, *, m, n, k, transpose_a=False, transpose_b=False):
    """C = op(A) op(B) for explicit m, n, k; None when m*n == 0."""
    return _enqueue(queue, operators, "pr_matmul_f32", MatmulRecord, m=_u64(m, "m"), n=_u64(n, "n"), k=_u64(k, "k"),
                    transpose_a=_flag(transpose_a, "transpose_a"), transpose_b=_flag(transpose_b, "transpose_b"),
                    a=a, b=b, c=c)


def bias_activation_into(queue, operators, x, bias, out, *, activation=Activation.NONE):
    """out = activation(x + bias[column]); bias may be None."""
    return _enqueue(queue, operators, "pr_bias_activation_f32", BiasActivationRecord,
                    activation=int(Activation(activation)), x=x, bias=bias, out=out)


def batched_matmul_into(queue, operators, a, b, c, *, batch, m, n, k):
    """C[z] = A[z] B[z] for rank-3 (possibly strided) [batch,m,k] x [batch,k,n]."""
    return _enqueue(queue, operators, "pr_batched_matmul_f32", BatchedMatmulRecord, batch=_u64(batch, "batch"),
                    m=_u64(m, "m"), n=_u64(n, "n"), k=_u64(k, "k"), a=a, b=b, c=c)


def reduce_rows_into(queue, operators, x, out, *, op=Reduce.SUM):
    """out[i] = sum or max of row i of x [rows, columns] in the fixed 256-lane order."""
    return _enqueue(queue, operators, "pr_reduce_rows_f32", ReduceRowsRecord, op=int(Reduce(op)), x=x, out=out)


def softmax_rows_into(queue, operators, x, out, *, scale=1.0, causal=False):
    """Softmax of scale*x over the last dimension of a rank-2 or rank-3 descriptor."""
    return _enqueue(queue, operators, "pr_softmax_rows_f32", SoftmaxRowsRecord, causal=_flag(causal, "causal"),
                    scale=_real(scale, "scale"), x=x, out=out)


def layer_norm_into(queue, operators, x, gamma, beta, out, *, epsilon=1e-5):
    """LayerNorm over the last dimension of x [rows, columns] with gamma, beta [columns]."""
    return _enqueue(queue, operators, "pr_layer_norm_f32", LayerNormRecord, epsilon=_real(epsilon, "epsilon"),
                    x=x, gamma=gamma, beta=beta, out=out)


def add_into(queue, operators, x, y, out):
    """out = x + y elementwise for equal-shape contiguous descriptors."""
    return _enqueue(queue, operators, "pr_add_f32", AddRecord, x=x, y=y, out=out)


# ---------------------------------------------------------------- tensors
class Tensor(DeviceValue):
    """A contiguous row-major FP32 tensor on one context."""
    _kind = "Tensor"

    @property
    def ndim(self):
        return len(self._shape)

    def descriptor(self):
        self._open()
        return TensorDescriptor(self._buffer, self._shape)

    def timing(self):
        self._open()
        return None if self._event is None else self._event.timing()


def tensor(values, *, shape, context, dtype=float32):
    """A new Tensor of `shape` holding the flat row-major host values."""
    if not isinstance(context, Context):
        raise TypeError("tensor needs an explicit Context")
    if dtype != float32:
        raise ValueError("tensor stores float32 only (pass dtype=paralyn_b200.float32)")
    dims, count = _dims(shape)
    data = host_fp32(values, "tensor")
    if data.nbytes != 4 * count:
        raise ValueError(f"{data.nbytes // 4} values cannot fill shape {dims}")
    return upload(Tensor, context, data, dims)


def _new(context, shape, device, submit):
    """A new Tensor of `shape` written by submit(provider, output descriptor)."""
    dims, count = _dims(shape)
    provider = operators_of(context)
    return produce(Tensor, context, dims, 4 * count, device,
                   lambda buffer: submit(provider, TensorDescriptor(buffer, dims)))


def matmul(a, b, *, transpose_a=False, transpose_b=False):
    """op(A) op(B) of rank-2 tensors (FP32 accumulation in increasing k)."""
    context = common_context((a, b), Tensor, "matmul")
    if a.ndim != 2 or b.ndim != 2:
        raise ValueError("matmul takes rank-2 tensors")
    m, k = a.shape[::-1] if _flag(transpose_a, "transpose_a") else a.shape
    k_b, n = b.shape[::-1] if _flag(transpose_b, "transpose_b") else b.shape
    if k != k_b:
        raise ValueError(f"matmul: inner extents {k} and {k_b} differ")
    return _new(context, (m, n), a.device, lambda r, c: matmul_into(
        r.queue, r.module, a.descriptor(), b.descriptor(), c, m=m, n=n, k=k, transpose_a=transpose_a,
        transpose_b=transpose_b))


def _bias_activation(x, bias, activation):
    operands = (x,) if bias is None else (x, bias)
    context = common_context(operands, Tensor, "bias_activation")
    return _new(context, x.shape, x.device, lambda r, out: bias_activation_into(
        r.queue, r.module, x.descriptor(), None if bias is None else bias.descriptor(), out,
        activation=activation))


def bias_add(x, bias, *, relu=False):
    """x[i, j] + bias[j], then ReLU when relu=True."""
    return _bias_activation(x, bias, Activation.RELU if _flag(relu, "relu") else Activation.NONE)


def relu(x):
    return _bias_activation(x, None, Activation.RELU)


def gelu(x):
    """The tanh-form GELU of every element."""
    return _bias_activation(x, None, Activation.GELU_TANH)


def bias_gelu(x, bias):
    return _bias_activation(x, bias, Activation.GELU_TANH)


def batched_matmul(a, b):
    """A[z] B[z] of contiguous rank-3 tensors [batch,m,k] x [batch,k,n]."""
    context = common_context((a, b), Tensor, "batched_matmul")
    if a.ndim != 3 or b.ndim != 3:
        raise ValueError("batched_matmul takes rank-3 tensors")
    batch, m, k = a.shape
    if b.shape[:2] != (batch, k):
        raise ValueError(f"batched_matmul: {a.shape} x {b.shape} do not chain")
    n = b.shape[2]
    return _new(context, (batch, m, n), a.device, lambda r, c: batched_matmul_into(
        r.queue, r.module, a.descriptor(), b.descriptor(), c, batch=batch, m=m, n=n, k=k))


def _rows(x, op):
    context = common_context((x,), Tensor, "row reduction")
    if x.ndim != 2:
        raise ValueError("row reductions take rank-2 tensors")
    return _new(context, (x.shape[0],), x.device,
                lambda r, out: reduce_rows_into(r.queue, r.module, x.descriptor(), out, op=op))


def row_sum(x):
    """Row sums in the fixed 256-lane order."""
    return _rows(x, Reduce.SUM)


def row_max(x):
    """Row maxima (NaN propagates, +0.0 wins over -0.0, -inf for empty rows)."""
    return _rows(x, Reduce.MAX)


def softmax(x, *, scale=1.0, causal=False):
    """Row softmax of scale*x over the last dimension."""
    context = common_context((x,), Tensor, "softmax")
    return _new(context, x.shape, x.device, lambda r, out: softmax_rows_into(
        r.queue, r.module, x.descriptor(), out, scale=scale, causal=causal))


def layer_norm(x, gamma, beta, *, epsilon=1e-5):
    """LayerNorm over the last dimension of a rank-2 tensor."""
    context = common_context((x, gamma, beta), Tensor, "layer_norm")
    return _new(context, x.shape, x.device, lambda r, out: layer_norm_into(
        r.queue, r.module, x.descriptor(), gamma.descriptor(), beta.descriptor(), out, epsilon=epsilon))


def residual_add(x, y):
    """x + y elementwise (equal shapes)."""
    context = common_context((x, y), Tensor, "residual_add")
    return _new(context, x.shape, x.device, lambda r, out: add_into(
        r.queue, r.module, x.descriptor(), y.descriptor(), out))
