"""FP32 tensors and the tensor-operator provider (include/paralyn/tensor.h).

Mirrors the reference's tensor API (bindings/python/paralyn/tensor.py): explicit
descriptors (buffer, byte offset, shape, strides), the *_into calls that take
descriptors and return an Event (or None when there is no GPU work), and the
high-level Tensor, tensor(), matmul(), layer_norm(), residual_add(), bias_add(),
relu(), gelu() that allocate distinct outputs on the inputs' context.
"""
from array import array as _host_array
import ctypes as _c
from contextlib import ExitStack
from dataclasses import dataclass
from enum import IntEnum
import os

from .native import (Context, Error, Event, Module, Queue, Status, Type, _int, library, f32)

float32 = "float32"
TENSOR_VERSION_1 = 1
MAX_RANK = 8
_MAX_ELEMENTS = (1 << 31) - 1


class Activation(IntEnum):
    NONE = 0
    RELU = 1
    GELU_TANH = 2


class Reduce(IntEnum):
    SUM = 0
    MAX = 1


class TensorDescRecord(_c.Structure):
    _fields_ = [("struct_size", _c.c_uint32), ("version", _c.c_uint32), ("buffer", _c.c_uint64),
                ("byte_offset", _c.c_uint64), ("dtype", _c.c_int), ("rank", _c.c_uint32),
                ("shape", _c.c_uint64 * MAX_RANK), ("strides", _c.c_int64 * MAX_RANK)]


_DESC = _c.POINTER(TensorDescRecord)


class MatmulRecord(_c.Structure):
    _fields_ = [("struct_size", _c.c_uint32), ("version", _c.c_uint32), ("m", _c.c_uint64),
                ("n", _c.c_uint64), ("k", _c.c_uint64), ("transpose_a", _c.c_uint32),
                ("transpose_b", _c.c_uint32), ("a", _DESC), ("b", _DESC), ("c", _DESC)]


class BiasActivationRecord(_c.Structure):
    _fields_ = [("struct_size", _c.c_uint32), ("version", _c.c_uint32), ("activation", _c.c_int),
                ("reserved", _c.c_uint32), ("x", _DESC), ("bias", _DESC), ("out", _DESC)]


class BatchedMatmulRecord(_c.Structure):
    _fields_ = [("struct_size", _c.c_uint32), ("version", _c.c_uint32), ("batch", _c.c_uint64),
                ("m", _c.c_uint64), ("n", _c.c_uint64), ("k", _c.c_uint64), ("a", _DESC), ("b", _DESC),
                ("c", _DESC)]


class ReduceRowsRecord(_c.Structure):
    _fields_ = [("struct_size", _c.c_uint32), ("version", _c.c_uint32), ("op", _c.c_int),
                ("reserved", _c.c_uint32), ("x", _DESC), ("out", _DESC)]


class SoftmaxRowsRecord(_c.Structure):
    _fields_ = [("struct_size", _c.c_uint32), ("version", _c.c_uint32), ("causal", _c.c_uint32),
                ("scale", _c.c_float), ("x", _DESC), ("out", _DESC)]


class LayerNormRecord(_c.Structure):
    _fields_ = [("struct_size", _c.c_uint32), ("version", _c.c_uint32), ("epsilon", _c.c_float),
                ("reserved", _c.c_uint32), ("x", _DESC), ("gamma", _DESC), ("beta", _DESC),
                ("out", _DESC)]


class AddRecord(_c.Structure):
    _fields_ = [("struct_size", _c.c_uint32), ("version", _c.c_uint32), ("x", _DESC), ("y", _DESC),
                ("out", _DESC)]


class CapabilitiesRecord(_c.Structure):
    _fields_ = [("struct_size", _c.c_uint32), ("version", _c.c_uint32), ("operations", _c.c_uint64),
                ("activations", _c.c_uint64), ("reductions", _c.c_uint64),
                ("max_tensor_elements", _c.c_uint64), ("max_row_operator_rows", _c.c_uint64),
                ("max_layer_norm_columns", _c.c_uint64)]


def _api(lib):
    if not getattr(lib, "_tensor_signatures", False):
        h, u32, u64, ptr = _c.c_uint64, _c.c_uint32, _c.c_uint64, _c.POINTER
        signatures = {
            "pr_tensor_desc_contiguous": (_c.c_int, [h, u64, _c.c_int, u32, ptr(u64), ptr(TensorDescRecord)]),
            "pr_tensor_desc_validate": (_c.c_int, [ptr(TensorDescRecord), ptr(u64)]),
            "pr_tensor_operators_artifact": (_c.c_int, [_c.c_void_p, u64, ptr(u64)]),
            "pr_tensor_operators_load": (_c.c_int, [h, ptr(h)]),
            "pr_matmul_f32": (_c.c_int, [h, h, ptr(MatmulRecord), ptr(h)]),
            "pr_bias_activation_f32": (_c.c_int, [h, h, ptr(BiasActivationRecord), ptr(h)]),
            "pr_layer_norm_f32": (_c.c_int, [h, h, ptr(LayerNormRecord), ptr(h)]),
            "pr_batched_matmul_f32": (_c.c_int, [h, h, ptr(BatchedMatmulRecord), ptr(h)]),
            "pr_reduce_rows_f32": (_c.c_int, [h, h, ptr(ReduceRowsRecord), ptr(h)]),
            "pr_softmax_rows_f32": (_c.c_int, [h, h, ptr(SoftmaxRowsRecord), ptr(h)]),
            "pr_add_f32": (_c.c_int, [h, h, ptr(AddRecord), ptr(h)]),
            "pr_tensor_operators_capabilities": (_c.c_int, [ptr(CapabilitiesRecord)]),
        }
        for name, (result, arguments) in signatures.items():
            function = getattr(lib.api, name)
            function.restype, function.argtypes = result, arguments
        lib._tensor_signatures = True
    return lib


def _shape(shape):
    if isinstance(shape, int) and not isinstance(shape, bool):
        shape = (shape,)
    if not isinstance(shape, (tuple, list)) or len(shape) > MAX_RANK:
        raise ValueError(f"shape must be a tuple of at most {MAX_RANK} dimensions")
    result = tuple(_int(d, 0, (1 << 63) - 1, "dimension") for d in shape)
    count = 1
    for d in result:
        count *= d
    if count > _MAX_ELEMENTS:
        raise ValueError("FP32 tensors support at most INT32_MAX elements")
    return result, count


@dataclass(frozen=True)
class TensorDescriptor:
    """Descriptor over a Buffer; strides in elements, None = contiguous row-major."""
    buffer: object
    shape: tuple
    byte_offset: int = 0
    strides: object = None

    def _native(self):
        # The record is built once per descriptor (descriptors are immutable) and
        # rebuilt only to report a closed buffer the same way as the first time.
        cached = self.__dict__.get("_record")
        if cached is not None and not self.buffer.closed:
            return cached
        record = self._build_native()
        object.__setattr__(self, "_record", record)
        return record

    def _build_native(self):
        lib = _api(self.buffer._lib)
        shape = tuple(self.shape)
        if len(shape) > MAX_RANK:
            raise ValueError(f"rank exceeds {MAX_RANK}")
        desc = TensorDescRecord()
        if self.strides is None:
            dims = (_c.c_uint64 * max(1, len(shape)))(*shape)
            lib.check(lib.api.pr_tensor_desc_contiguous(self.buffer.handle, self.byte_offset, Type.F32,
                                                        len(shape), dims, _c.byref(desc)))
            return desc
        if len(self.strides) != len(shape):
            raise ValueError("strides must have one entry per dimension")
        # A strided view may reach past the contiguous extent of its shape, so the
        # record is filled directly; the operators validate it against the buffer.
        desc.struct_size, desc.version = _c.sizeof(TensorDescRecord), TENSOR_VERSION_1
        desc.buffer, desc.byte_offset = self.buffer.handle, _int(self.byte_offset, 0, (1 << 64) - 1, "byte_offset")
        desc.dtype, desc.rank = Type.F32, len(shape)
        for index, (extent, stride) in enumerate(zip(shape, self.strides)):
            desc.shape[index] = _int(extent, 0, (1 << 64) - 1, "shape")
            desc.strides[index] = _int(stride, -(1 << 63), (1 << 63) - 1, "stride")
        return desc

    def required_bytes(self):
        lib = _api(self.buffer._lib)
        value = _c.c_uint64()
        lib.check(lib.api.pr_tensor_desc_validate(_c.byref(self._native()), _c.byref(value)))
        return value.value


def tensor_operators_artifact(library_path=None):
    """Exact bytes of the provider artifact."""
    lib = _api(library(library_path))
    size = _c.c_uint64()
    lib.check(lib.api.pr_tensor_operators_artifact(None, 0, _c.byref(size)))
    data = _c.create_string_buffer(size.value)
    lib.check(lib.api.pr_tensor_operators_artifact(data, size.value, _c.byref(size)))
    return data.raw[:size.value]


_OPERATION_BITS = ("matmul", "bias_activation", "batched_matmul", "reduce_rows", "softmax_rows",
                   "layer_norm", "add")


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
    lib.check(lib.api.pr_tensor_operators_capabilities(_c.byref(caps)))
    operations = frozenset(n for bit, n in enumerate(_OPERATION_BITS) if caps.operations >> bit & 1)
    activations = frozenset(a for a in Activation if caps.activations >> int(a) & 1)
    reductions = frozenset(r for r in Reduce if caps.reductions >> int(r) & 1)
    return TensorOperatorCapabilities(operations, activations, reductions, caps.max_tensor_elements,
                                      caps.max_row_operator_rows, caps.max_layer_norm_columns)


def load_tensor_operators(context):
    """Load the provider module; the caller owns it."""
    if not isinstance(context, Context):
        raise TypeError("load_tensor_operators requires a Context")
    lib = _api(context._lib)
    handle = _c.c_uint64()
    lib.check(lib.api.pr_tensor_operators_load(context.handle, _c.byref(handle)))
    return Module._adopt(lib, handle.value)


def _event(lib, handle):
    return Event._adopt(lib, handle) if handle else None


def _flag(value, label):
    if not isinstance(value, bool):
        raise TypeError(f"{label} must be a bool")
    return int(value)


def _real(value, label):
    if isinstance(value, bool) or not isinstance(value, (int, float)):
        raise TypeError(f"{label} must be a real number")
    return float(value)


def _pointer(record):
    """A ctypes pointer to a descriptor record, made once per record."""
    pointer = getattr(record, "_pointer", None)
    if pointer is None:
        pointer = record._pointer = _c.pointer(record)
    return pointer


def _submit(queue, operators, name, record):
    if not isinstance(queue, Queue) or not isinstance(operators, Module):
        raise TypeError(f"{name} requires a Queue and the tensor operator Module")
    lib = _api(queue._lib)
    handle = _c.c_uint64()
    lib.check(getattr(lib.api, name)(queue.handle, operators.handle, _c.byref(record), _c.byref(handle)))
    return _event(lib, handle.value)


def matmul_into(queue, operators, a, b, c, *, m, n, k, transpose_a=False, transpose_b=False):
    """C = op(A) op(B) with explicit m, n, k; returns an Event or None when m*n == 0."""
    descs = [x._native() for x in (a, b, c)]
    record = MatmulRecord(_c.sizeof(MatmulRecord), TENSOR_VERSION_1,
                          _int(m, 0, (1 << 64) - 1, "m"), _int(n, 0, (1 << 64) - 1, "n"),
                          _int(k, 0, (1 << 64) - 1, "k"), _flag(transpose_a, "transpose_a"),
                          _flag(transpose_b, "transpose_b"), *(_pointer(d) for d in descs))
    return _submit(queue, operators, "pr_matmul_f32", record)


def bias_activation_into(queue, operators, x, bias, out, *, activation=Activation.NONE):
    """out = act(x + bias[column]); bias may be None."""
    xd, od = x._native(), out._native()
    bd = bias._native() if bias is not None else None
    record = BiasActivationRecord(_c.sizeof(BiasActivationRecord), TENSOR_VERSION_1,
                                  int(Activation(activation)), 0, _pointer(xd),
                                  _pointer(bd) if bd is not None else None, _pointer(od))
    return _submit(queue, operators, "pr_bias_activation_f32", record)


def batched_matmul_into(queue, operators, a, b, c, *, batch, m, n, k):
    """C[z] = A[z] B[z] for rank-3 (possibly strided) descriptors [batch,m,k] x [batch,k,n]."""
    descs = [x._native() for x in (a, b, c)]
    record = BatchedMatmulRecord(_c.sizeof(BatchedMatmulRecord), TENSOR_VERSION_1,
                                 *(_int(v, 0, (1 << 64) - 1, label) for v, label in
                                   ((batch, "batch"), (m, "m"), (n, "n"), (k, "k"))),
                                 *(_pointer(d) for d in descs))
    return _submit(queue, operators, "pr_batched_matmul_f32", record)


def reduce_rows_into(queue, operators, x, out, *, op=Reduce.SUM):
    """out[i] = sum or max of row i of x [rows, columns] in the fixed 256-lane order."""
    xd, od = x._native(), out._native()
    record = ReduceRowsRecord(_c.sizeof(ReduceRowsRecord), TENSOR_VERSION_1, int(Reduce(op)), 0,
                              _pointer(xd), _pointer(od))
    return _submit(queue, operators, "pr_reduce_rows_f32", record)


def softmax_rows_into(queue, operators, x, out, *, scale=1.0, causal=False):
    """Row softmax of scale*x over the last dimension of a rank-2 or rank-3 descriptor."""
    xd, od = x._native(), out._native()
    record = SoftmaxRowsRecord(_c.sizeof(SoftmaxRowsRecord), TENSOR_VERSION_1, _flag(causal, "causal"),
                               _real(scale, "scale"), _pointer(xd), _pointer(od))
    return _submit(queue, operators, "pr_softmax_rows_f32", record)


def layer_norm_into(queue, operators, x, gamma, beta, out, *, epsilon=1e-5):
    """LayerNorm over the last dimension of x [rows, columns] with gamma/beta [columns]."""
    descs = [d._native() for d in (x, gamma, beta, out)]
    record = LayerNormRecord(_c.sizeof(LayerNormRecord), TENSOR_VERSION_1, _real(epsilon, "epsilon"), 0,
                             *(_pointer(d) for d in descs))
    return _submit(queue, operators, "pr_layer_norm_f32", record)


def add_into(queue, operators, x, y, out):
    """Elementwise out = x + y for equal-shape contiguous descriptors."""
    descs = [d._native() for d in (x, y, out)]
    record = AddRecord(_c.sizeof(AddRecord), TENSOR_VERSION_1, *(_pointer(d) for d in descs))
    return _submit(queue, operators, "pr_add_f32", record)


class _Operators:
    def __init__(self, context):
        with ExitStack() as acquired:
            self.module = acquired.enter_context(load_tensor_operators(context))
            self.queue = acquired.enter_context(context.queue())
            self._owners = acquired.pop_all()

    def close(self):
        self._owners.close()


def operators_of(context):
    """The context's cached (provider module, queue) pair."""
    context.handle
    resources = getattr(context, "_tensor_resources", None)
    if resources is None:
        resources = _Operators(context)
        context._tensor_resources = resources
    return resources


class Tensor:
    """Owned contiguous row-major FP32 tensor on one Context."""

    def __init__(self, *_, **__):
        raise TypeError("Use paralyn_b200.tensor(...) or tensor operators to create a Tensor")

    @classmethod
    def _adopt(cls, context, buffer, shape, event=None, device=None):
        value = cls.__new__(cls)
        value._context, value._buffer, value._event = context, buffer, event
        value._shape, value._closed = shape, False
        value._device = context.device if device is None else device
        return value

    def _open(self):
        if self.closed:
            raise Error(Status.INVALID_HANDLE, "Tensor", "tensor is closed")

    @property
    def closed(self):
        return getattr(self, "_closed", True)

    @property
    def shape(self):
        return self._shape

    @property
    def ndim(self):
        return len(self._shape)

    @property
    def size(self):
        count = 1
        for d in self._shape:
            count *= d
        return count

    @property
    def dtype(self):
        return float32

    @property
    def nbytes(self):
        return self.size * 4

    @property
    def device(self):
        return self._device

    @property
    def buffer(self):
        return self._buffer

    def descriptor(self):
        self._open()
        return TensorDescriptor(self._buffer, self._shape)

    def wait(self):
        self._open()
        return self._event.wait() if self._event is not None else None

    def timing(self):
        self._open()
        return self._event.timing() if self._event is not None else None

    def to_host(self):
        """Flat row-major array('f') copy."""
        self.wait()
        result = _host_array("f")
        result.frombytes(self._buffer.read())
        return result

    def close(self):
        if self.closed:
            return
        self._closed = True
        failure = None
        if self._event is not None:
            try:
                self._event.close()
            except Exception as error:
                failure = error
        try:
            self._buffer.close()
        except Exception as error:
            failure = failure or error
        if failure is not None:
            raise failure

    def __enter__(self):
        self._open()
        return self

    def __exit__(self, *_):
        self.close()

    def __del__(self, _write=os.write, _exit=os._exit):
        if not self.closed:
            try:
                self.close()
            except Exception as error:
                try:
                    _write(2, f"Paralyn fatal unhandled Tensor finalizer error: {error}\n".encode())
                finally:
                    _exit(1)


def tensor(values, *, shape, context, dtype=float32):
    """Copy flat row-major values (sequence, or native FP32 C-contiguous buffer)."""
    if not isinstance(context, Context):
        raise TypeError("tensor requires an explicit Context")
    context.handle
    if dtype != float32:
        raise ValueError("only explicit dtype=paralyn_b200.float32 is supported")
    shape, count = _shape(shape)
    if isinstance(values, (list, tuple)):
        data = memoryview(_host_array("f", (f32(v).value for v in values)))
    else:
        data = memoryview(values)
        if not data.c_contiguous:
            raise ValueError("tensor requires a C-contiguous host buffer")
        if data.itemsize != 4 or data.format not in ("f", "@f", "=f", "<f"):
            raise TypeError("buffer input must already contain native-endian FP32 values")
    if data.nbytes != count * 4:
        raise ValueError("value count must equal the product of the shape")
    buffer = context.buffer(count * 4)
    try:
        buffer.write(data)
        return Tensor._adopt(context, buffer, shape)
    except BaseException:
        buffer.close()
        raise


def _same_context(*tensors):
    for value in tensors:
        if not isinstance(value, Tensor):
            raise TypeError("tensor operators require Paralyn Tensors")
        value._open()
    context = tensors[0]._context
    if any(value._context is not context for value in tensors):
        raise Error(Status.CONTEXT_MISMATCH, "tensor operation", "inputs belong to different contexts")
    context.handle
    return context


def _output(context, shape, device, enqueue):
    buffer = context.buffer(4 * _shape(shape)[1])
    event = None
    try:
        event = enqueue(TensorDescriptor(buffer, shape))
        return Tensor._adopt(context, buffer, shape, event, device)
    except BaseException:
        try:
            if event is not None:
                event.close()
        finally:
            buffer.close()
        raise


def matmul(a, b, *, transpose_a=False, transpose_b=False):
    """C = op(A) op(B) on the GPU with FP32 accumulation in increasing k."""
    context = _same_context(a, b)
    if a.ndim != 2 or b.ndim != 2:
        raise ValueError("matmul requires rank-2 tensors")
    _flag(transpose_a, "transpose_a")
    _flag(transpose_b, "transpose_b")
    m, k = (a.shape[1], a.shape[0]) if transpose_a else a.shape
    kb, n = (b.shape[1], b.shape[0]) if transpose_b else b.shape
    if k != kb:
        raise ValueError(f"matmul inner dimensions differ ({k} != {kb})")
    r = operators_of(context)
    return _output(context, (m, n), a.device, lambda c: matmul_into(
        r.queue, r.module, a.descriptor(), b.descriptor(), c, m=m, n=n, k=k,
        transpose_a=transpose_a, transpose_b=transpose_b))


def _bias_activation(x, bias, activation):
    context = _same_context(x, *(() if bias is None else (bias,)))
    r = operators_of(context)
    return _output(context, x.shape, x.device, lambda out: bias_activation_into(
        r.queue, r.module, x.descriptor(), None if bias is None else bias.descriptor(), out,
        activation=activation))


def bias_add(x, bias, *, relu=False):
    """out[i, j] = x[i, j] + bias[j], optionally followed by ReLU."""
    if not isinstance(relu, bool):
        raise TypeError("relu must be a bool")
    return _bias_activation(x, bias, Activation.RELU if relu else Activation.NONE)


def relu(x):
    return _bias_activation(x, None, Activation.RELU)


def gelu(x):
    return _bias_activation(x, None, Activation.GELU_TANH)


def bias_gelu(x, bias):
    return _bias_activation(x, bias, Activation.GELU_TANH)


def batched_matmul(a, b):
    """C[i] = A[i] B[i] for contiguous rank-3 tensors [batch,m,k] x [batch,k,n]."""
    context = _same_context(a, b)
    if a.ndim != 3 or b.ndim != 3:
        raise ValueError("batched_matmul requires rank-3 tensors")
    batch, m, k = a.shape
    if b.shape[0] != batch or b.shape[1] != k:
        raise ValueError(f"batched_matmul shapes differ: {a.shape} x {b.shape}")
    n = b.shape[2]
    resources = operators_of(context)
    return _output(context, (batch, m, n), a.device, lambda c: batched_matmul_into(
        resources.queue, resources.module, a.descriptor(), b.descriptor(), c, batch=batch, m=m, n=n, k=k))


def _reduce(x, op):
    context = _same_context(x)
    if x.ndim != 2:
        raise ValueError("row reductions require rank-2 tensors")
    resources = operators_of(context)
    return _output(context, (x.shape[0],), x.device, lambda out: reduce_rows_into(
        resources.queue, resources.module, x.descriptor(), out, op=op))


def row_sum(x):
    """Row sums of a rank-2 tensor in the fixed 256-lane order."""
    return _reduce(x, Reduce.SUM)


def row_max(x):
    """Row maxima (NaN-propagating, +0.0 preferred over -0.0, -inf for empty rows)."""
    return _reduce(x, Reduce.MAX)


def softmax(x, *, scale=1.0, causal=False):
    """Numerically stable row softmax of scale*x over the last dimension."""
    context = _same_context(x)
    resources = operators_of(context)
    return _output(context, x.shape, x.device, lambda out: softmax_rows_into(
        resources.queue, resources.module, x.descriptor(), out, scale=scale, causal=causal))


def layer_norm(x, gamma, beta, *, epsilon=1e-5):
    """LayerNorm over the last dimension of a rank-2 tensor."""
    context = _same_context(x, gamma, beta)
    r = operators_of(context)
    return _output(context, x.shape, x.device, lambda out: layer_norm_into(
        r.queue, r.module, x.descriptor(), gamma.descriptor(), beta.descriptor(), out, epsilon=epsilon))


def residual_add(x, y):
    """Elementwise x + y of equal-shape tensors."""
    context = _same_context(x, y)
    r = operators_of(context)
    return _output(context, x.shape, x.device, lambda out: add_into(
        r.queue, r.module, x.descriptor(), y.descriptor(), out))
