"""Owned one-dimensional FP32 arrays and the array operators.

Mirrors the reference's array API (bindings/python/paralyn/array.py): asarray,
Array (shape/size/nbytes/wait/to_host/close), add and affine, launched through
pr_launch from the verified-IR operators module (array_add / array_affine, grid
ceil(n/256) x 256) on the context's queue. affine_scalar(a, scale, bias) is an
addition of this library: the affine map with a scalar addend, from the same
module. Sequence input is rounded to binary32 and copied; buffer input must be
native FP32 and C-contiguous; there is no broadcasting and no CPU fallback.
"""
from array import array as _host_array
from contextlib import ExitStack
import os
from pathlib import Path

from .native import Access, Context, Error, Module, Status, _int, f32, u32

float32 = "float32"
_MAX_ELEMENTS = (1 << 31) - 1
DEFAULT_OPERATORS = Path(__file__).resolve().parent / "data" / "operators.prk"


def operators_path():
    override = os.environ.get("PARALYN_OPERATORS")
    path = Path(override).resolve() if override else DEFAULT_OPERATORS
    if not path.is_file():
        raise FileNotFoundError("The array operator module is missing; run `python -m "
                                "paralyn_b200.build` or set PARALYN_OPERATORS to operators.prk")
    return path


class _Operators:
    def __init__(self, context):
        with ExitStack() as acquired:
            self.module = acquired.enter_context(Module.load_file(context, operators_path()))
            self.add = acquired.enter_context(self.module.kernel("array_add"))
            self.affine = acquired.enter_context(self.module.kernel("array_affine"))
            try:
                self.affine_scalar = acquired.enter_context(self.module.kernel("array_affine_scalar"))
            except Error:
                self.affine_scalar = None  # a reference-built module has only add/affine
            self.queue = acquired.enter_context(context.queue())
            self._owners = acquired.pop_all()

    def close(self):
        self._owners.close()


def _operators(context):
    context.handle
    resources = getattr(context, "_array_resources", None)
    if resources is None:
        resources = _Operators(context)
        context._array_resources = resources
    return resources


def _shape(shape, size):
    _int(size, 0, _MAX_ELEMENTS, "array length")
    if shape is None:
        return (size,)
    if not isinstance(shape, (tuple, list)) or len(shape) != 1:
        raise ValueError("only one-dimensional shape=(length,) is supported")
    length = _int(shape[0], 0, _MAX_ELEMENTS, "shape length")
    if length != size:
        raise ValueError("shape length must equal the number of input FP32 values")
    return (length,)


class Array:
    def __init__(self, *_, **__):
        raise TypeError("Use asarray with an explicit Context, or add/affine to create an Array")

    @classmethod
    def _adopt(cls, context, buffer, shape, event=None, device=None):
        value = cls.__new__(cls)
        value._context, value._buffer, value._event = context, buffer, event
        value._shape, value._closed = shape, False
        value._device = context.device if device is None else device
        return value

    def _open(self):
        if self.closed:
            raise Error(Status.INVALID_HANDLE, "Array", "array is closed")

    @property
    def closed(self):
        return getattr(self, "_closed", True)

    @property
    def shape(self):
        return self._shape

    @property
    def size(self):
        return self._shape[0]

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

    def wait(self):
        self._open()
        return self._event.wait() if self._event is not None else None

    def to_host(self):
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
                    _write(2, f"Paralyn fatal unhandled Array finalizer error: {error}\n".encode())
                finally:
                    _exit(1)


def asarray(values, *, context, dtype=float32, shape=None):
    """Copy host FP32 values into a new device array on `context`."""
    if not isinstance(context, Context):
        raise TypeError("asarray requires an explicit Context")
    context.handle
    if dtype != float32:
        raise ValueError("only explicit dtype=paralyn_b200.float32 is supported")
    if isinstance(values, (list, tuple)):
        _int(len(values), 0, _MAX_ELEMENTS, "array length")
        host = _host_array("f", (f32(v).value for v in values))
        data, count = memoryview(host), len(host)
    else:
        data = memoryview(values)
        if not data.c_contiguous or data.ndim != 1:
            raise ValueError("asarray requires a one-dimensional C-contiguous host buffer")
        if data.itemsize != 4 or data.format not in ("f", "@f", "=f", "<f"):
            raise TypeError("buffer input must already contain native-endian FP32 values")
        count = data.nbytes // 4
    actual = _shape(shape, count)
    buffer = context.buffer(count * 4)
    try:
        buffer.write(data)
        return Array._adopt(context, buffer, actual)
    except BaseException:
        buffer.close()
        raise


def _launch(a, inputs, kernel_of, scalars):
    context = a._context
    context.handle
    if a.size == 0:  # an empty result owns a zero-byte buffer and no GPU event
        return Array._adopt(context, context.buffer(0), a.shape, device=a.device)
    resources = _operators(context)
    kernel = kernel_of(resources)
    buffer = context.buffer(a.nbytes)
    event = None
    try:
        with ExitStack() as views:
            arguments = [views.enter_context(x._buffer.view(access=Access.READ)) for x in inputs]
            arguments.append(views.enter_context(buffer.view(access=Access.WRITE)))
            arguments += [u32(a.size), *scalars]
            event = resources.queue.launch(kernel, arguments, grid=((a.size + 255) // 256, 1, 1),
                                           block=(256, 1, 1))
        return Array._adopt(context, buffer, a.shape, event, a.device)
    except BaseException:
        try:
            if event is not None:
                event.close()
        finally:
            buffer.close()
        raise


def _pair(a, b):
    if not isinstance(a, Array) or not isinstance(b, Array):
        raise TypeError("array operators require two Paralyn Arrays")
    a._open()
    b._open()
    if a._context is not b._context:
        raise Error(Status.CONTEXT_MISMATCH, "array operation", "inputs belong to different contexts")
    if a.shape != b.shape:
        raise ValueError("array shapes must match exactly; broadcasting is unsupported")


def add(a, b):
    """Allocate and enqueue elementwise FP32 a + b (one rounding)."""
    _pair(a, b)
    return _launch(a, (a, b), lambda r: r.add, ())


def affine(a, b, scale):
    """Allocate and enqueue FP32 a*scale + b, rounded after the product and the sum."""
    _pair(a, b)
    return _launch(a, (a, b), lambda r: r.affine, (f32(scale),))


def affine_scalar(a, scale, bias):
    """Allocate and enqueue FP32 a*scale + bias with a scalar bias (8 bytes/element)."""
    if not isinstance(a, Array):
        raise TypeError("affine_scalar requires a Paralyn Array")
    a._open()

    def kernel(resources):
        if resources.affine_scalar is None:
            raise Error(Status.UNSUPPORTED, "affine_scalar",
                        "the loaded operators module has no array_affine_scalar kernel")
        return resources.affine_scalar
    return _launch(a, (a,), kernel, (f32(scale), f32(bias)))
