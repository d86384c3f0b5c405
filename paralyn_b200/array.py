"""One-dimensional FP32 arrays and the array operators add / affine.

The functions have the reference binding's names and meaning (package `paralyn`:
asarray, Array, add, affine): an Array is a device buffer of n FP32 values on one
context, and add / affine allocate the result and enqueue one launch of the
verified-IR operators module (array_add / array_affine: grid ceil(n/256) blocks of
256 threads, u32 element count) on the context's queue through pr_launch.
affine_scalar(a, scale, bias) is this library's addition: the affine map with a
scalar addend (8 bytes per element instead of 12), from the same module. List input
is rounded to binary32; buffer input must already be native FP32 and C-contiguous.
Shapes must match exactly (no broadcasting); there is no CPU fallback.
"""
from contextlib import ExitStack
import os
from pathlib import Path

from .native import Access, Error, Module, Status, _int, f32, u32
from .values import MAX_ELEMENTS, DeviceValue, common_context, float32, host_fp32, produce, upload

DEFAULT_OPERATORS = Path(__file__).resolve().parent / "data" / "operators.prk"


def operators_path():
    """PARALYN_OPERATORS, else the module paralyn_b200.build writes in-tree."""
    chosen = Path(os.environ.get("PARALYN_OPERATORS") or DEFAULT_OPERATORS).resolve()
    if not chosen.is_file():
        raise FileNotFoundError(f"no array operators module at {chosen}: run `python -m paralyn_b200.build` "
                                "or point PARALYN_OPERATORS at operators.prk")
    return chosen


class _ArrayKernels:
    """The operators module of one context, its kernels and the context's queue."""

    def __init__(self, context):
        with ExitStack() as held:
            module = held.enter_context(Module.load_file(context, operators_path()))
            self.kernels = {name: held.enter_context(module.kernel(name)) for name in ("array_add", "array_affine")}
            try:  # a module built by the reference's compiler has no scalar-addend kernel
                self.kernels["array_affine_scalar"] = held.enter_context(module.kernel("array_affine_scalar"))
            except Error:
                pass
            self.queue = held.enter_context(context.queue())
            self._held = held.pop_all()

    def close(self):
        self._held.close()


class Array(DeviceValue):
    """n FP32 values on one context (shape (n,))."""
    _kind = "Array"


def asarray(values, *, context, dtype=float32, shape=None):
    """A new Array on `context` holding a copy of the host values."""
    if dtype != float32:
        raise ValueError("asarray stores float32 only (pass dtype=paralyn_b200.float32)")
    data = host_fp32(values, "asarray")
    if data.ndim != 1:
        raise ValueError("asarray takes one-dimensional host data")
    count = _int(data.nbytes // 4, 0, MAX_ELEMENTS, "array length")
    if shape is not None:
        if not isinstance(shape, (tuple, list)) or len(shape) != 1:
            raise ValueError("an Array's shape is (length,)")
        if _int(shape[0], 0, MAX_ELEMENTS, "shape length") != count:
            raise ValueError(f"shape {tuple(shape)} does not hold the {count} values given")
    return upload(Array, context, data, (count,))


def _elementwise(kernel_name, inputs, scalars):
    """One launch of `kernel_name` over the first input's n elements into a new Array."""
    first = inputs[0]
    context = first._context
    n = first.size
    if n == 0:  # nothing to compute: an empty Array with a zero-byte buffer, no event
        return Array._adopt(context, context.buffer(0), first.shape, device=first.device)
    kernels = context.attached("array_kernels", _ArrayKernels)
    if kernel_name not in kernels.kernels:
        raise Error(Status.UNSUPPORTED, kernel_name, "the loaded operators module lacks this kernel")

    def enqueue(out):
        with ExitStack() as views:
            bound = [views.enter_context(x._buffer.view(access=Access.READ)) for x in inputs]
            bound.append(views.enter_context(out.view(access=Access.WRITE)))
            return kernels.queue.launch(kernels.kernels[kernel_name], bound + [u32(n), *scalars],
                                        grid=((n + 255) // 256, 1, 1), block=(256, 1, 1))
    return produce(Array, context, first.shape, 4 * n, first.device, enqueue)


def _same_shape(a, b, what):
    common_context((a, b), Array, what)
    if a.shape != b.shape:
        raise ValueError(f"{what}: shapes {a.shape} and {b.shape} differ (no broadcasting)")


def add(a, b):
    """A new Array with a[i] + b[i] (one FP32 rounding)."""
    _same_shape(a, b, "add")
    return _elementwise("array_add", (a, b), ())


def affine(a, b, scale):
    """A new Array with fl(fl(a[i] * scale) + b[i]) (no fused multiply-add)."""
    _same_shape(a, b, "affine")
    return _elementwise("array_affine", (a, b), (f32(scale),))


def affine_scalar(a, scale, bias):
    """A new Array with fl(fl(a[i] * scale) + bias), the addend a scalar."""
    common_context((a,), Array, "affine_scalar")
    return _elementwise("array_affine_scalar", (a,), (f32(scale), f32(bias)))
