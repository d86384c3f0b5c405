"""Bindings of the additive B200 entry points (include/paralyn/b200.h)."""
import ctypes as _c
from enum import IntEnum

from .native import Context, Event, Queue
from .tensor import TensorDescRecord, _api, _pointer

UNIFORM, NORMAL = 0, 1


class MatmulMode(IntEnum):
    AUTO = 0
    REFERENCE = 1
    FFMA = 2
    TF32X3 = 3


_B200_CALLS = """
pr_b200_matmul_mode_set h u32
pr_b200_matmul_mode_get h *u32
pr_b200_device_kernel_count h *u64
pr_b200_module_inspect ptr u64 str u64
pr_b200_buffer_export h ptr
pr_b200_buffer_import h ptr *h
pr_b200_layer_norm_gather_f32 h h ptr ptr u32 u64 *h
pr_b200_gather_rows_f32 h ptr ptr u32 u64 *h
pr_b200_buffer_write_async h h u64 ptr u64 *h
pr_b200_buffer_read_async h h u64 ptr u64 *h
pr_b200_host_register ptr u64
pr_b200_host_unregister ptr
pr_b200_marker h *h
pr_b200_selftest_bounded_wait h u64 *h
pr_b200_queue_hold h u64 *h
pr_b200_matmul_bias_activation_f32 h h ptr ptr u32 *h
pr_b200_matmul_prepare_f32 h h ptr u32 ptr *h
pr_b200_matmul_prepared_f32 h h ptr *h
pr_b200_matmul_prepared_bias_activation_f32 h h ptr ptr u32 *h
pr_b200_event_elapsed h h *f64
pr_b200_fill_synthetic_f32 h *TensorDescRecord u64 u64 u32 f32 f32 *h
"""


def _b200(lib):
    """`lib` with the tensor and the additive B200 entry points declared."""
    lib = _api(lib)
    if not lib.declares("pr_b200_marker"):
        lib.declare(_B200_CALLS)
        sizing = lib.api.pr_b200_matmul_prepared_bytes  # returns a size, not a status
        sizing.restype, sizing.argtypes = _c.c_uint64, [_c.c_uint64, _c.c_uint64]
    return lib


def set_matmul_mode(context, mode):
    lib = _b200(context._lib)
    lib.check(lib.api.pr_b200_matmul_mode_set(context.handle, int(MatmulMode(mode))))


def matmul_mode(context):
    lib = _b200(context._lib)
    value = _c.c_uint32()
    lib.check(lib.api.pr_b200_matmul_mode_get(context.handle, _c.byref(value)))
    return MatmulMode(value.value)


def device_kernel_count(context):
    """Device kernels the context has completed (waits for its queue)."""
    lib = _b200(context._lib)
    value = _c.c_uint64()
    lib.check(lib.api.pr_b200_device_kernel_count(context.handle, _c.byref(value)))
    return value.value


def fill_synthetic_into(queue, descriptor, *, seed, first_draw=0, distribution=UNIFORM, p0=1.0, p1=0.0):
    """Fill a contiguous tensor with the seeded stream (see paralyn_b200.synthetic)."""
    if not isinstance(queue, Queue):
        raise TypeError("fill_synthetic_into requires a Queue")
    lib = _b200(queue._lib)
    record = descriptor._native()
    handle = _c.c_uint64()
    lib.check(lib.api.pr_b200_fill_synthetic_f32(queue.handle, _c.byref(record), seed, first_draw,
                                                 distribution, p0, p1, _c.byref(handle)))
    return Event._adopt(lib, handle.value) if handle.value else None


PEER_HANDLE_BYTES = 72


def export_buffer(buffer):
    """Bytes another process passes to import_buffer to map this buffer (same node)."""
    lib = _b200(buffer._lib)
    out = _c.create_string_buffer(PEER_HANDLE_BYTES)
    lib.check(lib.api.pr_b200_buffer_export(buffer.handle, out))
    return out.raw


def import_buffer(context, handle):
    """A Buffer of `context` that refers to a peer process's exported buffer."""
    from .native import Buffer
    lib = _b200(context._lib)
    data = _c.create_string_buffer(bytes(handle), PEER_HANDLE_BYTES)
    result = _c.c_uint64()
    lib.check(lib.api.pr_b200_buffer_import(context.handle, data, _c.byref(result)))
    return Buffer._adopt(lib, result.value)


def layer_norm_gather_into(queue, operators, x, gamma, beta, out, gathered, *, row_offset, epsilon=1e-5):
    """LayerNorm of x's rows into `out`, each output row also written at row
    row_offset + i of every descriptor in `gathered` (local or imported)."""
    from .tensor import LayerNormRecord, TENSOR_VERSION_1
    lib = _b200(queue._lib)
    descs = [d._native() for d in (x, gamma, beta, out)]
    record = LayerNormRecord(_c.sizeof(LayerNormRecord), TENSOR_VERSION_1, float(epsilon), 0,
                             *(_pointer(d) for d in descs))
    natives = [g._native() for g in gathered]
    array = (_c.POINTER(TensorDescRecord) * max(1, len(natives)))(*(_pointer(d) for d in natives))
    handle = _c.c_uint64()
    lib.check(lib.api.pr_b200_layer_norm_gather_f32(queue.handle, operators.handle, _c.byref(record), array,
                                                    len(natives), row_offset, _c.byref(handle)))
    return Event._adopt(lib, handle.value) if handle.value else None


def gather_rows_into(queue, local, gathered, *, row_offset):
    """Write the rows of `local` (a [rows, columns] descriptor) at row row_offset + i of
    every descriptor in `gathered` (local or imported); returns the Event or None."""
    lib = _b200(queue._lib)
    source = local._native()
    natives = [g._native() for g in gathered]
    array = (_c.POINTER(TensorDescRecord) * max(1, len(natives)))(*(_pointer(d) for d in natives))
    handle = _c.c_uint64()
    lib.check(lib.api.pr_b200_gather_rows_f32(queue.handle, _c.byref(source), array, len(natives), row_offset,
                                              _c.byref(handle)))
    return Event._adopt(lib, handle.value) if handle.value else None


def _host_range(host, nbytes):
    """(address, bytes) of a numpy array, a ctypes object or a raw address + size."""
    if isinstance(host, int):
        if nbytes is None:
            raise ValueError("a raw host address needs nbytes")
        return host, int(nbytes)
    if hasattr(host, "__array_interface__"):
        import numpy as np
        array = np.asarray(host)
        if not array.flags.c_contiguous:
            raise ValueError("host array must be C-contiguous")
        return array.__array_interface__["data"][0], array.nbytes if nbytes is None else int(nbytes)
    return _c.addressof(host), _c.sizeof(host) if nbytes is None else int(nbytes)


def write_async(queue, buffer, source, *, offset=0, nbytes=None):
    """Stream-ordered copy of host memory into buffer[offset:offset+nbytes]; returns
    its Event (None for zero bytes). `source` must stay valid until the event completes."""
    lib = _b200(queue._lib)
    address, size = _host_range(source, nbytes)
    handle = _c.c_uint64()
    lib.check(lib.api.pr_b200_buffer_write_async(queue.handle, buffer.handle, offset, address, size,
                                                 _c.byref(handle)))
    if not handle.value:
        return None
    event = Event._adopt(lib, handle.value)
    event.host = source  # kept alive with the event
    return event


def read_async(queue, buffer, destination, *, offset=0, nbytes=None):
    """Stream-ordered copy of buffer[offset:offset+nbytes] into host memory."""
    lib = _b200(queue._lib)
    address, size = _host_range(destination, nbytes)
    handle = _c.c_uint64()
    lib.check(lib.api.pr_b200_buffer_read_async(queue.handle, buffer.handle, offset, address, size,
                                                _c.byref(handle)))
    if not handle.value:
        return None
    event = Event._adopt(lib, handle.value)
    event.host = destination
    return event


def host_register(host, nbytes=None, library_path=None):
    """Page-lock a host range (numpy array or address + nbytes) so copies overlap."""
    from .native import library
    lib = _b200(library(library_path))
    address, size = _host_range(host, nbytes)
    lib.check(lib.api.pr_b200_host_register(address, size))


def host_unregister(host, library_path=None):
    from .native import library
    lib = _b200(library(library_path))
    address, _ = _host_range(host, 0 if isinstance(host, int) else None)
    lib.check(lib.api.pr_b200_host_unregister(address))


def matmul_bias_activation_into(queue, operators, a, b, c, bias, *, m, n, k, transpose_a=False, transpose_b=False,
                                activation=0):
    """C = activation(op(A) op(B) + bias[column]) as one command (bias may be None);
    equal to matmul_into followed by bias_activation_into, bit for bit."""
    from .tensor import MatmulRecord, TENSOR_VERSION_1, Activation
    lib = _b200(queue._lib)
    descs = [x._native() for x in (a, b, c)]
    record = MatmulRecord(_c.sizeof(MatmulRecord), TENSOR_VERSION_1, m, n, k, int(bool(transpose_a)),
                          int(bool(transpose_b)), *(_pointer(d) for d in descs))
    bias_native = bias._native() if bias is not None else None
    handle = _c.c_uint64()
    lib.check(lib.api.pr_b200_matmul_bias_activation_f32(
        queue.handle, operators.handle, _c.byref(record),
        _c.byref(bias_native) if bias_native is not None else None, int(Activation(activation)), _c.byref(handle)))
    return Event._adopt(lib, handle.value) if handle.value else None


def matmul_prepared_bytes(lib, k, n):
    """Bytes of B's prepared form for a [k, n] B (0: k or n is 0 or above INT32_MAX)."""
    return int(_b200(lib).api.pr_b200_matmul_prepared_bytes(int(k), int(n)))


def matmul_prepare_into(queue, operators, b, prepared, *, transpose_b=False):
    """Enqueue B ([k, n], or [n, k] with transpose_b) into its prepared form in the
    1-D descriptor `prepared`; returns the Event."""
    lib = _b200(queue._lib)
    source, target = b._native(), prepared._native()
    handle = _c.c_uint64()
    lib.check(lib.api.pr_b200_matmul_prepare_f32(queue.handle, operators.handle, _c.byref(source),
                                                 int(bool(transpose_b)), _c.byref(target), _c.byref(handle)))
    return Event._adopt(lib, handle.value) if handle.value else None


def matmul_prepared_into(queue, operators, a, prepared, c, *, m, n, k, transpose_a=False):
    """C = op(A) B from B's prepared form (equal to matmul_into with that B, bit for
    bit in every matmul mode); returns the Event or None."""
    from .tensor import MatmulRecord, TENSOR_VERSION_1
    lib = _b200(queue._lib)
    descs = [x._native() for x in (a, prepared, c)]
    record = MatmulRecord(_c.sizeof(MatmulRecord), TENSOR_VERSION_1, m, n, k, int(bool(transpose_a)), 0,
                          *(_pointer(d) for d in descs))
    handle = _c.c_uint64()
    lib.check(lib.api.pr_b200_matmul_prepared_f32(queue.handle, operators.handle, _c.byref(record),
                                                  _c.byref(handle)))
    return Event._adopt(lib, handle.value) if handle.value else None


def matmul_prepared_bias_activation_into(queue, operators, a, prepared, c, bias, *, m, n, k, transpose_a=False,
                                         activation=0):
    """C = activation(op(A) B + bias[column]) from B's prepared form (bias may be
    None); equal to matmul_bias_activation_into with that B, bit for bit."""
    from .tensor import MatmulRecord, TENSOR_VERSION_1, Activation
    lib = _b200(queue._lib)
    descs = [x._native() for x in (a, prepared, c)]
    record = MatmulRecord(_c.sizeof(MatmulRecord), TENSOR_VERSION_1, m, n, k, int(bool(transpose_a)), 0,
                          *(_pointer(d) for d in descs))
    bias_native = bias._native() if bias is not None else None
    handle = _c.c_uint64()
    lib.check(lib.api.pr_b200_matmul_prepared_bias_activation_f32(
        queue.handle, operators.handle, _c.byref(record),
        _c.byref(bias_native) if bias_native is not None else None, int(Activation(activation)), _c.byref(handle)))
    return Event._adopt(lib, handle.value) if handle.value else None


class PreparedMatrix:
    """A right-hand matmul operand B prepared once for many products, in a buffer of
    its own (see pr_b200_matmul_prepare_f32). `descriptor` is what
    matmul_prepared_into takes; later changes to B do not reach it."""

    def __init__(self, queue, operators, context, b, *, k, n, transpose_b=False):
        from .tensor import TensorDescriptor
        self.k, self.n = int(k), int(n)
        size = matmul_prepared_bytes(queue._lib, self.k, self.n)
        if not size:
            raise ValueError("a prepared operand needs 1 <= k, n <= INT32_MAX")
        self.buffer = context.buffer(size)
        self.descriptor = TensorDescriptor(self.buffer, (size // 4,))
        try:
            event = matmul_prepare_into(queue, operators, b, self.descriptor, transpose_b=transpose_b)
            event.wait()
            event.close()
        except BaseException:
            self.buffer.close()
            raise

    def close(self):
        self.buffer.close()


def selftest_bounded_wait(queue, cycles):
    """Enqueue the bounded-wait probe (a wait that gives up after `cycles` SM cycles);
    waiting on the returned event raises the command's failure."""
    lib = _b200(queue._lib)
    handle = _c.c_uint64()
    lib.check(lib.api.pr_b200_selftest_bounded_wait(queue.handle, int(cycles), _c.byref(handle)))
    return Event._adopt(lib, handle.value)


def queue_hold(queue, seconds):
    """A command that keeps the queue's later device work waiting for `seconds` (at
    most 1) and then completes; returns its Event."""
    lib = _b200(queue._lib)
    handle = _c.c_uint64()
    lib.check(lib.api.pr_b200_queue_hold(queue.handle, int(round(seconds * 1e9)), _c.byref(handle)))
    return Event._adopt(lib, handle.value)


def marker(queue):
    """An empty command on the queue that records a device timestamp."""
    lib = _b200(queue._lib)
    handle = _c.c_uint64()
    lib.check(lib.api.pr_b200_marker(queue.handle, _c.byref(handle)))
    return Event._adopt(lib, handle.value)


def elapsed(first, second):
    """Device seconds between the completion of two markers of one context."""
    lib = _b200(first._lib)
    seconds = _c.c_double()
    lib.check(lib.api.pr_b200_event_elapsed(first.handle, second.handle, _c.byref(seconds)))
    return seconds.value


def last_variant(context, entry):
    """The implementation the library chose for the newest launch of provider entry
    `entry` on this context (from its evidence log), or None when there is none."""
    import json
    import shutil
    import tempfile
    from pathlib import Path
    root = Path(tempfile.mkdtemp(prefix="paralyn_evidence_"))
    try:
        context.write_evidence(str(root / "e"))
        launches = json.loads((root / "e" / "execution.json").read_text())["launches"]
    finally:
        shutil.rmtree(root, ignore_errors=True)
    for launch in reversed(launches):
        if launch["kernel"] == entry:
            return launch["variant"]
    return None


def inspect_module(data, library_path=None):
    """{kernel name: native implementation} for a module artifact, without a device."""
    from .native import library
    lib = _b200(library(library_path))
    data = bytes(data)
    report = _c.create_string_buffer(1 << 16)
    storage = _c.create_string_buffer(data, len(data)) if data else None
    lib.check(lib.api.pr_b200_module_inspect(storage, len(data), report, len(report)))
    pairs = [item.split("=", 1) for item in report.value.decode().split(";") if item]
    return dict(pairs)
