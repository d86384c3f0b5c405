"""ctypes binding of the native C ABI (include/paralyn/native.h).

The Python surface has the reference binding's names and meaning (package
`paralyn`: Context, Buffer, View, Module, Kernel, Queue, Event, i32/u32/f32,
Status, Error), so code written against it runs here. The implementation is this
package's own: the C records are declared from compact layout strings, every entry
point is typed from one signature table (`_CALLS`, shared with tensor.py and
b200.py), and every owned handle is released by `close()`, a `with` block, or a
garbage-collection finalizer; a release that fails inside a finalizer ends the
process, since the failure of GPU work that nobody waited for must not pass
silently. The library is the in-tree libparalyn_native.so built by
paralyn_b200.build, or PARALYN_LIBRARY. There is no CPU fallback: without the
library or a CUDA device every call fails with a structured Error.
"""
import ctypes as _c
from dataclasses import dataclass
from enum import IntEnum
import math
import os
from pathlib import Path
import sys
import weakref

ABI_VERSION = 1
_PACKAGE = Path(__file__).resolve().parent
DEFAULT_LIBRARY = _PACKAGE / "libparalyn_native.so"


# ---------------------------------------------------------------- ABI enumerations
class Status(IntEnum):
    SUCCESS = 0
    INVALID_ARGUMENT = 1
    INVALID_HANDLE = 2
    CONTEXT_MISMATCH = 3
    OUT_OF_BOUNDS = 4
    UNSUPPORTED = 5
    OUT_OF_MEMORY = 6
    COMPILATION_FAILED = 7
    EXECUTION_FAILED = 8
    DEVICE_UNAVAILABLE = 9
    INTERNAL_ERROR = 10


class Access(IntEnum):
    READ = 1
    WRITE = 2
    READ_WRITE = 3


class Type(IntEnum):
    I32 = 1
    U32 = 2
    F32 = 3
    BUFFER = 4


class ClockDomain(IntEnum):
    UNAVAILABLE = 0
    DURATION_ONLY = 1
    METAL_SYSTEM_MACH = 2


ARTIFACT_VERIFIED_IR = 1 << 0
ARTIFACT_MSL_SOURCE = 1 << 1
ARTIFACT_SPIRV_MSL = 1 << 2


class Error(RuntimeError):
    """A native call that did not succeed: `code` (Status), the failing `operation`
    as the library names it, and the library's `message`."""

    def __init__(self, code, operation, message):
        self.code, self.operation, self.message = Status(code), operation, message
        super().__init__(f"{operation} failed with {self.code.name}: {message}")


# ---------------------------------------------------------------- record layouts
# Layout strings list "name:type" fields in declaration order; char[N] is a fixed
# text field, ptr:<Record> a pointer to another record. The layouts are the C
# headers' (the records cross the ABI by address).
_SCALARS = {"u32": _c.c_uint32, "i32": _c.c_int32, "u64": _c.c_uint64, "i64": _c.c_int64,
            "f32": _c.c_float, "f64": _c.c_double, "enum": _c.c_int}


def layout(spec, **records):
    fields = []
    for item in spec.split():
        name, kind = item.split(":", 1)
        count = 1
        if kind.endswith("]"):
            kind, count = kind[:-1].split("[")
            count = int(count)
        if kind == "char":
            ctype = _c.c_char * count
        elif kind.startswith("ptr="):
            ctype = _c.POINTER(records[kind[4:]])
        else:
            ctype = _SCALARS[kind] if count == 1 else _SCALARS[kind] * count
        fields.append((name, ctype))
    return fields


class ErrorRecord(_c.Structure):
    _fields_ = layout("code:enum operation:char[64] message:char[1024]")


class DeviceRecord(_c.Structure):
    _fields_ = layout("name:char[256] backend:char[32] os:char[128] registry_id:u64 max_buffer_bytes:u64 "
                      "unified_memory:u32")


class Dim3(_c.Structure):
    _fields_ = layout("x:u32 y:u32 z:u32")


class ArgumentRecord(_c.Structure):
    _fields_ = layout("type:enum view:u64 i32:i32 u32:u32 f32:f32")


class ParameterRecord(_c.Structure):
    _fields_ = layout("name:char[4097] type:enum is_buffer:u32 access:enum")


class EventRecord(_c.Structure):
    _fields_ = layout("completed:u32 gpu_start_seconds:f64 gpu_end_seconds:f64")


class CapabilityRecord(_c.Structure):
    _fields_ = layout("struct_size:u32 version:u32 stable_id:char[128] backend:char[32] artifact_formats:u64 "
                      "scalar_types:u64 max_buffer_bytes:u64 max_threadgroup_memory_bytes:u64 max_block_x:u32 "
                      "max_block_y:u32 max_block_z:u32 max_buffer_bindings:u32 unified_memory:u32 reserved:u32")


class TimingRecord(_c.Structure):
    _fields_ = layout("struct_size:u32 version:u32 completed:u32 duration_valid:u32 timestamps_valid:u32 "
                      "clock_domain:enum duration_seconds:f64 start_seconds:f64 end_seconds:f64")


class BackendRecord(_c.Structure):
    _fields_ = layout("struct_size:u32 version:u32 backend:char[32] implemented:u32 available:u32 "
                      "device_count:u32 reserved:u32 driver_version:i32 compiler_version:i32 "
                      "driver_library:char[512] compiler_library:char[512] reason:char[1024]")


def versioned(record_type, version=1):
    """A zeroed record whose (struct_size, version) header is filled in."""
    record = record_type()
    record.struct_size, record.version = _c.sizeof(record_type), version
    return record


# ---------------------------------------------------------------- entry-point signatures
# One line per entry point: name, then its parameters. h = a 64-bit handle, u32 /
# u64 / f32 scalars, str = a NUL-terminated string, ptr = an untyped address,
# dim3 = a Dim3 by value, *X = a pointer to X (a scalar kind or a record name).
# Every entry point returns a pr_status, except where "-> u32" says otherwise.
_CALLS = """
pr_abi_version -> u32
pr_last_error *ErrorRecord
pr_backend_status_get str *BackendRecord
pr_device_count *u32
pr_device_get u32 *DeviceRecord
pr_device_capabilities_get u32 *CapabilityRecord
pr_context_create str *h
pr_context_device h *DeviceRecord
pr_context_capabilities h *CapabilityRecord
pr_context_synchronize h
pr_context_write_evidence h str
pr_release h
pr_buffer_create h u64 *h
pr_buffer_size h *u64
pr_view_create h u64 u64 u32 enum *h
pr_buffer_write h u64 ptr u64
pr_buffer_read h u64 ptr u64
pr_module_load h ptr u64 *h
pr_module_load_file h str *h
pr_module_kernel h str *h
pr_kernel_parameter_count h *u32
pr_kernel_parameter h u32 *ParameterRecord
pr_queue_get h *h
pr_queue_synchronize h
pr_launch h h dim3 dim3 *ArgumentRecord u32 *h
pr_event_wait h *EventRecord
pr_event_timing h *TimingRecord
pr_event_cancel h
"""
_KINDS = {"h": _c.c_uint64, "u32": _c.c_uint32, "u64": _c.c_uint64, "f32": _c.c_float, "f64": _c.c_double,
          "enum": _c.c_int, "str": _c.c_char_p, "ptr": _c.c_void_p, "dim3": Dim3}
_RECORDS = {cls.__name__: cls for cls in (ErrorRecord, DeviceRecord, ArgumentRecord, ParameterRecord, EventRecord,
                                          CapabilityRecord, TimingRecord, BackendRecord)}

# Entry points of include/paralyn/native.h and tensor.h (the reference ABI).
REFERENCE_SYMBOLS = (
    "pr_abi_version pr_add_f32 pr_backend_status_get pr_batched_matmul_f32 pr_bias_activation_f32 "
    "pr_buffer_create pr_buffer_read pr_buffer_size pr_buffer_write pr_context_capabilities "
    "pr_context_create pr_context_device pr_context_synchronize pr_context_write_evidence "
    "pr_device_capabilities_get pr_device_count pr_device_get pr_event_cancel pr_event_timing "
    "pr_event_wait pr_kernel_parameter pr_kernel_parameter_count pr_last_error pr_launch "
    "pr_layer_norm_f32 pr_matmul_f32 pr_module_kernel pr_module_load pr_module_load_file "
    "pr_queue_get pr_queue_synchronize pr_reduce_rows_f32 pr_release pr_softmax_rows_f32 "
    "pr_tensor_desc_contiguous pr_tensor_desc_validate pr_tensor_operators_artifact "
    "pr_tensor_operators_capabilities pr_tensor_operators_load pr_view_create").split()
B200_SYMBOLS = ("pr_b200_matmul_mode_set", "pr_b200_matmul_mode_get", "pr_b200_fill_synthetic_f32",
                "pr_b200_device_kernel_count", "pr_b200_module_inspect", "pr_b200_marker",
                "pr_b200_event_elapsed", "pr_b200_matmul_tf32x3_static_f32", "pr_b200_buffer_export",
                "pr_b200_buffer_import", "pr_b200_layer_norm_gather_f32", "pr_b200_buffer_write_async",
                "pr_b200_buffer_read_async", "pr_b200_host_register", "pr_b200_host_unregister",
                "pr_b200_selftest_bounded_wait", "pr_b200_matmul_bias_activation_f32", "pr_b200_gather_rows_f32",
                "pr_b200_matmul_prepared_bytes", "pr_b200_matmul_prepare_f32", "pr_b200_matmul_prepared_f32",
                "pr_b200_matmul_prepared_bias_activation_f32", "pr_b200_queue_hold")


def _ctype(kind, records):
    if kind.startswith("*"):
        return _c.POINTER(_ctype(kind[1:], records))
    return records[kind] if kind in records else _KINDS[kind]


class Library:
    """One loaded libparalyn_native.so. `api` exposes the typed entry points;
    `declare` adds signatures (tensor.py and b200.py declare theirs) and `check`
    turns a status into an Error carrying the library's last-error record."""

    def __init__(self, path):
        self.path = str(Path(path).resolve())
        self.api = _c.CDLL(self.path)
        self._records = dict(_RECORDS)
        self._declared = set()
        self.declare(_CALLS)
        found = self.api.pr_abi_version()
        if found != ABI_VERSION:
            raise RuntimeError(f"{self.path} implements ABI {found}; this binding speaks ABI {ABI_VERSION}")

    def declare(self, table, **records):
        self._records.update(records)
        for line in table.strip().splitlines():
            words = line.split()
            name, params = words[0], words[1:]
            result = _c.c_int
            if "->" in params:
                result = _ctype(params[-1], self._records)
                params = params[:params.index("->")]
            function = getattr(self.api, name)
            function.argtypes = [_ctype(p, self._records) for p in params]
            function.restype = result
            self._declared.add(name)

    def declares(self, name):
        return name in self._declared

    def last_error(self):
        record = ErrorRecord()
        if self.api.pr_last_error(_c.byref(record)) != Status.SUCCESS:
            return "native call", "the library's error record could not be read"
        return _decode(record.operation), _decode(record.message)

    def check(self, status):
        if status != Status.SUCCESS:
            raise Error(status, *self.last_error())

    def call(self, name, *args):
        self.check(getattr(self.api, name)(*args))

    def acquire(self, name, *args):
        """Calls an entry point whose last parameter receives a handle; returns it."""
        out = _c.c_uint64()
        self.call(name, *args, _c.byref(out))
        return out.value


_loaded = {}


def library(path=None):
    """The native library at `path`, else PARALYN_LIBRARY, else the in-tree build
    (loaded once per path)."""
    chosen = Path(path or os.environ.get("PARALYN_LIBRARY") or DEFAULT_LIBRARY).resolve()
    key = str(chosen)
    if key not in _loaded:
        if not chosen.is_file():
            raise FileNotFoundError(f"no native library at {chosen}: run `python -m paralyn_b200.build` "
                                    "or point PARALYN_LIBRARY at libparalyn_native.so")
        _loaded[key] = Library(chosen)
    return _loaded[key]


# ---------------------------------------------------------------- argument checks
def _decode(raw):
    return raw.decode("utf-8", errors="replace")


def _int(value, low, high, label):
    """`value` as an int in [low, high]; bools are not integers here."""
    if isinstance(value, bool) or not isinstance(value, int):
        raise TypeError(f"{label}: expected an integer, got {type(value).__name__}")
    if value < low or value > high:
        raise ValueError(f"{label}: {value} is outside [{low}, {high}]")
    return value


def _u64(value, label):
    return _int(value, 0, 2 ** 64 - 1, label)


def _encode(text, label):
    raw = os.fsencode(text)
    if 0 in raw:
        raise ValueError(f"{label}: embedded NUL byte")
    return raw


# ---------------------------------------------------------------- device and backend queries
@dataclass(frozen=True)
class Device:
    name: str
    backend: str
    os: str
    registry_id: int
    max_buffer_bytes: int
    unified_memory: bool

    @classmethod
    def _from(cls, r):
        return cls(_decode(r.name), _decode(r.backend), _decode(r.os), r.registry_id, r.max_buffer_bytes,
                   r.unified_memory != 0)


@dataclass(frozen=True)
class DeviceCapabilities:
    stable_id: str
    backend: str
    artifact_formats: int
    scalar_types: int
    max_buffer_bytes: int
    max_threadgroup_memory_bytes: int
    max_block: tuple
    max_buffer_bindings: int
    unified_memory: bool

    @classmethod
    def _from(cls, r):
        block = (r.max_block_x, r.max_block_y, r.max_block_z)
        return cls(_decode(r.stable_id), _decode(r.backend), r.artifact_formats, r.scalar_types,
                   r.max_buffer_bytes, r.max_threadgroup_memory_bytes, block, r.max_buffer_bindings,
                   r.unified_memory != 0)


@dataclass(frozen=True)
class EventTiming:
    """CUDA timing is duration-only: start/end stay None unless the record marks
    timestamps valid."""
    completed: bool
    duration_seconds: object
    start_seconds: object
    end_seconds: object
    clock_domain: ClockDomain

    @classmethod
    def _from(cls, r):
        stamps = (r.start_seconds, r.end_seconds) if r.timestamps_valid else (None, None)
        return cls(r.completed != 0, r.duration_seconds if r.duration_valid else None, *stamps,
                   ClockDomain(r.clock_domain))


@dataclass(frozen=True)
class BackendStatus:
    backend: str
    implemented: bool
    available: bool
    device_count: int
    driver_version: int
    compiler_version: int
    reason: str


def backend_status(name="cuda", path=None):
    lib = library(path)
    r = versioned(BackendRecord)
    lib.call("pr_backend_status_get", _encode(name, "backend name"), _c.byref(r))
    return BackendStatus(_decode(r.backend), r.implemented != 0, r.available != 0, r.device_count,
                         r.driver_version, r.compiler_version, _decode(r.reason))


def devices(path=None):
    lib = library(path)
    count = _c.c_uint32()
    lib.call("pr_device_count", _c.byref(count))
    found = []
    for index in range(count.value):
        r = DeviceRecord()
        lib.call("pr_device_get", index, _c.byref(r))
        found.append(Device._from(r))
    return tuple(found)


def device_capabilities(index=0, path=None):
    lib = library(path)
    r = versioned(CapabilityRecord)
    lib.call("pr_device_capabilities_get", _int(index, 0, 2 ** 32 - 1, "device index"), _c.byref(r))
    return DeviceCapabilities._from(r)


# ---------------------------------------------------------------- owned handles
def _release_at_collection(lib, handle, kind):
    """Finalizer of an owned handle that nobody closed."""
    status = lib.api.pr_release(handle)
    if status != Status.SUCCESS:
        operation, message = lib.last_error()
        sys.stderr.write(f"paralyn_b200: releasing an unclosed {kind} failed ({Status(status).name}, "
                         f"{operation}: {message}); a GPU failure nobody waited for ends the process\n")
        sys.stderr.flush()
        os._exit(1)


class Owned:
    """Holds one reference to a native handle until close(), the end of a `with`
    block, or garbage collection (not interpreter exit: the library drains its own
    work when the process ends)."""

    _handle = 0
    _finalizer = None

    def _own(self, lib, handle):
        self._lib, self._handle = lib, handle
        self._finalizer = weakref.finalize(self, _release_at_collection, lib, handle, type(self).__name__)
        self._finalizer.atexit = False

    @classmethod
    def _adopt(cls, lib, handle):
        value = cls.__new__(cls)
        value._own(lib, handle)
        return value

    @property
    def closed(self):
        return not self._handle

    @property
    def handle(self):
        if not self._handle:
            raise Error(Status.INVALID_HANDLE, type(self).__name__, "used after close()")
        return self._handle

    def close(self):
        """Releases the handle (idempotent); raises the release's failure, if any."""
        if not self._handle:
            return
        handle, self._handle = self._handle, 0
        self._finalizer.detach()
        self._lib.call("pr_release", handle)

    def __enter__(self):
        self.handle  # a closed object cannot enter a block
        return self

    def __exit__(self, *_):
        self.close()


class Context(Owned):
    """A device context with its one in-order queue. `selector` is "cuda:K" or
    "auto" (default: PARALYN_DEVICE, else "auto")."""

    def __init__(self, selector=None, *, library_path=None):
        lib = library(library_path)
        selector = os.environ.get("PARALYN_DEVICE", "auto") if selector is None else selector
        self._own(lib, lib.acquire("pr_context_create", _encode(selector, "device selector")))
        self._attached = {}  # per-context operator resources (tensor provider, array module)

    def attached(self, key, factory):
        """The context's resource under `key`, made by factory(context) on first use
        and closed before the context itself."""
        self.handle
        if key not in self._attached:
            self._attached[key] = factory(self)
        return self._attached[key]

    @property
    def device(self):
        r = DeviceRecord()
        self._lib.call("pr_context_device", self.handle, _c.byref(r))
        return Device._from(r)

    @property
    def capabilities(self):
        r = versioned(CapabilityRecord)
        self._lib.call("pr_context_capabilities", self.handle, _c.byref(r))
        return DeviceCapabilities._from(r)

    def buffer(self, size):
        return Buffer(self, size)

    def queue(self):
        return Queue(self)

    def synchronize(self):
        self._lib.call("pr_context_synchronize", self.handle)

    def write_evidence(self, directory):
        self._lib.call("pr_context_write_evidence", self.handle, _encode(directory, "evidence directory"))

    def close(self):
        errors = []
        for resource in reversed(list(getattr(self, "_attached", {}).values())):
            try:
                resource.close()
            except Exception as error:
                errors.append(error)
        self._attached = {}
        try:
            super().close()
        except Exception as error:
            errors.append(error)
        if errors:
            raise errors[0]


def _require(value, kind, what):
    if not isinstance(value, kind):
        raise TypeError(f"{what} requires a {kind.__name__}, got {type(value).__name__}")
    return value


class Buffer(Owned):
    """A device allocation of `size` bytes owned by a context."""

    def __init__(self, context, size):
        _require(context, Context, "Buffer")
        self._own(context._lib, context._lib.acquire("pr_buffer_create", context.handle, _u64(size, "buffer size")))

    @property
    def size(self):
        out = _c.c_uint64()
        self._lib.call("pr_buffer_size", self.handle, _c.byref(out))
        return out.value

    def write(self, data, *, offset=0):
        """Blocking copy of C-contiguous host bytes (any buffer-protocol object)."""
        bytes_view = memoryview(data)
        if not bytes_view.c_contiguous:
            raise ValueError("write: host data must be C-contiguous (no layout conversion is done)")
        bytes_view = bytes_view.cast("B")
        size = bytes_view.nbytes
        if size == 0:
            source = None
        elif bytes_view.readonly:
            source = _c.create_string_buffer(bytes_view.tobytes(), size)
        else:
            source = (_c.c_char * size).from_buffer(bytes_view)
        self._lib.call("pr_buffer_write", self.handle, _u64(offset, "write offset"), source, size)

    def write_from(self, address, nbytes, *, offset=0):
        """Blocking copy of nbytes from a raw host (or device) address."""
        self._lib.call("pr_buffer_write", self.handle, _u64(offset, "write offset"), _c.c_void_p(address),
                       _u64(nbytes, "byte count"))

    def read(self, size=None, *, offset=0):
        """Blocking copy of `size` bytes from `offset` (default: to the end) as bytes."""
        offset = _u64(offset, "read offset")
        total = self.size
        size = total - offset if size is None else _u64(size, "read size")
        if offset > total or size > total - offset:
            raise Error(Status.OUT_OF_BOUNDS, "Buffer.read",
                        f"bytes [{offset}, {offset + max(size, 0)}) are outside the {total}-byte buffer")
        out = bytearray(size)
        if size:
            self._lib.call("pr_buffer_read", self.handle, offset, (_c.c_char * size).from_buffer(out), size)
        return bytes(out)

    def read_into(self, address, nbytes, *, offset=0):
        """Blocking copy of nbytes into a raw host (or device) address."""
        self._lib.call("pr_buffer_read", self.handle, _u64(offset, "read offset"), _c.c_void_p(address),
                       _u64(nbytes, "byte count"))

    def view(self, *, offset=0, size=None, alignment=4, access=Access.READ_WRITE):
        return View(self, offset=offset, size=size, alignment=alignment, access=access)


class View(Owned):
    """A byte range of a buffer with an access mode: what kernels are bound to."""

    def __init__(self, buffer, *, offset=0, size=None, alignment=4, access=Access.READ_WRITE):
        _require(buffer, Buffer, "View")
        offset = _u64(offset, "view offset")
        if size is None:
            size = buffer.size - offset
            if size < 0:
                raise Error(Status.OUT_OF_BOUNDS, "View", f"offset {offset} is past the end of the buffer")
        handle = buffer._lib.acquire("pr_view_create", buffer.handle, offset, _u64(size, "view size"),
                                     _int(alignment, 0, 2 ** 32 - 1, "alignment"), Access(access))
        self._own(buffer._lib, handle)


class Module(Owned):
    """A loaded kernel module (.prk artifact)."""

    @classmethod
    def load_file(cls, context, path):
        _require(context, Context, "Module.load_file")
        return cls._adopt(context._lib, context._lib.acquire("pr_module_load_file", context.handle,
                                                             _encode(path, "module path")))

    @classmethod
    def load(cls, context, data):
        _require(context, Context, "Module.load")
        raw = bytes(memoryview(data))
        image = _c.create_string_buffer(raw, len(raw)) if raw else None
        return cls._adopt(context._lib, context._lib.acquire("pr_module_load", context.handle, image, len(raw)))

    def kernel(self, name):
        return Kernel._adopt(self._lib, self._lib.acquire("pr_module_kernel", self.handle,
                                                          _encode(name, "kernel name")))


@dataclass(frozen=True)
class Parameter:
    name: str
    type: Type
    is_buffer: bool
    access: Access


class Kernel(Owned):
    @property
    def parameters(self):
        count = _c.c_uint32()
        self._lib.call("pr_kernel_parameter_count", self.handle, _c.byref(count))
        found = []
        for index in range(count.value):
            r = ParameterRecord()
            self._lib.call("pr_kernel_parameter", self.handle, index, _c.byref(r))
            found.append(Parameter(_decode(r.name), Type(r.type), r.is_buffer != 0, Access(r.access)))
        return tuple(found)


# ---------------------------------------------------------------- scalar arguments
_FLT_MAX = 3.4028234663852886e38


def _as_i32(value):
    return _int(value, -2 ** 31, 2 ** 31 - 1, "i32")


def _as_u32(value):
    return _int(value, 0, 2 ** 32 - 1, "u32")


def _as_f32(value):
    if isinstance(value, bool) or not isinstance(value, (int, float)):
        raise TypeError(f"f32: expected an int or float, got {type(value).__name__}")
    value = float(value)
    if math.isfinite(value) and abs(value) > _FLT_MAX:
        raise ValueError(f"f32: {value} overflows binary32")
    return _c.c_float(value).value  # rounded to binary32 once, here


_SCALAR_RULES = {Type.I32: ("i32", _as_i32), Type.U32: ("u32", _as_u32), Type.F32: ("f32", _as_f32)}


@dataclass(frozen=True)
class Scalar:
    """A typed by-value kernel argument; the value is checked (and f32 rounded) once."""
    type: Type
    value: object

    def __post_init__(self):
        if self.type not in _SCALAR_RULES:
            raise ValueError("a Scalar is I32, U32 or F32")
        object.__setattr__(self, "value", _SCALAR_RULES[self.type][1](self.value))


def i32(value):
    return Scalar(Type.I32, value)


def u32(value):
    return Scalar(Type.U32, value)


def f32(value):
    return Scalar(Type.F32, value)


def _dims(value, label):
    if isinstance(value, int) and not isinstance(value, bool):
        value = (value, 1, 1)
    if not isinstance(value, (tuple, list)) or len(value) != 3:
        raise TypeError(f"{label}: expected an int or an (x, y, z) triple")
    return Dim3(*(_int(v, 0, 2 ** 32 - 1, label) for v in value))


class Queue(Owned):
    """A handle of the context's single in-order queue."""

    def __init__(self, context):
        _require(context, Context, "Queue")
        self._own(context._lib, context._lib.acquire("pr_queue_get", context.handle))

    def synchronize(self):
        self._lib.call("pr_queue_synchronize", self.handle)

    def launch(self, kernel, arguments, *, grid, block):
        """Enqueues `kernel` over grid x block with View and Scalar arguments in
        parameter order; returns the command's Event."""
        _require(kernel, Kernel, "launch")
        if kernel._lib is not self._lib:
            raise ValueError("launch: the kernel comes from another native library")
        arguments = list(arguments)
        packed = (ArgumentRecord * len(arguments))()
        for slot, argument in zip(packed, arguments):
            if isinstance(argument, View):
                if argument._lib is not self._lib:
                    raise ValueError("launch: a view comes from another native library")
                slot.type, slot.view = Type.BUFFER, argument.handle
            elif isinstance(argument, Scalar):
                slot.type = argument.type
                setattr(slot, _SCALAR_RULES[argument.type][0], argument.value)
            else:
                raise TypeError("launch: arguments are Views and i32/u32/f32 Scalars, got "
                                f"{type(argument).__name__}")
        handle = self._lib.acquire("pr_launch", self.handle, kernel.handle, _dims(grid, "grid"),
                                   _dims(block, "block"), packed, len(arguments))
        return Event._adopt(self._lib, handle)


@dataclass(frozen=True)
class EventInfo:
    completed: bool
    gpu_start_seconds: float
    gpu_end_seconds: float


class Event(Owned):
    """Completion of one queued command."""

    def wait(self):
        r = EventRecord()
        self._lib.call("pr_event_wait", self.handle, _c.byref(r))
        return EventInfo(r.completed != 0, r.gpu_start_seconds, r.gpu_end_seconds)

    def timing(self):
        """Waits for the command (raising its failure) and returns its timing."""
        r = versioned(TimingRecord)
        self._lib.call("pr_event_timing", self.handle, _c.byref(r))
        return EventTiming._from(r)

    def cancel(self):
        self._lib.call("pr_event_cancel", self.handle)
