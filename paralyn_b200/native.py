"""ctypes binding of the native C ABI (include/paralyn/native.h).

Mirrors the reference's Python binding (bindings/python/paralyn/__init__.py): the
same classes (Context, Buffer, View, Module, Kernel, Queue, Event), scalar
wrappers (i32/u32/f32), status codes, error type and ownership rules (explicit
close or context managers; a finalizer that cannot release terminates the
process). It loads the in-tree libparalyn_native.so built by paralyn_b200.build,
or PARALYN_LIBRARY. There is no CPU fallback: without the library or a CUDA
device every call fails loudly.
"""
import ctypes as _c
from dataclasses import dataclass
from enum import IntEnum
import math
import os
from pathlib import Path

ABI_VERSION = 1
_PACKAGE = Path(__file__).resolve().parent
DEFAULT_LIBRARY = _PACKAGE / "libparalyn_native.so"


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


class Error(RuntimeError):
    """A failed native call: status code, failing operation and message."""

    def __init__(self, code, operation, message):
        self.code = Status(code)
        self.operation = operation
        self.message = message
        super().__init__(f"{operation}: {message} [{self.code.name}]")


class ErrorRecord(_c.Structure):
    _fields_ = [("code", _c.c_int), ("operation", _c.c_char * 64), ("message", _c.c_char * 1024)]


class DeviceRecord(_c.Structure):
    _fields_ = [("name", _c.c_char * 256), ("backend", _c.c_char * 32), ("os", _c.c_char * 128),
                ("registry_id", _c.c_uint64), ("max_buffer_bytes", _c.c_uint64),
                ("unified_memory", _c.c_uint32)]


class Dim3(_c.Structure):
    _fields_ = [("x", _c.c_uint32), ("y", _c.c_uint32), ("z", _c.c_uint32)]


class ArgumentRecord(_c.Structure):
    _fields_ = [("type", _c.c_int), ("view", _c.c_uint64), ("i32", _c.c_int32),
                ("u32", _c.c_uint32), ("f32", _c.c_float)]


class ParameterRecord(_c.Structure):
    _fields_ = [("name", _c.c_char * 4097), ("type", _c.c_int), ("is_buffer", _c.c_uint32),
                ("access", _c.c_int)]


class EventRecord(_c.Structure):
    _fields_ = [("completed", _c.c_uint32), ("gpu_start_seconds", _c.c_double),
                ("gpu_end_seconds", _c.c_double)]


class CapabilityRecord(_c.Structure):
    _fields_ = [("struct_size", _c.c_uint32), ("version", _c.c_uint32),
                ("stable_id", _c.c_char * 128), ("backend", _c.c_char * 32),
                ("artifact_formats", _c.c_uint64), ("scalar_types", _c.c_uint64),
                ("max_buffer_bytes", _c.c_uint64), ("max_threadgroup_memory_bytes", _c.c_uint64),
                ("max_block_x", _c.c_uint32), ("max_block_y", _c.c_uint32),
                ("max_block_z", _c.c_uint32), ("max_buffer_bindings", _c.c_uint32),
                ("unified_memory", _c.c_uint32), ("reserved", _c.c_uint32)]


class TimingRecord(_c.Structure):
    _fields_ = [("struct_size", _c.c_uint32), ("version", _c.c_uint32), ("completed", _c.c_uint32),
                ("duration_valid", _c.c_uint32), ("timestamps_valid", _c.c_uint32),
                ("clock_domain", _c.c_int), ("duration_seconds", _c.c_double),
                ("start_seconds", _c.c_double), ("end_seconds", _c.c_double)]


class BackendRecord(_c.Structure):
    _fields_ = [("struct_size", _c.c_uint32), ("version", _c.c_uint32), ("backend", _c.c_char * 32),
                ("implemented", _c.c_uint32), ("available", _c.c_uint32),
                ("device_count", _c.c_uint32), ("reserved", _c.c_uint32),
                ("driver_version", _c.c_int32), ("compiler_version", _c.c_int32),
                ("driver_library", _c.c_char * 512), ("compiler_library", _c.c_char * 512),
                ("reason", _c.c_char * 1024)]


def versioned(record_type):
    record = record_type()
    record.struct_size, record.version = _c.sizeof(record_type), 1
    return record


def _text(raw):
    return raw.decode("utf-8", errors="replace")


def _int(value, low, high, label):
    if not isinstance(value, int) or isinstance(value, bool):
        raise TypeError(f"{label} requires an integer")
    if not low <= value <= high:
        raise ValueError(f"{label} must be in [{low}, {high}]")
    return value


def _u64(value, label):
    return _int(value, 0, (1 << 64) - 1, label)


def _cstring(value, label):
    data = os.fsencode(value)
    if b"\0" in data:
        raise ValueError(f"{label} contains a null byte")
    return data


_H, _U32, _U64, _P = _c.c_uint64, _c.c_uint32, _c.c_uint64, _c.POINTER
_SIGNATURES = {
    "pr_abi_version": (_U32, []),
    "pr_last_error": (_c.c_int, [_P(ErrorRecord)]),
    "pr_backend_status_get": (_c.c_int, [_c.c_char_p, _P(BackendRecord)]),
    "pr_device_count": (_c.c_int, [_P(_U32)]),
    "pr_device_get": (_c.c_int, [_U32, _P(DeviceRecord)]),
    "pr_device_capabilities_get": (_c.c_int, [_U32, _P(CapabilityRecord)]),
    "pr_context_create": (_c.c_int, [_c.c_char_p, _P(_H)]),
    "pr_context_device": (_c.c_int, [_H, _P(DeviceRecord)]),
    "pr_context_capabilities": (_c.c_int, [_H, _P(CapabilityRecord)]),
    "pr_context_synchronize": (_c.c_int, [_H]),
    "pr_context_write_evidence": (_c.c_int, [_H, _c.c_char_p]),
    "pr_release": (_c.c_int, [_H]),
    "pr_buffer_create": (_c.c_int, [_H, _U64, _P(_H)]),
    "pr_buffer_size": (_c.c_int, [_H, _P(_U64)]),
    "pr_view_create": (_c.c_int, [_H, _U64, _U64, _U32, _c.c_int, _P(_H)]),
    "pr_buffer_write": (_c.c_int, [_H, _U64, _c.c_void_p, _U64]),
    "pr_buffer_read": (_c.c_int, [_H, _U64, _c.c_void_p, _U64]),
    "pr_module_load": (_c.c_int, [_H, _c.c_void_p, _U64, _P(_H)]),
    "pr_module_load_file": (_c.c_int, [_H, _c.c_char_p, _P(_H)]),
    "pr_module_kernel": (_c.c_int, [_H, _c.c_char_p, _P(_H)]),
    "pr_kernel_parameter_count": (_c.c_int, [_H, _P(_U32)]),
    "pr_kernel_parameter": (_c.c_int, [_H, _U32, _P(ParameterRecord)]),
    "pr_queue_get": (_c.c_int, [_H, _P(_H)]),
    "pr_queue_synchronize": (_c.c_int, [_H]),
    "pr_launch": (_c.c_int, [_H, _H, Dim3, Dim3, _P(ArgumentRecord), _U32, _P(_H)]),
    "pr_event_wait": (_c.c_int, [_H, _P(EventRecord)]),
    "pr_event_timing": (_c.c_int, [_H, _P(TimingRecord)]),
    "pr_event_cancel": (_c.c_int, [_H]),
}
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
                "pr_b200_selftest_bounded_wait", "pr_b200_matmul_bias_activation_f32")


class Library:
    """One loaded libparalyn_native.so with typed entry points."""

    def __init__(self, path):
        self.path = str(Path(path).resolve())
        self.api = _c.CDLL(self.path)
        for name, (result, arguments) in _SIGNATURES.items():
            function = getattr(self.api, name)
            function.restype, function.argtypes = result, arguments
        version = self.api.pr_abi_version()
        if version != ABI_VERSION:
            raise RuntimeError(f"Paralyn ABI {version} is incompatible with binding ABI {ABI_VERSION}")

    def check(self, status):
        if status == Status.SUCCESS:
            return
        record = ErrorRecord()
        if self.api.pr_last_error(_c.byref(record)) == Status.SUCCESS:
            raise Error(status, _text(record.operation), _text(record.message))
        raise Error(status, "native call", "native error detail retrieval failed")


_libraries = {}


def library(path=None):
    """The native library: `path`, else PARALYN_LIBRARY, else the in-tree build."""
    if path is None:
        path = os.environ.get("PARALYN_LIBRARY") or DEFAULT_LIBRARY
    path = str(Path(path).resolve())
    if path not in _libraries:
        if not Path(path).is_file():
            raise FileNotFoundError(f"libparalyn_native.so not found at {path}; build it with "
                                    "`python -m paralyn_b200.build` or set PARALYN_LIBRARY")
        _libraries[path] = Library(path)
    return _libraries[path]


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
        return cls(_text(r.name), _text(r.backend), _text(r.os), r.registry_id, r.max_buffer_bytes,
                   bool(r.unified_memory))


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
        return cls(_text(r.stable_id), _text(r.backend), r.artifact_formats, r.scalar_types,
                   r.max_buffer_bytes, r.max_threadgroup_memory_bytes,
                   (r.max_block_x, r.max_block_y, r.max_block_z), r.max_buffer_bindings,
                   bool(r.unified_memory))


@dataclass(frozen=True)
class EventTiming:
    """Duration-only on CUDA: start/end are None unless the backend marks them valid."""
    completed: bool
    duration_seconds: object
    start_seconds: object
    end_seconds: object
    clock_domain: ClockDomain

    @classmethod
    def _from(cls, r):
        return cls(bool(r.completed), r.duration_seconds if r.duration_valid else None,
                   r.start_seconds if r.timestamps_valid else None,
                   r.end_seconds if r.timestamps_valid else None, ClockDomain(r.clock_domain))


@dataclass(frozen=True)
class BackendStatus:
    backend: str
    implemented: bool
    available: bool
    device_count: int
    driver_version: int
    compiler_version: int
    reason: str


ARTIFACT_VERIFIED_IR = 1 << 0
ARTIFACT_MSL_SOURCE = 1 << 1
ARTIFACT_SPIRV_MSL = 1 << 2


def backend_status(name="cuda", path=None):
    lib = library(path)
    record = versioned(BackendRecord)
    lib.check(lib.api.pr_backend_status_get(_cstring(name, "backend"), _c.byref(record)))
    return BackendStatus(_text(record.backend), bool(record.implemented), bool(record.available),
                         record.device_count, record.driver_version, record.compiler_version,
                         _text(record.reason))


def devices(path=None):
    lib = library(path)
    count = _c.c_uint32()
    lib.check(lib.api.pr_device_count(_c.byref(count)))
    result = []
    for index in range(count.value):
        record = DeviceRecord()
        lib.check(lib.api.pr_device_get(index, _c.byref(record)))
        result.append(Device._from(record))
    return tuple(result)


def device_capabilities(index=0, path=None):
    lib = library(path)
    record = versioned(CapabilityRecord)
    lib.check(lib.api.pr_device_capabilities_get(_int(index, 0, (1 << 32) - 1, "device index"),
                                                 _c.byref(record)))
    return DeviceCapabilities._from(record)


class Owned:
    """A native handle with one owned reference."""

    @classmethod
    def _adopt(cls, lib, handle):
        value = cls.__new__(cls)
        value._lib, value._handle = lib, handle
        return value

    @property
    def handle(self):
        if not getattr(self, "_handle", 0):
            raise Error(Status.INVALID_HANDLE, type(self).__name__, "object is closed")
        return self._handle

    @property
    def closed(self):
        return not getattr(self, "_handle", 0)

    def close(self):
        if self.closed:
            return
        handle, self._handle = self._handle, 0
        self._lib.check(self._lib.api.pr_release(handle))

    def __enter__(self):
        self.handle
        return self

    def __exit__(self, *_):
        self.close()

    def __del__(self, _write=os.write, _exit=os._exit):
        if not self.closed:
            try:
                self.close()
            except Exception as error:  # a lost GPU failure must not exit 0
                try:
                    _write(2, f"Paralyn fatal unhandled {type(self).__name__} finalizer error: "
                              f"{error}\n".encode("utf-8", errors="backslashreplace"))
                finally:
                    _exit(1)


class Context(Owned):
    """One device context with one ordered queue ("cuda:K" or "auto")."""

    def __init__(self, selector=None, *, library_path=None):
        if selector is None:
            selector = os.environ.get("PARALYN_DEVICE", "auto")
        self._lib, self._handle = library(library_path), 0
        handle = _c.c_uint64()
        self._lib.check(self._lib.api.pr_context_create(_cstring(selector, "selector"), _c.byref(handle)))
        self._handle = handle.value

    @property
    def device(self):
        record = DeviceRecord()
        self._lib.check(self._lib.api.pr_context_device(self.handle, _c.byref(record)))
        return Device._from(record)

    @property
    def capabilities(self):
        record = versioned(CapabilityRecord)
        self._lib.check(self._lib.api.pr_context_capabilities(self.handle, _c.byref(record)))
        return DeviceCapabilities._from(record)

    def buffer(self, size):
        return Buffer(self, size)

    def queue(self):
        return Queue(self)

    def synchronize(self):
        self._lib.check(self._lib.api.pr_context_synchronize(self.handle))

    def write_evidence(self, directory):
        self._lib.check(self._lib.api.pr_context_write_evidence(
            self.handle, _cstring(directory, "evidence directory")))

    def close(self):
        failure = None
        for name in ("_tensor_resources", "_array_resources"):
            resources = getattr(self, name, None)
            setattr(self, name, None)
            if resources is not None:
                try:
                    resources.close()
                except Exception as error:
                    failure = failure or error
        try:
            super().close()
        except Exception as error:
            failure = failure or error
        if failure is not None:
            raise failure


class Buffer(Owned):
    """Device allocation of `size` bytes owned by a context."""

    def __init__(self, context, size):
        if not isinstance(context, Context):
            raise TypeError("Buffer requires a Context")
        self._lib, self._handle = context._lib, 0
        handle = _c.c_uint64()
        self._lib.check(self._lib.api.pr_buffer_create(context.handle, _u64(size, "buffer size"),
                                                      _c.byref(handle)))
        self._handle = handle.value

    @property
    def size(self):
        value = _c.c_uint64()
        self._lib.check(self._lib.api.pr_buffer_size(self.handle, _c.byref(value)))
        return value.value

    def write(self, data, *, offset=0):
        view = memoryview(data)
        if not view.c_contiguous:
            raise ValueError("write requires C-contiguous host bytes; no layout conversion is performed")
        view = view.cast("B")
        if view.nbytes == 0:
            storage = None
        elif view.readonly:  # copy; writable host memory is passed without a copy
            storage = _c.create_string_buffer(view.tobytes(), view.nbytes)
        else:
            storage = (_c.c_char * view.nbytes).from_buffer(view)
        self._lib.check(self._lib.api.pr_buffer_write(self.handle, _u64(offset, "write offset"),
                                                     storage, view.nbytes))

    def write_from(self, address, nbytes, *, offset=0):
        """Blocking copy of nbytes from a raw host (or device) address."""
        self._lib.check(self._lib.api.pr_buffer_write(self.handle, _u64(offset, "write offset"),
                                                     _c.c_void_p(address), _u64(nbytes, "size")))

    def read(self, size=None, *, offset=0):
        offset = _u64(offset, "read offset")
        capacity = self.size
        if offset > capacity:
            raise Error(Status.OUT_OF_BOUNDS, "Buffer.read", "read offset exceeds buffer size")
        size = capacity - offset if size is None else _u64(size, "read size")
        if size > capacity - offset:
            raise Error(Status.OUT_OF_BOUNDS, "Buffer.read", "read exceeds buffer size")
        storage = bytearray(size)
        if size:
            target = (_c.c_char * size).from_buffer(storage)
            self._lib.check(self._lib.api.pr_buffer_read(self.handle, offset, target, size))
        return bytes(storage)

    def read_into(self, address, nbytes, *, offset=0):
        """Blocking copy of nbytes into a raw host (or device) address."""
        self._lib.check(self._lib.api.pr_buffer_read(self.handle, _u64(offset, "read offset"),
                                                    _c.c_void_p(address), _u64(nbytes, "size")))

    def view(self, *, offset=0, size=None, alignment=4, access=Access.READ_WRITE):
        return View(self, offset=offset, size=size, alignment=alignment, access=access)


class View(Owned):
    def __init__(self, buffer, *, offset=0, size=None, alignment=4, access=Access.READ_WRITE):
        if not isinstance(buffer, Buffer):
            raise TypeError("View requires a Buffer")
        self._lib, self._handle = buffer._lib, 0
        offset = _u64(offset, "view offset")
        if size is None:
            size = buffer.size - offset
            if size < 0:
                raise Error(Status.OUT_OF_BOUNDS, "View", "view offset exceeds buffer size")
        handle = _c.c_uint64()
        self._lib.check(self._lib.api.pr_view_create(
            buffer.handle, offset, _u64(size, "view size"), _int(alignment, 0, (1 << 32) - 1, "alignment"),
            Access(access), _c.byref(handle)))
        self._handle = handle.value


class Module(Owned):
    @classmethod
    def load_file(cls, context, path):
        if not isinstance(context, Context):
            raise TypeError("Module.load_file requires a Context")
        handle = _c.c_uint64()
        context._lib.check(context._lib.api.pr_module_load_file(
            context.handle, _cstring(path, "module path"), _c.byref(handle)))
        return cls._adopt(context._lib, handle.value)

    @classmethod
    def load(cls, context, data):
        if not isinstance(context, Context):
            raise TypeError("Module.load requires a Context")
        data = bytes(memoryview(data))
        storage = _c.create_string_buffer(data, len(data)) if data else None
        handle = _c.c_uint64()
        context._lib.check(context._lib.api.pr_module_load(context.handle, storage, len(data),
                                                        _c.byref(handle)))
        return cls._adopt(context._lib, handle.value)

    def kernel(self, name):
        handle = _c.c_uint64()
        self._lib.check(self._lib.api.pr_module_kernel(self.handle, _cstring(name, "kernel name"),
                                                      _c.byref(handle)))
        return Kernel._adopt(self._lib, handle.value)


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
        self._lib.check(self._lib.api.pr_kernel_parameter_count(self.handle, _c.byref(count)))
        result = []
        for index in range(count.value):
            record = ParameterRecord()
            self._lib.check(self._lib.api.pr_kernel_parameter(self.handle, index, _c.byref(record)))
            result.append(Parameter(_text(record.name), Type(record.type), bool(record.is_buffer),
                                    Access(record.access)))
        return tuple(result)


@dataclass(frozen=True)
class Scalar:
    type: Type
    value: object

    def __post_init__(self):
        if self.type == Type.I32:
            value = _int(self.value, -(1 << 31), (1 << 31) - 1, "i32")
        elif self.type == Type.U32:
            value = _int(self.value, 0, (1 << 32) - 1, "u32")
        elif self.type == Type.F32:
            if not isinstance(self.value, (int, float)) or isinstance(self.value, bool):
                raise TypeError("f32 requires an explicit integer or float value")
            value = float(self.value)
            if math.isfinite(value) and abs(value) > 3.4028234663852886e38:
                raise ValueError("f32 value exceeds the finite FP32 range")
            value = _c.c_float(value).value
        else:
            raise ValueError("Scalar type must be I32, U32 or F32")
        object.__setattr__(self, "value", value)


def i32(value):
    return Scalar(Type.I32, value)


def u32(value):
    return Scalar(Type.U32, value)


def f32(value):
    return Scalar(Type.F32, value)


def _dim3(value):
    if isinstance(value, int) and not isinstance(value, bool):
        value = (value, 1, 1)
    if not isinstance(value, (tuple, list)) or len(value) != 3:
        raise TypeError("dimensions require an integer or an (x, y, z) tuple")
    return Dim3(*(_int(v, 0, (1 << 32) - 1, "dimension") for v in value))


class Queue(Owned):
    """The context's single in-order queue."""

    def __init__(self, context):
        if not isinstance(context, Context):
            raise TypeError("Queue requires a Context")
        self._lib, self._handle = context._lib, 0
        handle = _c.c_uint64()
        self._lib.check(self._lib.api.pr_queue_get(context.handle, _c.byref(handle)))
        self._handle = handle.value

    def synchronize(self):
        self._lib.check(self._lib.api.pr_queue_synchronize(self.handle))

    def launch(self, kernel, arguments, *, grid, block):
        if not isinstance(kernel, Kernel):
            raise TypeError("launch requires a Kernel")
        if kernel._lib is not self._lib:
            raise ValueError("kernel and queue originate from different native libraries")
        arguments = tuple(arguments)
        native = (ArgumentRecord * len(arguments))()
        for index, argument in enumerate(arguments):
            if isinstance(argument, View):
                if argument._lib is not self._lib:
                    raise ValueError("view and queue originate from different native libraries")
                native[index].type, native[index].view = Type.BUFFER, argument.handle
            elif isinstance(argument, Scalar):
                native[index].type = argument.type
                setattr(native[index], {Type.I32: "i32", Type.U32: "u32", Type.F32: "f32"}[argument.type],
                        argument.value)
            else:
                raise TypeError("kernel arguments require View or explicit i32/u32/f32 values")
        handle = _c.c_uint64()
        self._lib.check(self._lib.api.pr_launch(self.handle, kernel.handle, _dim3(grid), _dim3(block),
                                               native, len(arguments), _c.byref(handle)))
        return Event._adopt(self._lib, handle.value)


@dataclass(frozen=True)
class EventInfo:
    completed: bool
    gpu_start_seconds: float
    gpu_end_seconds: float


class Event(Owned):
    def wait(self):
        record = EventRecord()
        self._lib.check(self._lib.api.pr_event_wait(self.handle, _c.byref(record)))
        return EventInfo(bool(record.completed), record.gpu_start_seconds, record.gpu_end_seconds)

    def timing(self):
        """Waits, propagates command failure, returns the duration-only timing record."""
        record = versioned(TimingRecord)
        self._lib.check(self._lib.api.pr_event_timing(self.handle, _c.byref(record)))
        return EventTiming._from(record)

    def cancel(self):
        self._lib.check(self._lib.api.pr_event_cancel(self.handle))
