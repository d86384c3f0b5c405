"""Device-resident FP32 values that own their buffer and the event that fills it.

Array (array.py) and Tensor (tensor.py) are both a DeviceValue: a buffer on one
context, a shape, and optionally the Event of the command that produces the
contents. Reading (`to_host`) or waiting first waits for that event, so a failed
command surfaces as its Error there. `close()` releases the event and then the
buffer; a value that nobody closed is released when it is collected, and a release
that fails at that point ends the process (the failed GPU work would otherwise be
lost without a trace).
"""
from array import array as _host_array
import os
import sys
import weakref

from .native import Context, Error, Status, _int, f32

float32 = "float32"
MAX_ELEMENTS = 2 ** 31 - 1


def _release_pair_at_collection(kind, event, buffer):
    try:
        for owned in (event, buffer):
            if owned is not None:
                owned.close()
    except Exception as error:
        sys.stderr.write(f"paralyn_b200: releasing an unclosed {kind} failed: {error}; "
                         "a GPU failure nobody waited for ends the process\n")
        sys.stderr.flush()
        os._exit(1)


class DeviceValue:
    """Base of Array and Tensor (created by the package's functions, not directly)."""

    _kind = "value"
    _finalizer = None

    def __init__(self, *_, **__):
        raise TypeError(f"a {type(self).__name__} is made by the package's functions "
                        "(asarray/tensor or an operator), not by calling the class")

    @classmethod
    def _adopt(cls, context, buffer, shape, event=None, device=None):
        value = cls.__new__(cls)
        value._context, value._buffer, value._event, value._shape = context, buffer, event, tuple(shape)
        value._device = device if device is not None else context.device
        value._finalizer = weakref.finalize(value, _release_pair_at_collection, cls._kind, event, buffer)
        value._finalizer.atexit = False
        return value

    @property
    def closed(self):
        return self._finalizer is None or not self._finalizer.alive

    def _open(self):
        if self.closed:
            raise Error(Status.INVALID_HANDLE, type(self).__name__, f"{self._kind} used after close()")

    @property
    def shape(self):
        return self._shape

    @property
    def size(self):
        count = 1
        for extent in self._shape:
            count *= extent
        return count

    @property
    def dtype(self):
        return float32

    @property
    def nbytes(self):
        return 4 * self.size

    @property
    def device(self):
        return self._device

    @property
    def buffer(self):
        return self._buffer

    def wait(self):
        """Waits for the producing command; None when there was no GPU work."""
        self._open()
        return None if self._event is None else self._event.wait()

    def to_host(self):
        """The contents as a flat row-major array('f') (waits first)."""
        self.wait()
        out = _host_array("f")
        out.frombytes(self._buffer.read())
        return out

    def close(self):
        if self.closed:
            return
        self._finalizer.detach()
        first = None
        for owned in (self._event, self._buffer):
            if owned is None:
                continue
            try:
                owned.close()
            except Exception as error:
                first = first or error
        if first is not None:
            raise first

    def __enter__(self):
        self._open()
        return self

    def __exit__(self, *_):
        self.close()


def host_fp32(values, label):
    """A memoryview of FP32 values: a list/tuple is rounded to binary32 element by
    element; anything else must already be a C-contiguous native-endian FP32 buffer."""
    if isinstance(values, (list, tuple)):
        _int(len(values), 0, MAX_ELEMENTS, f"{label} length")
        return memoryview(_host_array("f", [f32(v).value for v in values]))
    data = memoryview(values)
    if not data.c_contiguous:
        raise ValueError(f"{label}: host values must be C-contiguous")
    if data.itemsize != 4 or data.format not in ("f", "@f", "=f", "<f"):
        raise TypeError(f"{label}: host buffer must hold native-endian FP32 values")
    return data


def upload(cls, context, data, shape):
    """A new value of `cls` on `context` holding the bytes of `data`."""
    if not isinstance(context, Context):
        raise TypeError(f"{cls.__name__} creation needs an explicit Context")
    buffer = context.buffer(data.nbytes)
    try:
        buffer.write(data)
        return cls._adopt(context, buffer, shape)
    except BaseException:
        buffer.close()
        raise


def produce(cls, context, shape, nbytes, device, enqueue):
    """A new value of `cls` whose buffer (nbytes) is filled by enqueue(buffer), which
    returns the command's Event (or None when there is no GPU work)."""
    buffer = context.buffer(nbytes)
    event = None
    try:
        event = enqueue(buffer)
        return cls._adopt(context, buffer, shape, event, device)
    except BaseException:
        try:
            if event is not None:
                event.close()
        finally:
            buffer.close()
        raise


def common_context(values, kind, what):
    """The one context of open values of type `kind` (CONTEXT_MISMATCH otherwise)."""
    for value in values:
        if not isinstance(value, kind):
            raise TypeError(f"{what} takes {kind.__name__} operands, got {type(value).__name__}")
        value._open()
    context = values[0]._context
    if any(value._context is not context for value in values[1:]):
        raise Error(Status.CONTEXT_MISMATCH, what, "operands live on different contexts")
    context.handle
    return context
