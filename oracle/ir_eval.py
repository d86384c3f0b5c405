"""CPU evaluator of verified IR kernels: TEST INFRASTRUCTURE ONLY.

Restates the meaning the reference gives a verified IR kernel when it runs it
(compiler/codegen/cuda.cpp:24-80: FP32 + and * round separately as __fadd_rn and
__fmul_rn, integer + and * on 32-bit values, '<' compares, casts convert between
the integer types; compiler/ir/ir.cpp:70-180 for what verified IR may contain),
one thread at a time over a launch grid. Pure Python loops: small launches only.

Kernels are the tuples paralyn_b200.prk.serialize takes: (name, params, body) with
params (name, type, is_buffer, read_only) and statements
(kind, name, type, expression, target, body). Buffers are numpy arrays of the
parameter's element type; stores write into them. An access outside a buffer
raises IndexError (the GPU path reports it as an out-of-view access).
"""
import numpy as np

from paralyn_b200 import prk

_DTYPES = {prk.I32: np.int32, prk.U32: np.uint32, prk.F32: np.float32}


def _wrap(value, type_):
    if type_ == prk.U32:
        return int(value) & 0xFFFFFFFF
    if type_ == prk.I32:
        v = int(value) & 0xFFFFFFFF
        return v - (1 << 32) if v >= 1 << 31 else v
    return value


def _literal(type_, text):
    if type_ == prk.F32:
        return np.float32(float(text))
    if type_ == prk.BOOL:
        return text == "1"
    return _wrap(int(text), type_)


def _expr(e, env, buffers, thread):
    kind, type_, text, operands = e
    if kind == prk.LITERAL:
        return _literal(type_, text)
    if kind == prk.REF:
        return env[text]
    if kind == prk.BUILTIN:
        base, axis = text.split(".")
        return thread[base]["xyz".index(axis)]
    if kind == prk.CAST:
        return _wrap(_expr(operands[0], env, buffers, thread), type_)
    if kind == prk.BINARY:
        a = _expr(operands[0], env, buffers, thread)
        b = _expr(operands[1], env, buffers, thread)
        if text == "<":
            return bool(a < b)
        operand_type = operands[0][1]
        if operand_type == prk.F32:
            return np.float32(a + b) if text == "+" else np.float32(a * b)
        return _wrap(a + b if text == "+" else a * b, operand_type)
    if kind == prk.LOAD:
        buffer = buffers[operands[0][2]]
        index = int(_expr(operands[1], env, buffers, thread))
        if not 0 <= index < buffer.size:
            raise IndexError(f"load {operands[0][2]}[{index}] outside {buffer.size} elements")
        value = buffer[index]
        return np.float32(value) if buffer.dtype == np.float32 else int(value)
    raise ValueError(f"unknown expression kind {kind}")


def _run(body, env, buffers, thread):
    env = dict(env)
    for kind, name, type_, expression, target, inner in body:
        if kind == prk.LET:
            env[name] = _expr(expression, env, buffers, thread)
        elif kind == prk.STORE:
            buffer = buffers[target[3][0][2]]
            index = int(_expr(target[3][1], env, buffers, thread))
            value = _expr(expression, env, buffers, thread)
            if not 0 <= index < buffer.size:
                raise IndexError(f"store {target[3][0][2]}[{index}] outside {buffer.size} elements")
            buffer[index] = value
        elif _expr(expression, env, buffers, thread):
            _run(inner, env, buffers, thread)


def run(kernel, arguments, grid, block):
    """Runs `kernel` for every thread of grid x block in (z, y, x) block order and
    (z, y, x) thread order; `arguments` maps parameter names to numpy buffers or
    Python scalars. Returns the buffers (modified in place)."""
    _, params, body = kernel
    env, buffers = {}, {}
    for name, type_, is_buffer, _ in params:
        if is_buffer:
            buffers[name] = arguments[name]
            assert arguments[name].dtype == _DTYPES[type_]
        else:
            value = arguments[name]
            env[name] = np.float32(value) if type_ == prk.F32 else _wrap(value, type_)
    gx, gy, gz = grid
    bx, by, bz = block
    for z in range(gz):
        for y in range(gy):
            for x in range(gx):
                for tz in range(bz):
                    for ty in range(by):
                        for tx in range(bx):
                            thread = {"blockIdx": (x, y, z), "threadIdx": (tx, ty, tz),
                                      "blockDim": (bx, by, bz), "gridDim": (gx, gy, gz)}
                            _run(body, env, buffers, thread)
    return buffers
