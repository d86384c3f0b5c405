"""Writer for the verified-IR module container (.prk) used by the array operators.

The reference builds operators.prk by compiling bindings/python/operators.cu with
its Clang frontend (bindings/python/operators.cu:3-16). This library has no frontend:
the same kernels are constructed here as IR trees, exactly as the reference's
codegen tests build them by hand (tests/cuda/codegen_tests.cpp:53-76), and written
in container format 1 (compiler/ir/artifact.cpp:248-273: magic "PARALYN\\0",
u32 format 1, u32 numerical policy 1, kernels as length-prefixed little-endian
records). The native library maps these kernels to sm_100a kernels at load time.

Kernels written: array_add(a, b, out, n) and array_affine(a, b, out, n, scale)
as in the reference, plus array_affine_scalar(a, out, n, scale, bias), the affine
map with a scalar addend (8 bytes of HBM traffic per element instead of 12).
"""
from pathlib import Path
import struct

MAGIC = b"PARALYN\0"
FORMAT, POLICY = 1, 1
I32, U32, F32, BOOL = 0, 1, 2, 3
LITERAL, REF, BUILTIN, BINARY, CAST, LOAD = range(6)
LET, STORE, IF = range(3)


def expr(kind, type_, text="", *operands):
    return (kind, type_, text, tuple(operands))


def ref(name, type_):
    return expr(REF, type_, name)


def builtin(name):
    return expr(BUILTIN, U32, name)


def binary(op, type_, a, b):
    return expr(BINARY, type_, op, a, b)


def load(buffer, index):
    return expr(LOAD, F32, "", ref(buffer, F32), index)


def elementwise(name, params, value, index_type=U32):
    """Kernel: i = blockIdx.x * blockDim.x + threadIdx.x; if (i < n) out[i] = value(i)."""
    glob = binary("+", U32, binary("*", U32, builtin("blockIdx.x"), builtin("blockDim.x")),
                  builtin("threadIdx.x"))
    if index_type == I32:
        glob = expr(CAST, I32, "", glob)
    i = ref("i", index_type)
    let = (LET, "i", index_type, glob, None, ())
    store = (STORE, "", F32, value(i), load("out", i), ())
    guard = (IF, "", BOOL, binary("<", BOOL, i, ref("n", index_type)), None, (store,))
    return (name, tuple(params), (let, guard))


def operators():
    """The array operator kernels (names and parameter lists of operators.cu)."""
    ab = [("a", F32, True, True), ("b", F32, True, True), ("out", F32, True, False), ("n", U32, False, False)]
    add = elementwise("array_add", ab, lambda i: binary("+", F32, load("a", i), load("b", i)))
    affine = elementwise(
        "array_affine", ab + [("scale", F32, False, False)],
        lambda i: binary("+", F32, binary("*", F32, load("a", i), ref("scale", F32)), load("b", i)))
    scalar = elementwise(
        "array_affine_scalar",
        [("a", F32, True, True), ("out", F32, True, False), ("n", U32, False, False),
         ("scale", F32, False, False), ("bias", F32, False, False)],
        lambda i: binary("+", F32, binary("*", F32, load("a", i), ref("scale", F32)), ref("bias", F32)))
    return [add, affine, scalar]


def _u32(value):
    return struct.pack("<I", value)


def _string(text):
    data = text.encode()
    if len(data) > 4096 or b"\0" in data:
        raise ValueError("artifact strings are at most 4096 bytes without NUL")
    return _u32(len(data)) + data


def _expr(e):
    kind, type_, text, operands = e
    out = _u32(kind) + _u32(type_) + _string(text) + _u32(0) + _u32(0) + _u32(len(operands))
    return out + b"".join(_expr(o) for o in operands)


def _body(statements):
    out = _u32(len(statements))
    for kind, name, type_, expression, target, body in statements:
        out += _u32(kind)
        if kind == LET:
            out += _string(name) + _u32(type_) + _expr(expression)
        elif kind == STORE:
            out += _u32(type_) + _expr(expression) + _expr(target)
        else:
            out += _expr(expression) + _body(body)
    return out


def serialize(kernels):
    """Container bytes for (name, params, body) kernels; params are
    (name, type, is_buffer, read_only)."""
    if not kernels:
        raise ValueError("module contains no kernels")
    out = MAGIC + _u32(FORMAT) + _u32(POLICY) + _u32(len(kernels))
    for name, params, body in kernels:
        out += _string(name) + _u32(len(params))
        for pname, ptype, is_buffer, read_only in params:
            out += _string(pname) + _u32(ptype) + _u32((1 if is_buffer else 0) | (2 if read_only else 0))
        out += _body(body)
    return out


def write_operators(path):
    path = Path(path)
    data = serialize(operators())
    if not path.exists() or path.read_bytes() != data:
        path.parent.mkdir(parents=True, exist_ok=True)
        path.write_bytes(data)
    return path
