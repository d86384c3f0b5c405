"""Verified IR kernels that no built-in kernel implements, for the run-time
compiled path (CPU compile checks in test_jit.py, GPU runs in test_gpu_jit.py)."""
from paralyn_b200 import prk
from paralyn_b200.prk import BINARY, BOOL, CAST, F32, I32, IF, LET, LITERAL, LOAD, STORE, U32, builtin, expr, ref


def lit(value, type_):
    return expr(LITERAL, type_, str(value))


def bin_(op, type_, a, b):
    return expr(BINARY, BOOL if op == "<" else type_, op, a, b)


def load(buffer, type_, index):
    return expr(LOAD, type_, "", ref(buffer, type_), index)


def let(name, type_, value):
    return (LET, name, type_, value, None, ())


def store(buffer, type_, index, value):
    return (STORE, "", type_, value, load(buffer, type_, index), ())


def if_(condition, *body):
    return (IF, "", BOOL, condition, None, tuple(body))


def global_x(type_=U32):
    g = bin_("+", U32, bin_("*", U32, builtin("blockIdx.x"), builtin("blockDim.x")), builtin("threadIdx.x"))
    return expr(CAST, I32, "", g) if type_ == I32 else g


def strided_axpy():
    """out[2i] = x[i]*a + y[i]; out[2i+1] = v*v where v < 0 (i32 index)."""
    i, v = ref("i", I32), ref("v", F32)
    two_i = bin_("*", I32, lit(2, I32), i)
    body = (
        let("i", I32, global_x(I32)),
        if_(bin_("<", I32, i, expr(CAST, I32, "", ref("n", U32))),
            let("v", F32, bin_("+", F32, bin_("*", F32, load("x", F32, i), ref("a", F32)), load("y", F32, i))),
            store("out", F32, two_i, v),
            if_(bin_("<", F32, v, lit("0.0", F32)),
                store("out", F32, bin_("+", I32, two_i, lit(1, I32)), bin_("*", F32, v, v)))),
    )
    params = (("x", F32, True, True), ("y", F32, True, True), ("out", F32, True, False), ("n", U32, False, False),
              ("a", F32, False, False))
    return ("strided_axpy", params, body)


def integer_mix():
    """Wrapping u32 and i32 arithmetic: out_u[i] = a[i]*2654435761 + i,
    out_i[i] = b[i]*(-3) + 2147483647, out_i[n+i] = i32(a[i])."""
    i = ref("i", U32)
    body = (
        let("i", U32, global_x()),
        if_(bin_("<", U32, i, ref("n", U32)),
            store("out_u", U32, i, bin_("+", U32, bin_("*", U32, load("a", U32, i), lit(2654435761, U32)), i)),
            store("out_i", I32, i, bin_("+", I32, bin_("*", I32, load("b", I32, i), lit(-3, I32)),
                                        lit(2147483647, I32))),
            store("out_i", I32, bin_("+", U32, ref("n", U32), i), expr(CAST, I32, "", load("a", U32, i)))),
    )
    params = (("a", U32, True, True), ("b", I32, True, True), ("out_u", U32, True, False),
              ("out_i", I32, True, False), ("n", U32, False, False))
    return ("integer_mix", params, body)


def transpose_2d():
    """2-D grid: out[y*w + x] = src[x*h + y] for x < w, y < h."""
    x = bin_("+", U32, bin_("*", U32, builtin("blockIdx.x"), builtin("blockDim.x")), builtin("threadIdx.x"))
    y = bin_("+", U32, bin_("*", U32, builtin("blockIdx.y"), builtin("blockDim.y")), builtin("threadIdx.y"))
    rx, ry, w, h = ref("x", U32), ref("y", U32), ref("w", U32), ref("h", U32)
    body = (
        let("x", U32, x), let("y", U32, y),
        if_(bin_("<", U32, rx, w),
            if_(bin_("<", U32, ry, h),
                store("out", F32, bin_("+", U32, bin_("*", U32, ry, w), rx),
                      load("src", F32, bin_("+", U32, bin_("*", U32, rx, h), ry))))),
    )
    params = (("src", F32, True, True), ("out", F32, True, False), ("w", U32, False, False), ("h", U32, False, False))
    return ("transpose_2d", params, body)


def off_by_one():
    """Stores out[i + 1] under the guard i < n: the last thread addresses one past n."""
    i = ref("i", U32)
    body = (
        let("i", U32, global_x()),
        if_(bin_("<", U32, i, ref("n", U32)), store("out", F32, bin_("+", U32, i, lit(1, U32)), lit("2.5", F32))),
    )
    return ("off_by_one", (("out", F32, True, False), ("n", U32, False, False)), body)


def module(*kernels):
    return prk.serialize(list(kernels))
