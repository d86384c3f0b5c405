"""CPU oracle — TEST INFRASTRUCTURE ONLY (see oracle.c for what each function
restates from the reference and where).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import
this package, and only as the parity oracle or the timed CPU baseline; the product
(paralyn_b200 and libparalyn_native.so) never does.

liboracle.so is built by `make -C oracle`; `make -C oracle ref` also builds
oracle/_ref/libref.so from the reference's own sources when the reference
checkout is present (used to pin the oracle; absent on machines without it).
"""
import ctypes as _c
from pathlib import Path
import subprocess

import numpy as np

HERE = Path(__file__).resolve().parent
LIBRARY = HERE / "liboracle.so"
REF_LIBRARY = HERE / "_ref" / "libref.so"

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
_size = _c.c_size_t
_lib = None


def build():
    subprocess.run(["make", "-s", "-C", str(HERE), "all"], check=True)


def lib():
    global _lib
    if _lib is None:
        if not LIBRARY.exists():
            build()
        _lib = _c.CDLL(str(LIBRARY))
        sig = {
            "orc_threads": (_c.c_int, []),
            "orc_set_threads": (None, [_c.c_int]),
            "orc_add_f32": (None, [_f32p, _f32p, _f32p, _size]),
            "orc_add_f32_mt": (None, [_f32p, _f32p, _f32p, _size]),
            "orc_affine_f32": (None, [_f32p, _f32p, _f32p, _size, _c.c_float]),
            "orc_affine_f32_mt": (None, [_f32p, _f32p, _f32p, _size, _c.c_float]),
            "orc_affine_scalar_f32": (None, [_f32p, _f32p, _size, _c.c_float, _c.c_float]),
            "orc_affine_scalar_f32_mt": (None, [_f32p, _f32p, _size, _c.c_float, _c.c_float]),
            "orc_tree_sum_f32": (_c.c_float, [_f32p, _size]),
            "orc_layer_norm_f32": (None, [_f32p, _f32p, _f32p, _f32p, _size, _size, _c.c_float]),
            "orc_layer_norm_f32_mt": (None, [_f32p, _f32p, _f32p, _f32p, _size, _size, _c.c_float]),
            "orc_layer_norm_bound": (None, [_f32p, _f32p, _f32p, _size, _size, _c.c_double, _f64p,
                                            _f64p, _c.c_void_p]),
            "orc_matmul_f32": (None, [_f32p, _f32p, _f32p, _size, _size, _size, _c.c_int, _c.c_int]),
            "orc_matmul_f32_rows": (None, [_f32p, _f32p, _f32p, _size, _size, _size, _c.c_int,
                                           _c.c_int, _size, _size]),
            "orc_matmul_f32_rows_mt": (None, [_f32p, _f32p, _f32p, _size, _size, _size, _c.c_int,
                                              _c.c_int, _size, _size]),
            "orc_matmul_exact": (None, [_f32p, _f32p, _f64p, _f64p, _size, _size, _size, _c.c_int,
                                        _c.c_int]),
            "orc_bias_activation_f32": (None, [_f32p, _c.c_void_p, _f32p, _size, _size, _c.c_int]),
            "orc_reduce_rows_f32": (None, [_f32p, _f32p, _size, _size, _c.c_int]),
            "orc_softmax_bound": (None, [_f32p, _size, _size, _size, _c.c_int, _c.c_float, _f64p, _f64p,
                                         _c.c_void_p]),
            "orc_batched_matmul_f32": (None, [_f32p, _View, _f32p, _View, _f32p, _View, _size, _size, _size,
                                              _size]),
            "orc_batched_dot_bound": (None, [_f32p, _View, _f32p, _View, _size, _size, _size, _size, _f64p,
                                             _f64p, _f64p]),
            "orc_gelu_bound": (None, [_f32p, _size, _f64p, _f64p]),
            "orc_softmax_rows_f32_mt": (None, [_f32p, _f32p, _size, _size, _size, _c.c_int, _c.c_float]),
            "orc_reduce_rows_f32_mt": (None, [_f32p, _f32p, _size, _size, _c.c_int]),
            "orc_batched_matmul_f32_mt": (None, [_f32p, _View, _f32p, _View, _f32p, _View, _size, _size, _size,
                                                 _size]),
        }
        for name, (restype, argtypes) in sig.items():
            f = getattr(_lib, name)
            f.restype, f.argtypes = restype, argtypes
    return _lib


def _f32(x):
    return np.ascontiguousarray(x, dtype=np.float32)


def threads():
    return lib().orc_threads()


def use_all_cores():
    """Team size = the host threads this process may run on (ignores OMP_NUM_THREADS)."""
    import os
    lib().orc_set_threads(len(os.sched_getaffinity(0)))
    return threads()


def add(a, b, threaded=False):
    a, b = _f32(a), _f32(b)
    out = np.empty_like(a)
    (lib().orc_add_f32_mt if threaded else lib().orc_add_f32)(a, b, out, a.size)
    return out


def affine(a, b, scale, threaded=False):
    a, b = _f32(a), _f32(b)
    out = np.empty_like(a)
    (lib().orc_affine_f32_mt if threaded else lib().orc_affine_f32)(a, b, out, a.size, scale)
    return out


def affine_scalar(a, scale, bias, threaded=False):
    a = _f32(a)
    out = np.empty_like(a)
    (lib().orc_affine_scalar_f32_mt if threaded else lib().orc_affine_scalar_f32)(a, out, a.size, scale, bias)
    return out


def tree_sum(x):
    x = _f32(x)
    return np.float32(lib().orc_tree_sum_f32(x, x.size))


def layer_norm(x, gamma, beta, epsilon, threaded=False):
    """Reference-order FP32 LayerNorm of x [rows, columns]."""
    x, gamma, beta = _f32(x), _f32(gamma), _f32(beta)
    rows, columns = x.shape
    out = np.empty_like(x)
    (lib().orc_layer_norm_f32_mt if threaded else lib().orc_layer_norm_f32)(
        x, gamma, beta, out, rows, columns, epsilon)
    return out


def layer_norm_bound(x, gamma, beta, epsilon):
    """(value, error) float64 arrays: |FP32 result - value| <= error."""
    x, gamma, beta = _f32(x), _f32(gamma), _f32(beta)
    rows, columns = x.shape
    value = np.empty(x.shape, np.float64)
    error = np.empty(x.shape, np.float64)
    scratch = np.empty(4 * columns + 4, np.float64)
    lib().orc_layer_norm_bound(x, gamma, beta, rows, columns, float(epsilon), value, error,
                               scratch.ctypes.data)
    return value, error


def matmul(a, b, m, n, k, transpose_a=False, transpose_b=False, rows=None, threaded=False):
    """Sequential reference-order C[m,n]; `rows` = (begin, end) computes a row range only."""
    a, b = _f32(a), _f32(b)
    c = np.zeros((m, n), np.float32)
    begin, end = rows if rows is not None else (0, m)
    (lib().orc_matmul_f32_rows_mt if threaded else lib().orc_matmul_f32_rows)(
        a, b, c, m, n, k, int(transpose_a), int(transpose_b), begin, end)
    return c


def matmul_exact(a, b, m, n, k, transpose_a=False, transpose_b=False):
    """float64 (sum a*b, sum |a*b|) per output."""
    a, b = _f32(a), _f32(b)
    exact = np.empty((m, n), np.float64)
    magnitude = np.empty((m, n), np.float64)
    lib().orc_matmul_exact(a, b, exact, magnitude, m, n, k, int(transpose_a), int(transpose_b))
    return exact, magnitude


def bias_activation(x, bias, activation):
    x = _f32(x)
    rows, columns = x.shape
    out = np.empty_like(x)
    bias_arr = _f32(bias) if bias is not None else None
    lib().orc_bias_activation_f32(x, bias_arr.ctypes.data if bias_arr is not None else None, out,
                                  rows, columns, int(activation))
    return out


def reduce_rows(x, op, threaded=False):
    """Row sums (op 0) or maxima (op 1) of x [rows, columns] in the reference's fixed order."""
    x = _f32(x)
    rows, columns = x.shape
    out = np.empty(rows, np.float32)
    (lib().orc_reduce_rows_f32_mt if threaded else lib().orc_reduce_rows_f32)(x, out, rows, columns, int(op))
    return out


def softmax_rows(x, scale, causal=False, threaded=True):
    """FP32 row softmax in the reference's order with the C library's expf (all threads,
    or one with threaded=False; a timing baseline: parity checks use softmax_bound)."""
    x = _f32(x)
    rows, columns = x.shape[-2], x.shape[-1]
    out = np.empty_like(x)
    team = threads()
    if not threaded:
        lib().orc_set_threads(1)
    try:
        lib().orc_softmax_rows_f32_mt(x, out, int(np.prod(x.shape[:-1])), rows, columns, int(bool(causal)),
                                      float(scale))
    finally:
        lib().orc_set_threads(team)
    return out


def softmax_bound(x, scale, causal=False):
    """(value, error) float64 arrays for softmax over the last axis of x [..., rows, columns]
    (causal: row i of each batch keeps i + columns - rows + 1 leading entries)."""
    x = _f32(x)
    rows, columns = x.shape[-2], x.shape[-1]
    all_rows = int(np.prod(x.shape[:-1]))
    value = np.empty(x.shape, np.float64)
    error = np.empty(x.shape, np.float64)
    scratch = np.empty(4 * columns + 4, np.float64)
    lib().orc_softmax_bound(x, all_rows, rows, columns, int(bool(causal)), float(scale), value, error,
                            scratch.ctypes.data)
    return value, error


class _View(_c.Structure):
    _fields_ = [("offset", _c.c_int64), ("s0", _c.c_int64), ("s1", _c.c_int64), ("s2", _c.c_int64)]


def batched_matmul(a, a_view, b, b_view, c, c_view, batch, m, n, k):
    """Sequential reference-order C[z] = A[z] B[z] over strided views into flat storage;
    views are (element offset, (stride0, stride1, stride2)); writes only addressed elements of c."""
    a, b = _f32(a), _f32(b)
    assert c.dtype == np.float32 and c.flags.c_contiguous
    views = [_View(off, *strides) for off, strides in (a_view, b_view, c_view)]
    lib().orc_batched_matmul_f32(a, views[0], b, views[1], c, views[2], batch, m, n, k)
    return c


def batched_matmul_threaded(a, a_view, b, b_view, c, c_view, batch, m, n, k):
    """batched_matmul over all host threads (same per-element order)."""
    a, b = _f32(a), _f32(b)
    views = [_View(off, *strides) for off, strides in (a_view, b_view, c_view)]
    lib().orc_batched_matmul_f32_mt(a, views[0], b, views[1], c, views[2], batch, m, n, k)
    return c


def batched_dot_bound(a, a_view, b, b_view, batch, m, n, k, magnitude=False):
    """(value, error) float64 [batch, m, n] for the same products; with magnitude=True
    also sum |a*b| per output (for the FP32 GEMM contract 2*k*2^-24*sum|a||b|)."""
    a, b = _f32(a), _f32(b)
    value = np.empty((batch, m, n), np.float64)
    error = np.empty((batch, m, n), np.float64)
    mag = np.empty((batch, m, n), np.float64)
    va, vb = (_View(off, *strides) for off, strides in (a_view, b_view))
    lib().orc_batched_dot_bound(a, va, b, vb, batch, m, n, k, value, error, mag)
    return (value, error, mag) if magnitude else (value, error)


def gelu_bound(x):
    """(value, error) float64 arrays of the tanh-form GELU of the FP32 inputs x."""
    x = _f32(x)
    value = np.empty(x.shape, np.float64)
    error = np.empty(x.shape, np.float64)
    lib().orc_gelu_bound(x, x.size, value, error)
    return value, error


def within(gpu, value, error):
    """The reference's acceptance rule: |gpu - value| <= error + 2^-45 |value| + 2^-126; NaN fails."""
    gpu = np.asarray(gpu, np.float64)
    return np.abs(gpu - value) <= error + 2.0 ** -45 * np.abs(value) + 1.1754943508222875e-38


def matmul_tolerance(magnitude, k):
    """Per-element bound of the FP32 GEMM contract: 2 * k * 2^-24 * sum|a||b|."""
    return 2.0 * k * 2.0 ** -24 * magnitude


# ---- the reference's own code, compiled from its sources (oracle/_ref) ----
_ref = None
REF_BINDING = HERE / "_ref" / "bindings" / "python"
REF_QUALIFY = HERE / "_ref" / "scripts" / "qualify_cuda.py"


def reference_checkout():
    """Path of the reference checkout the oracle recipe builds from (PARALYN_REFERENCE,
    else the recipe's default), or None when no checkout is there."""
    import os
    path = os.environ.get("PARALYN_REFERENCE")
    if not path:
        try:
            path = subprocess.run(["make", "-s", "--no-print-directory", "-C", str(HERE), "print-reference"],
                                  check=True, capture_output=True, text=True).stdout.strip()
        except (OSError, subprocess.CalledProcessError):
            return None
    checkout = Path(path)
    return checkout if (checkout / "include" / "paralyn" / "native.h").exists() else None


def reference():
    """oracle/_ref/libref.so, or None when it was not built here."""
    global _ref
    if _ref is None and REF_LIBRARY.exists():
        _ref = _c.CDLL(str(REF_LIBRARY))
        _ref.ref_prk_emit_cuda.restype = _c.c_int
        _ref.ref_prk_emit_cuda.argtypes = [_c.c_char_p, _c.c_size_t, _c.c_char_p, _c.c_size_t]
        _ref.ref_tree_sum_f32.restype = _c.c_float
        _ref.ref_tree_sum_f32.argtypes = [_f32p, _c.c_size_t]
        _ref.ref_layer_norm_row.restype = None
        _ref.ref_layer_norm_row.argtypes = [_f32p, _f32p, _f32p, _c.c_size_t, _c.c_double, _f64p, _f64p]
        _ref.ref_tree_max_f32.restype = _c.c_float
        _ref.ref_tree_max_f32.argtypes = [_f32p, _c.c_size_t]
        _ref.ref_softmax_row.restype = None
        _ref.ref_softmax_row.argtypes = [_f32p, _c.c_size_t, _c.c_double, _c.c_size_t, _f64p, _f64p]
        _ref.ref_dot.restype = None
        _ref.ref_dot.argtypes = [_f32p, _f32p, _c.c_size_t, _c.POINTER(_c.c_double), _c.POINTER(_c.c_double)]
        _ref.ref_gelu.restype = None
        _ref.ref_gelu.argtypes = [_f32p, _c.c_size_t, _f64p, _f64p]
    return _ref
