"""The allocation-free matmul entry point, pr_b200_matmul_tf32x3_static_f32.

It exists for callers that cannot allocate device memory (a host framework that
owns all device memory and hands over only input/output pointers, or a loop that
must not call cudaMalloc): it runs the 3xTF32 tensor-core GEMM with its split
operands in a fixed 64 MiB array inside the library instead of the per-context
workspace pr_matmul_f32 grows. Here it is called through the C ABI on device
pointers and a CUDA stream owned by the caller (torch provides both), several times
in a row with different shapes and data, and each result is compared with the float64
product of the oracle within the FP32 GEMM tolerance 2*k*2^-24*sum|a||b| used by the
other matmul tests (and, as an extra check, with pr_matmul_f32 in TF32X3 mode within
twice that bound). Cases cover a C row stride that is not a multiple of four (the
kernel's scalar store path; the columns past n must stay untouched), a NULL stream
with a NULL status word, and odd m and n at a depth that fills the 64 MiB array to
within one 32-deep slice. This file is collected last.
"""
import ctypes as c

import numpy as np
import pytest

import oracle
import paralyn_b200 as p
from paralyn_b200 import synthetic

pytestmark = pytest.mark.gpu

LIMIT = 64 << 20


def static_entry():
    fn = p.library().api.pr_b200_matmul_tf32x3_static_f32
    fn.restype = c.c_int
    fn.argtypes = [c.c_void_p, c.c_void_p, c.c_void_p] + [c.c_uint64] * 6 + [c.c_uint32, c.c_uint32,
                                                                             c.c_void_p, c.c_void_p]
    return fn


def scratch_bytes(m, n, k):
    up = lambda v, to: -(-v // to) * to
    return 8 * up(k, 32) * (up(m, 128) + up(n, 256))


def through_pr_matmul(context, a, b, m, n, k, ta, tb):
    p.set_matmul_mode(context, p.MatmulMode.TF32X3)
    with p.tensor(a, shape=(k, m) if ta else (m, k), context=context) as da, \
            p.tensor(b, shape=(n, k) if tb else (k, n), context=context) as db, \
            p.matmul(da, db, transpose_a=ta, transpose_b=tb) as dc:
        return np.asarray(dc.to_host(), np.float32).reshape(m, n)


# (m, n, k, transpose_a, transpose_b, extra C columns, stream and status given, seed)
CASES = (
    (256, 384, 512, False, False, 0, True, 71),
    (640, 200, 1000, True, True, 0, True, 72),
    (200, 300, 700, False, True, 1, True, 73),     # ldc = 301: scalar stores
    (130, 17, 96, True, False, 3, False, 74),      # NULL stream, NULL status
    (17, 1, 21800, False, False, 0, False, 75),    # k_pad 21824: 8*21824*(128+256) bytes
)


def test_static_workspace_matches_the_oracle_on_calls_in_a_row():
    import torch
    torch.cuda.set_device(0)
    fn = static_entry()
    assert scratch_bytes(17, 1, 21800) <= LIMIT < scratch_bytes(17, 1, 21800 + 32)
    with p.Context("cuda:0") as context:
        for m, n, k, ta, tb, extra, given, seed in CASES:
            assert scratch_bytes(m, n, k) <= LIMIT
            a = synthetic.uniform(seed, 0, m * k)
            b = synthetic.uniform(seed, m * k, k * n)
            ldc = n + extra
            a_dev = torch.from_numpy(a).cuda()
            b_dev = torch.from_numpy(b).cuda()
            c_dev = torch.full((m, ldc), float("nan"), dtype=torch.float32, device="cuda")
            status = torch.zeros(1, dtype=torch.int32, device="cuda")
            lda, ldb = (m if ta else k), (k if tb else n)
            stream = c.c_void_p(torch.cuda.current_stream().cuda_stream) if given else None
            torch.cuda.synchronize()
            rc = fn(a_dev.data_ptr(), b_dev.data_ptr(), c_dev.data_ptr(), m, n, k, lda, ldb, ldc, int(ta), int(tb),
                    stream, c.c_void_p(status.data_ptr()) if given else None)
            assert rc == 0
            torch.cuda.synchronize()
            assert int(status.item()) == 0
            full = c_dev.cpu().numpy()
            got = full[:, :n]
            assert np.all(np.isnan(full[:, n:])), "columns past n were written"
            exact, magnitude = oracle.matmul_exact(a, b, m, n, k, ta, tb)
            tolerance = oracle.matmul_tolerance(magnitude, k)
            assert np.all(np.abs(got.astype(np.float64) - exact) <= tolerance)
            want = through_pr_matmul(context, a, b, m, n, k, ta, tb)
            assert np.all(np.abs(got.astype(np.float64) - want) <= 2 * tolerance)


def test_static_workspace_rejects_what_it_cannot_hold():
    fn = static_entry()
    dummy = c.c_void_p(256)  # never dereferenced: the shape checks fail first
    # 8 * 4096 * (4096 + 4096) bytes = 256 MiB > 64 MiB
    assert fn(dummy, dummy, dummy, 4096, 4096, 4096, 4096, 4096, 4096, 0, 0, None, None) == p.Status.OUT_OF_BOUNDS
    record = p.native.ErrorRecord()
    p.library().api.pr_last_error(c.byref(record))
    assert b"64 MiB" in record.message and record.operation == b"b200_matmul_tf32x3_static_f32"
    # one 32-deep slice past the array
    assert fn(dummy, dummy, dummy, 17, 1, 21800 + 32, 21832, 1, 1, 0, 0, None, None) == p.Status.OUT_OF_BOUNDS
    assert fn(dummy, dummy, dummy, 64, 64, 8, 8, 64, 64, 0, 0, None, None) == p.Status.UNSUPPORTED
    assert fn(None, dummy, dummy, 64, 64, 64, 64, 64, 64, 0, 0, None, None) == p.Status.INVALID_ARGUMENT
