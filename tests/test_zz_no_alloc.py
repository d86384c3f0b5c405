"""The allocation-free matmul entry point, pr_b200_matmul_tf32x3_static_f32.

It exists for callers that cannot allocate device memory (a host framework that
owns all device memory and hands over only input/output pointers, or a loop that
must not call cudaMalloc): it runs the 3xTF32 tensor-core GEMM with its split
operands in a fixed 64 MiB array inside the library instead of the per-context
workspace pr_matmul_f32 grows. Here it is called through the C ABI on device
pointers and a CUDA stream owned by the caller (torch provides both), twice in a
row with different shapes and data, and each result is compared with
pr_matmul_f32 (TF32X3 mode) on the same inputs within the FP32 GEMM tolerance
2*k*2^-24*sum|a||b| used by the other matmul tests. This file is collected last.
"""
import ctypes as c

import numpy as np
import pytest

import oracle
import paralyn_b200 as p
from paralyn_b200 import synthetic

pytestmark = pytest.mark.gpu


def static_entry():
    fn = p.library().api.pr_b200_matmul_tf32x3_static_f32
    fn.restype = c.c_int
    fn.argtypes = [c.c_void_p, c.c_void_p, c.c_void_p] + [c.c_uint64] * 6 + [c.c_uint32, c.c_uint32,
                                                                             c.c_void_p, c.c_void_p]
    return fn


def through_pr_matmul(context, a, b, m, n, k, ta, tb):
    p.set_matmul_mode(context, p.MatmulMode.TF32X3)
    with p.tensor(a, shape=(k, m) if ta else (m, k), context=context) as da, \
            p.tensor(b, shape=(n, k) if tb else (k, n), context=context) as db, \
            p.matmul(da, db, transpose_a=ta, transpose_b=tb) as dc:
        return np.asarray(dc.to_host(), np.float32).reshape(m, n)


def test_static_workspace_matches_pr_matmul_on_two_calls():
    import torch
    torch.cuda.set_device(0)
    fn = static_entry()
    stream = torch.cuda.current_stream()
    cases = ((256, 384, 512, False, False, 71), (640, 200, 1000, True, True, 72))
    with p.Context("cuda:0") as context:
        for m, n, k, ta, tb, seed in cases:
            a = synthetic.uniform(seed, 0, m * k)
            b = synthetic.uniform(seed, m * k, k * n)
            a_dev = torch.from_numpy(a).cuda()
            b_dev = torch.from_numpy(b).cuda()
            c_dev = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
            status = torch.zeros(1, dtype=torch.int32, device="cuda")
            lda, ldb = (m if ta else k), (k if tb else n)
            rc = fn(a_dev.data_ptr(), b_dev.data_ptr(), c_dev.data_ptr(), m, n, k, lda, ldb, n, int(ta), int(tb),
                    c.c_void_p(stream.cuda_stream), c.c_void_p(status.data_ptr()))
            assert rc == 0
            torch.cuda.synchronize()
            assert int(status.item()) == 0
            got = c_dev.cpu().numpy()
            want = through_pr_matmul(context, a, b, m, n, k, ta, tb)
            _, magnitude = oracle.matmul_exact(a, b, m, n, k, ta, tb)
            tolerance = oracle.matmul_tolerance(magnitude, k)
            assert np.all(np.abs(got.astype(np.float64) - want) <= tolerance)


def test_static_workspace_rejects_what_it_cannot_hold():
    fn = static_entry()
    dummy = c.c_void_p(256)  # never dereferenced: the shape checks fail first
    # 8 * 4096 * (4096 + 4096) bytes = 256 MiB > 64 MiB
    assert fn(dummy, dummy, dummy, 4096, 4096, 4096, 4096, 4096, 4096, 0, 0, None, None) == p.Status.OUT_OF_BOUNDS
    record = p.native.ErrorRecord()
    p.library().api.pr_last_error(c.byref(record))
    assert b"64 MiB" in record.message and record.operation == b"b200_matmul_tf32x3_static_f32"
    assert fn(dummy, dummy, dummy, 64, 64, 8, 8, 64, 64, 0, 0, None, None) == p.Status.UNSUPPORTED
    assert fn(None, dummy, dummy, 64, 64, 64, 64, 64, 64, 0, 0, None, None) == p.Status.INVALID_ARGUMENT
