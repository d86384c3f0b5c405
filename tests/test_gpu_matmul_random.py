"""Seeded random shapes through every form of the tensor-core GEMM.

The tensor-core path picks its form from the shape and layout: 64-, 128- or 256-column
tiles, A split in shared memory or by the split pass, narrow C computed transposed, a
split k-range tail, batched tile numbering, 128-bit or 32-bit operand splits. These
cases draw sizes, transposes, batch strides and byte offsets at random (fixed seeds) in
TF32X3 mode and check every output against the oracle's float64 sums with the FP32
contract |C - exact| <= 2 k 2^-24 sum|a||b|, and that no byte outside C changes.
"""
import importlib

import numpy as np
import pytest

import oracle
import paralyn_b200 as p

pytestmark = pytest.mark.gpu
T = importlib.import_module("paralyn_b200.tensor")
CANARY = np.float32(-4321.0)


def draw(rng):
    """(batch, m, n, k, transpose_a, transpose_b, element offsets of A, B, C)."""
    batch = int(rng.choice([1, 1, 2, 3]))
    m = int(rng.choice([int(rng.integers(1, 300)), int(rng.integers(300, 1000))]))
    n = int(rng.choice([int(rng.integers(1, 140)), int(rng.integers(140, 520))]))
    k = int(rng.choice([int(rng.integers(16, 100)), int(rng.integers(100, 800))]))
    if rng.random() < 0.5:  # 16-byte aligned rows: the raw-box forms become eligible
        k = (k + 3) // 4 * 4
    offsets = [int(rng.choice([0, 0, 1, 2, 4])) for _ in range(3)]
    return batch, m, n, k, bool(rng.random() < 0.3), bool(rng.random() < 0.3), offsets


def run_case(context, seed):
    rng = np.random.default_rng(seed)
    batch, m, n, k, ta, tb, (oa, ob, oc) = draw(rng)
    res = T.operators_of(context)
    a = rng.uniform(-1, 1, batch * m * k).astype(np.float32)
    b = rng.uniform(-1, 1, batch * k * n).astype(np.float32)
    bufs = []

    def upload(values, offset):
        data = np.concatenate([np.full(offset, CANARY, np.float32), values, np.full(3, CANARY, np.float32)])
        buf = context.buffer(data.nbytes)
        buf.write(data)
        bufs.append(buf)
        return buf

    try:
        ab, bb = upload(a, oa), upload(b, ob)
        cb = upload(np.full(batch * m * n, CANARY, np.float32), oc)
        # A[z] stored [m, k] (or [k, m] when transposed), B[z] [k, n] (or [n, k]).
        a_view = (oa, (m * k, 1, m) if ta else (m * k, k, 1))
        b_view = (ob, (k * n, 1, k) if tb else (k * n, n, 1))
        if batch == 1:
            event = T.matmul_into(res.queue, res.module, T.TensorDescriptor(ab, (k, m) if ta else (m, k), 4 * oa),
                                  T.TensorDescriptor(bb, (n, k) if tb else (k, n), 4 * ob),
                                  T.TensorDescriptor(cb, (m, n), 4 * oc), m=m, n=n, k=k, transpose_a=ta,
                                  transpose_b=tb)
        else:
            event = T.batched_matmul_into(res.queue, res.module,
                                          T.TensorDescriptor(ab, (batch, m, k), 4 * oa, a_view[1]),
                                          T.TensorDescriptor(bb, (batch, k, n), 4 * ob, b_view[1]),
                                          T.TensorDescriptor(cb, (batch, m, n), 4 * oc), batch=batch, m=m, n=n, k=k)
        event.wait()
        event.close()
        out = np.frombuffer(cb.read(), np.float32)
        assert np.all(out[:oc] == CANARY) and np.all(out[oc + batch * m * n:] == CANARY), "bytes outside C changed"
        got = out[oc:oc + batch * m * n].reshape(batch, m, n).astype(np.float64)
        value, _, magnitude = oracle.batched_dot_bound(np.concatenate([np.zeros(oa, np.float32), a]), a_view,
                                                       np.concatenate([np.zeros(ob, np.float32), b]), b_view,
                                                       batch, m, n, k, magnitude=True)
        bad = np.abs(got - value) > oracle.matmul_tolerance(magnitude, k)
        assert not bad.any(), (seed, batch, m, n, k, ta, tb, oa, ob, oc, int(bad.sum()))
    finally:
        for buf in bufs:
            buf.close()


@pytest.mark.parametrize("block", range(8))
def test_random_shapes_meet_fp32_contract(context, block):
    p.set_matmul_mode(context, p.MatmulMode.TF32X3)
    try:
        for seed in range(1000 + 40 * block, 1040 + 40 * block):
            run_case(context, seed)
    finally:
        p.set_matmul_mode(context, p.MatmulMode.AUTO)
