"""GPU parity of the transformer-block operators: pr_batched_matmul_f32,
pr_reduce_rows_f32 and pr_softmax_rows_f32.

Cases mirror the reference's tests/native/transformer_ops_tests.cpp:113-390:
shapes, strided and broadcast views, the attention head split, element offsets
inside buffers (canary values around every output must survive), empty inputs,
and the NaN / infinity / signed-zero policies. Expectations come from the oracle,
which is pinned to the reference's own code (tests/test_oracle.py):
  * batched matmul in REFERENCE mode and row reductions: bit-identical to the
    sequential / fixed-tree FP32 order; batched matmul in AUTO and TF32X3 modes
    (FFMA or the 3xTF32 tensor-core kernel): within the FP32 GEMM contract
    |err| <= 2 k 2^-24 sum|a b|;
  * softmax: within the reference's float64 bound (exp budgeted at 4 ulp,
    division at 2.5 ulp), masked columns exactly +0.0.
Every case runs once with 16-byte-aligned rows (warp-per-row kernels) and once at
the reference's odd element offsets (block-per-row kernels).
"""
import importlib
from collections import namedtuple

import numpy as np
import pytest

import oracle
import paralyn_b200 as p
from paralyn_b200 import synthetic

pytestmark = pytest.mark.gpu
T = importlib.import_module("paralyn_b200.tensor")
CANARY = np.float32(12345.0)
View = namedtuple("View", "shape strides offset")


def contiguous3(d0, d1, d2, offset=0):
    return View((d0, d1, d2), (d1 * d2, d2, 1), offset)


def upload(context, values, offset=0):
    data = np.concatenate([np.full(offset, 777.0, np.float32), np.asarray(values, np.float32).ravel()])
    buf = context.buffer(max(16, data.nbytes))
    if data.size:
        buf.write(data)
    return buf


def output(context, count):
    buf = context.buffer(max(16, 4 * count))
    buf.write(np.full(max(4, count), CANARY, np.float32))
    return buf


def read(buf, count):
    return np.frombuffer(buf.read(), np.float32)[:count].copy()


def descriptor(buf, view):
    return T.TensorDescriptor(buf, view.shape, 4 * view.offset, view.strides)


@pytest.fixture()
def ops(context):
    return T.operators_of(context)


# ---------------------------------------------------------------- batched matmul
def batched_case(context, ops, mode, batch, m, n, k, av, a, bv, b, cv, c_storage):
    p.set_matmul_mode(context, mode)
    bufs = [upload(context, a), upload(context, b), output(context, c_storage)]
    try:
        event = T.batched_matmul_into(ops.queue, ops.module, descriptor(bufs[0], av), descriptor(bufs[1], bv),
                                      descriptor(bufs[2], cv), batch=batch, m=m, n=n, k=k)
        got = read(bufs[2], c_storage)
        want = np.full(c_storage, CANARY, np.float32)
        if not batch * m * n:
            assert event is None and got.tobytes() == want.tobytes()
            return
        event.wait()
        event.close()
        oracle.batched_matmul(a, (av.offset, av.strides), b, (bv.offset, bv.strides), want,
                              (cv.offset, cv.strides), batch, m, n, k)
        if mode == p.MatmulMode.REFERENCE:
            assert got.tobytes() == want.tobytes()
            return
        addressed = np.zeros(c_storage, bool)
        index = (cv.offset + np.arange(batch)[:, None, None] * cv.strides[0]
                 + np.arange(m)[None, :, None] * cv.strides[1] + np.arange(n)[None, None, :] * cv.strides[2])
        addressed[index.ravel()] = True
        assert got[~addressed].tobytes() == want[~addressed].tobytes()  # canaries untouched
        value, _, magnitude = oracle.batched_dot_bound(a, (av.offset, av.strides), b, (bv.offset, bv.strides),
                                                       batch, m, n, k, magnitude=True)
        assert np.all(np.abs(got[index] - value) <= oracle.matmul_tolerance(magnitude, k))
    finally:
        p.set_matmul_mode(context, p.MatmulMode.AUTO)
        for buf in bufs:
            buf.close()


BATCHED_SHAPES = [(1, 1, 1, 1), (3, 17, 13, 5), (4, 33, 31, 47), (2, 1, 65, 16), (1, 16, 16, 16),
                  (2, 129, 70, 257), (5, 16, 17, 0), (0, 4, 4, 4), (3, 0, 5, 2), (3, 5, 0, 2), (1, 1, 1, 300),
                  (8, 128, 128, 64), (6, 200, 136, 72), (3, 300, 520, 96)]
MODES = [p.MatmulMode.REFERENCE, p.MatmulMode.AUTO, p.MatmulMode.TF32X3]


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("shape", BATCHED_SHAPES)
def test_batched_matmul_layouts(context, ops, mode, shape):
    batch, m, n, k = shape
    seed = 100 + BATCHED_SHAPES.index(shape)
    a = synthetic.uniform(seed, 0, 3 + batch * m * k)
    b = synthetic.uniform(seed, 1 << 30, 1 + batch * k * n)
    # contiguous views at element offsets 3 / 1 / 2
    batched_case(context, ops, mode, batch, m, n, k, contiguous3(batch, m, k, 3), a, contiguous3(batch, k, n, 1), b,
                 contiguous3(batch, m, n, 2), 2 + batch * m * n)
    # B stored [batch, n, k] and viewed as [batch, k, n]
    bt = View((batch, k, n), (n * k, 1, k), 0)
    batched_case(context, ops, mode, batch, m, n, k, contiguous3(batch, m, k), a, bt, b, contiguous3(batch, m, n),
                 batch * m * n)
    if batch > 1 and k:  # B broadcast over the batch (stride 0)
        batched_case(context, ops, mode, batch, m, n, k, contiguous3(batch, m, k), a, View((batch, k, n), (0, n, 1), 0),
                     b, contiguous3(batch, m, n), batch * m * n)


@pytest.mark.parametrize("mode", MODES)
def test_batched_matmul_attention_views(context, ops, mode):
    # QKV stored [T, 3HD]; Q_h [H,T,D] and K_h^T [H,D,T] are strided views, the scores
    # are contiguous [H,T,T]; probs x V_h lands in head-concatenated [T, HD] columns.
    T_, H, D = 19, 3, 7
    W = 3 * H * D
    qkv = synthetic.uniform(77, 0, T_ * W)
    batched_case(context, ops, mode, H, T_, T_, D, View((H, T_, D), (D, W, 1), 0), qkv,
                 View((H, D, T_), (D, 1, W), H * D), qkv, contiguous3(H, T_, T_), H * T_ * T_)
    probs = synthetic.uniform(78, 0, H * T_ * T_)
    batched_case(context, ops, mode, H, T_, D, T_, contiguous3(H, T_, T_), probs,
                 View((H, T_, D), (D, W, 1), 2 * H * D), qkv, View((H, T_, D), (D, H * D, 1), 0), T_ * H * D)
    # a column-major output and operands that are neither rows nor columns (generic kernel)
    a = synthetic.uniform(79, 0, 2 * 9 * 5 * 2)
    b = synthetic.uniform(80, 0, 2 * 5 * 6 * 3)
    batched_case(context, ops, mode, 2, 9, 6, 5, View((2, 9, 5), (90, 10, 2), 0), a, View((2, 5, 6), (90, 18, 3), 0), b,
                 View((2, 9, 6), (54, 1, 9), 0), 2 * 54)


def test_batched_matmul_zero_depth_fills_addressed_elements(context, ops):
    batched_case(context, ops, p.MatmulMode.AUTO, 2, 3, 4, 0, contiguous3(2, 3, 0), np.zeros(1, np.float32),
                 contiguous3(2, 0, 4), np.zeros(1, np.float32), View((2, 3, 4), (40, 10, 2), 1), 80)


def test_batched_matmul_rejects_overlapping_outputs(context, ops):
    a, b, c = upload(context, np.ones(8)), upload(context, np.ones(8)), output(context, 16)
    try:
        with pytest.raises(p.Error) as error:
            T.batched_matmul_into(ops.queue, ops.module, descriptor(a, contiguous3(2, 2, 2)),
                                  descriptor(b, contiguous3(2, 2, 2)), descriptor(c, View((2, 2, 2), (1, 2, 1), 0)),
                                  batch=2, m=2, n=2, k=2)
        assert error.value.code == p.Status.INVALID_ARGUMENT
    finally:
        for buf in (a, b, c):
            buf.close()


# ---------------------------------------------------------------- row reductions
REDUCE_SHAPES = [(1, 1), (3, 255), (5, 256), (2, 257), (7, 1000), (64, 3), (4, 0), (0, 5), (1, 100003), (2, 513),
                 (300, 4096), (1000, 64)]


def reduce_case(context, ops, x, rows, cols, op, x_offset, out_offset):
    xb, ob = upload(context, x, x_offset), output(context, out_offset + rows)
    try:
        xd = T.TensorDescriptor(xb, (rows, cols), 4 * x_offset)
        od = T.TensorDescriptor(ob, (rows,), 4 * out_offset)
        event = T.reduce_rows_into(ops.queue, ops.module, xd, od, op=op)
        got = read(ob, out_offset + rows)
        if not rows:
            assert event is None
            return
        event.wait()
        event.close()
        assert np.all(got[:out_offset] == CANARY)
        want = oracle.reduce_rows(np.asarray(x, np.float32).reshape(rows, cols), int(op))
        got = got[out_offset:]
        assert np.array_equal(np.isnan(got), np.isnan(want))
        finite = ~np.isnan(want)
        assert got[finite].tobytes() == want[finite].tobytes()
    finally:
        xb.close()
        ob.close()


@pytest.mark.parametrize("offsets", [(0, 0), (5, 1)])
@pytest.mark.parametrize("op", [p.Reduce.SUM, p.Reduce.MAX])
@pytest.mark.parametrize("shape", REDUCE_SHAPES)
def test_reduce_rows_fixed_order(context, ops, shape, op, offsets):
    rows, cols = shape
    x = synthetic.uniform(300 + REDUCE_SHAPES.index(shape), 0, rows * cols, 4.0)
    reduce_case(context, ops, x, rows, cols, op, *offsets)


@pytest.mark.parametrize("cols", [1000, 70001, 4096])
def test_reduce_rows_mixed_magnitudes(context, ops, cols):
    rows = 3
    x = synthetic.uniform(390 + cols, 0, rows * cols, 1.0)
    x = (x / np.float32(3.0) * np.ldexp(np.float32(1.0), (np.arange(x.size) % 41) - 20).astype(np.float32))
    x = x.astype(np.float32)
    for offsets in ((0, 0), (1, 0)):
        reduce_case(context, ops, x, rows, cols, p.Reduce.SUM, *offsets)


@pytest.mark.parametrize("cols", [700, 2048])
def test_reduce_rows_specials_in_long_rows(context, ops, cols):
    # The same special values spread over several 256-column chunks: each reference
    # lane's chain, the tree and the NaN / signed-zero rules must hold across chunks.
    nan, inf = np.nan, np.inf
    rng = np.random.default_rng(cols)
    x = rng.uniform(-2, 2, (6, cols)).astype(np.float32)
    x[0, cols - 5] = nan
    x[1, :] = -0.0
    x[1, 257] = 0.0
    x[2, :] = -0.0
    x[3, 3] = inf
    x[3, cols - 1] = -inf
    x[4, :] = -inf
    x[5, 100] = inf
    x[5, 600 % cols] = inf
    for offsets in ((0, 0), (1, 3)):
        for op in (p.Reduce.SUM, p.Reduce.MAX):
            reduce_case(context, ops, x.ravel(), 6, cols, op, *offsets)


def test_reduce_rows_specials(context, ops):
    nan, inf = np.nan, np.inf
    x = np.array([[1, nan, -2, 3], [-0.0, 0.0, -0.0, -1], [-0.0, -0.0, -3, -1], [inf, -inf, 1, 2],
                  [-inf, -inf, -inf, -inf], [inf, 1, inf, 0]], np.float32)
    for offsets in ((0, 0), (1, 3)):
        for op in (p.Reduce.SUM, p.Reduce.MAX):
            reduce_case(context, ops, x, 6, 4, op, *offsets)


# ---------------------------------------------------------------- softmax
SOFTMAX_CASES = [(1, 1, 1, 1.0, 4.0, False, False), (1, 3, 17, 1.0, 4.0, False, False),
                 (1, 5, 256, 0.125, 16.0, False, False), (1, 2, 1000, 1.0, 8.0, False, False),
                 (1, 1, 100003, 1.0, 30.0, False, False), (4, 9, 9, 0.35355339, 8.0, True, True),
                 (2, 5, 12, 1.0, 8.0, True, True), (3, 7, 7, 3.0, 4.0, False, True), (1, 1, 300, 1.0, 100.0, True, False),
                 (1, 17, 17, 1.0, 60.0, True, False), (1, 0, 5, 1.0, 1.0, False, False), (1, 3, 0, 1.0, 1.0, False, False),
                 (0, 3, 3, 1.0, 1.0, True, True), (8, 128, 128, 0.125, 8.0, True, True), (2, 64, 2048, 1.0, 8.0, False, True),
                 (1, 33, 4096, 1.0, 8.0, False, False), (2, 40, 2048, 0.125, 8.0, True, True),
                 (1, 1300, 1300, 1.0, 8.0, True, False), (1, 20, 3000, 1.0, 8.0, True, False)]


def softmax_case(context, ops, x, batch, rows, cols, scale, causal, rank3, x_offset, out_offset):
    shape = (batch, rows, cols) if rank3 else (rows, cols)
    count = batch * rows * cols
    xb, ob = upload(context, x, x_offset), output(context, out_offset + count)
    try:
        event = T.softmax_rows_into(ops.queue, ops.module, T.TensorDescriptor(xb, shape, 4 * x_offset),
                                    T.TensorDescriptor(ob, shape, 4 * out_offset), scale=scale, causal=causal)
        got = read(ob, out_offset + count)
        if not count:
            assert event is None
            return None
        event.wait()
        event.close()
        assert np.all(got[:out_offset] == CANARY)
        return got[out_offset:].reshape(batch * rows, cols)
    finally:
        xb.close()
        ob.close()


@pytest.mark.parametrize("offsets", [(0, 0), (2, 1)])
@pytest.mark.parametrize("case", SOFTMAX_CASES)
def test_softmax_within_reference_bound(context, ops, case, offsets):
    batch, rows, cols, scale, magnitude, causal, rank3 = case
    if not rank3:
        batch = 1
    x = synthetic.uniform(500 + SOFTMAX_CASES.index(case), 0, batch * rows * cols, magnitude)
    got = softmax_case(context, ops, x, batch, rows, cols, scale, causal, rank3, *offsets)
    if got is None:
        return
    value, error = oracle.softmax_bound(x.reshape(batch, rows, cols), np.float32(scale), causal)
    value, error = value.reshape(got.shape), error.reshape(got.shape)
    visible = np.ones(got.shape, bool)
    if causal:
        r = np.arange(batch * rows) % rows
        visible = np.arange(cols)[None, :] < (r + (cols - rows) + 1)[:, None]
    assert got[~visible].tobytes() == np.zeros(int((~visible).sum()), np.float32).tobytes()
    assert np.all(oracle.within(got[visible], value[visible], error[visible]))


def test_softmax_specials(context, ops):
    nan, inf = np.nan, np.inf
    x = np.array([[1, nan, 2, 0.5], [1, inf, 2, 0.5], [-inf, -inf, -inf, -inf], [0, -inf, 0, -inf]], np.float32)
    for offsets in ((0, 0), (2, 1)):
        got = softmax_case(context, ops, x, 1, 4, 4, 1.0, False, False, *offsets)
        assert np.all(np.isnan(got[:3]))
        assert got[3, 1] == 0.0 and not np.signbit(got[3, 1]) and got[3, 3] == 0.0 and not np.signbit(got[3, 3])
        half_v, half_e = oracle.softmax_bound(np.zeros((1, 2), np.float32), 1.0)
        assert np.all(oracle.within(got[3, [0, 2]], half_v.ravel(), half_e.ravel()))
        # causal: a NaN in a masked position never enters the row
        got = softmax_case(context, ops, np.array([1, nan, 2, 3], np.float32), 1, 2, 2, 1.0, True, False, *offsets)
        assert got[0, 0] == 1.0 and got[0, 1] == 0.0 and not np.isnan(got[1]).any()
        # scale * x overflows to +inf: a NaN row
        got = softmax_case(context, ops, np.array([3e38, 1.0], np.float32), 1, 1, 2, 4.0, False, False, *offsets)
        assert np.isnan(got).all()


@pytest.mark.parametrize("cols", [600, 1024, 2048, 2052])
def test_softmax_specials_in_long_rows(context, ops, cols):
    # Rows over 512 columns take the three-pass streamed kernel (the offset case the
    # one-block-per-row kernel): a NaN or +inf in any
    # visible column makes the row NaN, an all -inf row is NaN, -inf entries of a
    # finite row become +0.0, and a NaN in a causally masked column never enters.
    nan, inf = np.nan, np.inf
    rng = np.random.default_rng(cols)
    x = rng.uniform(-4, 4, (6, cols)).astype(np.float32)
    x[0, cols - 3] = nan
    x[1, 300] = inf
    x[2, :] = -inf
    x[3, ::3] = -inf
    x[4, cols // 2] = nan  # row 4 of 6 with causal masking sees cols - 1 columns
    x[5, 7] = -inf
    for offsets in ((0, 0), (2, 1)):
        got = softmax_case(context, ops, x, 1, 6, cols, 0.5, False, False, *offsets)
        assert np.all(np.isnan(got[:3]))
        assert np.all(got[3, ::3] == 0.0) and not np.any(np.signbit(got[3, ::3]))
        value, error = oracle.softmax_bound(x[3:], np.float32(0.5))
        assert np.all(oracle.within(got[3:6][:, :], value, error)[np.isfinite(value)])
        # causal over 6 rows: row r keeps r + cols - 6 + 1 leading columns
        xc = x.copy()
        xc[4, cols - 1] = nan  # masked for row 4 (it keeps cols - 1 columns)
        xc[4, cols // 2] = 1.0
        got = softmax_case(context, ops, xc, 1, 6, cols, 0.5, True, False, *offsets)
        assert not np.isnan(got[4]).any() and got[4, cols - 1] == 0.0
        vc, ec = oracle.softmax_bound(xc, np.float32(0.5), causal=True)
        assert np.all(oracle.within(got[4], vc[4], ec[4]))


@pytest.mark.parametrize("scale,causal,shape,code", [
    (0.0, False, (2, 4), p.Status.INVALID_ARGUMENT), (float("inf"), False, (2, 4), p.Status.INVALID_ARGUMENT),
    (1.0, True, (4, 2), p.Status.INVALID_ARGUMENT)])
def test_softmax_rejections(context, ops, scale, causal, shape, code):
    xb, ob = upload(context, np.ones(8)), output(context, 8)
    try:
        with pytest.raises(p.Error) as error:
            T.softmax_rows_into(ops.queue, ops.module, T.TensorDescriptor(xb, shape), T.TensorDescriptor(ob, shape),
                                scale=scale, causal=causal)
        assert error.value.code == code
    finally:
        xb.close()
        ob.close()


def test_high_level_helpers(context):
    x = synthetic.uniform(900, 0, 6 * 40, 3.0).reshape(6, 40)
    with p.tensor(x.ravel(), shape=(6, 40), context=context) as t, p.row_sum(t) as s, p.row_max(t) as m, \
            p.softmax(t, scale=0.5) as y:
        assert np.asarray(s.to_host(), np.float32).tobytes() == oracle.reduce_rows(x, 0).tobytes()
        assert np.asarray(m.to_host(), np.float32).tobytes() == oracle.reduce_rows(x, 1).tobytes()
        value, error = oracle.softmax_bound(x.reshape(1, 6, 40), np.float32(0.5))
        assert np.all(oracle.within(np.asarray(y.to_host(), np.float32), value.ravel(), error.ravel()))
    a = synthetic.uniform(901, 0, 2 * 5 * 3).reshape(2, 5, 3)
    b = synthetic.uniform(902, 0, 2 * 3 * 4).reshape(2, 3, 4)
    p.set_matmul_mode(context, p.MatmulMode.REFERENCE)
    try:
        with p.tensor(a.ravel(), shape=(2, 5, 3), context=context) as ta, \
                p.tensor(b.ravel(), shape=(2, 3, 4), context=context) as tb, p.batched_matmul(ta, tb) as c:
            want = np.zeros(40, np.float32)
            oracle.batched_matmul(a, (0, (15, 3, 1)), b, (0, (12, 4, 1)), want, (0, (20, 4, 1)), 2, 5, 4, 3)
            assert np.asarray(c.to_host(), np.float32).tobytes() == want.tobytes()
    finally:
        p.set_matmul_mode(context, p.MatmulMode.AUTO)
