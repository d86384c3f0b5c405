"""GPU parity of pr_matmul_f32 against the oracle.

Modes (paralyn/b200.h): REFERENCE must equal the sequential FP32 checker bit for
bit (tests/native/tensor_tests.cpp:62-85,143-146); FFMA, TF32X3 and AUTO must
satisfy the FP32 contract |C - C_exact| <= 2*K*2^-24*sum|a||b| per element.
Shapes follow the reference suite ({1,15,16,17,33,47,65,129,257,300}, all four
transpose combinations, byte offsets and canaries, tensor_tests.cpp:121-151); the
MLP output SHA-256 of docs/tensors-matmul.md:79 is reproduced in REFERENCE mode;
the 4096^3 benchmark shape is checked on sampled rows.
"""
import hashlib
import importlib

import numpy as np
import pytest

import oracle
import paralyn_b200 as p
from paralyn_b200 import synthetic

from test_oracle import MLP_OUTPUT_SHA256, mlp_inputs

pytestmark = pytest.mark.gpu
T = importlib.import_module("paralyn_b200.tensor")
SIZES = (1, 15, 16, 17, 33, 47, 65, 129, 257, 300)


def gpu_matmul(context, a, b, m, n, k, ta=False, tb=False):
    """Matmul through descriptors with 12-byte offsets and canaries (tensor_tests.cpp:126-136)."""
    res = T.operators_of(context)
    canary = np.float32(-777.0)

    def upload(values, before, after):
        data = np.concatenate([np.full(before, canary, np.float32), values.ravel(), np.full(after, canary, np.float32)])
        buf = context.buffer(data.nbytes)
        buf.write(data)
        return buf

    ab, bb = upload(a, 3, 2), upload(b, 1, 5)
    cb = upload(np.full(m * n, 12345.0, np.float32), 3, 4)
    event = T.matmul_into(res.queue, res.module, T.TensorDescriptor(ab, (k, m) if ta else (m, k), 12),
                          T.TensorDescriptor(bb, (n, k) if tb else (k, n), 4),
                          T.TensorDescriptor(cb, (m, n), 12), m=m, n=n, k=k, transpose_a=ta, transpose_b=tb)
    out = np.frombuffer(cb.read(), np.float32)
    assert np.all(out[:3] == canary) and np.all(out[-4:] == canary), "canary overwritten"
    c = out[3:3 + m * n].reshape(m, n).copy()
    for x in (event, ab, bb, cb):
        if x is not None:
            x.close()
    return event, c


@pytest.mark.parametrize("ta", (False, True))
@pytest.mark.parametrize("tb", (False, True))
def test_reference_order_is_bit_exact(context, ta, tb):
    p.set_matmul_mode(context, p.MatmulMode.REFERENCE)
    for i, (m, n, k) in enumerate([(s, t, u) for s in SIZES for t in SIZES[::3] for u in SIZES[1::3]]):
        a = synthetic.uniform(1000 + i, 0, m * k)
        b = synthetic.uniform(2000 + i, 0, k * n)
        event, c = gpu_matmul(context, a, b, m, n, k, ta, tb)
        assert event is not None
        assert c.tobytes() == oracle.matmul(a, b, m, n, k, ta, tb).tobytes(), (m, n, k, ta, tb)


@pytest.mark.parametrize("mode", (p.MatmulMode.FFMA, p.MatmulMode.TF32X3, p.MatmulMode.AUTO))
@pytest.mark.parametrize("ta,tb", ((False, False), (True, False), (False, True), (True, True)))
def test_fast_modes_meet_fp32_contract(context, mode, ta, tb):
    p.set_matmul_mode(context, mode)
    for i, (m, n, k) in enumerate(((1, 1, 1), (17, 33, 15), (129, 300, 257), (300, 129, 64), (256, 256, 512),
                                   (130, 260, 1000))):
        a = synthetic.uniform(3000 + i, 0, m * k)
        b = synthetic.uniform(4000 + i, 0, k * n)
        _, c = gpu_matmul(context, a, b, m, n, k, ta, tb)
        exact, magnitude = oracle.matmul_exact(a, b, m, n, k, ta, tb)
        bound = oracle.matmul_tolerance(magnitude, k)
        assert np.all(np.abs(c.astype(np.float64) - exact) <= bound), (mode, m, n, k)


def test_empty_and_k0(context):
    p.set_matmul_mode(context, p.MatmulMode.AUTO)
    event, c = gpu_matmul(context, np.zeros(0, np.float32), np.zeros(0, np.float32), 3, 5, 0)
    assert event is not None and np.all(c == 0.0) and not np.signbit(c).any()
    event, _ = gpu_matmul(context, np.zeros(0, np.float32), np.zeros(10, np.float32), 0, 5, 2)
    assert event is None


def test_mlp_golden_hash_on_gpu(context):
    p.set_matmul_mode(context, p.MatmulMode.REFERENCE)
    x, w1, b1, w2, b2 = mlp_inputs()
    with p.tensor(x, shape=(64, 257), context=context) as tx, p.tensor(w1, shape=(257, 130), context=context) as tw1, \
            p.tensor(b1, shape=(130,), context=context) as tb1, p.tensor(w2, shape=(130, 11), context=context) as tw2, \
            p.tensor(b2, shape=(11,), context=context) as tb2:
        with p.matmul(tx, tw1) as z1, p.bias_add(z1, tb1, relu=True) as h, p.matmul(h, tw2) as z2, \
                p.bias_add(z2, tb2) as y:
            out = np.asarray(y.to_host(), np.float32)
    assert hashlib.sha256(out.astype("<f4").tobytes()).hexdigest() == MLP_OUTPUT_SHA256


@pytest.mark.parametrize("mode", (p.MatmulMode.AUTO, p.MatmulMode.FFMA))
def test_benchmark_shape_sampled_rows(context, mode):
    # C = A B, M = N = K = 4096, A, B ~ U[-1,1) from seed 3 (one stream: A then B).
    p.set_matmul_mode(context, mode)
    m = n = k = 4096
    a = synthetic.uniform(3, 0, m * k)
    b = synthetic.uniform(3, m * k, k * n)
    with p.tensor(a, shape=(m, k), context=context) as ta, p.tensor(b, shape=(k, n), context=context) as tb, \
            p.matmul(ta, tb) as tc:
        c = np.asarray(tc.to_host(), np.float32).reshape(m, n)
    rows = np.array([0, 1, 127, 128, 2047, 4000, 4095])
    exact, magnitude = oracle.matmul_exact(a.reshape(m, k)[rows].ravel(), b, len(rows), n, k)
    assert np.all(np.abs(c[rows].astype(np.float64) - exact) <= oracle.matmul_tolerance(magnitude, k))


def test_matmul_validation(context):
    res = T.operators_of(context)
    buf = context.buffer(4096)
    d = T.TensorDescriptor
    with pytest.raises(p.Error) as error:  # C overlapping A
        T.matmul_into(res.queue, res.module, d(buf, (4, 4)), d(buf, (4, 4), 64), d(buf, (4, 4), 32), m=4, n=4, k=4)
    assert error.value.code == p.Status.INVALID_ARGUMENT and error.value.operation == "matmul_f32"
    with pytest.raises(p.Error) as error:  # C in A's allocation at disjoint bytes
        T.matmul_into(res.queue, res.module, d(buf, (4, 4)), d(buf, (4, 4), 64), d(buf, (4, 4), 1024), m=4, n=4, k=4)
    assert error.value.code == p.Status.UNSUPPORTED
    c = context.buffer(64)
    with pytest.raises(p.Error) as error:  # shape disagreement
        T.matmul_into(res.queue, res.module, d(buf, (4, 3)), d(buf, (4, 4), 64), d(c, (4, 4)), m=4, n=4, k=4)
    assert error.value.code == p.Status.INVALID_ARGUMENT
    with pytest.raises(p.Error) as error:
        T.matmul_into(res.queue, res.module, d(buf, (4, 4)), d(buf, (4, 4), 64), d(c, (4, 4)), m=4, n=4, k=4 + (1 << 31))
    assert error.value.code in (p.Status.UNSUPPORTED, p.Status.INVALID_ARGUMENT)
    c.close()
    buf.close()


@pytest.mark.parametrize("m,n,k", [(2432, 2048, 1024), (4096, 4096, 256), (4096, 4096, 40), (128 * 150, 256, 96),
                                   (2048, 1024, 1024), (512, 512, 512), (1000, 60, 4000), (5000, 128, 512),
                                   (300, 64, 4096), (256 * 150, 33, 128)])
def test_split_tail_tiles_meet_fp32_contract(context, m, n, k):
    # Tile counts just above a multiple of the 148 persistent CTAs, or below it: the
    # tiles of the last (or only), mostly idle round are cut into k-ranges whose
    # partial sums are added by a second kernel. Rows sampled from every tile row,
    # all columns checked.
    p.set_matmul_mode(context, p.MatmulMode.TF32X3)
    try:
        a = synthetic.uniform(7000 + k, 0, m * k)
        b = synthetic.uniform(8000 + k, 0, k * n)
        with p.tensor(a, shape=(m, k), context=context) as ta, p.tensor(b, shape=(k, n), context=context) as tb, \
                p.matmul(ta, tb) as tc:
            c = np.asarray(tc.to_host(), np.float32).reshape(m, n)
        rows = np.unique(np.concatenate([np.arange(0, m, 128), np.arange(127, m, 128), [m - 1]]))
        exact, magnitude = oracle.matmul_exact(a.reshape(m, k)[rows].ravel(), b, len(rows), n, k)
        assert np.all(np.abs(c[rows].astype(np.float64) - exact) <= oracle.matmul_tolerance(magnitude, k))
    finally:
        p.set_matmul_mode(context, p.MatmulMode.AUTO)


@pytest.mark.parametrize("mode", (p.MatmulMode.REFERENCE, p.MatmulMode.FFMA, p.MatmulMode.TF32X3, p.MatmulMode.AUTO))
@pytest.mark.parametrize("m,n,k,ta,tb", [(129, 65, 257, False, False), (300, 260, 96, True, False),
                                         (2432, 2048, 256, False, True), (64, 40, 0, False, False),
                                         (300, 64, 96, False, False), (1000, 100, 2048, False, True),
                                         (600, 300, 512, False, False)])
def test_fused_bias_activation_equals_two_commands(context, mode, m, n, k, ta, tb):
    # One command (GEMM epilogue adds the bias and applies the activation) against
    # pr_matmul_f32 followed by pr_bias_activation_f32: identical bits, every mode,
    # including the split tail tiles (2432 x 2048), k = 0, narrow C computed
    # transposed (n = 64 and n = 100, the latter with split k-ranges) and CTA pairs
    # converting A in shared memory (600 x 300: two column tiles), whose fused
    # epilogue runs on sixteen warps per CTA.
    p.set_matmul_mode(context, mode)
    res = T.operators_of(context)
    D = T.TensorDescriptor
    try:
        a = synthetic.uniform(900 + m, 0, m * k, 2.0)
        b = synthetic.uniform(901 + n, 0, k * n, 2.0)
        bias = synthetic.uniform(902, 0, n, 1.0)
        bufs = [context.buffer(max(16, a.nbytes)), context.buffer(max(16, b.nbytes)), context.buffer(bias.nbytes),
                context.buffer(4 * m * n), context.buffer(4 * m * n), context.buffer(4 * m * n)]
        for buf, host in zip(bufs, (a, b, bias)):
            if host.size:
                buf.write(host)
        da = D(bufs[0], (k, m) if ta else (m, k))
        db = D(bufs[1], (n, k) if tb else (k, n))
        dbias = D(bufs[2], (n,))
        for activation in (p.Activation.NONE, p.Activation.RELU, p.Activation.GELU_TANH):
            for with_bias in (True, False):
                e1 = T.matmul_into(res.queue, res.module, da, db, D(bufs[3], (m, n)), m=m, n=n, k=k,
                                   transpose_a=ta, transpose_b=tb)
                e2 = T.bias_activation_into(res.queue, res.module, D(bufs[3], (m, n)), dbias if with_bias else None,
                                            D(bufs[4], (m, n)), activation=activation)
                e3 = p.b200.matmul_bias_activation_into(res.queue, res.module, da, db, D(bufs[5], (m, n)),
                                                        dbias if with_bias else None, m=m, n=n, k=k, transpose_a=ta,
                                                        transpose_b=tb, activation=activation)
                e3.wait()
                for e in (e1, e2, e3):
                    e.close()
                two = np.frombuffer(bufs[4].read(), np.float32)
                one = np.frombuffer(bufs[5].read(), np.float32)
                assert one.tobytes() == two.tobytes(), (mode, activation, with_bias)
        for buf in bufs:
            buf.close()
    finally:
        p.set_matmul_mode(context, p.MatmulMode.AUTO)


def test_fused_mlp_reproduces_the_golden_hash(context):
    # The reference's MLP (docs/tensors-matmul.md:79) with both layers' bias (+ ReLU)
    # fused into the GEMM: the published output SHA-256 in REFERENCE mode.
    p.set_matmul_mode(context, p.MatmulMode.REFERENCE)
    res = T.operators_of(context)
    try:
        x, w1, b1, w2, b2 = mlp_inputs()
        with p.tensor(x, shape=(64, 257), context=context) as tx, p.tensor(w1, shape=(257, 130), context=context) as tw1, \
                p.tensor(b1, shape=(130,), context=context) as tb1, p.tensor(w2, shape=(130, 11), context=context) as tw2, \
                p.tensor(b2, shape=(11,), context=context) as tb2:
            h, y = context.buffer(4 * 64 * 130), context.buffer(4 * 64 * 11)
            D = T.TensorDescriptor
            e1 = p.b200.matmul_bias_activation_into(res.queue, res.module, tx.descriptor(), tw1.descriptor(),
                                                    D(h, (64, 130)), tb1.descriptor(), m=64, n=130, k=257,
                                                    activation=p.Activation.RELU)
            e2 = p.b200.matmul_bias_activation_into(res.queue, res.module, D(h, (64, 130)), tw2.descriptor(),
                                                    D(y, (64, 11)), tb2.descriptor(), m=64, n=11, k=130)
            e2.wait()
            out = np.frombuffer(y.read(), np.float32)
            for obj in (e1, e2, h, y):
                obj.close()
        assert hashlib.sha256(out.astype("<f4").tobytes()).hexdigest() == MLP_OUTPUT_SHA256
    finally:
        p.set_matmul_mode(context, p.MatmulMode.AUTO)


def aligned_matmul(context, a, b, m, n, k, ta):
    """C = op(A) B with every operand at byte offset 0 (16-byte aligned rows when k % 4 == 0)."""
    res = T.operators_of(context)
    bufs = [context.buffer(4 * x.size) for x in (a, b)] + [context.buffer(4 * m * n)]
    try:
        bufs[0].write(np.ascontiguousarray(a.T if ta else a).ravel())
        bufs[1].write(b.ravel())
        event = T.matmul_into(res.queue, res.module, T.TensorDescriptor(bufs[0], (k, m) if ta else (m, k)),
                              T.TensorDescriptor(bufs[1], (k, n)), T.TensorDescriptor(bufs[2], (m, n)),
                              m=m, n=n, k=k, transpose_a=ta)
        event.wait()
        event.close()
        return np.frombuffer(bufs[2].read(), np.float32).reshape(m, n).copy()
    finally:
        for buf in bufs:
            buf.close()


@pytest.mark.parametrize("m,n,k", [(1, 1, 16), (16, 16, 16), (129, 65, 260), (257, 100, 96), (300, 129, 64),
                                   (2048, 64, 2048), (1000, 512, 100), (4096, 200, 1024), (777, 48, 520),
                                   (37888, 64, 64)])
def test_a_split_in_shared_memory_equals_the_split_pass(context, m, n, k):
    # A stored [m, k] with 16-byte aligned rows is loaded raw and split into its TF32
    # pair inside the GEMM kernel: as the A operand when at most two column tiles
    # re-read it, as the 256-wide B operand of C^T when n <= 128 (on 64-row tiles of
    # C^T, M = 64 MMAs, when n <= 64). Stored [k, m] it goes
    # through the separate split pass into 128 x BN tiles of C. Same conversion, same
    # products in the same order and, at these sizes, the same k-ranges for the
    # split tail: equal bits. (Where the two tilings cut k differently the partial
    # sums round differently; the split-tail test bounds those cases.)
    p.set_matmul_mode(context, p.MatmulMode.TF32X3)
    try:
        a = synthetic.uniform(9100 + m, 0, m * k).reshape(m, k)
        b = synthetic.uniform(9200 + n, 0, k * n).reshape(k, n)
        raw = aligned_matmul(context, a, b, m, n, k, False)
        split = aligned_matmul(context, a, b, m, n, k, True)
        assert raw.tobytes() == split.tobytes()
        rows = np.unique(np.concatenate([np.arange(0, m, 97), [m - 1]]))
        exact, magnitude = oracle.matmul_exact(a[rows].ravel(), b.ravel(), len(rows), n, k)
        assert np.all(np.abs(raw[rows].astype(np.float64) - exact) <= oracle.matmul_tolerance(magnitude, k))
    finally:
        p.set_matmul_mode(context, p.MatmulMode.AUTO)


def test_tallest_narrow_product_runs_on_the_tensor_cores(context, tmp_path):
    # m = 1,048,560 (the most rows the reference's launch geometry, ceil(m/16) grid
    # rows, admits) x 64 x 16: computed transposed, A's rows loaded raw as the 256-wide
    # MMA side (4096 tiles of D).
    import json
    m, n, k = 65535 * 16, 64, 16
    p.set_matmul_mode(context, p.MatmulMode.TF32X3)
    try:
        a = synthetic.uniform(9300, 0, m * k)
        b = synthetic.uniform(9301, 0, k * n)
        with p.tensor(a, shape=(m, k), context=context) as ta, p.tensor(b, shape=(k, n), context=context) as tb, \
                p.matmul(ta, tb) as tc:
            c = np.asarray(tc.to_host(), np.float32).reshape(m, n)
        rows = np.unique(np.concatenate([np.arange(0, m, 9973), [m - 1]]))
        exact, magnitude = oracle.matmul_exact(a.reshape(m, k)[rows].ravel(), b, len(rows), n, k)
        assert np.all(np.abs(c[rows].astype(np.float64) - exact) <= oracle.matmul_tolerance(magnitude, k))
        context.write_evidence(str(tmp_path / "e"))
        launches = json.loads((tmp_path / "e" / "execution.json").read_text())["launches"]
        assert [l["variant"] for l in launches if l["kernel"] == "paralyn_matmul_f32"][-1] == "tcgen05_tf32x3"
    finally:
        p.set_matmul_mode(context, p.MatmulMode.AUTO)


@pytest.mark.parametrize("mode", (p.MatmulMode.REFERENCE, p.MatmulMode.FFMA, p.MatmulMode.TF32X3))
def test_nonfinite_inputs_per_mode(context, mode):
    # Row 0 of A holds +inf, row 1 a NaN, the rest finite; B is finite and nonzero.
    # REFERENCE / FFMA: row 0 is +-inf (IEEE, sequential order), row 1 NaN. An explicit
    # TF32X3 request: the infinite operand's low half is inf - inf, so row 0 is NaN as
    # well. Rows without exceptional inputs are unaffected in every mode.
    m, n, k = 130, 70, 64
    a = synthetic.uniform(9400, 0, m * k).reshape(m, k)
    b = np.abs(synthetic.uniform(9401, 0, k * n).reshape(k, n)) + np.float32(0.5)
    a[0, 5] = np.inf
    a[1, 9] = np.nan
    p.set_matmul_mode(context, mode)
    try:
        c = aligned_matmul(context, a, b, m, n, k, False)
    finally:
        p.set_matmul_mode(context, p.MatmulMode.AUTO)
    assert np.isnan(c[1]).all()
    if mode == p.MatmulMode.TF32X3:
        assert np.isnan(c[0]).all()
    else:
        assert np.all(c[0] == np.inf)
    exact, magnitude = oracle.matmul_exact(a[2:].ravel(), b.ravel(), m - 2, n, k)
    assert np.all(np.abs(c[2:].astype(np.float64) - exact) <= oracle.matmul_tolerance(magnitude, k))


def same_specials_and_contract(c, a, b, m, n, k):
    """c has the reference order's +-inf / NaN pattern (oracle sequential product) and
    its finite entries are within the FP32 contract of the float64 product."""
    want = oracle.matmul(a, b, m, n, k)
    special = ~np.isfinite(want)
    assert np.array_equal(np.isnan(c), np.isnan(want))
    assert np.array_equal(c[np.isinf(want)], want[np.isinf(want)])
    exact, magnitude = oracle.matmul_exact(a, b, m, n, k)
    finite = ~special
    assert np.all(np.isfinite(c[finite]))
    err = np.abs(c[finite].astype(np.float64) - exact[finite])
    assert np.all(err <= oracle.matmul_tolerance(magnitude, k)[finite])


# AUTO picks the 3xTF32 kernel for these shapes; an infinite operand (or one whose TF32
# high part rounds to infinity) raises the command's non-finite word in the split pass
# or in the GEMM's shared-memory converter, and the guarded FFMA kernel recomputes C in
# IEEE order, so +-inf propagate as in the reference (docs/tensors-matmul.md:80).
#   (300, 260, 96): A converted in shared memory (two column tiles), B split
#   (300, 1000, 96): both operands split
#   (4096, 100, 96): the transposed form (n <= 128: A's rows converted as the wide side)
#   (4096, 64, 96): the same on 64-row tiles (n <= 64: M = 64 MMAs)
@pytest.mark.parametrize("m,n,k", [(300, 260, 96), (300, 1000, 96), (4096, 100, 96), (4096, 64, 96)])
@pytest.mark.parametrize("where", ("a", "b", "huge"))
def test_auto_mode_propagates_infinities_like_the_reference(context, m, n, k, where):
    a = synthetic.uniform(9500, 0, m * k).reshape(m, k)
    b = synthetic.uniform(9501, 0, k * n).reshape(k, n)
    if where == "a":
        a[0, 5], a[m - 1, k - 1], a[m // 2, 0] = np.inf, -np.inf, np.nan
    elif where == "b":
        b[3, 0], b[k - 1, n - 1] = np.inf, -np.inf
    else:  # finite, but its TF32 high part rounds to infinity; every product stays finite
        a[2, 7] = np.finfo(np.float32).max
        b[7, :] = np.float32(0.25)
    p.set_matmul_mode(context, p.MatmulMode.AUTO)
    c = aligned_matmul(context, a, b, m, n, k, False)
    assert p.b200.last_variant(context, "paralyn_matmul_f32") == "tcgen05_tf32x3"
    same_specials_and_contract(c, a.ravel(), b.ravel(), m, n, k)
    if where == "huge":
        assert np.all(np.isfinite(c))


def test_auto_mode_with_finite_operands_is_the_tf32x3_result(context):
    # The guarded FFMA kernel leaves C alone when no operand held an infinity: AUTO and
    # an explicit TF32X3 request give the same bits.
    m, n, k = 300, 1000, 96
    a = synthetic.uniform(9510, 0, m * k).reshape(m, k)
    b = synthetic.uniform(9511, 0, k * n).reshape(k, n)
    results = []
    for mode in (p.MatmulMode.AUTO, p.MatmulMode.TF32X3):
        p.set_matmul_mode(context, mode)
        results.append(aligned_matmul(context, a, b, m, n, k, False))
    p.set_matmul_mode(context, p.MatmulMode.AUTO)
    assert results[0].tobytes() == results[1].tobytes()


def test_auto_mode_batched_propagates_infinities(context):
    batch, m, n, k = 3, 256, 256, 64
    a = synthetic.uniform(9520, 0, batch * m * k).reshape(batch, m, k)
    b = synthetic.uniform(9521, 0, batch * k * n).reshape(batch, k, n)
    a[1, 4, 2] = np.inf
    b[2, 9, 17] = -np.inf
    p.set_matmul_mode(context, p.MatmulMode.AUTO)
    with p.tensor(a.ravel(), shape=(batch, m, k), context=context) as ta, \
            p.tensor(b.ravel(), shape=(batch, k, n), context=context) as tb, p.batched_matmul(ta, tb) as tc:
        c = np.asarray(tc.to_host(), np.float32).reshape(batch, m, n)
    assert p.b200.last_variant(context, "paralyn_batched_matmul_f32") == "batched_tcgen05_tf32x3"
    for z in range(batch):
        want = oracle.matmul(a[z].ravel(), b[z].ravel(), m, n, k)
        if np.all(np.isfinite(want)):
            exact, magnitude = oracle.matmul_exact(a[z].ravel(), b[z].ravel(), m, n, k)
            assert np.all(np.abs(c[z] - exact) <= oracle.matmul_tolerance(magnitude, k))
        else:
            same_specials_and_contract(c[z], a[z].ravel(), b[z].ravel(), m, n, k)


# The TMA-fed SIMT kernel (gemm_simt_tma, FFMA mode): operands with 16-byte aligned
# bases and row strides (k % 4 == 0 for A stored [m][k], m % 4 == 0 for A stored
# [k][m], n % 4 == 0 for B) and B not transposed. Its k loop runs in 32-deep slices
# with zero-filled tails, every output adding its products in increasing k.
TMA_SHAPES = {False: ((1, 4, 4), (17, 132, 36), (129, 260, 100), (300, 128, 64), (257, 300, 1000), (128, 128, 32)),
              True: ((4, 4, 1), (20, 132, 33), (132, 260, 100), (300, 128, 17), (256, 300, 1000), (128, 128, 32))}


@pytest.mark.parametrize("ta", (False, True))
def test_aligned_operands_reference_order(context, ta):
    # The aligned shapes the TMA-fed kernel takes in FFMA mode, in the reference order
    # (the register-staged kernel): a rounded product, then a rounded sum, per k, bit
    # for bit as the oracle's loop.
    p.set_matmul_mode(context, p.MatmulMode.REFERENCE)
    try:
        for i, (m, n, k) in enumerate(TMA_SHAPES[ta]):
            a = synthetic.uniform(9600 + i, 0, m * k).reshape(k, m).T.copy() if ta else \
                synthetic.uniform(9600 + i, 0, m * k).reshape(m, k)
            b = synthetic.uniform(9700 + i, 0, k * n).reshape(k, n)
            c = aligned_matmul(context, a, b, m, n, k, ta)
            assert p.b200.last_variant(context, "paralyn_matmul_f32") == "simt_reference_order", (m, n, k)
            want = oracle.matmul(np.ascontiguousarray(a.T if ta else a).ravel(), b.ravel(), m, n, k, ta, False)
            assert c.tobytes() == want.tobytes(), (m, n, k, ta)
    finally:
        p.set_matmul_mode(context, p.MatmulMode.AUTO)


@pytest.mark.parametrize("ta", (False, True))
def test_tma_fed_simt_kernel_ffma_contract(context, ta):
    p.set_matmul_mode(context, p.MatmulMode.FFMA)
    try:
        for i, (m, n, k) in enumerate(TMA_SHAPES[ta]):
            a = synthetic.uniform(9800 + i, 0, m * k).reshape(m, k)
            b = synthetic.uniform(9900 + i, 0, k * n).reshape(k, n)
            c = aligned_matmul(context, a, b, m, n, k, ta)
            assert p.b200.last_variant(context, "paralyn_matmul_f32") == "simt_tma_ffma", (m, n, k)
            exact, magnitude = oracle.matmul_exact(a.ravel(), b.ravel(), m, n, k)
            assert np.all(np.abs(c.astype(np.float64) - exact) <= oracle.matmul_tolerance(magnitude, k))
    finally:
        p.set_matmul_mode(context, p.MatmulMode.AUTO)


ALIGNED_PRODUCT = """
import hashlib, sys
import numpy as np
import paralyn_b200 as p
from paralyn_b200 import synthetic
m, n, k = 4096, 4096, 2048
with p.Context("cuda:0") as ctx:
    p.set_matmul_mode(ctx, p.MatmulMode.TF32X3)
    a, b = synthetic.uniform(9700, 0, m * k), synthetic.uniform(9701, 0, k * n)
    with p.tensor(a, shape=(m, k), context=ctx) as ta, p.tensor(b, shape=(k, n), context=ctx) as tb, \\
            p.matmul(ta, tb) as tc:
        c = np.asarray(tc.to_host(), np.float32)
    rows = np.arange(0, m, 251)
    print(hashlib.sha256(c.tobytes()).hexdigest(), ",".join(map(str, rows)))
    np.save(sys.argv[1], c.reshape(m, n)[rows])
"""


def test_round_alignment_changes_no_bits(tmp_path):
    # The CTA pairs' round alignment (products with k >= 2048: 256 tiles of 256 x 256
    # here, three rounds and a split tail on 74 pairs) only delays producers; the same
    # product with it off (PARALYN_GEMM_WAVE_WAIT_US=0, read once per process) and at
    # its default gives the same bits, and sampled rows meet the FP32 contract.
    import os
    import subprocess
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    digests = []
    for wait in ("0", "50"):
        env = dict(os.environ, PARALYN_GEMM_WAVE_WAIT_US=wait)
        out = subprocess.run([sys.executable, "-c", ALIGNED_PRODUCT, str(tmp_path / f"rows{wait}.npy")], env=env,
                             cwd=root, capture_output=True, text=True, timeout=600)
        assert out.returncode == 0, out.stderr[-2000:]
        digests.append(out.stdout.split()[0])
    assert digests[0] == digests[1]
    m, n, k = 4096, 4096, 2048
    rows = np.arange(0, m, 251)
    got = np.load(tmp_path / "rows50.npy")
    a, b = synthetic.uniform(9700, 0, m * k).reshape(m, k), synthetic.uniform(9701, 0, k * n)
    exact, magnitude = oracle.matmul_exact(a[rows].ravel(), b, len(rows), n, k)
    assert np.all(np.abs(got.astype(np.float64) - exact) <= oracle.matmul_tolerance(magnitude, k))
