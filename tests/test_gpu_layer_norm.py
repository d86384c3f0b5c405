"""GPU parity of row LayerNorm (pr_layer_norm_f32) against the oracle.

Expected results: bit-exact with the oracle's reference-order FP32 LayerNorm
(runtime/tensor.cpp:276-299), and inside the reference's float64 bound
(examples/native/transformer_reference.hpp:133-157, pinned in
tests/golden/reference_vectors.npz). Cases: the shapes, centers and epsilons of
tests/native/transformer_ops_tests.cpp:397-400, the non-finite policy of :428-445,
the 16384 x 4096 benchmark configuration, and widths that exercise both the
warp-per-row and the block-per-row kernels.
"""
import importlib
from pathlib import Path

import numpy as np
import pytest

import oracle
import paralyn_b200 as p
from paralyn_b200 import synthetic

pytestmark = pytest.mark.gpu
GOLDEN = np.load(Path(__file__).with_name("golden") / "reference_vectors.npz")
T = importlib.import_module("paralyn_b200.tensor")
LN_KEYS = sorted({k.rsplit("_", 1)[0] for k in GOLDEN.files if k.startswith("ln_")})


def run(context, x, g, b, eps, pads=(1, 0, 3, 2)):
    """LayerNorm through descriptors with byte offsets and canaries around the output."""
    rows, cols = x.shape
    t = T
    res = t.operators_of(context)
    canary = np.float32(-777.0)

    def upload(values, pad):
        data = np.concatenate([np.full(pad, canary, np.float32), values.ravel(), np.full(2, canary, np.float32)])
        buf = context.buffer(data.nbytes)
        buf.write(data)
        return buf

    xb, gb, bb = upload(x, pads[0]), upload(g, pads[1]), upload(b, pads[2])
    ob = upload(np.zeros(rows * cols, np.float32), pads[3])
    event = t.layer_norm_into(res.queue, res.module, t.TensorDescriptor(xb, (rows, cols), 4 * pads[0]),
                              t.TensorDescriptor(gb, (cols,), 4 * pads[1]),
                              t.TensorDescriptor(bb, (cols,), 4 * pads[2]),
                              t.TensorDescriptor(ob, (rows, cols), 4 * pads[3]), epsilon=float(eps))
    out = np.frombuffer(ob.read(), np.float32)
    assert np.all(out[:pads[3]] == canary) and np.all(out[-2:] == canary)
    result = out[pads[3]:pads[3] + rows * cols].reshape(rows, cols).copy()
    for x_ in (event, xb, gb, bb, ob):
        if x_ is not None:
            x_.close()
    return event, result


@pytest.mark.parametrize("key", LN_KEYS)
def test_reference_cases_bit_exact_and_within_bound(context, key):
    x, g, b = GOLDEN[key + "_x"], GOLDEN[key + "_gamma"], GOLDEN[key + "_beta"]
    eps = GOLDEN[key + "_eps"][0]
    _, out = run(context, x, g, b, eps)
    assert out.tobytes() == oracle.layer_norm(x, g, b, eps).tobytes()
    value, error = GOLDEN[key + "_value"], GOLDEN[key + "_error"]
    assert np.all(np.abs(out.astype(np.float64) - value) <= error + 2.0 ** -45 * np.abs(value) + 1.2e-38)


@pytest.mark.parametrize("rows,cols", [(5, 1000), (1, 100003), (7, 4096), (3, 4100), (9, 2048), (2, 12),
                                       (33, 768), (4, 8192), (6, 257)])
def test_widths_bit_exact(context, rows, cols):
    x = (synthetic.normal(21, 0, rows * cols, 0.5, 3.0)).reshape(rows, cols)
    g, b = synthetic.normal(22, 0, cols, 1.0, 0.5), synthetic.normal(23, 0, cols, 0.0, 0.5)
    _, out = run(context, x, g, b, np.float32(1e-5))
    assert out.tobytes() == oracle.layer_norm(x, g, b, np.float32(1e-5)).tobytes()


def test_nonfinite_policy(context):
    nan, inf = np.float32("nan"), np.float32("inf")
    x = np.array([[1, nan, 2, 3], [1, inf, 2, 3], [5, 5, 5, 5], [1, 2, 3, 4]], np.float32)
    g = np.array([1, 2, nan, 1], np.float32)
    b = np.array([0.25, -0.5, 0, nan], np.float32)
    _, out = run(context, x, g, b, np.float32(1e-5))
    assert np.isnan(out[:2]).all()
    assert out[2, 0] == 0.25 and out[2, 1] == -0.5 and np.isnan(out[2, 2:]).all()
    assert not np.isnan(out[3, :2]).any() and np.isnan(out[3, 2:]).all()


@pytest.mark.parametrize("cols", [2048, 4096])
def test_nonfinite_policy_in_wide_rows(context, cols):
    # The same policy on the shared-memory streamed kernel (1024 < columns <= 4096):
    # NaN / inf rows are all NaN, a constant row is exactly beta, and a NaN in gamma or
    # beta reaches only its column; finite results equal the oracle bit for bit.
    nan, inf = np.float32("nan"), np.float32("inf")
    x = synthetic.normal(24, 0, 4 * cols, 0.5, 2.0).reshape(4, cols)
    x[0, 1500] = nan
    x[1, 3] = inf
    x[2, :] = 5.0
    g = synthetic.normal(25, 0, cols, 1.0, 0.25)
    b = synthetic.normal(26, 0, cols, 0.0, 0.25)
    g[2000 % cols] = nan
    b[cols - 7] = nan
    _, out = run(context, x, g, b, np.float32(1e-5))
    want = oracle.layer_norm(x, g, b, np.float32(1e-5))
    assert np.isnan(out[:2]).all()
    bad = np.zeros(cols, bool)
    bad[[2000 % cols, cols - 7]] = True
    assert np.isnan(out[2:, bad]).all() and not np.isnan(out[2:, ~bad]).any()
    assert out[2, ~bad].tobytes() == b[~bad].tobytes()
    assert np.array_equal(np.isnan(out), np.isnan(want))
    assert out[~np.isnan(want)].tobytes() == want[~np.isnan(want)].tobytes()


def test_empty_shapes_make_no_event(context):
    for rows, cols in ((0, 8), (3, 0)):
        x = np.zeros((rows, cols), np.float32)
        event, _ = run(context, x, np.zeros(cols, np.float32), np.zeros(cols, np.float32), 1e-5)
        assert event is None


def test_benchmark_configuration_bit_exact(context):
    # X[16384 x 4096] ~ N(0,1), gamma ~ N(1,0.02), beta ~ N(0,0.02), eps 1e-5, seed 2.
    rows, cols = 16384, 4096
    x = synthetic.normal(2, 0, rows * cols).reshape(rows, cols)
    g = synthetic.normal(2, 2 * rows * cols, cols, 1.0, 0.02)
    b = synthetic.normal(2, 2 * rows * cols + 2 * cols, cols, 0.0, 0.02)
    with p.tensor(x, shape=(rows, cols), context=context) as tx, \
            p.tensor(g, shape=(cols,), context=context) as tg, \
            p.tensor(b, shape=(cols,), context=context) as tb, \
            p.layer_norm(tx, tg, tb, epsilon=1e-5) as ty:
        out = np.asarray(ty.to_host(), np.float32).reshape(rows, cols)
        timing = ty.timing()
        assert timing.completed and timing.duration_seconds > 0
    assert out.tobytes() == oracle.layer_norm(x, g, b, np.float32(1e-5), threaded=True).tobytes()


def test_validation_statuses(context):
    import importlib
    t = importlib.import_module("paralyn_b200.tensor")
    res = t.operators_of(context)
    buf = context.buffer(64)
    other = p.Context("cuda:0")
    foreign = other.buffer(64)
    d = t.TensorDescriptor
    cases = [
        # overlapping output and input: in-place is rejected
        ((d(buf, (2, 4)), d(buf, (4,)), d(buf, (4,)), d(buf, (2, 4))), p.Status.INVALID_ARGUMENT),
        # gamma of the wrong length
        ((d(buf, (2, 2)), d(buf, (3,)), d(buf, (2,)), d(foreign, (2, 2))), p.Status.INVALID_ARGUMENT),
        # a buffer of another context
        ((d(buf, (2, 2)), d(buf, (2,)), d(buf, (2,)), d(foreign, (2, 2))), p.Status.CONTEXT_MISMATCH),
        # non-contiguous input
        ((d(buf, (2, 2), strides=(1, 2)), d(buf, (2,)), d(buf, (2,), 32), d(foreign, (2, 2))),
         p.Status.UNSUPPORTED),
    ]
    for (x, g, b, o), status in cases:
        with pytest.raises(p.Error) as error:
            t.layer_norm_into(res.queue, res.module, x, g, b, o)
        assert error.value.code == status and error.value.operation == "layer_norm_f32"
    # Only modules returned by pr_tensor_operators_load are providers.
    impostor = p.Module.load(context, p.tensor_operators_artifact())
    with pytest.raises(p.Error) as error:
        t.layer_norm_into(res.queue, impostor, d(buf, (1, 2)), d(buf, (2,), 8), d(buf, (2,), 16),
                          d(context.buffer(8), (1, 2)))
    assert error.value.code == p.Status.INVALID_ARGUMENT
    impostor.close()
    foreign.close()
    other.close()
    buf.close()
