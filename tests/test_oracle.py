"""The CPU oracle pinned against the reference's own code and golden values.

Pins: tree_sum_f32 and the float64 LayerNorm bound from the reference's
examples/native/transformer_reference.hpp (run here through oracle/_ref, stored in
tests/golden/reference_vectors.npz by tests/golden/make_golden.py); the exact
expected values of tests/native/array_tests.cpp:22-27; the independent affine
checker of scripts/qualify_cuda.py:93; and the published MLP output SHA-256 of
docs/tensors-matmul.md:79, which pins the sequential FP32 GEMM order and ReLU.
"""
import hashlib
from pathlib import Path

import numpy as np
import pytest

import oracle
from paralyn_b200 import synthetic

GOLDEN = np.load(Path(__file__).with_name("golden") / "reference_vectors.npz")
TREE_LENGTHS = (1, 7, 255, 256, 257, 1000, 4096, 100003)
LN_KEYS = sorted({k.rsplit("_", 1)[0] for k in GOLDEN.files if k.startswith("ln_")})


@pytest.mark.parametrize("index,n", list(enumerate(TREE_LENGTHS)))
def test_tree_sum_matches_reference_bitwise(index, n):
    x = GOLDEN[f"tree_{n}_x"] if f"tree_{n}_x" in GOLDEN.files else synthetic.uniform(100 + index, 0, n, 4.0)
    assert oracle.tree_sum(x).tobytes() == GOLDEN[f"tree_{n}_sum"].tobytes()


@pytest.mark.parametrize("key", LN_KEYS)
def test_layer_norm_bound_restatement_matches_reference(key):
    x, g, b = GOLDEN[key + "_x"], GOLDEN[key + "_gamma"], GOLDEN[key + "_beta"]
    eps = float(GOLDEN[key + "_eps"][0])
    value, error = oracle.layer_norm_bound(x, g, b, eps)
    np.testing.assert_allclose(value, GOLDEN[key + "_value"], rtol=1e-13, atol=0)
    np.testing.assert_allclose(error, GOLDEN[key + "_error"], rtol=1e-12, atol=0)


@pytest.mark.parametrize("key", LN_KEYS)
def test_layer_norm_fp32_within_reference_bound(key):
    x, g, b = GOLDEN[key + "_x"], GOLDEN[key + "_gamma"], GOLDEN[key + "_beta"]
    eps = GOLDEN[key + "_eps"][0]
    out = oracle.layer_norm(x, g, b, eps).astype(np.float64)
    value, error = GOLDEN[key + "_value"], GOLDEN[key + "_error"]
    slack = 2.0 ** -45 * np.abs(value) + 1.1754943508222875e-38
    assert np.all(np.abs(out - value) <= error + slack)


def test_layer_norm_tree_is_the_reference_tree():
    # mean of the reference order equals tree_sum_f32 / n exactly.
    x = synthetic.normal(7, 0, 3 * 1000, 0.0, 1.0).reshape(3, 1000)
    g, b = np.ones(1000, np.float32), np.zeros(1000, np.float32)
    out = oracle.layer_norm(x, g, b, np.float32(1e-5))
    for r in range(3):
        mean = np.float32(oracle.tree_sum(x[r]) / np.float32(1000))
        d = (x[r] - mean).astype(np.float32)
        var = np.float32(oracle.tree_sum((d * d).astype(np.float32)) / np.float32(1000))
        rstd = np.float32(np.float32(1.0) / np.sqrt(np.float32(var + np.float32(1e-5))))
        expected = ((d * rstd).astype(np.float32) * g + b).astype(np.float32)
        assert expected.tobytes() == out[r].tobytes()


def test_layer_norm_specials():
    # transformer_ops_tests.cpp:428-445: a NaN/Inf row is all NaN, a constant row is
    # exactly beta, a NaN in gamma or beta affects only its column.
    nan, inf = np.float32("nan"), np.float32("inf")
    x = np.array([[1, nan, 2, 3], [1, inf, 2, 3], [5, 5, 5, 5], [1, 2, 3, 4]], np.float32)
    g = np.array([1, 2, nan, 1], np.float32)
    b = np.array([0.25, -0.5, 0, nan], np.float32)
    out = oracle.layer_norm(x, g, b, np.float32(1e-5))
    assert np.isnan(out[:2]).all()
    assert out[2, 0] == 0.25 and out[2, 1] == -0.5 and np.isnan(out[2, 2:]).all()
    assert not np.isnan(out[3, :2]).any() and np.isnan(out[3, 2:]).all()


@pytest.mark.parametrize("n", (0, 1, 17, 256, 257, 1003, 1000003))
def test_array_chain_matches_reference_expected_values(n):
    # array_tests.cpp:22-27: expected = (a + b) * 0.5 + (a * -2 + b) in FP32.
    i = np.arange(n)
    a = ((i % 61) - 30).astype(np.float32) * np.float32(0.5)
    b = ((i % 37) - 18).astype(np.float32) * np.float32(0.25)
    expected = ((a + b) * np.float32(0.5) + (a * np.float32(-2) + b)).astype(np.float32)
    summed, scaled = oracle.add(a, b), oracle.affine(a, b, -2.0)
    assert oracle.affine(summed, scaled, 0.5).tobytes() == expected.tobytes()


def test_affine_matches_independent_checker():
    # scripts/qualify_cuda.py:93: expected = f32(f32(a * scale) + b), no contraction.
    rng = np.random.default_rng(3)
    a = (rng.integers(-4096, 4096, 65537) * 0.125).astype(np.float32)
    b = (rng.integers(-4096, 4096, 65537) * 0.0625).astype(np.float32)
    for scale in (0.5, -1.25, 3.0, 0.1):
        s = np.float32(scale)
        expected = ((a * s).astype(np.float32) + b).astype(np.float32)
        assert oracle.affine(a, b, s).tobytes() == expected.tobytes()
        assert oracle.affine_scalar(a, s, np.float32(-0.25)).tobytes() == \
            ((a * s).astype(np.float32) + np.float32(-0.25)).astype(np.float32).tobytes()


def _xorshift_values(state, count, scale):
    out = np.empty(count, np.float32)
    for i in range(count):
        state ^= (state << 13) & 0xFFFFFFFF
        state ^= state >> 17
        state ^= (state << 5) & 0xFFFFFFFF
        out[i] = np.float32((state >> 16) - 32768) / np.float32(32768.0) * np.float32(scale)
    return out, state


def mlp_inputs(batch=64, inputs=257, hidden=130, outputs=11, seed=2026):
    """examples/native/mlp.cpp:20-70 inputs (xorshift32, drawn in order x, W1, b1, W2, b2)."""
    state = seed
    x, state = _xorshift_values(state, batch * inputs, 1.0)
    w1, state = _xorshift_values(state, inputs * hidden, 0.0625)
    b1, state = _xorshift_values(state, hidden, 0.25)
    w2, state = _xorshift_values(state, hidden * outputs, 0.0625)
    b2, state = _xorshift_values(state, outputs, 0.25)
    return x, w1, b1, w2, b2


MLP_OUTPUT_SHA256 = "3ecb2b1d71d52f4a83f8e6e4cc1f953b189d97c3f434cbd77126e46559a5b073"


def test_mlp_golden_hash_pins_sequential_gemm():
    x, w1, b1, w2, b2 = mlp_inputs()
    z1 = oracle.matmul(x, w1, 64, 130, 257)
    h = oracle.bias_activation(z1, b1, 1)
    z2 = oracle.matmul(h, w2, 64, 11, 130)
    y = oracle.bias_activation(z2, b2, 0)
    assert hashlib.sha256(y.astype("<f4").tobytes()).hexdigest() == MLP_OUTPUT_SHA256


@pytest.mark.parametrize("ta", (False, True))
@pytest.mark.parametrize("tb", (False, True))
@pytest.mark.parametrize("shape", ((1, 1, 1), (15, 17, 33), (65, 47, 129), (17, 300, 16)))
def test_matmul_sequential_within_gamma_bound(shape, ta, tb):
    m, n, k = shape
    a = synthetic.uniform(11, 0, m * k)
    b = synthetic.uniform(12, 0, k * n)
    c = oracle.matmul(a, b, m, n, k, ta, tb)
    exact, magnitude = oracle.matmul_exact(a, b, m, n, k, ta, tb)
    u = 2.0 ** -24
    assert np.all(np.abs(c - exact) <= k * u / (1 - k * u) * magnitude)
    rows = oracle.matmul(a, b, m, n, k, ta, tb, rows=(0, m), threaded=True)
    assert rows.tobytes() == c.tobytes()


def test_threaded_variants_are_bitwise_equal():
    x = synthetic.normal(3, 0, 64 * 512).reshape(64, 512)
    g, b = synthetic.normal(4, 0, 512, 1.0, 0.02), synthetic.normal(5, 0, 512, 0.0, 0.02)
    assert oracle.layer_norm(x, g, b, 1e-5).tobytes() == oracle.layer_norm(x, g, b, 1e-5, threaded=True).tobytes()
    a, c = synthetic.uniform(1, 0, 100001), synthetic.uniform(2, 0, 100001)
    assert oracle.add(a, c).tobytes() == oracle.add(a, c, threaded=True).tobytes()
    assert oracle.affine(a, c, 1.5).tobytes() == oracle.affine(a, c, 1.5, threaded=True).tobytes()


def test_relu_semantics():
    x = np.array([[-1.0, -0.0, 0.0, np.nan, -np.inf, 2.0]], np.float32)
    out = oracle.bias_activation(x, None, 1)
    assert out[0, 0] == 0.0 and not np.signbit(out[0, 0])
    assert np.signbit(out[0, 1])  # -0.0 is not less than zero: passes through
    assert np.isnan(out[0, 3]) and out[0, 4] == 0.0 and out[0, 5] == 2.0


def test_reference_sources_reproduce_fixture(reference_checkout):
    ref = oracle.reference()
    if ref is None:
        pytest.skip("oracle/_ref not built")
    x = synthetic.uniform(100 + 7, 0, 100003, 4.0)
    assert np.float32(ref.ref_tree_sum_f32(x, x.size)).tobytes() == GOLDEN["tree_100003_sum"].tobytes()


# ---- transformer-block row operators and the batched matmul ----
SM_KEYS = sorted({k.rsplit("_", 1)[0] for k in GOLDEN.files if k.startswith("sm_")})
DOT_LENGTHS = sorted(int(k.split("_")[1]) for k in GOLDEN.files if k.startswith("dot_") and k.endswith("_a"))


@pytest.mark.parametrize("index,n", list(enumerate(TREE_LENGTHS)))
def test_tree_max_matches_reference_bitwise(index, n):
    x = synthetic.uniform(100 + index, 0, n, 4.0)
    got = oracle.reduce_rows(x.reshape(1, n), 1)
    assert got.tobytes() == GOLDEN[f"tmax_{n}"].tobytes()


def test_reduce_specials_match_reference():
    x = GOLDEN["tmax_special_x"]
    got = oracle.reduce_rows(x, 1)
    want = GOLDEN["tmax_special_max"]
    assert np.array_equal(np.isnan(got), np.isnan(want))
    finite = ~np.isnan(want)
    assert got[finite].tobytes() == want[finite].tobytes()  # signed zeros included
    sums = oracle.reduce_rows(x, 0)  # reference expectations, transformer_ops_tests.cpp:293-298
    assert np.isnan(sums[0]) and sums[1] == -1.0 and sums[2] == -4.0 and np.isnan(sums[3])
    assert sums[4] == -np.inf and sums[5] == np.inf
    assert oracle.reduce_rows(np.zeros((3, 0), np.float32), 0).tobytes() == np.zeros(3, np.float32).tobytes()
    assert np.all(oracle.reduce_rows(np.zeros((2, 0), np.float32), 1) == -np.inf)


@pytest.mark.parametrize("key", SM_KEYS)
def test_softmax_bound_restatement_matches_reference(key):
    x = GOLDEN[key + "_x"]
    scale, causal = GOLDEN[key + "_meta"]
    batch, rows, cols = (int(v) for v in key[3:].split("x"))
    value, error = oracle.softmax_bound(x.reshape(batch, rows, cols), np.float32(scale), bool(causal))
    np.testing.assert_allclose(value.reshape(x.shape), GOLDEN[key + "_value"], rtol=1e-13, atol=0)
    np.testing.assert_allclose(error.reshape(x.shape), GOLDEN[key + "_error"], rtol=1e-12, atol=0)


@pytest.mark.parametrize("k", DOT_LENGTHS)
def test_dot_bound_matches_reference(k):
    a, b = GOLDEN[f"dot_{k}_a"], GOLDEN[f"dot_{k}_b"]
    value, error = oracle.batched_dot_bound(a, (0, (0, 0, 1)), b, (0, (0, 1, 0)), 1, 1, 1, k)
    np.testing.assert_allclose(value.ravel(), GOLDEN[f"dot_{k}_value"], rtol=1e-13, atol=0)
    np.testing.assert_allclose(error.ravel(), GOLDEN[f"dot_{k}_error"], rtol=1e-12, atol=0)


def test_batched_matmul_strided_views_follow_the_sequential_order():
    # attention-style head split (tests/native/transformer_ops_tests.cpp:194-206): Q_h and
    # K_h^T are strided views into one [T, 3HD] storage.
    T_, H, D = 19, 3, 7
    W = 3 * H * D
    qkv = synthetic.uniform(77, 0, T_ * W, 1.0)
    c = np.full(H * T_ * T_, 12345.0, np.float32)
    oracle.batched_matmul(qkv, (0, (D, W, 1)), qkv, (H * D, (D, 1, W)), c, (0, (T_ * T_, T_, 1)), H, T_, T_, D)
    q = qkv.reshape(T_, 3, H, D)[:, 0].transpose(1, 0, 2)  # [H, T, D]
    k = qkv.reshape(T_, 3, H, D)[:, 1].transpose(1, 0, 2)
    for h in range(H):
        want = oracle.matmul(np.ascontiguousarray(q[h]), np.ascontiguousarray(k[h]), T_, T_, D, transpose_b=True)
        assert c.reshape(H, T_, T_)[h].tobytes() == want.tobytes()
    # a strided output writes only the addressed elements
    out = np.full(80, 12345.0, np.float32)
    oracle.batched_matmul(np.zeros(1, np.float32), (0, (0, 0, 1)), np.zeros(1, np.float32), (0, (0, 1, 0)), out,
                          (1, (40, 10, 2)), 2, 3, 4, 0)
    addressed = {1 + z * 40 + i * 10 + j * 2 for z in range(2) for i in range(3) for j in range(4)}
    for idx in range(80):
        assert out[idx] == (0.0 if idx in addressed else 12345.0)


def test_gelu_bound_matches_reference():
    x = GOLDEN["gelu_x"]
    value, error = oracle.gelu_bound(x)
    np.testing.assert_allclose(value, GOLDEN["gelu_value"], rtol=1e-13, atol=1e-300)
    np.testing.assert_allclose(error, GOLDEN["gelu_error"], rtol=1e-12, atol=1e-300)
