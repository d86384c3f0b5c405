"""Parity of the benchmarked chain configuration at full size.

Y = LayerNorm(X W) with X [65536 x 4096] ~ N(0, 1), W [4096 x 4096] ~ N(0, 1/4096),
gamma = 1, beta = 0, eps = 1e-5, seed 4, in the default matmul mode (AUTO: the
persistent 3xTF32 tcgen05 kernel, whose last round of tiles runs as k-ranges added by
the split fixup), exactly as bench.py's chain workload runs it: ChainShard with
device-generated inputs, one rank.

Sampled rows (the first and last row of every tile row whose tiles are cut into
k-ranges, for each tile geometry the GEMM may use: 128-row tiles on one SM or 256-row
tiles on a CTA pair; the first and last rows of the matrix and of the first tiles;
seeded random rows; at least 64 in all) are read back with their X rows and the whole
W, and checked:
  * Z within the FP32 GEMM contract |Z - Z_exact| <= 2*k*2^-24*sum|x||w| of the
    float64 product (reference tests/native/tensor_tests.cpp:62-85,
    docs/tensors-matmul.md:75-77);
  * Y bit-identical with the oracle's reference-order LayerNorm of the GPU's own Z
    rows (reference runtime/tensor.cpp:276-299), and within the reference's float64
    LayerNorm bound of those rows (examples/native/transformer_reference.hpp:133-147);
  * Y within that bound plus the propagated GEMM error of the float64 LayerNorm of the
    float64 product: with t_j = |Z_j - Z_exact_j|, the mean moves by at most mean(t),
    each centred value d_j by t_j + mean(t), the variance by at most
    V = mean(2|d_j|(t_j + mean t) + (t_j + mean t)^2), so |dY_j| <= r'(t_j + mean t)
    + |d_j| |r' - r| with r = 1/sqrt(var + eps) and r' = 1/sqrt(var - V + eps).
"""
import numpy as np
import pytest

import oracle
import paralyn_b200 as p
from paralyn_b200 import shard

pytestmark = pytest.mark.gpu

ROWS, K, N = 65536, 4096, 4096
BN = 256
# The tile geometries the GEMM may use here: (tile rows, raster group, concurrent
# units): the one-SM kernel (128-row tiles, one per SM) and the CTA-pair kernel
# (256-row tiles, one per pair of SMs, with any of its raster group sizes).
GEOMETRIES = lambda sm_count: ((128, 8, sm_count),) + tuple((256, g, sm_count // 2) for g in (1, 2, 4, 8, 16))


def split_tile_rows(tm, group, units):
    """First rows of the tiles the persistent kernel cuts into k-ranges: tiles = R*G + r
    with 2r <= G puts the last r tiles (in the grouped raster order) into k-ranges."""
    tiles_m, tiles_n = ROWS // tm, N // BN
    tiles = tiles_m * tiles_n
    r = tiles % units
    if r == 0 or 2 * r > units:
        return set()
    out = set()
    per_group = group * tiles_n
    for tile in range(tiles - r, tiles):
        first_m = (tile // per_group) * group
        rows_in_group = min(group, tiles_m - first_m)
        out.add((first_m + (tile % per_group) % rows_in_group) * tm)
    return out


def sampled_rows(sm_count):
    rows = {0, 1, 127, 128, 255, 256, ROWS - 1}
    for tm, group, units in GEOMETRIES(sm_count):
        for first in split_tile_rows(tm, group, units):
            rows |= {first, first + tm - 1}
    rng = np.random.default_rng(2026)
    while len(rows) < 64:
        rows.add(int(rng.integers(0, ROWS)))
    return sorted(rows)


def layer_norm_f64(z, eps=1e-5):
    mean = z.mean(axis=1, keepdims=True)
    var = ((z - mean) ** 2).mean(axis=1, keepdims=True)
    return (z - mean) / np.sqrt(var + eps)


def propagated(z_exact, t, eps=1e-5):
    """Bound on |LN(z_exact + delta) - LN(z_exact)| for |delta| <= t (float64, per row)."""
    mean = z_exact.mean(axis=1, keepdims=True)
    d = np.abs(z_exact - mean)
    var = (d ** 2).mean(axis=1, keepdims=True)
    shift = t + t.mean(axis=1, keepdims=True)
    v = (2 * d * shift + shift ** 2).mean(axis=1, keepdims=True)
    assert np.all(var - v + eps > 0)
    r, r_low = 1 / np.sqrt(var + eps), 1 / np.sqrt(var - v + eps)
    return r_low * shift + d * (r_low - r)


def test_chain_configuration_auto_mode(context):
    import torch
    sm_count = torch.cuda.get_device_properties(0).multi_processor_count
    p.set_matmul_mode(context, p.MatmulMode.AUTO)
    chain = shard.ChainShard(context, ROWS, K, N, 1, 0, seed=4, w_std=1.0 / 64.0)
    try:
        chain.fill_synthetic()
        mm, ln = chain.step()
        ln.wait()
        variant = p.b200.last_variant(context, "paralyn_matmul_f32")
        mm.close()
        ln.close()
        assert variant is not None and "tf32x3" in variant, variant
        rows = sampled_rows(sm_count)
        assert any(split_tile_rows(*geometry) for geometry in GEOMETRIES(sm_count))
        w = np.frombuffer(chain.w.read(), np.float32)
        x = np.stack([np.frombuffer(chain.x.read(4 * K, offset=4 * r * K), np.float32) for r in rows])
        z = np.stack([np.frombuffer(chain.z.read(4 * N, offset=4 * r * N), np.float32) for r in rows])
        y = np.stack([np.frombuffer(chain.y.read(4 * N, offset=4 * r * N), np.float32) for r in rows])
    finally:
        chain.close()
    count = len(rows)
    exact, magnitude = oracle.matmul_exact(x.ravel(), w, count, N, K)
    error = np.abs(z.astype(np.float64) - exact)
    assert np.all(error <= oracle.matmul_tolerance(magnitude, K)), \
        f"worst row {rows[int(np.argmax(np.max(error / oracle.matmul_tolerance(magnitude, K), axis=1)))]}"
    gamma, beta = np.ones(N, np.float32), np.zeros(N, np.float32)
    want = oracle.layer_norm(z, gamma, beta, np.float32(1e-5))
    assert y.tobytes() == want.tobytes()
    value, bound = oracle.layer_norm_bound(z, gamma, beta, 1e-5)
    assert np.all(oracle.within(y, value, bound))
    y_exact = layer_norm_f64(exact)
    assert np.all(np.abs(y - y_exact) <= bound + propagated(exact, error) + 2.0 ** -45 * np.abs(y_exact))
