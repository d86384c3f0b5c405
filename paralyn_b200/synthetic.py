"""Seeded synthetic inputs on the host (numpy), the same stream the device
generator pr_b200_fill_synthetic_f32 produces.

SplitMix64 with state `seed`: draw d is mix(seed + (d + 1) * 0x9E3779B97F4A7C15).
  uniform(seed, first, count, scale): scale * (int(draw >> 40) - 2^23) * 2^-23,
      a 24-bit dyadic value in scale * [-1, 1), exact in FP32;
  normal(seed, first, count, mean, std): sample i uses draws first + 2i and
      first + 2i + 1: u1 = ((d0 >> 11) + 1) 2^-53, u2 = (d1 >> 11) 2^-53,
      float32(mean + std * sqrt(-2 ln u1) cos(2 pi u2)) computed in float64.
A workload draws its tensors in order from one stream per seed: each tensor's
`first` is the number of draws the tensors before it consumed.
"""
import numpy as np

GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def draws(seed, first, count):
    """`count` raw 64-bit draws starting at draw index `first`."""
    index = np.arange(first + 1, first + 1 + count, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = np.uint64(seed) + index * GOLDEN
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
    return z ^ (z >> np.uint64(31))


def uniform(seed, first, count, scale=1.0):
    d = draws(seed, first, count)
    u = ((d >> np.uint64(40)).astype(np.int64) - (1 << 23)).astype(np.float32) * np.float32(2.0 ** -23)
    return (np.float32(scale) * u).astype(np.float32)


def normal(seed, first, count, mean=0.0, std=1.0):
    d = draws(seed, first, 2 * count)
    u1 = ((d[0::2] >> np.uint64(11)) + np.uint64(1)).astype(np.float64) * 2.0 ** -53
    u2 = (d[1::2] >> np.uint64(11)).astype(np.float64) * 2.0 ** -53
    v = np.sqrt(-2.0 * np.log(u1)) * np.cos(6.283185307179586 * u2)
    return (np.float64(np.float32(mean)) + np.float64(np.float32(std)) * v).astype(np.float32)


def uniform_draws(count):
    return count


def normal_draws(count):
    return 2 * count
