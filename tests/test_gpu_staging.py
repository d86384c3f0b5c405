"""Blocking copies from and to pageable host memory (the reference binding's numpy
arrays) go through the library's pinned staging ring: contents must round-trip
exactly at sizes that span several slots, at unaligned offsets and lengths."""
import numpy as np
import pytest

import paralyn_b200 as p

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("nbytes,offset", [(4 << 20, 0), ((48 << 20) + 4 * 7, 4 * 3), ((100 << 20) + 12, 16)])
def test_pageable_round_trip(context, nbytes, offset):
    rng = np.random.default_rng(nbytes)
    data = rng.integers(0, 256, nbytes, dtype=np.uint8)
    buf = context.buffer(offset + nbytes + 64)
    try:
        buf.write_from(data.ctypes.data, nbytes, offset=offset)
        back = np.empty(nbytes, np.uint8)
        buf.read_into(back.ctypes.data, nbytes, offset=offset)
        assert np.array_equal(back, data)
        half = np.frombuffer(buf.read(nbytes // 2, offset=offset), np.uint8)
        assert np.array_equal(half, data[:nbytes // 2])
    finally:
        buf.close()
