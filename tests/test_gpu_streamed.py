"""Stream-ordered host copies (pr_b200_buffer_write_async / read_async).

The copies run on the GPU's copy engines, concurrently with kernels on other
bytes, and the runtime orders them against every earlier command that touches
the same bytes. These tests enqueue whole dependency chains without any host
wait in between and check that every result is the one a blocking, in-order
execution gives: round trips, read-after-write through a kernel, write-after-read
of a kernel's input, write-after-read of a download, and the pipelined row-sliced
GEMM -> LayerNorm chain against the oracle.
"""
import importlib

import numpy as np
import pytest

import oracle
import paralyn_b200 as p
from paralyn_b200 import b200, shard, synthetic

pytestmark = pytest.mark.gpu
T = importlib.import_module("paralyn_b200.tensor")


def registered(*arrays):
    for a in arrays:
        b200.host_register(a)
    return arrays


def test_round_trip_pinned_and_pageable(context):
    queue = T.operators_of(context).queue
    n = 1 << 22
    src = synthetic.uniform(5, 0, n, 4.0)
    buf = context.buffer(4 * n + 256)
    for pin in (True, False):
        host_in, host_out = src.copy(), np.zeros(n, np.float32)
        if pin:
            registered(host_in, host_out)
        try:
            up = b200.write_async(queue, buf, host_in, offset=256)
            down = b200.read_async(queue, buf, host_out, offset=256)  # same bytes: after the upload
            down.wait()
            assert host_out.tobytes() == src.tobytes()
            info = up.timing()
            assert info.completed and info.duration_seconds > 0
            up.close()
            down.close()
        finally:
            if pin:
                b200.host_unregister(host_in)
                b200.host_unregister(host_out)
    assert b200.write_async(queue, buf, src, offset=0, nbytes=0) is None
    with pytest.raises(p.Error) as error:
        b200.write_async(queue, buf, src, offset=512)  # past the end
    assert error.value.code == p.Status.OUT_OF_BOUNDS
    with pytest.raises(p.Error) as error:
        b200.host_register(src, 0)
    assert error.value.code == p.Status.INVALID_ARGUMENT
    buf.close()


def test_hazards_through_a_kernel(context):
    # upload X1, Y = 1.5 X - 0.25, download Y -> o1, upload X2 (must wait for the
    # kernel still reading X1), Y = ... (must wait for the download of Y), download
    # Y -> o2; nothing waits on the host until the end.
    queue = T.operators_of(context).queue
    n = 1 << 24
    module = p.Module.load_file(context, p.array.operators_path())
    kernel = module.kernel("array_affine_scalar")
    x, y = context.buffer(4 * n), context.buffer(4 * n)
    xv, yv = x.view(access=p.Access.READ), y.view(access=p.Access.WRITE)
    inputs = [synthetic.uniform(6, 0, n, 4.0), synthetic.uniform(6, n, n, 4.0)]
    outputs = [np.zeros(n, np.float32), np.zeros(n, np.float32)]
    registered(*inputs, *outputs)
    try:
        events = []
        for host_in, host_out in zip(inputs, outputs):
            events.append(b200.write_async(queue, x, host_in))
            events.append(queue.launch(kernel, [xv, yv, p.u32(n), p.f32(1.5), p.f32(-0.25)],
                                       grid=((n + 255) // 256, 1, 1), block=(256, 1, 1)))
            events.append(b200.read_async(queue, y, host_out))
        events[-1].wait()
        for host_in, host_out in zip(inputs, outputs):
            want = oracle.affine_scalar(host_in, np.float32(1.5), np.float32(-0.25))
            assert host_out.tobytes() == want.tobytes()
        for e in events:
            e.close()
    finally:
        for a in inputs + outputs:
            b200.host_unregister(a)
    for obj in (xv, yv, x, y, module):
        obj.close()


def test_blocking_copies_and_markers_follow_async_ones(context):
    queue = T.operators_of(context).queue
    n = 1 << 22
    src = synthetic.uniform(7, 0, n)
    (pinned,) = registered(src.copy())
    buf = context.buffer(4 * n)
    try:
        up = b200.write_async(queue, buf, pinned)
        mark = b200.marker(queue)  # a marker follows every earlier command, copies included
        mark.wait()
        assert up.wait().completed
        back = np.frombuffer(buf.read(), np.float32)  # the blocking read drains the queue first
        assert back.tobytes() == src.tobytes()
        for e in (up, mark):
            e.close()
    finally:
        b200.host_unregister(pinned)
    buf.close()


@pytest.mark.parametrize("slices", [1, 3, 8])
def test_pipelined_chain_matches_oracle(context, slices):
    rows, k, n = 700, 64, 96
    p.set_matmul_mode(context, p.MatmulMode.REFERENCE)
    try:
        chain = shard.ChainShard(context, rows, k, n, seed=4)
        chain.fill_synthetic()
        x = synthetic.normal(4, 0, rows * k)
        w = synthetic.normal(4, 2 * rows * k, k * n, 0.0, 1.0 / 64.0)
        z = oracle.matmul(x, w, rows, n, k)
        want = oracle.layer_norm(z, np.ones(n, np.float32), np.zeros(n, np.float32), np.float32(1e-5))
        x_host = x.copy()
        y_host = np.full(rows * n, np.nan, np.float32)
        registered(x_host, y_host)
        try:
            chain.x.write(np.zeros(rows * k, np.float32))  # the device copy must come from x_host
            events = chain.step_from_host(x_host.ctypes.data, y_host.ctypes.data, slices=slices)
            events[-1].wait()
            assert y_host.tobytes() == want.reshape(-1).tobytes()
            for e in events:
                e.close()
        finally:
            b200.host_unregister(x_host)
            b200.host_unregister(y_host)
        chain.close()
    finally:
        p.set_matmul_mode(context, p.MatmulMode.AUTO)
