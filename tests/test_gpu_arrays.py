"""GPU parity of the 1-D array path (add / affine / scalar affine) against the oracle.

Cases follow the reference's own suites: the sizes and expected values of
tests/native/array_tests.cpp:22-27, and the launch matrix of
scripts/qualify_cuda.py:61-108,171 (sizes x view offsets x {add, affine} x {u32, i32}
index kernels, block 128, guard sentinels around every view). Integer-exact
arithmetic: every comparison is bit-for-bit.
"""
import numpy as np
import pytest

import oracle
import paralyn_b200 as p
from paralyn_b200 import prk, synthetic

pytestmark = pytest.mark.gpu


def host(buffer):
    return np.frombuffer(buffer.read(), np.float32)


def test_array_chain_reference_values(context):
    for n in (0, 1, 17, 256, 257, 1003, 1000003):
        i = np.arange(n)
        a_host = ((i % 61) - 30).astype(np.float32) * np.float32(0.5)
        b_host = ((i % 37) - 18).astype(np.float32) * np.float32(0.25)
        a = p.asarray(a_host, context=context)
        b = p.asarray(b_host, context=context)
        assert a.shape == (n,) and a.nbytes == 4 * n and a.wait() is None
        summed, scaled = p.add(a, b), p.affine(a, b, -2)
        chained = p.affine(summed, scaled, 0.5)
        for value in (summed, scaled, chained):
            info = value.wait()
            assert (info is not None) == bool(n)
            if n:
                timing = value._event.timing()
                assert timing.completed and timing.duration_seconds > 0
                assert timing.clock_domain == p.ClockDomain.DURATION_ONLY and timing.start_seconds is None
        expected = oracle.affine(oracle.add(a_host, b_host), oracle.affine(a_host, b_host, -2.0), 0.5)
        assert np.asarray(chained.to_host(), np.float32).tobytes() == expected.tobytes()
        for value in (a, b, summed, scaled, chained):
            value.close()


def test_same_input_alias(context):
    with p.asarray([1, 2, 3], context=context) as a:
        with p.add(a, a) as doubled:
            assert list(doubled.to_host()) == [2, 4, 6]


def test_mismatched_arrays_are_rejected(context):
    with p.asarray([1, 2, 3], context=context) as a, p.asarray([1], context=context) as short:
        with pytest.raises(ValueError):
            p.add(a, short)
    with p.Context("cuda:0") as other, p.asarray([1, 2, 3], context=context) as a, \
            p.asarray([1, 2, 3], context=other) as foreign:
        with pytest.raises(p.Error) as error:
            p.add(a, foreign)
        assert error.value.code == p.Status.CONTEXT_MISMATCH


def qualification_module(context):
    kernels = prk.operators()[:2] + [
        prk.elementwise("vector_add", [("a", prk.F32, True, True), ("b", prk.F32, True, True),
                                       ("out", prk.F32, True, False), ("n", prk.I32, False, False)],
                        lambda i: prk.binary("+", prk.F32, prk.load("a", i), prk.load("b", i)), prk.I32),
        prk.elementwise("affine", [("a", prk.F32, True, True), ("b", prk.F32, True, True),
                                   ("out", prk.F32, True, False), ("n", prk.I32, False, False),
                                   ("scale", prk.F32, False, False)],
                        lambda i: prk.binary("+", prk.F32, prk.binary("*", prk.F32, prk.load("a", i),
                                                                     prk.ref("scale", prk.F32)),
                                             prk.load("b", i)), prk.I32)]
    return p.Module.load(context, prk.serialize(kernels))


@pytest.mark.parametrize("name", ("array_add", "array_affine", "vector_add", "affine"))
def test_qualification_matrix(context, name):
    module = qualification_module(context)
    kernel = module.kernel(name)
    params = kernel.parameters
    assert [x.access for x in params[:3]] == [p.Access.READ, p.Access.READ, p.Access.WRITE]
    queue = context.queue()
    rng = np.random.default_rng(abs(hash(name)) % 1000)
    sentinel = np.float32(-7777.5)
    for n in (1, 127, 128, 129, 1000, 65537, 1000003):
        for offset in (0, 3):
            guard = 5
            total = n + offset + guard
            a = (rng.integers(-4096, 4096, total) * 0.125).astype(np.float32)
            b = (rng.integers(-4096, 4096, total) * 0.0625).astype(np.float32)
            scale = np.float32(rng.choice([0.5, -1.25, 3.0, 0.1]))
            buffers = [context.buffer(total * 4) for _ in range(3)]
            buffers[0].write(a)
            buffers[1].write(b)
            buffers[2].write(np.full(total, sentinel, np.float32))
            start, size = offset * 4, n * 4
            views = [buffers[0].view(offset=start, size=size, access=p.Access.READ),
                     buffers[1].view(offset=start, size=size, access=p.Access.READ),
                     buffers[2].view(offset=start, size=size, access=p.Access.WRITE)]
            count = p.i32(n) if params[3].type == p.Type.I32 else p.u32(n)
            args = views + [count] + ([p.f32(float(scale))] if "affine" in name else [])
            event = queue.launch(kernel, args, grid=((n + 127) // 128, 1, 1), block=(128, 1, 1))
            assert event.timing().completed
            out = host(buffers[2])
            inside = slice(offset, offset + n)
            if "affine" in name:
                want = oracle.affine(a[inside], b[inside], scale)
            else:
                want = oracle.add(a[inside], b[inside])
            assert out[inside].tobytes() == want.tobytes(), (name, n, offset)
            assert np.all(out[:offset] == sentinel) and np.all(out[offset + n:] == sentinel)
            for x in views + buffers + [event]:
                x.close()
    kernel.close()
    queue.close()
    module.close()


def test_launch_geometry_bounds_the_written_range(context):
    module = p.Module.load_file(context, p.array.operators_path())
    kernel, queue = module.kernel("array_add"), context.queue()
    n = 10000
    a, b = synthetic.uniform(5, 0, n), synthetic.uniform(6, 0, n)
    bufs = [context.buffer(n * 4) for _ in range(3)]
    bufs[0].write(a)
    bufs[1].write(b)
    bufs[2].write(np.full(n, 9.0, np.float32))
    views = [x.view() for x in bufs]
    # 13 blocks of 256 lanes cover only 3328 elements; the rest stays untouched.
    queue.launch(kernel, views + [p.u32(n)], grid=(13, 2, 1), block=(256, 1, 1)).wait()
    out = host(bufs[2])
    assert out[:3328].tobytes() == oracle.add(a[:3328], b[:3328]).tobytes()
    assert np.all(out[3328:] == 9.0)
    # n larger than the views: refused before anything runs.
    with pytest.raises(p.Error) as error:
        queue.launch(kernel, views + [p.u32(n + 1)], grid=(100, 1, 1), block=(256, 1, 1))
    assert error.value.code == p.Status.OUT_OF_BOUNDS and error.value.operation == "launch"
    # Reference launch checks (backends/cuda/engine.cpp:597-616).
    for grid, block in (((0, 1, 1), (256, 1, 1)), ((1, 1, 1), (2048, 1, 1)), ((1, 1, 1), (0, 1, 1))):
        with pytest.raises(p.Error) as error:
            queue.launch(kernel, views + [p.u32(n)], grid=grid, block=block)
        assert error.value.code == p.Status.INVALID_ARGUMENT
    with pytest.raises(p.Error) as error:
        queue.launch(kernel, views[:2] + [p.u32(n)], grid=(1, 1, 1), block=(256, 1, 1))
    assert error.value.code == p.Status.INVALID_ARGUMENT
    read_only_out = bufs[2].view(access=p.Access.READ)
    with pytest.raises(p.Error) as error:
        queue.launch(kernel, views[:2] + [read_only_out, p.u32(n)], grid=(40, 1, 1), block=(256, 1, 1))
    assert error.value.code == p.Status.INVALID_ARGUMENT
    for x in views + bufs + [read_only_out, kernel, queue, module]:
        x.close()


def test_i32_index_overflow_is_refused(context):
    module = qualification_module(context)
    kernel, queue = module.kernel("vector_add"), context.queue()
    bufs = [context.buffer(64) for _ in range(3)]
    views = [x.view() for x in bufs]
    # 2^31 + 1024 threads along x would produce negative i32 indices.
    with pytest.raises(p.Error) as error:
        queue.launch(kernel, views + [p.i32(16)], grid=((1 << 31) // 1024 + 1, 1, 1), block=(1024, 1, 1))
    assert error.value.code == p.Status.OUT_OF_BOUNDS
    queue.launch(kernel, views + [p.i32(-5)], grid=(1, 1, 1), block=(32, 1, 1)).wait()
    for x in views + bufs + [kernel, queue, module]:
        x.close()


def test_add_config_bit_exact(context):
    # vector add, n = 1,048,576, a, b ~ U[-1,1) from seed 0.
    n = 1 << 20
    a, b = synthetic.uniform(0, 0, n), synthetic.uniform(0, n, n)
    with p.asarray(a, context=context) as da, p.asarray(b, context=context) as db, p.add(da, db) as c:
        assert np.asarray(c.to_host(), np.float32).tobytes() == oracle.add(a, b).tobytes()


def test_affine_config_bit_exact(context):
    # y = 1.5 x - 0.25, n = 2^26, x ~ U[-4,4) from seed 1: scalar-bias kernel and
    # the reference-API affine(x, b = -0.25, 1.5).
    n = 1 << 26
    x = synthetic.uniform(1, 0, n, 4.0)
    want = oracle.affine_scalar(x, np.float32(1.5), np.float32(-0.25), threaded=True)
    with p.asarray(x, context=context) as dx:
        with p.affine_scalar(dx, 1.5, -0.25) as y:
            assert np.asarray(y.to_host(), np.float32).tobytes() == want.tobytes()
        with p.asarray(np.full(n, -0.25, np.float32), context=context) as db, p.affine(dx, db, 1.5) as y:
            assert np.asarray(y.to_host(), np.float32).tobytes() == want.tobytes()


def test_misaligned_views_take_the_scalar_path(context):
    module = p.Module.load_file(context, p.array.operators_path())
    kernel, queue = module.kernel("array_affine"), context.queue()
    n = 100001
    a, b = synthetic.uniform(8, 0, n + 8), synthetic.uniform(9, 0, n + 8)
    bufs = [context.buffer((n + 8) * 4) for _ in range(3)]
    bufs[0].write(a)
    bufs[1].write(b)
    bufs[2].write(np.zeros(n + 8, np.float32))
    # a at +1 element, b at +2, out at +3: no common 16-byte phase.
    views = [bufs[0].view(offset=4, size=n * 4), bufs[1].view(offset=8, size=n * 4),
             bufs[2].view(offset=12, size=n * 4)]
    queue.launch(kernel, views + [p.u32(n), p.f32(0.75)], grid=((n + 255) // 256, 1, 1), block=(256, 1, 1)).wait()
    out = host(bufs[2])[3:3 + n]
    assert out.tobytes() == oracle.affine(a[1:1 + n], b[2:2 + n], np.float32(0.75)).tobytes()
    for x in views + bufs + [kernel, queue, module]:
        x.close()
