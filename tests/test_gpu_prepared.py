"""Prepared right-hand operands (pr_b200_matmul_prepare_f32 / _prepared_f32 /
_prepared_bias_activation_f32) on a device.

A product from B's prepared form must equal pr_matmul_f32 with that B bit for bit in
every matmul mode (the reference order against the oracle as well), through each
kernel form the shape selects: the SIMT kernels (small shapes, FFMA, REFERENCE), the
one-SM tensor-core kernel with the split pass over A or A converted in shared memory,
the transposed form (n <= 128), and the CTA-pair kernel (m >= 256, n > 128). Infinities
of B propagate in AUTO as through pr_matmul_f32. The fused form (bias and activation in
the GEMM epilogue) equals pr_b200_matmul_bias_activation_f32 with that B bit for bit the
same way. A tensor prepared for another (k, n),
or never prepared, fails the command when it runs; the host-side checks reject wrong
sizes, alignments and flags before anything is enqueued.
"""
import ctypes as c
import importlib

import numpy as np
import pytest

import oracle
import paralyn_b200 as p
from paralyn_b200 import b200, shard, synthetic
from paralyn_b200.native import ErrorRecord, Event

pytestmark = pytest.mark.gpu
T = importlib.import_module("paralyn_b200.tensor")
MODES = (p.MatmulMode.AUTO, p.MatmulMode.REFERENCE, p.MatmulMode.FFMA, p.MatmulMode.TF32X3)

# (m, n, k, transpose_a, transpose_b)
SHAPES = ((5, 7, 3, False, False),         # SIMT in every mode
          (300, 129, 64, False, False),    # one-SM kernel, A converted in shared memory
          (257, 300, 1000, True, True),    # split pass over A stored [k, m]; B prepared from [n, k]
          (130, 64, 96, False, True),      # transposed form (n <= 128)
          (1000, 4096, 512, False, False),  # CTA pairs
          (513, 1000, 33, False, False))   # AUTO declines (k < 64): FFMA from the prepared copy


def products(context, a, b, m, n, k, ta, tb, mode):
    """(pr_matmul_f32 result, prepared-form result) for the same operands and mode."""
    res = T.operators_of(context)
    p.set_matmul_mode(context, mode)
    bufs = [context.buffer(4 * a.size), context.buffer(4 * b.size), context.buffer(4 * m * n),
            context.buffer(4 * m * n)]
    try:
        bufs[0].write(a.ravel())
        bufs[1].write(b.ravel())
        ad = T.TensorDescriptor(bufs[0], (k, m) if ta else (m, k))
        bd = T.TensorDescriptor(bufs[1], (n, k) if tb else (k, n))
        plain = T.matmul_into(res.queue, res.module, ad, bd, T.TensorDescriptor(bufs[2], (m, n)), m=m, n=n, k=k,
                              transpose_a=ta, transpose_b=tb)
        prepared = b200.PreparedMatrix(res.queue, res.module, context, bd, k=k, n=n, transpose_b=tb)
        try:
            bufs[1].write(np.full(b.size, np.nan, np.float32))  # later changes to B do not reach it
            event = b200.matmul_prepared_into(res.queue, res.module, ad, prepared.descriptor,
                                              T.TensorDescriptor(bufs[3], (m, n)), m=m, n=n, k=k, transpose_a=ta)
            event.wait()
            event.close()
            variant = b200.last_variant(context, "b200_matmul_prepared_f32")
        finally:
            prepared.close()
        plain.wait()
        plain.close()
        want = np.frombuffer(bufs[2].read(), np.float32).reshape(m, n).copy()
        got = np.frombuffer(bufs[3].read(), np.float32).reshape(m, n).copy()
        return want, got, variant
    finally:
        p.set_matmul_mode(context, p.MatmulMode.AUTO)
        for buf in bufs:
            buf.close()


@pytest.mark.parametrize("m,n,k,ta,tb", SHAPES)
def test_prepared_product_equals_matmul_in_every_mode(context, m, n, k, ta, tb):
    a = synthetic.uniform(7100 + m, 0, m * k).reshape(k, m) if ta else \
        synthetic.uniform(7100 + m, 0, m * k).reshape(m, k)
    b = synthetic.uniform(7200 + n, 0, k * n).reshape(n, k) if tb else \
        synthetic.uniform(7200 + n, 0, k * n).reshape(k, n)
    for mode in MODES:
        want, got, variant = products(context, a, b, m, n, k, ta, tb, mode)
        assert got.tobytes() == want.tobytes(), (m, n, k, ta, tb, mode, variant)
        if mode == p.MatmulMode.REFERENCE:
            exact = oracle.matmul(a.ravel(), np.ascontiguousarray(b.T if tb else b).ravel(), m, n, k, ta, False)
            assert got.tobytes() == exact.tobytes()
        tensor_cores = (mode == p.MatmulMode.TF32X3 and k >= 16) or \
            (mode == p.MatmulMode.AUTO and k >= 64 and m * n >= 128 * 256)
        assert (variant == "tcgen05_tf32x3") == tensor_cores, (m, n, k, mode, variant)


def test_infinite_weights_propagate_in_auto(context):
    m, n, k = 512, 512, 256
    a = synthetic.uniform(7301, 0, m * k).reshape(m, k)
    b = synthetic.uniform(7302, 0, k * n).reshape(k, n)
    b[3, 5] = np.inf
    b[100, 7] = -np.inf
    want, got, variant = products(context, a, b, m, n, k, False, False, p.MatmulMode.AUTO)
    assert variant == "tcgen05_tf32x3"
    assert got.tobytes() == want.tobytes()
    assert np.isinf(got[:, 5]).all() and np.isinf(got[:, 7]).all()
    assert not np.isnan(got).any()


def test_chain_with_prepared_weights_equals_the_plain_chain(context):
    rows, k, n = 1024, 512, 768
    results = []
    for prepared in (False, True):
        chain = shard.ChainShard(context, rows, k, n, seed=11, w_std=1.0 / 32.0)
        try:
            chain.fill_synthetic()
            if prepared:
                chain.prepare_weights()
            for e in chain.step():
                e.wait()
                e.close()
            results.append((chain.z.read(), chain.y.read()))
        finally:
            chain.close()
    assert results[0] == results[1]


def fused_products(context, a, b, bias, m, n, k, ta, mode, activation):
    """(pr_b200_matmul_bias_activation_f32 result, prepared-form result, variant) for
    the same operands, bias (or None), activation and mode."""
    res = T.operators_of(context)
    p.set_matmul_mode(context, mode)
    bufs = [context.buffer(4 * a.size), context.buffer(4 * b.size), context.buffer(4 * n),
            context.buffer(4 * m * n), context.buffer(4 * m * n)]
    try:
        bufs[0].write(a.ravel())
        bufs[1].write(b.ravel())
        ad = T.TensorDescriptor(bufs[0], (k, m) if ta else (m, k))
        bd = T.TensorDescriptor(bufs[1], (k, n))
        bias_d = None
        if bias is not None:
            bufs[2].write(bias)
            bias_d = T.TensorDescriptor(bufs[2], (n,))
        plain = b200.matmul_bias_activation_into(res.queue, res.module, ad, bd, T.TensorDescriptor(bufs[3], (m, n)),
                                                 bias_d, m=m, n=n, k=k, transpose_a=ta, activation=activation)
        prepared = b200.PreparedMatrix(res.queue, res.module, context, bd, k=k, n=n)
        try:
            event = b200.matmul_prepared_bias_activation_into(
                res.queue, res.module, ad, prepared.descriptor, T.TensorDescriptor(bufs[4], (m, n)), bias_d,
                m=m, n=n, k=k, transpose_a=ta, activation=activation)
            event.wait()
            event.close()
            variant = b200.last_variant(context, "b200_matmul_prepared_bias_activation_f32")
        finally:
            prepared.close()
        plain.wait()
        plain.close()
        want = np.frombuffer(bufs[3].read(), np.float32).reshape(m, n).copy()
        got = np.frombuffer(bufs[4].read(), np.float32).reshape(m, n).copy()
        return want, got, variant
    finally:
        p.set_matmul_mode(context, p.MatmulMode.AUTO)
        for buf in bufs:
            buf.close()


# (m, n, k, transpose_a): SIMT, A converted in shared memory, split A stored [k, m],
# the transposed form, CTA pairs
FUSED_SHAPES = ((5, 7, 3, False), (300, 129, 64, False), (257, 300, 1000, True), (130, 64, 96, False),
                (1000, 4096, 512, False))


@pytest.mark.parametrize("m,n,k,ta", FUSED_SHAPES)
def test_prepared_bias_activation_equals_the_fused_product(context, m, n, k, ta):
    a = synthetic.uniform(7500 + m, 0, m * k).reshape((k, m) if ta else (m, k))
    b = synthetic.uniform(7600 + n, 0, k * n).reshape(k, n)
    bias = synthetic.uniform(7700 + n, 0, n)
    cases = [(mode, T.Activation.GELU_TANH, bias) for mode in MODES] + \
        [(p.MatmulMode.AUTO, T.Activation.RELU, bias), (p.MatmulMode.AUTO, T.Activation.NONE, None),
         (p.MatmulMode.TF32X3, T.Activation.GELU_TANH, None)]
    for mode, activation, bias_values in cases:
        want, got, variant = fused_products(context, a, b, bias_values, m, n, k, ta, mode, activation)
        assert got.tobytes() == want.tobytes(), (m, n, k, ta, mode, activation, variant)
        tensor_cores = (mode == p.MatmulMode.TF32X3 and k >= 16) or \
            (mode == p.MatmulMode.AUTO and k >= 64 and m * n >= 128 * 256)
        assert (variant == "tcgen05_tf32x3") == tensor_cores, (m, n, k, mode, variant)


# ---- validation ----
class Calls:
    def __init__(self, context):
        self.context = context
        self.lib = b200._b200(context._lib)
        res = T.operators_of(context)
        self.queue, self.module = res.queue.handle, res.module.handle
        self.buffers = []

    def buf(self, nbytes):
        b = self.context.buffer(nbytes)
        self.buffers.append(b)
        return b

    def desc(self, buf, shape, offset=0):
        return T.TensorDescRecord.from_buffer_copy(T.TensorDescriptor(buf, shape, offset)._native())

    def prepare(self, b, tb, prepared):
        out = c.c_uint64(99)
        status = self.lib.api.pr_b200_matmul_prepare_f32(self.queue, self.module, c.byref(b), tb,
                                                          c.byref(prepared), c.byref(out))
        return status, out.value, self.operation()

    def product(self, record):
        out = c.c_uint64(99)
        status = self.lib.api.pr_b200_matmul_prepared_f32(self.queue, self.module, c.byref(record), c.byref(out))
        return status, out.value, self.operation()

    def fused(self, record, bias, activation):
        out = c.c_uint64(99)
        status = self.lib.api.pr_b200_matmul_prepared_bias_activation_f32(
            self.queue, self.module, c.byref(record), c.byref(bias) if bias is not None else None, activation,
            c.byref(out))
        return status, out.value, self.operation()

    def operation(self):
        err = ErrorRecord()
        self.lib.api.pr_last_error(c.byref(err))
        return err.operation.decode()

    def close(self):
        for b in self.buffers:
            b.close()


def record(m, n, k, a, prepared, cc, ta=0, tb=0):
    rec = T.MatmulRecord(c.sizeof(T.MatmulRecord), 1, m, n, k, ta, tb, c.pointer(a), c.pointer(prepared),
                         c.pointer(cc))
    rec._keep = (a, prepared, cc)
    return rec


def test_prepare_and_product_validation(context):
    S = p.Status
    calls = Calls(context)
    try:
        k, n, m = 64, 96, 32
        size = b200.matmul_prepared_bytes(context._lib, k, n)
        b = calls.desc(calls.buf(4 * k * n), (k, n))
        room = calls.buf(size + 256)
        good = calls.desc(room, (size // 4,))
        # the prepare call: transpose flag, prepared size, rank, alignment, aliasing
        assert calls.prepare(b, 2, good)[:2] == (S.INVALID_ARGUMENT, 0)
        assert calls.prepare(b, 0, calls.desc(room, (size // 4 - 1,)))[:2] == (S.INVALID_ARGUMENT, 0)
        assert calls.prepare(b, 0, calls.desc(calls.buf(size), (size // 8, 2)))[:2] == (S.INVALID_ARGUMENT, 0)
        assert calls.prepare(b, 0, calls.desc(room, (size // 4,), 16)) == (S.INVALID_ARGUMENT, 0, "matmul_prepare_f32")
        shared = calls.buf(4 * k * n + size)
        assert calls.prepare(calls.desc(shared, (k, n)), 0, calls.desc(shared, (size // 4,), 4 * k * n))[:2] == \
            (S.UNSUPPORTED, 0)
        status, event, _ = calls.prepare(b, 0, good)
        assert status == S.SUCCESS and event != 0
        ev = Event._adopt(calls.lib, event)
        ev.wait()
        ev.close()
        a = calls.desc(calls.buf(4 * m * k), (m, k))
        cc = calls.desc(calls.buf(4 * m * n), (m, n))
        # the product: transpose_b, the prepared shape, then pr_matmul_f32's shape rules
        assert calls.product(record(m, n, k, a, good, cc, tb=1)) == (S.INVALID_ARGUMENT, 0, "matmul_prepared_f32")
        wide = calls.desc(calls.buf(4 * m * (n + 1)), (m, n + 1))
        assert calls.product(record(m, n + 1, k, a, good, wide))[:2] == (S.INVALID_ARGUMENT, 0)
        assert calls.product(record(m, n, k, calls.desc(calls.buf(4 * m * k), (k, m)), good, cc))[:2] == \
            (S.INVALID_ARGUMENT, 0)
        assert calls.product(record(m, n, k, a, calls.desc(room, (size // 4,), 16), cc))[:2] == \
            (S.INVALID_ARGUMENT, 0)
        status, event, _ = calls.product(record(m, n, k, a, good, cc))
        assert status == S.SUCCESS and event != 0
        ev = Event._adopt(calls.lib, event)
        ev.wait()
        ev.close()
        # no rows: no command and no event
        assert calls.product(record(0, n, k, calls.desc(calls.buf(4), (0, k)), good,
                                    calls.desc(calls.buf(4), (0, n))))[:2] == (S.SUCCESS, 0)
        # the fused form: the product's rules, then the activation and the bias shape
        op = "matmul_prepared_bias_activation_f32"
        bias = calls.desc(calls.buf(4 * n), (n,))
        assert calls.fused(record(m, n, k, a, good, cc, tb=1), bias, 2) == (S.INVALID_ARGUMENT, 0, op)
        assert calls.fused(record(m, n, k, a, good, cc), bias, 3) == (S.INVALID_ARGUMENT, 0, op)
        assert calls.fused(record(m, n, k, a, good, cc), calls.desc(calls.buf(4 * n + 4), (n + 1,)), 2) == \
            (S.INVALID_ARGUMENT, 0, op)
        assert calls.fused(record(m, n, k, a, calls.desc(room, (size // 4,), 16), cc), bias, 2)[:2] == \
            (S.INVALID_ARGUMENT, 0)
        for with_bias in (bias, None):
            status, event, _ = calls.fused(record(m, n, k, a, good, cc), with_bias, 2)
            assert status == S.SUCCESS and event != 0
            ev = Event._adopt(calls.lib, event)
            ev.wait()
            ev.close()
    finally:
        calls.close()


@pytest.mark.parametrize("prepare", (True, False))
def test_product_with_a_tensor_not_prepared_for_its_shape_fails(prepare):
    # (k, n) = (64, 256) and (32, 512) have prepared forms of the same size: the host
    # checks pass and the header check in the command fails it. A context of its own:
    # the failure is sticky.
    assert b200.matmul_prepared_bytes(p.library(), 64, 256) == b200.matmul_prepared_bytes(p.library(), 32, 512)
    with p.Context("cuda:0") as ctx:
        res = T.operators_of(ctx)
        size = b200.matmul_prepared_bytes(ctx._lib, 64, 256)
        bufs = [ctx.buffer(4 * 64 * 256), ctx.buffer(size), ctx.buffer(4 * 300 * 32), ctx.buffer(4 * 300 * 512)]
        bufs[0].write(synthetic.uniform(7401, 0, 64 * 256))
        bufs[1].write(np.zeros(size // 4, np.float32))
        prepared = T.TensorDescriptor(bufs[1], (size // 4,))
        if prepare:
            e = b200.matmul_prepare_into(res.queue, res.module, T.TensorDescriptor(bufs[0], (64, 256)), prepared)
            e.wait()
            e.close()
        event = b200.matmul_prepared_into(res.queue, res.module, T.TensorDescriptor(bufs[2], (300, 32)), prepared,
                                          T.TensorDescriptor(bufs[3], (300, 512)), m=300, n=512, k=32)
        with pytest.raises(p.Error) as error:
            event.wait()
        assert error.value.code == p.Status.EXECUTION_FAILED
        assert "prepared operand" in str(error.value)
        for obj in [event] + bufs:
            try:
                obj.close()
            except p.Error:
                pass
    with p.Context("cuda:0") as ctx, p.asarray(np.ones(1000, np.float32), context=ctx) as a, p.add(a, a) as b:
        assert np.all(np.asarray(b.to_host(), np.float32) == 2.0)
