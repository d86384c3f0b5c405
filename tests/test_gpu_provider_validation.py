"""The tensor provider's validation contract, operator by operator, on a device.

Each case takes a valid call of one operator (pr_matmul_f32, pr_bias_activation_f32,
pr_batched_matmul_f32, pr_reduce_rows_f32, pr_softmax_rows_f32, pr_layer_norm_f32,
pr_add_f32) and breaks one thing; the call must fail with the reference's status
(runtime/tensor.cpp:448-1038), name the operation in pr_last_error, and leave the
event output 0. Precedence cases break two things and pin which check runs first:
the event output, then the record, the record's scalars, operand presence, each
operand's descriptor, the shape relations, output/input aliasing, handle ownership
(queue, operator module, tensor buffers), and only then the zero-work decision.
"""
import ctypes as c
import importlib

import pytest

import paralyn_b200 as p
from paralyn_b200.native import ErrorRecord

T = importlib.import_module("paralyn_b200.tensor")

pytestmark = pytest.mark.gpu
S = p.Status


class Env:
    def __init__(self, context):
        self.context = context
        self.lib = T._api(context._lib)
        res = T.operators_of(context)
        self.queue, self.module = res.queue.handle, res.module.handle
        self.buffers = []

    def buf(self, nbytes, context=None):
        b = (context or self.context).buffer(nbytes)
        self.buffers.append(b)
        return b

    def desc(self, buf, shape, offset=0, strides=None):
        record = T.TensorDescriptor(buf, shape, offset, strides)._native()
        return T.TensorDescRecord.from_buffer_copy(record)

    def close(self):
        for b in self.buffers:
            b.close()


@pytest.fixture()
def env(context):
    e = Env(context)
    yield e
    e.close()


def call(env, entry, record, queue=None, module=None, event=True):
    out = c.c_uint64(99)
    status = getattr(env.lib.api, entry)(env.queue if queue is None else queue,
                                         env.module if module is None else module,
                                         c.byref(record) if record is not None else None,
                                         c.byref(out) if event else None)
    err = ErrorRecord()
    env.lib.api.pr_last_error(c.byref(err))
    return status, out.value, err.operation.decode()


def ptr(d):
    return c.pointer(d) if d is not None else None


# ---- builders of one valid call per operator: (entry, operation, record) ----
def matmul(env, m=4, n=4, k=4, ta=0, tb=0, a=None, b=None, cc=None):
    A = a or env.desc(env.buf(4 * m * k), (k, m) if ta else (m, k))
    B = b or env.desc(env.buf(4 * k * n), (n, k) if tb else (k, n))
    C = cc or env.desc(env.buf(max(4, 4 * m * n)), (m, n))
    rec = T.MatmulRecord(c.sizeof(T.MatmulRecord), 1, m, n, k, ta, tb, ptr(A), ptr(B), ptr(C))
    rec._keep = (A, B, C)
    return rec


def bias_act(env, rows=4, cols=8, bias=True, act=1):
    X = env.desc(env.buf(4 * rows * cols), (rows, cols))
    O = env.desc(env.buf(4 * rows * cols), (rows, cols))
    Bv = env.desc(env.buf(4 * cols), (cols,)) if bias else None
    rec = T.BiasActivationRecord(c.sizeof(T.BiasActivationRecord), 1, act, 0, ptr(X), ptr(Bv), ptr(O))
    rec._keep = (X, O, Bv)
    return rec


def batched(env, batch=2, m=4, n=4, k=4):
    A = env.desc(env.buf(4 * batch * m * k), (batch, m, k))
    B = env.desc(env.buf(4 * batch * k * n), (batch, k, n))
    C = env.desc(env.buf(4 * batch * m * n), (batch, m, n))
    rec = T.BatchedMatmulRecord(c.sizeof(T.BatchedMatmulRecord), 1, batch, m, n, k, ptr(A), ptr(B), ptr(C))
    rec._keep = (A, B, C)
    return rec


def reduce_rows(env, rows=4, cols=8, op=0):
    X = env.desc(env.buf(max(4, 4 * rows * cols)), (rows, cols))
    O = env.desc(env.buf(max(4, 4 * rows)), (rows,))
    rec = T.ReduceRowsRecord(c.sizeof(T.ReduceRowsRecord), 1, op, 0, ptr(X), ptr(O))
    rec._keep = (X, O)
    return rec


def softmax(env, shape=(4, 8), causal=0, scale=1.0):
    count = 1
    for d in shape:
        count *= d
    X = env.desc(env.buf(max(4, 4 * count)), shape)
    O = env.desc(env.buf(max(4, 4 * count)), shape)
    rec = T.SoftmaxRowsRecord(c.sizeof(T.SoftmaxRowsRecord), 1, causal, scale, ptr(X), ptr(O))
    rec._keep = (X, O)
    return rec


def layer_norm(env, rows=4, cols=8, eps=1e-5):
    X = env.desc(env.buf(max(4, 4 * rows * cols)), (rows, cols))
    G = env.desc(env.buf(max(4, 4 * cols)), (cols,))
    Bt = env.desc(env.buf(max(4, 4 * cols)), (cols,))
    O = env.desc(env.buf(max(4, 4 * rows * cols)), (rows, cols))
    rec = T.LayerNormRecord(c.sizeof(T.LayerNormRecord), 1, eps, 0, ptr(X), ptr(G), ptr(Bt), ptr(O))
    rec._keep = (X, G, Bt, O)
    return rec


def add(env, shape=(4, 8)):
    count = 1
    for d in shape:
        count *= d
    X, Y, O = (env.desc(env.buf(max(4, 4 * count)), shape) for _ in range(3))
    rec = T.AddRecord(c.sizeof(T.AddRecord), 1, ptr(X), ptr(Y), ptr(O))
    rec._keep = (X, Y, O)
    return rec


OPS = {"matmul": ("pr_matmul_f32", "matmul_f32", matmul, ("a", "b"), "c"),
       "bias_activation": ("pr_bias_activation_f32", "bias_activation_f32", bias_act, ("x", "bias"), "out"),
       "batched_matmul": ("pr_batched_matmul_f32", "batched_matmul_f32", batched, ("a", "b"), "c"),
       "reduce_rows": ("pr_reduce_rows_f32", "reduce_rows_f32", reduce_rows, ("x",), "out"),
       "softmax": ("pr_softmax_rows_f32", "softmax_rows_f32", softmax, ("x",), "out"),
       "layer_norm": ("pr_layer_norm_f32", "layer_norm_f32", layer_norm, ("x", "gamma", "beta"), "out"),
       "add": ("pr_add_f32", "add_f32", add, ("x", "y"), "out")}


def expect(env, name, record, status, **kw):
    entry, operation = OPS[name][:2]
    got, event, op = call(env, entry, record, **kw)
    assert got == status, (name, S(got).name, S(status).name)
    assert event == 0 if kw.get("event", True) else True
    if status != S.SUCCESS:
        assert op == operation


def replace(record, field, desc):
    setattr(record, field, ptr(desc))
    record._keep = record._keep + (desc,)


@pytest.mark.parametrize("name", list(OPS))
def test_valid_call_succeeds(env, name):
    entry, _, build, _, _ = OPS[name]
    status, event, _ = call(env, entry, build(env))
    assert status == S.SUCCESS and event != 0
    env.lib.api.pr_event_wait(event, None)
    env.lib.api.pr_release(event)


@pytest.mark.parametrize("name", list(OPS))
def test_record_header(env, name):
    build = OPS[name][2]
    expect(env, name, build(env), S.INVALID_ARGUMENT, event=False)
    expect(env, name, None, S.INVALID_ARGUMENT)
    rec = build(env)
    rec.version = 2
    expect(env, name, rec, S.UNSUPPORTED)
    rec = build(env)
    rec.struct_size = 8
    expect(env, name, rec, S.INVALID_ARGUMENT)
    rec = build(env)
    rec.version = 2
    expect(env, name, rec, S.INVALID_ARGUMENT, event=False)  # the event output is checked first


@pytest.mark.parametrize("name", list(OPS))
def test_operands(env, name):
    _, _, build, inputs, output = OPS[name]
    for field in inputs[:1] + (output,):
        rec = build(env)
        setattr(rec, field, None)
        expect(env, name, rec, S.INVALID_ARGUMENT)
        rec = build(env)
        bad = T.TensorDescRecord.from_buffer_copy(getattr(rec, field).contents)
        bad.version = 2
        replace(rec, field, bad)
        expect(env, name, rec, S.UNSUPPORTED)
        rec = build(env)
        bad = T.TensorDescRecord.from_buffer_copy(getattr(rec, field).contents)
        bad.dtype = p.Type.I32
        replace(rec, field, bad)
        expect(env, name, rec, S.UNSUPPORTED)
        rec = build(env)
        bad = T.TensorDescRecord.from_buffer_copy(getattr(rec, field).contents)
        bad.byte_offset += 2
        replace(rec, field, bad)
        expect(env, name, rec, S.INVALID_ARGUMENT)
        rec = build(env)
        bad = T.TensorDescRecord.from_buffer_copy(getattr(rec, field).contents)
        bad.byte_offset += 4  # one element past the end of its buffer
        replace(rec, field, bad)
        expect(env, name, rec, S.OUT_OF_BOUNDS)
        rec = build(env)
        bad = T.TensorDescRecord.from_buffer_copy(getattr(rec, field).contents)
        bad.buffer = 987654321
        replace(rec, field, bad)
        expect(env, name, rec, S.INVALID_HANDLE)
        rec = build(env)
        bad = T.TensorDescRecord.from_buffer_copy(getattr(rec, field).contents)
        bad.strides[0] = -1
        replace(rec, field, bad)
        expect(env, name, rec, S.UNSUPPORTED)
        rec = build(env)
        bad = T.TensorDescRecord.from_buffer_copy(getattr(rec, field).contents)
        bad.rank = 9
        replace(rec, field, bad)
        expect(env, name, rec, S.INVALID_ARGUMENT)


@pytest.mark.parametrize("name", [n for n in OPS if n not in ("batched_matmul", "add", "softmax")])
def test_wrong_rank_and_layout(env, name):
    _, _, build, inputs, output = OPS[name]
    rec = build(env)
    src = getattr(rec, inputs[0]).contents
    shape = tuple(src.shape[i] for i in range(src.rank))
    flat = env.desc(env.buf(4 * max(1, shape[0] * (shape[1] if len(shape) > 1 else 1)) * 2),
                    (shape[0] * (shape[1] if len(shape) > 1 else 1),))
    if len(shape) > 1:
        replace(rec, inputs[0], flat)
        expect(env, name, rec, S.INVALID_ARGUMENT)  # rank
        rec = build(env)
        strided = env.desc(env.buf(4 * 4 * shape[0] * shape[1]), shape, 0, (1, shape[0]))
        replace(rec, inputs[0], strided)
        expect(env, name, rec, S.UNSUPPORTED)  # not contiguous row-major


@pytest.mark.parametrize("name", list(OPS))
def test_aliasing_and_ownership(env, name, context):
    entry, _, build, inputs, output = OPS[name]
    rec = build(env)
    src = getattr(rec, output).contents
    shared = T.TensorDescRecord.from_buffer_copy(src)
    first_input = getattr(rec, inputs[0]).contents
    shared.buffer = first_input.buffer  # the output inside an input's allocation
    big = env.buf(1 << 16)
    inp = T.TensorDescRecord.from_buffer_copy(first_input)
    inp.buffer, inp.byte_offset = big.handle, 0
    out_overlap = T.TensorDescRecord.from_buffer_copy(src)
    out_overlap.buffer, out_overlap.byte_offset = big.handle, 4
    replace(rec, inputs[0], inp)
    replace(rec, output, out_overlap)
    expect(env, name, rec, S.INVALID_ARGUMENT)  # overlapping bytes
    out_disjoint = T.TensorDescRecord.from_buffer_copy(src)
    out_disjoint.buffer, out_disjoint.byte_offset = big.handle, 1 << 15
    replace(rec, output, out_disjoint)
    expect(env, name, rec, S.UNSUPPORTED)  # same allocation, disjoint bytes
    with p.Context("cuda:0") as other:
        foreign = other.buffer(1 << 16)
        rec = build(env)
        moved = T.TensorDescRecord.from_buffer_copy(getattr(rec, output).contents)
        moved.buffer, moved.byte_offset = foreign.handle, 0
        replace(rec, output, moved)
        expect(env, name, rec, S.CONTEXT_MISMATCH)
        other_ops = T.load_tensor_operators(other)
        expect(env, name, build(env), S.CONTEXT_MISMATCH, module=other_ops.handle)
        other_ops.close()
        foreign.close()
    expect(env, name, build(env), S.INVALID_HANDLE, queue=123456789)
    expect(env, name, build(env), S.INVALID_HANDLE, module=123456789)
    impostor = p.Module.load(context, p.tensor_operators_artifact())
    expect(env, name, build(env), S.INVALID_ARGUMENT, module=impostor.handle)
    impostor.close()


def test_operator_scalars(env):
    expect(env, "matmul", matmul(env, ta=2), S.INVALID_ARGUMENT)
    expect(env, "matmul", matmul(env, m=1 << 31, n=1, k=1, a=env.desc(env.buf(4), (1, 1)),
                                 b=env.desc(env.buf(4), (1, 1)), cc=env.desc(env.buf(4), (1, 1))), S.UNSUPPORTED)
    rec = matmul(env)
    replace(rec, "a", env.desc(env.buf(64), (4, 3)))
    expect(env, "matmul", rec, S.INVALID_ARGUMENT)  # shape relation
    expect(env, "bias_activation", bias_act(env, act=3), S.INVALID_ARGUMENT)
    rec = bias_act(env)
    rec.reserved = 1
    expect(env, "bias_activation", rec, S.INVALID_ARGUMENT)
    rec = bias_act(env)
    replace(rec, "bias", env.desc(env.buf(64), (7,)))
    expect(env, "bias_activation", rec, S.INVALID_ARGUMENT)
    rec = batched(env)
    overlapping = env.desc(env.buf(4 * 64), (2, 4, 4), 0, (0, 4, 1))  # both matrices at the same bytes
    replace(rec, "c", overlapping)
    expect(env, "batched_matmul", rec, S.INVALID_ARGUMENT)
    rec = batched(env)
    replace(rec, "a", env.desc(env.buf(4 * 2 * 4 * 4), (2, 4, 4), 0, (16, 1, 4)))  # transposed view: accepted
    status, event, _ = call(env, "pr_batched_matmul_f32", rec)
    assert status == S.SUCCESS and event
    env.lib.api.pr_release(event)
    expect(env, "reduce_rows", reduce_rows(env, op=2), S.INVALID_ARGUMENT)
    rec = reduce_rows(env)
    rec.reserved = 3
    expect(env, "reduce_rows", rec, S.INVALID_ARGUMENT)
    expect(env, "reduce_rows", reduce_rows(env, rows=16777216, cols=0), S.UNSUPPORTED)
    expect(env, "softmax", softmax(env, causal=2), S.INVALID_ARGUMENT)
    expect(env, "softmax", softmax(env, scale=0.0), S.INVALID_ARGUMENT)
    expect(env, "softmax", softmax(env, scale=float("nan")), S.INVALID_ARGUMENT)
    expect(env, "softmax", softmax(env, shape=(2, 2, 2, 2)), S.INVALID_ARGUMENT)
    expect(env, "softmax", softmax(env, shape=(8, 4), causal=1), S.INVALID_ARGUMENT)  # columns < rows
    rec = softmax(env)
    replace(rec, "out", env.desc(env.buf(4 * 32), (8, 4)))
    expect(env, "softmax", rec, S.INVALID_ARGUMENT)
    expect(env, "layer_norm", layer_norm(env, eps=0.0), S.INVALID_ARGUMENT)
    expect(env, "layer_norm", layer_norm(env, eps=float("inf")), S.INVALID_ARGUMENT)
    rec = layer_norm(env)
    rec.reserved = 1
    expect(env, "layer_norm", rec, S.INVALID_ARGUMENT)
    expect(env, "layer_norm", layer_norm(env, rows=1, cols=(1 << 24) + 1), S.UNSUPPORTED)
    rec = add(env)
    replace(rec, "y", env.desc(env.buf(4 * 32), (8, 4)))
    expect(env, "add", rec, S.INVALID_ARGUMENT)


def test_zero_work_and_its_precedence(env):
    # No output elements: success with event 0 and nothing submitted...
    for name, rec in (("matmul", matmul(env, m=0, n=4, k=4)), ("reduce_rows", reduce_rows(env, rows=0)),
                      ("softmax", softmax(env, shape=(0, 8))), ("layer_norm", layer_norm(env, rows=0)),
                      ("add", add(env, shape=(0,))), ("batched_matmul", batched(env, batch=0)),
                      ("bias_activation", bias_act(env, rows=0))):
        expect(env, name, rec, S.SUCCESS)
    # ...but only after the handles are checked.
    expect(env, "matmul", matmul(env, m=0, n=4, k=4), S.INVALID_HANDLE, queue=123456789)
    expect(env, "layer_norm", layer_norm(env, rows=0), S.INVALID_HANDLE, module=123456789)
    # k == 0 is work: C is filled with +0.0.
    status, event, _ = call(env, "pr_matmul_f32", matmul(env, m=4, n=4, k=0))
    assert status == S.SUCCESS and event
    env.lib.api.pr_release(event)


def test_check_precedence(env):
    # operand descriptor errors come before handle ownership
    rec = matmul(env)
    bad = T.TensorDescRecord.from_buffer_copy(rec.a.contents)
    bad.version = 2
    replace(rec, "a", bad)
    expect(env, "matmul", rec, S.UNSUPPORTED, queue=123456789)
    # record scalars come before the operands' descriptors
    rec = layer_norm(env, eps=-1.0)
    bad = T.TensorDescRecord.from_buffer_copy(rec.x.contents)
    bad.version = 2
    replace(rec, "x", bad)
    expect(env, "layer_norm", rec, S.INVALID_ARGUMENT)
    # shape relations come before aliasing: a mis-shaped C in A's allocation at
    # disjoint bytes fails on its shape, not as a shared allocation
    big = env.buf(4096)
    rec = matmul(env, a=env.desc(big, (4, 4)), cc=env.desc(big, (2, 8), 1024))
    expect(env, "matmul", rec, S.INVALID_ARGUMENT)
    rec = matmul(env, a=env.desc(big, (4, 4)), cc=env.desc(big, (4, 4), 1024))
    expect(env, "matmul", rec, S.UNSUPPORTED)
    # aliasing comes before ownership: an overlapping output with an invalid queue
    rec = add(env)
    replace(rec, "out", T.TensorDescRecord.from_buffer_copy(rec.x.contents))
    expect(env, "add", rec, S.INVALID_ARGUMENT, queue=123456789)
