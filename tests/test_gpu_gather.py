"""Row-sharded results gathered over NVLink.

pr_b200_layer_norm_gather_f32: each rank normalizes its rows [r0, r1) and the same
kernel writes every output row into each rank's gathered [rows, columns] tensor (its
own and the peers', mapped with pr_b200_buffer_export / pr_b200_buffer_import).
pr_b200_gather_rows_f32: the same gathered output for any row shard, here a GEMM
shard's C (reference-order matmul, so the gathered product is checkable bit for bit).
After all ranks' commands have completed, every gathered tensor must equal the
unsharded oracle result, bit for bit. One-GPU cases gather into local buffers; the
two-GPU case spawns one process per GPU (needs a box with at least two B200s,
skipped otherwise).
"""
import importlib
import multiprocessing as mp

import numpy as np
import pytest

import oracle
import paralyn_b200 as p
from paralyn_b200 import shard, synthetic

pytestmark = pytest.mark.gpu
T = importlib.import_module("paralyn_b200.tensor")


def inputs(rows, cols):
    x = synthetic.normal(31, 0, rows * cols, 0.25, 2.0).reshape(rows, cols)
    g = synthetic.normal(32, 0, cols, 1.0, 0.1)
    b = synthetic.normal(33, 0, cols, 0.0, 0.1)
    return x, g, b


@pytest.mark.parametrize("rows,cols", [(96, 4096), (50, 2000), (33, 700)])
def test_gather_into_local_buffers(context, rows, cols):
    x, g, b = inputs(rows, cols)
    want = oracle.layer_norm(x, g, b, np.float32(1e-5))
    res = T.operators_of(context)
    gathered = [context.buffer(rows * cols * 4), context.buffer((rows + 3) * cols * 4)]
    for world in (1, 3):
        for rank in range(world):
            r0, r1 = shard.row_range(rows, world, rank)
            with p.tensor(x[r0:r1].ravel(), shape=(r1 - r0, cols), context=context) as tx, \
                    p.tensor(g, shape=(cols,), context=context) as tg, \
                    p.tensor(b, shape=(cols,), context=context) as tb:
                out = context.buffer(max(1, (r1 - r0) * cols * 4))
                event = p.b200.layer_norm_gather_into(
                    res.queue, res.module, tx.descriptor(), tg.descriptor(), tb.descriptor(),
                    T.TensorDescriptor(out, (r1 - r0, cols)),
                    [T.TensorDescriptor(gathered[0], (rows, cols)),
                     T.TensorDescriptor(gathered[1], (rows, cols), 3 * cols * 4)], row_offset=r0)
                event.wait()
                local = np.frombuffer(out.read(), np.float32).reshape(r1 - r0, cols)
                assert local.tobytes() == want[r0:r1].tobytes()
                event.close()
                out.close()
        first = np.frombuffer(gathered[0].read(), np.float32).reshape(rows, cols)
        second = np.frombuffer(gathered[1].read(), np.float32)[3 * cols:].reshape(rows, cols)
        assert first.tobytes() == want.tobytes() and second.tobytes() == want.tobytes()
    with pytest.raises(p.Error) as error:  # rows past the end of the gathered tensor
        with p.tensor(x.ravel(), shape=(rows, cols), context=context) as tx, \
                p.tensor(g, shape=(cols,), context=context) as tg, p.tensor(b, shape=(cols,), context=context) as tb:
            out = context.buffer(rows * cols * 4)
            try:
                p.b200.layer_norm_gather_into(res.queue, res.module, tx.descriptor(), tg.descriptor(),
                                              tb.descriptor(), T.TensorDescriptor(out, (rows, cols)),
                                              [T.TensorDescriptor(gathered[0], (rows, cols))], row_offset=1)
            finally:
                out.close()
    assert error.value.code == p.Status.OUT_OF_BOUNDS
    for buf in gathered:
        buf.close()


@pytest.mark.parametrize("rows,cols,k", [(96, 4096, 64), (50, 2001, 33), (7, 12, 5)])
def test_gemm_shards_gathered_into_local_buffers(context, rows, cols, k):
    a = synthetic.uniform(41, 0, rows * k).reshape(rows, k)
    b = synthetic.uniform(42, 0, k * cols).reshape(k, cols)
    p.set_matmul_mode(context, p.MatmulMode.REFERENCE)
    want = oracle.matmul(a.ravel(), b.ravel(), rows, cols, k)
    res = T.operators_of(context)
    gathered = [context.buffer(rows * cols * 4), context.buffer((rows + 2) * cols * 4)]
    try:
        for world in (1, 2, 3):
            for buf in gathered:
                buf.write(np.full(buf.size // 4, np.nan, np.float32))
            with p.tensor(b.ravel(), shape=(k, cols), context=context) as tb:
                for rank in range(world):
                    r0, r1 = shard.row_range(rows, world, rank)
                    with p.tensor(a[r0:r1].ravel(), shape=(r1 - r0, k), context=context) as ta, \
                            p.matmul(ta, tb) as c:
                        event = p.b200.gather_rows_into(
                            res.queue, c.descriptor(),
                            [T.TensorDescriptor(gathered[0], (rows, cols)),
                             T.TensorDescriptor(gathered[1], (rows, cols), 2 * cols * 4)], row_offset=r0)
                        event.wait()
                        assert p.b200.last_variant(context, "b200_gather_rows_f32") in ("vec4", "scalar")
                        event.close()
            first = np.frombuffer(gathered[0].read(), np.float32).reshape(rows, cols)
            second = np.frombuffer(gathered[1].read(), np.float32)[2 * cols:].reshape(rows, cols)
            assert first.tobytes() == want.tobytes() and second.tobytes() == want.tobytes()
        with pytest.raises(p.Error) as error:  # rows past the end of the gathered tensor
            with p.tensor(a.ravel(), shape=(rows, k), context=context) as ta, \
                    p.tensor(b.ravel(), shape=(k, cols), context=context) as tb, p.matmul(ta, tb) as c:
                p.b200.gather_rows_into(res.queue, c.descriptor(), [T.TensorDescriptor(gathered[0], (rows, cols))],
                                        row_offset=1)
        assert error.value.code == p.Status.OUT_OF_BOUNDS
        with pytest.raises(p.Error) as error:  # two gathered tensors over the same bytes
            with p.tensor(a.ravel(), shape=(rows, k), context=context) as ta, \
                    p.tensor(b.ravel(), shape=(k, cols), context=context) as tb, p.matmul(ta, tb) as c:
                target = T.TensorDescriptor(gathered[0], (rows, cols))
                p.b200.gather_rows_into(res.queue, c.descriptor(), [target, target], row_offset=0)
        assert error.value.code == p.Status.INVALID_ARGUMENT
    finally:
        p.set_matmul_mode(context, p.MatmulMode.AUTO)
        for buf in gathered:
            buf.close()


ROWS, COLS = 257, 4096


def _rank(rank, world, handles, barrier, results):
    import numpy as np
    import paralyn_b200 as p
    from paralyn_b200 import shard, synthetic
    T = importlib.import_module("paralyn_b200.tensor")
    try:
        ctx = p.Context(f"cuda:{rank}")
        x, g, b = inputs(ROWS, COLS)
        r0, r1 = shard.row_range(ROWS, world, rank)
        mine = ctx.buffer(ROWS * COLS * 4)
        mine.write(np.full(ROWS * COLS, np.nan, np.float32))
        handles[rank] = p.b200.export_buffer(mine)
        barrier.wait(timeout=120)
        peers = [p.b200.import_buffer(ctx, handles[r]) for r in range(world) if r != rank]
        res = T.operators_of(ctx)
        tx = p.tensor(x[r0:r1].ravel(), shape=(r1 - r0, COLS), context=ctx)
        tg = p.tensor(g, shape=(COLS,), context=ctx)
        tb = p.tensor(b, shape=(COLS,), context=ctx)
        out = ctx.buffer((r1 - r0) * COLS * 4)
        targets = [T.TensorDescriptor(buf, (ROWS, COLS)) for buf in [mine] + peers]
        event = p.b200.layer_norm_gather_into(res.queue, res.module, tx.descriptor(), tg.descriptor(),
                                              tb.descriptor(), T.TensorDescriptor(out, (r1 - r0, COLS)),
                                              targets, row_offset=r0)
        event.wait()
        barrier.wait(timeout=120)  # every rank's rows have landed everywhere
        gathered = np.frombuffer(mine.read(), np.float32).reshape(ROWS, COLS)
        want = oracle.layer_norm(x, g, b, np.float32(1e-5))
        ok_ln = gathered.tobytes() == want.tobytes()
        barrier.wait(timeout=120)  # everyone has read the LayerNorm before it is overwritten
        # A GEMM shard (reference order) gathered with pr_b200_gather_rows_f32.
        k = 64
        am = synthetic.uniform(43, 0, ROWS * k).reshape(ROWS, k)
        bm = synthetic.uniform(44, 0, k * COLS).reshape(k, COLS)
        p.set_matmul_mode(ctx, p.MatmulMode.REFERENCE)
        with p.tensor(am[r0:r1].ravel(), shape=(r1 - r0, k), context=ctx) as ta, \
                p.tensor(bm.ravel(), shape=(k, COLS), context=ctx) as tbm, p.matmul(ta, tbm) as c:
            gevent = p.b200.gather_rows_into(res.queue, c.descriptor(), targets, row_offset=r0)
            gevent.wait()
            gevent.close()
        barrier.wait(timeout=120)
        gathered = np.frombuffer(mine.read(), np.float32).reshape(ROWS, COLS)
        ok_mm = gathered.tobytes() == oracle.matmul(am.ravel(), bm.ravel(), ROWS, COLS, k).tobytes()
        results.put((rank, ok_ln and ok_mm))
        barrier.wait(timeout=120)  # nobody unmaps while a peer may still read
        for obj in [event, out, tx, tg, tb] + peers:
            obj.close()
        mine.close()
        ctx.close()
    except Exception as error:  # reported to the parent, which fails the test
        results.put((rank, repr(error)))


def test_gather_across_two_gpus():
    if len(p.devices()) < 2:
        pytest.skip("needs two GPUs")
    world = 2
    spawn = mp.get_context("spawn")
    with spawn.Manager() as manager:
        handles = manager.list([None] * world)
        barrier = spawn.Barrier(world)
        results = spawn.Queue()
        procs = [spawn.Process(target=_rank, args=(r, world, handles, barrier, results)) for r in range(world)]
        for proc in procs:
            proc.start()
        outcome = dict(results.get(timeout=300) for _ in range(world))
        for proc in procs:
            proc.join(timeout=120)
    assert outcome == {0: True, 1: True}, outcome
