"""Row-sharded LayerNorm with the output gathered over NVLink (pr_b200_layer_norm_gather_f32).

Each rank normalizes its rows [r0, r1) and the same kernel writes every output row
into each rank's gathered [rows, columns] tensor (its own and the peers', mapped
with pr_b200_buffer_export / pr_b200_buffer_import). After all ranks' commands have
completed, every gathered tensor must equal the unsharded LayerNorm of the oracle,
bit for bit. One-GPU cases gather into local buffers; the two-GPU case spawns one
process per GPU (needs a box with at least two B200s, skipped otherwise).
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


ROWS, COLS = 257, 4096


def _rank(rank, world, handles, barrier, results):
    import numpy as np
    import paralyn_b200 as p
    from paralyn_b200 import shard
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
        results.put((rank, gathered.tobytes() == want.tobytes()))
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
