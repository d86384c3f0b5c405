"""GPU checks of the runtime around the kernels: events and duration-only timing,
evidence export, ordering on the context queue, the synthetic input generator, the
row-sharded GEMM -> LayerNorm chain on one device, and device-kernel accounting."""
import importlib
import json

import numpy as np
import pytest

import oracle
import paralyn_b200 as p
from paralyn_b200 import synthetic

pytestmark = pytest.mark.gpu
T = importlib.import_module("paralyn_b200.tensor")


def test_context_reports_b200(context):
    device = context.device
    assert device.backend == "CUDA" and device.registry_id == 0x4355444100000001
    caps = context.capabilities
    assert caps.stable_id.startswith("cuda:uuid:") and caps.artifact_formats == p.ARTIFACT_VERIFIED_IR
    assert caps.max_block[0] == 1024 and caps.max_buffer_bytes > 100 << 30


def test_evidence_lists_every_launch(context, tmp_path):
    with p.asarray([1.0, 2.0], context=context) as a, p.add(a, a) as b:
        b.wait()
    context.write_evidence(str(tmp_path / "evidence"))
    record = json.loads((tmp_path / "evidence" / "execution.json").read_text())
    assert record["backend"] == "CUDA" and record["cpu_fallback"] is False
    launch = record["launches"][-1]
    assert launch["kernel"] == "array_add" and launch["command_status"] == "completed"
    assert launch["gpu_duration_valid"] and launch["device_kernels"] == 1
    with pytest.raises(p.Error) as error:  # not new or empty
        context.write_evidence(str(tmp_path / "evidence"))
    assert error.value.code == p.Status.INVALID_ARGUMENT


def test_release_and_cancel_semantics(context):
    a = p.asarray(np.ones(1000, np.float32), context=context)
    b = p.add(a, a)
    with pytest.raises(p.Error) as error:
        b._event.cancel()
    assert error.value.code == p.Status.UNSUPPORTED
    b.close()
    b.close()  # idempotent
    with pytest.raises(p.Error):
        b.to_host()
    a.close()


def test_queue_orders_dependent_work(context):
    x = synthetic.uniform(40, 0, 1 << 22)
    arrays = [p.asarray(x, context=context)]
    for i in range(8):
        arrays.append(p.affine(arrays[-1], arrays[0], 0.5))
    want = x
    for _ in range(8):
        want = oracle.affine(want, x, 0.5)
    assert np.asarray(arrays[-1].to_host(), np.float32).tobytes() == want.tobytes()
    for a in arrays:
        a.close()


@pytest.mark.parametrize("distribution", (p.b200.UNIFORM, p.b200.NORMAL))
def test_synthetic_generator_matches_host_stream(context, distribution):
    count, first = 100003, 12345
    buf = context.buffer(count * 4)
    event = p.fill_synthetic_into(context.queue(), T.TensorDescriptor(buf, (count,)), seed=7,
                                  first_draw=first, distribution=distribution, p0=4.0 if not distribution else 0.5,
                                  p1=2.0)
    event.wait()
    out = np.frombuffer(buf.read(), np.float32)
    if distribution == p.b200.UNIFORM:
        assert out.tobytes() == synthetic.uniform(7, first, count, 4.0).tobytes()
    else:  # float64 log/cos may differ in the last double bit; after rounding to FP32:
        want = synthetic.normal(7, first, count, 0.5, 2.0)
        assert np.mean(out == want) > 0.999 and np.max(np.abs(out - want)) <= 1e-6
    event.close()
    buf.close()


def test_sharded_chain_rows_match_the_whole(context):
    # GEMM -> LayerNorm on row shards [r0, r1) of X equals the same rows of the
    # unsharded result: the sharded path has no exchange step.
    rows, k, n = 96, 256, 512
    x = synthetic.normal(4, 0, rows * k)
    w = synthetic.normal(4, 2 * rows * k, k * n, 0.0, 1.0 / 64.0)
    gamma, beta = np.ones(n, np.float32), np.zeros(n, np.float32)
    p.set_matmul_mode(context, p.MatmulMode.REFERENCE)
    full_z = oracle.matmul(x, w, rows, n, k)
    full = oracle.layer_norm(full_z, gamma, beta, np.float32(1e-5))
    from paralyn_b200 import shard
    with p.tensor(w, shape=(k, n), context=context) as tw, p.tensor(gamma, shape=(n,), context=context) as tg, \
            p.tensor(beta, shape=(n,), context=context) as tb:
        for world in (1, 2, 4):
            for rank in range(world):
                r0, r1 = shard.row_range(rows, world, rank)
                with p.tensor(x[r0 * k:r1 * k], shape=(r1 - r0, k), context=context) as tx, \
                        p.matmul(tx, tw) as z, p.layer_norm(z, tg, tb, epsilon=1e-5) as y:
                    out = np.asarray(y.to_host(), np.float32).reshape(r1 - r0, n)
                assert out.tobytes() == full[r0:r1].tobytes()


def test_device_kernel_count_advances(context):
    before = p.device_kernel_count(context)
    with p.asarray(np.ones(4096, np.float32), context=context) as a, p.add(a, a) as b:
        b.wait()
    assert p.device_kernel_count(context) == before + 1


def test_bounded_wait_failure_path():
    # A wait nothing completes gives up after ~1 ms of SM cycles: the kernel records
    # its status and returns, the command fails and the GPU stays healthy (a new
    # context works). A context of its own: the failure is sticky.
    with p.Context("cuda:0") as ctx:
        queue = ctx.queue()
        event = p.b200.selftest_bounded_wait(queue, 2_000_000)
        with pytest.raises(p.Error) as error:
            event.wait()
        assert error.value.code == p.Status.EXECUTION_FAILED
        assert "abandoned a bounded wait" in str(error.value)
        for obj in (event, queue):
            try:
                obj.close()
            except p.Error:
                pass
    with p.Context("cuda:0") as ctx, p.asarray(np.ones(1000, np.float32), context=ctx) as a, p.add(a, a) as b:
        assert np.all(np.asarray(b.to_host(), np.float32) == 2.0)


def test_queue_hold_delays_later_commands(context):
    # The hold keeps later commands waiting for its duration (device timer), then the
    # queue runs on; lengths above one second are refused before anything is enqueued.
    queue = context.queue()
    before = p.b200.marker(queue)
    hold = p.b200.queue_hold(queue, 0.005)
    after = p.b200.marker(queue)
    assert p.b200.elapsed(before, after) >= 0.0045
    with pytest.raises(p.Error) as error:
        p.b200.queue_hold(queue, 1.5)
    assert error.value.code == p.Status.INVALID_ARGUMENT
    for e in (before, hold, after, queue):
        e.close()
