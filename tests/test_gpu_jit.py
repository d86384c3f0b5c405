"""GPU runs of run-time compiled IR: kernels outside the native built-ins are
compiled by NVRTC for sm_100a at module load and launched with the caller's grid.
Results must equal the CPU evaluation of the same IR (oracle/ir_eval.py) bit for
bit; an access outside a bound view is skipped on the device and fails the
command with a clear error instead of touching other memory."""
import json

import numpy as np
import pytest

from oracle import ir_eval
import paralyn_b200 as p
from paralyn_b200 import prk, synthetic

import jit_kernels as jk

pytestmark = pytest.mark.gpu
SCALAR = {prk.I32: p.i32, prk.U32: p.u32, prk.F32: p.f32}


def launch(context, module, kernel, arrays, scalars, grid, block):
    """Runs `kernel` (IR tuple) of `module` on device copies of `arrays`; returns the
    device results and the event's launch variant."""
    name, params, _ = kernel
    buffers, views, args = {}, [], []
    try:
        for pname, ptype, is_buffer, read_only in params:
            if is_buffer:
                host = arrays[pname]
                buffers[pname] = context.buffer(host.nbytes)
                buffers[pname].write(host)
                view = buffers[pname].view(access=p.Access.READ if read_only else p.Access.READ_WRITE)
                views.append(view)
                args.append(view)
            else:
                args.append(SCALAR[ptype](scalars[pname]))
        queue = context.queue()
        try:
            event = queue.launch(module.kernel(name), args, grid=grid, block=block)
            event.wait()
            event.close()
        finally:
            queue.close()
        return {k: np.frombuffer(b.read(), arrays[k].dtype).copy() for k, b in buffers.items()}
    finally:
        for v in views:
            v.close()
        for b in buffers.values():
            b.close()


def check(context, kernel, arrays, scalars, grid, block):
    data = jk.module(kernel)
    with p.Module.load(context, data) as module:
        got = launch(context, module, kernel, arrays, scalars, grid, block)
    want = ir_eval.run(kernel, {**{k: v.copy() for k, v in arrays.items()}, **scalars}, grid, block)
    for name, value in want.items():
        assert got[name].tobytes() == value.tobytes(), name


def test_strided_axpy(context):
    n = 1000
    arrays = {"x": synthetic.uniform(11, 0, n, 3.0), "y": synthetic.uniform(12, 0, n, 3.0),
              "out": np.full(2 * n, 7.0, np.float32)}
    check(context, jk.strided_axpy(), arrays, {"n": n, "a": -1.75}, ((n + 255) // 256, 1, 1), (256, 1, 1))


def test_integer_wrap(context):
    n = 5000
    rng = np.random.default_rng(5)
    arrays = {"a": rng.integers(0, 2 ** 32, n, dtype=np.uint64).astype(np.uint32),
              "b": rng.integers(-2 ** 31, 2 ** 31, n, dtype=np.int64).astype(np.int32),
              "out_u": np.zeros(n, np.uint32), "out_i": np.zeros(2 * n, np.int32)}
    check(context, jk.integer_mix(), arrays, {"n": n}, ((n + 127) // 128, 1, 1), (128, 1, 1))


def test_two_dimensional_grid(context):
    w, h = 37, 21
    arrays = {"src": synthetic.uniform(13, 0, w * h), "out": np.full(w * h, -1.0, np.float32)}
    check(context, jk.transpose_2d(), arrays, {"w": w, "h": h}, (3, 2, 1), (16, 16, 1))


def test_native_and_compiled_kernels_share_a_module(context, tmp_path):
    n = 4096
    kernels = [prk.operators()[0], jk.strided_axpy()]
    with p.Module.load(context, jk.module(*kernels)) as module:
        a, b = synthetic.uniform(14, 0, n), synthetic.uniform(15, 0, n)
        got = launch(context, module, kernels[0], {"a": a, "b": b, "out": np.zeros(n, np.float32)}, {"n": n},
                     (n // 256, 1, 1), (256, 1, 1))
        assert got["out"].tobytes() == (a + b).astype(np.float32).tobytes()
        launch(context, module, kernels[1], {"x": a, "y": b, "out": np.zeros(2 * n, np.float32)}, {"n": n, "a": 2.0},
               (n // 256, 1, 1), (256, 1, 1))
    context.write_evidence(str(tmp_path / "e"))
    launches = json.loads((tmp_path / "e" / "execution.json").read_text())["launches"]
    variants = {l["kernel"]: l["variant"] for l in launches}
    assert variants["strided_axpy"] == "nvrtc_sm_100a" and variants["array_add"] != "nvrtc_sm_100a"


def test_out_of_view_store_is_skipped_and_reported():
    # A context of its own: the failed command makes the context's failure sticky.
    n = 100
    with p.Context("cuda:0") as context:
        kernel = jk.off_by_one()
        with p.Module.load(context, jk.module(kernel)) as module:
            out = context.buffer(4 * n)
            out.write(np.zeros(n, np.float32))
            view = out.view(access=p.Access.READ_WRITE)
            queue = context.queue()
            event = queue.launch(module.kernel("off_by_one"), [view, p.u32(n)], grid=(1, 1, 1), block=(128, 1, 1))
            with pytest.raises(p.Error) as error:
                event.wait()
            assert "outside its bound views" in str(error.value)
            for obj in (event, queue, view, out):
                try:
                    obj.close()
                except p.Error:
                    pass
