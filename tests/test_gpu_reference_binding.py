"""The reference's own Python client code running on a B200 through this library.

Two programs of the reference run unchanged from the copies the oracle recipe stages
into oracle/_ref (`make -C oracle binding`: bindings/python/paralyn and
scripts/qualify_cuda.py), each in a child process with PARALYN_LIBRARY pointing at
libparalyn_native.so and PARALYN_OPERATORS at this repository's operators.prk:

  * the binding's array and tensor calls (asarray/add/affine, tensor/matmul/
    layer_norm/bias_add/relu/row_sum/residual_add) on cuda:0, checked against the
    oracle: bit-exact where the reference's arithmetic is, the matmul bit-exact in
    the reference summation order (PARALYN_MATMUL_MODE=reference) and within
    2*k*2^-24*sum|a||b| in the default mode;
  * the qualification harness's own launch_case (reference
    scripts/qualify_cuda.py:60-111): array_add and array_affine at n = 1, 127, 128,
    129, 1000, 65537 and 1000003, view offsets 0 and 3, 28 launches each compared
    bit for bit with the harness's independent FP32 reference including guard
    sentinels, then the harness's evidence and timing checks (:163-169): no CPU
    fallback, backend CUDA, no test double, duration-only timing. The harness's
    `paralyn devices` / `paralyn doctor` steps call the reference's command-line tool,
    which is outside this path, and are not run.
"""
import os
from pathlib import Path
import subprocess
import sys

import pytest

import oracle
import paralyn_b200 as p

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]

BINDING_SCRIPT = r'''
import sys
sys.path[:0] = [sys.argv[1], sys.argv[2]]
import numpy as np
import paralyn as ref
import oracle
from paralyn_b200 import synthetic

mode = sys.argv[3]
with ref.Context("cuda:0") as ctx:
    assert ctx.device.backend == "CUDA"
    for n in (1, 1000, 1000003):
        a, b = synthetic.uniform(11, 0, n, 4.0), synthetic.uniform(11, n, n)
        da, db = ref.asarray(a, context=ctx), ref.asarray(b, context=ctx)
        s, f = ref.add(da, db), ref.affine(da, db, 1.5)
        assert np.asarray(s.to_host(), np.float32).tobytes() == oracle.add(a, b).tobytes()
        assert np.asarray(f.to_host(), np.float32).tobytes() == oracle.affine(a, b, 1.5).tobytes()
        for value in (f, s, db, da):
            value.close()
    m, n, k = 129, 300, 257
    a, b = synthetic.uniform(12, 0, m * k), synthetic.uniform(12, m * k, k * n)
    bias = synthetic.uniform(12, m * k + k * n, n)
    ta, tb = ref.tensor(a, shape=(m, k), context=ctx), ref.tensor(b, shape=(k, n), context=ctx)
    tbias = ref.tensor(bias, shape=(n,), context=ctx)
    c = ref.matmul(ta, tb)
    got = np.asarray(c.to_host(), np.float32).reshape(m, n)
    exact, magnitude = oracle.matmul_exact(a, b, m, n, k)
    assert np.all(np.abs(got - exact) <= oracle.matmul_tolerance(magnitude, k))
    if mode == "reference":
        assert got.tobytes() == oracle.matmul(a, b, m, n, k).tobytes()
    biased = ref.bias_add(c, tbias, relu=True)
    want = oracle.bias_activation(got, bias, 1)
    assert np.asarray(biased.to_host(), np.float32).tobytes() == want.ravel().tobytes()
    rows, cols = 37, 4096
    x = synthetic.normal(13, 0, rows * cols).reshape(rows, cols)
    g, be = synthetic.normal(13, 1 << 20, cols, 1.0, 0.02), synthetic.normal(13, 1 << 21, cols, 0.0, 0.02)
    tx = ref.tensor(x.ravel(), shape=(rows, cols), context=ctx)
    tg, tbe = ref.tensor(g, shape=(cols,), context=ctx), ref.tensor(be, shape=(cols,), context=ctx)
    y = ref.layer_norm(tx, tg, tbe, epsilon=1e-5)
    assert np.asarray(y.to_host(), np.float32).tobytes() == oracle.layer_norm(x, g, be, np.float32(1e-5)).tobytes()
    sums = ref.row_sum(tx)
    assert np.asarray(sums.to_host(), np.float32).tobytes() == oracle.reduce_rows(x, 0).tobytes()
    res = ref.residual_add(tx, y)
    want = oracle.add(x.ravel(), np.asarray(y.to_host(), np.float32))
    assert np.asarray(res.to_host(), np.float32).tobytes() == want.tobytes()
    for value in (res, sums, y, tbe, tg, tx, biased, c, tbias, tb, ta):
        value.close()
print("binding ok", mode)
'''

QUALIFY_SCRIPT = r'''
import importlib.util, json, sys, tempfile
from pathlib import Path
sys.path[:0] = [sys.argv[1]]
spec = importlib.util.spec_from_file_location("qualify_cuda", sys.argv[2])
q = importlib.util.module_from_spec(spec)
spec.loader.exec_module(q)
import paralyn as pr
results = []
with pr.Context("cuda:0") as context:
    assert context.device.backend == "CUDA"
    with pr.Module.load_file(context, sys.argv[3]) as module, context.queue() as queue:
        kernels = {name: module.kernel(name) for name in ("array_add", "array_affine")}
        seed = 20260928
        for name in kernels:
            for n in (1, 127, 128, 129, 1000, 65537, 1000003):
                for offset in (0, 3):
                    results.append(q.launch_case(pr, context, queue, kernels, name, n, seed, offset, "u32"))
                    seed += 1
        for kernel in kernels.values():
            kernel.close()
    out = Path(tempfile.mkdtemp()) / "native"
    context.write_evidence(str(out))
execution = json.loads((out / "execution.json").read_text())
assert execution["cpu_fallback"] is False
assert execution["backend"] == "CUDA" and execution["test_double"] is False
for event in results:
    assert event["completed"] and event["duration_valid"] and not event["timestamps_valid"] \
        and event["clock_domain"] == 1, event
print("qualified", len(results), sum(r["checked_values"] for r in results))
'''


def staged():
    if not (oracle.REF_BINDING / "paralyn" / "__init__.py").exists() or not oracle.REF_QUALIFY.exists():
        pytest.skip("the reference binding is not staged (make -C oracle binding needs the checkout)")


def run(script, *args, mode=None):
    env = dict(os.environ, PARALYN_LIBRARY=str(p.native.DEFAULT_LIBRARY),
               PARALYN_OPERATORS=str(p.array.DEFAULT_OPERATORS))
    env.pop("PARALYN_MATMUL_MODE", None)
    if mode:
        env["PARALYN_MATMUL_MODE"] = mode
    result = subprocess.run([sys.executable, "-c", script, *map(str, args)], env=env, capture_output=True,
                            text=True, timeout=600)
    assert result.returncode == 0, result.stdout + result.stderr
    return result.stdout


@pytest.mark.parametrize("mode", ("reference", "auto"))
def test_reference_binding_calls_on_device(mode):
    staged()
    assert f"binding ok {mode}" in run(BINDING_SCRIPT, oracle.REF_BINDING, ROOT, mode, mode=mode)


def test_reference_qualification_harness():
    staged()
    out = run(QUALIFY_SCRIPT, oracle.REF_BINDING, oracle.REF_QUALIFY, p.array.DEFAULT_OPERATORS)
    words = out.split()
    assert words[0] == "qualified" and int(words[1]) == 28 and int(words[2]) > 2 * 2 * 1066000
