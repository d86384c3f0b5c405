"""The CTA-pair GEMM splitting A itself, ahead of use, equals the split pass bit for bit.

For a product whose A is one matrix stored [m][k] with 16-byte aligned rows, the pair
kernel's converter warps write A's TF32 pair into global memory a work unit ahead of
the TMA loads (claimed 8-row parts, no split pass over A). The pair they write is the
split pass's, so C must be identical to a run with PARALYN_GEMM_SPLIT_AHEAD=0 (which
the library reads once per process: each run is a fresh process). The run without
the split pass enqueues one kernel fewer per command. Shapes cover rows past m inside
the last 128-row band, k tails inside the last 32-column block, one and several
waves of tiles, split-K tail units, and an infinite element of A in AUTO mode.
"""
import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

import oracle
from paralyn_b200 import synthetic

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]

RUN = r"""
import importlib, json, sys
import numpy as np
import paralyn_b200 as p
from paralyn_b200 import synthetic
T = importlib.import_module("paralyn_b200.tensor")
m, n, k, inf, out = int(sys.argv[1]), int(sys.argv[2]), int(sys.argv[3]), int(sys.argv[4]), sys.argv[5]
a = synthetic.uniform(8101 + m, 0, m * k).reshape(m, k)
b = synthetic.uniform(8102 + n, 0, k * n).reshape(k, n)
if inf:
    a[m // 2, k // 3] = np.inf
with p.Context("cuda:0") as ctx:
    res = T.operators_of(ctx)
    bufs = [ctx.buffer(4 * m * k), ctx.buffer(4 * k * n), ctx.buffer(4 * m * n)]
    bufs[0].write(a.ravel())
    bufs[1].write(b.ravel())
    runs = []
    for _ in range(2):  # the second call reuses the workspace and its claim words
        before = p.device_kernel_count(ctx)
        e = T.matmul_into(res.queue, res.module, T.TensorDescriptor(bufs[0], (m, k)),
                          T.TensorDescriptor(bufs[1], (k, n)), T.TensorDescriptor(bufs[2], (m, n)), m=m, n=n, k=k)
        e.wait()
        e.close()
        runs.append((p.device_kernel_count(ctx) - before, bufs[2].read()))
    assert runs[0][1] == runs[1][1]
    open(out, "wb").write(runs[0][1])
    print(json.dumps({"kernels": runs[0][0], "variant": p.b200.last_variant(ctx, "paralyn_matmul_f32")}))
    for buf in bufs:
        buf.close()
"""


def run(tmp_path, m, n, k, inf, ahead):
    out = tmp_path / f"c_{m}_{n}_{k}_{inf}_{ahead}.bin"
    env = dict(os.environ, PARALYN_GEMM_SPLIT_AHEAD="1" if ahead else "0")
    proc = subprocess.run([sys.executable, "-c", RUN, str(m), str(n), str(k), str(inf), str(out)], cwd=ROOT,
                          env=env, capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stderr[-2000:]
    info = json.loads(proc.stdout.strip().splitlines()[-1])
    return info, out.read_bytes()


@pytest.mark.parametrize("m,n,k,inf", [(777, 600, 1000, 0), (300, 4096, 64, 0), (2048, 1024, 260, 0),
                                       (40000, 768, 512, 0), (1000, 1000, 4096, 1)])
def test_split_ahead_equals_the_split_pass(tmp_path, m, n, k, inf):
    ahead, c_ahead = run(tmp_path, m, n, k, inf, True)
    plain, c_plain = run(tmp_path, m, n, k, inf, False)
    assert ahead["variant"] == plain["variant"] == "tcgen05_tf32x3"
    assert ahead["kernels"] == plain["kernels"] - 1  # no split pass over A
    assert c_ahead == c_plain
    c = np.frombuffer(c_ahead, np.float32).reshape(m, n)
    a = synthetic.uniform(8101 + m, 0, m * k).reshape(m, k)
    b = synthetic.uniform(8102 + n, 0, k * n).reshape(k, n)
    if inf:  # row m // 2 holds the infinity: +-inf in every column (NaN where b is 0)
        assert np.all(np.isinf(c[m // 2]) | (b[k // 3] == 0))
    rows = sorted({0, 1, 127, 128, 255, 256, m // 2, m - 1} - ({m // 2} if inf else set()))
    exact, magnitude = oracle.matmul_exact(a[rows].ravel(), b.ravel(), len(rows), n, k)
    assert np.all(np.abs(c[rows].astype(np.float64) - exact) <= oracle.matmul_tolerance(magnitude, k))
