"""Run-time compiled IR (CPU side): kernels that no built-in implements are
compiled by NVRTC straight to sm_100a cubins when a module is loaded or inspected,
and the CPU evaluator of IR (oracle/ir_eval.py) that the GPU tests compare with is
checked against the oracle's own array kernels."""
import numpy as np

import oracle
from oracle import ir_eval
import paralyn_b200 as p
from paralyn_b200 import prk, synthetic

import jit_kernels as jk


def test_unmatched_ir_compiles_for_sm_100a():
    data = jk.module(jk.strided_axpy(), jk.integer_mix(), jk.transpose_2d(), jk.off_by_one(), prk.operators()[0])
    assert p.inspect_module(data) == {"strided_axpy": "nvrtc_sm_100a", "integer_mix": "nvrtc_sm_100a",
                                      "transpose_2d": "nvrtc_sm_100a", "off_by_one": "nvrtc_sm_100a",
                                      "array_add": "ir.add.u32"}


def test_evaluator_matches_the_array_oracle():
    n = 777
    a, b = synthetic.uniform(1, 0, n), synthetic.uniform(2, 0, n)
    out = np.zeros(n, np.float32)
    add, affine = prk.operators()[:2]
    ir_eval.run(add, {"a": a, "b": b, "out": out, "n": n}, ((n + 63) // 64, 1, 1), (64, 1, 1))
    assert out.tobytes() == oracle.add(a, b).tobytes()
    ir_eval.run(affine, {"a": a, "b": b, "out": out, "n": n, "scale": 1.5}, ((n + 63) // 64, 1, 1), (64, 1, 1))
    assert out.tobytes() == oracle.affine(a, b, np.float32(1.5)).tobytes()


def test_evaluator_integer_wrap_and_strides():
    n = 40
    a = np.arange(n, dtype=np.uint32) * np.uint32(123456789)
    b = (np.arange(n, dtype=np.int32) - 20) * np.int32(100000000)
    out_u, out_i = np.zeros(n, np.uint32), np.zeros(2 * n, np.int32)
    ir_eval.run(jk.integer_mix(), {"a": a, "b": b, "out_u": out_u, "out_i": out_i, "n": n}, (2, 1, 1), (32, 1, 1))
    want_u = [(int(v) * 2654435761 + i) & 0xFFFFFFFF for i, v in enumerate(a)]
    want_i = [(int(v) * -3 + 2147483647) & 0xFFFFFFFF for v in b]
    assert np.array_equal(out_u, np.array(want_u, np.uint32))
    assert np.array_equal(out_i[:n], np.array(want_i, np.uint32).view(np.int32))
    assert np.array_equal(out_i[n:], a.view(np.int32))
    x, y = synthetic.uniform(3, 0, 50), synthetic.uniform(4, 0, 50)
    out = np.full(100, 7.0, np.float32)
    ir_eval.run(jk.strided_axpy(), {"x": x, "y": y, "out": out, "n": 50, "a": -2.0}, (1, 1, 1), (64, 1, 1))
    v = (x * np.float32(-2.0) + y).astype(np.float32)
    assert out[0::2].tobytes() == v.tobytes()
    assert np.all(out[1::2][v >= 0] == 7.0) and out[1::2][v < 0].tobytes() == (v[v < 0] * v[v < 0]).tobytes()
