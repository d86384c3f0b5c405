"""Regenerates tests/golden/reference_vectors.npz from the reference's OWN code.

Run in a checkout where the reference is present (it compiles oracle/_ref from the
reference sources: `make -C oracle ref`):

    python tests/golden/make_golden.py

Contents (inputs are seeded synthetic data from paralyn_b200.synthetic):
  tree_<n>_x / tree_<n>_sum   the reference's tree_sum_f32 of synthetic.uniform(100+i, 0, n, 4)
                              (examples/native/transformer_reference.hpp:172-181)
  ln_<r>x<c>_{x,gamma,beta,value,error,eps}
                              the reference's float64 LayerNorm bound layer_norm_row
                              (same header :133-147) on the LayerNorm test shapes of
                              tests/native/transformer_ops_tests.cpp:397-400
  tmax_<n>                    the reference's tree_max_f32 of the same tree inputs (:182-191)
  tmax_special_{x,max}        tree_max_f32 of the NaN / signed-zero / infinity rows of
                              tests/native/transformer_ops_tests.cpp:277-283
  sm_<b>x<r>x<c>_{x,value,error,meta}
                              the reference's float64 softmax_row bound (same header
                              :122-132) on the softmax test shapes of
                              tests/native/transformer_ops_tests.cpp:341-350 (columns
                              <= 1000); meta = (scale, causal)
  dot_<k>_{a,b,value,error}   the reference's float64 dot bound (same header :101-111)
  gelu_{x,value,error}        the reference's float64 GELU bound (same header :113-121) on
                              synthetic.uniform(900, 0, 1000, 8) and the saturation and
                              special points of tests/native/transformer_ops_tests.cpp:482-499
  prk_emit_cuda_sha256        SHA-256 of the CUDA the reference's codegen emits for
                              paralyn_b200.prk.operators() (must equal the reference's
                              reviewed goldens tests/cuda/golden/array_{add,affine}.cu)
GPU machines have no reference checkout, so the GPU tests read these vectors.
"""
import ctypes
import hashlib
from pathlib import Path
import subprocess
import sys

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import oracle  # noqa: E402
from paralyn_b200 import prk, synthetic  # noqa: E402

TREE_LENGTHS = (1, 7, 255, 256, 257, 1000, 4096, 100003)
# (rows, columns, center, magnitude, epsilon) of the reference LayerNorm test cases.
LN_CASES = ((1, 1, 0.0, 1.0, 1e-5), (3, 17, 0.5, 2.0, 1e-5), (4, 256, 0.0, 1.0, 1e-5),
            (2, 257, -3.0, 4.0, 1e-6), (5, 1000, 0.0, 1.0, 1e-5), (3, 64, 1000.0, 1.0, 1e-5),
            (2, 48, 0.0, 1e-3, 1e-2))


# (batch, rows, columns, scale, magnitude, causal) of the reference softmax cases with
# at most 1000 columns.
SOFTMAX_CASES = ((1, 1, 1, 1.0, 4.0, False), (1, 3, 17, 1.0, 4.0, False), (1, 5, 256, 0.125, 16.0, False),
                 (1, 2, 1000, 1.0, 8.0, False), (4, 9, 9, 0.35355339, 8.0, True), (2, 5, 12, 1.0, 8.0, True),
                 (3, 7, 7, 3.0, 4.0, False), (1, 1, 300, 1.0, 100.0, True), (1, 17, 17, 1.0, 60.0, True))
DOT_LENGTHS = (1, 5, 16, 47, 257, 300)


def main():
    subprocess.run(["make", "-s", "-C", str(ROOT / "oracle"), "all", "ref"], check=True)
    ref = oracle.reference()
    if ref is None:
        raise SystemExit("oracle/_ref/libref.so was not built (is the reference checkout present?)")
    out = {}
    for i, n in enumerate(TREE_LENGTHS):
        x = synthetic.uniform(100 + i, 0, n, 4.0)
        if n <= 4096:  # larger inputs are regenerated from the same seeded stream
            out[f"tree_{n}_x"] = x
        out[f"tree_{n}_sum"] = np.array([ref.ref_tree_sum_f32(x, n)], np.float32)
    for i, (rows, cols, center, magnitude, eps) in enumerate(LN_CASES):
        x = (synthetic.uniform(200 + i, 0, rows * cols, magnitude) + np.float32(center)).astype(np.float32)
        g = synthetic.uniform(300 + i, 0, cols, 2.0)
        b = synthetic.uniform(400 + i, 0, cols, 0.5)
        value = np.empty((rows, cols), np.float64)
        error = np.empty((rows, cols), np.float64)
        for r in range(rows):
            v = np.empty(cols, np.float64)
            e = np.empty(cols, np.float64)
            # epsilon enters as double(float epsilon), as in transformer_ops_tests.cpp:418
            ref.ref_layer_norm_row(np.ascontiguousarray(x[r * cols:(r + 1) * cols]), g, b, cols,
                                   float(np.float32(eps)), v, e)
            value[r], error[r] = v, e
        key = f"ln_{rows}x{cols}"
        out[key + "_x"] = x.reshape(rows, cols)
        out[key + "_gamma"], out[key + "_beta"] = g, b
        out[key + "_value"], out[key + "_error"] = value, error
        out[key + "_eps"] = np.array([eps], np.float32)
    for i, n in enumerate(TREE_LENGTHS):
        x = synthetic.uniform(100 + i, 0, n, 4.0)
        out[f"tmax_{n}"] = np.array([ref.ref_tree_max_f32(x, n)], np.float32)
    nan, inf = np.float32(np.nan), np.float32(np.inf)
    special = np.array([[1, nan, -2, 3], [-0.0, 0.0, -0.0, -1], [-0.0, -0.0, -3, -1], [inf, -inf, 1, 2],
                        [-inf, -inf, -inf, -inf], [inf, 1, inf, 0]], np.float32)
    out["tmax_special_x"] = special
    out["tmax_special_max"] = np.array([ref.ref_tree_max_f32(np.ascontiguousarray(r), 4) for r in special],
                                       np.float32)
    for i, (batch, rows, cols, scale, magnitude, causal) in enumerate(SOFTMAX_CASES):
        x = synthetic.uniform(500 + i, 0, batch * rows * cols, magnitude).reshape(batch * rows, cols)
        value = np.empty_like(x, dtype=np.float64)
        error = np.empty_like(x, dtype=np.float64)
        for r in range(batch * rows):
            visible = (r % rows) + (cols - rows) + 1 if causal else cols
            ref.ref_softmax_row(np.ascontiguousarray(x[r]), cols, float(np.float32(scale)), visible, value[r], error[r])
        key = f"sm_{batch}x{rows}x{cols}"
        out[key + "_x"], out[key + "_value"], out[key + "_error"] = x, value, error
        out[key + "_meta"] = np.array([np.float32(scale), float(causal)], np.float64)
    for i, k in enumerate(DOT_LENGTHS):
        a = synthetic.uniform(600 + i, 0, k, 2.0)
        b = synthetic.uniform(700 + i, 0, k, 3.0)
        v, e = ctypes.c_double(), ctypes.c_double()
        ref.ref_dot(a, b, k, ctypes.byref(v), ctypes.byref(e))
        out[f"dot_{k}_a"], out[f"dot_{k}_b"] = a, b
        out[f"dot_{k}_value"] = np.array([v.value])
        out[f"dot_{k}_error"] = np.array([e.value])
    gx = np.concatenate([synthetic.uniform(900, 0, 1000, 8.0),
                         np.array([30, -30, 0, -0.0, 1e-20, -1e-3, 5.5, -5.5], np.float32)]).astype(np.float32)
    gv, ge = np.empty(gx.size, np.float64), np.empty(gx.size, np.float64)
    ref.ref_gelu(gx, gx.size, gv, ge)
    out["gelu_x"], out["gelu_value"], out["gelu_error"] = gx, gv, ge
    data = prk.serialize(prk.operators()[:2])
    text = ctypes.create_string_buffer(1 << 16)
    if ref.ref_prk_emit_cuda(data, len(data), text, len(text)) != 0:
        raise SystemExit("reference rejected the operators module: " + text.value.decode())
    out["prk_emit_cuda_sha256"] = np.frombuffer(hashlib.sha256(text.value).digest(), np.uint8)
    np.savez_compressed(Path(__file__).with_name("reference_vectors.npz"), **out)
    print("wrote", len(out), "arrays")


if __name__ == "__main__":
    main()
