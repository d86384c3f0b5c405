"""The reference's own native C++ examples on this library.

oracle/Makefile (target `examples`) compiles examples/native/mlp.cpp and
examples/native/transformer_block.cpp from the reference's sources, with its
header-only C++ wrappers, and links them against paralyn_b200/libparalyn_native.so.
Run unchanged on a B200 they check themselves: the MLP against its float64 bound
(docs/tensors-matmul.md), the pre-LN encoder block every stage against its float64
running bound and its exported evidence against the GPU launches it made. In the
reference summation order the MLP's output hash is the published golden value.
Skipped where the examples were not built (no reference checkout at build time).
"""
import json
import os
import subprocess
from pathlib import Path

import pytest

from test_oracle import MLP_OUTPUT_SHA256

pytestmark = pytest.mark.gpu
REF = Path(__file__).resolve().parent.parent / "oracle" / "_ref"


def run_example(name, args, env_extra, timeout=600):
    exe = REF / name
    if not exe.exists():
        pytest.skip(f"{name} was not built (oracle/Makefile examples)")
    env = dict(os.environ, **env_extra)
    result = subprocess.run([str(exe), *args], env=env, capture_output=True, text=True, timeout=timeout)
    assert result.returncode == 0, result.stdout + result.stderr
    return result.stdout


def test_reference_mlp_example_in_reference_order(tmp_path):
    out = run_example("native_mlp", ["--artifacts", str(tmp_path)], {"PARALYN_MATMUL_MODE": "reference"})
    assert "Verification: PASS" in out
    report = json.loads((tmp_path / "mlp-report.json").read_text())
    assert report["output_sha256"] == MLP_OUTPUT_SHA256
    execution = json.loads((tmp_path / "execution.json").read_text())
    assert len(execution["launches"]) == 4 and execution["cpu_fallback"] is False


@pytest.mark.parametrize("mode", ["auto", "reference"])
def test_reference_mlp_example(tmp_path, mode):
    out = run_example("native_mlp", ["--batch", "300", "--in", "520", "--hidden", "260", "--out", "70"],
                      {"PARALYN_MATMUL_MODE": mode})
    assert "Verification: PASS" in out


@pytest.mark.parametrize("mode", ["auto", "reference"])
def test_reference_transformer_block_example(tmp_path, mode):
    out = run_example("native_transformer_block", ["--artifacts", str(tmp_path)], {"PARALYN_MATMUL_MODE": mode})
    assert "Verification: PASS" in out


def test_reference_transformer_block_example_on_tensor_cores(tmp_path):
    # T=128, d=128, 4 heads, d_ff=512: AUTO runs the QKV and MLP up-projections on the
    # 3xTF32 kernel. (From d_model = 256 the example's own end-to-end bound evaluates to
    # NaN in every mode, the bit-exact reference order included, so it cannot pass.)
    out = run_example("native_transformer_block", ["--tokens", "128", "--model", "128", "--heads", "4",
                                                   "--ff", "512", "--artifacts", str(tmp_path)],
                      {"PARALYN_MATMUL_MODE": "auto"}, timeout=1200)
    assert "Verification: PASS" in out
