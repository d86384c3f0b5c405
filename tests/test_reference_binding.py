"""The reference's own Python binding (bindings/python/paralyn) driving this library.

The drop-in claim at the binding level: with PARALYN_LIBRARY pointing at
libparalyn_native.so from this repository, the reference package loads it (its ABI
check and signature tables, reference bindings/python/paralyn/__init__.py:137-177),
and its device-free calls behave as on the reference. The binding runs unchanged from
the copy the oracle recipe stages into oracle/_ref (`make -C oracle binding`); where
that copy is absent the test skips. The device half is tests/test_gpu_reference_binding.py.
"""
import os
import subprocess
import sys

import pytest

import oracle
import paralyn_b200 as p

SCRIPT = r'''
import sys
sys.path.insert(0, sys.argv[1])
import paralyn as ref
assert ref.ABI_VERSION == 1
caps = ref.tensor_operators_capabilities()
assert {"matmul", "layer_norm", "add"} <= caps.operations, caps
assert caps.max_layer_norm_columns == 2 ** 24
art = ref.tensor_operators_artifact()
assert art[:8] == b"PARALYNB"
print("loaded", len(ref.devices()))
'''


def binding_environment():
    return dict(os.environ, PARALYN_LIBRARY=str(p.native.DEFAULT_LIBRARY),
                PARALYN_OPERATORS=str(p.array.DEFAULT_OPERATORS))


def test_reference_binding_loads_this_library():
    if not (oracle.REF_BINDING / "paralyn" / "__init__.py").exists():
        pytest.skip("the reference binding is not staged (make -C oracle binding needs the checkout)")
    result = subprocess.run([sys.executable, "-c", SCRIPT, str(oracle.REF_BINDING)], env=binding_environment(),
                            capture_output=True, text=True, timeout=120)
    assert result.returncode == 0, result.stderr
    assert result.stdout.split()[0] == "loaded"
