"""The reference's own Python binding (bindings/python/paralyn) driving this library.

The drop-in claim at the binding level: with PARALYN_LIBRARY pointing at
libparalyn_native.so from this repository, the reference package loads it (its ABI
check and signature tables, reference bindings/python/paralyn/__init__.py:137-177),
and its device-free calls behave as on the reference. Runs only where the reference
checkout exists; GPU machines have no reference checkout.
"""
import os
import subprocess
import sys

import pytest

import paralyn_b200 as p

SCRIPT = r'''
import sys
sys.path.insert(0, "/root/reference/bindings/python")
import paralyn as ref
assert ref.ABI_VERSION == 1
caps = ref.tensor_operators_capabilities()
assert {"matmul", "layer_norm", "add"} <= caps.operations, caps
assert caps.max_layer_norm_columns == 2 ** 24
art = ref.tensor_operators_artifact()
assert art[:8] == b"PARALYNB"
devices = ref.devices()
try:
    ctx = ref.Context("cuda:0")
except ref.Error as error:
    assert error.code == ref.Status.DEVICE_UNAVAILABLE and error.operation == "context_create", error
    print("no-device", len(devices))
else:
    a = ref.asarray([1.0, 2.0, 3.0], context=ctx)
    b = ref.add(a, a)
    assert list(b.to_host()) == [2.0, 4.0, 6.0]
    x = ref.tensor([1.0, 2.0, 3.0, 4.0], shape=(2, 2), context=ctx)
    y = ref.matmul(x, x)
    assert list(y.to_host()) == [7.0, 10.0, 15.0, 22.0]
    for value in (b, a, y, x):
        value.close()
    ctx.close()
    print("device", len(devices))
'''


def test_reference_binding_loads_this_library(reference_checkout):
    env = dict(os.environ, PARALYN_LIBRARY=str(p.native.DEFAULT_LIBRARY),
               PARALYN_OPERATORS=str(p.array.DEFAULT_OPERATORS))
    result = subprocess.run([sys.executable, "-c", SCRIPT], env=env, capture_output=True, text=True, timeout=120)
    assert result.returncode == 0, result.stderr
    assert result.stdout.strip().split()[0] in ("no-device", "device")
