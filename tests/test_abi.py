"""The drop-in C-ABI boundary, checked without a GPU.

The library must load, export every entry point the include/ headers declare
(the 40 reference symbols of include/paralyn/native.h and tensor.h, plus the
additive include/paralyn/b200.h), keep the reference record layouts, and report
device absence and argument errors with the reference's statuses and operations.
"""
import ctypes as c
from pathlib import Path
import re

import pytest

import paralyn_b200 as p
import importlib
from paralyn_b200 import prk

native_module = importlib.import_module("paralyn_b200.native")
tensor = importlib.import_module("paralyn_b200.tensor")

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    names = set()
    for header in (ROOT / "include" / "paralyn").glob("*.h"):
        names |= set(re.findall(r"^(?:pr_status|uint32_t|uint64_t)\s+(pr_\w+)\(", header.read_text(), re.M))
    return names


def test_headers_declare_reference_symbols():
    declared = declared_symbols()
    assert set(native_module.REFERENCE_SYMBOLS) <= declared
    assert len(native_module.REFERENCE_SYMBOLS) == 40
    assert set(native_module.B200_SYMBOLS) == {name for name in declared if name.startswith("pr_b200_")}


def test_library_exports_every_declared_symbol(lib):
    for name in sorted(declared_symbols()):
        assert hasattr(lib.api, name), name


def test_library_exports_only_the_abi(lib):
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", lib.path], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    assert exported == declared_symbols()


def test_record_layouts():
    assert c.sizeof(native_module.ErrorRecord) == 1092
    assert c.sizeof(native_module.ArgumentRecord) == 32
    assert native_module.ArgumentRecord.f32.offset == 24
    assert c.sizeof(native_module.ParameterRecord) == 4112
    assert c.sizeof(native_module.DeviceRecord) == 440
    assert c.sizeof(native_module.CapabilityRecord) == 224
    assert c.sizeof(native_module.TimingRecord) == 48
    assert c.sizeof(native_module.BackendRecord) == 2112
    assert c.sizeof(tensor.TensorDescRecord) == 160
    assert c.sizeof(tensor.MatmulRecord) == 64
    assert c.sizeof(tensor.LayerNormRecord) == 48
    assert c.sizeof(tensor.AddRecord) == 32
    assert c.sizeof(tensor.CapabilitiesRecord) == 56


def test_abi_version(lib):
    assert lib.api.pr_abi_version() == 1


def test_backend_status_queries(lib):
    cuda = p.backend_status("cuda")
    assert cuda.implemented and cuda.compiler_version >= 12000
    metal = p.backend_status("metal")
    assert not metal.implemented and "Metal" in metal.reason
    hip = p.backend_status("hip")
    assert not hip.implemented
    with pytest.raises(p.Error) as error:
        p.backend_status("opencl")
    assert error.value.code == p.Status.INVALID_ARGUMENT and error.value.operation == "backend_status_get"


def test_versioned_query_rejects_unknown_version(lib):
    record = native_module.versioned(native_module.BackendRecord) if hasattr(native_module, "versioned") else None
    record = native_module.versioned(native_module.BackendRecord)
    record.version = 2
    assert lib.api.pr_backend_status_get(b"cuda", c.byref(record)) == p.Status.UNSUPPORTED
    record.version, record.struct_size = 1, 8
    assert lib.api.pr_backend_status_get(b"cuda", c.byref(record)) == p.Status.INVALID_ARGUMENT


@pytest.mark.skipif(p.backend_status().available, reason="a CUDA device is present")
def test_no_device_is_an_explicit_error(lib):
    assert p.devices() == ()
    with pytest.raises(p.Error) as error:
        p.Context("cuda:0")
    assert error.value.code == p.Status.DEVICE_UNAVAILABLE
    assert error.value.operation == "context_create"
    assert "no CPU fallback" in error.value.message


def test_selector_validation(lib):
    handle = c.c_uint64(123)
    for selector, status in ((b"cuda:", p.Status.DEVICE_UNAVAILABLE), (b"cuda:x", p.Status.DEVICE_UNAVAILABLE),
                             (b"hip:0", p.Status.DEVICE_UNAVAILABLE), (b"metal:0", p.Status.DEVICE_UNAVAILABLE)):
        assert lib.api.pr_context_create(selector, c.byref(handle)) == status
        assert handle.value == 0
    assert lib.api.pr_context_create(b"auto", None) == p.Status.INVALID_ARGUMENT


def test_success_clears_last_error(lib):
    assert lib.api.pr_release(99999) == p.Status.INVALID_HANDLE
    record = native_module.ErrorRecord()
    lib.api.pr_last_error(c.byref(record))
    assert record.code == p.Status.INVALID_HANDLE and record.operation == b"release"
    count = c.c_uint32()
    assert lib.api.pr_device_count(c.byref(count)) == p.Status.SUCCESS
    lib.api.pr_last_error(c.byref(record))
    assert record.code == 0 and record.operation == b"" and record.message == b""
    assert lib.api.pr_last_error(None) == p.Status.INVALID_ARGUMENT


def test_invalid_handles_are_rejected(lib):
    size = c.c_uint64()
    assert lib.api.pr_buffer_size(12345, c.byref(size)) == p.Status.INVALID_HANDLE
    view = c.c_uint64()
    assert lib.api.pr_view_create(12345, 0, 4, 4, 3, c.byref(view)) == p.Status.INVALID_HANDLE
    assert lib.api.pr_event_wait(12345, None) == p.Status.INVALID_HANDLE
    assert lib.api.pr_queue_synchronize(0) == p.Status.INVALID_HANDLE


def test_descriptor_helpers_without_device(lib):
    lib = tensor._api(lib)
    desc = tensor.TensorDescRecord()
    shape = (c.c_uint64 * 3)(2, 3, 2)
    assert lib.api.pr_tensor_desc_contiguous(7, 8, p.Type.F32, 3, shape, c.byref(desc)) == 0
    assert desc.struct_size == 160 and desc.version == 1 and list(desc.strides[:4]) == [6, 2, 1, 0]
    assert lib.api.pr_tensor_desc_contiguous(7, 0, p.Type.F32, 9, shape, c.byref(desc)) == p.Status.INVALID_ARGUMENT
    # Validation needs the buffer: an unknown handle is reported as such.
    assert lib.api.pr_tensor_desc_contiguous(7, 8, p.Type.F32, 3, shape, c.byref(desc)) == 0
    assert lib.api.pr_tensor_desc_validate(c.byref(desc), None) == p.Status.INVALID_HANDLE
    bad = tensor.TensorDescRecord.from_buffer_copy(desc)
    bad.version = 2
    assert lib.api.pr_tensor_desc_validate(c.byref(bad), None) == p.Status.UNSUPPORTED
    bad = tensor.TensorDescRecord.from_buffer_copy(desc)
    bad.dtype = p.Type.I32
    assert lib.api.pr_tensor_desc_validate(c.byref(bad), None) == p.Status.UNSUPPORTED
    bad = tensor.TensorDescRecord.from_buffer_copy(desc)
    bad.byte_offset = 2
    assert lib.api.pr_tensor_desc_validate(c.byref(bad), None) == p.Status.INVALID_ARGUMENT
    bad = tensor.TensorDescRecord.from_buffer_copy(desc)
    bad.shape[5] = 1
    assert lib.api.pr_tensor_desc_validate(c.byref(bad), None) == p.Status.INVALID_ARGUMENT
    bad = tensor.TensorDescRecord.from_buffer_copy(desc)
    bad.strides[1] = -1
    assert lib.api.pr_tensor_desc_validate(c.byref(bad), None) == p.Status.UNSUPPORTED


def test_provider_artifact_and_capabilities(lib):
    artifact = p.tensor_operators_artifact()
    assert artifact[:8] == b"PARALYNB"
    entries = p.inspect_module(artifact)
    assert {"paralyn_matmul_f32", "paralyn_layer_norm_f32", "paralyn_add_f32",
            "paralyn_fill_f32"} <= set(entries)
    caps = p.tensor_operators_capabilities()
    assert {"matmul", "layer_norm", "add", "bias_activation"} <= caps.operations
    assert caps.max_tensor_elements == 2 ** 31 - 1
    assert caps.max_row_operator_rows == 16777215 and caps.max_layer_norm_columns == 2 ** 24
    lib = tensor._api(lib)
    size = c.c_uint64()
    small = c.create_string_buffer(4)
    assert lib.api.pr_tensor_operators_artifact(small, 4, c.byref(size)) == p.Status.OUT_OF_BOUNDS


def test_tensor_operator_records_are_checked_first(lib):
    lib = tensor._api(lib)
    event = c.c_uint64(77)
    record = tensor.LayerNormRecord(c.sizeof(tensor.LayerNormRecord), 2)
    assert lib.api.pr_layer_norm_f32(1, 2, c.byref(record), c.byref(event)) == p.Status.UNSUPPORTED
    assert event.value == 0
    record = tensor.LayerNormRecord(c.sizeof(tensor.LayerNormRecord), 1, float("nan"))
    assert lib.api.pr_layer_norm_f32(1, 2, c.byref(record), c.byref(event)) == p.Status.INVALID_ARGUMENT
    err = native_module.ErrorRecord()
    lib.api.pr_last_error(c.byref(err))
    assert err.operation == b"layer_norm_f32"
    mm = tensor.MatmulRecord(c.sizeof(tensor.MatmulRecord), 1, 1, 1, 1, 2, 0)
    assert lib.api.pr_matmul_f32(1, 2, c.byref(mm), c.byref(event)) == p.Status.INVALID_ARGUMENT


def test_module_inspection_maps_operators():
    entries = p.inspect_module(prk.serialize(prk.operators()))
    assert entries == {"array_add": "ir.add.u32", "array_affine": "ir.affine.u32",
                       "array_affine_scalar": "ir.affine_scalar.u32"}


def test_prepared_operand_sizes(lib):
    from paralyn_b200 import b200
    assert b200.matmul_prepared_bytes(lib, 4096, 4096) == 256 + 4 * 4096 * 4096 + 8 * 4096 * 4096
    assert b200.matmul_prepared_bytes(lib, 33, 300) == 256 + -(-4 * 33 * 300 // 256) * 256 + 8 * 512 * 64
    assert b200.matmul_prepared_bytes(lib, 64, 256) == b200.matmul_prepared_bytes(lib, 32, 512)
    for k, n in ((0, 5), (5, 0), (1 << 31, 5), (5, 1 << 31)):
        assert b200.matmul_prepared_bytes(lib, k, n) == 0


def test_integration_c_examples_compile(tmp_path):
    # The C fragments of INTEGRATION.md, inside a function that declares what they use,
    # compile against include/ (gcc, C11, warnings as errors).
    import shutil
    import subprocess
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not found")
    text = (ROOT / "INTEGRATION.md").read_text()
    blocks = re.findall(r"```c\n(.*?)```", text, re.S)
    assert blocks
    for i, body in enumerate(blocks):
        source = tmp_path / f"example{i}.c"
        source.write_text(
            '#include "paralyn/native.h"\n#include "paralyn/tensor.h"\n#include "paralyn/b200.h"\n'
            "void example(pr_context ctx, pr_queue queue, pr_module operators, pr_buffer w_buf, uint64_t m,\n"
            "             uint64_t n, uint64_t k, pr_tensor_desc_v1 x, pr_tensor_desc_v1 y, pr_tensor_desc_v1 bias) {\n"
            + body + "}\n")
        out = subprocess.run([gcc, "-std=c11", "-Wall", "-Werror", "-fsyntax-only", "-I", str(ROOT / "include"),
                              str(source)], capture_output=True, text=True)
        assert out.returncode == 0, out.stderr


def test_integration_binding_stubs_cover_every_b200_entry():
    # The ctypes stubs INTEGRATION.md gives a maintainer parse as Python and name every
    # pr_b200_* function include/paralyn/b200.h declares, and nothing else.
    import ast
    text = (ROOT / "INTEGRATION.md").read_text()
    stubs = next(b for b in re.findall(r"```python\n(.*?)```", text, re.S) if "optional = {" in b)
    tree = ast.parse(stubs)
    names = set()
    for node in ast.walk(tree):
        if isinstance(node, ast.Dict):
            names |= {k.value for k in node.keys if isinstance(k, ast.Constant) and isinstance(k.value, str)}
    header = (ROOT / "include" / "paralyn" / "b200.h").read_text()
    declared = set(re.findall(r"\b(pr_b200_\w+)\s*\(", header))
    assert names == declared, (sorted(declared - names), sorted(names - declared))
