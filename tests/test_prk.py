"""The verified-IR module path (.prk) of the array operators, without a GPU.

operators.prk written by paralyn_b200.prk must be accepted by the reference's own
deserializer and produce, through the reference's CUDA codegen, exactly its
reviewed golden kernels (tests/cuda/golden/array_{add,affine}.cu); the hash of that
output is pinned in tests/golden/reference_vectors.npz. The native library's own
parser/verifier/matcher is exercised through pr_b200_module_inspect, including the
rejections the reference's loader makes (compiler/ir/artifact.cpp:275-313,
compiler/ir/ir.cpp:254-267).
"""
import ctypes
import hashlib
from pathlib import Path
import struct

import numpy as np
import pytest

import oracle
import paralyn_b200 as p
from paralyn_b200 import prk

GOLDEN = np.load(Path(__file__).with_name("golden") / "reference_vectors.npz")


def inspect(data):
    return p.inspect_module(data)


def status_of(data):
    try:
        inspect(data)
        return p.Status.SUCCESS
    except p.Error as error:
        return error.code


def test_operators_module_is_accepted_by_reference_codegen(reference_checkout):
    ref = oracle.reference()
    if ref is None:
        pytest.skip("oracle/_ref not built")
    data = prk.serialize(prk.operators()[:2])
    text = ctypes.create_string_buffer(1 << 16)
    assert ref.ref_prk_emit_cuda(data, len(data), text, len(text)) == 0, text.value
    digest = hashlib.sha256(text.value).digest()
    assert digest == bytes(GOLDEN["prk_emit_cuda_sha256"])
    golden = b"".join((reference_checkout / "tests" / "cuda" / "golden" / f"{name}.cu").read_bytes()
                      for name in ("array_add", "array_affine"))
    assert text.value == golden


def test_scalar_affine_kernel_is_valid_reference_ir(reference_checkout):
    ref = oracle.reference()
    if ref is None:
        pytest.skip("oracle/_ref not built")
    data = prk.serialize(prk.operators())
    text = ctypes.create_string_buffer(1 << 16)
    assert ref.ref_prk_emit_cuda(data, len(data), text, len(text)) == 0, text.value
    assert b"uc_kernel_array_affine_scalar" in text.value
    assert b"__fadd_rn(__fmul_rn(uc_arg_0[uc_local_0], uc_arg_3), uc_arg_4)" in text.value


def test_operators_map_to_native_kernels():
    assert inspect(prk.serialize(prk.operators())) == {
        "array_add": "ir.add.u32", "array_affine": "ir.affine.u32",
        "array_affine_scalar": "ir.affine_scalar.u32"}


def i32_kernels():
    ab = [("a", prk.F32, True, True), ("b", prk.F32, True, True), ("out", prk.F32, True, False),
          ("n", prk.I32, False, False)]
    add = prk.elementwise("vector_add", ab, lambda i: prk.binary("+", prk.F32, prk.load("a", i), prk.load("b", i)),
                          index_type=prk.I32)
    affine = prk.elementwise(
        "affine", ab + [("scale", prk.F32, False, False)],
        lambda i: prk.binary("+", prk.F32, prk.binary("*", prk.F32, prk.load("a", i), prk.ref("scale", prk.F32)),
                             prk.load("b", i)), index_type=prk.I32)
    return [add, affine]


def test_i32_index_variants_map(reference_checkout=None):
    # examples/native/kernels.cu: vector_add / affine with an int index and count.
    assert inspect(prk.serialize(i32_kernels())) == {"vector_add": "ir.add.i32", "affine": "ir.affine.i32"}


def test_commuted_operands_still_match():
    k = prk.elementwise(
        "swapped", [("a", prk.F32, True, True), ("b", prk.F32, True, True), ("out", prk.F32, True, False),
                    ("n", prk.U32, False, False), ("scale", prk.F32, False, False)],
        lambda i: prk.binary("+", prk.F32, prk.load("b", i),
                             prk.binary("*", prk.F32, prk.ref("scale", prk.F32), prk.load("a", i))))
    assert inspect(prk.serialize([k])) == {"swapped": "ir.affine.u32"}


def test_other_verified_ir_is_compiled_at_run_time():
    k = prk.elementwise(
        "array_mul", [("a", prk.F32, True, True), ("b", prk.F32, True, True), ("out", prk.F32, True, False),
                      ("n", prk.U32, False, False)],
        lambda i: prk.binary("*", prk.F32, prk.load("a", i), prk.load("b", i)))
    assert status_of(prk.serialize([k])) == p.Status.SUCCESS
    assert inspect(prk.serialize([k])) == {"array_mul": "nvrtc_sm_100a"}


def test_malformed_containers_fail_compilation():
    good = prk.serialize(prk.operators())
    assert status_of(b"") == p.Status.COMPILATION_FAILED
    assert status_of(b"PARALYX\0" + good[8:]) == p.Status.COMPILATION_FAILED  # magic
    assert status_of(good[:8] + struct.pack("<I", 2) + good[12:]) == p.Status.COMPILATION_FAILED  # format
    assert status_of(good[:12] + struct.pack("<I", 2) + good[16:]) == p.Status.COMPILATION_FAILED  # policy
    assert status_of(good[:-1]) == p.Status.COMPILATION_FAILED  # truncated
    assert status_of(good + b"\0") == p.Status.COMPILATION_FAILED  # trailing data
    empty = prk.MAGIC + struct.pack("<III", 1, 1, 0)
    assert status_of(empty) == p.Status.COMPILATION_FAILED  # no kernels
    duplicate = prk.serialize([prk.operators()[0], prk.operators()[0]])
    assert status_of(duplicate) == p.Status.COMPILATION_FAILED


def test_invalid_ir_fails_verification():
    # Store into a read-only buffer.
    k = prk.elementwise("bad", [("a", prk.F32, True, True), ("b", prk.F32, True, True),
                                ("out", prk.F32, True, True), ("n", prk.U32, False, False)],
                        lambda i: prk.binary("+", prk.F32, prk.load("a", i), prk.load("b", i)))
    assert status_of(prk.serialize([k])) == p.Status.COMPILATION_FAILED
    # Reference to an undefined symbol.
    k = prk.elementwise("bad", [("a", prk.F32, True, True), ("out", prk.F32, True, False),
                                ("n", prk.U32, False, False)],
                        lambda i: prk.binary("+", prk.F32, prk.load("a", i), prk.ref("ghost", prk.F32)))
    assert status_of(prk.serialize([k])) == p.Status.COMPILATION_FAILED


def test_msl_executables_are_metal_only():
    # The reference's CUDA engine rejects PARALYNX executables as Metal-specific
    # (backends/cuda/engine.cpp:588-592).
    assert status_of(b"PARALYNX" + b"\0" * 64) == p.Status.UNSUPPORTED


def test_committed_operator_module_is_current():
    path = Path(p.__file__).with_name("data") / "operators.prk"
    assert path.read_bytes() == prk.serialize(prk.operators())
