"""The drop-in boundary, checked without a GPU.

* libopl_b200.so loads and exports every opl_* function declared in
  include/operatorlib/opl_capi.h and every operatorlib:: launcher of
  include/operatorlib/operators.h (reference operators.h:13-44).
* Argument validation happens before any CUDA call and returns
  cudaErrorInvalidValue (1) exactly where the reference does
  (src/*.cu launchers; operators.h:10-11).
* The torch binding library loads and registers the six schemas verbatim
  (reference python/operatorlib_binding.cpp:190-197).
"""
from __future__ import annotations

import re
import subprocess
from pathlib import Path

import pytest

import operatorlib

REPO = Path(__file__).resolve().parents[1]
INVALID = 1


def declared_capi():
    text = (REPO / "include" / "operatorlib" / "opl_capi.h").read_text()
    return sorted(set(re.findall(r"\b(opl_[a-z0-9_]+)\s*\(", text)))


def test_capi_exports_every_declared_symbol():
    lib = operatorlib.capi()
    names = declared_capi()
    assert "opl_softmax_f32" in names and len(names) >= 12
    for name in names:
        assert hasattr(lib, name), name


def test_cpp_api_symbols_exported():
    out = subprocess.run(["nm", "-DC", str(operatorlib.LIB_PATH)],
                         capture_output=True, text=True, check=True).stdout
    for sig in [
        "operatorlib::reduce_sum_f32(float const*, float*, unsigned long, CUstream_st*)",
        "operatorlib::softmax_f32(float const*, float*, int, int, CUstream_st*)",
        "operatorlib::transpose_f32(float const*, float*, int, int, CUstream_st*)",
        "operatorlib::rmsnorm_f32(float const*, float const*, float*, int, int, float, CUstream_st*)",
        "operatorlib::gemm_f32(float const*, float const*, float*, int, int, int, CUstream_st*)",
        "operatorlib::gemm_f16(__half const*, __half const*, float*, int, int, int, CUstream_st*)",
        "operatorlib::attention_f32(float const*, float const*, float const*, float*, int, int, int, int, bool, CUstream_st*)",
        "operatorlib::attention_f16(__half const*, __half const*, __half const*, float*, int, int, int, int, bool, CUstream_st*)",
    ]:
        assert sig in out, sig


def test_version_names_sm100a():
    assert "sm_100a" in operatorlib.version()


FAKE = 0x1000  # never dereferenced: validation rejects before any launch


@pytest.mark.parametrize("call", [
    lambda L: L.opl_reduce_sum_f32(None, FAKE, 10, None),
    lambda L: L.opl_reduce_sum_f32(FAKE, None, 10, None),
    lambda L: L.opl_reduce_sum_f32(FAKE, FAKE, 0, None),
    lambda L: L.opl_reduce_sum_partial_f64(FAKE, FAKE, 0, None),
    lambda L: L.opl_softmax_f32(FAKE, FAKE, 0, 5, None),
    lambda L: L.opl_softmax_f32(FAKE, FAKE, 5, -1, None),
    lambda L: L.opl_softmax_f32(None, FAKE, 5, 5, None),
    lambda L: L.opl_transpose_f32(FAKE, FAKE, 3, 0, None),
    lambda L: L.opl_transpose_f32(FAKE, None, 3, 3, None),
    lambda L: L.opl_rmsnorm_f32(FAKE, FAKE, FAKE, 2, 8, 0.0, None),
    lambda L: L.opl_rmsnorm_f32(FAKE, FAKE, FAKE, 2, 8, -1e-5, None),
    lambda L: L.opl_rmsnorm_f32(FAKE, FAKE, FAKE, 2, 8, float("nan"), None),
    lambda L: L.opl_rmsnorm_f32(FAKE, None, FAKE, 2, 8, 1e-5, None),
    lambda L: L.opl_rmsnorm_f32(FAKE, FAKE, FAKE, 0, 8, 1e-5, None),
    lambda L: L.opl_gemm_f32(FAKE, FAKE, FAKE, 0, 4, 4, None),
    lambda L: L.opl_gemm_f32(FAKE, None, FAKE, 4, 4, 4, None),
    lambda L: L.opl_gemm_f16(FAKE, FAKE, FAKE, 4, 4, -4, None),
    lambda L: L.opl_gemm_f16(None, FAKE, FAKE, 4, 4, 4, None),
    lambda L: L.opl_attention_f32(FAKE, FAKE, FAKE, FAKE, 1, 1, 8, 129, 0, None),
    lambda L: L.opl_attention_f32(FAKE, FAKE, FAKE, FAKE, 1, 1, 8, 0, 0, None),
    lambda L: L.opl_attention_f16(FAKE, FAKE, FAKE, FAKE, 1, 1, 8, 129, 1, None),
    lambda L: L.opl_attention_f16(FAKE, FAKE, None, FAKE, 1, 1, 8, 64, 1, None),
    lambda L: L.opl_attention_f16(FAKE, FAKE, FAKE, FAKE, 0, 1, 8, 64, 1, None),
])
def test_invalid_arguments_rejected_before_launch(call):
    assert call(operatorlib.capi()) == INVALID


def test_error_string_and_exception_text():
    lib = operatorlib.capi()
    assert lib.opl_error_string(INVALID).decode() == "invalid argument"
    with pytest.raises(operatorlib.OplError, match="softmax launch failed: invalid argument"):
        operatorlib.check("softmax", INVALID)


def test_torch_binding_registers_reference_schemas():
    import torch

    operatorlib.load_operatorlib()
    expected = {
        "reduce_sum": "operatorlib::reduce_sum(Tensor input) -> Tensor",
        "softmax": "operatorlib::softmax(Tensor input) -> Tensor",
        "transpose": "operatorlib::transpose(Tensor input) -> Tensor",
        "rmsnorm": "operatorlib::rmsnorm(Tensor input, Tensor weight, float epsilon=1.0000000000000001e-05) -> Tensor",
        "gemm": "operatorlib::gemm(Tensor a, Tensor b) -> Tensor",
        "attention": "operatorlib::attention(Tensor q, Tensor k, Tensor v, bool causal=False) -> Tensor",
    }
    for name, schema in expected.items():
        op = getattr(torch.ops.operatorlib, name)
        assert str(op.default._schema) == schema


def test_torch_binding_has_no_cpu_kernel():
    """CUDA dispatch key only, like the reference (binding:199-206)."""
    import torch

    operatorlib.load_operatorlib()
    with pytest.raises(NotImplementedError):
        torch.ops.operatorlib.softmax(torch.ones(2, 3))
