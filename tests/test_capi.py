"""The C ABI library loads, exports every declared entry point, and rejects
contract violations before touching a GPU (CPU-only checks)."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

import sdc_b200
from sdc_b200 import capi

HEADER = Path(__file__).resolve().parents[1] / "include" / "sdc_b200.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return re.findall(r"^(?:const char\*|int64_t|size_t|int)\s+(sdc_\w+)\s*\(", text, flags=re.M)


def test_every_declared_symbol_is_exported_and_bound():
    names = declared_functions()
    assert len(names) >= 20
    lib = ctypes.CDLL(str(sdc_b200.LIB_PATH))
    for name in names:
        assert hasattr(lib, name), name
    assert sorted(names) == sorted(capi.PROTOTYPES)


def test_host_layout_functions():
    lib = capi.lib()
    assert lib.sdc_nvfp4_scale_size(130, 64) == 1024
    assert lib.sdc_nvfp4_scale_offset(33, 1, 64) == 16 + 4 + 1
    idx = (ctypes.c_int64 * (3 * 4))()
    capi.check(lib.sdc_nvfp4_scale_layout(3, 64, ctypes.cast(idx, ctypes.c_void_p)))
    assert list(idx) == [0, 1, 2, 3, 16, 17, 18, 19, 32, 33, 34, 35]
    assert lib.sdc_nvfp4_scale_layout(3, 63, None) == capi.SDC_ERR_INVALID


def test_argument_contracts_are_checked_before_launch():
    lib = capi.lib()
    fake = 1 << 20  # never dereferenced: validation fails first
    rc = lib.sdc_abft_fp8_gemm(fake, fake, 136, 144, 128, fake, 0, fake, 0, -1, 0, None, fake, fake, fake, None)
    assert rc == capi.SDC_ERR_INVALID and "fault" in capi.last_error()
    rc = lib.sdc_abft_fp8_gemm(fake, fake, 136, 144, 128, fake, 2, fake, -1, -1, -1, None, fake, fake, fake, None)
    assert rc == capi.SDC_ERR_UNKNOWN_ALGORITHM and "Unknown compiled ABFT algorithm ID" in capi.last_error()
    rc = lib.sdc_fp8_gemm(fake, fake, 136, 144, 100, fake, fake, None)
    assert rc == capi.SDC_ERR_INVALID and "multiple of 16" in capi.last_error()
    rc = lib.sdc_nvfp4_gemm(fake, fake, fake, fake, 136, 144, 48, fake, fake, None)
    assert rc == capi.SDC_ERR_INVALID and "multiple of 32" in capi.last_error()
    rc = lib.sdc_abft_finalize(7, fake, fake, fake, 1, 16, 16, None, 0, fake, fake, 0.0, 0.0, fake, 0, 0, None,
                               None, None, 0, fake, fake, fake, fake, 64, None)
    assert rc == capi.SDC_ERR_UNKNOWN_ALGORITHM
    rc = lib.sdc_fp8_block_gemm(fake, fake, fake, fake, 136, 144, 192, fake, None)
    assert rc == capi.SDC_ERR_INVALID and "multiple of 128" in capi.last_error()
    rc = lib.sdc_abft_fp8_block_gemm(fake, fake, fake, fake, 136, 144, 256, 0, fake, 136, 0, 0, None, fake, fake,
                                     fake, None)
    assert rc == capi.SDC_ERR_INVALID and "fault" in capi.last_error()
    rc = lib.sdc_quantize_fp8_block(fake, 0, 4, 128, 64, fake, fake, None)
    assert rc == capi.SDC_ERR_INVALID and "1 x 128 or 128 x 128" in capi.last_error()
    assert lib.sdc_test_set_watchdog(0, -1) == capi.SDC_ERR_INVALID and "pace_extra" in capi.last_error()
    assert lib.sdc_test_set_watchdog(0, 0) == capi.SDC_OK
    assert lib.sdc_abft_finalize_workspace_bytes(0, 300, 4) == 2 * ((300 + 63) // 64) * 4
    assert lib.sdc_abft_workspace_bytes(0, 256, 64, 128, 0) == 2 * 2 * 2 * 128 * 4


REFERENCE_SCHEMAS = {
    # src/cutlass_gemm/csrc/bindings.cpp:45-62 of the reference.
    "mm": "mm(Tensor a, Tensor b) -> Tensor",
    "fp8_mm": "fp8_mm(Tensor a, Tensor b_rows, Tensor alpha) -> Tensor",
    "nvfp4_mm": "nvfp4_mm(Tensor a_packed, Tensor b_packed, Tensor sfa, Tensor sfb, int k, Tensor alpha) -> Tensor",
    "abft_finalize": "abft_finalize(Tensor partials, Tensor tile_flags, int n, float atol, float rtol, Tensor(a)? reference, bool diagnostics, int algorithm=0, Tensor? thresholds=None) -> (Tensor(a), Tensor, Tensor, Tensor, Tensor, Tensor)",
    "abft_finalize_reference": "abft_finalize_reference(Tensor observed, Tensor predicted, Tensor magnitude, Tensor hit, Tensor nonfinite, int n, float atol, float rtol, Tensor(a)? reference, bool diagnostics, int algorithm=0, Tensor? thresholds=None) -> (Tensor(a), Tensor, Tensor, Tensor, Tensor, Tensor)",
    "abft_fp8_mm": "abft_fp8_mm(Tensor a, Tensor b_rows, Tensor alpha, Tensor weights, int row, int col, int bit, int algorithm=0, Tensor(a!)? nonfinite=None) -> (Tensor, Tensor, Tensor)",
    "abft_nvfp4_mm": "abft_nvfp4_mm(Tensor a_packed, Tensor b_packed, Tensor sfa, Tensor sfb, int k, Tensor alpha, Tensor weights, int row, int col, int bit, int algorithm=0, Tensor(a!)? nonfinite=None) -> (Tensor, Tensor, Tensor)",
    "nvfp4_scale_layout": "nvfp4_scale_layout(int m, int n, int k) -> (Tensor, Tensor, int, int)",
}
# Block-scaled FP8 ops (no reference counterpart) follow the FP8 ops' argument
# order with the fp32 block scales in place of alpha.
BLOCK_SCALED = {
    "fp8_block_mm": "fp8_block_mm(Tensor a, Tensor b_rows, Tensor scale_a, Tensor scale_b) -> Tensor",
    "abft_fp8_block_mm": "abft_fp8_block_mm(Tensor a, Tensor b_rows, Tensor scale_a, Tensor scale_b, Tensor weights, int row, int col, int bit, int algorithm=0, Tensor(a!)? nonfinite=None) -> (Tensor, Tensor, Tensor)",
    "quantize_fp8_block": "quantize_fp8_block(Tensor x, int block_rows) -> (Tensor, Tensor)",
}
# Input-fused ops keep the reference's arguments and add one trailing default.
EXTENDED = {
    "abft_fp8_reference_mm": "abft_fp8_reference_mm(Tensor a, Tensor b_rows, Tensor alpha, Tensor weights, int row, int col, int bit, int algorithm=0, Tensor(a!)? nonfinite=None",
    "abft_nvfp4_reference_mm": "abft_nvfp4_reference_mm(Tensor a_packed, Tensor b_packed, Tensor sfa, Tensor sfb, int k, Tensor alpha, Tensor weights, int row, int col, int bit, int algorithm=0, Tensor(a!)? nonfinite=None",
}


def test_torch_op_schemas_match_reference_bindings():
    sdc_b200.load()
    for name, schema in REFERENCE_SCHEMAS.items():
        assert str(getattr(torch.ops.sdc_cutlass, name).default._schema) == "sdc_cutlass::" + schema
    for name, schema in BLOCK_SCALED.items():
        assert str(getattr(torch.ops.sdc_cutlass, name).default._schema) == "sdc_cutlass::" + schema
    for name, prefix in EXTENDED.items():
        schema = str(getattr(torch.ops.sdc_cutlass, name).default._schema)
        assert schema.startswith("sdc_cutlass::" + prefix + ", int layout=0)")


def test_scale_layout_op_runs_on_cpu():
    ia, ib, sa, sb = torch.ops.sdc_cutlass.nvfp4_scale_layout(160, 192, 256)
    assert ia.shape == (160, 16) and ib.shape == (192, 16)
    assert (sa, sb) == (2 * 128 * 16, 2 * 128 * 16)
    assert ia[33, 5].item() == (33 % 32) * 16 + 4 + 1 + 512
    with pytest.raises(RuntimeError, match="multiple of 32"):
        torch.ops.sdc_cutlass.nvfp4_scale_layout(160, 192, 48)
