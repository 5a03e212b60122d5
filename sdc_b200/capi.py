"""ctypes binding of the sdc_b200 C ABI (include/sdc_b200.h).

This is the stub a non-torch host (or the reference's own Python, via ctypes)
uses to call the kernels directly: plain device pointers as integers, sizes
and a CUDA stream handle. Every declared function gets its prototype here; a
CPU test checks the list against the header and the exported symbols.
"""
from __future__ import annotations

import ctypes
from functools import lru_cache

from . import LIB_PATH

_int = ctypes.c_int
_i64 = ctypes.c_int64
_size = ctypes.c_size_t
_float = ctypes.c_float
_vp = ctypes.c_void_p

SDC_OK = 0
SDC_ERR_INVALID = 1
SDC_ERR_UNSUPPORTED_DEVICE = 2
SDC_ERR_CUDA = 3
SDC_ERR_WORKSPACE = 4
SDC_ERR_UNKNOWN_ALGORITHM = 5
SDC_LAYOUT_TILE = 0
SDC_LAYOUT_KSLICE = 1

PROTOTYPES = {
    "sdc_last_error": (ctypes.c_char_p, []),
    "sdc_device_check": (_int, [_int]),
    "sdc_read_device_error": (_int, [_vp, _vp]),
    "sdc_test_set_watchdog": (_int, [ctypes.c_uint64, ctypes.c_int32]),
    "sdc_test_set_kslice_path": (_int, [_int]),
    "sdc_quantize_workspace_bytes": (_size, [_i64, _i64]),
    "sdc_quantize_fp8": (_int, [_vp, _int, _i64, _i64, _int, _float, _vp, _vp, _vp, _size, _vp]),
    "sdc_quantize_nvfp4": (_int, [_vp, _int, _i64, _i64, _int, _float, _vp, _vp, _vp, _vp, _vp, _size, _vp]),
    "sdc_quantize_fp8_global_amax": (_int, [_vp, _int, _i64, _i64, _vp, _vp, _vp, _vp]),
    "sdc_quantize_nvfp4_global_amax": (_int, [_vp, _int, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _vp]),
    "sdc_nvfp4_scale_offset": (_i64, [_i64, _i64, _i64]),
    "sdc_nvfp4_scale_size": (_i64, [_i64, _i64]),
    "sdc_nvfp4_scale_layout": (_int, [_i64, _i64, _vp]),
    "sdc_nvfp4_pack_scales": (_int, [_vp, _i64, _i64, _vp, _vp]),
    "sdc_fp8_gemm": (_int, [_vp, _vp, _i64, _i64, _i64, _vp, _vp, _vp]),
    "sdc_nvfp4_gemm": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _vp, _vp]),
    "sdc_abft_workspace_bytes": (_size, [_int, _i64, _i64, _i64, _int]),
    "sdc_abft_fp8_gemm": (_int, [_vp, _vp, _i64, _i64, _i64, _vp, _int, _vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp]),
    "sdc_abft_fp8_reference_gemm": (_int, [_vp, _vp, _i64, _i64, _i64, _vp, _int, _vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _int, _vp, _size, _vp]),
    "sdc_abft_nvfp4_gemm": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _int, _vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp]),
    "sdc_abft_nvfp4_reference_gemm": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _int, _vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _int, _vp, _size, _vp]),
    "sdc_quantize_fp8_block": (_int, [_vp, _int, _i64, _i64, _int, _vp, _vp, _vp]),
    "sdc_fp8_block_gemm": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _vp]),
    "sdc_abft_fp8_block_gemm": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _int, _vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp]),
    "sdc_abft_fp8_block_reference_gemm": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _int, _vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _size, _vp]),
    "sdc_abft_correct_fp8_block": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp]),
    "sdc_bf16_gemm": (_int, [_vp, _vp, _i64, _i64, _i64, _vp, _vp]),
    "sdc_abft_reference_gemm_rows": (_int, [_int, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _int, _vp, _i64, _i64,
                                             _i64, _vp, _vp, _vp, _vp, _vp, _vp, _int, _vp, _vp, _size, _vp]),
    "sdc_abft_row_workspace_bytes": (_size, [_i64, _i64]),
    "sdc_abft_row_reference": (_int, [_int, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _size, _vp]),
    "sdc_abft_locate2d_workspace_bytes": (_size, []),
    "sdc_abft_locate2d": (_int, [_vp, _i64, _vp, _vp, _i64, ctypes.c_float, ctypes.c_float, _vp, _vp, _int, _i64,
                                 _vp, _vp, _vp, _vp, _vp, _vp, _vp, _size, _vp]),
    "sdc_abft_augment_encode": (_int, [_vp, _i64, _i64, _int, _vp, _vp, _vp]),
    "sdc_abft_augmented_workspace_bytes": (_size, [_int, _i64, _i64]),
    "sdc_abft_bf16_augmented_gemm": (_int, [_vp, _vp, _i64, _i64, _i64, _int, _vp, _i64, _i64, _i64, _vp, _vp, _vp,
                                            _vp, _vp, _vp, _vp, _size, _vp]),
    "sdc_abft_finalize_workspace_bytes": (_size, [_int, _i64, _i64]),
    "sdc_abft_finalize": (_int, [_int, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _i64, _vp, _vp, _float, _float, _vp, _int, _int, _vp, _vp, _vp, _int, _vp, _vp, _vp, _vp, _size, _vp]),
    "sdc_abft_finalize_noalloc": (_int, [_int, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _i64, _vp, _vp, _float, _float, _vp, _int, _int, _vp, _vp, _vp, _int, _vp, _vp, _vp, _vp]),
    "sdc_abft_locate": (_int, [_vp, _vp, _vp, _i64, _i64, _vp, _vp, _vp]),
    "sdc_abft_correct_fp8": (_int, [_vp, _vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _vp]),
    "sdc_abft_correct_nvfp4": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _vp]),
}


@lru_cache(maxsize=1)
def lib() -> ctypes.CDLL:
    handle = ctypes.CDLL(str(LIB_PATH))
    for name, (restype, argtypes) in PROTOTYPES.items():
        fn = getattr(handle, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return handle


def last_error() -> str:
    return lib().sdc_last_error().decode()


def check(status: int) -> None:
    if status != SDC_OK:
        raise RuntimeError(f"sdc_b200 status {status}: {last_error()}")
