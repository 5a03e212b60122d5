"""ctypes loader for the C oracle (cref.c). Test infrastructure only.

The shared object is built on first use with the system C compiler into
``oracle/_build/`` (``-O2 -ffp-contract=off`` keeps every fp32 operation a
single IEEE operation; ``fmaf`` is C99's correctly rounded fused multiply-add).
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SRC = HERE / "cref.c"
LIB = HERE / "_build" / "liboracle.so"
_lib = None


def build() -> Path:
    if not LIB.exists() or LIB.stat().st_mtime < SRC.stat().st_mtime:
        LIB.parent.mkdir(parents=True, exist_ok=True)
        subprocess.run(["gcc", "-O2", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared",
                        str(SRC), "-o", str(LIB), "-lm"], check=True)
    return LIB


def lib():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(str(build()))
        u8 = ctypes.POINTER(ctypes.c_uint8)
        f32 = ctypes.POINTER(ctypes.c_float)
        i64 = ctypes.c_int64
        for name in ("oracle_tile_reference", "oracle_kslice_reference"):
            fn = getattr(_lib, name)
            fn.argtypes = [ctypes.c_int, u8, u8, u8, u8, i64, i64, i64, f32, ctypes.c_int,
                           ctypes.c_float, f32, f32, i64]
            fn.restype = ctypes.c_int
        _lib.oracle_gemm_f64.argtypes = [ctypes.c_int, u8, u8, u8, u8, i64, i64, i64,
                                         ctypes.POINTER(ctypes.c_double)]
        _lib.oracle_gemm_f64.restype = ctypes.c_int
    return _lib


def _u8(x):
    if x is None:
        return ctypes.POINTER(ctypes.c_uint8)()
    x = np.ascontiguousarray(x)
    # fp32 block scales travel as their bytes.
    x = x.view(np.uint8) if x.dtype == np.float32 else x.astype(np.uint8, copy=False)
    return x.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)), x


def _ptr(x):
    return _u8(x) if x is not None else (ctypes.POINTER(ctypes.c_uint8)(), None)


KINDS = {"fp8": 0, "nvfp4": 1, "fp8_block": 2}


def input_reference(kind, a, sfa, b, sfb, m, n, k, weights, alpha, padded_n, layout="tile"):
    """Predicted/magnitude partials [C, Tm, padded_n] (float32).

    kind: "fp8" (a: uint8 e4m3 [m,k], b: [n,k]), "nvfp4" (packed [rows,k/2]
    plus scale atoms) or "fp8_block" (e4m3 plus fp32 scales [m, k/128] and
    [ceil(n/128), k/128]). layout "tile" is the reference's per-M-tile layout.
    """
    weights = np.ascontiguousarray(weights, dtype=np.float32)
    channels = weights.shape[0]
    tiles = (m + 127) // 128
    pred = np.zeros((channels, tiles, padded_n), np.float32)
    mag = np.zeros_like(pred)
    pa, ka = _ptr(a)
    pb, kb = _ptr(b)
    psa, ksa = _ptr(sfa)
    psb, ksb = _ptr(sfb)
    fn = lib().oracle_tile_reference if layout == "tile" else lib().oracle_kslice_reference
    f32 = ctypes.POINTER(ctypes.c_float)
    rc = fn(KINDS[kind], pa, psa, pb, psb, m, n, k, weights.ctypes.data_as(f32), channels,
            ctypes.c_float(np.float32(alpha)), pred.ctypes.data_as(f32), mag.ctypes.data_as(f32), padded_n)
    if rc:
        raise MemoryError("oracle allocation failed")
    return pred, mag


def gemm_f64(kind, a, sfa, b, sfb, m, n, k):
    """Exact-product float64 accumulation of the decoded operands, [m, n]."""
    out = np.zeros((m, n), np.float64)
    pa, ka = _ptr(a)
    pb, kb = _ptr(b)
    psa, ksa = _ptr(sfa)
    psb, ksb = _ptr(sfb)
    rc = lib().oracle_gemm_f64(KINDS[kind], pa, psa, pb, psb, m, n, k,
                               out.ctypes.data_as(ctypes.POINTER(ctypes.c_double)))
    if rc:
        raise MemoryError("oracle allocation failed")
    return out
