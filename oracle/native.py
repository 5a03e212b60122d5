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
        _lib.oracle_tile_reference_subset.argtypes = [ctypes.c_int, u8, u8, u8, u8, i64, i64, i64, f32, ctypes.c_int,
                                                      ctypes.c_float, ctypes.POINTER(ctypes.c_int64), i64, f32, f32,
                                                      i64]
        _lib.oracle_tile_reference_subset.restype = ctypes.c_int
        _lib.oracle_observed_epilogue.argtypes = [f32, i64, i64, f32, ctypes.c_int, f32, i64]
        _lib.oracle_observed_epilogue.restype = ctypes.c_int
        _lib.oracle_row_observed.argtypes = [f32, i64, i64, f32]
        _lib.oracle_row_observed.restype = ctypes.c_int
        _lib.oracle_row_reference.argtypes = [ctypes.c_int, u8, u8, u8, u8, i64, i64, i64, ctypes.c_float, f32, f32]
        _lib.oracle_row_reference.restype = ctypes.c_int
        u16 = ctypes.POINTER(ctypes.c_uint16)
        _lib.oracle_augment_encode.argtypes = [u16, i64, i64, u16, ctypes.c_int, u16]
        _lib.oracle_augment_encode.restype = ctypes.c_int
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


def tile_reference_subset(kind, a, sfa, b, sfb, m, n, k, weights, alpha, padded_n, tiles):
    """TILE-layout predicted/magnitude for the listed M-tiles only: [C, len(tiles), padded_n]."""
    weights = np.ascontiguousarray(weights, dtype=np.float32)
    channels = weights.shape[0]
    tiles = np.ascontiguousarray(tiles, dtype=np.int64)
    pred = np.zeros((channels, tiles.size, padded_n), np.float32)
    mag = np.zeros_like(pred)
    pa, ka = _ptr(a)
    pb, kb = _ptr(b)
    psa, ksa = _ptr(sfa)
    psb, ksb = _ptr(sfb)
    f32 = ctypes.POINTER(ctypes.c_float)
    rc = lib().oracle_tile_reference_subset(KINDS[kind], pa, psa, pb, psb, m, n, k, weights.ctypes.data_as(f32),
                                            channels, ctypes.c_float(np.float32(alpha)),
                                            tiles.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)), tiles.size,
                                            pred.ctypes.data_as(f32), mag.ctypes.data_as(f32), padded_n)
    if rc:
        raise MemoryError("oracle allocation failed")
    return pred, mag


def observed_epilogue(values, weights, padded_n):
    """Observed checksum partials [C, Tm, padded_n] of the fp32 values [m, n]
    the epilogue summed, in the sm_100a epilogue's exact reduction order."""
    values = np.ascontiguousarray(values, dtype=np.float32)
    weights = np.ascontiguousarray(weights, dtype=np.float32)
    m, n = values.shape
    channels = weights.shape[0]
    out = np.zeros((channels, (m + 127) // 128, padded_n), np.float32)
    f32 = ctypes.POINTER(ctypes.c_float)
    lib().oracle_observed_epilogue(values.ctypes.data_as(f32), m, n, weights.ctypes.data_as(f32), channels,
                                   out.ctypes.data_as(f32), padded_n)
    return out


def decoded(kind, codes, scales, rows, k, operand="a", start=0, stop=None):
    """Exact fp32 values of rows [start, stop) of a quantised operand with
    ``rows`` rows and K = k: e4m3 codes; packed e2m1 codes times their ue4m3
    scale (atom layout); or block-scaled e4m3 codes times their fp32 scale
    (1 x 128 for operand "a", 128 x 128 for "b")."""
    from . import formats
    from .quant import scale_layout

    stop = rows if stop is None else stop
    if kind == "fp8":
        return formats.e4m3_decode(np.asarray(codes, np.uint8).reshape(rows, k)[start:stop])
    if kind == "fp8_block":
        block_rows = 1 if operand == "a" else 128
        scales = np.asarray(scales, np.float32)
        idx = np.arange(start, stop) // block_rows
        expanded = np.repeat(scales[idx], 128, axis=1)
        return (formats.e4m3_decode(np.asarray(codes, np.uint8).reshape(rows, k)[start:stop]) * expanded).astype(
            np.float32)
    packed = np.asarray(codes, np.uint8).reshape(rows, k // 2)[start:stop]
    vals = formats.e2m1_decode(formats.unpack_e2m1(packed))
    s = formats.e4m3_decode(np.asarray(scales, np.uint8)[scale_layout(rows, k)[start:stop]])
    return (vals.reshape(stop - start, k // 16, 16) * s[..., None]).reshape(stop - start, k).astype(np.float32)


def gemm_rows_f64(kind, a, sfa, b, sfb, m, n, k, rows, chunk=2048):
    """Float64 reference rows of the decoded product (exact products, the sum
    in float64) and the same rows of |A| |B| (for error bounds): ([r, n], [r, n])."""
    rows = np.asarray(rows, np.int64)
    av = np.concatenate([decoded(kind, a, sfa, m, k, "a", int(r), int(r) + 1) for r in rows]).astype(np.float64)
    out = np.zeros((rows.size, n))
    bound = np.zeros((rows.size, n))
    for c0 in range(0, n, chunk):
        c1 = min(n, c0 + chunk)
        bv = decoded(kind, b, sfb, n, k, "b", c0, c1).astype(np.float64)
        out[:, c0:c1] = av @ bv.T
        bound[:, c0:c1] = np.abs(av) @ np.abs(bv).T
    return out, bound


def augment_encode(a_bits, w_bits):
    """Checksum rows of the augmented BF16 GEMM as bf16 bit patterns
    [C * ceil(m/128), k] from bf16 bits A [m, k] and weights [C, m]."""
    a_bits = np.ascontiguousarray(a_bits, dtype=np.uint16)
    w_bits = np.ascontiguousarray(w_bits, dtype=np.uint16)
    m, k = a_bits.shape
    channels = w_bits.shape[0]
    q = np.zeros((channels * ((m + 127) // 128), k), np.uint16)
    u16 = ctypes.POINTER(ctypes.c_uint16)
    rc = lib().oracle_augment_encode(a_bits.ctypes.data_as(u16), m, k, w_bits.ctypes.data_as(u16), channels,
                                     q.ctypes.data_as(u16))
    if rc:
        raise MemoryError("oracle allocation failed")
    return q


def row_observed(values):
    """Row sums per 64-column block, [ceil(n/64), m], of the fp32 values [m, n]
    the epilogue summed (columns ascending from +0)."""
    values = np.ascontiguousarray(values, dtype=np.float32)
    m, n = values.shape
    out = np.zeros(((n + 63) // 64, m), np.float32)
    f32 = ctypes.POINTER(ctypes.c_float)
    lib().oracle_row_observed(values.ctypes.data_as(f32), m, n, out.ctypes.data_as(f32))
    return out


def row_reference(kind, a, sfa, b, sfb, m, n, k, alpha):
    """(predicted_rows, magnitude_rows) [m] of the row checksums (alpha * A . e^T B
    and |alpha| * |A| . e^T |B|) in the library's order."""
    pred = np.zeros(m, np.float32)
    mag = np.zeros(m, np.float32)
    pa, ka = _ptr(a)
    pb, kb = _ptr(b)
    psa, ksa = _ptr(sfa)
    psb, ksb = _ptr(sfb)
    f32 = ctypes.POINTER(ctypes.c_float)
    rc = lib().oracle_row_reference(KINDS[kind], pa, psa, pb, psb, m, n, k, ctypes.c_float(np.float32(alpha)),
                                    pred.ctypes.data_as(f32), mag.ctypes.data_as(f32))
    if rc:
        raise MemoryError("oracle allocation failed")
    return pred, mag
