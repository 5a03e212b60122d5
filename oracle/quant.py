"""Quantisation and scale layout, restated in numpy. Test infrastructure only.

Follows src/cutlass_gemm/quantization.py of the reference:
  _multiplier (:99-112), quantize FP8 (:114-140), NVFP4 (:141-165),
  dequantize (:166-185);
the scale scatter of src/cutlass_gemm/backend.py:124-127; and the CUTLASS
Sm1xxBlkScaledConfig<16> K-major layout the reference's
src/cutlass_gemm/csrc/gemm/nvfp4.cu:122-147 evaluates (pinned against CUTLASS
itself in tests/golden/sf_layout.json).
"""
from __future__ import annotations

import numpy as np

from .formats import e2m1_decode, e2m1_encode, e4m3_decode, e4m3_encode, pack_e2m1, unpack_e2m1

FLT_MAX = np.float32(np.finfo(np.float32).max)
ONE_SIXTH_F32 = np.float32(1.0 / 6.0)


def multiplier(values, precision, global_scale="amax"):
    """st: limit / amax(|x|) in fp32 (1 if amax == 0), or the fixed scale."""
    values = np.asarray(values, np.float32)
    if isinstance(global_scale, str):
        if global_scale != "amax":
            raise ValueError("global_scale must be 'amax' or a positive finite number")
        amax = np.float32(np.max(np.abs(values))) if not np.isnan(values).any() else np.float32(np.nan)
        limit = np.float32(448.0 if precision == "fp8" else 6.0 * 448.0)
        return np.float32(1.0) if amax == 0 else np.float32(limit / amax)
    return np.float32(global_scale)


def quantize_fp8(x, global_scale="amax"):
    """Returns (codes uint8 [R,C], st float32)."""
    x = np.asarray(x, np.float32)
    st = multiplier(x, "fp8", global_scale)
    return e4m3_encode(x * st), st


def quantize_nvfp4(x, global_scale="amax"):
    """Returns (packed codes uint8 [R,C/2], scales uint8 [R,C/16], st float32)."""
    x = np.asarray(x, np.float32)
    rows, cols = x.shape
    if cols % 16:
        raise ValueError("nonempty input columns must be divisible by 16")
    st = multiplier(x, "nvfp4", global_scale)
    blocks = x.reshape(rows, cols // 16, 16)
    amax16 = np.abs(blocks).max(axis=-1)
    scale_values = amax16 * np.float32(st * ONE_SIXTH_F32)
    scales = e4m3_encode(scale_values)
    decoded = e4m3_decode(scales)
    with np.errstate(divide="ignore", over="ignore", invalid="ignore"):
        acc = (np.float32(1.0) / decoded) * st
    acc = np.where(acc > FLT_MAX, FLT_MAX, acc).astype(np.float32)  # clamp_max; NaN passes
    normalized = (blocks * acc[..., None]).reshape(rows, cols)
    return pack_e2m1(e2m1_encode(normalized)), scales, st


def quantize_fp8_block(x, block_rows):
    """Block-scaled FP8: one fp32 scale per (block_rows x 128) block.

    The reference quantises FP8 tensorwise only; this restates the recipe
    named by the benchmark configuration (1 x 128 activation blocks,
    128 x 128 weight blocks): d = amax(|x_block|) / 448 in fp32 (1 when the
    block is all zero), code = e4m3_rn_satfinite(x / d). Returns
    (codes uint8 [R, C], scales float32 [ceil(R / block_rows), C / 128]).
    """
    x = np.asarray(x, np.float32)
    rows, cols = x.shape
    if cols % 128:
        raise ValueError("nonempty input columns must be divisible by 128")
    if block_rows not in (1, 128):
        raise ValueError("block_rows must be 1 or 128")
    row_blocks = -(-rows // block_rows)
    padded = np.zeros((row_blocks * block_rows, cols), np.float32)
    padded[:rows] = x
    blocks = padded.reshape(row_blocks, block_rows, cols // 128, 128)
    amax = np.abs(blocks).max(axis=(1, 3)).astype(np.float32)
    scales = np.where(amax == 0, np.float32(1.0), amax / np.float32(448.0)).astype(np.float32)
    expanded = np.repeat(np.repeat(scales, block_rows, axis=0)[:rows], 128, axis=1)
    return e4m3_encode(x / expanded), scales


def dequantize_fp8_block(codes, scales, block_rows):
    rows, cols = np.asarray(codes).shape
    expanded = np.repeat(np.repeat(np.asarray(scales, np.float32), block_rows, axis=0)[:rows], 128, axis=1)
    return e4m3_decode(codes) * expanded


def dequantize_fp8(codes, st):
    return e4m3_decode(codes) / np.float32(st)


def dequantize_nvfp4(packed, scales, st):
    vals = e2m1_decode(unpack_e2m1(packed))
    rows, cols = vals.shape
    s = e4m3_decode(scales)
    return (vals.reshape(rows, cols // 16, 16) * s[..., None]).reshape(rows, cols) / np.float32(st)


def sf_offset(row, block, k):
    """Byte offset of natural scale (row, block) in the 128x4 atom layout."""
    row = np.asarray(row, np.int64)
    block = np.asarray(block, np.int64)
    k_atoms = (k + 63) // 64
    return ((row >> 7) * k_atoms + (block >> 2)) * 512 + (row & 31) * 16 + ((row >> 5) & 3) * 4 + (block & 3)


def sf_size(rows, k):
    return ((rows + 127) // 128) * 128 * ((k + 63) // 64) * 4


def scale_layout(rows, k):
    r, b = np.meshgrid(np.arange(rows), np.arange(k // 16), indexing="ij")
    return sf_offset(r, b, k)


def pack_scales(scales, k):
    """Natural [rows, k/16] scales -> zero-padded atom layout bytes."""
    scales = np.asarray(scales, np.uint8)
    rows = scales.shape[0]
    out = np.zeros(sf_size(rows, k), np.uint8)
    out[scale_layout(rows, k).reshape(-1)] = scales.reshape(-1)
    return out


def unpack_scales(packed, rows, k):
    return np.asarray(packed, np.uint8)[scale_layout(rows, k)]
