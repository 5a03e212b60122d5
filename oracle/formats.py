"""Narrow float formats, restated in numpy. Test infrastructure only.

The reference converts with the CuTe DSL ``cute.testing._convert`` kernel
(call sites src/cutlass_gemm/quantization.py:33-54,137,149,157), which lowers
to PTX ``cvt.rn.satfinite.{e4m3x2,e2m1x2}.f32``: round to nearest, ties to
even, finite overflow saturates to the largest finite value, NaN stays NaN.
(torch's own ``.to(float8_e4m3fn)`` is *not* used: on the CPU it returns NaN
above 448.) Decodes follow the formats' definitions and the reference's e2m1
table (src/abft/operands.py:109).
"""
from __future__ import annotations

import numpy as np

E2M1_VALUES = np.array([0., .5, 1., 1.5, 2., 3., 4., 6., -0., -.5, -1., -1.5, -2., -3., -4., -6.],
                       dtype=np.float32)


def _round_grid(mag, min_exp, mantissa_bits, max_value):
    """RNE of non-negative float64 ``mag`` onto a binary float grid, saturating."""
    mag = np.asarray(mag, np.float64)
    with np.errstate(divide="ignore", invalid="ignore"):
        exp = np.floor(np.log2(np.where(mag > 0, mag, 1.0)))
    exp = np.maximum(exp, min_exp)
    quantum = np.exp2(exp - mantissa_bits)
    rounded = np.rint(mag / quantum) * quantum  # division by a power of two is exact
    return np.minimum(rounded, max_value)


def e4m3_encode(x):
    """fp32 -> e4m3fn byte (uint8), RN-even, satfinite (|x| >= 448 -> 448)."""
    x = np.asarray(x, np.float32)
    sign = np.signbit(x)
    mag = np.abs(x.astype(np.float64))
    nan = np.isnan(x)
    r = _round_grid(np.where(nan, 0, mag), -6, 3, 448.0)
    # Encode: subnormals are m * 2^-9 (m < 8); normals 2^(e-7) * (1 + m/8).
    sub = r < 2.0 ** -6
    m_sub = np.rint(r / 2.0 ** -9).astype(np.int64)
    with np.errstate(divide="ignore", invalid="ignore"):
        e = np.floor(np.log2(np.where(sub, 1.0, r))).astype(np.int64)
    man = np.rint((np.where(sub, 1.0, r) / np.exp2(e) - 1.0) * 8).astype(np.int64)
    code = np.where(sub, m_sub, ((e + 7) << 3) | man)
    code = np.where(nan, 0x7F, code) | np.where(sign & ~nan, 0x80, 0)
    return code.astype(np.uint8)


def e4m3_decode(b):
    b = np.asarray(b, np.uint8).astype(np.int64)
    sign = np.where(b & 0x80, -1.0, 1.0)
    exp = (b >> 3) & 0xF
    man = b & 7
    val = np.where(exp == 0, man * 2.0 ** -9, (1 + man / 8.0) * np.exp2(exp - 7.0))
    val = np.where((exp == 0xF) & (man == 7), np.nan, val)
    return (sign * val).astype(np.float32)


def e2m1_encode(x):
    """fp32 -> e2m1 nibble (uint8 0..15), RN-even, satfinite (|x| > 6 -> 6)."""
    x = np.asarray(x, np.float32)
    sign = np.signbit(x)
    mag = np.abs(x.astype(np.float64))
    nan = np.isnan(x)
    r = _round_grid(np.where(nan, 0, mag), 0, 1, 6.0)
    # magnitudes {0,.5,1,1.5,2,3,4,6} -> codes 0..7
    lookup = {0.0: 0, 0.5: 1, 1.0: 2, 1.5: 3, 2.0: 4, 3.0: 5, 4.0: 6, 6.0: 7}
    code = np.vectorize(lambda v: lookup[float(v)], otypes=[np.int64])(r) if r.size else r.astype(np.int64)
    # NaN has no e2m1 encoding; the hardware conversion yields the max magnitude.
    code = np.where(nan, 7, code)
    return (code | np.where(sign, 8, 0)).astype(np.uint8)


def e2m1_decode(nibbles):
    return E2M1_VALUES[np.asarray(nibbles, np.uint8) & 15]


def pack_e2m1(nibbles):
    """[rows, 2c] nibbles -> [rows, c] bytes, even column in the low nibble."""
    n = np.asarray(nibbles, np.uint8)
    return (n[:, 0::2] | (n[:, 1::2] << 4)).astype(np.uint8)


def unpack_e2m1(packed):
    p = np.asarray(packed, np.uint8)
    out = np.empty((p.shape[0], p.shape[1] * 2), np.uint8)
    out[:, 0::2] = p & 15
    out[:, 1::2] = p >> 4
    return out


def bf16_round(x):
    """fp32 -> bf16 value (as fp32), round to nearest even."""
    x = np.ascontiguousarray(x, np.float32)
    bits = x.view(np.uint32).astype(np.uint64)
    rounded = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16) << 16
    out = rounded.astype(np.uint32).view(np.float32)
    return np.where(np.isnan(x), x, out)
