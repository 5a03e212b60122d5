"""Operand quantisation on the sm_100a kernels.

Mirrors src/cutlass_gemm/quantization.py of the reference (``quantize``,
``dequantize``, ``QuantizedMatrix``): same precisions, the same ``st``
multiplier policy (``"amax"`` or a positive finite number), the same code and
natural scale layouts. The work is one fused CUDA pass per operand (amax,
scale, round-to-nearest-even saturating cast, packing) instead of torch ops
plus a CuTe conversion kernel; NVFP4 additionally emits its scales directly
in the 128x4 atom layout the block-scaled MMA consumes (``scales_mma``), which
replaces the reference's host index table and scatter.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from numbers import Real

import torch

from .. import ops, require_device


@dataclass(frozen=True)
class QuantizedMatrix:
    """Codes reconstruct as ``decoded_codes * scales / multiplier``.

    Tensorwise FP8 has no block scales. NVFP4 codes hold two E2M1 values per
    byte (even column in the low nibble); ``scales`` holds E4M3 bytes in
    natural ``[rows, columns // 16]`` order and ``scales_mma`` the same bytes
    in the MMA scale-factor layout. ``multiplier`` is a 0-d CUDA float32
    tensor. Block-scaled FP8 (``block_rows`` 1 or 128) holds fp32 ``scales``
    ``[ceil(rows / block_rows), columns // 128]`` and a multiplier of 1.
    """

    codes: torch.Tensor
    scales: torch.Tensor | None
    multiplier: torch.Tensor
    precision: str
    shape: tuple[int, int]
    scales_mma: torch.Tensor | None = None
    block_rows: int | None = None


def _fixed_scale(policy):
    if isinstance(policy, str):
        if policy != "amax":
            raise ValueError("global_scale must be 'amax' or a positive finite number")
        return None
    if isinstance(policy, bool) or not isinstance(policy, Real):
        raise ValueError("global_scale must be 'amax' or a positive finite number")
    if not math.isfinite(policy) or policy <= 0:
        raise ValueError("global_scale must be positive and finite")
    return float(policy)


@torch.no_grad()
def quantize(matrix, precision, global_scale="amax", *, amax=None):
    """Quantize a 2-D CUDA FP32/BF16 matrix to FP8 (tensorwise) or NVFP4.

    ``amax`` (extension): a 0-d CUDA fp32 tensor holding max |x| of a larger
    matrix this one is a row shard of; with the "amax" policy the multiplier
    then comes from it (no host read), so the shard's codes equal the same
    rows of the whole matrix quantised at once."""
    if matrix.device.type != "cuda" or matrix.ndim != 2:
        raise ValueError("quantize requires a two-dimensional CUDA tensor")
    if matrix.dtype not in {torch.float32, torch.bfloat16}:
        raise ValueError("quantize requires FP32 or BF16 input")
    precision = "nvfp4" if precision == "fp4" else precision
    if precision not in {"fp8", "nvfp4"}:
        raise ValueError("precision must be fp8 or nvfp4")
    rows, columns = matrix.shape
    alignment = 4 if precision == "fp8" else 16
    if rows == 0 or columns == 0 or columns % alignment:
        raise ValueError(f"nonempty input columns must be divisible by {alignment}")
    fixed = _fixed_scale(global_scale)
    if amax is not None and fixed is not None:
        raise ValueError("a global amax only applies to the amax policy")
    require_device(matrix.device)
    if amax is not None:
        amax = amax.detach().to(device=matrix.device, dtype=torch.float32).reshape(())
    if precision == "fp8":
        codes, st = ops.quantize_fp8(matrix, fixed, amax)
        return QuantizedMatrix(codes, None, st, precision, (rows, columns))
    codes, scales, packed, st = ops.quantize_nvfp4(matrix, fixed, amax)
    return QuantizedMatrix(codes, scales, st, precision, (rows, columns), packed)


@torch.no_grad()
def quantize_blockwise(matrix, block_rows):
    """Block-scaled FP8: one fp32 scale per (block_rows x 128) block,
    d = amax / 448 (1 for an all-zero block), code = e4m3(x / d). Activations
    use block_rows=1 (1 x 128), weights stored as rows [N, K] 128 (128 x 128).
    The reference quantises FP8 tensorwise only; this is the block recipe of
    the FP8 benchmark configuration."""
    if matrix.device.type != "cuda" or matrix.ndim != 2:
        raise ValueError("quantize requires a two-dimensional CUDA tensor")
    if matrix.dtype not in {torch.float32, torch.bfloat16}:
        raise ValueError("quantize requires FP32 or BF16 input")
    if block_rows not in (1, 128):
        raise ValueError("block_rows must be 1 or 128")
    rows, columns = matrix.shape
    if rows == 0 or columns == 0 or columns % 128:
        raise ValueError("nonempty input columns must be divisible by 128")
    require_device(matrix.device)
    codes, scales = ops.quantize_fp8_block(matrix, block_rows)
    one = torch.ones((), device=matrix.device, dtype=torch.float32)
    return QuantizedMatrix(codes, scales, one, "fp8", (rows, columns), None, block_rows)


_E2M1 = (0., .5, 1., 1.5, 2., 3., 4., 6., -0., -.5, -1., -1.5, -2., -3., -4., -6.)


@torch.no_grad()
def dequantize(matrix: QuantizedMatrix):
    """Decode to float32 (reference checks only; exact for these formats)."""
    if matrix.precision == "fp8" and matrix.block_rows:
        scales = matrix.scales.repeat_interleave(matrix.block_rows, 0)[:matrix.shape[0]]
        return matrix.codes.view(torch.float8_e4m3fn).float() * scales.repeat_interleave(128, 1)
    if matrix.precision == "fp8":
        values = matrix.codes.view(torch.float8_e4m3fn).float()
    else:
        table = torch.tensor(_E2M1, device=matrix.codes.device)
        packed = matrix.codes
        nibbles = torch.stack((packed & 15, packed >> 4), dim=-1).reshape(packed.shape[0], -1).long()
        values = table[nibbles]
        scales = matrix.scales.view(torch.float8_e4m3fn).float()
        values = (values.reshape(*scales.shape, 16) * scales.unsqueeze(-1)).reshape(matrix.shape)
    return values / matrix.multiplier
