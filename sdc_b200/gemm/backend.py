"""Unprotected GEMM entry and NVFP4 scale-layout helpers.

Mirrors src/cutlass_gemm/backend.py of the reference: ``require_device``,
``_scale_layout``, ``_pack_scales`` and ``gemm(a, b, precision, scaling,
global_scale)`` with the same precision/scaling pairs and output contracts
(FP8: fp32 column-major; NVFP4 and BF16: bf16 row-major). The reference's
FP32 SIMT GEMM is outside this path and raises. Extension:
FP8 with ``scaling="blockwise"`` (1 x 128 A / 128 x 128 B fp32 block scales,
bf16 row-major output).
"""
from __future__ import annotations

from functools import lru_cache

import torch

from .. import ops
from .. import require_device as _require

SCALING = {"fp32": "none", "bf16": "none", "fp8": "tensorwise", "nvfp4": "block16"}
SCALINGS = {"fp32": {"none"}, "bf16": {"none"}, "fp8": {"tensorwise", "blockwise"}, "nvfp4": {"block16"}}


def require_device(device):
    _require(device)


@lru_cache(maxsize=128)
def _scale_layout(m, n, k, device):
    """Natural-scale -> atom-layout indices (CPU op), moved to ``device``."""
    ia, ib, size_a, size_b = ops.nvfp4_scale_layout(m, n, k)
    return ia.to(device), ib.to(device), size_a, size_b


def _pack_scales(scales, indices, size):
    storage = torch.zeros(size, device=scales.device, dtype=torch.uint8)
    storage.scatter_(0, indices.flatten(), scales.view(torch.uint8).flatten())
    return storage


def mm(a, b):
    """The reference's FP32/BF16 GEMM entry: BF16 runs on the tcgen05 BF16
    GEMM (fp32 accumulation, bf16 row-major output); the FP32 SIMT GEMM is
    outside this library's path and raises after the device check."""
    require_device(a.device)
    if a.dtype == torch.bfloat16 and b.dtype == torch.bfloat16:
        return ops.mm(a, b)
    raise NotImplementedError("FP32 legacy GEMMs are not part of the sdc_b200 path")


def gemm(a, b, precision, scaling, global_scale="amax"):
    """A @ B through the quantised sm_100a kernel selected by precision."""
    if precision not in SCALINGS or scaling not in SCALINGS[precision]:
        raise ValueError(f"GEMM precision and scaling do not match: {precision}/{scaling}")
    if a.ndim != 2 or b.ndim != 2 or a.shape[1] != b.shape[0] or a.device != b.device:
        raise ValueError("GEMM inputs must be two matching matrices on one device")
    if precision in {"fp32", "bf16"}:
        dtype = torch.float32 if precision == "fp32" else torch.bfloat16
        return mm(a.to(dtype), b.to(dtype))
    require_device(a.device)
    from .quantization import quantize, quantize_blockwise

    if scaling == "blockwise":
        qa, qb = quantize_blockwise(a.contiguous(), 1), quantize_blockwise(b.T.contiguous(), 128)
        return ops.fp8_block_mm(qa.codes.view(torch.float8_e4m3fn), qb.codes.view(torch.float8_e4m3fn),
                                qa.scales, qb.scales)
    qa = quantize(a.contiguous(), precision, global_scale)
    qb = quantize(b.T.contiguous(), precision, global_scale)
    alpha = (qa.multiplier * qb.multiplier).reciprocal()
    if precision == "fp8":
        return ops.fp8_mm(qa.codes.view(torch.float8_e4m3fn), qb.codes.view(torch.float8_e4m3fn), alpha)
    return ops.nvfp4_mm(qa.codes, qb.codes, qa.scales_mma, qb.scales_mma, a.shape[1], alpha)
