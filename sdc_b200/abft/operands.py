"""Prepared GEMM operands: quantise once, run native kernels, decode K blocks.

Mirrors src/abft/operands.py of the reference (``PreparedGemm``): the same
fields, ``prepare`` (FP8/NVFP4 through this library's quantizer, B transposed
to K-major rows), ``raw_native`` / ``collected_native`` /
``collected_reference_native`` op routing, the CPU-capable ``decode_block``
and ``injected`` input-code bit flips (NVFP4 nibble rule). BF16 operands run on
the tcgen05 BF16 GEMM (``raw_native``) and the augmented ABFT GEMM
(``augmented_native`` / ``augmented_compact``); FP32 operands are kept for
the separate reference mode and CPU tests, their native GEMMs are outside
this path. Extension: FP8 ``scaling="blockwise"`` (1 x 128 A and
128 x 128 B fp32 block scales in ``sfa``/``sfb``, no alpha) routes to the
block-scaled ops, whose input-fused prediction has the K-slice layout only.
"""
from __future__ import annotations

from dataclasses import dataclass, replace
from typing import Any

import torch

SCALING = {"fp32": "none", "bf16": "none", "fp8": "tensorwise", "nvfp4": "block16"}
SCALINGS = {"fp32": {"none"}, "bf16": {"none"}, "fp8": {"tensorwise", "blockwise"}, "nvfp4": {"block16"}}
INPUT_REFERENCE_PRECISIONS = frozenset({"fp8", "nvfp4"})
LAYOUTS = {"tile": 0, "kslice": 1}
_E2M1 = (0., .5, 1., 1.5, 2., 3., 4., 6., -0., -.5, -1., -1.5, -2., -3., -4., -6.)


def _ops():
    from .. import ops
    return ops


@dataclass
class PreparedGemm:
    a: torch.Tensor
    b: torch.Tensor
    precision: str
    m: int
    n: int
    k: int
    qa: Any = None
    qb: Any = None
    alpha: Any = None
    sfa: Any = None
    sfb: Any = None
    scaling: str = ""

    def __post_init__(self):
        if not self.scaling:
            self.scaling = SCALING[self.precision]

    @property
    def blockwise(self):
        return self.scaling == "blockwise"

    @classmethod
    def prepare(cls, a, b, precision, scaling, global_scale="amax"):
        if precision not in SCALINGS or scaling not in SCALINGS[precision]:
            raise ValueError("Incompatible precision/scaling")
        if a.ndim != 2 or b.ndim != 2 or a.shape[1] != b.shape[0] or a.device != b.device:
            raise ValueError("GEMM requires compatible matrices on one device")
        m, k = a.shape
        n = b.shape[1]
        if min(m, n, k) <= 0:
            raise ValueError("Empty GEMM is not supported")
        if precision == "bf16":
            # The sm_100a GEMM reads A row-major and B as K-major rows, i.e.
            # B [K, N] column-major: repack once here instead of every call.
            a, b = a.to(torch.bfloat16).contiguous(), b.to(torch.bfloat16)
            if not b.T.is_contiguous():
                b = b.T.contiguous().T
            return cls(a, b, precision, m, n, k)
        if precision == "fp32":
            return cls(a.float(), b.float(), precision, m, n, k)
        from .. import require_device
        from ..gemm.quantization import quantize, quantize_blockwise

        require_device(a.device)
        if scaling == "blockwise":
            qa, qb = quantize_blockwise(a.contiguous(), 1), quantize_blockwise(b.T.contiguous(), 128)
            return cls(qa.codes, qb.codes, precision, m, n, k, qa, qb, None, qa.scales, qb.scales, scaling)
        qa = quantize(a.contiguous(), precision, global_scale)
        qb = quantize(b.T.contiguous(), precision, global_scale)
        alpha = (qa.multiplier * qb.multiplier).reciprocal()
        prepared = cls(qa.codes, qb.codes, precision, m, n, k, qa, qb, alpha)
        if precision == "nvfp4":
            prepared.sfa, prepared.sfb = qa.scales_mma, qb.scales_mma
        return prepared

    def _native_args(self):
        if self.blockwise:
            return (self.a.view(torch.float8_e4m3fn), self.b.view(torch.float8_e4m3fn), self.sfa, self.sfb)
        if self.precision == "fp8":
            return (self.a.view(torch.float8_e4m3fn), self.b.view(torch.float8_e4m3fn), self.alpha)
        if self.precision == "nvfp4":
            return (self.a, self.b, self.sfa, self.sfb, self.k, self.alpha)
        raise NotImplementedError(f"native {self.precision} GEMMs are outside the FP8/NVFP4 path")

    def raw_native(self):
        if self.precision in {"fp32", "bf16"}:
            from ..gemm import backend
            return backend.mm(self.a, self.b)
        ops = _ops()
        gemm = ops.fp8_block_mm if self.blockwise else ops.fp8_mm if self.precision == "fp8" else ops.nvfp4_mm
        return gemm(*self._native_args())

    def collected_native(self, weights, fault=(-1, -1, -1), *, algorithm=0, nonfinite=None):
        """Output, observed partials and hit (epilogue checksums only)."""
        ops = _ops()
        if self.precision in {"fp32", "bf16"}:
            from .. import require_device
            require_device(self.a.device)
            return ops.abft_mm(self.a, self.b, weights, *fault, algorithm, nonfinite)
        op = (ops.abft_fp8_block_mm if self.blockwise else ops.abft_fp8_mm if self.precision == "fp8"
              else ops.abft_nvfp4_mm)
        return op(*self._native_args(), weights, *fault, algorithm, nonfinite)

    def collected_reference_native(self, weights, fault=(-1, -1, -1), *, algorithm=0, nonfinite=None,
                                   layout="tile"):
        """Output, observed, hit, predicted and magnitude partials."""
        if self.precision not in INPUT_REFERENCE_PRECISIONS:
            raise NotImplementedError(f"input_fused reference is not implemented for {self.precision}")
        ops = _ops()
        if self.blockwise:
            if layout != "kslice":
                raise NotImplementedError("block-scaled FP8 computes its input-fused prediction in the kslice "
                                          "layout only")
            return ops.abft_fp8_block_reference_mm(*self._native_args(), weights, *fault, algorithm, nonfinite)
        op = ops.abft_fp8_reference_mm if self.precision == "fp8" else ops.abft_nvfp4_reference_mm
        return op(*self._native_args(), weights, *fault, algorithm, nonfinite, LAYOUTS[layout])

    def collected_rows_native(self, weights, fault=(-1, -1, -1), *, algorithm=0, nonfinite=None, layout="tile"):
        """``collected_reference_native`` plus the row checksums: observed
        row sums per 64-column block [ceil(N/64), M], predicted row sums
        alpha * A (B^T e) [M] and their magnitude [M]."""
        if self.precision not in INPUT_REFERENCE_PRECISIONS:
            raise NotImplementedError(f"row checksums are not implemented for {self.precision}")
        ops = _ops()
        a, b = self.a, self.b
        if self.blockwise:
            if layout != "kslice":
                raise NotImplementedError("block-scaled FP8 computes its input-fused prediction in the kslice "
                                          "layout only")
            args = (2, a.view(torch.float8_e4m3fn), self.sfa, b.view(torch.float8_e4m3fn), self.sfb, self.k, None)
        elif self.precision == "fp8":
            args = (0, a.view(torch.float8_e4m3fn), None, b.view(torch.float8_e4m3fn), None, self.k, self.alpha)
        else:
            args = (1, a, self.sfa, b, self.sfb, self.k, self.alpha)
        return ops.abft_reference_rows_mm(*args, weights, *fault, algorithm, nonfinite, LAYOUTS[layout])

    def augmented_native(self, weights, fault=(-1, -1, -1), *, algorithm=0):
        """Output, observed, hit, predicted and magnitude partials of the
        augmented BF16 GEMM (the checksum rows are extra M-tiles of the same
        tcgen05 GEMM; magnitude is the output-side sum |w v|)."""
        if self.precision != "bf16":
            raise ValueError("augmented currently requires BF16 GEMM")
        from .. import require_device
        require_device(self.a.device)
        return _ops().abft_augmented_mm(self.a, self.b, weights, *fault, algorithm)

    def augmented_compact(self, weights, fault=(-1, -1, -1), *, algorithm=0):
        """Output, packed partials [3, C, Tm, padded_N] and per-tile flags of
        the augmented BF16 GEMM (the native engine's form)."""
        if self.precision != "bf16":
            raise ValueError("augmented currently requires BF16 GEMM")
        return _ops().abft_augmented_compact(self.a, self.b, weights, *fault, algorithm)

    def decode_block(self, start, end):
        """Decoded fp32 A[:, start:end] and B[start:end, :] (works on the CPU)."""
        if not 0 <= start < end <= self.k:
            raise ValueError("Invalid K block")
        if self.precision == "nvfp4" and (start % 16 or end % 16):
            raise ValueError("NVFP4 reference blocks must align to block16 scales")
        if self.precision in {"fp32", "bf16"}:
            return self.a[:, start:end].float(), self.b[start:end, :].float()

        def decode(codes, q):
            if self.blockwise:
                scales = q.scales[:, start // 128:(end + 127) // 128].repeat_interleave(q.block_rows, 0)
                scales = scales[:codes.shape[0]].repeat_interleave(128, 1)
                offset = start - (start // 128) * 128
                return codes[:, start:end].view(torch.float8_e4m3fn).float() * scales[:, offset:offset + end - start]
            if self.precision == "fp8":
                return codes[:, start:end].view(torch.float8_e4m3fn).float() / q.multiplier
            packed = codes[:, start // 2:end // 2]
            nibbles = torch.stack((packed & 15, packed >> 4), dim=-1).reshape(codes.shape[0], end - start).long()
            values = torch.tensor(_E2M1, device=codes.device)[nibbles]
            scales = q.scales[:, start // 16:end // 16].view(torch.float8_e4m3fn).float()
            blocks = values.reshape(values.shape[0], -1, 16) * scales.unsqueeze(-1)
            return blocks.reshape_as(values) / q.multiplier

        return decode(self.a, self.qa), decode(self.b, self.qb).T

    def injected(self, config):
        """Copy of the operands with one input-code bit flipped (the clean
        buffers are untouched). Logical B coordinates map to the B rows."""
        if config.location not in {"a", "b"}:
            raise ValueError("Prepared input injection requires location a or b")
        rows, cols = (self.m, self.k) if config.location == "a" else (self.k, self.n)
        width = {"fp32": 32, "bf16": 16, "fp8": 8, "nvfp4": 4}[self.precision]
        if config.row >= rows or config.col >= cols or config.bit >= width:
            raise ValueError("Input fault coordinate/bit outside actual representation")
        target = (self.a if config.location == "a" else self.b).clone()
        row, col = config.row, config.col
        if config.location == "b" and self.precision in {"fp8", "nvfp4"}:
            row, col = col, row
        if self.precision == "nvfp4":
            target[row, col // 2] ^= 1 << (config.bit + 4 * (col % 2))
        else:
            dtype = {32: torch.int32, 16: torch.int16, 8: torch.uint8}[width]
            mask = 1 << config.bit
            if width > 8 and config.bit == width - 1:
                mask = -(1 << config.bit)
            target.view(dtype)[row, col] ^= mask
        return replace(self, **{config.location: target})
