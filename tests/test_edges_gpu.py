"""Ragged and minimal shapes on every kind: M, N around the 128-row tile and
the 256-row CTA pair, the smallest K each format allows. The protected output
equals the unprotected one bit for bit, the K-slice partials equal the C
oracle bit for bit, the output is within the fp32 accumulation bound of the
float64 product, and no clean run raises a flag."""
import numpy as np
import pytest
import torch

import sdc_b200  # noqa: F401  (registers torch.ops.sdc_cutlass)
from oracle import native
from sdc_b200.gemm.quantization import quantize, quantize_blockwise

pytestmark = pytest.mark.gpu
ops = torch.ops.sdc_cutlass
DEV = "cuda"

SHAPES = [(1, 8), (127, 1), (129, 129), (255, 300), (257, 64), (385, 257)]
MIN_K = {"fp8": 16, "nvfp4": 32, "fp8_block": 128}


def _np(t):
    return t.detach().cpu().numpy()


def _case(kind, m, n, k, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    a = torch.randn(m, k, device=DEV, generator=g)
    b = torch.randn(n, k, device=DEV, generator=g)
    if kind == "fp8_block":
        qa, qb = quantize_blockwise(a, 1), quantize_blockwise(b, 128)
        args = (qa.codes.view(torch.float8_e4m3fn), qb.codes.view(torch.float8_e4m3fn), qa.scales, qb.scales)
        oracle_in = (_np(qa.codes), _np(qa.scales), _np(qb.codes), _np(qb.scales))
        return args, oracle_in, 1.0, (ops.fp8_block_mm, ops.abft_fp8_block_reference_mm, ())
    qa, qb = quantize(a, kind), quantize(b, kind)
    alpha = (qa.multiplier * qb.multiplier).reciprocal()
    if kind == "fp8":
        args = (qa.codes.view(torch.float8_e4m3fn), qb.codes.view(torch.float8_e4m3fn), alpha)
        oracle_in = (_np(qa.codes), None, _np(qb.codes), None)
        return args, oracle_in, float(_np(alpha)), (ops.fp8_mm, ops.abft_fp8_reference_mm, (1,))
    args = (qa.codes, qb.codes, qa.scales_mma, qb.scales_mma, k, alpha)
    oracle_in = (_np(qa.codes), _np(qa.scales_mma), _np(qb.codes), _np(qb.scales_mma))
    return args, oracle_in, float(_np(alpha)), (ops.nvfp4_mm, ops.abft_nvfp4_reference_mm, (1,))


@pytest.mark.parametrize("kind", ["fp8", "nvfp4", "fp8_block"])
@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("k_blocks", [1, 3])
def test_ragged_shapes_all_kinds(kind, shape, k_blocks):
    m, n = shape
    k = MIN_K[kind] * k_blocks
    args, (oa, osa, ob, osb), alpha, (plain, reference, layout) = _case(kind, m, n, k, seed=m * 7 + n + k)
    rows = torch.arange(m, device=DEV, dtype=torch.float32)
    weights = torch.stack((torch.ones(m, device=DEV), rows + 1))
    nonfinite = torch.zeros(1, dtype=torch.int32, device=DEV)
    base = plain(*args)
    out, obs, hit, pred, mag = reference(*args, weights, -1, -1, -1, 0, nonfinite, *layout)
    assert torch.equal(out, base)
    assert hit.item() == 0 and nonfinite.item() == 0
    epred, emag = native.input_reference(kind, oa, osa, ob, osb, m, n, k, _np(weights), alpha, pred.shape[-1],
                                         "kslice")
    assert np.array_equal(_np(pred), epred) and np.array_equal(_np(mag), emag)
    exact = native.gemm_f64(kind, oa, osa, ob, osb, m, n, k) * alpha
    bound = native.gemm_f64(kind, *_abs(kind, oa, osa, ob, osb), m, n, k) * abs(alpha)
    got = _np(out.float()).astype(np.float64)
    bf16 = out.dtype == torch.bfloat16
    limit = 2 * k * 2.0 ** -24 * bound + (2.0 ** -8 * np.abs(exact) if bf16 else 0) + 1e-6
    assert np.all(np.abs(got - exact) <= limit)
    packet = ops.abft_finalize_reference(obs, pred, mag, hit, nonfinite, n, 1e-3, 1e-4, None, False)
    assert not packet[3][0].item(), "clean run flagged"


def _abs(kind, a, sa, b, sb):
    if kind == "nvfp4":
        return a & 0x77, sa, b & 0x77, sb
    return a & 0x7F, sa, b & 0x7F, sb
