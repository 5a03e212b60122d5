"""Seeded bit-flip campaign: the GPU's detection decision equals the oracle's.

For every flip (uniform row and column, bit uniform in 20-30, seeded) the
protected GEMM runs on the GPU with the fault injected in the epilogue, then
finalize and the device locator. The oracle recomputes the decision from its
own partials:
* tensorwise FP8 (fp32 output): the observed checksums are recomputed from
  the stored output in the epilogue's exact reduction order
  (``native.observed_epilogue``) and must equal the GPU's bit for bit; the
  predicted/magnitude partials come from ``cref.c``;
* NVFP4 and block-scaled FP8 (bf16 output, so the fp32 values are not
  stored): the GPU's observed partials with the oracle's predicted/magnitude.
``oracle.abft.finalize_serial`` and ``oracle.abft.locate`` then give the
reference packet and location, which must equal the GPU's bit for bit, at the
reference's thresholds and at a tight one. Whenever the oracle locates the
fault, the single-element correction runs and must restore the clean value.
"""
import numpy as np
import pytest
import torch

import sdc_b200  # noqa: F401  (registers torch.ops.sdc_cutlass)
from oracle import abft as oabft
from oracle import native
from sdc_b200.gemm.quantization import quantize, quantize_blockwise

pytestmark = pytest.mark.gpu
ops = torch.ops.sdc_cutlass
DEV = "cuda"
THRESHOLDS = ((1e-3, 1e-4), (0.0, 1e-6))


def _np(t):
    return t.detach().cpu().numpy()


def _setup(kind, m, n, k, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    a = torch.randn(m, k, device=DEV, generator=g, dtype=torch.bfloat16)
    b = torch.randn(n, k, device=DEV, generator=g, dtype=torch.bfloat16)
    if kind == "fp8_block":
        qa, qb = quantize_blockwise(a, 1), quantize_blockwise(b, 128)
        args = (qa.codes.view(torch.float8_e4m3fn), qb.codes.view(torch.float8_e4m3fn), qa.scales, qb.scales)
        oracle_in = (_np(qa.codes), _np(qa.scales), _np(qb.codes), _np(qb.scales))
        return args, oracle_in, np.float32(1.0), ops.abft_fp8_block_reference_mm, (), ops.abft_fp8_block_correct
    qa, qb = quantize(a, kind), quantize(b, kind)
    alpha = (qa.multiplier * qb.multiplier).reciprocal()
    if kind == "fp8":
        args = (qa.codes.view(torch.float8_e4m3fn), qb.codes.view(torch.float8_e4m3fn), alpha)
        oracle_in = (_np(qa.codes), None, _np(qb.codes), None)
        return args, oracle_in, np.float32(_np(alpha)), ops.abft_fp8_reference_mm, (1,), ops.abft_fp8_correct
    args = (qa.codes, qb.codes, qa.scales_mma, qb.scales_mma, k, alpha)
    oracle_in = (_np(qa.codes), _np(qa.scales_mma), _np(qb.codes), _np(qb.scales_mma))
    return args, oracle_in, np.float32(_np(alpha)), ops.abft_nvfp4_reference_mm, (1,), ops.abft_nvfp4_correct


def _packet_equal(gpu, expected):
    ref, res, thr, flags, hit, loc = expected
    assert np.array_equal(_np(gpu[0]).view(np.uint32), ref.view(np.uint32))
    assert np.array_equal(_np(gpu[1]).view(np.uint32), res.view(np.uint32))
    assert np.array_equal(_np(gpu[2]).view(np.uint32), thr.view(np.uint32))
    assert _np(gpu[3]).tolist() == flags.tolist()
    assert int(gpu[4].item()) == int(hit[0])


@pytest.mark.parametrize("kind,shape,flips", [("fp8", (1024, 768, 1024), 64), ("fp8", (2304, 1280, 2048), 64),
                                              ("nvfp4", (1024, 1024, 1024), 32),
                                              ("fp8_block", (1280, 1024, 1024), 32)])
def test_seeded_flips_decided_like_the_oracle(kind, shape, flips):
    m, n, k = shape
    args, (a, sfa, b, sfb), alpha, fused, layout, correct = _setup(kind, m, n, k, seed=sum(shape))
    weights = torch.stack((torch.ones(m, device=DEV), torch.arange(1, m + 1, device=DEV, dtype=torch.float32)))
    w = _np(weights)
    nonfinite = torch.zeros(1, dtype=torch.int32, device=DEV)
    clean, obs, hit, pred, mag = fused(*args, weights, -1, -1, -1, 0, nonfinite, *layout)
    padded = pred.shape[-1]
    epred, emag = native.input_reference(kind, a, sfa, b, sfb, m, n, k, w, alpha, padded, "kslice")
    assert np.array_equal(_np(pred), epred) and np.array_equal(_np(mag), emag)
    clean_np = _np(clean.float())
    rng = np.random.default_rng(sum(shape) + flips)
    located_count = detected_count = 0
    for _ in range(flips):
        row, col, bit = int(rng.integers(0, m)), int(rng.integers(0, n)), int(rng.integers(20, 31))
        out, obs, hit, pred, mag = fused(*args, weights, row, col, bit, 0, nonfinite, *layout)
        assert hit.item() == 1
        out_np = _np(out.float())
        if kind == "fp8":
            # The stored fp32 output is exactly what the epilogue summed.
            eobs = native.observed_epilogue(out_np, w, padded)
            assert np.array_equal(_np(obs).view(np.uint32), eobs.view(np.uint32))
        else:
            eobs = _np(obs)
        with np.errstate(invalid="ignore", over="ignore"):
            stored_nonfinite = not np.isfinite(out_np).all()
        assert nonfinite.item() == int(stored_nonfinite)
        for atol, rtol in THRESHOLDS:
            packet = ops.abft_finalize_reference(obs, pred, mag, hit, nonfinite, n, atol, rtol, None, True)
            expected = oabft.finalize_serial(eobs, epred, emag, n, atol=np.float32(atol), rtol=np.float32(rtol),
                                             hit=1, nonfinite=stored_nonfinite)
            _packet_equal(packet, expected)
            location, located = ops.abft_locate(packet[1], packet[2], packet[3], m)
            ok, loc = oabft.locate(expected[1], expected[2], bool(expected[3][0]), bool(expected[3][1]), m)
            assert bool(located.item()) == ok and location.tolist() == list(loc)
            detected_count += bool(expected[3][0])
            if not ok:
                continue
            located_count += 1
            assert loc == (row, col)
            fixed = out.clone()
            corrected = correct(*args, location, located, fixed)
            assert corrected.item()
            fixed_np = _np(fixed.float())
            # Only the located element changes, and it returns to the clean
            # value up to the fp32 accumulation order (and the bf16 cast).
            mask = np.ones((m, n), bool)
            mask[row, col] = False
            assert np.array_equal(fixed_np[mask], out_np[mask])
            _, bound = native.gemm_rows_f64(kind, a, sfa, b, sfb, m, n, k, [row])
            tol = 4 * k * 2.0 ** -24 * float(bound[0, col]) * abs(float(alpha)) + 1e-6
            if kind != "fp8":
                tol += 2.0 ** -7 * abs(float(clean_np[row, col]))
            assert abs(float(fixed_np[row, col]) - float(clean_np[row, col])) <= tol
    # The campaign exercises every branch: detections, locations and misses.
    assert detected_count > 0 and located_count > 0
