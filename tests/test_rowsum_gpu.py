"""Row checksums and two-dimensional localisation (extension).

The GEMM epilogue's row sums per 64-column block, the input-side row
prediction alpha * A . (e^T B) with its magnitude, and the locator that
takes one failing row and one failing column as the faulty element. Checked
against the C oracle (bit for bit where the arithmetic is the library's own
fixed order), against float64 where the tensor cores' accumulation is
involved, and end to end: a flipped accumulator bit is found at its exact
(row, column) and repaired by the single-element correction, including
flips too small for the two-channel ratio locator.
"""
import numpy as np
import pytest
import torch

import sdc_b200  # noqa: F401
from oracle import native
from sdc_b200 import ops
from sdc_b200.gemm.quantization import quantize, quantize_blockwise

pytestmark = pytest.mark.gpu
DEV = "cuda"
KIND = {"fp8": 0, "nvfp4": 1, "fp8_block": 2}


def _np(t):
    return t.detach().cpu().numpy()


def _case(precision, m, n, k, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    a = torch.randn(m, k, device=DEV, generator=g)
    b = torch.randn(n, k, device=DEV, generator=g)
    rows = torch.arange(1, m + 1, device=DEV, dtype=torch.float32)
    weights = torch.stack((torch.ones_like(rows), rows))
    if precision == "fp8_block":
        qa, qb = quantize_blockwise(a, 1), quantize_blockwise(b, 128)
        args = (qa.codes, qa.scales, qb.codes, qb.scales, k, None)
        oracle_in = (_np(qa.codes), _np(qa.scales), _np(qb.codes), _np(qb.scales), 1.0)
        correct = lambda loc, ok, out: ops.abft_fp8_block_correct(  # noqa: E731
            qa.codes.view(torch.float8_e4m3fn), qb.codes.view(torch.float8_e4m3fn), qa.scales, qb.scales, loc, ok,
            out)
    else:
        qa, qb = quantize(a, precision), quantize(b, precision)
        alpha = (qa.multiplier * qb.multiplier).reciprocal()
        if precision == "fp8":
            args = (qa.codes, None, qb.codes, None, k, alpha)
            oracle_in = (_np(qa.codes), None, _np(qb.codes), None, float(alpha))
            correct = lambda loc, ok, out: ops.abft_fp8_correct(  # noqa: E731
                qa.codes.view(torch.float8_e4m3fn), qb.codes.view(torch.float8_e4m3fn), alpha, loc, ok, out)
        else:
            args = (qa.codes, qa.scales_mma, qb.codes, qb.scales_mma, k, alpha)
            oracle_in = (_np(qa.codes), _np(qa.scales_mma), _np(qb.codes), _np(qb.scales_mma), float(alpha))
            correct = lambda loc, ok, out: ops.abft_nvfp4_correct(  # noqa: E731
                qa.codes, qb.codes, qa.scales_mma, qb.scales_mma, k, alpha, loc, ok, out)
    return args, weights, oracle_in, correct


def _run(precision, args, weights, fault=(-1, -1, -1)):
    a, sa, b, sb, k, alpha = args
    if precision != "nvfp4":
        a, b = a.view(torch.float8_e4m3fn), b.view(torch.float8_e4m3fn)
    return ops.abft_reference_rows_mm(KIND[precision], a, sa, b, sb, k, alpha, weights, *fault, 0, None, 1)


@pytest.mark.parametrize("precision", ["fp8", "nvfp4", "fp8_block"])
@pytest.mark.parametrize("shape", [(136, 144, 256), (300, 200, 512), (96, 80, 640), (1024, 768, 1024),
                                   (2560, 640, 2048), (136, 72, 25088)])
def test_row_prediction_bit_exact_and_observation_within_bound(precision, shape):
    m, n, k = shape
    args, weights, (a, sa, b, sb, alpha), _ = _case(precision, m, n, k, seed=m + n)
    out, obs, hit, pred, mag, row_obs, row_pred, row_mag = _run(precision, args, weights)
    torch.cuda.synchronize()
    assert hit.item() == 0 and row_obs.shape == ((n + 63) // 64, m)
    epred, emag = native.row_reference(precision, a, sa, b, sb, m, n, k, alpha)
    np.testing.assert_array_equal(_np(row_pred), epred)
    np.testing.assert_array_equal(_np(row_mag), emag)
    if precision == "fp8":
        # fp32 output: the epilogue summed exactly these values.
        np.testing.assert_array_equal(_np(row_obs), native.row_observed(_np(out)))
    # Against float64 row sums of the exact product (fp32 accumulation bound).
    rows = np.arange(0, m, max(1, m // 64))
    exact, bound = native.gemm_rows_f64(precision, a, sa, b, sb, m, n, k, rows)
    total = _np(row_obs).astype(np.float64).sum(axis=0)[rows]
    scale = abs(alpha)
    assert np.all(np.abs(total - scale * exact.sum(axis=1)) <= (k + n + 64) * 2.0 ** -24 * scale * bound.sum(axis=1)
                  + 1e-6)
    # Clean run: no row fails at a tight relative tolerance.
    packet = ops.abft_finalize_reference(obs, pred, mag, hit, torch.zeros(1, dtype=torch.int32, device=DEV), n,
                                         1e-3, 1e-5, None, True)
    location, located, row_flags, row_res, row_thr = ops.abft_locate2d(row_obs, row_pred, row_mag, 1e-3, 1e-5,
                                                                       packet[1], packet[2], packet[3])
    assert not bool(row_flags[0]) and not bool(row_flags[1]) and not bool(located)
    assert location.tolist() == [-1, -1]


@pytest.mark.parametrize("precision", ["fp8", "nvfp4", "fp8_block"])
@pytest.mark.parametrize("bit", [21, 23, 25, 27, 30])
def test_single_flip_located_in_two_dimensions_and_corrected(precision, bit):
    m, n, k = 520, 384, 512
    args, weights, _, correct = _case(precision, m, n, k, seed=7)
    clean = _run(precision, args, weights)[0].clone()
    positions = [(0, 0), (519, 383), (260, 129), (131, 7)]
    located_any = 0
    for row, col in positions:
        out, obs, hit, pred, mag, row_obs, row_pred, row_mag = _run(precision, args, weights, (row, col, bit))
        nonfinite = torch.zeros(1, dtype=torch.int32, device=DEV)
        packet = ops.abft_finalize_reference(obs, pred, mag, hit, nonfinite, n, 1e-3, 1e-5, None, True)
        location, located, row_flags, _, _ = ops.abft_locate2d(row_obs, row_pred, row_mag, 1e-3, 1e-5, packet[1],
                                                               packet[2], packet[3])
        torch.cuda.synchronize()
        assert hit.item() == 1
        if not bool(packet[3][0]):
            continue  # the flip moved the value by less than the threshold (a tiny element)
        if bool(packet[3][1]):
            assert not bool(located)  # non-finite output: never located
            continue
        assert bool(row_flags[0]), "the row sum must fail with the column"
        assert bool(located) and location.tolist() == [row, col]
        located_any += 1
        fixed = correct(location, located, out)
        torch.cuda.synchronize()
        assert bool(fixed)
        # The element is recomputed on CUDA cores (another fp32 summation
        # order than the tensor cores'); every other element is untouched.
        torch.testing.assert_close(out.float(), clean.float(), rtol=1e-2, atol=1e-3)
        diff = (out.float() != clean.float())
        assert int(diff.sum()) <= 1 and (int(diff.sum()) == 0 or bool(diff[row, col]))
    assert located_any >= 2


def test_two_failing_rows_are_not_located():
    precision, m, n, k = "fp8", 256, 256, 256
    args, weights, _, _ = _case(precision, m, n, k, seed=3)
    out, obs, hit, pred, mag, row_obs, row_pred, row_mag = _run(precision, args, weights)
    row_obs = row_obs.clone()
    row_obs[0, 5] += 1e3
    row_obs[2, 77] += 1e3
    packet = ops.abft_finalize_reference(obs, pred, mag, hit, torch.zeros(1, dtype=torch.int32, device=DEV), n,
                                         1e-3, 1e-5, None, True)
    location, located, row_flags, row_res, _ = ops.abft_locate2d(row_obs, row_pred, row_mag, 1e-3, 1e-5, packet[1],
                                                                 packet[2], packet[3])
    torch.cuda.synchronize()
    assert bool(row_flags[0]) and not bool(located) and location.tolist() == [-1, -1]
    assert abs(float(row_res[5]) - 1e3) < 1.0 and abs(float(row_res[77]) - 1e3) < 1.0


def test_row_checksum_errors():
    a = torch.zeros(128, 64, dtype=torch.uint8, device=DEV).view(torch.float8_e4m3fn)
    w = torch.ones(2, 128, device=DEV)
    alpha = torch.ones((), device=DEV)
    with pytest.raises(RuntimeError, match="kind must be"):
        ops.abft_reference_rows_mm(5, a, None, a, None, 64, alpha, w, -1, -1, -1, 0, None, 1)
    with pytest.raises(RuntimeError, match="need alpha"):
        ops.abft_reference_rows_mm(0, a, None, a, None, 64, None, w, -1, -1, -1, 0, None, 1)
    a128 = torch.zeros(128, 128, dtype=torch.uint8, device=DEV).view(torch.float8_e4m3fn)
    with pytest.raises(RuntimeError, match="K-slice layout only"):
        ops.abft_reference_rows_mm(2, a128, torch.ones(128, 1, device=DEV), a128, torch.ones(1, 1, device=DEV), 128,
                                   None, w, -1, -1, -1, 0, None, 0)


def _engine_cfg(**changes):
    return {"method": "classic", "implementation": "native", "reference_mode": "input_fused", "on_error": "report",
            "atol": 1e-3, "rtol": 1e-5, "reference_layout": "kslice", "row_checksums": True, **changes}


@pytest.mark.parametrize("precision,scaling", [("fp8", "tensorwise"), ("nvfp4", "block16"), ("fp8", "blockwise")])
@pytest.mark.parametrize("method", ["classic", "sum"])
def test_engine_row_checksums_locate_and_correct(precision, scaling, method):
    """The engine option: the clean output is the plain GEMM's, bit for bit;
    a flip is located from the row and column checksums (the one-channel Sum
    policy included, which cannot locate by itself) and repaired in place."""
    from sdc_b200.abft import execute_prepared
    from sdc_b200.abft.operands import PreparedGemm

    m, n, k = 520, 384, 512
    g = torch.Generator(device=DEV).manual_seed(21)
    a, b = torch.randn(m, k, device=DEV, generator=g), torch.randn(k, n, device=DEV, generator=g)
    prepared = PreparedGemm.prepare(a, b, precision, scaling)
    clean = prepared.raw_native()
    output, report = execute_prepared(prepared, _engine_cfg(method=method))
    assert torch.equal(output, clean) and not report.detected and not report.located
    assert report.context["location_assumption"] == "row_and_column_checksums"
    values = clean.float()
    row, col = divmod(int(((values.abs() >= 4) & (values.abs() < 256)).reshape(-1).nonzero()[37, 0]), n)
    fault = {"location": "accumulator", "row": row, "col": col, "bit": 27}
    output, report = execute_prepared(prepared, _engine_cfg(method=method, recovery="correct", diagnostics=True),
                                      fault)
    assert report.detected and report.located and report.location.tolist() == [row, col]
    assert report.recovered and report.context["recovery_action"] == "located_element_recomputed"
    assert report.row_residual.shape == (m,) and abs(float(report.row_residual[row])) > float(report.row_threshold[row])
    torch.testing.assert_close(output.float(), clean.float(), rtol=1e-2, atol=1e-3)
    output, report = execute_prepared(prepared, _engine_cfg(method=method, recovery="recompute"), fault)
    assert report.recovered and torch.equal(output, clean)
