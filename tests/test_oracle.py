"""The CPU oracle checked against the reference's known answers and fixtures.

Every expectation here comes from the reference (meiyou666/SDC): its tests'
literal known-answer vectors (cited per test), CUTLASS's scale layout
(golden/sf_layout.json) and runs of its own CPU ABFT path
(golden/config1_trials.json, golden/engine_cases.json, see make_golden.py).
"""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import abft, cpu_path, formats, native, quant

GOLDEN = Path(__file__).parent / "golden"


# --- casts and quantisation (tests/cutlass_gemm/test_low_precision_cuda.py:24-53)

NVFP4_VALUES = np.array([
    [0., .5, 1., 1.5, 2., 3., 4., 6., -0., -.5, -1., -1.5, -2., -3., -4., -6.],
    [0., .25, .75, 1.25, 1.75, 2.5, 3.5, 5., -0., -.25, -.75, -1.25, -1.75, -2.5, -3.5, -6.],
], np.float32)
NVFP4_CODES = np.array([
    [0x10, 0x32, 0x54, 0x76, 0x98, 0xBA, 0xDC, 0xFE],
    [0x00, 0x22, 0x44, 0x66, 0x88, 0xAA, 0xCC, 0xFE],
], np.uint8)


def test_nvfp4_known_codes_midpoints_and_scale_byte():
    codes, scales, st = quant.quantize_nvfp4(NVFP4_VALUES, 1.0)
    assert np.array_equal(codes, NVFP4_CODES)
    assert np.array_equal(scales, np.full((2, 1), 0x38, np.uint8))
    assert st == 1.0
    neg, _, _ = quant.quantize_nvfp4(-NVFP4_VALUES, 1.0)
    assert np.array_equal(neg, NVFP4_CODES ^ 0x88)
    decoded = quant.dequantize_nvfp4(codes, scales, st)
    assert np.array_equal(decoded[0], NVFP4_VALUES[0])
    assert np.signbit(decoded[0, 8]) and not np.signbit(decoded[0, 0])


def test_nvfp4_zero_input_and_exact_block_scales():
    codes, scales, st = quant.quantize_nvfp4(np.zeros((4, 64), np.float32))
    assert st == 1.0 and not codes.any() and not scales.any()
    blocks = np.repeat(np.array([6., 12., 3., 0.], np.float32), 16).reshape(1, 64)
    codes, scales, st = quant.quantize_nvfp4(blocks)
    assert st == 224.0
    assert np.array_equal(scales, np.array([[0x76, 0x7E, 0x6E, 0]], np.uint8))
    assert np.array_equal(quant.dequantize_nvfp4(codes, scales, st), blocks)


def test_e4m3_cast_is_rne_and_saturating():
    # Representable values round-trip; midpoints go to the even mantissa;
    # overflow saturates to 448 (the reference's satfinite conversion) and
    # values below half the smallest subnormal flush to (signed) zero.
    grid = formats.e4m3_decode(np.arange(256, dtype=np.uint8))
    finite = np.isfinite(grid)
    assert np.array_equal(formats.e4m3_decode(formats.e4m3_encode(grid[finite])), grid[finite])
    assert formats.e4m3_encode(np.float32(1.0625)) == 0x38      # 1 + 1/16: tie -> 1.0 (even)
    assert formats.e4m3_encode(np.float32(1.1875)) == 0x3A      # 1 + 3/16: tie -> 1.25 (even)
    assert formats.e4m3_encode(np.float32(500.0)) == 0x7E       # saturates to 448
    assert formats.e4m3_encode(np.float32(-1e30)) == 0xFE
    assert formats.e4m3_encode(np.float32(2.0 ** -10)) == 0x00  # tie between 0 and 2^-9 -> 0
    assert formats.e4m3_encode(np.float32(-2.0 ** -11)) == 0x80
    assert formats.e4m3_encode(np.float32(np.nan)) == 0x7F


def test_fp8_multiplier_policy():
    x = np.array([[1., -3.5, 0.25, 2.]], np.float32)
    codes, st = quant.quantize_fp8(x)
    assert st == np.float32(448.0) / np.float32(3.5)
    assert np.array_equal(codes, formats.e4m3_encode(x * st))
    assert quant.quantize_fp8(np.zeros((1, 4), np.float32))[1] == 1.0
    assert quant.quantize_fp8(x, 2.0)[1] == 2.0


def test_fp8_reference_decode_with_multipliers():
    # tests/abft/test_framework.py:213-225: codes of 2 and 4 with multipliers
    # 2 and 4 decode to ones; Classic expected = [[96,96],[192,192]].
    a = formats.e4m3_encode(np.full((3, 32), 2., np.float32))
    b = formats.e4m3_encode(np.full((2, 32), 4., np.float32))
    da, db = quant.dequantize_fp8(a, 2.0), quant.dequantize_fp8(b, 4.0)
    expected = abft.classic_weights(3) @ (da @ db.T)
    assert np.array_equal(expected, [[96., 96.], [192., 192.]])


def test_nvfp4_two_block_reference_and_nibble_flip():
    # tests/abft/test_framework.py:42-71: packed 0x22 codes with block scales
    # (2, 4) and multiplier 2 decode to ones then twos; flipping bit 0 of
    # logical column 0 / 1 gives 0x23 / 0x32.
    packed = np.full((3, 16), 0x22, np.uint8)
    scales = formats.e4m3_encode(np.array([[2., 4.]] * 3, np.float32))
    a = quant.dequantize_nvfp4(packed, scales, 2.0)
    assert np.array_equal(a[:, :16], np.ones((3, 16))) and np.array_equal(a[:, 16:], np.full((3, 16), 2.))
    for col, expected in ((0, 0x23), (1, 0x32)):
        flipped = packed.copy()
        flipped[0, col // 2] ^= 1 << (0 + 4 * (col % 2))
        assert flipped[0, 0] == expected


# --- scale layout (CUTLASS Sm1xxBlkScaledConfig, nvfp4.cu:122-147) ----------

def test_scale_layout_matches_cutlass():
    for case in json.loads((GOLDEN / "sf_layout.json").read_text()):
        rows, k = case["rows"], case["k"]
        assert quant.sf_size(rows, k) == case["size"]
        assert quant.scale_layout(rows, k).reshape(-1).tolist() == case["offsets"]


def test_pack_scales_round_trip():
    rng = np.random.default_rng(5)
    scales = rng.integers(1, 255, (200, 9), dtype=np.uint8)
    packed = quant.pack_scales(scales, 144)
    assert packed.size == quant.sf_size(200, 144)
    assert np.array_equal(quant.unpack_scales(packed, 200, 144), scales)
    assert np.count_nonzero(packed) == np.count_nonzero(scales)


# --- finalize policy (tests/cutlass_gemm/test_abft_finalize_gpu.py) ----------

def _packet(observed, predicted, magnitude, n, **kw):
    return abft.finalize_serial(observed, predicted, magnitude, n, **kw)


def test_finalize_threshold_strict_greater_than():
    # :246-256 - |res| == thr is clean, the next float above is detected.
    for above in (False, True):
        obs = np.zeros((1, 1, 16), np.float32)
        v = np.float32(1.0)
        if above:
            v = np.nextafter(v, np.float32(np.inf))
        obs[0, 0, 15] = v
        packet = _packet(obs, np.zeros_like(obs), np.zeros_like(obs), 16, atol=1.0, rtol=0.0)
        assert bool(packet[3][0]) == above


def test_finalize_threshold_is_multiply_then_add_not_fma():
    # :279-294
    magnitude = rtol = np.float32(1 + 2 ** -23)
    atol = np.float32(2 ** -24)
    separate = np.float32(1 + 2 ** -22)
    fused = np.float32(1 + 3 * 2 ** -23)
    obs = np.zeros((1, 1, 16), np.float32)
    mag = np.zeros_like(obs)
    mag[0, 0, 15] = magnitude
    obs[0, 0, 15] = fused
    packet = _packet(obs, np.zeros_like(obs), mag, 16, atol=atol, rtol=rtol)
    assert packet[2][0, 15] == separate and packet[3][0]


def test_finalize_order_sensitive_serial_sum():
    # :464 - a column [2^24, 1, -2^24] sums to 0 serially (the 1 is lost).
    obs = np.zeros((1, 3, 4), np.float32)
    obs[0, :, 0] = [2 ** 24, 1, -(2 ** 24)]
    packet = _packet(obs, np.zeros_like(obs), np.zeros_like(obs), 4, atol=0.5, rtol=0.0)
    assert packet[1][0, 0] == 0.0 and not packet[3][0]


def test_finalize_subnormal_and_maximum_tolerances():
    obs = np.zeros((1, 1, 16), np.float32)
    mag = np.zeros_like(obs)
    mag[0, 0, 15] = 1
    obs[0, 0, 15] = 2.0 ** -149
    packet = _packet(obs, np.zeros_like(obs), mag, 16, atol=0.0, rtol=np.float32(2.0 ** -149))
    assert packet[2][0, 15] == np.float32(2.0 ** -149) and not packet[3][0]
    big = np.zeros((1, 1, 16), np.float32)
    big[0, 0, 15] = np.finfo(np.float32).max
    packet = _packet(big, np.zeros_like(big), np.zeros_like(big), 16, atol=np.finfo(np.float32).max, rtol=0.0)
    assert not packet[3][0] and not packet[3][1]


# --- locator (tests/abft/test_framework.py:88-94, 136-144) -------------------

def test_accumulator_detection_and_location():
    a, b = torch.ones(3, 16), torch.ones(16, 2)
    _, report, _ = cpu_path.execute(a, b, fault=(1, 0, 31))
    assert report["detected"] and report["located"] and report["location"] == [1, 0]
    assert report["fault_hit"] == 1


def test_ambiguous_numeric_location_rejected():
    m = 3
    weights = abft.classic_weights(m)
    expected = weights @ np.full((3, 2), 16., np.float32)
    observed = expected.copy()
    observed[:, 0] += [1., 2.]
    residual = (observed - expected).astype(np.float32)
    threshold = np.full((2, 2), 0.4, np.float32)
    located, loc = abft.locate(residual, threshold, True, False, m)
    assert not located and loc == (-1, -1)


def test_numpy_locator_matches_torch_locator():
    rng = np.random.default_rng(11)
    for trial in range(200):
        m, n = 300, 40
        residual = np.zeros((2, n), np.float32)
        col = int(rng.integers(0, n))
        row = int(rng.integers(0, m))
        delta = np.float32(rng.choice([-1, 1]) * 10 ** rng.uniform(-3, 3))
        residual[0, col] = delta
        residual[1, col] = np.float32((row + 1) * delta) * np.float32(1 + rng.normal() * 1e-6)
        threshold = np.abs(rng.normal(size=(2, n))).astype(np.float32) * np.float32(10 ** rng.uniform(-6, -1))
        failed = np.abs(residual) > threshold
        detected = bool(failed.any())
        located, loc = abft.locate(residual, threshold, detected, False, m)
        ref = cpu_path.verify(torch.tensor(residual), torch.zeros(1), torch.zeros(2, n),
                              torch.zeros(2, n), 0.0, 0.0, m, locate=True)
        # Re-run the torch locator on the same residual/threshold tensors.
        res_t, thr_t = torch.tensor(residual), torch.tensor(threshold)
        columns = (res_t.abs() > thr_t).any(dim=0)
        c = columns.to(torch.int64).argmax()
        d0, d1 = res_t[:, c].unbind()
        ratio = d1 / torch.where(d0 == 0, torch.ones_like(d0), d0)
        r = ratio.round().to(torch.int64) - 1
        ok = detected and int(columns.sum()) == 1 and bool(d0.abs() > thr_t[0, c])
        ok = ok and 0 <= int(r) < m and bool((d1 - (r + 1).float() * d0).abs() <= thr_t[1, c] + (r + 1).abs().float() * thr_t[0, c])
        unc = (thr_t[1, c] + ratio.abs() * thr_t[0, c]) / (d0.abs() - thr_t[0, c]).clamp_min(torch.finfo(torch.float32).tiny)
        ok = ok and bool((ratio - (r + 1)).abs() + unc < 0.5)
        assert located == ok, (trial, located, ok)
        if ok:
            assert loc == (int(r), int(c))
        del ref


# --- the reference's CPU path (fixtures from make_golden.py) -----------------

def test_cpu_path_reproduces_reference_config1_trials():
    data = json.loads((GOLDEN / "config1_trials.json").read_text())
    g = torch.Generator().manual_seed(data["seed"])
    m, n, k = data["shape"]
    a = torch.rand(m, k, generator=g) * 2 - 1
    b = torch.rand(k, n, generator=g) * 2 - 1
    state = None
    for trial in data["trials"]:
        f = trial["fault"]
        fault = (f["row"], f["col"], f["bit"]) if f else (-1, -1, -1)
        _, report, state = cpu_path.execute(a, b, atol=data["atol"], rtol=data["rtol"], fault=fault, state=state)
        assert report["detected"] == trial["detected"]
        assert report["located"] == trial["located"]
        assert report["location"] == trial["location"]
    clean = data["trials"][:50]
    assert not any(t["detected"] for t in clean)  # zero false positives


def test_cpu_path_reproduces_reference_engine_cases():
    for case in json.loads((GOLDEN / "engine_cases.json").read_text()):
        g = torch.Generator().manual_seed(case["seed"])
        a = torch.randn(64, 80, generator=g)
        b = torch.randn(80, 96, generator=g)
        f = case["fault"]
        fault = (f["row"], f["col"], f["bit"]) if f else (-1, -1, -1)
        _, report, _ = cpu_path.execute(a, b, atol=1e-4, rtol=1e-4, fault=fault, block_k=32, recovery="recompute")
        assert (report["detected"], report["located"], report["location"], report["recovered"]) == (
            case["detected"], case["located"], case["location"], case["recovered"])


# --- C oracle of the input-fused checksum ------------------------------------

@pytest.mark.parametrize("kind", ["fp8", "nvfp4"])
def test_c_oracle_tile_reference_matches_float64(kind):
    rng = np.random.default_rng(7)
    m, n, k = 200, 72, 96
    if kind == "fp8":
        a = formats.e4m3_encode(rng.normal(size=(m, k)).astype(np.float32) * 8)
        b = formats.e4m3_encode(rng.normal(size=(n, k)).astype(np.float32) * 8)
        sfa = sfb = None
        da, db = formats.e4m3_decode(a), formats.e4m3_decode(b)
    else:
        a, sa, _ = quant.quantize_nvfp4(rng.normal(size=(m, k)).astype(np.float32))
        b, sb, _ = quant.quantize_nvfp4(rng.normal(size=(n, k)).astype(np.float32))
        sfa, sfb = quant.pack_scales(sa, k), quant.pack_scales(sb, k)
        da, db = quant.dequantize_nvfp4(a, sa, 1.0), quant.dequantize_nvfp4(b, sb, 1.0)
    w = rng.normal(size=(2, m)).astype(np.float32)
    pn = 128
    pred, mag = native.input_reference(kind, a, sfa, b, sfb, m, n, k, w, 0.5, pn, "tile")
    for t in range(2):
        rows = slice(128 * t, min(m, 128 * t + 128))
        exact = (w[:, rows].astype(np.float64) @ da[rows].astype(np.float64)) @ db.T.astype(np.float64) * 0.5
        exact_mag = (np.abs(w[:, rows]).astype(np.float64) @ np.abs(da[rows]).astype(np.float64)) @ np.abs(db.T).astype(np.float64) * 0.5
        assert np.all(np.abs(pred[:, t, :n] - exact) <= 1e-5 * exact_mag + 1e-6)
        assert np.allclose(mag[:, t, :n], exact_mag, rtol=1e-5)
    assert not pred[:, :, n:].any() and not mag[:, :, n:].any()
    kpred, kmag = native.input_reference(kind, a, sfa, b, sfb, m, n, k, w, 0.5, pn, "kslice")
    assert np.allclose(kpred.sum(axis=1), pred.sum(axis=1), rtol=1e-5, atol=1e-4 * mag.sum(axis=1).max())
    assert np.allclose(kmag.sum(axis=1), mag.sum(axis=1), rtol=1e-5)


# --- block-scaled FP8 (1 x 128 activations, 128 x 128 weights) -----------------

def test_fp8_block_quantizer_known_answers():
    x = np.zeros((3, 256), np.float32)
    x[0, :128] = np.linspace(-1, 1, 128, dtype=np.float32) * 896  # amax 896 -> d = 2
    x[1, 130] = -3.0  # block (1, 1): d = 3 / 448
    codes, scales = quant.quantize_fp8_block(x, 1)
    assert scales.shape == (3, 2) and scales.dtype == np.float32
    assert scales[0, 0] == 2.0 and scales[1, 1] == np.float32(3.0) / np.float32(448.0)
    assert scales[0, 1] == scales[2, 0] == scales[2, 1] == 1.0  # all-zero blocks keep d = 1
    assert codes[0, 0] == 0xFE and codes[0, 127] == 0x7E  # -/+448
    assert codes[1, 130] == 0xFE and not codes[2].any()
    dq = quant.dequantize_fp8_block(codes, scales, 1)
    assert np.all(np.abs(dq - x) <= np.abs(x) * 2.0 ** -4 + 1e-30)


def test_fp8_block_quantizer_weight_blocks_and_ragged_rows():
    rng = np.random.default_rng(3)
    x = rng.normal(size=(200, 384)).astype(np.float32)
    codes, scales = quant.quantize_fp8_block(x, 128)
    assert scales.shape == (2, 3)
    for rb in range(2):
        for kb in range(3):
            block = x[128 * rb:128 * rb + 128, 128 * kb:128 * kb + 128]
            assert scales[rb, kb] == np.float32(np.abs(block).max()) / np.float32(448.0)
            d = scales[rb, kb]
            assert np.array_equal(codes[128 * rb:128 * rb + 128, 128 * kb:128 * kb + 128],
                                  formats.e4m3_encode(block / d))
    # Every block's largest magnitude maps onto the top code 448 exactly.
    assert (formats.e4m3_decode(codes) == 448).sum() + (formats.e4m3_decode(codes) == -448).sum() >= 6
    with pytest.raises(ValueError):
        quant.quantize_fp8_block(x[:, :100], 1)


def test_c_oracle_block_scaled_matches_float64():
    rng = np.random.default_rng(11)
    m, n, k = 200, 160, 256
    a, sa = quant.quantize_fp8_block(rng.normal(size=(m, k)).astype(np.float32), 1)
    b, sb = quant.quantize_fp8_block(rng.normal(size=(n, k)).astype(np.float32), 128)
    da, db = quant.dequantize_fp8_block(a, sa, 1), quant.dequantize_fp8_block(b, sb, 128)
    out = native.gemm_f64("fp8_block", a, sa, b, sb, m, n, k)
    assert np.allclose(out, da.astype(np.float64) @ db.T.astype(np.float64), rtol=1e-12, atol=1e-12)
    w = rng.normal(size=(2, m)).astype(np.float32)
    pred, mag = native.input_reference("fp8_block", a, sa, b, sb, m, n, k, w, 1.0, 256, "kslice")
    exact = w.astype(np.float64) @ out
    exact_mag = (np.abs(w).astype(np.float64) @ np.abs(da).astype(np.float64)) @ np.abs(db.T).astype(np.float64)
    assert np.all(np.abs(pred.sum(axis=1)[:, :n] - exact) <= 1e-5 * exact_mag + 1e-6)
    assert np.allclose(mag.sum(axis=1)[:, :n], exact_mag, rtol=1e-5)
    assert not pred[:, :, n:].any()


# --- row checksums (extension) ----------------------------------------------

@pytest.mark.parametrize("kind", ["fp8", "nvfp4", "fp8_block"])
def test_c_oracle_row_checksums_match_float64(kind):
    rng = np.random.default_rng(13)
    m, n, k = 150, 200, 256
    if kind == "fp8":
        a = formats.e4m3_encode(rng.normal(size=(m, k)).astype(np.float32) * 8)
        b = formats.e4m3_encode(rng.normal(size=(n, k)).astype(np.float32) * 8)
        sfa = sfb = None
        da, db = formats.e4m3_decode(a), formats.e4m3_decode(b)
    elif kind == "nvfp4":
        a, sa, _ = quant.quantize_nvfp4(rng.normal(size=(m, k)).astype(np.float32))
        b, sb, _ = quant.quantize_nvfp4(rng.normal(size=(n, k)).astype(np.float32))
        sfa, sfb = quant.pack_scales(sa, k), quant.pack_scales(sb, k)
        da, db = quant.dequantize_nvfp4(a, sa, 1.0), quant.dequantize_nvfp4(b, sb, 1.0)
    else:
        a, sfa = quant.quantize_fp8_block(rng.normal(size=(m, k)).astype(np.float32), 1)
        b, sfb = quant.quantize_fp8_block(rng.normal(size=(n, k)).astype(np.float32), 128)
        da, db = quant.dequantize_fp8_block(a, sfa, 1), quant.dequantize_fp8_block(b, sfb, 128)
    alpha = 1.0 if kind == "fp8_block" else 0.25
    pred, mag = native.row_reference(kind, a, sfa, b, sfb, m, n, k, alpha)
    exact = da.astype(np.float64) @ db.astype(np.float64).sum(axis=0) * alpha
    exact_mag = np.abs(da).astype(np.float64) @ np.abs(db).astype(np.float64).sum(axis=0) * alpha
    assert np.all(np.abs(pred - exact) <= 1e-5 * exact_mag + 1e-6)
    assert np.allclose(mag, exact_mag, rtol=1e-5)
    # Observed row sums: per 64-column block, the columns added in ascending order from +0.
    values = rng.normal(size=(m, n)).astype(np.float32)
    blocks = native.row_observed(values)
    assert blocks.shape == (4, m)
    for j in range(4):
        acc = np.zeros(m, np.float32)
        for c in range(64 * j, min(n, 64 * j + 64)):
            acc = acc + values[:, c]
        assert np.array_equal(blocks[j], acc)
