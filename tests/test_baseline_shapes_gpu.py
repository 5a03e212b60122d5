"""Parity at the benchmark configurations' own shapes.

Every shape the benchmark times is checked here against the CPU oracle:
block-scaled FP8 8192^3 (configuration 1, the headline), tensorwise FP8
8192^3 (the reference's FP8 semantics), NVFP4 16384^3 (configuration 2), and
two Qwen2.5-7B layer shapes of configuration 3 (down: K = 18944; gate + up
fused: N = 37888), all with M = 16384 tokens where the configuration says so.
At these sizes the persistent kernel walks many tiles per CTA and the K-slice
layout gives each tile several slices, which the small-shape tests do not.

Bars (the same as at small shapes):
* quantised codes and scales bit-exact against the oracle quantiser, on
  sampled rows, with the global multiplier recomputed from the full tensor;
* K-slice predicted / magnitude partials bit-exact against ``cref.c`` (all
  slots), TILE-layout partials bit-exact on sampled tiles (the reference's
  own layout, tensorwise FP8 and NVFP4);
* output rows (a sampled set plus one whole M-tile) within the fp32
  accumulation bound of the float64 product of the decoded operands (plus
  the bf16 half-ulp where the output is bf16);
* the observed checksum of the whole tile within the same bound summed over
  its rows;
* the clean run is not flagged at the reference's thresholds, and its
  residual stays far below them (the measured ratio is printed).
"""
import numpy as np
import pytest
import torch

import sdc_b200  # noqa: F401  (registers torch.ops.sdc_cutlass)
from oracle import native, quant
from sdc_b200.gemm.quantization import quantize, quantize_blockwise

pytestmark = pytest.mark.gpu
ops = torch.ops.sdc_cutlass
DEV = "cuda"

CASES = [
    pytest.param("fp8_block", (8192, 8192, 8192), 1.0, id="config1-fp8-block-8192"),
    pytest.param("fp8", (8192, 8192, 8192), 1.0, id="fp8-tensorwise-8192"),
    pytest.param("nvfp4", (16384, 16384, 16384), 1.0, id="config2-nvfp4-16384"),
    pytest.param("fp8_block", (16384, 3584, 18944), 0.02, id="qwen-down-K18944-fp8-block"),
    pytest.param("nvfp4", (16384, 37888, 3584), 0.02, id="qwen-gate-up-N37888-nvfp4"),
]


def _np(t):
    return t.detach().cpu().numpy()


def _sample_rows(m, seed):
    rng = np.random.default_rng(seed)
    fixed = [0, 1, 127, 128, 255, m // 2, m - 129, m - 1]
    return np.unique(np.concatenate([fixed, rng.integers(0, m, 40)]))


def _operands(kind, m, n, k, b_std, seed):
    """Seeded bf16 N(0,1) activations [m, k] and N(0, b_std) weights [n, k],
    quantised on the device; returns (op args, oracle inputs, alpha, raw bf16)."""
    g = torch.Generator(device=DEV).manual_seed(seed)
    a = torch.randn(m, k, device=DEV, generator=g, dtype=torch.bfloat16)
    b = (torch.randn(n, k, device=DEV, generator=g, dtype=torch.bfloat16) * b_std).to(torch.bfloat16)
    if kind == "fp8_block":
        qa, qb = quantize_blockwise(a, 1), quantize_blockwise(b, 128)
        args = (qa.codes.view(torch.float8_e4m3fn), qb.codes.view(torch.float8_e4m3fn), qa.scales, qb.scales)
        oracle_in = (_np(qa.codes), _np(qa.scales), _np(qb.codes), _np(qb.scales))
        alpha = np.float32(1.0)
    else:
        qa, qb = quantize(a, kind), quantize(b, kind)
        alpha_t = (qa.multiplier * qb.multiplier).reciprocal()
        alpha = np.float32(_np(alpha_t))
        if kind == "fp8":
            args = (qa.codes.view(torch.float8_e4m3fn), qb.codes.view(torch.float8_e4m3fn), alpha_t)
            oracle_in = (_np(qa.codes), None, _np(qb.codes), None)
        else:
            args = (qa.codes, qb.codes, qa.scales_mma, qb.scales_mma, k, alpha_t)
            oracle_in = (_np(qa.codes), _np(qa.scales_mma), _np(qb.codes), _np(qb.scales_mma))
    return args, oracle_in, alpha, (a, b), (qa, qb)


def _check_quantised_rows(kind, raw, quantised, oracle_in, k, seed):
    """Codes and scales of sampled rows (whole 128-row groups for the 128 x 128
    weight blocks) against the oracle quantiser, with the tensorwise
    multiplier recomputed from the whole tensor."""
    for x, q, codes, scales, operand in ((raw[0], quantised[0], oracle_in[0], oracle_in[1], "a"),
                                         (raw[1], quantised[1], oracle_in[2], oracle_in[3], "b")):
        rows = x.shape[0]
        if kind == "fp8_block" and operand == "b":
            groups = np.unique(np.concatenate([[0, rows // 128 // 2, (rows - 1) // 128],
                                               np.random.default_rng(seed).integers(0, (rows + 127) // 128, 3)]))
            sample = np.concatenate([np.arange(g * 128, min(rows, g * 128 + 128)) for g in groups])
        else:
            sample = _sample_rows(rows, seed)
        values = _np(x[torch.from_numpy(sample).to(DEV)].float())
        if kind == "fp8_block":
            block_rows = 1 if operand == "a" else 128
            ecodes, escales = quant.quantize_fp8_block(values, block_rows)
            assert np.array_equal(codes[sample], ecodes)
            assert np.array_equal(scales[np.unique(sample // block_rows)], escales)
            continue
        amax = np.float32(_np(x.abs().max().float()))
        limit = np.float32(448.0 if kind == "fp8" else 6.0 * 448.0)
        st = np.float32(1.0) if amax == 0 else np.float32(limit / amax)
        assert _np(q.multiplier) == st
        if kind == "fp8":
            ecodes, _ = quant.quantize_fp8(values, float(st))
            assert np.array_equal(codes[sample], ecodes)
        else:
            ecodes, escales, _ = quant.quantize_nvfp4(values, float(st))
            assert np.array_equal(codes[sample], ecodes)
            assert np.array_equal(quant.unpack_scales(scales, rows, k)[sample], escales)


@pytest.mark.parametrize("kind,shape,b_std", CASES)
def test_parity_at_benchmark_shape(kind, shape, b_std):
    m, n, k = shape
    seed = m + n + k
    args, oracle_in, alpha, raw, quantised = _operands(kind, m, n, k, b_std, seed)
    _check_quantised_rows(kind, raw, quantised, oracle_in, k, seed)
    del raw, quantised
    weights = torch.stack((torch.ones(m, device=DEV), torch.arange(1, m + 1, device=DEV, dtype=torch.float32)))
    nonfinite = torch.zeros(1, dtype=torch.int32, device=DEV)
    if kind == "fp8_block":
        out, obs, hit, pred, mag = ops.abft_fp8_block_reference_mm(*args, weights, -1, -1, -1, 0, nonfinite)
    elif kind == "fp8":
        out, obs, hit, pred, mag = ops.abft_fp8_reference_mm(*args, weights, -1, -1, -1, 0, nonfinite, 1)
    else:
        out, obs, hit, pred, mag = ops.abft_nvfp4_reference_mm(*args, weights, -1, -1, -1, 0, nonfinite, 1)
    packet = ops.abft_finalize_reference(obs, pred, mag, hit, nonfinite, n, 1e-3, 1e-4, None, True)
    torch.cuda.synchronize()
    padded = pred.shape[-1]
    a, sfa, b, sfb = oracle_in
    w = _np(weights)

    # K-slice partials, every slot, bit for bit.
    epred, emag = native.input_reference(kind, a, sfa, b, sfb, m, n, k, w, alpha, padded, "kslice")
    assert np.array_equal(_np(pred), epred)
    assert np.array_equal(_np(mag), emag)
    del epred, emag

    # Sampled output rows and one whole M-tile against float64.
    tile = (m // 128) // 2
    rows = np.unique(np.concatenate([_sample_rows(m, seed), np.arange(128 * tile, 128 * tile + 128)]))
    exact, bound = native.gemm_rows_f64(kind, a, sfa, b, sfb, m, n, k, rows)
    exact *= float(alpha)
    bound *= abs(float(alpha))
    got = _np(out[torch.from_numpy(rows).to(DEV)].float()).astype(np.float64)
    accumulation = 2 * k * 2.0 ** -24 * bound
    cast = 2.0 ** -8 * np.abs(exact) if kind != "fp8" else 0.0
    assert np.all(np.abs(got - exact) <= accumulation + cast + 1e-6)

    # Observed checksum of that tile: sum over its rows of w * value (fp32
    # values before the output cast), within the summed accumulation bound.
    in_tile = (rows >= 128 * tile) & (rows < 128 * tile + 128)
    wt = w[:, rows[in_tile]].astype(np.float64)
    expected_obs = wt @ exact[in_tile]
    obs_tol = np.abs(wt) @ accumulation[in_tile] + 2.0 ** -20 * (np.abs(wt) @ np.abs(exact[in_tile])) + 1e-3
    assert np.all(np.abs(_np(obs[:, tile, :n]).astype(np.float64) - expected_obs) <= obs_tol)

    # Clean run: not flagged, and the residual is far below the threshold.
    flags = _np(packet[3])
    assert not flags[0] and not flags[1] and hit.item() == 0
    residual, threshold = _np(packet[1]).astype(np.float64), _np(packet[2]).astype(np.float64)
    ratio = np.abs(residual) / np.maximum(_np(packet[0][1]).astype(np.float64), 1e-30)
    print(f"{kind} {shape}: clean max |res|/thr = {np.max(np.abs(residual) / threshold):.3e}, "
          f"max |res|/mag = {ratio.max():.3e}")
    assert np.max(np.abs(residual) / threshold) < 1e-2

    # The reference's own layout (TILE) on sampled tiles: the same output and
    # observation, per-tile partials bit for bit.
    if kind != "fp8_block":
        tiles = np.unique([0, tile, (m + 127) // 128 - 1])
        fused = ops.abft_fp8_reference_mm if kind == "fp8" else ops.abft_nvfp4_reference_mm
        out0, obs0, hit0, pred0, mag0 = fused(*args, weights, -1, -1, -1, 0, None, 0)
        assert torch.equal(out0, out) and torch.equal(obs0, obs) and hit0.item() == 0
        sel = torch.from_numpy(tiles).to(DEV)
        tpred, tmag = native.tile_reference_subset(kind, a, sfa, b, sfb, m, n, k, w, alpha, padded, tiles)
        assert np.array_equal(_np(pred0[:, sel]), tpred)
        assert np.array_equal(_np(mag0[:, sel]), tmag)
