"""Augmented BF16 ABFT (the reference's reference_mode="augmented") on sm_100a.

The checksum rows q = bf16(w^T A_t) of every 128-row M-tile are encoded by
one kernel and multiplied by B as extra M-tiles of the same tcgen05 BF16
GEMM. Checked against the C oracle and float64:

* the BF16 GEMM (``sdc_cutlass::mm``) against float64 within bf16 output
  rounding plus fp32 accumulation;
* the encoding, bit for bit against ``oracle.native.augment_encode`` (same
  fp32 fma order, one round-to-nearest-even);
* predicted partials against float64 q B (q from the oracle, exact input);
* observed and output-magnitude partials against float64 sums over the
  float64 product, within the fp32 accumulation bound;
* the clean residual against the float64 encoding residual sum_k e_k b_k,
  e = (w^T A)_f64 - q (the only error the augmented check tolerates);
* compact and separate outputs identical; tile flags; fault detection,
  non-finite outputs, recovery and error messages through the engine.
"""
import ctypes

import numpy as np
import pytest
import torch

import sdc_b200  # noqa: F401
from oracle import native as oracle
from sdc_b200 import capi, ops
from sdc_b200.abft import execute, execute_prepared
from sdc_b200.abft.operands import PreparedGemm

pytestmark = pytest.mark.gpu

U = 2.0 ** -24  # fp32 unit roundoff


def _operands(m, n, k, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    a = (torch.randn(m, k, generator=g) * scale).to(torch.bfloat16)
    b = (torch.randn(k, n, generator=g) * scale).to(torch.bfloat16)
    return a, b


def _weights(m, channels):
    rows = torch.arange(1, m + 1, dtype=torch.float32)
    w = torch.stack((torch.ones_like(rows), rows)) if channels == 2 else torch.ones(1, m)
    return w.to(torch.bfloat16)


def _bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _f64(t):
    return t.float().double().numpy()


@pytest.mark.parametrize("m,n,k", [(256, 256, 512), (300, 200, 136), (1, 8, 8), (1024, 1536, 2048),
                                   (129, 1000, 4104)])
@pytest.mark.parametrize("layout", ["rr", "cr", "rc"])
def test_bf16_mm_matches_float64(m, n, k, layout):
    a, b = _operands(m, n, k, seed=m + n + k)
    ad, bd = a.cuda(), b.cuda()
    if layout[0] == "c":
        ad = ad.T.contiguous().T
    if layout[1] == "c":
        bd = bd.T.contiguous().T
    d = ops.mm(ad, bd)
    torch.cuda.synchronize()
    ref = _f64(a) @ _f64(b)
    bound = np.abs(_f64(a)) @ np.abs(_f64(b))
    err = np.abs(d.cpu().double().numpy() - ref)
    # One bf16 rounding of the output (2^-9 relative) plus fp32 accumulation.
    assert np.all(err <= 2.0 ** -8 * np.abs(ref) + (k + 16) * U * bound + 1e-30)
    assert d.dtype == torch.bfloat16 and d.shape == (m, n) and d.is_contiguous()


@pytest.mark.parametrize("m,k,channels", [(300, 136, 2), (1024, 1024, 2), (128, 4096, 1), (77, 8, 2)])
def test_encoding_bit_exact_against_oracle(m, k, channels):
    a, _ = _operands(m, 8, k, seed=7 * m + k, scale=3.0)
    w = _weights(m, channels)
    tiles = (m + 127) // 128
    q = torch.empty(channels * tiles, k, dtype=torch.bfloat16, device="cuda")
    ad, wd = a.cuda(), w.cuda()
    algorithm = 0 if channels == 2 else 1
    capi.check(capi.lib().sdc_abft_augment_encode(ad.data_ptr(), m, k, algorithm, wd.data_ptr(), q.data_ptr(),
                                                   torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    expected = oracle.augment_encode(_bits(a), _bits(w))
    np.testing.assert_array_equal(_bits(q.cpu()), expected)


def _augmented(a, b, w, fault=(-1, -1, -1), algorithm=0):
    return ops.abft_augmented_mm(a.cuda(), b.cuda(), w.cuda(), *fault, algorithm)


@pytest.mark.parametrize("m,n,k,channels", [(256, 256, 512, 2), (300, 200, 136, 2), (1024, 640, 1024, 1),
                                            (520, 1100, 2056, 2), (1, 8, 8, 2)])
def test_partials_against_oracle_and_float64(m, n, k, channels):
    a, b = _operands(m, n, k, seed=11 * m + n)
    w = _weights(m, channels)
    d, observed, hit, predicted, magnitude = _augmented(a, b, w, algorithm=0 if channels == 2 else 1)
    torch.cuda.synchronize()
    tiles, padded = (m + 127) // 128, ((n + 127) // 128) * 128
    assert observed.shape == predicted.shape == magnitude.shape == (channels, tiles, padded)
    assert hit.item() == 0
    av, bv, wv = _f64(a), _f64(b), _f64(w)
    q = oracle.augment_encode(_bits(a), _bits(w)).view(np.int16)
    qv = torch.from_numpy(q).view(torch.bfloat16).double().numpy()
    prod = av @ bv
    prod_bound = np.abs(av) @ np.abs(bv)
    obs, pred, mag = (x.cpu().double().numpy() for x in (observed, predicted, magnitude))
    for field in (obs, pred, mag):
        assert np.all(field[:, :, n:] == 0.0)
    for t in range(tiles):
        rows = slice(t * 128, min(m, t * 128 + 128))
        for c in range(channels):
            qrow = qv[t * channels + c]
            ref_pred = qrow @ bv
            tol_pred = (k + 16) * U * (np.abs(qrow) @ np.abs(bv)) + 1e-30
            assert np.all(np.abs(pred[c, t, :n] - ref_pred) <= tol_pred)
            wr = wv[c, rows]
            ref_obs = wr @ prod[rows]
            ref_mag = np.abs(wr) @ np.abs(prod[rows])
            tol = (k + 256) * U * (np.abs(wr) @ prod_bound[rows]) + 1e-30
            assert np.all(np.abs(obs[c, t, :n] - ref_obs) <= tol)
            assert np.all(np.abs(mag[c, t, :n] - ref_mag) <= tol)
            # The clean residual is the encoding's: sum_k (w^T A - q)_k B_k.
            encoding_residual = (wr @ av[rows] - qrow) @ bv
            assert np.all(np.abs((obs[c, t, :n] - pred[c, t, :n]) - encoding_residual) <= tol + tol_pred)
    ref = prod
    assert np.all(np.abs(d.cpu().double().numpy() - ref) <= 2.0 ** -8 * np.abs(ref) + (k + 16) * U * prod_bound)


def test_compact_matches_separate_and_flags_the_fault_tile():
    m, n, k = 700, 900, 1024
    a, b = _operands(m, n, k, seed=5)
    w = _weights(m, 2)
    fault = (333, 517, 30)
    d1, observed, hit, predicted, magnitude = _augmented(a, b, w, fault)
    d2, partials, tile_flags = ops.abft_augmented_compact(a.cuda(), b.cuda(), w.cuda(), *fault, 0)
    torch.cuda.synchronize()
    assert torch.equal(d1.view(torch.int16), d2.view(torch.int16))
    assert torch.equal(partials[0], observed) and torch.equal(partials[1], predicted)
    assert torch.equal(partials[2], magnitude)
    assert hit.item() == 1
    flags = tile_flags.cpu()
    assert flags.shape == ((m + 127) // 128, (n + 127) // 128)
    expected = torch.zeros_like(flags)
    expected[333 // 128, 517 // 128] = 1
    assert torch.equal(flags, expected)


def test_nonfinite_output_flags_its_tile_and_is_detected():
    m, n, k = 256, 384, 64
    a, b = _operands(m, n, k, seed=9)
    clean = (a.float() @ b.float())
    # An element whose fp32 accumulator has exponent 127 (|v| in [1, 2)):
    # flipping bit 30 sets the exponent to all ones (inf or NaN).
    candidates = ((clean.abs() > 1.1) & (clean.abs() < 1.9)).nonzero()
    row, col = (int(x) for x in candidates[len(candidates) // 2])
    w = _weights(m, 2)
    d, partials, tile_flags = ops.abft_augmented_compact(a.cuda(), b.cuda(), w.cuda(), row, col, 30, 0)
    torch.cuda.synchronize()
    assert not torch.isfinite(d[row, col].float())
    assert tile_flags[row // 128, col // 128].item() == 3
    ref, residual, threshold, flags, hit, location = ops.abft_finalize(partials, tile_flags, n, 1e-3, 1e-2, None,
                                                                       True, 0, None)
    detected, nonfinite = flags[0].item(), flags[1].item()
    assert detected and nonfinite and hit.item() == 1


def _config(**changes):
    cfg = {"method": "classic", "reference_mode": "augmented", "threshold_scale": "output",
           "implementation": "native", "atol": 1e-3, "rtol": 1e-2, "on_error": "report", "diagnostics": True}
    cfg.update(changes)
    return cfg


@pytest.mark.parametrize("method", ["classic", "sum"])
def test_engine_clean_call_passes_and_fault_is_detected(method):
    m, n, k = 1024, 768, 1536
    a, b = _operands(m, n, k, seed=21)
    a, b = a.cuda(), b.cuda()
    out, report = execute(a, b, "bf16", "none", abft_config=_config(method=method))
    assert not bool(report.detected) and not bool(report.nonfinite) and not bool(report.located)
    assert report.execution_path == "augmented_native"
    ctx = report.context
    assert ctx["reference_algorithm"] == "augmented_gemm" and ctx["checksum_input_precision"] == "bf16"
    assert ctx["augmented_rows_per_data_tile"] == (2 if method == "classic" else 1)
    assert ctx["location_assumption"] == "disabled_for_low_precision_encoding"
    torch.testing.assert_close(out, ops.mm(a, b), rtol=0, atol=0)
    fault = {"location": "accumulator", "row": 700, "col": 5, "bit": 28}
    out2, report2 = execute(a, b, "bf16", "none", abft_config=_config(method=method), fault_config=fault)
    assert bool(report2.detected) and int(report2.fault_hit.item()) == 1 and not bool(report2.located)
    assert report2.residual.shape == (2 if method == "classic" else 1, n)


def test_engine_recompute_recovers_the_clean_output():
    m, n, k = 512, 512, 512
    a, b = _operands(m, n, k, seed=33)
    a, b = a.cuda(), b.cuda()
    fault = {"location": "accumulator", "row": 100, "col": 200, "bit": 29}
    out, report = execute(a, b, "bf16", "none", abft_config=_config(recovery="recompute"), fault_config=fault)
    assert bool(report.detected) and bool(report.recovered) and not bool(report.recheck_failed)
    assert report.context["recovery_action"] == "full_recompute"
    torch.testing.assert_close(out, ops.mm(a, b), rtol=0, atol=0)


def test_python_implementation_uses_the_separate_augmented_outputs():
    m, n, k = 384, 256, 256
    a, b = _operands(m, n, k, seed=41)
    prepared = PreparedGemm.prepare(a.cuda(), b.cuda(), "bf16", "none")
    cfg = _config(implementation="reference")
    out, report = execute_prepared(prepared, cfg)
    assert report.execution_path == "instrumented" and not bool(report.detected)
    _, native_report = execute_prepared(prepared, _config())
    # Same kernel, same evidence; only the order of the sum over M-tiles
    # differs (torch reduction vs the finalize's ascending fp32 sum).
    magnitude = (native_report.threshold - 1e-3) / 1e-2
    assert torch.all((report.residual - native_report.residual).abs() <= 1e-6 * magnitude + 1e-6)


def test_errors_are_reported_before_launch():
    a = torch.zeros(128, 12, dtype=torch.bfloat16, device="cuda")
    b = torch.zeros(12, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError, match="multiple of 8"):
        ops.mm(a, b)
    a8, b8 = torch.zeros(128, 16, dtype=torch.bfloat16, device="cuda"), torch.zeros(16, 64, dtype=torch.bfloat16,
                                                                                     device="cuda")
    with pytest.raises(RuntimeError, match="weights must be contiguous BF16"):
        ops.abft_augmented_mm(a8, b8, torch.ones(2, 128, device="cuda"), -1, -1, -1, 0)
    with pytest.raises(RuntimeError, match="fault must be all -1"):
        ops.abft_augmented_mm(a8, b8, _weights(128, 2).cuda(), 128, 0, 1, 0)
    with pytest.raises(RuntimeError, match="BF16"):
        ops.mm(a8.float(), b8.float())
    lib = capi.lib()
    rc = lib.sdc_abft_augment_encode(a8.data_ptr(), 128, 12, 0, a8.data_ptr(), a8.data_ptr(), None)
    assert rc != 0 and "multiple of 8" in capi.last_error()
    assert ctypes.c_size_t(lib.sdc_abft_augmented_workspace_bytes(7, 128, 16)).value == 0
