"""ABFT epilogue, finalize and localisation, restated. Test infrastructure only.

* ``epilogue``        — src/cutlass_gemm/csrc/abft/common/sm120_epilogue.cuh:52-151:
  v = alpha * acc (fp32), optional XOR of one bit at (row, col), observed
  column projection sum_rows w_c[row] * v per 128-row tile, then the cast.
* ``finalize_serial`` — src/cutlass_gemm/csrc/abft/common/finalize.cu:90-135 with
  the policy of policy.cuh:54-63 (serial ascending-tile fp32 adds, threshold
  = atol + (rtol * mag) as two rounded ops, strict ``>``), i.e. the same
  oracle the reference's tests use (tests/cutlass_gemm/test_abft_finalize_gpu.py:420-449).
* ``locate``          — the Classic ratio locator of src/abft/methods.py:201-237,
  in fp32 op for op.
"""
from __future__ import annotations

import numpy as np

from .formats import bf16_round


def epilogue(dot, alpha, weights, fault=(-1, -1, -1), out="f32", padded_n=None):
    """Epilogue of one GEMM given exact dot products ``dot`` [M, N].

    Returns (output fp32 values as stored, observed [C, Tm, Np] float64 sums of
    fp32 products, hit, nonfinite). ``dot`` must be exactly representable in
    fp32 for bit-exact outputs (integer/dyadic test data).
    """
    m, n = dot.shape
    v = (np.float32(alpha) * dot.astype(np.float32)).astype(np.float32)
    row, col, bit = fault
    hit = 0
    if bit >= 0:
        bits = v.view(np.uint32)
        bits[row, col] ^= np.uint32(1 << bit)
        hit = 1
    stored = v if out == "f32" else bf16_round(v)
    with np.errstate(invalid="ignore"):
        nonfinite = int(not np.isfinite(stored).all())
    weights = np.asarray(weights, np.float32)
    c = weights.shape[0]
    tiles = (m + 127) // 128
    np_ = padded_n if padded_n is not None else n
    observed = np.zeros((c, tiles, np_), np.float64)
    with np.errstate(invalid="ignore", over="ignore"):
        for t in range(tiles):
            rows = slice(t * 128, min(m, t * 128 + 128))
            prod = weights[:, rows, None].astype(np.float32) * v[None, rows, :]
            observed[:, t, :n] = prod.astype(np.float64).sum(axis=1)
    return stored, observed, hit, nonfinite


def finalize_serial(observed, predicted, magnitude, n, atol, rtol, reference=None, diagnostics=True,
                    hit=0, nonfinite=False, thresholds=None):
    """Bit-exact packet (reference, residual, threshold, flags, hit, location)."""
    obs_p = np.asarray(observed, np.float32)[..., :n]
    c, tiles = obs_p.shape[:2]
    obs = np.zeros((c, n), np.float32)
    for t in range(tiles):
        obs = obs + obs_p[:, t]
    if reference is None:
        ref = np.zeros((2, c, n), np.float32)
        pred_p = np.asarray(predicted, np.float32)[..., :n]
        mag_p = np.asarray(magnitude, np.float32)[..., :n]
        for t in range(tiles):
            ref[0] = ref[0] + pred_p[:, t]
            ref[1] = ref[1] + mag_p[:, t]
    else:
        ref = np.array(reference, np.float32, copy=True)
    pred, mag = ref[0], ref[1]
    with np.errstate(invalid="ignore", over="ignore"):
        residual = (obs - pred).astype(np.float32)
        if thresholds is None:
            threshold = (mag * np.float32(rtol)).astype(np.float32) + np.float32(atol)
        else:
            threshold = np.broadcast_to(np.asarray(thresholds, np.float32), (c, n)).copy()
        threshold = threshold.astype(np.float32)
        finite = (np.isfinite(obs).all() and np.isfinite(ref).all() and np.isfinite(residual).all()
                  and np.isfinite(threshold).all())
        has_nonfinite = bool(nonfinite) or not finite
        detected = has_nonfinite or bool((np.abs(residual) > threshold).any()) or bool((threshold < 0).any())
    flags = np.array([detected, has_nonfinite, False, False, False])
    empty = np.zeros(0, np.float32)
    return (ref, residual if diagnostics else empty, threshold if diagnostics else empty, flags,
            np.array([int(bool(hit))], np.int32), np.array([-1, -1], np.int64))


def locate(residual, threshold, detected, nonfinite, m):
    """Classic.verify localisation: returns (located, (row, col))."""
    residual = np.asarray(residual, np.float32)
    threshold = np.asarray(threshold, np.float32)
    failed = np.abs(residual) > threshold
    columns = failed.any(axis=0)
    col = int(np.argmax(columns)) if columns.size else 0
    d0, d1 = residual[0, col], residual[1, col]
    t0, t1 = threshold[0, col], threshold[1, col]
    with np.errstate(all="ignore"):
        ratio = np.float32(d1 / (np.float32(1) if d0 == 0 else d0))
        if not np.isfinite(ratio):
            return False, (-1, -1)
        row = int(np.rint(ratio)) - 1
        rp1 = np.float32(row + 1)
        consistency = np.float32(abs(np.float32(d1 - np.float32(rp1 * d0))))
        allowance = np.float32(t1 + np.float32(abs(rp1) * t0))
        located = bool(detected) and not bool(nonfinite) and int(columns.sum()) == 1 and abs(d0) > t0
        located = located and 0 <= row < m and consistency <= allowance
        denom = max(np.float32(abs(d0) - t0), np.float32(np.finfo(np.float32).tiny))
        uncertainty = np.float32(np.float32(t1 + np.float32(abs(ratio) * t0)) / np.float32(denom))
        located = located and np.float32(np.float32(abs(np.float32(ratio - rp1))) + uncertainty) < 0.5
    return located, ((row, col) if located else (-1, -1))


def classic_weights(m):
    """Classic projection weights [ones; 1..M] (src/abft/methods.py:162-164)."""
    return np.stack([np.ones(m, np.float32), np.arange(1, m + 1, dtype=np.float32)])


def sum_weights(m):
    """Sum projection weights (src/abft/methods.py:252-253)."""
    return np.ones((1, m), np.float32)
