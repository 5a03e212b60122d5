"""The reference's CPU/torch ABFT path, restated. Test infrastructure only.

Restates ``abft.execute(a, b, "fp32", "none", abft_config={"method": "classic",
...}, reference_mm=torch.mm, collector_fn=collect)`` of the reference:
  PreparedGemm.prepare fp32 (src/abft/operands.py:28-41),
  Classic.prepare K-chunked expected/magnitude (src/abft/methods.py:181-197),
  the CPU collector of tests/abft/test_framework.py:14-22 (C = A @ B, XOR of
  one fp32 bit, partials = W @ C),
  Classic.propagate / verify incl. the ratio locator (src/abft/methods.py:198-241),
  and the recompute-and-recheck retry (src/abft/engine.py:274-291).
The torch CPU ops are the same ones the reference calls, so results are bit
for bit those of the reference on the same machine. This is the timed CPU
baseline of bench.py and the checker of the config-1 golden trials.
"""
from __future__ import annotations

import torch


def classic_weights(m, dtype=torch.float32):
    return torch.stack((torch.ones(m, dtype=dtype), torch.arange(1, m + 1, dtype=dtype)))


def prepare(a, b, weights, block_k=256):
    m, k = a.shape
    n = b.shape[1]
    expected = torch.zeros((weights.shape[0], n), dtype=torch.float32)
    magnitude = torch.zeros_like(expected)
    for start in range(0, k, block_k):
        end = min(k, start + block_k)
        ab, bb = a[:, start:end].contiguous(), b[start:end, :].contiguous()
        expected += torch.mm(torch.mm(weights, ab).contiguous(), bb)
        magnitude += torch.mm(torch.mm(weights.abs(), ab.abs()).contiguous(), bb.abs().contiguous())
    return expected, magnitude


def collect(a, b, weights, fault):
    output = a @ b
    row, col, bit = fault
    if row >= 0:
        mask = 1 << bit if bit < 31 else -(1 << 31)
        output.view(torch.int32)[row, col] ^= mask
    return output, (weights @ output).unsqueeze(1), int(row >= 0)


def verify(observed, output, expected, magnitude, atol, rtol, m, locate=True):
    residual = observed - expected
    threshold = atol + rtol * magnitude
    nonfinite = (~torch.isfinite(observed)).any() | (~torch.isfinite(expected)).any()
    nonfinite |= (~torch.isfinite(threshold)).any() | (~torch.isfinite(output)).any()
    nonfinite |= (~torch.isfinite(residual)).any()
    failed = residual.abs() > threshold
    detected = failed.any() | nonfinite
    result = {"detected": bool(detected), "nonfinite": bool(nonfinite), "located": False,
              "location": [-1, -1], "residual": residual, "threshold": threshold}
    if not locate:
        return result
    columns = failed.any(dim=0)
    col = columns.to(torch.int64).argmax()
    d0, d1 = residual[:, col].unbind()
    ratio = d1 / torch.where(d0 == 0, torch.ones_like(d0), d0)
    row = ratio.round().to(torch.int64) - 1
    consistency = (d1 - (row + 1).float() * d0).abs()
    allowance = threshold[1, col] + (row + 1).abs().float() * threshold[0, col]
    located = detected & ~nonfinite & (columns.sum() == 1) & (d0.abs() > threshold[0, col])
    located &= (row >= 0) & (row < m) & (consistency <= allowance)
    uncertainty = (threshold[1, col] + ratio.abs() * threshold[0, col]) / (
        d0.abs() - threshold[0, col]).clamp_min(torch.finfo(torch.float32).tiny)
    located &= (ratio - (row + 1)).abs() + uncertainty < 0.5
    result["located"] = bool(located)
    result["location"] = [int(row), int(col)] if bool(located) else [-1, -1]
    return result


def execute(a, b, atol=1e-4, rtol=1e-4, fault=(-1, -1, -1), block_k=256, recovery="none", state=None):
    """One protected fp32 GEMM on the CPU. Returns (output, report dict, state).

    ``state`` (weights, expected, magnitude) may be passed back in to reuse the
    input-side reference across trials on the same operands, as a caller of
    execute_prepared would.
    """
    a = a.float()
    b = b.float()
    m, n = a.shape[0], b.shape[1]
    if state is None:
        weights = classic_weights(m)
        expected, magnitude = prepare(a, b, weights, block_k)
        state = (weights, expected, magnitude)
    weights, expected, magnitude = state
    output, partials, hit = collect(a, b, weights, fault)
    observed = partials.sum(dim=1)[:, :n]
    report = verify(observed, output, expected, magnitude, atol, rtol, m)
    report["fault_hit"] = hit
    report["recovered"] = False
    if recovery == "recompute" and report["detected"]:
        replacement, retry_partials, _ = collect(a, b, weights, (-1, -1, -1))
        checked = verify(retry_partials.sum(dim=1)[:, :n], replacement, expected, magnitude, atol, rtol, m,
                         locate=False)
        report["recovered"] = not checked["detected"]
        if report["recovered"]:
            output = replacement
    return output, report, state
