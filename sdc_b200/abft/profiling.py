"""Per-stage profile of one ABFT execution with the PyTorch profiler.

The interface follows the reference's src/abft/profiling.py (``STAGES``,
``summarize_profile``, ``profile_prepared``, ``print_profile``): the engine
opens a profiler scope named ``abft.<stage>`` around each of its phases (the
``profile_scope`` argument of ``execute_prepared``), and a profiled run of
``repeats`` unprotected and protected calls in alternating order is reduced
to per-stage statistics. A stage's GPU time is the device activity the
profiler correlates with its scope (kernels and copies, without host launch
gaps); its CPU time is the scope's host duration (submission, waits and the
profiler's own cost, overlapping the GPU work). Nothing here synchronises
inside the profiled region.
"""
from __future__ import annotations

import math
import statistics

# Stage -> what it covers. Stages a path does not run are left out of its
# summary; ``abft.total`` encloses the others and is not their sum.
STAGES = {
    "baseline.gemm": "unprotected GEMM",
    "abft.reference": "checksum weights and reference preparation",
    "abft.fault_prepare": "fault-injected operand copies (reference path)",
    "abft.execute": "protected GEMM call (checksums, prediction, status words)",
    "abft.finalize": "device finalize: column merge, thresholds, non-finite rule, flags",
    "abft.merge_reference": "predicted checksum and magnitude merge",
    "abft.merge_observed": "observed checksum merge",
    "abft.detect": "threshold comparison and non-finite detection",
    "abft.locate": "error location",
    "abft.verify": "method detection and location together",
    "abft.recover_recheck": "recovery and recheck",
    "abft.report_flags": "report status tensors",
    "abft.total": "whole protected call",
}

# Kernels of this library that run the GEMM itself (the rest of a stage's
# GPU activity is reported beside them).
_GEMM_KERNELS = ("gemm_kernel",)


def _stats(values):
    if not values or any(not math.isfinite(v) or v < 0 for v in values):
        raise ValueError("Profile timings must be finite and nonnegative")
    return {"median": statistics.median(values), "mean": statistics.mean(values), "min": min(values),
            "max": max(values), "samples": list(values)}


def _gemm_kernel_us(event):
    """Device time of this library's GEMM kernels under ``event`` (its own
    correlated kernels and those of its child scopes)."""
    own = sum(k.duration for k in getattr(event, "kernels", ()) if any(name in k.name for name in _GEMM_KERNELS))
    return own + sum(_gemm_kernel_us(child) for child in getattr(event, "cpu_children", ()))


def _device_us(event):
    value = getattr(event, "device_time_total", None)
    return getattr(event, "cuda_time_total", 0.0) if value is None else value


def summarize_profile(events, repeats, *, input_fused, native=False):
    """Per-stage statistics from profiler events. Only CPU-side scope events
    are counted (a scope's device time already includes its kernels), and
    every stage the path must run needs exactly ``repeats`` samples."""
    scopes = {name: [] for name in STAGES}
    for event in events:
        device_type = getattr(getattr(event, "device_type", None), "name", "CPU")
        if event.name in scopes and device_type == "CPU":
            scopes[event.name].append(event)
    required = {"baseline.gemm", "abft.reference", "abft.execute", "abft.total"}
    required.add("abft.finalize" if native else "abft.verify")
    for name in sorted(required):
        if len(scopes[name]) != repeats:
            raise RuntimeError(f"Incomplete profile: {name}, expected {repeats} samples")
    if not sum(_device_us(e) for e in scopes["baseline.gemm"]):
        raise RuntimeError("CUDA activity timings are unavailable; check the PyTorch profiler's CUPTI support")
    rows = []
    for name, label in STAGES.items():
        samples = scopes[name]
        if not samples:
            continue
        if len(samples) % repeats:
            raise RuntimeError(f"Incomplete profile: {name}, {len(samples)} samples for {repeats} repeats")
        row = {"stage": name, "label": label, "calls_per_repeat": len(samples) // repeats,
               "gpu_active_ms": _stats([_device_us(e) / 1000 for e in samples]),
               "cpu_scope_ms": _stats([e.cpu_time_total / 1000 for e in samples])}
        if name in {"baseline.gemm", "abft.execute"}:
            gemm = [_gemm_kernel_us(e) for e in samples]
            if all(v > 0 for v in gemm):
                row["gemm_kernel_ms"] = _stats([v / 1000 for v in gemm])
                row["other_gpu_activity_ms"] = _stats([max(0.0, _device_us(e) - v) / 1000
                                                       for e, v in zip(samples, gemm, strict=True)])
        rows.append(row)
    fused = ("the checksums, the projection and the prediction run inside the GEMM kernel (abft.execute); "
             "finalize is one further kernel" if native and input_fused else
             "separate reference and verification stages")
    return {"repeats": repeats, "stages": rows,
            "gpu_scope": "device activity correlated with each CPU scope; host launch gaps excluded",
            "cpu_scope": "host time of each scope, including submission, waits and profiler overhead",
            "exclusions": ["compilation", "operand preparation and quantisation", "warm-up", "printing",
                           "report serialisation"],
            "fused_scope": fused}


def _compare(expected, actual):
    """Whether the protected call's output equals the unprotected one bit for
    bit, and their largest finite absolute difference."""
    import torch

    same = expected.shape == actual.shape and expected.dtype == actual.dtype
    if same:
        as_int = {1: torch.uint8, 2: torch.int16, 4: torch.int32, 8: torch.int64}[expected.element_size()]
        same = bool(torch.equal(expected.contiguous().view(as_int), actual.contiguous().view(as_int)))
    diff = (expected.float() - actual.float()).abs()
    finite = diff[diff.isfinite()]
    return {"bit_identical": same, "max_abs_diff": float(finite.max()) if finite.numel() else 0.0}


def profile_prepared(prepared, config, *, warmup, repeats):
    """Profile ``repeats`` unprotected and protected calls on prepared
    operands (the order alternates per repeat, as in the paired timings),
    after ``warmup`` calls of each under throw-away scope names. The output
    comparison and the last report are read after the profiler has stopped."""
    import torch

    from .config import parse_abft_config
    from .engine import execute_prepared

    cfg = parse_abft_config(config)
    record = torch.profiler.record_function
    device = prepared.a.device
    activities = [torch.profiler.ProfilerActivity.CPU, torch.profiler.ProfilerActivity.CUDA]
    torch.cuda.synchronize(device)
    with torch.profiler.profile(activities=activities) as profiler:
        for _ in range(warmup):
            prepared.raw_native()
            execute_prepared(prepared, abft_config=cfg, profile_scope=lambda name: record("warmup." + name))
        torch.cuda.synchronize(device)
        for index in range(repeats):
            order = ("baseline", "protected") if index % 2 == 0 else ("protected", "baseline")
            for name in order:
                if name == "baseline":
                    with record("baseline.gemm"):
                        plain = prepared.raw_native()
                else:
                    with record("abft.total"):
                        output, report = execute_prepared(prepared, abft_config=cfg, profile_scope=record)
        torch.cuda.synchronize(device)
    result = summarize_profile(profiler.events(), repeats,
                               input_fused=cfg.reference_mode in {"input_fused", "augmented"},
                               native=cfg.implementation == "native")
    result["last_output_comparison"] = _compare(plain, output)
    result["last_report"] = report.to_record()
    return result


def print_profile(result):
    """A fixed-width table of the median GPU and CPU time per stage."""
    print(f"{'stage':22s} {'gpu ms (median)':>16s} {'cpu ms (median)':>16s}  what")
    for row in result["stages"]:
        print(f"{row['stage']:22s} {row['gpu_active_ms']['median']:16.4f} {row['cpu_scope_ms']['median']:16.4f}"
              f"  {row['label']}")
