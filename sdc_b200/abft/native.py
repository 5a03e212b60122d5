"""Native executions: the fused sm_100a GEMM, the device finalize and locator.

The host resolves the method's compiled policy once per call; the kernels
never call back into Python, and every decision stays a device tensor until
a caller asks for it (recovery and ``on_error="raise"`` are the only host
reads). One call is:

1. the builtin projection weights W [C, M] (``WeightCache``: made once per
   policy, device and M, shared across streams with an event);
2. the input-fused GEMM (``reference_layout`` "tile": the reference's
   per-M-tile predicted partials; "kslice": computed inside the GEMM launch)
   with the epilogue fault, if this call's fault fires;
3. the device finalize (threshold atol + rtol * magnitude, or the method's
   own thresholds), then optionally the device ratio locator (policy 0);
4. on detection with ``recovery``: either the located element recomputed on
   the device (``"correct"``), or a full recompute judged against the first
   call's reference (``"recompute"``, and ``"correct"`` when nothing was
   located); then the engine's shared tail (commit, diagnostics, raise).

The augmented BF16 mode (``execute_augmented``) follows the same steps with
BF16 encoding weights, the compact augmented GEMM and the packed finalize.
Both mirror src/abft/native.py of the reference (``_builtin_weights``,
``_execute_native``).
"""
from __future__ import annotations

import time
from collections import OrderedDict
from threading import Lock

import torch

from .engine import AbftReport, _finish, _injection, _Plan, _selected, _Timer, call_context
from .methods import Classic, Sum, get_method


class WeightCache:
    """Least-recently-used cache of the builtin projection weights, bounded
    by entry count and bytes. An entry remembers the stream that made it: a
    consumer on another stream first waits for that work (event) and marks
    the tensor as used on its own stream."""

    def __init__(self, max_entries=32, max_bytes=16 * 1024 * 1024):
        self.max_entries, self.max_bytes = max_entries, max_bytes
        self._entries = OrderedDict()  # key -> (weights, ready event, producing stream handle)
        self._lock = Lock()

    def peek(self, key):
        with self._lock:
            entry = self._entries.get(key)
            return None if entry is None else entry[0]

    def weights(self, method, prepared, policy, dtype=torch.float32):
        device = torch.device(prepared.a.device)
        stream = torch.cuda.current_stream(device)
        key = (policy.algorithm, stream.device.index, prepared.m, dtype)
        with self._lock:
            entry = self._entries.pop(key, None)
            if entry is None:
                made = method.projection_weights(prepared).to(dtype).contiguous()
                ready = torch.cuda.Event()
                ready.record(stream)
                entry = (made, ready, stream.cuda_stream)
            if entry[0].numel() * entry[0].element_size() <= self.max_bytes:
                self._entries[key] = entry
                self._evict()
        weights, ready, producer = entry
        if producer != stream.cuda_stream:
            stream.wait_event(ready)
            weights.record_stream(stream)
        return weights

    def _evict(self):
        while len(self._entries) > self.max_entries or sum(
                item[0].numel() * item[0].element_size() for item in self._entries.values()) > self.max_bytes:
            self._entries.popitem(last=False)


WEIGHTS = WeightCache()


def _method_state(method, prepared, cfg, policy):
    """Weights (and optional thresholds) of this call. Only unmodified
    builtin methods use the cache; plugins prepare their own. The augmented
    mode encodes with BF16 weights (the input format of A)."""
    augmented = cfg.reference_mode == "augmented"
    customised = any(hook in vars(method) for hook in ("projection_weights", "prepare_fused", "prepare_augmented"))
    if type(method) in {Classic, Sum} and not method.stateful and not customised:
        dtype = torch.bfloat16 if augmented else torch.float32
        return {"weights": WEIGHTS.weights(method, prepared, policy, dtype), "m": prepared.m, "n": prepared.n,
                **({"augmented": True} if augmented else {})}
    return method.prepare_augmented(prepared, cfg) if augmented else method.prepare_fused(prepared, cfg)


def _check_state(state, prepared, policy, dtype=torch.float32):
    weights = state["weights"]
    if (weights.ndim != 2 or weights.shape != (policy.channels, prepared.m) or weights.dtype != dtype
            or weights.device != prepared.a.device or not weights.is_contiguous()):
        raise ValueError("Native method weights do not match compiled policy channels/format/device")
    thresholds = state.get("thresholds")
    if thresholds is not None and (not isinstance(thresholds, torch.Tensor) or thresholds.dtype != torch.float32
                                   or thresholds.device != prepared.a.device or not thresholds.is_contiguous()
                                   or thresholds.shape not in {(1,), (policy.channels, prepared.n)}):
        raise ValueError("Native method thresholds must be contiguous FP32 [1] or [channels,N] on the operand "
                         "device")
    return weights, thresholds


def _decisions(packet, statistics):
    """Report tensors from a finalize packet (reference, residual, threshold,
    flags, hit, location)."""
    reference, residual, threshold, flags, hit, location = packet
    detected, nonfinite, located, recovered, recheck_failed = flags.unbind()
    tensors = {"detected": detected, "nonfinite": nonfinite, "located": located, "recovered": recovered,
               "recheck_failed": recheck_failed, "fault_hit": hit, "location": location}
    if statistics:
        tensors.update(residual=residual, threshold=threshold)
    return reference, tensors, (residual, threshold, flags)


def execute_input_fused(prepared, cfg, fault, context, *, method=None, policy=None, profile_scope=None):
    from .. import ops, require_device

    if method is None:
        method = get_method(cfg.method)
        if method.stateful:
            raise ValueError("Stateful native methods require a retained method_instance or MethodSession")
    policy = method.validate_execution(prepared, cfg) if policy is None else policy
    if cfg.reference_mode != "input_fused":
        raise NotImplementedError("native executions on B200 use the input_fused reference")
    rows = cfg.row_checksums
    locate = (cfg.locate and policy.algorithm == 0) or rows
    statistics = cfg.diagnostics or method.needs_diagnostics or locate
    require_device(prepared.a.device)
    plan = _Plan(prepared, cfg, fault, context, method, policy, _selected(fault, context))
    injection = _injection(prepared, fault, plan.selected, accumulator_only=True)
    timer = _Timer(cfg.timing, prepared.a.device, profile_scope)
    started = time.perf_counter()

    with timer.phase("reference"):
        plan.state = _method_state(method, prepared, cfg, policy)
        weights, thresholds = _check_state(plan.state, prepared, policy)

    def gemm(injected):
        nonfinite = torch.empty(1, device=prepared.a.device, dtype=torch.int32)
        if rows:
            output, observed, hit, predicted, magnitude, *row_evidence = prepared.collected_rows_native(
                weights, injected, algorithm=policy.algorithm, nonfinite=nonfinite, layout=cfg.reference_layout)
            return output, (observed, predicted, magnitude, hit, nonfinite), row_evidence
        output, observed, hit, predicted, magnitude = prepared.collected_reference_native(
            weights, injected, algorithm=policy.algorithm, nonfinite=nonfinite, layout=cfg.reference_layout)
        return output, (observed, predicted, magnitude, hit, nonfinite), None

    def finalize(evidence, reference):
        return ops.abft_finalize_reference(*evidence, prepared.n, cfg.atol, cfg.rtol, reference, statistics,
                                           policy.algorithm, thresholds)

    def decide(evidence, row_evidence, reference):
        """Column decisions from the finalize; with row checksums, the row
        check is merged in and the location is the failing (row, column)
        pair, if exactly one of each failed."""
        reference, tensors, (residual, threshold, flags) = _decisions(finalize(evidence, reference), statistics)
        if row_evidence is not None:
            location, located, row_flags, row_residual, row_threshold = ops.abft_locate2d(
                *row_evidence, cfg.atol, cfg.rtol, residual, threshold, flags, policy.algorithm)
            tensors["detected"] = tensors["detected"] | row_flags[0]
            tensors["nonfinite"] = tensors["nonfinite"] | row_flags[1]
            tensors["location"], tensors["located"] = location, located
            if cfg.diagnostics:
                tensors.update(row_residual=row_residual, row_threshold=row_threshold)
        return reference, tensors, (residual, threshold, flags)

    with timer.phase("execute"):
        output, evidence, row_evidence = gemm(injection)
    with timer.phase("finalize"):
        first_reference, tensors, (residual, threshold, flags) = decide(evidence, row_evidence, None)
    del evidence, row_evidence
    if locate and not rows:
        with timer.phase("locate"):
            tensors["location"], tensors["located"] = ops.abft_locate(residual, threshold, flags, prepared.m)
    plan.state = {**plan.state, "reference": first_reference}
    described = call_context(prepared, cfg, fault, context, plan.selected, output, method)
    described["reference_operand_reuse"] = "mainloop_shared_operands"
    described["threshold_source"] = "method_state" if thresholds is not None else "config_atol_rtol"
    if rows:
        described["location_assumption"] = "row_and_column_checksums"
    report = AbftReport(tensors, described, cfg.method, "input_fused_native", timer.events)

    def recheck():
        if cfg.recovery == "correct" and locate and bool(tensors["located"].item()):
            # Only the located element is recomputed, in place.
            correct = (ops.abft_fp8_block_correct if getattr(prepared, "blockwise", False) else
                       ops.abft_fp8_correct if prepared.precision == "fp8" else ops.abft_nvfp4_correct)
            fixed = correct(*prepared._native_args(), tensors["location"], tensors["located"], output)
            tensors["recovered"], tensors["recheck_failed"] = fixed, ~fixed
            report.context["recovery_action"] = "located_element_recomputed"
            return None, None
        replacement, retry_evidence, retry_rows = gemm((-1, -1, -1))
        _, checked, _ = decide(retry_evidence, retry_rows, first_reference)
        report.context["recovery_action"] = "full_recompute"
        return replacement, checked

    return _finish(plan, report, output, recheck, timer, started)


def execute_augmented(prepared, cfg, fault, context, *, method=None, policy=None, profile_scope=None):
    """The augmented BF16 execution: one launch computes the output, the
    observed and output-magnitude partials (data tiles' epilogue) and the
    predicted partials (the BF16 checksum rows as extra M-tiles), with
    per-tile fault/non-finite flags; then the packed device finalize. No
    locator: BF16-rounded checksum rows and row numbers cannot place a
    single element. Recovery is the full recompute judged against the first
    call's reference (``"correct"`` falls back to it, nothing is located)."""
    from .. import ops, require_device

    if method is None:
        method = get_method(cfg.method)
        if method.stateful:
            raise ValueError("Stateful native methods require a retained method_instance or MethodSession")
    policy = method.validate_execution(prepared, cfg) if policy is None else policy
    if cfg.reference_mode != "augmented" or prepared.precision != "bf16":
        raise ValueError("augmented currently requires BF16 GEMM")
    statistics = cfg.diagnostics or method.needs_diagnostics
    require_device(prepared.a.device)
    plan = _Plan(prepared, cfg, fault, context, method, policy, _selected(fault, context))
    injection = _injection(prepared, fault, plan.selected, accumulator_only=True)
    timer = _Timer(cfg.timing, prepared.a.device, profile_scope)
    started = time.perf_counter()

    with timer.phase("reference"):
        plan.state = _method_state(method, prepared, cfg, policy)
        weights, thresholds = _check_state(plan.state, prepared, policy, torch.bfloat16)

    def gemm(injected):
        output, partials, tile_flags = prepared.augmented_compact(weights, injected, algorithm=policy.algorithm)
        return output, (partials, tile_flags)

    def finalize(evidence, reference):
        return ops.abft_finalize(*evidence, prepared.n, cfg.atol, cfg.rtol, reference, statistics,
                                 policy.algorithm, thresholds)

    with timer.phase("execute"):
        output, evidence = gemm(injection)
    with timer.phase("finalize"):
        first_reference, tensors, _ = _decisions(finalize(evidence, None), statistics)
    del evidence
    plan.state = {**plan.state, "reference": first_reference}
    described = call_context(prepared, cfg, fault, context, plan.selected, output, method)
    described["reference_operand_reuse"] = "checksum_rows_as_extra_m_tiles"
    described["threshold_source"] = "method_state" if thresholds is not None else "config_atol_rtol"
    report = AbftReport(tensors, described, cfg.method, "augmented_native", timer.events)

    def recheck():
        replacement, retry_evidence = gemm((-1, -1, -1))
        _, checked, _ = _decisions(finalize(retry_evidence, first_reference), statistics)
        report.context["recovery_action"] = "full_recompute"
        return replacement, checked

    return _finish(plan, report, output, recheck, timer, started)
