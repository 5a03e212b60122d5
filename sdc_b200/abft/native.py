"""Native ABFT executions: fused sm_100a GEMM + device finalize.

Mirrors src/abft/native.py of the reference (``_execute_native``,
``execute_input_fused``, the builtin-weight cache and ``_tensors``): the host
resolves the method's compiled policy once, the kernels never call Python
hooks, and every decision stays a device tensor until the caller asks for it
(``bool(detected)`` is the one host read, taken only when recovery or
``on_error="raise"`` needs it). Extensions over the reference:

* the prediction layout (``AbftConfig.reference_layout``) is passed to the
  GEMM op; "kslice" computes the prediction inside the GEMM;
* ``AbftConfig.locate`` runs the device Classic locator after finalize
  (policy 0 only), filling ``located``/``location``;
* ``recovery="correct"`` recomputes just the located element on the device
  and falls back to the reference's full recompute + recheck otherwise.
"""
from __future__ import annotations

import time
from collections import OrderedDict
from contextlib import contextmanager, nullcontext
from threading import Lock

import torch

from .methods import Classic, Sum, get_method

_weights = OrderedDict()
_weights_lock = Lock()
_MAX_WEIGHT_ENTRIES = 32
_MAX_WEIGHT_BYTES = 16 * 1024 * 1024


def _builtin_weights(method, prepared, cfg, policy):
    """Projection weights for the builtin formulas, cached per (policy, stream,
    m); plugin or overridden preparations are never cached."""
    custom = any(name in vars(method) for name in ("projection_weights", "prepare_fused"))
    if type(method) not in {Classic, Sum} or method.stateful or custom:
        return method.prepare_fused(prepared, cfg)
    device = torch.device(prepared.a.device)
    stream = torch.cuda.current_stream(device)
    key = (policy.algorithm, stream.device.index, prepared.m)
    with _weights_lock:
        entry = _weights.pop(key, None)
        if entry is None:
            weights = method.projection_weights(prepared).to(torch.float32).contiguous()
            ready = torch.cuda.Event()
            ready.record(stream)
            entry = (weights, ready, stream.cuda_stream)
        weights, ready, owner = entry
        if weights.numel() * 4 <= _MAX_WEIGHT_BYTES:
            _weights[key] = entry
            while (len(_weights) > _MAX_WEIGHT_ENTRIES or
                   sum(item[0].numel() * 4 for item in _weights.values()) > _MAX_WEIGHT_BYTES):
                _weights.popitem(last=False)
        if owner != stream.cuda_stream:
            stream.wait_event(ready)
            weights.record_stream(stream)
    return {"weights": weights, "m": prepared.m, "n": prepared.n}


def _tensors(finalized, diagnostics):
    reference, residual, threshold, flags, hit, location = finalized
    detected, nonfinite, located, recovered, recheck_failed = flags.unbind()
    tensors = dict(detected=detected, nonfinite=nonfinite, located=located, recovered=recovered,
                   recheck_failed=recheck_failed, fault_hit=hit, location=location)
    if diagnostics:
        tensors.update(residual=residual, threshold=threshold)
    return reference, tensors, (residual, threshold, flags)


def _execute_native(prepared, cfg, fault, context, *, method=None, policy=None, profile_scope=None):
    from .. import ops, require_device
    from .engine import AbftError, AbftReport, _commit_method, _report_context, _selected

    if method is None:
        method = get_method(cfg.method)
        if method.stateful:
            raise ValueError("Stateful native methods require a retained method_instance or MethodSession")
    policy = method.validate_execution(prepared, cfg) if policy is None else policy
    if cfg.reference_mode != "input_fused":
        raise NotImplementedError("native executions on B200 use the input_fused reference")
    algorithm = policy.algorithm
    locate = cfg.locate and algorithm == 0
    need_statistics = cfg.diagnostics or method.needs_diagnostics or locate
    require_device(prepared.a.device)
    selected = _selected(fault, context)
    injection = (-1, -1, -1)
    if selected:
        if fault.location != "accumulator":
            raise ValueError("native fused GEMM accepts only accumulator faults")
        if fault.row >= prepared.m or fault.col >= prepared.n or fault.bit >= 32:
            raise ValueError("Accumulator fault coordinate/bit outside FP32 output")
        injection = (fault.row, fault.col, fault.bit)
    started = time.perf_counter()
    events = []
    scope = profile_scope or nullcontext

    @contextmanager
    def phase(name):
        with scope("abft." + name):
            mark = None
            if cfg.timing and prepared.a.is_cuda:
                mark = torch.cuda.Event(enable_timing=True)
                mark.record(torch.cuda.current_stream(prepared.a.device))
            yield
            if mark is not None:
                end = torch.cuda.Event(enable_timing=True)
                end.record(torch.cuda.current_stream(prepared.a.device))
                events.append((name, mark, end))

    with phase("reference"):
        state = _builtin_weights(method, prepared, cfg, policy)
        weights = state["weights"]
        if (weights.ndim != 2 or weights.shape != (policy.channels, prepared.m) or
                weights.dtype != torch.float32 or weights.device != prepared.a.device or
                not weights.is_contiguous()):
            raise ValueError("Native method weights do not match compiled policy channels/format/device")
        thresholds = state.get("thresholds")
        if thresholds is not None and (
            not isinstance(thresholds, torch.Tensor) or thresholds.dtype != torch.float32 or
            thresholds.device != prepared.a.device or not thresholds.is_contiguous() or
            thresholds.shape not in {(1,), (policy.channels, prepared.n)}
        ):
            raise ValueError("Native method thresholds must be contiguous FP32 [1] or [channels,N] on the operand device")
        finalize_args = (algorithm, thresholds)

    def run(fault_tuple):
        nonfinite = torch.empty(1, device=prepared.a.device, dtype=torch.int32)
        output, observed, hit, predicted, magnitude = prepared.collected_reference_native(
            weights, fault_tuple, algorithm=algorithm, nonfinite=nonfinite, layout=cfg.reference_layout)
        return output, (observed, predicted, magnitude, hit, nonfinite)

    def finalize(evidence, first_reference):
        return ops.abft_finalize_reference(*evidence, prepared.n, cfg.atol, cfg.rtol, first_reference,
                                           need_statistics, *finalize_args)

    with phase("execute"):
        output, evidence = run(injection)
    with phase("finalize"):
        reference, tensors, (residual, threshold, flags) = _tensors(finalize(evidence, None), need_statistics)
    if locate:
        with phase("locate"):
            location, located = ops.abft_locate(residual, threshold, flags, prepared.m)
            tensors.update(location=location, located=located)
    state = {**state, "reference": reference}
    del evidence
    report_context = _report_context(prepared, cfg, fault, context, selected, output, method)
    report_context["reference_operand_reuse"] = "mainloop_shared_operands"
    report_context["threshold_source"] = "method_state" if thresholds is not None else "config_atol_rtol"
    report = AbftReport(tensors, report_context, cfg.method, "input_fused_native", events)
    if cfg.recovery in {"recompute", "correct"} and bool(tensors["detected"].item()):
        with phase("recover_recheck"):
            if cfg.recovery == "correct" and locate and bool(tensors["located"].item()):
                correct = (ops.abft_fp8_block_correct if getattr(prepared, "blockwise", False) else
                           ops.abft_fp8_correct if prepared.precision == "fp8" else ops.abft_nvfp4_correct)
                corrected = correct(*prepared._native_args(), tensors["location"], tensors["located"], output)
                tensors["recovered"] = corrected
                tensors["recheck_failed"] = ~corrected
                report.context["recovery_action"] = "located_element_recomputed"
            else:
                replacement, retry_evidence = run((-1, -1, -1))
                _, checked, _ = _tensors(finalize(retry_evidence, reference), need_statistics)
                tensors["recheck_failed"] = checked["detected"]
                tensors["recovered"] = ~checked["detected"]
                if need_statistics:
                    tensors["retry_residual"] = checked["residual"]
                if not bool(checked["detected"].item()):
                    output = replacement
                report.context["recovery_action"] = "full_recompute"
    with phase("state_update") if method.stateful or method.needs_diagnostics else nullcontext():
        _commit_method(method, state, tensors, context, prepared)
    if not cfg.diagnostics:
        for key in ("residual", "threshold", "retry_residual"):
            tensors.pop(key, None)
    should_raise = (cfg.on_error == "raise" and bool(tensors["detected"].item())
                    and not bool(tensors["recovered"].item()))
    report.host_seconds = time.perf_counter() - started
    if should_raise:
        raise AbftError(report)
    return output, report


def execute_input_fused(prepared, cfg, fault, context, *, method=None, policy=None, profile_scope=None):
    return _execute_native(prepared, cfg, fault, context, method=method, policy=policy,
                           profile_scope=profile_scope)
