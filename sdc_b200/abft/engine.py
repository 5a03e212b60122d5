"""One protected GEMM call: plan, evidence, decision, recovery, report.

``execute`` quantises (prepares) the operands once and hands them to
``execute_prepared``. A call is planned once (``_Plan``: method, compiled
policy, whether the configured fault fires, the injection) and then runs on
one of two evidence sources:

* native (``implementation="native"``): the fused sm_100a GEMM, the device
  finalize and, optionally, the device locator (``native.py``);
* reference (``implementation="reference"``): the method's Python hooks,
  with the caller-supplied seams ``raw_fn``, ``reference_mm``,
  ``collector_fn`` and ``reference_collector_fn`` standing in for the GEMM
  (which is how the whole engine runs on a CPU).

Both paths finish the same way (``_finish``): an optional recompute against
the first reference, one ``commit`` of the decisions to the method, the
diagnostics policy and the raise policy. Decisions stay device tensors; the
host reads one only when recovery or ``on_error="raise"`` needs it, and
``AbftReport.to_record`` is the explicit synchronisation point for logging.

The call signatures, report fields, report context keys and error messages
are those of the reference's ``abft`` engine (src/abft/engine.py), so
callers and logs written for it keep working.
"""
from __future__ import annotations

import math
import time
from contextlib import contextmanager, nullcontext
from dataclasses import asdict, dataclass, field

import torch

from ..gemm import backend
from .config import parse_abft_config, parse_fault_config
from .methods import get_method, validate_method_instance
from .operands import INPUT_REFERENCE_PRECISIONS, SCALING, PreparedGemm

NO_FAULT = (-1, -1, -1)
DECISION_KEYS = ("detected", "nonfinite", "located", "location", "recovered", "recheck_failed", "residual",
                 "threshold", "retry_residual")
DIAGNOSTIC_KEYS = ("residual", "threshold", "retry_residual")
CONTEXT_KEYS_FOR_METHODS = ("layer", "role", "call_index", "execution_kind", "retry", "scale_profile")


@dataclass
class AbftReport:
    """Decision tensors of one call (attribute access: ``report.detected``)
    plus its context; device tensors until ``to_record`` reads them."""

    tensors: dict
    context: dict
    method: str
    execution_path: str
    timing_events: list = field(default_factory=list)
    host_seconds: float = 0.0

    def __getattr__(self, name):
        tensors = self.__dict__.get("tensors", {})
        if name in tensors:
            return tensors[name]
        raise AttributeError(name)

    def to_record(self):
        """Plain, strict-JSON record (the explicit device-to-host sync).
        Non-finite numbers become null and their paths are listed under
        ``nonfinite_metrics``."""
        record = {name: value.detach().cpu().tolist() for name, value in self.tensors.items()}
        record.update(context=self.context, method=self.method, execution_path=self.execution_path,
                      host_seconds=self.host_seconds)
        if self.timing_events:
            self.timing_events[-1][2].synchronize()
            record["timing_ms"] = {name: begin.elapsed_time(end) for name, begin, end in self.timing_events}
        nonfinite = {}
        record = _strict_json(record, "", nonfinite)
        if nonfinite:
            record["nonfinite_metrics"] = nonfinite
        return record


def _strict_json(value, path, nonfinite):
    if isinstance(value, float) and not math.isfinite(value):
        nonfinite[path] = str(value)
        return None
    if isinstance(value, dict):
        return {key: _strict_json(item, f"{path}.{key}" if path else str(key), nonfinite)
                for key, item in value.items()}
    if isinstance(value, (list, tuple)):
        return [_strict_json(item, f"{path}[{index}]", nonfinite) for index, item in enumerate(value)]
    return value


class AbftError(RuntimeError):
    def __init__(self, report):
        super().__init__("ABFT detected an unrecovered anomaly")
        self.report = report


def _selected(fault, context):
    """Whether the configured fault fires on this call: its call index,
    layer and role (when given) must match, and never on a retry."""
    if fault.location == "none" or context.get("retry", False):
        return False
    if context.get("call_index", 1) != fault.call_index:
        return False
    return all(wanted is None or context.get(name) == wanted for name, wanted in (("layer", fault.layer),
                                                                                 ("role", fault.role)))


def _injection(prepared, fault, selected, accumulator_only=False):
    """The (row, col, bit) XOR the epilogue applies, or NO_FAULT."""
    if not selected:
        return NO_FAULT
    if fault.location != "accumulator":
        if accumulator_only:
            raise ValueError("native fused GEMM accepts only accumulator faults")
        return NO_FAULT
    if fault.row >= prepared.m or fault.col >= prepared.n or fault.bit >= 32:
        raise ValueError("Accumulator fault coordinate/bit outside FP32 output")
    return (fault.row, fault.col, fault.bit)


class _Timer:
    """Named phases timed with CUDA events on the operand stream (when
    ``timing`` is on) and wrapped in the caller's profiler scope."""

    def __init__(self, enabled, device, scope=None):
        self.enabled = enabled and device.type == "cuda"
        self.device = device
        self.scope = scope or nullcontext
        self.events = []

    def _event(self):
        event = torch.cuda.Event(enable_timing=True)
        event.record(torch.cuda.current_stream(self.device))
        return event

    @contextmanager
    def phase(self, name):
        with self.scope("abft." + name):
            begin = self._event() if self.enabled else None
            yield
            if begin is not None:
                self.events.append((name, begin, self._event()))


def call_context(prepared, cfg, fault, context, selected, output, method=None):
    """The report context: the caller's context plus what ran and how."""
    augmented = cfg.reference_mode == "augmented"
    fused = cfg.reference_mode in {"input_fused", "augmented"}
    native = cfg.implementation == "native"
    policy = getattr(method, "compiled_policy", None)
    channels = policy.channels if policy is not None else getattr(method, "channels", 2)
    if not selected:
        injection_point = "none"
    elif fault.location == "accumulator":
        injection_point = "post_alpha_fp32_epilogue_before_output_cast"
    else:
        injection_point = "prepared_input_codes"
    if augmented:
        # BF16-rounded checksum rows and row numbers: no single-element ratio.
        location = "disabled_for_low_precision_encoding"
    elif native:
        location = "device_ratio_locator" if cfg.locate and channels == 2 else "disabled_for_native_policy"
    else:
        location = "disabled_for_detection_only_method" if channels == 1 else "single_output_element"
    if augmented:
        algorithm = "augmented_gemm"
    else:
        algorithm = "input_fused_fp32_projection" if fused else "separate_projection_arithmetic"
    described = {
        "fault": asdict(fault), "fault_selected": selected, "precision": prepared.precision,
        "scaling": getattr(prepared, "scaling", SCALING[prepared.precision]),
        "reference_mode": cfg.reference_mode, "implementation": cfg.implementation,
        "threshold_scale": cfg.threshold_scale, "checksum_input_precision": "bf16" if augmented else "fp32",
        "reference_algorithm": algorithm,
        "reference_layout": cfg.reference_layout if fused and not augmented else None,
        "augmented_rows_per_data_tile": channels if augmented else 0,
        "compiled_policy": policy.metadata() if policy is not None else None,
        "verification_backend": "cuda_policy" if native else "python_method",
        "compiled_reference_format": dict(policy.reference_formats).get(cfg.reference_mode) if policy else None,
        "protection_scope": "computation_after_input_load" if fused else "prepared_inputs_and_computation",
        "m": prepared.m, "n": prepared.n, "k": prepared.k, "input_precision": prepared.precision,
        "accumulator_precision": "fp32", "output_precision": str(output.dtype), "check_precision": "fp32",
        "injection_point": injection_point, "fault_hit_meaning": "injection_executed_not_output_damage",
        "location_assumption": location,
    }
    return {**context, **described}


def commit_decisions(method, state, tensors, context, prepared):
    """Hand the final decisions of the whole transaction to the method once."""
    decisions = {key: tensors[key] for key in DECISION_KEYS if key in tensors}
    if "threshold" not in decisions and isinstance(state, dict) and state.get("thresholds") is not None:
        decisions["threshold"] = state["thresholds"]
    metadata = {key: context[key] for key in CONTEXT_KEYS_FOR_METHODS if key in context}
    metadata.update(precision=prepared.precision, device=str(prepared.a.device), m=prepared.m, n=prepared.n,
                    k=prepared.k, scaling=getattr(prepared, "scaling", SCALING[prepared.precision]))
    method.commit(state, decisions, metadata)


def _finish(plan, report, output, recheck, timer, started):
    """Shared tail of both paths. ``recheck()`` runs the clean recompute and
    returns (replacement output, its decision tensors)."""
    tensors, method, cfg = report.tensors, plan.method, plan.cfg
    if method is not None and cfg.recovery in {"recompute", "correct"} and bool(tensors["detected"].item()):
        with timer.phase("recover_recheck"):
            replacement, checked = recheck()
            if replacement is not None:
                tensors["recheck_failed"] = checked["detected"]
                tensors["recovered"] = ~checked["detected"]
                if "residual" in checked:
                    tensors["retry_residual"] = checked["residual"]
                if not bool(checked["detected"].item()):
                    output = replacement
    if method is not None:
        tracked = method.stateful or method.needs_diagnostics
        with timer.phase("state_update") if tracked else nullcontext():
            commit_decisions(method, plan.state, tensors, plan.context, plan.prepared)
    if not cfg.diagnostics:
        for key in DIAGNOSTIC_KEYS:
            tensors.pop(key, None)
    report.host_seconds = time.perf_counter() - started
    if method is not None and cfg.on_error == "raise" and bool((tensors["detected"] & ~tensors["recovered"]).item()):
        raise AbftError(report)
    return output, report


@dataclass
class _Plan:
    prepared: PreparedGemm
    cfg: object
    fault: object
    context: dict
    method: object
    policy: object
    selected: bool
    state: object = None


def _default_context(context):
    return {"layer": None, "role": None, "call_index": 1, "execution_kind": "forward", "retry": False,
            **dict(context or {})}


@torch.no_grad()
def execute(a, b, precision, scaling, global_scale="amax", abft_config=None, fault_config=None, context=None, *,
            raw_fn=None, reference_mm=None, collector_fn=None, reference_collector_fn=None, method_instance=None):
    """Protected ``a @ b`` (a: [M, K], b: [K, N]): prepare (quantise) once,
    then execute the prepared GEMM. Returns (output, report or None)."""
    cfg, fault = parse_abft_config(abft_config), parse_fault_config(fault_config)
    if cfg.method == "none" and method_instance is not None:
        raise ValueError("method_instance requires an enabled ABFT method")
    if cfg.method == "none" and raw_fn is None and not _selected(fault, _default_context(context)):
        return backend.gemm(a, b, precision, scaling, global_scale), None
    prepared = PreparedGemm.prepare(a, b, precision, scaling, global_scale)
    return execute_prepared(prepared, cfg, fault, context, raw_fn=raw_fn, reference_mm=reference_mm,
                            collector_fn=collector_fn, reference_collector_fn=reference_collector_fn,
                            method_instance=method_instance)


@torch.no_grad()
def execute_prepared(prepared, abft_config=None, fault_config=None, context=None, *, raw_fn=None,
                     reference_mm=None, collector_fn=None, reference_collector_fn=None, profile_scope=None,
                     method_instance=None):
    """Execute prepared operands without quantising again (see ``execute``)."""
    cfg, fault = parse_abft_config(abft_config), parse_fault_config(fault_config)
    seams = {"raw_fn": raw_fn, "reference_mm": reference_mm, "collector_fn": collector_fn,
             "reference_collector_fn": reference_collector_fn}
    if cfg.reference_mode == "augmented" and prepared.precision != "bf16":
        raise ValueError("augmented currently requires BF16 GEMM")
    if cfg.reference_mode in {"input_fused", "augmented"}:
        if (cfg.reference_mode == "input_fused" and prepared.precision not in INPUT_REFERENCE_PRECISIONS
                and reference_collector_fn is None):
            raise NotImplementedError(f"input_fused reference is not implemented for {prepared.precision}")
        if fault.location in {"a", "b"}:
            raise ValueError("input_fused protects computation only; input memory faults require separate reference")
    context = _default_context(context)
    selected = _selected(fault, context)
    if cfg.implementation == "native" and any(seam is not None for seam in seams.values()):
        raise ValueError("native implementation does not accept reference collector overrides")
    if cfg.method == "none" and method_instance is not None:
        raise ValueError("method_instance requires an enabled ABFT method")
    if cfg.method == "none" and not selected:
        return (raw_fn(prepared) if raw_fn else prepared.raw_native()), None
    method = None
    if cfg.method != "none":
        if method_instance is not None:
            method = validate_method_instance(cfg.method, method_instance)
        else:
            method = get_method(cfg.method)
    if method is not None and method.stateful and method_instance is None:
        raise ValueError("Stateful ABFT methods require a retained method_instance or MethodSession")
    policy = method.validate_execution(prepared, cfg) if method is not None else None
    plan = _Plan(prepared, cfg, fault, context, method, policy, selected)
    if cfg.implementation == "native":
        from .native import execute_augmented, execute_input_fused

        run = execute_augmented if cfg.reference_mode == "augmented" else execute_input_fused
        return run(prepared, cfg, fault, context, method=method, policy=policy, profile_scope=profile_scope)
    return _run_reference(plan, seams, profile_scope)


def _run_reference(plan, seams, profile_scope):
    """The Python implementation: evidence through the seams (or the native
    collectors), decisions through the method's hooks."""
    prepared, cfg, fault, method = plan.prepared, plan.cfg, plan.fault, plan.method
    device = prepared.a.device
    algorithm = plan.policy.algorithm if plan.policy is not None else 0
    augmented = cfg.reference_mode == "augmented"
    fused_reference = cfg.reference_mode in {"input_fused", "augmented"}
    timer = _Timer(cfg.timing, device, profile_scope)
    started = time.perf_counter()
    if method is not None:
        method._profile_scope = timer.scope

    with timer.phase("reference"):
        if method is None:
            plan.state = None
        elif augmented:
            plan.state = method.prepare_augmented(prepared, cfg)
        elif fused_reference:
            plan.state = method.prepare_fused(prepared, cfg)
        else:
            plan.state = method.prepare(prepared, cfg, seams["reference_mm"])
    with timer.phase("fault_prepare"):
        input_fault = plan.selected and fault.location in {"a", "b"}
        active = prepared.injected(fault) if input_fault else prepared
        injection = _injection(prepared, fault, plan.selected)
    weights = plan.state["weights"] if plan.state else torch.zeros((2, prepared.m), device=device,
                                                                    dtype=torch.float32)

    def observe(operands, injected):
        """(output, observed partials, hit) of the epilogue checksums."""
        if seams["collector_fn"] is not None:
            return seams["collector_fn"](operands, weights, injected)
        return operands.collected_native(weights, injected, algorithm=algorithm)

    def observe_with_reference(operands, injected):
        """(output, observed, hit, predicted, magnitude) of the input-fused GEMM."""
        if seams["reference_collector_fn"] is not None:
            return seams["reference_collector_fn"](operands, weights, injected)
        if augmented:
            return operands.augmented_native(weights, injected, algorithm=algorithm)
        return operands.collected_reference_native(weights, injected, algorithm=algorithm,
                                                   layout=cfg.reference_layout)

    instrumented = method is not None or injection[0] >= 0
    with timer.phase("execute"):
        if fused_reference:
            output, partials, hit, predicted, magnitude = observe_with_reference(active, injection)
        elif instrumented:
            output, partials, hit = observe(active, injection)
        else:
            output = seams["raw_fn"](active) if seams["raw_fn"] else active.raw_native()
            hit = torch.zeros(1, device=device, dtype=torch.int32)
        if input_fault:
            hit = torch.ones(1, device=device, dtype=torch.int32)
    with timer.phase("verify"):
        if fused_reference:
            with timer.scope("abft.merge_reference"):
                plan.state = method.bind_reference(predicted, magnitude, plan.state)
        if method is not None:
            with timer.scope("abft.merge_observed"):
                observed = method.propagate(partials, plan.state)
            with timer.scope("abft.method_verify"):
                tensors = method.verify(observed, output, plan.state, cfg)
        else:
            no = torch.zeros((), device=device, dtype=torch.bool)
            tensors = {"detected": no, "nonfinite": (~torch.isfinite(output)).any(), "located": no,
                       "location": torch.full((2,), -1, device=device, dtype=torch.int64)}
        with timer.scope("abft.report_flags"):
            tensors.update(fault_hit=hit, recovered=torch.zeros((), device=device, dtype=torch.bool),
                           recheck_failed=torch.zeros((), device=device, dtype=torch.bool))
    report = AbftReport(tensors, call_context(prepared, cfg, fault, plan.context, plan.selected, output, method),
                        cfg.method, "instrumented" if instrumented else "raw", timer.events)

    def recheck():
        # The clean operands again; the first reference stays the judge.
        if fused_reference:
            replacement, retry_partials, _, _, _ = observe_with_reference(prepared, NO_FAULT)
        elif seams["collector_fn"] is None:
            replacement, retry_partials, _ = method.recover(prepared, plan.state)
        else:
            replacement, retry_partials, _ = observe(prepared, NO_FAULT)
        return replacement, method.verify(method.propagate(retry_partials, plan.state), replacement, plan.state,
                                          cfg)

    return _finish(plan, report, output, recheck, timer, started)
