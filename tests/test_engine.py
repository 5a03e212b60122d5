"""CPU contract tests of the ABFT engine mirror (sdc_b200.abft).

The engine's reference implementation runs on the CPU through the same
dependency-injection seams the reference's own tests use
(tests/abft/test_framework.py:14-26): an fp32 collector computing C = A @ B,
one XOR'd fp32 bit and the W @ C partials. Decisions are checked against the
reference engine's recorded outcomes (golden/engine_cases.json,
golden/config1_trials.json, made by golden/make_golden.py).
"""
import json
import math
from pathlib import Path
from types import SimpleNamespace

import pytest
import torch

from sdc_b200.abft import AbftConfig, FaultConfig, execute, execute_prepared, parse_abft_config
from sdc_b200.abft import engine, methods
from sdc_b200.abft.engine import AbftError, _selected
from sdc_b200.abft.methods import Classic, CompiledPolicy, Sum, get_method, register_method
from sdc_b200.abft.operands import PreparedGemm

GOLDEN = Path(__file__).parent / "golden"


def collect(operands, weights, fault):
    a, b = operands.decode_block(0, operands.k)
    output = a @ b
    row, col, bit = fault
    if row >= 0:
        output.view(torch.int32)[row, col] ^= (1 << bit) if bit < 31 else -(1 << 31)
    return output, (weights @ output).unsqueeze(1), torch.tensor([int(row >= 0)])


def run(a, b, **kwargs):
    return execute(a, b, "fp32", "none", reference_mm=torch.mm, collector_fn=collect, **kwargs)


# --- golden outcomes of the reference engine ---------------------------------

def test_engine_reproduces_reference_engine_cases():
    for case in json.loads((GOLDEN / "engine_cases.json").read_text()):
        g = torch.Generator().manual_seed(case["seed"])
        a = torch.randn(64, 80, generator=g)
        b = torch.randn(80, 96, generator=g)
        cfg = {"method": "classic", "atol": 1e-4, "rtol": 1e-4, "diagnostics": True, "on_error": "report",
               "reference_block_k": 32, "recovery": "recompute"}
        _, report = run(a, b, abft_config=cfg, fault_config=case["fault"])
        rec = report.to_record()
        assert (bool(rec["detected"]), bool(rec["located"]), rec["location"], bool(rec["recovered"])) == (
            case["detected"], case["located"], case["location"], case["recovered"]), case["seed"]


def test_engine_reproduces_config1_golden_trials():
    data = json.loads((GOLDEN / "config1_trials.json").read_text())
    g = torch.Generator().manual_seed(data["seed"])
    a = torch.rand(1024, 1024, generator=g) * 2 - 1
    b = torch.rand(1024, 1024, generator=g) * 2 - 1
    cfg = {"method": "classic", "atol": data["atol"], "rtol": data["rtol"], "diagnostics": True,
           "on_error": "report"}
    prepared = PreparedGemm.prepare(a, b, "fp32", "none")
    picked = data["trials"][:3] + data["trials"][50:62]
    for trial in picked:
        _, report = execute_prepared(prepared, cfg, trial["fault"], reference_mm=torch.mm, collector_fn=collect)
        rec = report.to_record()
        assert bool(rec["detected"]) == trial["detected"]
        assert bool(rec["located"]) == trial["located"]
        assert rec["location"] == trial["location"]
        ratio = float((report.residual.abs() / report.threshold).max())
        assert ratio == pytest.approx(trial["max_ratio"], rel=1e-6)


# --- operands -------------------------------------------------------------------

@pytest.mark.parametrize("precision,bit", [("fp32", 31), ("bf16", 15)])
@pytest.mark.parametrize("location", ["a", "b"])
def test_input_fault_copies_and_leaves_clean_operands(precision, bit, location):
    a, b = torch.ones(3, 16), torch.ones(16, 2)
    prepared = PreparedGemm.prepare(a, b, precision, "none")
    faulty = prepared.injected(FaultConfig(location=location, row=0, col=0, bit=bit))
    assert getattr(faulty, location)[0, 0] == -1 and getattr(prepared, location)[0, 0] == 1
    other = "b" if location == "a" else "a"
    assert getattr(faulty, other) is getattr(prepared, other)


def _nvfp4_operands():
    # 0x22 = two e2m1 codes of 1.0; block scales 2 and 4; multiplier 2.
    def meta(rows):
        return SimpleNamespace(scales=torch.tensor([[2., 4.]] * rows).to(torch.float8_e4m3fn).view(torch.uint8),
                               multiplier=torch.tensor(2.))
    a = torch.full((3, 16), 0x22, dtype=torch.uint8)
    b = torch.full((2, 16), 0x22, dtype=torch.uint8)
    return PreparedGemm(a, b, "nvfp4", 3, 2, 32, meta(3), meta(2))


@pytest.mark.parametrize("col,expected", [(0, 0x23), (1, 0x32)])
def test_nvfp4_fault_flips_one_nibble(col, expected):
    clean = _nvfp4_operands()
    assert clean.injected(FaultConfig(location="a", col=col, bit=0)).a[0, 0] == expected
    assert clean.injected(FaultConfig(location="b", row=col, col=1, bit=0)).b[1, 0] == expected
    assert clean.a[0, 0] == 0x22 and clean.b[1, 0] == 0x22


def test_nvfp4_decode_applies_block_scales_and_b_orientation():
    prepared = _nvfp4_operands()
    a, b = prepared.decode_block(0, 32)
    assert torch.equal(a[:, :16], torch.ones(3, 16)) and torch.equal(a[:, 16:], torch.full((3, 16), 2.))
    assert b.shape == (32, 2)
    state = Classic().prepare(prepared, AbftConfig(reference_block_k=16), torch.mm)
    assert torch.equal(state["expected"], state["weights"] @ (a @ b))
    with pytest.raises(ValueError, match="block16"):
        prepared.decode_block(1, 17)


def test_separate_reference_is_chunked(monkeypatch):
    torch.manual_seed(3)
    prepared = PreparedGemm.prepare(torch.randn(4, 48), torch.randn(48, 3), "bf16", "none")
    calls = []
    decode = prepared.decode_block
    monkeypatch.setattr(prepared, "decode_block", lambda s, e: calls.append((s, e)) or decode(s, e))
    state = Classic().prepare(prepared, AbftConfig(reference_block_k=16), torch.mm)
    assert calls == [(0, 16), (16, 32), (32, 48)]
    torch.testing.assert_close(state["expected"], state["weights"] @ (prepared.a.float() @ prepared.b.float()))


# --- decisions ------------------------------------------------------------------

def test_accumulator_fault_detected_and_located():
    _, report = run(torch.ones(3, 16), torch.ones(16, 2), abft_config={"method": "classic", "on_error": "report"},
                    fault_config={"location": "accumulator", "row": 1, "col": 0, "bit": 31})
    assert report.detected and report.located
    assert report.location.tolist() == [1, 0]
    assert report.to_record()["fault_hit"] == [1]


def test_fault_only_run_uses_fp32_zero_weights():
    prepared = PreparedGemm.prepare(torch.ones(3, 16), torch.ones(16, 2), "fp32", "none")

    def collector(operands, weights, fault):
        assert weights.dtype == torch.float32 and not weights.any()
        return collect(operands, weights, fault)

    output, report = execute_prepared(prepared, "none", {"location": "accumulator", "row": 1, "col": 0, "bit": 31},
                                      collector_fn=collector)
    expected = torch.full((3, 2), 16.)
    expected[1, 0] = -16.
    assert torch.equal(output, expected)
    assert report.context["fault_selected"] and not report.detected


@pytest.mark.parametrize("value", [math.nan, math.inf, -math.inf])
def test_nonfinite_is_detected_and_never_located(value):
    method = Classic()
    prepared = PreparedGemm.prepare(torch.ones(3, 16), torch.ones(16, 2), "fp32", "none")
    cfg = AbftConfig()
    state = method.prepare(prepared, cfg, torch.mm)
    output = prepared.a @ prepared.b
    output[1, 0] = value
    result = method.verify(state["weights"] @ output, output, state, cfg)
    assert result["detected"] and result["nonfinite"] and not result["located"]


def test_inconsistent_ratio_is_not_located():
    method = Classic()
    prepared = PreparedGemm.prepare(torch.ones(3, 16), torch.ones(16, 2), "fp32", "none")
    cfg = AbftConfig(atol=0.4, rtol=0.)
    state = method.prepare(prepared, cfg, torch.mm)
    observed = state["expected"].clone()
    observed[:, 0] += torch.tensor([1., 2.])
    result = method.verify(observed, prepared.a @ prepared.b, state, cfg)
    assert result["detected"] and not result["located"]


def test_recovery_recomputes_from_clean_operands(monkeypatch):
    prepared_calls = []
    original = PreparedGemm.prepare.__func__
    monkeypatch.setattr(PreparedGemm, "prepare",
                        classmethod(lambda cls, *args: prepared_calls.append(1) or original(cls, *args)))
    a, b = torch.ones(3, 16), torch.ones(16, 2)
    output, report = run(a, b, abft_config={"method": "classic", "recovery": "recompute"},
                         fault_config={"location": "a", "bit": 31})
    assert len(prepared_calls) == 1
    assert report.detected and report.recovered and not report.recheck_failed
    assert torch.equal(output, a @ b)


def test_failed_recheck_raises_with_report():
    def broken(operands, weights, fault):
        output, partials, hit = collect(operands, weights, fault)
        return output, partials + 100, hit

    with pytest.raises(AbftError) as error:
        execute(torch.ones(3, 16), torch.ones(16, 2), "fp32", "none",
                abft_config={"method": "classic", "recovery": "recompute"}, reference_mm=torch.mm,
                collector_fn=broken)
    assert error.value.report.recheck_failed and not error.value.report.recovered


def test_disabled_method_calls_plain_backend_without_preparing(monkeypatch):
    sentinel = torch.ones(1)
    monkeypatch.setattr(engine.backend, "gemm", lambda *args: sentinel)
    monkeypatch.setattr(PreparedGemm, "prepare", lambda *args: pytest.fail("prepared"))
    output, report = execute(torch.ones(3, 16), torch.ones(16, 2), "fp32", "none")
    assert output is sentinel and report is None


def test_report_policy_takes_no_host_sync(monkeypatch):
    monkeypatch.setattr(torch.Tensor, "item", lambda *args: pytest.fail("implicit sync"))
    _, report = run(torch.ones(3, 16), torch.ones(16, 2), abft_config={"method": "classic", "on_error": "report"})
    assert report.method == "classic" and report.execution_path == "instrumented"


def test_registered_plugin_method_runs(monkeypatch):
    monkeypatch.setattr(methods, "_METHODS", dict(methods._METHODS))

    class Plugin(Classic):
        def verify(self, *args):
            return {**super().verify(*args), "plugin_used": torch.tensor(True)}

    register_method("test_plugin", Plugin)
    _, report = run(torch.ones(3, 16), torch.ones(16, 2), abft_config="test_plugin")
    assert report.plugin_used
    with pytest.raises(ValueError, match="duplicate"):
        register_method("test_plugin", Plugin)


@pytest.mark.parametrize("context,fires", [
    ({}, True), ({"call_index": 2}, False), ({"retry": True}, False),
    ({"layer": "mlp"}, True), ({"layer": "attn"}, False), ({"role": "dgrad"}, False)])
def test_fault_fires_only_on_its_call_layer_and_role(context, fires):
    fault = FaultConfig(location="accumulator", layer=None if "layer" not in context else "mlp", role="forward")
    full = {"call_index": 1, "role": "forward", **context}
    assert _selected(fault, full) == fires


def test_record_is_strict_json_with_nonfinite_paths():
    def nan_collector(operands, weights, fault):
        output, partials, hit = collect(operands, weights, fault)
        output[0, 0] = math.nan
        return output, weights @ output, hit

    _, report = execute(torch.ones(3, 16), torch.ones(16, 2), "fp32", "none",
                        abft_config={"method": "classic", "on_error": "report", "diagnostics": True},
                        reference_mm=torch.mm, collector_fn=lambda o, w, f: (lambda r: (r[0], r[1].unsqueeze(1),
                                                                                         r[2]))(nan_collector(o, w, f)))
    record = report.to_record()
    json.dumps(record, allow_nan=False)
    assert record["nonfinite"] and any(key.startswith("residual") for key in record["nonfinite_metrics"])


@pytest.mark.parametrize("diagnostics", [False, True])
def test_diagnostics_and_precision_metadata(diagnostics):
    _, report = run(torch.ones(3, 16), torch.ones(16, 2),
                    abft_config={"method": "classic", "diagnostics": diagnostics})
    assert ("residual" in report.tensors) == diagnostics
    assert report.context["precision"] == "fp32" and report.context["accumulator_precision"] == "fp32"
    assert report.context["reference_algorithm"] == "separate_projection_arithmetic"


# --- input_fused through the reference seams -------------------------------------

def _fused_collector(corrupt_predicted=0.0, calls=None):
    def collector(operands, weights, fault):
        if calls is not None:
            calls.append(fault)
        output, observed, hit = collect(operands, weights, fault)
        a, b = operands.decode_block(0, operands.k)
        predicted = (weights @ a @ b).unsqueeze(1) + corrupt_predicted
        magnitude = (weights.abs() @ a.abs() @ b.abs()).unsqueeze(1)
        return output, observed, hit, predicted, magnitude
    return collector


def test_input_fused_reference_controls_verification():
    a, b = torch.ones(3, 16), torch.ones(16, 2)
    cfg = {"method": "classic", "reference_mode": "input_fused", "on_error": "report"}
    _, clean = execute(a, b, "fp32", "none", abft_config=cfg, reference_collector_fn=_fused_collector())
    _, shifted = execute(a, b, "fp32", "none", abft_config=cfg, reference_collector_fn=_fused_collector(1.0))
    assert not clean.detected and shifted.detected
    assert clean.context["reference_algorithm"] == "input_fused_fp32_projection"


def test_input_fused_retry_reuses_first_reference():
    calls = []
    a, b = torch.ones(3, 16), torch.ones(16, 2)
    cfg = {"method": "classic", "reference_mode": "input_fused", "recovery": "recompute"}
    output, report = execute(a, b, "fp32", "none", abft_config=cfg,
                             fault_config={"location": "accumulator", "row": 2, "col": 1, "bit": 30},
                             reference_collector_fn=_fused_collector(calls=calls))
    assert calls == [(2, 1, 30), (-1, -1, -1)]
    assert report.detected and report.recovered and torch.equal(output, a @ b)


@pytest.mark.parametrize("location", ["a", "b"])
def test_input_fused_rejects_input_memory_faults(location):
    with pytest.raises(ValueError, match="computation only"):
        execute(torch.ones(3, 16), torch.ones(16, 2), "fp32", "none",
                abft_config={"method": "classic", "reference_mode": "input_fused"},
                fault_config={"location": location}, reference_collector_fn=_fused_collector())


def test_input_fused_needs_fp8_or_nvfp4_without_a_collector():
    with pytest.raises(NotImplementedError, match="input_fused reference is not implemented for fp32"):
        execute(torch.ones(3, 16), torch.ones(16, 2), "fp32", "none",
                abft_config={"method": "classic", "reference_mode": "input_fused"})


# --- methods and policies ----------------------------------------------------------

@pytest.mark.parametrize("algorithm,channels", [(0, 1), (1, 2), (2, 1), (True, 2), (0.0, 2)])
def test_compiled_policy_requires_an_installed_pair(algorithm, channels):
    with pytest.raises(ValueError, match="installed CUDA"):
        CompiledPolicy(algorithm, channels)


def test_sum_detects_without_locating():
    method = get_method("sum")
    assert isinstance(method, Sum) and method.compiled_policy == CompiledPolicy(1, 1)
    _, report = run(torch.ones(3, 16), torch.ones(16, 2), abft_config={"method": "sum", "on_error": "report"},
                    fault_config={"location": "accumulator", "row": 1, "col": 0, "bit": 31})
    assert report.detected and not report.located and report.location.tolist() == [-1, -1]


@pytest.mark.parametrize("name", ["classic", "sum"])
def test_methods_reject_parameters(name):
    with pytest.raises(ValueError, match="does not accept method parameters"):
        run(torch.ones(3, 16), torch.ones(16, 2), abft_config={"method": name, "parameters": {"x": 1}})


def test_subclass_must_opt_in_to_a_native_policy(monkeypatch):
    monkeypatch.setattr(methods, "_METHODS", dict(methods._METHODS))

    class Custom(Classic):
        def verify(self, *args):
            return super().verify(*args)

    register_method("custom", Custom)
    prepared = PreparedGemm.prepare(torch.ones(3, 16), torch.ones(16, 2), "fp32", "none")
    cfg = parse_abft_config({"method": "custom", "implementation": "native", "reference_mode": "input_fused"})
    with pytest.raises(ValueError, match="no explicit compiled CUDA policy"):
        get_method("custom").validate_execution(prepared, cfg)


def test_method_instance_must_match_configuration():
    with pytest.raises(ValueError, match="does not match"):
        run(torch.ones(3, 16), torch.ones(16, 2), abft_config="classic", method_instance=get_method("sum"))
    with pytest.raises(ValueError, match="requires an enabled"):
        run(torch.ones(3, 16), torch.ones(16, 2), method_instance=get_method("classic"))


def test_stateful_method_needs_a_retained_instance(monkeypatch):
    monkeypatch.setattr(methods, "_METHODS", dict(methods._METHODS))

    class Adaptive(Classic):
        stateful = True

    register_method("adaptive", Adaptive)
    with pytest.raises(ValueError, match="retained method_instance"):
        run(torch.ones(3, 16), torch.ones(16, 2), abft_config="adaptive")
    _, report = run(torch.ones(3, 16), torch.ones(16, 2), abft_config="adaptive",
                    method_instance=get_method("adaptive"))
    assert not report.detected


def test_commit_sees_decisions_once_after_retry(monkeypatch):
    monkeypatch.setattr(methods, "_METHODS", dict(methods._METHODS))
    commits = []

    class Recording(Classic):
        def commit(self, state, decision, context):
            commits.append((sorted(decision), context["precision"]))

    register_method("recording", Recording)
    run(torch.ones(3, 16), torch.ones(16, 2), abft_config={"method": "recording", "recovery": "recompute"},
        fault_config={"location": "accumulator", "row": 0, "col": 1, "bit": 30})
    assert len(commits) == 1 and "recovered" in commits[0][0] and commits[0][1] == "fp32"


def test_native_rejects_collector_overrides():
    codes = torch.zeros((3, 16), dtype=torch.uint8)
    prepared = PreparedGemm(codes, codes[:2], "fp8", 3, 2, 16)
    with pytest.raises(ValueError, match="does not accept reference collector overrides"):
        execute_prepared(prepared, {"method": "classic", "implementation": "native",
                                    "reference_mode": "input_fused"}, collector_fn=collect)


# --- configuration -------------------------------------------------------------------

@pytest.mark.parametrize("value", [
    {"method": "classic", "atol": -1}, {"method": "classic", "rtol": math.inf}, {"method": "classic", "atol": True},
    {"method": "classic", "recovery": "retry"}, {"method": "classic", "on_error": "ignore"},
    {"method": "classic", "reference_block_k": 8}, {"method": "classic", "timing": 1},
    {"method": "classic", "reference_mode": "other"}, {"method": "none", "reference_mode": "input_fused"},
    {"method": "classic", "reference_mode": "augmented"}, {"method": "none", "implementation": "native"},
    {"method": "classic", "unknown": 1}, {"method": "classic", "parameters": {"x": math.nan}},
    {"method": "classic", "parameters": {1: 2}}, {"method": "classic", "reference_layout": "rows"},
    {"method": "classic", "locate": "yes"}, {"method": ""}, {"method": "classic", "row_checksums": 1},
    {"method": "classic", "row_checksums": True},
    {"method": "classic", "row_checksums": True, "implementation": "native", "reference_mode": "direct"}])
def test_invalid_configurations_rejected(value):
    with pytest.raises(ValueError):
        parse_abft_config(value)


def test_configuration_defaults_and_extensions():
    cfg = parse_abft_config("classic")
    assert (cfg.atol, cfg.rtol, cfg.recovery, cfg.on_error, cfg.reference_block_k) == (1e-4, 1e-4, "none", "raise", 256)
    assert (cfg.reference_layout, cfg.locate) == ("tile", False)
    assert parse_abft_config({"method": "classic", "recovery": "correct", "locate": True,
                              "reference_layout": "kslice"}).recovery == "correct"
    assert AbftConfig().parameters is not AbftConfig().parameters
    rows = parse_abft_config({"method": "sum", "implementation": "native", "reference_mode": "input_fused",
                              "row_checksums": True})
    assert rows.row_checksums and not cfg.row_checksums


def test_profile_summary_per_stage():
    """summarize_profile: stage statistics from CPU scope events, the GEMM
    kernels' share (own and child scopes), and a loud error when a stage the
    path must run is missing a sample."""
    from types import SimpleNamespace

    from sdc_b200.abft import profiling

    cpu = SimpleNamespace(name="CPU")

    def scope(name, device_us, cpu_us, kernels=(), children=()):
        return SimpleNamespace(name=name, device_type=cpu, device_time_total=device_us, cpu_time_total=cpu_us,
                               kernels=[SimpleNamespace(name=k, duration=d) for k, d in kernels],
                               cpu_children=list(children))

    events = []
    for i in range(2):
        launch = scope("sdc_cutlass::abft_fp8_reference_mm", 50.0, 5.0, kernels=[("sdc::gemm_kernel<0,2>", 45.0)])
        events += [scope("baseline.gemm", 40.0 + i, 6.0, kernels=[("sdc::gemm_kernel<0,0>", 40.0 + i)]),
                   scope("abft.reference", 0.0, 2.0), scope("abft.execute", 55.0, 20.0, children=[launch]),
                   scope("abft.finalize", 9.0, 15.0), scope("abft.total", 64.0, 40.0),
                   SimpleNamespace(name="abft.total", device_type=SimpleNamespace(name="CUDA"))]
    result = profiling.summarize_profile(events, 2, input_fused=True, native=True)
    rows = {row["stage"]: row for row in result["stages"]}
    assert set(rows) == {"baseline.gemm", "abft.reference", "abft.execute", "abft.finalize", "abft.total"}
    assert rows["baseline.gemm"]["gpu_active_ms"]["samples"] == [0.040, 0.041]
    assert rows["abft.execute"]["gemm_kernel_ms"]["median"] == 0.045
    assert abs(rows["abft.execute"]["other_gpu_activity_ms"]["median"] - 0.010) < 1e-12
    assert rows["abft.finalize"]["cpu_scope_ms"]["median"] == 0.015
    with pytest.raises(RuntimeError, match="Incomplete profile: abft.finalize"):
        profiling.summarize_profile([e for e in events if e.name != "abft.finalize"], 2, input_fused=True,
                                    native=True)
