"""GPU tests of the ABFT engine mirror on the native sm_100a path.

``execute(..., implementation="native")`` must give the unprotected GEMM's
output bit for bit when clean, detect an accumulator fault, locate it with
``locate=True`` and repair it (``recovery="recompute"``: bit-exact clean
output; ``"correct"``: the located element recomputed). The Python
``reference`` implementation fed by the same native collectors must reach the
same decisions.
"""
import pytest
import torch

import sdc_b200
from sdc_b200.abft import execute, execute_prepared
from sdc_b200.abft.engine import AbftError
from sdc_b200.abft.methods import get_method
from sdc_b200.abft.operands import PreparedGemm
from sdc_b200.gemm import backend

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
SCALING = {"fp8": "tensorwise", "nvfp4": "block16"}


def _operands(m, n, k, seed=5):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return torch.randn(m, k, device=DEV, generator=g), torch.randn(k, n, device=DEV, generator=g)


def _cfg(**changes):
    return {"method": "classic", "implementation": "native", "reference_mode": "input_fused",
            "on_error": "report", "atol": 1e-3, "rtol": 1e-4, "diagnostics": True, **changes}


def _fault_near(clean, row, col):
    """The first output element at or after (row, col) (row-major order)
    with 4 <= |v| < 256, and exponent bit 27: those values have exponent bits
    26..29 clear, so the flip scales the element by 2^16 and the checksum
    change is large, finite and locatable."""
    values = clean.float().reshape(-1)
    start = row * clean.shape[1] + col
    ok = (values[start:].abs() >= 4) & (values[start:].abs() < 256)
    index = start + int(ok.nonzero()[0, 0])
    return index // clean.shape[1], index % clean.shape[1], 27


@pytest.mark.parametrize("precision", ["fp8", "nvfp4"])
@pytest.mark.parametrize("layout", ["tile", "kslice"])
def test_native_clean_output_is_the_unprotected_gemm(precision, layout):
    a, b = _operands(384, 520, 512)
    plain = backend.gemm(a, b, precision, SCALING[precision])
    output, report = execute(a, b, precision, SCALING[precision], abft_config=_cfg(reference_layout=layout))
    assert torch.equal(output, plain)
    assert not report.detected and not report.nonfinite
    assert report.execution_path == "input_fused_native"
    record = report.to_record()
    assert record["context"]["reference_layout"] == layout and record["fault_hit"] == [0]


@pytest.mark.parametrize("precision", ["fp8", "nvfp4"])
@pytest.mark.parametrize("recovery", ["recompute", "correct"])
def test_native_fault_detected_located_and_repaired(precision, recovery):
    m, n, k = 520, 384, 512
    a, b = _operands(m, n, k, seed=9)
    prepared = PreparedGemm.prepare(a, b, precision, SCALING[precision])
    clean = prepared.raw_native()
    row, col, bit = _fault_near(clean, 389, 201)
    fault = {"location": "accumulator", "row": row, "col": col, "bit": bit}
    output, report = execute_prepared(prepared, _cfg(locate=True, recovery=recovery, reference_layout="kslice"),
                                      fault)
    assert report.detected and report.fault_hit.item() == 1
    assert report.located and report.location.tolist() == [row, col]
    assert report.recovered and not report.recheck_failed
    if recovery == "recompute":
        assert torch.equal(output, clean)
        assert report.context["recovery_action"] == "full_recompute"
    else:
        assert report.context["recovery_action"] == "located_element_recomputed"
        torch.testing.assert_close(output.float(), clean.float(), rtol=1e-2, atol=1e-3)


@pytest.mark.parametrize("precision", ["fp8", "nvfp4"])
def test_native_unrecovered_fault_raises(precision):
    a, b = _operands(256, 256, 256, seed=3)
    prepared = PreparedGemm.prepare(a, b, precision, SCALING[precision])
    row, col, bit = _fault_near(prepared.raw_native(), 17, 33)
    with pytest.raises(AbftError) as error:
        execute_prepared(prepared, _cfg(on_error="raise"),
                         {"location": "accumulator", "row": row, "col": col, "bit": bit})
    assert error.value.report.detected and not error.value.report.recovered


@pytest.mark.parametrize("precision", ["fp8", "nvfp4"])
def test_native_sum_policy_detects_without_location(precision):
    a, b = _operands(256, 320, 256, seed=4)
    prepared = PreparedGemm.prepare(a, b, precision, SCALING[precision])
    row, col, bit = _fault_near(prepared.raw_native(), 5, 6)
    _, report = execute_prepared(prepared, _cfg(method="sum", locate=True),
                                 {"location": "accumulator", "row": row, "col": col, "bit": bit})
    assert report.detected and not report.located and report.location.tolist() == [-1, -1]
    assert report.context["compiled_policy"]["id"] == 1


@pytest.mark.parametrize("precision", ["fp8", "nvfp4"])
def test_python_reference_implementation_agrees_with_native(precision):
    a, b = _operands(264, 272, 288, seed=11)
    prepared = PreparedGemm.prepare(a, b, precision, SCALING[precision])
    row, col, bit = _fault_near(prepared.raw_native(), 100, 200)
    fault = {"location": "accumulator", "row": row, "col": col, "bit": bit}
    for layout in ("tile", "kslice"):
        native_out, native = execute_prepared(prepared, _cfg(locate=True, reference_layout=layout), fault)
        python_out, python = execute_prepared(prepared, _cfg(implementation="reference", reference_layout=layout),
                                              fault)
        assert torch.equal(native_out, python_out)
        assert bool(native.detected) == bool(python.detected) is True
        assert native.location.tolist() == python.location.tolist() == [row, col]
        # Totals are summed in a different order (serial vs torch.sum): equal
        # up to rounding, far below the detection threshold, off the faulty column.
        clean_cols = torch.arange(prepared.n, device=DEV) != col
        diff = (native.residual - python.residual).abs()[:, clean_cols]
        assert (diff <= native.threshold[:, clean_cols]).all()


def test_native_weights_are_cached_per_stream():
    from sdc_b200.abft import native

    a, b = _operands(128, 128, 128)
    prepared = PreparedGemm.prepare(a, b, "fp8", "tensorwise")
    execute_prepared(prepared, _cfg())
    key = (0, torch.device(DEV).index or 0, 128, torch.float32)
    first = native.WEIGHTS.peek(key)
    execute_prepared(prepared, _cfg())
    assert first is not None and native.WEIGHTS.peek(key) is first
    assert torch.equal(first, get_method("classic").projection_weights(prepared))


def test_timing_events_are_reported():
    a, b = _operands(256, 256, 256)
    _, report = execute(a, b, "fp8", "tensorwise", abft_config=_cfg(timing=True, locate=True))
    timing = report.to_record()["timing_ms"]
    assert {"reference", "execute", "finalize", "locate"} <= set(timing)
    assert all(value >= 0 for value in timing.values())
    assert sdc_b200.LIB_PATH.exists()


def test_stage_profile_of_a_native_call():
    """profile_prepared: every native stage appears with one sample per
    repeat, the GEMM kernels account for most of abft.execute, and the clean
    protected output equals the unprotected GEMM's."""
    from sdc_b200.abft.profiling import profile_prepared

    a, b = _operands(512, 512, 512, seed=12)
    prepared = PreparedGemm.prepare(a, b, "fp8", "tensorwise")
    result = profile_prepared(prepared, _cfg(reference_layout="kslice"), warmup=2, repeats=4)
    rows = {row["stage"]: row for row in result["stages"]}
    for stage in ("baseline.gemm", "abft.reference", "abft.execute", "abft.finalize", "abft.total"):
        assert stage in rows and len(rows[stage]["gpu_active_ms"]["samples"]) == 4 * rows[stage]["calls_per_repeat"]
    assert rows["abft.execute"]["gemm_kernel_ms"]["median"] > 0
    assert rows["baseline.gemm"]["gemm_kernel_ms"]["median"] > 0
    assert result["last_output_comparison"]["bit_identical"]
    assert result["last_report"]["detected"] in (False, [False])
