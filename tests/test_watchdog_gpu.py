"""An expired bounded wait is reported in-band, never as a clean result.

Every wait in the GEMM kernels gives up after a time limit and unwinds. The
test hook ``sdc_test_set_watchdog`` shortens that limit to 1 ms and makes the
prediction warps' pacing target unreachable (a flag that nothing sets; the
in-GEMM prediction path is forced with ``sdc_test_set_kslice_path``), so
the wait runs out on purpose; nothing faults or hangs the GPU. The launch
must then report itself through its own outputs: bit 1 of ``hit``, the
non-finite flag, and finalize's verdict detected + nonfinite, plus the
watchdog code for the host. A normal call afterwards is clean and equal to
the call before.
"""
import ctypes

import pytest
import torch

import sdc_b200  # noqa: F401  (registers torch.ops.sdc_cutlass)
from sdc_b200 import capi
from sdc_b200.gemm.quantization import quantize, quantize_blockwise

pytestmark = pytest.mark.gpu
ops = torch.ops.sdc_cutlass
DEV = "cuda"
WAIT_PACE = 8  # watchdog code of the prediction warps' pacing wait


def _watchdog():
    code = ctypes.c_int32(-1)
    capi.check(capi.lib().sdc_read_device_error(torch.cuda.current_stream().cuda_stream, ctypes.byref(code)))
    return code.value


def _call(kind, m, n, k):
    g = torch.Generator(device=DEV).manual_seed(m + n + k)
    a = torch.randn(m, k, device=DEV, generator=g)
    b = torch.randn(n, k, device=DEV, generator=g)
    weights = torch.stack((torch.ones(m, device=DEV), torch.arange(1, m + 1, device=DEV, dtype=torch.float32)))
    if kind == "fp8_block":
        qa, qb = quantize_blockwise(a, 1), quantize_blockwise(b, 128)
        args = (qa.codes.view(torch.float8_e4m3fn), qb.codes.view(torch.float8_e4m3fn), qa.scales, qb.scales)
        fused, extra = ops.abft_fp8_block_reference_mm, ()
    else:
        qa, qb = quantize(a, kind), quantize(b, kind)
        alpha = (qa.multiplier * qb.multiplier).reciprocal()
        if kind == "fp8":
            args = (qa.codes.view(torch.float8_e4m3fn), qb.codes.view(torch.float8_e4m3fn), alpha)
            fused = ops.abft_fp8_reference_mm
        else:
            args = (qa.codes, qb.codes, qa.scales_mma, qb.scales_mma, k, alpha)
            fused = ops.abft_nvfp4_reference_mm
        extra = (1,)  # the K-slice layout: prediction warps inside the GEMM

    def run():
        nonfinite = torch.zeros(1, dtype=torch.int32, device=DEV)
        out, obs, hit, pred, mag = fused(*args, weights, -1, -1, -1, 0, nonfinite, *extra)
        packet = ops.abft_finalize_reference(obs, pred, mag, hit, nonfinite, n, 1e-3, 1e-4, None, True)
        torch.cuda.synchronize()
        return out, hit.item(), nonfinite.item(), packet[3].tolist(), packet[4].item()

    return run


# A single CTA (M <= 128) and CTA pairs, all three GEMM kinds.
@pytest.mark.parametrize("kind,shape", [("fp8", (128, 512, 1024)), ("fp8_block", (1024, 1024, 1024)),
                                        ("nvfp4", (512, 768, 512))])
def test_expired_wait_is_reported_in_band(kind, shape):
    run = _call(kind, *shape)
    assert _watchdog() == 0
    # The pacing wait belongs to the in-GEMM prediction path (these short M
    # would otherwise run the standalone K-slice kernels, which never wait).
    capi.check(capi.lib().sdc_test_set_kslice_path(1))
    try:
        _expire_and_recover(run)
    finally:
        capi.check(capi.lib().sdc_test_set_kslice_path(0))


def _expire_and_recover(run):
    clean, hit, nonfinite, flags, hit_out = run()
    assert hit == 0 and nonfinite == 0 and flags == [False] * 5
    try:
        capi.check(capi.lib().sdc_test_set_watchdog(1_000_000, 1 << 20))
        _, hit, nonfinite, flags, hit_out = run()
    finally:
        capi.check(capi.lib().sdc_test_set_watchdog(0, 0))
    assert hit & 2, "the aborted launch must mark hit bit 1"
    assert nonfinite == 1
    assert flags[0] and flags[1], "finalize must report an aborted launch as detected and nonfinite"
    assert hit_out == 0  # no fault was injected
    assert _watchdog() == WAIT_PACE
    again, hit, nonfinite, flags, _ = run()
    assert hit == 0 and nonfinite == 0 and flags == [False] * 5
    assert torch.equal(again, clean)
    assert _watchdog() == 0

