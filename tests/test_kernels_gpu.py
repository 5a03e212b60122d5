"""Parity of the sm_100a kernels with the CPU oracle (through the C ABI).

Bars: quantised codes/scales/multipliers, finalize packets, input-fused
checksum partials (TILE layout) and outputs on exactly representable data are
bit-exact; observed projections (tensor-core / reduction order unpinned in
the reference) match float64 within the reference tests' own tolerance
rtol 2e-5, atol 2e-3 (tests/cutlass_gemm/test_abft_gpu.py:61-68).
"""
import numpy as np
import pytest
import torch

import sdc_b200  # noqa: F401  (registers torch.ops.sdc_cutlass)
from oracle import abft as oabft
from oracle import formats, native, quant
from sdc_b200.gemm.quantization import quantize

pytestmark = pytest.mark.gpu
ops = torch.ops.sdc_cutlass
DEV = "cuda"


def _np(t):
    return t.detach().cpu().numpy()


# ------------------------------------------------------------- quantise ----

@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", [(1, 16), (7, 48), (160, 256), (257, 1040), (1024, 4096)])
@pytest.mark.parametrize("scale", ["amax", 3.0])
def test_quantize_bit_exact(dtype, shape, scale):
    g = torch.Generator(device=DEV).manual_seed(shape[0] * 31 + shape[1])
    x = (torch.randn(shape, device=DEV, generator=g) * 3).to(dtype)
    x[0, 0] = 50.0  # saturating values for a fixed scale
    ref_in = _np(x.float())
    q8 = quantize(x, "fp8", scale)
    codes, st = quant.quantize_fp8(ref_in, scale)
    assert np.array_equal(_np(q8.codes), codes) and _np(q8.multiplier) == st
    q4 = quantize(x, "nvfp4", scale)
    codes, scales, st = quant.quantize_nvfp4(ref_in, scale)
    assert np.array_equal(_np(q4.codes), codes)
    assert np.array_equal(_np(q4.scales), scales)
    assert _np(q4.multiplier) == st
    assert np.array_equal(_np(q4.scales_mma), quant.pack_scales(scales, shape[1]))


def test_quantize_known_answers_on_device():
    # tests/cutlass_gemm/test_low_precision_cuda.py:24-53 of the reference.
    values = torch.tensor([
        [0., .5, 1., 1.5, 2., 3., 4., 6., -0., -.5, -1., -1.5, -2., -3., -4., -6.],
        [0., .25, .75, 1.25, 1.75, 2.5, 3.5, 5., -0., -.25, -.75, -1.25, -1.75, -2.5, -3.5, -6.],
    ], device=DEV)
    expected = torch.tensor([[0x10, 0x32, 0x54, 0x76, 0x98, 0xBA, 0xDC, 0xFE],
                             [0x00, 0x22, 0x44, 0x66, 0x88, 0xAA, 0xCC, 0xFE]], dtype=torch.uint8, device=DEV)
    q = quantize(values, "nvfp4", 1.0)
    assert torch.equal(q.codes, expected)
    assert torch.equal(q.scales, torch.full((2, 1), 0x38, dtype=torch.uint8, device=DEV))
    assert torch.equal(quantize(-values, "nvfp4", 1.0).codes, expected ^ 0x88)
    zeros = quantize(torch.zeros(4, 64, device=DEV), "nvfp4")
    assert zeros.multiplier.item() == 1.0 and not zeros.codes.any() and not zeros.scales.any()
    blocks = torch.tensor([6., 12., 3., 0.], device=DEV).repeat_interleave(16).reshape(1, 64)
    scaled = quantize(blocks, "nvfp4")
    assert scaled.multiplier.item() == 224.0
    assert torch.equal(scaled.scales, torch.tensor([[0x76, 0x7E, 0x6E, 0]], dtype=torch.uint8, device=DEV))


def test_quantize_rejects_bad_input():
    with pytest.raises(ValueError, match="divisible by 16"):
        quantize(torch.ones(4, 8, device=DEV), "nvfp4")
    with pytest.raises(ValueError, match="positive"):
        quantize(torch.ones(4, 16, device=DEV), "fp8", -1.0)


# ------------------------------------------------------------- finalize ----

def _partials(tiles, n, channels=2, random=False, seed=529):
    padded = ((n + 127) // 128) * 128
    g = torch.Generator().manual_seed(seed)
    shape = (3, channels, tiles, padded)
    if random:
        p = torch.randn(shape, generator=g)
    else:
        p = torch.randint(-8, 9, shape, generator=g).float() / 8
        p[0].copy_(p[1])
    p[2].abs_()
    p[..., n:] = float("nan")
    return p


def _assert_packet(actual, expected):
    for a, e in zip(actual, expected, strict=True):
        a = _np(a)
        e = np.asarray(e)
        assert a.shape == e.shape, (a.shape, e.shape)
        if a.dtype == np.bool_:
            assert np.array_equal(a, e.astype(bool))
        else:
            assert np.array_equal(a.view(np.uint8), e.astype(a.dtype).view(np.uint8))


@pytest.mark.parametrize("algorithm,channels", [(0, 2), (1, 1)])
@pytest.mark.parametrize("tiles,n", [(1, 16), (3, 65), (17, 1024), (33, 257), (1, 8193), (9, 1025)])
def test_finalize_bit_exact_vs_serial_oracle(algorithm, channels, tiles, n):
    p = _partials(tiles, n, channels, random=True)
    p[0, 0, : min(3, tiles), 0] = torch.tensor([2.0 ** 24, 1, -(2.0 ** 24)])[: min(3, tiles)]
    pc = p.to(DEV)
    flags = torch.zeros(tiles, (n + 127) // 128, dtype=torch.int32, device=DEV)
    packed = ops.abft_finalize(pc, flags, n, 0.125, 0.25, None, True, algorithm)
    expected = oabft.finalize_serial(_np(p[0]), _np(p[1]), _np(p[2]), n, atol=0.125, rtol=0.25)
    _assert_packet(packed, expected)
    hit = torch.zeros(1, dtype=torch.int32, device=DEV)
    for pad in (64, 128):
        padded_n = ((n + pad - 1) // pad) * pad
        generic = ops.abft_finalize_reference(pc[0, ..., :padded_n].contiguous(), pc[1, ..., :padded_n].contiguous(),
                                              pc[2, ..., :padded_n].contiguous(), hit, hit.clone(), n, 0.125, 0.25,
                                              None, True, algorithm)
        _assert_packet(generic, expected)


def test_finalize_retry_reference_alias_thresholds_and_flags():
    n, tiles = 257, 33
    p = _partials(tiles, n).to(DEV)
    flags = torch.zeros(tiles, 3, dtype=torch.int32, device=DEV)
    first = ops.abft_finalize(p, flags, n, 0.0, 0.25, None, True)
    saved = first[0].clone()
    retry = p.clone()
    retry[0, 1, 0, n - 1] += 32
    retry[1].fill_(float("nan"))
    retry[2].fill_(float("inf"))
    out = ops.abft_finalize(retry, flags, n, 0.0, 0.25, first[0], True)
    assert out[0].data_ptr() == first[0].data_ptr() and torch.equal(first[0], saved)
    assert out[1][1, n - 1].item() == 32 and out[3].tolist() == [True, False, False, False, False]
    thr = torch.full((2, n), 8.0, device=DEV)
    thr[1, n - 1] = 0.5
    over = ops.abft_finalize(retry, flags, n, 1e12, 1e12, first[0], True, 0, thr)
    assert over[3][0].item() and torch.equal(over[2], thr)
    flags[-1, -1] = 3
    status = ops.abft_finalize(p, flags, n, 0.0, 0.25, None, False)
    assert status[1].numel() == 0 and status[3].tolist() == [True, True, False, False, False]
    assert status[4].item() == 1 and status[5].tolist() == [-1, -1]


def test_finalize_invalid_inputs_rejected():
    p = _partials(2, 144).to(DEV)
    flags = torch.zeros(2, 2, dtype=torch.int32, device=DEV)
    with pytest.raises(RuntimeError, match="Unknown compiled ABFT algorithm ID"):
        ops.abft_finalize(p, flags, 144, 0.0, 0.0, None, True, 2**32)
    with pytest.raises(RuntimeError, match="tolerances"):
        ops.abft_finalize(p, flags, 144, float("nan"), 0.0, None, True)
    with pytest.raises(RuntimeError, match="padded_N"):
        ops.abft_finalize(p, flags, 257, 0.0, 0.0, None, True)
    with pytest.raises(RuntimeError, match="same CUDA device"):
        ops.abft_finalize(p, flags.cpu(), 144, 0.0, 0.0, None, True)
    first = ops.abft_finalize(p, flags, 144, 0.0, 0.0, None, True)
    with pytest.raises(RuntimeError, match="overlap|memory location"):
        ops.abft_finalize(p, flags, 144, 0.0, 0.0, first[0], True, 0, first[0][0])


def test_finalize_cuda_graph_replay_reads_updated_thresholds():
    n = 145
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        p = _partials(3, n).to(DEV)
        p[0, -1, -1, n - 1] += 4
        flags = torch.zeros(3, 2, dtype=torch.int32, device=DEV)
        thr = torch.full((2, n), 8.0, device=DEV)
        for _ in range(3):
            ops.abft_finalize(p, flags, n, 0.125, 0.25, None, True, 0, thr)
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            out = ops.abft_finalize(p, flags, n, 0.125, 0.25, None, True, 0, thr)
        graph.replay()
        stream.synchronize()
        assert not out[3][0].item()
        thr.fill_(0.5)
        graph.replay()
        stream.synchronize()
        assert out[3][0].item()


def test_finalize_through_raw_c_abi():
    from sdc_b200 import capi

    n, tiles = 300, 5
    p = _partials(tiles, n, random=True).to(DEV)
    padded = p.shape[-1]
    obs, pred, mag = (p[i].contiguous() for i in range(3))
    hit = torch.zeros(1, dtype=torch.int32, device=DEV)
    nonfinite = torch.zeros(1, dtype=torch.int32, device=DEV)
    ref = torch.empty(2, 2, n, device=DEV)
    res = torch.empty(2, n, device=DEV)
    thr = torch.empty(2, n, device=DEV)
    flags = torch.empty(5, dtype=torch.uint8, device=DEV)
    hit_out = torch.empty(1, dtype=torch.int32, device=DEV)
    loc = torch.empty(2, dtype=torch.int64, device=DEV)
    lib = capi.lib()
    ws_bytes = lib.sdc_abft_finalize_workspace_bytes(0, n, tiles)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=DEV)
    stream = torch.cuda.current_stream().cuda_stream
    capi.check(lib.sdc_abft_finalize(0, obs.data_ptr(), pred.data_ptr(), mag.data_ptr(), tiles, padded, n, None, 0,
                                     hit.data_ptr(), nonfinite.data_ptr(), 0.125, 0.25, ref.data_ptr(), 0, 1,
                                     res.data_ptr(), thr.data_ptr(), None, 0, flags.data_ptr(), hit_out.data_ptr(),
                                     loc.data_ptr(), ws.data_ptr(), ws_bytes, stream))
    expected = oabft.finalize_serial(_np(p[0]), _np(p[1]), _np(p[2]), n, atol=0.125, rtol=0.25)
    _assert_packet((ref, res, thr, flags.bool(), hit_out, loc), expected)


# ---------------------------------------------------------------- GEMMs ----

def _integer_case(precision, m, n, k, unit=False, seed=2026):
    """Integer operands with exactly representable codes and products
    (the reference's _prepare, tests/cutlass_gemm/test_abft_gpu.py:17-53)."""
    torch.manual_seed(seed)
    a = torch.randint(-2, 3, (m, k), device=DEV).float()
    b = torch.randint(-2, 3, (n, k), device=DEV).float()
    a[:, ::16] = 6
    b[:, ::16] = 6
    if unit:
        a.zero_()
        b.zero_()
        a[:, 0] = 1
        b[:, 0] = 1
    qa, qb = quantize(a, precision, 1.0), quantize(b, precision, 1.0)
    alpha = torch.tensor(1.0 if unit else 0.25, device=DEV)
    dot = _np(a).astype(np.float64) @ _np(b).astype(np.float64).T
    return qa, qb, alpha, dot


def _args(precision, qa, qb, alpha, k):
    if precision == "fp8":
        return (qa.codes.view(torch.float8_e4m3fn), qb.codes.view(torch.float8_e4m3fn), alpha)
    return (qa.codes, qb.codes, qa.scales_mma, qb.scales_mma, k, alpha)


def _ops(precision):
    if precision == "fp8":
        return ops.fp8_mm, ops.abft_fp8_mm, ops.abft_fp8_reference_mm, 64
    return ops.nvfp4_mm, ops.abft_nvfp4_mm, ops.abft_nvfp4_reference_mm, 128


def _oracle_inputs(precision, qa, qb):
    if precision == "fp8":
        return _np(qa.codes), None, _np(qb.codes), None
    return _np(qa.codes), _np(qa.scales_mma), _np(qb.codes), _np(qb.scales_mma)


def _assert_observed(observed, weights, values, n, tile_n):
    m = values.shape[0]
    assert observed.dtype == torch.float32
    assert observed.shape == (weights.shape[0], (m + 127) // 128, ((n + tile_n - 1) // tile_n) * tile_n)
    obs = _np(observed).astype(np.float64)
    w = _np(weights).astype(np.float64)
    for t in range(obs.shape[1]):
        rows = slice(128 * t, min(m, 128 * t + 128))
        expected = w[:, rows] @ values[rows].astype(np.float64)
        assert np.allclose(obs[:, t, :n], expected, rtol=2e-5, atol=2e-3)
    assert np.count_nonzero(obs[:, :, n:]) == 0


@pytest.mark.parametrize("precision", ["fp8", "nvfp4"])
@pytest.mark.parametrize("shape", [(128, 128, 128), (136, 144, 128), (264, 272, 288), (300, 520, 1024)])
def test_gemm_and_projection_exact(precision, shape):
    m, n, k = shape
    qa, qb, alpha, dot = _integer_case(precision, m, n, k)
    base, fused, _, tile_n = _ops(precision)
    args = _args(precision, qa, qb, alpha, k)
    weights = torch.randn(2, m, device=DEV)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        baseline = base(*args)
        output, observed, hit = fused(*args, weights, -1, -1, -1)
    stream.synchronize()
    stored, _, _, _ = oabft.epilogue(dot, 0.25, _np(weights), out="f32" if precision == "fp8" else "bf16")
    assert output.stride() == baseline.stride()
    assert torch.equal(output, baseline)
    assert np.array_equal(_np(output.float()), stored)
    assert hit.item() == 0
    values = (np.float32(0.25) * dot.astype(np.float32))
    _assert_observed(observed, weights, values, n, tile_n)


@pytest.mark.parametrize("precision", ["fp8", "nvfp4"])
@pytest.mark.parametrize("location", [(0, 0), (127, 127), (128, 128), (135, 143)])
def test_bitflip_exact_global_position_and_projection(precision, location):
    m, n, k = 136, 144, 128
    qa, qb, alpha, dot = _integer_case(precision, m, n, k)
    _, fused, _, tile_n = _ops(precision)
    weights = torch.randn(2, m, device=DEV)
    row, col = location
    output, observed, hit = fused(*_args(precision, qa, qb, alpha, k), weights, row, col, 31)
    stored, _, ohit, _ = oabft.epilogue(dot, 0.25, _np(weights), (row, col, 31),
                                        out="f32" if precision == "fp8" else "bf16")
    assert hit.item() == 1 == ohit
    assert np.array_equal(_np(output.float()), stored)
    values = np.float32(0.25) * dot.astype(np.float32)
    values[row, col] = -values[row, col]
    _assert_observed(observed, weights, values, n, tile_n)


@pytest.mark.parametrize("precision", ["fp8", "nvfp4"])
def test_projection_precedes_output_rounding(precision):
    # tests/cutlass_gemm/test_abft_gpu.py:114-129: a bit-0 flip is invisible
    # in bf16 but exact in the fp32 projection of an isolated row.
    m, n, k = 136, 144, 128
    qa, qb, alpha, dot = _integer_case(precision, m, n, k)
    _, fused, _, _ = _ops(precision)
    row, col = 128, 128
    weights = torch.zeros(2, m, device=DEV)
    weights[:, row] = torch.tensor([1., -2.], device=DEV)
    args = _args(precision, qa, qb, alpha, k)
    original, _, _ = fused(*args, weights, -1, -1, -1)
    output, observed, hit = fused(*args, weights, row, col, 0)
    value = np.float32(0.25) * np.float32(dot[row, col])
    flipped = np.array([value], np.float32).view(np.uint32) ^ 1
    flipped = flipped.view(np.float32)[0]
    assert hit.item() == 1
    if precision == "nvfp4":
        assert torch.equal(output, original)
    assert np.array_equal(_np(observed[:, row // 128, col]), _np(weights[:, row]) * flipped)


@pytest.mark.parametrize("precision", ["fp8", "nvfp4"])
def test_nonfinite_injection_is_not_masked(precision):
    m, n, k = 136, 144, 128
    qa, qb, alpha, dot = _integer_case(precision, m, n, k, unit=True)
    _, fused, _, _ = _ops(precision)
    value = np.float32(dot[128, 128])
    bits = int(np.array([value], np.float32).view(np.uint32)[0])
    bit = next(b for b in range(23, 31) if ((bits ^ (1 << b)) & 0x7F800000) == 0x7F800000)
    nonfinite = torch.zeros(1, dtype=torch.int32, device=DEV)
    output, observed, hit = fused(*_args(precision, qa, qb, alpha, k), torch.ones(2, m, device=DEV), 128, 128, bit,
                                  0, nonfinite)
    assert hit.item() == 1 and nonfinite.item() == 1
    assert not torch.isfinite(output[128, 128].float())
    assert not torch.isfinite(observed[:, 1, 128]).any()
    output[128, 128] = 0
    assert torch.isfinite(output.float()).all()


@pytest.mark.parametrize("precision", ["fp8", "nvfp4"])
@pytest.mark.parametrize("fault", [(0, -1, -1), (-1, 0, 0), (136, 0, 0), (0, 144, 0), (0, 0, 32), (0, 0, -2)])
def test_invalid_fault_rejected(precision, fault):
    qa, qb, alpha, _ = _integer_case(precision, 136, 144, 128)
    _, fused, _, _ = _ops(precision)
    with pytest.raises(RuntimeError, match="fault"):
        fused(*_args(precision, qa, qb, alpha, 128), torch.randn(2, 136, device=DEV), *fault)


@pytest.mark.parametrize("precision", ["fp8", "nvfp4"])
@pytest.mark.parametrize("invalid", ["dtype", "shape", "noncontiguous", "cpu"])
def test_invalid_weights_rejected(precision, invalid):
    qa, qb, alpha, _ = _integer_case(precision, 136, 144, 128)
    _, fused, _, _ = _ops(precision)
    weights = torch.randn(2, 136, device=DEV)
    if invalid == "dtype":
        weights = weights.bfloat16()
    elif invalid == "shape":
        weights = weights[:, :-1].contiguous()
    elif invalid == "noncontiguous":
        weights = torch.ones(136, 2, device=DEV).T
    else:
        weights = weights.cpu()
    with pytest.raises(RuntimeError, match="weights|CUDA device"):
        fused(*_args(precision, qa, qb, alpha, 128), weights, -1, -1, -1)


def _dyadic_weights(m):
    # Signed, unequal, global-row weights (tests/cutlass_gemm/test_fp8_input_reference_gpu.py:14-20).
    rows = torch.arange(m, device=DEV, dtype=torch.int64)
    return torch.stack(((rows * 7 % 29 - 14).float() / 8, (rows * 11 % 37 - 18).float() / 16))


def _varying_case(precision, m, n, k):
    """Heterogeneous block scales (tests/cutlass_gemm/test_nvfp4_input_reference_gpu.py:60-81)."""
    def values(rows, phase):
        row = torch.arange(rows, device=DEV)[:, None]
        col = torch.arange(k, device=DEV)[None, :]
        exponent = ((row * 3 + col // 16 + phase) % 11 - 5).float()
        pattern = ((row + col * 7 + phase) % 13 - 6).float()
        return (pattern * torch.pow(2.0, exponent)).contiguous()
    qa, qb = quantize(values(m, 0), precision), quantize(values(n, 3), precision)
    alpha = (qa.multiplier * qb.multiplier).reciprocal()
    return qa, qb, alpha


@pytest.mark.parametrize("precision", ["fp8", "nvfp4"])
@pytest.mark.parametrize("shape", [(136, 144, 64), (136, 144, 288), (136, 144, 1024), (2048, 2048, 512),
                                   (300, 200, 96)])
@pytest.mark.parametrize("layout", [0, 1])
def test_input_reference_bit_exact_vs_oracle(precision, shape, layout):
    m, n, k = shape
    if precision == "nvfp4" and k % 32:
        pytest.skip("NVFP4 needs K % 32 == 0")
    qa, qb, alpha = _varying_case(precision, m, n, k)
    base, observe, reference, tile_n = _ops(precision)
    args = _args(precision, qa, qb, alpha, k)
    weights = _dyadic_weights(m)
    old = base(*args)
    old_out, old_obs, old_hit = observe(*args, weights, -1, -1, -1)
    out, obs, hit, pred, mag = reference(*args, weights, -1, -1, -1, 0, None, layout)
    assert torch.equal(out, old) and torch.equal(out, old_out) and torch.equal(obs, old_obs)
    assert hit.item() == old_hit.item() == 0
    a, sfa, b, sfb = _oracle_inputs(precision, qa, qb)
    padded = pred.shape[-1]
    epred, emag = native.input_reference(precision, a, sfa, b, sfb, m, n, k, _np(weights), _np(alpha), padded,
                                         "tile" if layout == 0 else "kslice")
    assert np.array_equal(_np(pred), epred)
    assert np.array_equal(_np(mag), emag)
    # Clean run: the epilogue's observation agrees with the input prediction.
    tol = 2e-5 * _np(mag).sum(axis=1) + 1e-3
    assert np.all(np.abs(_np(obs).sum(axis=1) - _np(pred).sum(axis=1)) <= tol)


@pytest.mark.parametrize("precision", ["fp8", "nvfp4"])
@pytest.mark.parametrize("shape,layout", [((2560, 4352, 2048), 1), ((2560, 4352, 512), 0), ((640, 33024, 1024), 1)])
def test_persistent_multi_tile_per_cta_bit_exact(precision, shape, layout):
    # More tiles than SMs: every CTA walks several tiles, the accumulator
    # buffers rotate and the prediction warps skip across many pipeline phases.
    m, n, k = shape
    qa, qb, alpha = _varying_case(precision, m, n, k)
    base, _, reference, _ = _ops(precision)
    args = _args(precision, qa, qb, alpha, k)
    weights = _dyadic_weights(m)
    out, obs, hit, pred, mag = reference(*args, weights, -1, -1, -1, 0, None, layout)
    assert torch.equal(out, base(*args))
    a, sfa, b, sfb = _oracle_inputs(precision, qa, qb)
    epred, emag = native.input_reference(precision, a, sfa, b, sfb, m, n, k, _np(weights), _np(alpha),
                                         pred.shape[-1], "tile" if layout == 0 else "kslice")
    assert np.array_equal(_np(pred), epred)
    assert np.array_equal(_np(mag), emag)
    tol = 2e-5 * _np(mag).sum(axis=1) + 1e-3
    assert np.all(np.abs(_np(obs).sum(axis=1) - _np(pred).sum(axis=1)) <= tol)
    from sdc_b200 import capi
    import ctypes
    code = ctypes.c_int32(-1)
    capi.check(capi.lib().sdc_read_device_error(torch.cuda.current_stream().cuda_stream, ctypes.byref(code)))
    assert code.value == 0, f"a bounded wait expired (watchdog code {code.value})"


@pytest.mark.parametrize("precision", ["fp8", "nvfp4"])
@pytest.mark.parametrize("shape", [(136, 144, 288), (300, 200, 96), (2560, 4352, 2048), (640, 33024, 1024),
                                   (5000, 640, 512)])
def test_kslice_standalone_and_fused_paths_are_bit_identical(precision, shape):
    # The K-slice prediction runs inside the GEMM (path 1), as two kernels
    # before an observed-only GEMM (path 2), or inside the GEMM from a
    # projection computed before it (path 3); all must give the oracle's
    # partials bit for bit, and the same output and observation.
    from sdc_b200 import capi

    m, n, k = shape
    qa, qb, alpha = _varying_case(precision, m, n, k)
    _, _, reference, _ = _ops(precision)
    args = _args(precision, qa, qb, alpha, k)
    weights = _dyadic_weights(m)
    lib = capi.lib()
    results = []
    try:
        for mode in (1, 2, 3):
            capi.check(lib.sdc_test_set_kslice_path(mode))
            results.append([x.clone() for x in reference(*args, weights, -1, -1, -1, 0, None, 1)])
            torch.cuda.synchronize()
    finally:
        capi.check(lib.sdc_test_set_kslice_path(0))
    (out1, obs1, hit1, pred1, mag1) = results[0]
    for out2, obs2, hit2, pred2, mag2 in results[1:]:
        assert torch.equal(out1, out2) and torch.equal(obs1, obs2) and hit1.item() == hit2.item() == 0
        assert torch.equal(pred1, pred2) and torch.equal(mag1, mag2)
    a, sfa, b, sfb = _oracle_inputs(precision, qa, qb)
    epred, emag = native.input_reference(precision, a, sfa, b, sfb, m, n, k, _np(weights), _np(alpha),
                                         pred1.shape[-1], "kslice")
    assert np.array_equal(_np(pred2), epred)
    assert np.array_equal(_np(mag2), emag)


@pytest.mark.parametrize("precision", ["fp8", "nvfp4"])
def test_epilogue_fault_changes_only_observation(precision):
    m, n, k = 136, 144, 288
    qa, qb, alpha = _varying_case(precision, m, n, k)
    _, _, reference, _ = _ops(precision)
    args = _args(precision, qa, qb, alpha, k)
    weights = _dyadic_weights(m)
    clean, obs, hit, pred, mag = reference(*args, weights, -1, -1, -1)
    out, fobs, fhit, fpred, fmag = reference(*args, weights, m - 1, n - 1, 31)
    assert hit.item() == 0 and fhit.item() == 1
    assert torch.equal(fpred, pred) and torch.equal(fmag, mag)
    expected = clean.clone()
    expected[m - 1, n - 1] = -expected[m - 1, n - 1]
    assert torch.equal(out, expected)
    assert torch.all(fobs[:, 1, n - 1] != obs[:, 1, n - 1])
    unchanged = fobs.clone()
    unchanged[:, 1, n - 1] = obs[:, 1, n - 1]
    assert torch.equal(unchanged, obs)


@pytest.mark.parametrize("precision", ["fp8", "nvfp4"])
def test_random_normal_outputs_within_fp32_accumulation_tolerance(precision):
    m, n, k = 1024, 768, 2048
    g = torch.Generator(device=DEV).manual_seed(3)
    a = torch.randn(m, k, device=DEV, generator=g, dtype=torch.bfloat16)
    b = torch.randn(n, k, device=DEV, generator=g, dtype=torch.bfloat16)
    qa, qb = quantize(a, precision), quantize(b, precision)
    alpha = (qa.multiplier * qb.multiplier).reciprocal()
    base, _, _, _ = _ops(precision)
    out = base(*_args(precision, qa, qb, alpha, k)).float()
    oa, osfa, ob, osfb = _oracle_inputs(precision, qa, qb)
    exact = native.gemm_f64(precision, oa, osfa, ob, osfb, m, n, k) * float(_np(alpha))
    bound = native.gemm_f64(precision, *_abs_operands(precision, oa, osfa, ob, osfb), m, n, k) * float(_np(alpha))
    err = np.abs(_np(out).astype(np.float64) - exact)
    # fp32 accumulation over K plus the output cast (bf16 half-ulp for NVFP4).
    limit = 2 * k * 2.0 ** -24 * bound + (2.0 ** -8 * np.abs(exact) if precision == "nvfp4" else 0) + 1e-6
    assert np.all(err <= limit)


def _abs_operands(precision, a, sfa, b, sfb):
    if precision == "fp8":
        return a & 0x7F, None, b & 0x7F, None
    return a & 0x77, sfa, b & 0x77, sfb


# ------------------------------------------------------ locate / correct ----

@pytest.mark.parametrize("precision", ["fp8", "nvfp4"])
def test_end_to_end_detect_locate_correct(precision):
    m, n, k = 520, 384, 512
    g = torch.Generator(device=DEV).manual_seed(9)
    a = torch.randn(m, k, device=DEV, generator=g)
    b = torch.randn(n, k, device=DEV, generator=g)
    qa, qb = quantize(a, precision), quantize(b, precision)
    alpha = (qa.multiplier * qb.multiplier).reciprocal()
    _, _, reference, _ = _ops(precision)
    args = _args(precision, qa, qb, alpha, k)
    weights = torch.stack((torch.ones(m, device=DEV), torch.arange(1, m + 1, device=DEV, dtype=torch.float32)))
    clean, *_ = reference(*args, weights, -1, -1, -1)
    row, col = 389, 201
    # The highest exponent bit below 30 that is clear in the clean value: the
    # flip scales it by 2^(2^(bit-23)), far above every threshold (so the ratio
    # locator must succeed), and keeps the row-weighted checksum finite.
    bits = int(np.array([clean[row, col].float().item()], np.float32).view(np.uint32)[0])
    bit = next(b for b in range(29, 24, -1) if not bits & (1 << b))
    nonfinite = torch.zeros(1, dtype=torch.int32, device=DEV)
    out, obs, hit, pred, mag = reference(*args, weights, row, col, bit, 0, nonfinite)
    packet = ops.abft_finalize_reference(obs, pred, mag, hit, nonfinite, n, 1e-3, 1e-4, None, True)
    assert packet[3][0].item() and not packet[3][1].item()
    location, located = ops.abft_locate(packet[1], packet[2], packet[3], m)
    ok, loc = oabft.locate(_np(packet[1]), _np(packet[2]), True, False, m)
    assert ok and located.item()
    assert location.tolist() == list(loc) == [row, col]
    fixed = out.clone()
    if precision == "fp8":
        corrected = ops.abft_fp8_correct(*args, location, located, fixed)
    else:
        corrected = ops.abft_nvfp4_correct(*args, location, located, fixed)
    assert corrected.item()
    torch.testing.assert_close(fixed.float(), clean.float(), rtol=1e-2, atol=1e-3)
    clean_packet = ops.abft_finalize_reference(*reference(*args, weights, -1, -1, -1, 0, nonfinite)[1:2],
                                               pred, mag, torch.zeros_like(hit), nonfinite, n, 1e-3, 1e-4, None, True)
    assert not clean_packet[3][0].item()
