#!/usr/bin/env python
"""Benchmark of the ABFT-protected FP8 / NVFP4 GEMM path on B200.

Metric: ABFT NVFP4/FP8 GEMM TFLOPS, % overhead vs the
unprotected kernel, detection recall. One step = one protected GEMM on
operands already quantised and resident in HBM: the input-fused ABFT GEMM
(tcgen05 mainloop, fused observed-checksum epilogue, input-side projection
and prediction in the K-slice layout) and the device finalize that merges
the partials and decides. Throughput counts only the useful 2*M*N*K flops.

Headline workload (config[1]): FP8 e4m3, M=N=K=8192, 1 x 128 (A) and
128 x 128 (B) fp32 block scales, fp32 accumulation, bf16 output. Measured in
the same run: the NVFP4 workload of config[2] (M=N=K=16384, e2m1 + ue4m3/16 +
fp32 global scale, bf16 out) under "nvfp4", and the reference's own FP8
semantics (tensorwise scale, fp32 output) at 8192^3 under "fp8_tensorwise".
Operands are seeded bf16 N(0,1) matrices drawn on the host, so the reference
arm can quantise exactly the same ones.

Detection (rank 0): the configuration's schedule of 1000 GEMMs, each on fresh
seeded operands, with seeded accumulator bit flips at rate 1e-3 per GEMM (at
least one per schedule): false positives and the clean residual margins
max |res|/thr and max |res|/mag; and a per-bit campaign (bits 20-31) on the
headline operands with recall per bit and per class, where a flip counts as
detectable when its own perturbation w_c * delta, computed from the flipped
value, clears the threshold by more than the clean residual. The thresholds
are atol + rtol * |w|^T |A| |B| with rtol calibrated per format from
measured clean margins (CALIBRATED_RTOL), not the reference's debug default.

Multi-GPU (python -m torch.distributed.run ... bench.py --gpus N): each rank
protects its own M-shard (8192 rows x N=K=8192, weak scaling: the job's M is
8192*N). Each step's verdict (detected, hit, max |res|/thr, max |res|) goes
into a ring of per-step status rows that the ranks all-reduce (MAX) over
NCCL once per 16 steps and at the end of the timed region, the path's only
exchange. Time is the max over ranks.

--impl reference times the reference's own CPU/torch ABFT path (restated in
oracle/cpu_path.py, bit-identical to it) on this host's cores, on the
dequantised operands of the same seed and configuration.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

METRIC = "ABFT NVFP4/FP8 GEMM TFLOPS, % overhead vs unprotected, detection recall"
UNIT = "TFLOPS"
# Relative thresholds of the benchmark's detector, per format. Calibrated on
# B200 from 1000 clean GEMMs per format at the configuration's shape, each on
# fresh seeded operands: the largest clean max |res| / |w|^T|A||B| was
# 6.5e-10 (block-scaled FP8 8192^3), 9.2e-10 (tensorwise FP8 8192^3) and
# 3.7e-10 (NVFP4 16384^3), so rtol = 1e-8 keeps a safety factor of at least
# 10.8 (every run reports the margin it measures again in "fault_schedule").
CALIBRATED_RTOL = {"fp8_block": 1e-8, "fp8": 1e-8, "nvfp4": 1e-8}
# Configuration 5 (training): gradient GEMMs (K up to 16384 tokens, values
# with a wide dynamic range) leave a larger clean residual than N(0,1)
# operands; `--workload train --calibrate` measures max |res| / magnitude per
# role (one B200, 4 steps of 507 GEMMs: forward 4.7e-8, dgrad 1.2e-6, wgrad
# 2.3e-6), and this tolerance is that maximum times a safety factor of 4.
TRAIN_RTOL = 1e-5
ATOL = 1e-3
SEEDS = {"fp8_block": 1, "fp8": 3, "nvfp4": 2}
SIZES = {"fp8_block": 8192, "fp8": 8192, "nvfp4": 16384}
EXCHANGE_EVERY = 16


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return data["bf16_tflops"], data["hbm_gbs"], "measured"
    return 1590.0, 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled during the timed region.
    The timed region starts only after the first sample has been written."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        deadline = time.time() + 10.0
        while self.proc is not None and time.time() < deadline and os.path.getsize(self.file.name) == 0:
            time.sleep(0.02)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            self.proc.wait(timeout=5)

    def summary(self):
        self.file.flush()
        rows = []
        for line in Path(self.file.name).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        sm_max = max(float(r[2]) for r in rows if r[2].replace(".", "").isdigit())
        loaded = [s for s in sm if s > 0.5 * sm_max] or sm
        reasons = set()
        for r in rows:
            for name, flag in (("hw_slowdown", r[5]), ("hw_thermal_slowdown", r[6]),
                               ("sw_thermal_slowdown", r[7]), ("sw_power_cap", r[8])):
                if flag.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": sm_max, "reasons": sorted(reasons),
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())}


# Workload formats: (quantisation precision, description).
FORMATS = {"fp8_block": ("fp8", "fp8 block-scaled 1x128 / 128x128, bf16 out"),
           "fp8": ("fp8", "fp8 tensorwise, fp32 out"),
           "nvfp4": ("nvfp4", "nvfp4 block16, bf16 out")}


def workload_name(precision, size):
    kind, rest = FORMATS[precision][1].split(" ", 1)
    return f"{kind} M=N=K={size} {rest}"


def bench_config(precision, size, world):
    """The config dict both arms print (the reference arm runs the same workload)."""
    return {"workload": workload_name(precision, size) + " ABFT (Classic, K-slice input reference) + finalize",
            "per_gpu": f"M=N=K={size}", "parallelism": f"M-shard x{world}, NCCL all-reduce of detection status",
            "operands": f"seeded bf16 N(0,1) A [M,K] and B [N,K] drawn on the host (seed {SEEDS[precision]}"
                        f" + 1000*rank), quantised once",
            "l2": "working set (A+B codes, output) > 126 MB L2; no explicit flush"}


def host_operands(m, n, k, seed, b_std=1.0):
    """Seeded bf16 A [m, k] and B rows [n, k] on the host (both arms use these)."""
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(m, k, generator=g, dtype=torch.bfloat16)
    b = torch.randn(n, k, generator=g, dtype=torch.bfloat16)
    if b_std != 1.0:
        b = (b.float() * b_std).to(torch.bfloat16)
    return a, b


def quantise(precision, a, b):
    """Device bf16 A [m,k], B rows [n,k] -> (op args, (qa, qb))."""
    from sdc_b200.gemm.quantization import quantize, quantize_blockwise

    if precision == "fp8_block":
        qa, qb = quantize_blockwise(a, 1), quantize_blockwise(b, 128)
        return (qa.codes.view(torch.float8_e4m3fn), qb.codes.view(torch.float8_e4m3fn), qa.scales, qb.scales), (qa, qb)
    qa, qb = quantize(a, precision), quantize(b, precision)
    alpha = (qa.multiplier * qb.multiplier).reciprocal()
    if precision == "fp8":
        return (qa.codes.view(torch.float8_e4m3fn), qb.codes.view(torch.float8_e4m3fn), alpha), (qa, qb)
    return (qa.codes, qb.codes, qa.scales_mma, qb.scales_mma, a.shape[1], alpha), (qa, qb)


def _dequantize_row(q, row):
    """Decoded row of a QuantizedMatrix (codes * block scales / multiplier)."""
    import dataclasses

    from sdc_b200.gemm.quantization import dequantize

    if q.precision == "fp8" and q.block_rows:
        scales = q.scales[row // q.block_rows:row // q.block_rows + 1]
        return q.codes[row:row + 1].view(torch.float8_e4m3fn).float() * scales.repeat_interleave(128, 1)
    one = dataclasses.replace(q, codes=q.codes[row:row + 1],
                              scales=None if q.scales is None else q.scales[row:row + 1], shape=(1, q.shape[1]))
    return dequantize(one)


class Protected:
    """One protected GEMM step on resident operands (the hot path)."""

    def __init__(self, precision, m, n, k, device, seed, layout=1, atol=ATOL, rtol=None, b_std=1.0, operands=None):
        self.ops = torch.ops.sdc_cutlass
        self.precision, self.m, self.n, self.k, self.device = precision, m, n, k, device
        if operands is None:
            operands = host_operands(m, n, k, seed, b_std)
        a, b = (t.to(device) for t in operands)
        self.args, self.quantised = quantise(precision, a, b)
        del a, b
        self.weights = torch.stack((torch.ones(m, device=device),
                                    torch.arange(1, m + 1, device=device, dtype=torch.float32)))
        self.nonfinite = torch.zeros(1, dtype=torch.int32, device=device)
        self.atol = atol
        self.rtol = CALIBRATED_RTOL[precision] if rtol is None else rtol
        ops = self.ops
        if precision == "fp8_block":  # K-slice is the block-scaled op's only layout
            self.fused, self.plain = ops.abft_fp8_block_reference_mm, ops.fp8_block_mm
            self.layout_args = ()
        else:
            self.fused = ops.abft_fp8_reference_mm if precision == "fp8" else ops.abft_nvfp4_reference_mm
            self.plain = ops.fp8_mm if precision == "fp8" else ops.nvfp4_mm
            self.layout_args = (layout,)

    def requantise(self, a, b):
        self.args, self.quantised = quantise(self.precision, a, b)

    def step_rows(self, fault=(-1, -1, -1)):
        """The step with row checksums: the protected GEMM whose epilogue also
        sums the output rows, the row prediction alpha * A (B^T e), the
        finalize and the two-dimensional locator."""
        if self.precision == "fp8_block":
            a, b, sa, sb = self.args
            rows_args = (2, a, sa, b, sb, self.k, None)
        elif self.precision == "fp8":
            a, b, alpha = self.args
            rows_args = (0, a, None, b, None, self.k, alpha)
        else:
            a, b, sa, sb, k, alpha = self.args
            rows_args = (1, a, sa, b, sb, k, alpha)
        out, obs, hit, pred, mag, row_obs, row_pred, row_mag = self.ops.abft_reference_rows_mm(
            *rows_args, self.weights, *fault, 0, self.nonfinite, 1)
        packet = self.ops.abft_finalize_reference(obs, pred, mag, hit, self.nonfinite, self.n, self.atol,
                                                  self.rtol, None, True)
        location, located, row_flags, _, _ = self.ops.abft_locate2d(row_obs, row_pred, row_mag, self.atol,
                                                                    self.rtol, packet[1], packet[2], packet[3])
        return out, packet, (location, located, row_flags)

    def step(self, fault=(-1, -1, -1), diagnostics=True):
        out, obs, hit, pred, mag = self.fused(*self.args, self.weights, *fault, 0, self.nonfinite, *self.layout_args)
        packet = self.ops.abft_finalize_reference(obs, pred, mag, hit, self.nonfinite, self.n, self.atol,
                                                  self.rtol, None, diagnostics)
        return out, packet

    def unprotected(self):
        return self.plain(*self.args)

    def fused_only(self):
        """The step's dominant kernel alone: the protected GEMM without finalize."""
        return self.fused(*self.args, self.weights, -1, -1, -1, 0, self.nonfinite, *self.layout_args)

    def exact_value(self, row, col):
        """Float64 dot product of the decoded operands at (row, col), times alpha:
        the fp32 value the epilogue sees, up to the accumulation order."""
        qa, qb = self.quantised
        return float((_dequantize_row(qa, row).double() * _dequantize_row(qb, col).double()).sum())


def timed(fn, steps, warmup, stream):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        fn()
    end.record(stream)
    end.synchronize()
    return start.elapsed_time(end) / 1e3


def paired_overhead(prot, steps, rounds=5):
    """Protected vs unprotected step, alternating blocks so both see the same
    clocks and temperature (the reference times paired, alternating calls)."""
    stream = torch.cuda.current_stream()
    n = max(2, steps // rounds)
    t_prot = t_plain = 0.0
    for _ in range(rounds):
        t_prot += timed(prot.step, n, 1, stream)
        t_plain += timed(prot.unprotected, n, 1, stream)
    return t_prot / (rounds * n), t_plain / (rounds * n)


def timed_flushed(fns, iters, stream, flush):
    """Mean device seconds per call of each function in ``fns``, one call at
    a time with L2 flushed (a write larger than L2) before each, outside the
    timed interval; the functions alternate so they share clocks."""
    totals = [0.0] * len(fns)
    for _ in range(iters):
        for i, fn in enumerate(fns):
            flush.add_(1)
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(stream)
            fn()
            end.record(stream)
            end.synchronize()
            totals[i] += start.elapsed_time(end) / 1e3
    return [t / iters for t in totals]


# Published augmented-mode timings of the reference at M=N=K=2048 on an RTX
# 5090 (its own benchmark, BF16): augmented ABFT vs the unprotected GEMM.
REFERENCE_AUGMENTED_2048 = {"gpu": "RTX 5090", "protected_us": 137.872, "unprotected_us": 98.895}


def augmented_bf16(device, stream, sizes=(2048, 8192), iters=20):
    """The augmented BF16 ABFT GEMM (Classic, compact form + packed finalize)
    against the unprotected BF16 GEMM of this library at M=N=K = each size,
    L2 flushed before every call; plus the clean calls' largest
    |residual| / magnitude (what the relative threshold must clear)."""
    from sdc_b200 import ops

    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)
    bf16_peak, _, basis = measured_peaks()
    out = {}
    for size in sizes:
        g = torch.Generator().manual_seed(size)
        a = torch.randn(size, size, generator=g).to(torch.bfloat16).to(device)
        b_kn = torch.randn(size, size, generator=g).to(torch.bfloat16).to(device).T.contiguous().T
        rows = torch.arange(1, size + 1, device=device, dtype=torch.float32)
        w = torch.stack((torch.ones_like(rows), rows)).to(torch.bfloat16)
        worst = torch.zeros((), device=device)

        def protected():
            _, partials, flags = ops.abft_augmented_compact(a, b_kn, w, -1, -1, -1, 0)
            packet = ops.abft_finalize(partials, flags, size, 0.0, 0.0, None, True, 0, None)
            return partials, packet

        def plain():
            ops.mm(a, b_kn)

        def library():  # cuBLAS through torch: an anchor for the plain GEMM, not this library
            torch.matmul(a, b_kn)

        for _ in range(3):
            partials, packet = protected()
            plain()
            mag = partials[2].sum(dim=1)[:, :size]
            torch.maximum(worst, (packet[1].abs() / mag.clamp_min(1e-30)).amax(), out=worst)
        library()
        t_prot, t_plain, t_lib = timed_flushed([protected, plain, library], iters, stream, flush)
        # Host enqueue time of one eager call (no synchronisation inside).
        host = []
        for fn in (protected, plain):
            torch.cuda.synchronize()
            flush.add_(1)  # keeps the GPU busy so the enqueue never waits on it
            t0 = time.perf_counter()
            fn()
            host.append(time.perf_counter() - t0)
        torch.cuda.synchronize()
        # The same calls captured once in CUDA graphs and replayed: device
        # time without the host's per-call work.
        graphs = []
        for fn in (protected, plain):
            side = torch.cuda.Stream(device)
            side.wait_stream(stream)
            with torch.cuda.stream(side):
                fn()
            stream.wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                fn()
            graphs.append(graph)
        t_prot_graph, t_plain_graph = timed_flushed([g.replay for g in graphs], iters, stream, flush)
        del graphs
        flops = 2.0 * size ** 3
        out[str(size)] = {
            "protected_us": t_prot * 1e6, "unprotected_us": t_plain * 1e6, "time_ratio": t_prot / t_plain,
            "overhead_pct": 100.0 * (t_prot / t_plain - 1.0),
            "protected_tflops": flops / t_prot / 1e12, "unprotected_tflops": flops / t_plain / 1e12,
            "unprotected_frac_of_bf16_peak": flops / t_plain / 1e12 / bf16_peak,
            "cublas_bf16_us": t_lib * 1e6,
            "host_enqueue_us": {"protected": host[0] * 1e6, "unprotected": host[1] * 1e6},
            "graph_replay": {"protected_us": t_prot_graph * 1e6, "unprotected_us": t_plain_graph * 1e6,
                             "time_ratio": t_prot_graph / t_plain_graph},
            "clean_max_res_over_magnitude": float(worst),
            "launches_per_call": {"protected": 3, "unprotected": 1},
        }
        del a, b_kn
    out["method"] = (f"{iters} alternating calls each, L2 flushed before every call (256 MB write, untimed), "
                     "CUDA events per call; protected = encode + augmented GEMM + finalize (one "
                     "launch)")
    out["peak_basis"] = f"{basis} bf16 dense burst ({bf16_peak} TFLOP/s)"
    out["reference_published_2048"] = {**REFERENCE_AUGMENTED_2048,
                                       "time_ratio": REFERENCE_AUGMENTED_2048["protected_us"]
                                       / REFERENCE_AUGMENTED_2048["unprotected_us"]}
    return out


def profiled_traffic(precision, size):
    """DRAM bytes (read + write) of one protected-GEMM launch of this workload,
    from the committed same-size ncu capture summary (profiles/traffic.json),
    or None when no capture of this exact workload exists."""
    path = ROOT / "profiles" / "traffic.json"
    if not path.exists():
        return None, None
    entry = json.loads(path.read_text()).get(f"{precision}_{size}")
    if not entry:
        return None, None
    return entry["dram_bytes_read"] + entry["dram_bytes_write"], entry["source"]


# Kernels this library launches per protected step: the GEMM (projection and
# K-slice prediction fused into it) + the finalize (its last block also
# writes the flags).
LAUNCHES_PER_STEP = 2


def _flip(value, bit):
    import numpy as np

    bits = np.array([value], np.float32).view(np.uint32) ^ np.uint32(1 << bit)
    return float(bits.view(np.float32)[0])


def detection_campaign(prot, flips_per_bit, seed):
    """Per-bit recall on the headline operands (bits 20-31). A flip is
    detectable when, for some channel c, |w_c[row] * delta| exceeds the clean
    threshold plus the clean residual of that column, where delta is the
    flipped minus the clean fp32 value (from the decoded operands,
    independently of the checksum arithmetic); undetectable when it is below
    the threshold minus the clean residual for every channel; ambiguous
    otherwise. Non-finite flipped values are detectable (non-finite rule)."""
    g = torch.Generator().manual_seed(seed)
    clean_out, clean_packet = prot.step()
    residual0 = clean_packet[1].double().cpu()
    threshold0 = clean_packet[2].double().cpu()
    per_bit = {}
    totals = {"flips": 0, "detected": 0, "detectable": 0, "detected_detectable": 0, "undetectable": 0,
              "detected_undetectable": 0, "ambiguous": 0}
    classes = {"exponent": [0, 0, 0, 0], "high_mantissa": [0, 0, 0, 0], "sign": [0, 0, 0, 0]}
    for bit in range(20, 32):
        stats = [0, 0, 0, 0]  # flips, detected, detectable, detected among detectable
        for _ in range(flips_per_bit):
            row = int(torch.randint(0, prot.m, (1,), generator=g))
            col = int(torch.randint(0, prot.n, (1,), generator=g))
            if prot.precision == "fp8":
                value = float(clean_out[row, col])  # fp32 output: exactly the epilogue's value
            else:
                value = float(torch.tensor(prot.exact_value(row, col), dtype=torch.float32))
            flipped = _flip(value, bit)
            _, packet = prot.step((row, col, bit))
            hit = bool(packet[3][0])
            if not math.isfinite(flipped):
                status = "detectable"
            else:
                delta = abs(flipped - value)
                perturb = [delta, (row + 1.0) * delta]
                clean = [abs(float(residual0[c, col])) for c in range(2)]
                thr = [float(threshold0[c, col]) for c in range(2)]
                if any(perturb[c] > thr[c] + clean[c] for c in range(2)):
                    status = "detectable"
                elif all(perturb[c] < thr[c] - clean[c] for c in range(2)):
                    status = "undetectable"
                else:
                    status = "ambiguous"
            stats[0] += 1
            stats[1] += hit
            totals["flips"] += 1
            totals["detected"] += hit
            if status == "detectable":
                stats[2] += 1
                stats[3] += hit
                totals["detectable"] += 1
                totals["detected_detectable"] += hit
            elif status == "undetectable":
                totals["undetectable"] += 1
                totals["detected_undetectable"] += hit
            else:
                totals["ambiguous"] += 1
        per_bit[bit] = {"flips": stats[0], "detected": stats[1], "detectable": stats[2],
                        "detected_detectable": stats[3]}
        cls = "sign" if bit == 31 else "exponent" if bit >= 23 else "high_mantissa"
        for i in range(4):
            classes[cls][i] += stats[i]
    by_class = {name: {"flips": v[0], "detected": v[1], "recall": v[1] / max(v[0], 1), "detectable": v[2],
                       "recall_detectable": v[3] / max(v[2], 1)} for name, v in classes.items()}
    return {"flips_per_bit": flips_per_bit, "per_bit": per_bit, "by_class": by_class, **totals,
            "recall_all": totals["detected"] / max(totals["flips"], 1),
            "recall_detectable": totals["detected_detectable"] / max(totals["detectable"], 1),
            "missed_detectable": totals["detectable"] - totals["detected_detectable"],
            "detectable_rule": "|w_c delta| > thr_c + |clean res_c| for some channel c, delta from the decoded "
                               "operands (independent of the checksum arithmetic); non-finite flips detectable",
            "clean_flagged": bool(clean_packet[3][0])}


def row_checksum_leg(prot, steps, seed, flips=48, rounds=5):
    """Row checksums with two-dimensional localisation: the step's cost
    against the column-only step and the unprotected GEMM (paired
    alternating blocks), and a localisation campaign of single accumulator
    flips (bits 23-30 at seeded positions): of the flips the columns
    detected, how many the row/column pair located at the exact element,
    against the two-channel ratio locator on the same packets."""
    stream = torch.cuda.current_stream()
    n = max(2, steps // rounds)
    t_rows = t_cols = t_plain = 0.0
    for _ in range(rounds):
        t_rows += timed(prot.step_rows, n, 1, stream)
        t_cols += timed(prot.step, n, 1, stream)
        t_plain += timed(prot.unprotected, n, 1, stream)
    t_rows, t_cols, t_plain = (t / (rounds * n) for t in (t_rows, t_cols, t_plain))
    g = torch.Generator().manual_seed(seed)
    counts = {"flips": 0, "column_detected": 0, "row_detected": 0, "located_2d": 0, "located_2d_exact": 0,
              "located_ratio": 0, "located_ratio_exact": 0}
    _, clean_packet, (_, clean_located, clean_rows) = prot.step_rows()
    for i in range(flips):
        row = int(torch.randint(0, prot.m, (1,), generator=g))
        col = int(torch.randint(0, prot.n, (1,), generator=g))
        bit = 23 + i % 8
        _, packet, (location, located, row_flags) = prot.step_rows((row, col, bit))
        ratio_location, ratio_located = prot.ops.abft_locate(packet[1], packet[2], packet[3], prot.m)
        counts["flips"] += 1
        if not bool(packet[3][0]):
            continue
        counts["column_detected"] += 1
        counts["row_detected"] += bool(row_flags[0])
        counts["located_2d"] += bool(located)
        counts["located_2d_exact"] += location.tolist() == [row, col]
        counts["located_ratio"] += bool(ratio_located)
        counts["located_ratio_exact"] += ratio_location.tolist() == [row, col]
    return {"ms_per_step": t_rows * 1e3, "column_only_ms_per_step": t_cols * 1e3,
            "unprotected_ms_per_step": t_plain * 1e3,
            "overhead_pct": 100.0 * (t_rows / t_plain - 1.0),
            "added_over_column_only_pct": 100.0 * (t_rows / t_cols - 1.0),
            "clean_flagged": bool(clean_packet[3][0]) or bool(clean_rows[0]) or bool(clean_located),
            "localisation": counts,
            "method": "paired alternating blocks; flips of the fp32 accumulator, bits 23-30, seeded positions"}


def fault_schedule(prot, seed, gemms=1000, rate=1e-3):
    """The configurations' schedule: ``gemms`` protected GEMMs, each on fresh
    seeded operands of the workload's shape drawn on the device, each carrying
    one seeded accumulator flip (uniform row, column and bit in [0, 32)) with
    probability ``rate``; when the draws give none, one GEMM of the schedule
    (drawn uniformly) carries one, so every schedule injects. Verdicts and the
    clean residual margins stay on the device until the end."""
    g = torch.Generator().manual_seed(seed + 7919)
    draws = torch.rand(gemms, generator=g) < rate
    if not bool(draws.any()):
        draws[int(torch.randint(0, gemms, (1,), generator=g))] = True
    faults = {}
    for i in draws.nonzero().flatten().tolist():
        faults[i] = (int(torch.randint(0, prot.m, (1,), generator=g)), int(torch.randint(0, prot.n, (1,), generator=g)),
                     int(torch.randint(0, 32, (1,), generator=g)))
    device = prot.device
    flags = torch.zeros(gemms, dtype=torch.bool, device=device)
    nonfinite = torch.zeros(gemms, dtype=torch.bool, device=device)
    ratio_thr = torch.zeros(gemms, dtype=torch.float64, device=device)
    ratio_mag = torch.zeros(gemms, dtype=torch.float64, device=device)
    dev_gen = torch.Generator(device=device)
    saved = prot.args, prot.quantised
    for i in range(gemms):
        dev_gen.manual_seed(seed * 100003 + i)
        a = torch.randn(prot.m, prot.k, device=device, generator=dev_gen, dtype=torch.bfloat16)
        b = torch.randn(prot.n, prot.k, device=device, generator=dev_gen, dtype=torch.bfloat16)
        prot.requantise(a, b)
        del a, b
        _, packet = prot.step(faults.get(i, (-1, -1, -1)))
        flags[i] = packet[3][0]
        nonfinite[i] = packet[3][1]
        res = packet[1].abs().double()
        ratio_thr[i] = (res / packet[2].double()).amax()
        ratio_mag[i] = (res / packet[0][1].double().clamp_min(1e-30)).amax()
    prot.args, prot.quantised = saved
    flags, nonfinite = flags.cpu(), nonfinite.cpu()
    ratio_thr, ratio_mag = ratio_thr.cpu(), ratio_mag.cpu()
    clean = torch.ones(gemms, dtype=torch.bool)
    clean[list(faults)] = False
    return {"gemms": gemms, "rate": rate, "faulted": len(faults), "detected": int(flags[~clean].sum()),
            "faults": [{"gemm": i, "row": r, "col": c, "bit": bit, "detected": bool(flags[i]),
                        "nonfinite": bool(nonfinite[i])} for i, (r, c, bit) in sorted(faults.items())],
            "clean": int(clean.sum()), "false_positives": int(flags[clean].sum()),
            "clean_max_res_over_thr": float(ratio_thr[clean].max()),
            "clean_max_res_over_mag": float(ratio_mag[clean].max()),
            "clean_p50_res_over_mag": float(ratio_mag[clean].median()),
            "operands": "fresh seeded N(0,1) bf16 operands per GEMM (device generator)"}


# Qwen2.5-7B linear layers at T = 16384 tokens: (name, M, N, K).
QWEN_SHAPES = (("qkv", 16384, 4608, 3584), ("o", 16384, 3584, 3584), ("gate_up", 16384, 37888, 3584),
               ("down", 16384, 3584, 18944))


def qwen_sweep(args, device, stream, rank, world, dist):
    """Protected vs unprotected GEMM on the Qwen linear shapes, rows of the
    activations sharded over the ranks (the shape's M split into 128-aligned
    blocks); time = max over ranks. gate and up share K and the activation,
    so they run as one N = 2*18944 GEMM."""
    from sdc_b200.abft.distributed import shard_rows

    out = {}
    for precision in FORMATS:
        if args.format not in ("all", precision):
            continue
        rows = {}
        total_flops = total_prot = total_plain = 0.0
        for name, m, n, k in QWEN_SHAPES:
            start, stop = shard_rows(m, world, rank)
            g = torch.Generator(device=device).manual_seed(7 + rank)
            a = torch.randn(stop - start, k, device=device, generator=g, dtype=torch.bfloat16)
            b = (torch.randn(n, k, device=device, generator=g, dtype=torch.bfloat16) * 0.02).to(torch.bfloat16)
            prot = Protected(precision, stop - start, n, k, device, 0, operands=(a, b))
            del a, b
            # Paired, alternating blocks (as for the headline), so that both
            # arms see the same clocks under the power cap.
            step_t, plain_t = paired_overhead(prot, 3 * args.sweep_steps, rounds=3)
            t = torch.tensor([step_t, plain_t], device=device)
            if dist is not None:
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
            t_prot, t_plain = (float(v) for v in t.tolist())
            flops = 2.0 * m * n * k
            rows[name] = {"m": m, "n": n, "k": k, "tflops": flops / t_prot / 1e12,
                          "unprotected_tflops": flops / t_plain / 1e12,
                          "overhead_pct": 100.0 * (t_prot / t_plain - 1.0)}
            total_flops += flops
            total_prot += t_prot
            total_plain += t_plain
            del prot
        torch.cuda.empty_cache()
        out[precision] = {"layers": rows, "tflops": total_flops / total_prot / 1e12,
                          "overhead_pct": 100.0 * (total_prot / total_plain - 1.0)}
    out["config"] = (f"T=16384 tokens, activations N(0,1), weights N(0,0.02), bf16 before quantisation; "
                     f"M sharded over {world} rank(s); 3 alternating blocks of {args.sweep_steps} protected and "
                     f"{args.sweep_steps} unprotected steps per shape")
    return out


ABFT_PUBLIC = {"method": "classic", "implementation": "native", "reference_mode": "input_fused",
               "reference_layout": "kslice", "on_error": "report", "recovery": "none", "diagnostics": False}


def e2e_run(precision, host_a, host_b_kn, device, atol, rtol, steps, stream):
    """``steps`` clean end-to-end protected GEMMs through the public API
    (sdc_b200.abft.execute: quantise both operands, protected GEMM,
    finalize) from pinned host bf16 operands, with the output
    and the verdict copied back to pinned host memory every step. Step i+1's
    host-to-device copies run on a copy stream (two buffer sets) and step i's
    device-to-host copies on another while the compute stream works.
    Returns (seconds per step from CUDA events on the compute stream, bytes
    copied back per step, steps flagged)."""
    from sdc_b200.abft import execute

    scaling = {"fp8_block": "blockwise", "fp8": "tensorwise", "nvfp4": "block16"}[precision]
    quant = FORMATS[precision][0]
    cfg = dict(ABFT_PUBLIC, atol=atol, rtol=rtol)
    copy_in, copy_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    dev_a = [torch.empty_like(host_a, device=device) for _ in range(2)]
    dev_b = [torch.empty_like(host_b_kn, device=device) for _ in range(2)]
    m, n = host_a.shape[0], host_b_kn.shape[1]
    out_dtype = torch.float32 if precision == "fp8" else torch.bfloat16
    out_host = [torch.empty((m, n), dtype=out_dtype).pin_memory() for _ in range(2)]
    flags_host = torch.empty((steps, 2), dtype=torch.bool).pin_memory()
    copied = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]

    def issue_copy(i):
        slot = i % 2
        with torch.cuda.stream(copy_in):
            if i >= 2:
                copy_in.wait_event(free[slot])
            dev_a[slot].copy_(host_a, non_blocking=True)
            dev_b[slot].copy_(host_b_kn, non_blocking=True)
            copied[slot].record(copy_in)

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record(stream)
    with torch.cuda.stream(copy_in):
        copy_in.wait_event(start)
    issue_copy(0)
    for i in range(steps):
        if i + 1 < steps:
            issue_copy(i + 1)
        slot = i % 2
        stream.wait_event(copied[slot])
        out, report = execute(dev_a[slot], dev_b[slot], quant, scaling, abft_config=cfg)
        free[slot].record(stream)
        copy_out.wait_stream(stream)
        with torch.cuda.stream(copy_out):
            # Same-stream order keeps out_host[slot] from being overwritten
            # before the previous copy into it has finished.
            out_host[slot].copy_(out, non_blocking=True)
            flags_host[i, 0].copy_(report.detected.reshape(()), non_blocking=True)
            flags_host[i, 1].copy_(report.nonfinite.reshape(()), non_blocking=True)
        out.record_stream(copy_out)
    stream.wait_stream(copy_out)
    end.record(stream)
    end.synchronize()
    return (start.elapsed_time(end) / 1e3 / steps, m * n * out_host[0].element_size() + 2,
            int(flags_host[:, 0].sum()))


def library_ceiling(device, stream):
    """Library GEMMs at the workloads' shapes on the same box, as achievable
    anchors beside the 2x / 4x bf16 denominators (torch._scaled_mm, i.e.
    cuBLASLt). Each entry is TFLOP/s, or the error when the library rejects
    the form."""
    out = {}
    size = 8192
    g = torch.Generator(device=device).manual_seed(5)
    a = torch.randn(size, size, device=device, generator=g).to(torch.float8_e4m3fn)
    b = torch.randn(size, size, device=device, generator=g).to(torch.float8_e4m3fn)
    one = torch.ones((), device=device)
    flops = 2.0 * size ** 3

    def measure(name, fn, flop):
        try:
            fn()
            seconds = timed(fn, 20, 3, stream) / 20
            out[name] = {"tflops": flop / seconds / 1e12}
        except Exception as error:  # the library may not offer this form
            out[name] = {"error": str(error).splitlines()[0][:200]}

    measure("fp8_tensorwise_8192_bf16out", lambda: torch._scaled_mm(a, b.t(), scale_a=one, scale_b=one,
                                                                     out_dtype=torch.bfloat16), flops)
    # 1 x 128 activation and 128 x 128 weight scales: the scale layouts the
    # library accepts differ between versions, so the known forms are tried.
    sa = torch.rand(size, size // 128, device=device) + 0.5
    sb = torch.rand(size // 128, size // 128, device=device) + 0.5
    forms = (("row-major", lambda: (sa, sb)), ("a outer-dim-major", lambda: (sa.t().contiguous().t(), sb)),
             ("both outer-dim-major", lambda: (sa.t().contiguous().t(), sb.t().contiguous().t())))
    name = "fp8_blockwise_1x128_128x128_8192_bf16out"
    errors = []
    for form, scales in forms:
        s_a, s_b = scales()
        measure(name, lambda: torch._scaled_mm(a, b.t(), scale_a=s_a, scale_b=s_b, out_dtype=torch.bfloat16), flops)
        if "tflops" in out[name]:
            out[name]["scale_form"] = form
            break
        errors.append(f"{form}: {out[name]['error']}")
    else:
        out[name] = {"error": "; ".join(errors)}
    del a, b
    n4 = 16384
    try:
        codes = torch.randint(0, 256, (n4, n4 // 2), device=device, dtype=torch.uint8)
        scales = torch.full((n4 * n4 // 16,), 0x38, device=device, dtype=torch.uint8)
        fa = codes.view(torch.float4_e2m1fn_x2)
        sfa = scales.view(torch.float8_e4m3fn)
        measure("nvfp4_16384_bf16out", lambda: torch._scaled_mm(fa, fa.t(), scale_a=sfa, scale_b=sfa,
                                                                 out_dtype=torch.bfloat16), 2.0 * n4 ** 3)
    except Exception as error:
        out["nvfp4_16384_bf16out"] = {"error": str(error).splitlines()[0][:200]}
    torch.cuda.empty_cache()
    return out


def run_ours(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    import sdc_b200

    sdc_b200.require_device(device)
    dist = None
    # The result is the only line on stdout: libraries (NCCL prints its
    # version) write to stderr instead while this run lasts.
    result_fd = os.dup(1)
    os.dup2(2, 1)
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    stream = torch.cuda.current_stream(device)
    bf16_peak, hbm_peak, basis = measured_peaks()
    results = {}
    for precision in ("fp8_block", "fp8", "nvfp4"):
        if args.format not in ("all", precision):
            continue
        size = args.size or SIZES[precision]
        m = n = k = size
        if args.shape:
            m, n, k = (int(x) for x in args.shape.split(","))
        prot = Protected(precision, m, n, k, device, SEEDS[precision] + 1000 * rank, rtol=args.rtol)
        flops = 2.0 * m * n * k
        ring = torch.zeros(EXCHANGE_EVERY, 4, dtype=torch.float32, device=device)
        exchanged = torch.zeros(4, dtype=torch.float32, device=device)
        counter = [0]

        def exchange():
            dist.all_reduce(ring, op=dist.ReduceOp.MAX)
            torch.maximum(exchanged, ring.amax(dim=0), out=exchanged)
            ring.zero_()

        def step():
            _, packet = prot.step()
            if dist is not None:
                # This step's verdict and residual norms into the ring; the
                # ranks exchange the ring once per EXCHANGE_EVERY steps.
                slot = counter[0] % EXCHANGE_EVERY
                res = packet[1].abs()
                ring[slot, 0] = packet[3][0].float()
                ring[slot, 1] = packet[4][0].float()
                ring[slot, 2] = (res / packet[2]).amax()
                ring[slot, 3] = res.amax()
                counter[0] += 1
                if counter[0] % EXCHANGE_EVERY == 0:
                    exchange()

        for _ in range(args.warmup):
            step()
        if dist is not None and counter[0] % EXCHANGE_EVERY:
            exchange()
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        counter[0] = 0
        with ClockSampler(local) as clocks:
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(stream)
            for _ in range(args.steps):
                step()
            if dist is not None and counter[0] % EXCHANGE_EVERY:
                exchange()
            end.record(stream)
            end.synchronize()
        elapsed = start.elapsed_time(end) / 1e3
        torch.cuda.synchronize()
        if dist is not None:
            t = torch.tensor([elapsed], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            elapsed = float(t.item())
        step_paired, plain_paired = paired_overhead(prot, args.steps)
        t_fused = timed(prot.fused_only, args.steps, 2, stream)
        per_step = elapsed / args.steps
        fp8 = precision.startswith("fp8")
        peak = bf16_peak * (2 if fp8 else 4)
        traffic, traffic_source = profiled_traffic(precision, size)
        entry = {
            "workload": workload_name(precision, size),
            "tflops": world * flops / per_step / 1e12,
            "ms_per_step": per_step * 1e3,
            "unprotected_tflops": flops / plain_paired / 1e12,
            "overhead_pct": 100.0 * (step_paired / plain_paired - 1.0),
            "overhead_method": "paired alternating blocks of protected (GEMM + finalize) and unprotected steps",
            "roofline": {"bound": "tensor", "achieved": flops / (t_fused / args.steps) / 1e12, "peak": peak,
                         "unit": "TFLOP/s", "frac": flops / (t_fused / args.steps) / 1e12 / peak,
                         "kernel": "protected GEMM (gemm_kernel with checksums, projection and prediction)",
                         "traffic": traffic, "traffic_source": traffic_source,
                         "algorithmic_flops": flops,
                         "peak_basis": f"{2 if fp8 else 4}x {basis} bf16 dense burst "
                                       f"({bf16_peak} TFLOP/s) of measured; nominal dense {4500 if fp8 else 9000}"},
            "thresholds": {"atol": prot.atol, "rtol": prot.rtol, "rule": "thr = atol + rtol * |w|^T|A||B|"},
            "clocks": clocks.summary(),
        }
        if dist is not None:
            verdict = exchanged.tolist()
            entry["exchanged_status"] = {"detected": verdict[0], "fault_hit": verdict[1],
                                         "max_res_over_thr": verdict[2], "max_abs_res": verdict[3],
                                         "method": f"ring of per-step [detected, hit, max|res|/thr, max|res|], "
                                                   f"MAX all-reduce every {EXCHANGE_EVERY} steps"}
        if rank == 0 and not args.no_detection:
            entry["detection"] = detection_campaign(prot, args.flips_per_bit, SEEDS[precision])
            entry["fault_schedule"] = fault_schedule(prot, SEEDS[precision], gemms=args.schedule_gemms)
        if rank == 0 and not args.no_rows:
            entry["row_checksums"] = row_checksum_leg(prot, args.steps, SEEDS[precision] + 7)
        if not args.no_e2e:  # every rank: its own shard end to end, time = max over ranks
            host_a, host_b = host_operands(m, n, k, SEEDS[precision] + 1000 * rank)
            host_a = host_a.pin_memory()
            host_b_kn = host_b.T.contiguous().pin_memory()  # the public API's B is [K, N]
            e2e_run(precision, host_a, host_b_kn, device, prot.atol, prot.rtol, 3, stream)  # warm-up
            e_steps = max(3, args.steps // 4)
            t0 = time.perf_counter()
            e_time, d2h, e_flagged = e2e_run(precision, host_a, host_b_kn, device, prot.atol, prot.rtol, e_steps,
                                             stream)
            wall = (time.perf_counter() - t0) / e_steps
            if dist is not None:
                t = torch.tensor([e_time], device=device)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                e_time = float(t.item())
            entry["e2e"] = {"value": world * flops / e_time / 1e12, "unit": UNIT,
                            "h2d_bytes_per_step": world * (host_a.numel() * 2 + host_b.numel() * 2),
                            "d2h_bytes_per_step": world * d2h, "host_wall_s_per_step": wall,
                            "clean_steps_flagged": e_flagged,
                            "api": "sdc_b200.abft.execute (quantise + protected GEMM + finalize), host buffers in "
                                   "and out",
                            "pipeline": "step i+1's host-to-device copies and step i's device-to-host copies "
                                        "overlap the compute"}
        results[precision] = entry
        del prot
        torch.cuda.empty_cache()
    sweep = None if args.no_sweep else qwen_sweep(args, device, stream, rank, world, dist)
    augmented = None if (args.no_augmented or rank != 0) else augmented_bf16(
        device, stream, tuple(int(x) for x in args.augmented_sizes.split(",")), args.augmented_iters)
    ceiling = None if (args.no_ceiling or rank != 0) else library_ceiling(device, stream)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    head_key = "fp8_block" if "fp8_block" in results else "fp8" if "fp8" in results else "nvfp4"
    head = results[head_key]
    line = {
        "metric": METRIC, "value": head["tflops"], "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "e2m1" if head_key == "nvfp4" else "e4m3", "data": "synthetic",
        "config": bench_config(head_key, args.size or SIZES[head_key], world),
        "overhead_pct": head["overhead_pct"], "unprotected_tflops": head["unprotected_tflops"],
        "roofline": head["roofline"], "clocks": head["clocks"],
        "gpu_launches": LAUNCHES_PER_STEP * args.steps,
        "e2e": head.get("e2e"), "detection": head.get("detection"), "fault_schedule": head.get("fault_schedule"),
        "thresholds": head["thresholds"], "row_checksums": head.get("row_checksums"),
    }
    if "exchanged_status" in head:
        line["exchanged_status"] = head["exchanged_status"]
    for key, name in (("fp8", "fp8_tensorwise"), ("nvfp4", "nvfp4")):
        if key in results and results[key] is not head:
            line[name] = results[key]
    if sweep is not None:
        line["qwen2.5_7b_linears"] = sweep
    if ceiling is not None:
        line["library_ceiling"] = ceiling
    if augmented is not None:
        line["augmented_bf16"] = augmented
    if not args.no_cpu_baseline and world == 1:
        line["cpu_baseline"] = cpu_baseline(args.cpu_sample_rows, args.size or SIZES[head_key])
    sys.stdout.flush()
    os.write(result_fd, (json.dumps(line) + "\n").encode())


def reference_operands(precision, size, rows):
    """The workload's operands as the reference's CPU path gets them: the same
    seeded bf16 matrices, quantised by the oracle's restatement of the format
    (bit-identical to the device quantiser) and dequantised to fp32. Returns
    (A rows [rows, K] fp32, B [K, N] fp32)."""
    import numpy as np

    from oracle import quant

    full_a, b = host_operands(size, size, size, SEEDS[precision])
    full_a = full_a.float().numpy()
    a = full_a[:rows]
    b = b.float().numpy()
    if precision == "fp8_block":
        ca, sa = quant.quantize_fp8_block(a, 1)
        cb, sb = quant.quantize_fp8_block(b, 128)
        da, db = quant.dequantize_fp8_block(ca, sa, 1), quant.dequantize_fp8_block(cb, sb, 128)
    elif precision == "fp8":
        # The multiplier of A is the whole matrix's: amax over all rows.
        ca, st_a = quant.quantize_fp8(a, float(quant.multiplier(full_a, "fp8")))
        cb, st_b = quant.quantize_fp8(b)
        da, db = quant.dequantize_fp8(ca, st_a), quant.dequantize_fp8(cb, st_b)
    else:
        ca, sa, st_a = quant.quantize_nvfp4(a, float(quant.multiplier(full_a, "nvfp4")))
        cb, sb, st_b = quant.quantize_nvfp4(b)
        da, db = quant.dequantize_nvfp4(ca, sa, st_a), quant.dequantize_nvfp4(cb, sb, st_b)
    return torch.from_numpy(np.ascontiguousarray(da, np.float32)), torch.from_numpy(
        np.ascontiguousarray(db.T, np.float32))


def cpu_baseline(rows, size, min_seconds=10.0):
    """The reference's CPU/torch ABFT path on rows of the headline workload's
    dequantised operands, repeated until about ``min_seconds`` of CPU work."""
    from oracle import cpu_path

    torch.set_num_threads(os.cpu_count() or 1)
    rows = min(rows, size)
    a, b = reference_operands("fp8_block", size, rows)
    cpu_path.execute(a[:64], b[:, :64], block_k=256)  # warm the BLAS
    calls = 0
    t0 = time.perf_counter()
    while True:
        _, report, _ = cpu_path.execute(a, b, atol=ATOL, rtol=CALIBRATED_RTOL["fp8_block"], block_k=256)
        calls += 1
        seconds = time.perf_counter() - t0
        if seconds >= min_seconds:
            break
    return {"value": 2.0 * rows * size * size * calls / seconds / 1e12, "unit": UNIT,
            "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"dequantised block-scaled fp32 {rows}x{size}x{size} ({rows} of the {size} rows of the "
                      f"headline workload, same seed), Classic, {calls} protected GEMMs in {seconds:.1f} s",
            "detected": report["detected"]}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    from oracle import cpu_path

    torch.set_num_threads(os.cpu_count() or 1)
    precision = "fp8_block" if args.format == "all" else args.format
    size = args.size or SIZES[precision]
    rows = min(args.cpu_sample_rows, size)
    a, b = reference_operands(precision, size, rows)
    rtol = CALIBRATED_RTOL[precision] if args.rtol is None else args.rtol
    for _ in range(args.warmup):
        cpu_path.execute(a, b, atol=ATOL, rtol=rtol)
    report = {"detected": False}
    t0 = time.perf_counter()
    for _ in range(args.steps):
        # Each step is a whole protected GEMM: prepare (the input-side
        # reference), collect and verify, as abft.execute does per call.
        _, report, _ = cpu_path.execute(a, b, atol=ATOL, rtol=rtol)
    seconds = (time.perf_counter() - t0) / max(args.steps, 1)
    value = 2.0 * rows * size * size / seconds / 1e12
    sample = (f"dequantised {FORMATS[precision][1].split(',')[0]} fp32 operands of the same seed, "
              f"{rows}x{size}x{size} ({rows} of the {size} rows of the workload) per step")
    print(json.dumps({
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": seconds * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic", "impl": "reference",
        "config": bench_config(precision, size, world),
        "reference_path": "abft.execute CPU path (reference_mm=torch.mm; the reference's only CPU implementation "
                          "computes the protected GEMM in fp32), restated in oracle/cpu_path.py",
        "thresholds": {"atol": ATOL, "rtol": rtol}, "clean_detected": report["detected"],
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# Qwen2.5-0.5B shapes (configuration 5): layers, hidden, intermediate, heads, KV heads, vocab.
QWEN05B = dict(num_hidden_layers=24, hidden_size=896, intermediate_size=4864, num_attention_heads=14,
               num_key_value_heads=2, vocab_size=151936, rope_theta=1e6, rms_norm_eps=1e-6,
               tie_word_embeddings=True, max_position_embeddings=32768)


def build_train_model(device, seed, layers=None, shapes=None, calibrate=False):
    """Random-init Qwen2 causal LM (transformers config, fp32 master weights)
    with every nn.Linear replaced by the protected NVFP4 linear."""
    from transformers import Qwen2Config, Qwen2ForCausalLM

    from sdc_b200.gemm.linear import install

    cfg = dict(QWEN05B if shapes is None else shapes)
    if layers is not None:
        cfg["num_hidden_layers"] = layers
    torch.manual_seed(seed)
    model = Qwen2ForCausalLM(Qwen2Config(**cfg, attn_implementation="sdpa")).to(device)
    # Detect and log (the configuration asks for detections per layer); no
    # recovery, so no GEMM waits on its own verdict and the host never syncs
    # inside the step.
    # Thresholds: the NVFP4 calibration (rtol, the clean residual of an fp32
    # accumulation is ~1e-9 of the magnitude) and no absolute floor, since
    # gradient GEMMs have outputs far below any fixed atol (a zero column has
    # a zero residual).
    abft = {"method": "classic", "implementation": "native", "reference_mode": "input_fused",
            "reference_layout": "kslice", "on_error": "report", "recovery": "none", "locate": True,
            "atol": 0.0, "rtol": TRAIN_RTOL}
    if calibrate:
        # threshold = magnitude: the reports' residual / threshold is the
        # clean |residual| / magnitude the relative tolerance must clear.
        abft.update(rtol=1.0, diagnostics=True)
    install(model, "nvfp4", "block16", abft_config=abft, report_max_records=4096)
    return model


def clean_ratio(report):
    """max |residual| / magnitude of a diagnostics report made with rtol 1, atol 0."""
    res, thr = report.tensors["residual"].abs(), report.tensors["threshold"]
    return float(torch.where(thr > 0, res / thr, torch.zeros_like(res)).max())


def train_reports(model):
    """(layer, role, detected, located, fault_hit) per protected GEMM call recorded since the last reset."""
    from sdc_b200.gemm.linear import ProtectedLinear

    protection = next(m.protection for m in model.modules() if isinstance(m, ProtectedLinear))
    rows = []
    for report in protection.reports:
        ctx = report.context
        rows.append((ctx.get("layer"), ctx.get("role"), bool(report.detected), bool(report.located),
                     int(report.fault_hit.reshape(-1)[0]) if report.fault_hit is not None else 0,
                     ctx.get("call_index")))
    protection.reports.clear()
    return protection, rows


def run_train(args):
    """Configuration 5: one data-parallel training step of a Qwen2.5-0.5B-shaped
    model with NVFP4 ABFT on every linear (forward, dgrad, wgrad GEMMs),
    synthetic uniform token ids, seeded Bernoulli accumulator faults per GEMM;
    detections are counted per layer and role. Prints one JSON line."""
    from sdc_b200.abft.config import parse_fault_config

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    result_fd = os.dup(1)
    os.dup2(2, 1)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
    model = build_train_model(device, 1234, calibrate=args.calibrate)
    if dist is not None:
        model = torch.nn.parallel.DistributedDataParallel(model, device_ids=[local])
    optimizer = torch.optim.AdamW(model.parameters(), lr=1e-4)
    batch, seq = args.micro_batch, args.seq_len
    g = torch.Generator(device=device).manual_seed(100 + rank)
    tokens = torch.randint(0, QWEN05B["vocab_size"], (batch, seq), device=device, generator=g)
    schedule = torch.Generator().manual_seed(7 + rank)
    stream = torch.cuda.current_stream(device)
    core = model.module if dist is not None else model
    gemms_per_step = None
    per_layer = {}
    faults = detected = 0
    fault_log = []

    def step():
        optimizer.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = model(input_ids=tokens, labels=tokens).loss
        loss.backward()
        optimizer.step()
        return loss

    def arm_faults(protection, first_call, count):
        # One seeded Bernoulli(rate) draw per GEMM of the coming step; the
        # session injects at most one fault per step (the first drawn).
        hits = (torch.rand(count, generator=schedule) < args.fault_rate).nonzero().flatten().tolist()
        if not hits:
            protection.fault = parse_fault_config(None)
            return None
        call = first_call + hits[0] + 1
        bit = int(torch.randint(0, 32, (1,), generator=schedule))
        protection.fault = parse_fault_config({"location": "accumulator",
                                               "row": int(torch.randint(0, 128, (1,), generator=schedule)),
                                               "col": int(torch.randint(0, 128, (1,), generator=schedule)),
                                               "bit": bit, "call_index": call})
        armed_bits[call] = bit
        return call

    losses = []
    armed_bits = {}
    ratios = {}  # role -> max clean |residual| / magnitude (--calibrate)
    for i in range(args.warmup + args.steps):
        protection, _ = train_reports(core)
        if gemms_per_step is not None and i >= args.warmup:
            faults += arm_faults(protection, protection.call_index, gemms_per_step) is not None
        if i == args.warmup:
            torch.cuda.synchronize()
            if dist is not None:
                dist.barrier()
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(stream)
        first = protection.call_index
        losses.append(step().detach())
        if args.calibrate:
            for report in protection.reports:
                role = report.context.get("role")
                ratios[role] = max(ratios.get(role, 0.0), clean_ratio(report))
        protection, rows = train_reports(core)
        gemms_per_step = protection.call_index - first
        if i >= args.warmup:
            for layer, role, det, loc, hit, call in rows:
                if det:
                    key = f"{layer}:{role}"
                    per_layer[key] = per_layer.get(key, 0) + 1
                    detected += 1
                if hit:
                    fault_log.append({"rank": rank, "step": i - args.warmup, "layer": layer, "role": role,
                                      "bit": armed_bits.get(call), "detected": det, "located": loc})
    end.record(stream)
    end.synchronize()
    elapsed = start.elapsed_time(end) / 1e3
    if dist is not None:
        t = torch.tensor([elapsed, faults, detected], device=device, dtype=torch.float64)
        dist.all_reduce(t[:1], op=dist.ReduceOp.MAX)
        dist.all_reduce(t[1:], op=dist.ReduceOp.SUM)
        elapsed, faults, detected = float(t[0]), int(t[1]), int(t[2])
        logs = [None] * world
        dist.all_gather_object(logs, (fault_log, per_layer, ratios))
        for _, _, r in logs:
            for role, value in r.items():
                ratios[role] = max(ratios.get(role, 0.0), value)
        fault_log = [entry for log, _, _ in logs for entry in log]
        per_layer = {}
        for _, counts, _ in logs:
            for key, value in counts.items():
                per_layer[key] = per_layer.get(key, 0) + value
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    tokens_per_step = batch * seq * world
    line = {"metric": "Qwen2.5-0.5B NVFP4 ABFT training step throughput",
            "value": tokens_per_step * args.steps / elapsed,
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": elapsed / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "e2m1", "data": "synthetic",
            "config": {"workload": "configuration 5: Qwen2.5-0.5B shapes (24 layers, hidden 896, intermediate 4864, "
                                   "14/2 heads of dim 64, vocab 151936), random init, uniform token ids",
                       "micro_batch": batch, "seq_len": seq, "parallelism": f"dp{world}",
                       "protected_gemms_per_step": gemms_per_step, "fault_rate_per_gemm": args.fault_rate},
            "thresholds": {"atol": 0.0, "rtol": 1.0 if args.calibrate else TRAIN_RTOL},
            "clean_max_res_over_magnitude": ratios if args.calibrate else None,
            "faults_injected": faults, "detections": detected, "detections_per_layer_role": per_layer,
            "faults": fault_log,
            "faults_detected": sum(entry["detected"] for entry in fault_log),
            "false_detections": detected - sum(entry["detected"] for entry in fault_log),
            "loss_first": float(losses[0]), "loss_last": float(losses[-1])}
    sys.stdout.flush()
    os.write(result_fd, (json.dumps(line) + "\n").encode())


def main():
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=300)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=["ours", "reference"], default="ours")
    parser.add_argument("--format", choices=["all", "fp8_block", "fp8", "nvfp4"], default="all",
                        help="fp8_block = config[1] (headline), fp8 = tensorwise FP8, nvfp4 = config[2]")
    parser.add_argument("--flips-per-bit", type=int, default=24)
    parser.add_argument("--schedule-gemms", type=int, default=1000)
    parser.add_argument("--rtol", type=float, default=None, help="override the calibrated relative threshold")
    parser.add_argument("--cpu-sample-rows", type=int, default=8192)
    parser.add_argument("--no-detection", action="store_true")
    parser.add_argument("--no-e2e", action="store_true")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-ceiling", action="store_true", help="skip the library GEMM anchors")
    parser.add_argument("--no-sweep", action="store_true", help="skip the Qwen2.5-7B linear-shape sweep")
    parser.add_argument("--sweep-steps", type=int, default=10)
    parser.add_argument("--no-augmented", action="store_true", help="skip the augmented BF16 ABFT leg")
    parser.add_argument("--no-rows", action="store_true",
                        help="skip the row-checksum (two-dimensional localisation) leg")
    parser.add_argument("--augmented-only", action="store_true",
                        help="run only the augmented BF16 leg and print its object (profiling; not a bench line)")
    parser.add_argument("--augmented-sizes", default="2048,8192")
    parser.add_argument("--augmented-iters", type=int, default=20)
    parser.add_argument("--workload", choices=["gemm", "train"], default="gemm",
                        help="gemm: the ABFT GEMM benchmark (default); train: configuration 5 training step")
    parser.add_argument("--micro-batch", type=int, default=8)
    parser.add_argument("--seq-len", type=int, default=2048)
    parser.add_argument("--fault-rate", type=float, default=1e-4)
    parser.add_argument("--calibrate", action="store_true",
                        help="train workload: no detection threshold, report the clean residual / magnitude")
    parser.add_argument("--size", type=int, default=0,
                        help="override M=N=K of the workloads (profiling captures and CPU tests; not a bench line)")
    parser.add_argument("--shape", default="",
                        help="M,N,K of the GEMM step (profiling captures at one layer's shard shape; not a bench line; "
                             "the end-to-end leg needs --no-e2e)")
    args = parser.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.augmented_only:
        device = torch.device("cuda", 0)
        torch.cuda.set_device(device)
        result = augmented_bf16(device, torch.cuda.current_stream(device),
                                tuple(int(x) for x in args.augmented_sizes.split(",")), args.augmented_iters)
        print(json.dumps({"augmented_bf16": result}))
    elif args.impl == "reference":
        run_reference(args)
    elif args.workload == "train":
        run_train(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
