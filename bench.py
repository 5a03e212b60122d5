#!/usr/bin/env python
"""Benchmark of the ABFT-protected FP8 / NVFP4 GEMM path on B200.

Metric: ABFT NVFP4/FP8 GEMM TFLOPS, % overhead vs the
unprotected kernel, detection recall. One step = one protected GEMM on
operands already quantised and resident in HBM: the input-fused ABFT GEMM
(tcgen05 mainloop, fused observed-checksum epilogue, input-side prediction in
the K-slice layout) followed by the device finalize that merges partials and
decides. Throughput counts only the useful 2*M*N*K flops.

Headline workload (config[1]): FP8 e4m3, M=N=K=8192, 1 x 128 (A) and
128 x 128 (B) fp32 block scales, fp32 accumulation, bf16 output. Measured in
the same run: the NVFP4 workload of config[2] (M=N=K=16384, e2m1 + ue4m3/16 +
fp32 global scale, bf16 out) under "nvfp4", and the reference's own FP8
semantics (tensorwise scale, fp32 output) at 8192^3 under "fp8_tensorwise".

Multi-GPU (python -m torch.distributed.run ... bench.py --gpus N): each rank
protects its own M-shard (8192 rows x N=K=8192, weak scaling: the job's M is
8192*N) and the ranks all-reduce (MAX) their detection status words over
NCCL after every step, the path's only exchange. Time is the max over ranks.

--impl reference times the reference's own CPU/torch ABFT path (restated in
oracle/cpu_path.py, bit-identical to it) on this host's cores instead.
"""
from __future__ import annotations

import argparse
import json
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


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return data["bf16_tflops"], data["hbm_gbs"], "measured"
    return 1590.0, 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled during the timed region."""

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
        time.sleep(0.15)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
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


# Workload formats: (quantisation precision, bench key, description).
FORMATS = {"fp8_block": ("fp8", "fp8 block-scaled 1x128 / 128x128, bf16 out"),
           "fp8": ("fp8", "fp8 tensorwise, fp32 out"),
           "nvfp4": ("nvfp4", "nvfp4 block16, bf16 out")}


def make_operands(precision, m, n, k, device, seed, b_std=1.0):
    """Seeded N(0,1) bf16 A [m,k] and B_rows [n,k] (synthetic, BASELINE shapes) quantised once."""
    from sdc_b200.gemm.quantization import quantize, quantize_blockwise

    g = torch.Generator(device=device).manual_seed(seed)
    a = torch.randn(m, k, device=device, generator=g, dtype=torch.bfloat16)
    b = torch.randn(n, k, device=device, generator=g, dtype=torch.bfloat16)
    if b_std != 1.0:
        b = b * b_std
    if precision == "fp8_block":
        qa, qb = quantize_blockwise(a, 1), quantize_blockwise(b, 128)
        return (qa.codes.view(torch.float8_e4m3fn), qb.codes.view(torch.float8_e4m3fn), qa.scales, qb.scales)
    qa, qb = quantize(a, precision), quantize(b, precision)
    alpha = (qa.multiplier * qb.multiplier).reciprocal()
    if precision == "fp8":
        args = (qa.codes.view(torch.float8_e4m3fn), qb.codes.view(torch.float8_e4m3fn), alpha)
    else:
        args = (qa.codes, qb.codes, qa.scales_mma, qb.scales_mma, k, alpha)
    del a, b
    return args


class Protected:
    """One protected GEMM step on resident operands (the hot path)."""

    def __init__(self, precision, m, n, k, device, seed, layout=1, atol=1e-3, rtol=1e-4, b_std=1.0):
        self.ops = torch.ops.sdc_cutlass
        self.precision, self.m, self.n, self.k = precision, m, n, k
        self.args = make_operands(precision, m, n, k, device, seed, b_std)
        self.weights = torch.stack((torch.ones(m, device=device),
                                    torch.arange(1, m + 1, device=device, dtype=torch.float32)))
        self.nonfinite = torch.zeros(1, dtype=torch.int32, device=device)
        self.atol, self.rtol = atol, rtol
        ops = self.ops
        if precision == "fp8_block":  # K-slice is the block-scaled op's only layout
            self.fused, self.observe, self.plain = (ops.abft_fp8_block_reference_mm, ops.abft_fp8_block_mm,
                                                    ops.fp8_block_mm)
            self.layout_args = ()
        else:
            self.fused = ops.abft_fp8_reference_mm if precision == "fp8" else ops.abft_nvfp4_reference_mm
            self.observe = ops.abft_fp8_mm if precision == "fp8" else ops.abft_nvfp4_mm
            self.plain = ops.fp8_mm if precision == "fp8" else ops.nvfp4_mm
            self.layout_args = (layout,)

    def step(self, fault=(-1, -1, -1)):
        out, obs, hit, pred, mag = self.fused(*self.args, self.weights, *fault, 0, self.nonfinite, *self.layout_args)
        packet = self.ops.abft_finalize_reference(obs, pred, mag, hit, self.nonfinite, self.n, self.atol,
                                                  self.rtol, None, True)
        return out, packet

    def unprotected(self):
        return self.plain(*self.args)

    def gemm_only(self):
        return self.observe(*self.args, self.weights, -1, -1, -1)

    def fused_only(self):
        """The step's dominant kernel alone: the protected GEMM without finalize."""
        return self.fused(*self.args, self.weights, -1, -1, -1, 0, self.nonfinite, *self.layout_args)


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


def profiled_traffic(name):
    """DRAM bytes (read + write) of one protected-GEMM launch from the committed
    ncu summary (first value column of its full-capture table), or None."""
    import re

    path = ROOT / "profiles" / name
    if not path.exists():
        return None
    total = 0.0
    for metric in ("dram__bytes_read.sum", "dram__bytes_write.sum"):
        m = re.search(rf"\| {re.escape(metric)} \| ([0-9.]+) MB", path.read_text())
        if m is None:
            return None
        total += float(m.group(1)) * 1e6
    return total


# Kernels this library launches per protected step: the K-slice projection
# of A (kslice_project + kslice_band_sum), the GEMM (prediction fused into
# it), finalize_columns + finalize_flags.
LAUNCHES_PER_STEP = 5


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


def detection_campaign(prot, flips, seed):
    """Seeded single-bit accumulator flips (bits 23-30 exponent, 20-22 high
    mantissa) at uniform (row, col); recall over all flips and over flips
    whose checksum perturbation exceeds the threshold."""
    g = torch.Generator().manual_seed(seed)
    clean_out, clean_packet = prot.step()
    residual0 = clean_packet[1].clone()
    threshold0 = clean_packet[2].clone()
    detected = detectable = 0
    by_class = {"exponent": [0, 0], "high_mantissa": [0, 0]}
    for _ in range(flips):
        row = int(torch.randint(0, prot.m, (1,), generator=g))
        col = int(torch.randint(0, prot.n, (1,), generator=g))
        bit = int(torch.randint(20, 31, (1,), generator=g))
        _, packet = prot.step((row, col, bit))
        flags = packet[3].tolist()
        hit = bool(flags[0])
        # Detectable: the flip's own checksum perturbation exceeds the clean threshold.
        delta = (packet[1][:, col] - residual0[:, col]).abs()
        can = bool((delta > threshold0[:, col]).any()) or bool(flags[1])
        detected += hit
        detectable += can
        cls = "exponent" if bit >= 23 else "high_mantissa"
        by_class[cls][0] += hit
        by_class[cls][1] += 1
    clean_runs = 8
    false_positives = sum(bool(prot.step()[1][3][0]) for _ in range(clean_runs))
    return {"flips": flips, "detected": detected, "detectable": detectable,
            "recall_all": detected / max(flips, 1), "recall_detectable": min(detected, detectable) / max(detectable, 1),
            "by_class": {k: {"detected": v[0], "flips": v[1]} for k, v in by_class.items()},
            "clean_runs": clean_runs + 1, "false_positives": false_positives + int(bool(clean_packet[3][0])),
            "schedule": fault_schedule(prot, residual0, threshold0, seed)}


def fault_schedule(prot, residual0, threshold0, seed, gemms=1000, rate=1e-3):
    """The configurations' schedule: ``gemms`` protected GEMMs, each carrying
    one seeded accumulator flip with probability ``rate`` (uniform row,
    column and bit in [0, 32)); every GEMM's verdict is read back."""
    g = torch.Generator().manual_seed(seed + 7919)
    faulted = detected = detectable = false_positives = 0
    for _ in range(gemms):
        fault = (-1, -1, -1)
        if float(torch.rand((), generator=g)) < rate:
            fault = (int(torch.randint(0, prot.m, (1,), generator=g)), int(torch.randint(0, prot.n, (1,), generator=g)),
                     int(torch.randint(0, 32, (1,), generator=g)))
        _, packet = prot.step(fault)
        flag = bool(packet[3][0])
        if fault[0] < 0:
            false_positives += flag
            continue
        faulted += 1
        detected += flag
        col = fault[1]
        delta = (packet[1][:, col] - residual0[:, col]).abs()
        detectable += bool((delta > threshold0[:, col]).any()) or bool(packet[3][1])
    return {"gemms": gemms, "rate": rate, "faulted": faulted, "detected": detected, "detectable": detectable,
            "false_positives": false_positives, "clean": gemms - faulted}


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
            prot = Protected(precision, stop - start, n, k, device, 7 + rank, b_std=0.02)
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


def e2e_step(precision, a, b, weights, nonfinite, atol, rtol):
    """Public-API protected GEMM on device bf16 operands (quantise, protected
    GEMM, finalize); returns the flags packet tensor and the output."""
    from sdc_b200.gemm.quantization import quantize, quantize_blockwise

    ops = torch.ops.sdc_cutlass
    if precision == "fp8_block":
        qa, qb = quantize_blockwise(a, 1), quantize_blockwise(b, 128)
        res = ops.abft_fp8_block_reference_mm(qa.codes.view(torch.float8_e4m3fn), qb.codes.view(torch.float8_e4m3fn),
                                              qa.scales, qb.scales, weights, -1, -1, -1, 0, nonfinite)
    else:
        qa, qb = quantize(a, precision), quantize(b, precision)
        alpha = (qa.multiplier * qb.multiplier).reciprocal()
        if precision == "fp8":
            res = ops.abft_fp8_reference_mm(qa.codes.view(torch.float8_e4m3fn), qb.codes.view(torch.float8_e4m3fn),
                                            alpha, weights, -1, -1, -1, 0, nonfinite, 1)
        else:
            res = ops.abft_nvfp4_reference_mm(qa.codes, qb.codes, qa.scales_mma, qb.scales_mma, a.shape[1], alpha,
                                              weights, -1, -1, -1, 0, nonfinite, 1)
    out, obs, hit, pred, mag = res
    packet = ops.abft_finalize_reference(obs, pred, mag, hit, nonfinite, b.shape[0], atol, rtol, None, False)
    return packet[3], out


def e2e_run(precision, host_a, host_b, device, weights, nonfinite, atol, rtol, steps, stream):
    """``steps`` end-to-end protected GEMMs from pinned host bf16 operands:
    each step copies its A and B to the device (on a copy stream, one step
    ahead, into one of two buffer sets) and reads its flags back to pinned
    host memory. Returns seconds per step (CUDA events on the compute stream)."""
    copy = torch.cuda.Stream(device)
    dev_a = [torch.empty_like(host_a, device=device) for _ in range(2)]
    dev_b = [torch.empty_like(host_b, device=device) for _ in range(2)]
    flags_host = torch.empty((steps, 5), dtype=torch.bool).pin_memory()
    copied = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]

    def issue_copy(i):
        slot = i % 2
        with torch.cuda.stream(copy):
            if i >= 2:
                copy.wait_event(free[slot])
            dev_a[slot].copy_(host_a, non_blocking=True)
            dev_b[slot].copy_(host_b, non_blocking=True)
            copied[slot].record(copy)

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record(stream)
    with torch.cuda.stream(copy):
        copy.wait_event(start)
    issue_copy(0)
    for i in range(steps):
        if i + 1 < steps:
            issue_copy(i + 1)
        slot = i % 2
        stream.wait_event(copied[slot])
        flags, _ = e2e_step(precision, dev_a[slot], dev_b[slot], weights, nonfinite, atol, rtol)
        free[slot].record(stream)
        flags_host[i].copy_(flags, non_blocking=True)
    end.record(stream)
    end.synchronize()
    assert not flags_host[:, 0].any(), "a clean end-to-end run was flagged"
    return start.elapsed_time(end) / 1e3 / steps


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
    for precision, size, seed in (("fp8_block", args.size or 8192, 1), ("fp8", args.size or 8192, 3),
                                  ("nvfp4", args.size or 16384, 2)):
        if args.format not in ("all", precision):
            continue
        m = n = k = size
        prot = Protected(precision, m, n, k, device, seed + 1000 * rank)
        flops = 2.0 * m * n * k
        status = torch.zeros(2, dtype=torch.int32, device=device)

        def step():
            _, packet = prot.step()
            if dist is not None:
                status[0] = packet[3][0].to(torch.int32)
                status[1] = packet[4][0]
                dist.all_reduce(status, op=dist.ReduceOp.MAX)

        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        with ClockSampler(local) as clocks:
            elapsed = timed(step, args.steps, 0, stream)
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
        profile = {("fp8_block", 8192): "gemm_fp8block_8192_abft.md",
                   ("fp8", 8192): "gemm_fp8_8192_abft.md"}.get((precision, size))
        entry = {
            "workload": f"{FORMATS[precision][1].split(' ', 1)[0]} M=N=K={size} {FORMATS[precision][1].split(' ', 1)[1]}",
            "tflops": world * flops / per_step / 1e12,
            "ms_per_step": per_step * 1e3,
            "unprotected_tflops": flops / plain_paired / 1e12,
            "overhead_pct": 100.0 * (step_paired / plain_paired - 1.0),
            "overhead_method": "paired alternating blocks of protected (GEMM + finalize) and unprotected steps",
            "roofline": {"bound": "tensor", "achieved": flops / (t_fused / args.steps) / 1e12, "peak": peak,
                         "unit": "TFLOP/s", "frac": flops / (t_fused / args.steps) / 1e12 / peak,
                         "kernel": "protected GEMM (gemm_kernel with checksums, projection and prediction)",
                         "traffic": profiled_traffic(profile) if profile else None,
                         "traffic_source": f"profiles/{profile} (ncu dram bytes of one launch)" if profile else None,
                         "algorithmic_flops": flops,
                         "peak_basis": f"{2 if fp8 else 4}x {basis} bf16 dense burst "
                                       f"({bf16_peak} TFLOP/s); nominal dense {4500 if fp8 else 9000}"},
            "clocks": clocks.summary(),
        }
        if rank == 0 and not args.no_detection:
            entry["detection"] = detection_campaign(prot, args.flips, seed)
        if not args.no_e2e:  # every rank: its own shard end to end, time = max over ranks
            host_a = torch.randn(m, k, dtype=torch.bfloat16).pin_memory()
            host_b = torch.randn(n, k, dtype=torch.bfloat16).pin_memory()
            w = prot.weights
            e2e_run(precision, host_a, host_b, device, w, prot.nonfinite, prot.atol, prot.rtol, 3, stream)  # warm-up
            e_steps = max(3, args.steps // 4)
            t0 = time.perf_counter()
            e_time = e2e_run(precision, host_a, host_b, device, w, prot.nonfinite, prot.atol, prot.rtol, e_steps,
                             stream)
            if dist is not None:
                t = torch.tensor([e_time], device=device)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                e_time = float(t.item())
            entry["e2e"] = {"value": world * flops / e_time / 1e12, "unit": UNIT,
                            "h2d_bytes_per_step": world * (host_a.numel() * 2 + host_b.numel() * 2),
                            "d2h_bytes_per_step": world * 5, "host_wall_s_per_step": (time.perf_counter() - t0) / e_steps,
                            "pipeline": "step i+1's host-to-device copies overlap step i's compute (two buffer sets)"}
        results[precision] = entry
        del prot
        torch.cuda.empty_cache()
    sweep = None if args.no_sweep else qwen_sweep(args, device, stream, rank, world, dist)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    head = results.get("fp8_block") or results.get("fp8") or results["nvfp4"]
    line = {
        "metric": METRIC, "value": head["tflops"], "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "e2m1" if head is results.get("nvfp4") else "e4m3", "data": "synthetic",
        "config": {"workload": head["workload"] + " ABFT (Classic, K-slice input reference) + finalize",
                   "per_gpu": head["workload"].split(" ")[1],
                   "parallelism": f"M-shard x{world}, NCCL all-reduce of detection status",
                   "l2": "working set (A+B codes, output) > 126 MB L2; no explicit flush"},
        "overhead_pct": head["overhead_pct"], "unprotected_tflops": head["unprotected_tflops"],
        "roofline": head["roofline"], "clocks": head["clocks"],
        "gpu_launches": LAUNCHES_PER_STEP * args.steps,
        "e2e": head.get("e2e"), "detection": head.get("detection"),
    }
    for key, name in (("fp8", "fp8_tensorwise"), ("nvfp4", "nvfp4")):
        if key in results and results[key] is not head:
            line[name] = results[key]
    if sweep is not None:
        line["qwen2.5_7b_linears"] = sweep
    if not args.no_cpu_baseline and world == 1:
        line["cpu_baseline"] = cpu_baseline(args.cpu_sample_rows)
    sys.stdout.flush()
    os.write(result_fd, (json.dumps(line) + "\n").encode())


def cpu_baseline(rows, min_seconds=10.0):
    """The reference's CPU/torch ABFT path on rows of the 8192^3 workload
    (all 8192 by default), repeated until about ``min_seconds`` of CPU work."""
    from oracle import cpu_path

    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(0)
    k = n = 8192
    a = torch.randn(rows, k, generator=g)
    b = torch.randn(k, n, generator=g)
    cpu_path.execute(a[:64], b[:, :64], block_k=256)  # warm the BLAS
    calls = 0
    t0 = time.perf_counter()
    while True:
        _, report, _ = cpu_path.execute(a, b, atol=1e-3, rtol=1e-4, block_k=256)
        calls += 1
        seconds = time.perf_counter() - t0
        if seconds >= min_seconds:
            break
    return {"value": 2.0 * rows * n * k * calls / seconds / 1e12, "unit": UNIT, "cores": torch.get_num_threads(),
            "kind": "port", "sample": f"fp32 {rows}x{n}x{k} ({rows} of the 8192 rows of the workload), Classic, "
                                      f"{calls} protected GEMMs in {seconds:.1f} s",
            "detected": report["detected"]}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import cpu_path

    torch.set_num_threads(os.cpu_count() or 1)
    rows, k, n = args.cpu_sample_rows, 8192, 8192
    g = torch.Generator().manual_seed(0)
    a = torch.randn(rows, k, generator=g)
    b = torch.randn(k, n, generator=g)
    for _ in range(max(1, min(args.warmup, 2))):
        cpu_path.execute(a, b, atol=1e-3, rtol=1e-4)
    steps = max(1, min(args.steps, 5))
    t0 = time.perf_counter()
    for _ in range(steps):
        cpu_path.execute(a, b, atol=1e-3, rtol=1e-4)
    seconds = (time.perf_counter() - t0) / steps
    value = 2.0 * rows * n * k / seconds / 1e12
    sample = f"fp32 {rows}x{n}x{k} ({rows} of the 8192 rows of the workload) per step"
    print(json.dumps({
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
        "steps": steps, "warmup": args.warmup, "ms_per_step": seconds * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic", "impl": "reference",
        "config": {"workload": "fp8 M=N=K=8192 block-scaled 1x128 / 128x128, bf16 out"
                               " ABFT (Classic, K-slice input reference) + finalize",
                   "reference_path": "abft.execute CPU path (reference_mm=torch.mm; the reference's only CPU "
                                     "implementation computes the protected GEMM in fp32), restated in "
                                     "oracle/cpu_path.py"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# Qwen2.5-0.5B shapes (configuration 5): layers, hidden, intermediate, heads, KV heads, vocab.
QWEN05B = dict(num_hidden_layers=24, hidden_size=896, intermediate_size=4864, num_attention_heads=14,
               num_key_value_heads=2, vocab_size=151936, rope_theta=1e6, rms_norm_eps=1e-6,
               tie_word_embeddings=True, max_position_embeddings=32768)


def build_train_model(device, seed, layers=None, shapes=None):
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
    abft = {"method": "classic", "implementation": "native", "reference_mode": "input_fused",
            "reference_layout": "kslice", "on_error": "report", "recovery": "none", "locate": True,
            "atol": 1e-3, "rtol": 1e-4}
    install(model, "nvfp4", "block16", abft_config=abft, report_max_records=4096)
    return model


def train_reports(model):
    """(layer, role, detected, located, fault_hit) per protected GEMM call recorded since the last reset."""
    from sdc_b200.gemm.linear import ProtectedLinear

    protection = next(m.protection for m in model.modules() if isinstance(m, ProtectedLinear))
    rows = []
    for report in protection.reports:
        ctx = report.context
        rows.append((ctx.get("layer"), ctx.get("role"), bool(report.detected), bool(report.located),
                     int(report.fault_hit.reshape(-1)[0]) if report.fault_hit is not None else 0))
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
    model = build_train_model(device, 1234)
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
        protection.fault = parse_fault_config({"location": "accumulator", "row": int(torch.randint(0, 128, (1,), generator=schedule)),
                                               "col": int(torch.randint(0, 128, (1,), generator=schedule)),
                                               "bit": bit, "call_index": call})
        return call

    losses = []
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
        protection, rows = train_reports(core)
        gemms_per_step = protection.call_index - first
        if i >= args.warmup:
            for layer, role, det, loc, hit in rows:
                if det:
                    key = f"{layer}:{role}"
                    per_layer[key] = per_layer.get(key, 0) + 1
                    detected += 1
    end.record(stream)
    end.synchronize()
    elapsed = start.elapsed_time(end) / 1e3
    if dist is not None:
        t = torch.tensor([elapsed, faults, detected], device=device, dtype=torch.float64)
        dist.all_reduce(t[:1], op=dist.ReduceOp.MAX)
        dist.all_reduce(t[1:], op=dist.ReduceOp.SUM)
        elapsed, faults, detected = float(t[0]), int(t[1]), int(t[2])
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    tokens_per_step = batch * seq * world
    line = {"metric": "Qwen2.5-0.5B NVFP4 ABFT training step throughput", "value": tokens_per_step * args.steps / elapsed,
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": elapsed / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "e2m1", "data": "synthetic",
            "config": {"workload": "configuration 5: Qwen2.5-0.5B shapes (24 layers, hidden 896, intermediate 4864, "
                                   "14/2 heads of dim 64, vocab 151936), random init, uniform token ids",
                       "micro_batch": batch, "seq_len": seq, "parallelism": f"dp{world}",
                       "protected_gemms_per_step": gemms_per_step, "fault_rate_per_gemm": args.fault_rate},
            "faults_injected": faults, "detections": detected, "detections_per_layer_role": per_layer,
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
    parser.add_argument("--flips", type=int, default=64)
    parser.add_argument("--cpu-sample-rows", type=int, default=8192)
    parser.add_argument("--no-detection", action="store_true")
    parser.add_argument("--no-e2e", action="store_true")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-sweep", action="store_true", help="skip the Qwen2.5-7B linear-shape sweep")
    parser.add_argument("--sweep-steps", type=int, default=10)
    parser.add_argument("--workload", choices=["gemm", "train"], default="gemm",
                        help="gemm: the ABFT GEMM benchmark (default); train: configuration 5 training step")
    parser.add_argument("--micro-batch", type=int, default=8)
    parser.add_argument("--seq-len", type=int, default=2048)
    parser.add_argument("--fault-rate", type=float, default=1e-4)
    parser.add_argument("--size", type=int, default=0,
                        help="override M=N=K of both workloads (profiling captures; not a bench line)")
    args = parser.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "train":
        run_train(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
