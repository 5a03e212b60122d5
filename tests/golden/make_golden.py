"""Regenerates the committed golden fixtures in this directory.

Run in a container that has the reference checkout (meiyou666/SDC) and
nvcc; the fixtures it writes are small JSON files the tests read, so neither
the reference nor a compiler is needed where the tests run.

* sf_layout.json      CUTLASS Sm1xxBlkScaledConfig<16> scale-factor byte
                      offsets (the layout the reference's nvfp4 operators
                      use), evaluated by sf_layout_golden.cu against the CuTe
                      headers vendored in this image.
* config1_trials.json The reference's own CPU ABFT path (abft.execute with
                      reference_mm=torch.mm and the CPU collector of its
                      tests/abft/test_framework.py) on BASELINE config 1:
                      1024^3 fp32, A and B uniform[-1, 1] from seed 0,
                      Classic, atol 0, rtol 1e-5; 50 clean trials and 50
                      accumulator bit flips with (row, col) uniform and bit in
                      20..30 drawn from seed 1. One record per trial.
* engine_cases.json   Small reference runs: detection/location outcomes of the
                      reference engine for seeded 64x96x80 problems.

Usage: python tests/golden/make_golden.py --reference /path/to/SDC
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent


def sf_layout(cutlass_include: str) -> None:
    with tempfile.TemporaryDirectory() as tmp:
        exe = Path(tmp) / "sf_golden"
        subprocess.run(["nvcc", "-std=c++17", "-Wno-deprecated-gpu-targets", "-I", cutlass_include,
                        str(HERE / "sf_layout_golden.cu"), "-o", str(exe)], check=True)
        data = json.loads(subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout)
    (HERE / "sf_layout.json").write_text(json.dumps(data))


def reference_trials(reference: Path) -> None:
    sys.path.insert(0, str(reference / "src"))
    import torch
    from abft.engine import execute  # the reference's engine

    def collect(operands, weights, fault):
        # The reference's CPU collector (tests/abft/test_framework.py:14-22).
        a, b = operands.decode_block(0, operands.k)
        output = a @ b
        row, col, bit = fault
        if row >= 0:
            mask = 1 << bit if bit < 31 else -(1 << 31)
            output.view(torch.int32)[row, col] ^= mask
        return output, (weights @ output).unsqueeze(1), torch.tensor([int(row >= 0)])

    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(0)
    a = torch.rand(1024, 1024, generator=g) * 2 - 1
    b = torch.rand(1024, 1024, generator=g) * 2 - 1
    fg = torch.Generator().manual_seed(1)
    cfg = {"method": "classic", "atol": 0.0, "rtol": 1e-5, "diagnostics": True, "on_error": "report"}
    trials = []
    for i in range(100):
        fault = None
        if i >= 50:
            row = int(torch.randint(0, 1024, (1,), generator=fg))
            col = int(torch.randint(0, 1024, (1,), generator=fg))
            bit = int(torch.randint(20, 31, (1,), generator=fg))
            fault = {"location": "accumulator", "row": row, "col": col, "bit": bit}
        out, report = execute(a, b, "fp32", "none", abft_config=cfg, fault_config=fault,
                              reference_mm=torch.mm, collector_fn=collect)
        rec = report.to_record()
        residual = report.tensors["residual"]
        threshold = report.tensors["threshold"]
        trials.append({
            "fault": fault,
            "detected": bool(rec["detected"]),
            "nonfinite": bool(rec["nonfinite"]),
            "located": bool(rec["located"]),
            "location": rec["location"],
            "max_ratio": float((residual.abs() / threshold).max()),
        })
    (HERE / "config1_trials.json").write_text(json.dumps({
        "shape": [1024, 1024, 1024], "seed": 0, "fault_seed": 1, "atol": 0.0, "rtol": 1e-5,
        "trials": trials}, indent=1))


def engine_cases(reference: Path) -> None:
    sys.path.insert(0, str(reference / "src"))
    import torch
    from abft.engine import execute

    def collect(operands, weights, fault):
        a, b = operands.decode_block(0, operands.k)
        output = a @ b
        row, col, bit = fault
        if row >= 0:
            mask = 1 << bit if bit < 31 else -(1 << 31)
            output.view(torch.int32)[row, col] ^= mask
        return output, (weights @ output).unsqueeze(1), torch.tensor([int(row >= 0)])

    cases = []
    for seed in range(12):
        g = torch.Generator().manual_seed(100 + seed)
        a = torch.randn(64, 80, generator=g)
        b = torch.randn(80, 96, generator=g)
        fault = None
        if seed % 3:
            fault = {"location": "accumulator", "row": (7 * seed) % 64, "col": (11 * seed) % 96,
                     "bit": [31, 30, 26, 22, 29, 23][seed % 6]}
        cfg = {"method": "classic", "atol": 1e-4, "rtol": 1e-4, "diagnostics": True, "on_error": "report",
               "reference_block_k": 32, "recovery": "recompute"}
        out, report = execute(a, b, "fp32", "none", abft_config=cfg, fault_config=fault,
                              reference_mm=torch.mm, collector_fn=collect)
        rec = report.to_record()
        cases.append({"seed": 100 + seed, "fault": fault, "detected": bool(rec["detected"]),
                      "located": bool(rec["located"]), "location": rec["location"],
                      "recovered": bool(rec["recovered"])})
    (HERE / "engine_cases.json").write_text(json.dumps(cases, indent=1))


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, type=Path)
    parser.add_argument("--cutlass-include", default=str(
        Path(sys.prefix) / "lib/python3.12/site-packages/flashinfer/data/cutlass/include"))
    args = parser.parse_args()
    sf_layout(args.cutlass_include)
    reference_trials(args.reference)
    engine_cases(args.reference)


if __name__ == "__main__":
    main()
