"""In-tree build of the sdc_b200 native libraries.

Two shared objects are produced next to this file:

* ``libsdc_b200.so`` — every CUDA kernel and the C ABI declared in
  ``include/sdc_b200.h``, compiled by nvcc for sm_100a only. It links the
  CUDA runtime statically and reaches the driver's tensor-map encoder through
  ``cudaGetDriverEntryPoint``, so it has no torch or libcuda link dependency.
* ``_sdc_ops.so`` — the thin torch extension registering the reference's
  ``sdc_cutlass::*`` operator schemas on top of that ABI (loaded with
  ``torch.ops.load_library``; it has no Python module of its own).

Builds are incremental on source modification times, so importing the package
on a machine that received prebuilt objects never invokes a compiler.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
INCLUDE = ROOT / "include"
LIB = HERE / "libsdc_b200.so"
OPS = HERE / "_sdc_ops.so"

CUDA_SOURCES = [
    "status.cu",
    "finalize.cu",
    "quantize.cu",
    "tile_reference.cu",
    "gemm.cu",
    "api.cu",
    "locate.cu",
    "augmented.cu",
    "kslice.cu",
    "rowsum.cu",
]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    return str(Path(home) / "bin" / "nvcc")


def _stale(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return True
    built = target.stat().st_mtime
    return any(s.stat().st_mtime > built for s in sources)


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} (exit {proc.returncode})")
    if verbose and (proc.stdout or proc.stderr):
        sys.stderr.write(proc.stdout + proc.stderr)


def build_library(verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    headers = sorted(CSRC.glob("*.cuh")) + [INCLUDE / "sdc_b200.h"]
    sources = [CSRC / s for s in CUDA_SOURCES]
    objdir = ROOT / "_build" / "obj"
    objdir.mkdir(parents=True, exist_ok=True)
    objects = []
    procs = []
    for src in sources:
        obj = objdir / (src.stem + ".o")
        objects.append(obj)
        if _stale(obj, [src, *headers]) or ptxas_verbose:
            cmd = [_nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                   "--expt-relaxed-constexpr", "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
            if ptxas_verbose:
                cmd += ["-Xptxas", "-v"]
            if verbose:
                print(" ".join(cmd), flush=True)
            procs.append((cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)))
    failed = False
    for cmd, proc in procs:
        out, err = proc.communicate()
        if proc.returncode != 0 or ptxas_verbose or verbose:
            sys.stderr.write(out + err)
        failed |= proc.returncode != 0
    if failed:
        raise RuntimeError("nvcc failed")
    if _stale(LIB, objects):
        _run([_nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", str(LIB), *map(str, objects),
              "-cudart", "static"], verbose)
    return LIB


def build_ops(verbose: bool = False) -> Path:
    import torch
    from torch.utils import cpp_extension

    src = CSRC / "torch_ops.cpp"
    if not _stale(OPS, [src, INCLUDE / "sdc_b200.h", LIB]):
        return OPS
    includes = []
    for path in cpp_extension.include_paths("cuda"):
        includes += ["-isystem", path]
    libdirs = [f"-L{p}" for p in cpp_extension.library_paths("cuda")]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_API_INCLUDE_EXTENSION_H", "-DTORCH_EXTENSION_NAME=_sdc_ops",
           *includes, "-I", str(INCLUDE), str(src), "-o", str(OPS), *libdirs,
           f"-L{HERE}", "-lsdc_b200", "-Wl,-rpath,$ORIGIN",
           "-lc10", "-ltorch", "-ltorch_cpu", "-lc10_cuda", "-ltorch_cuda"]
    _run(cmd, verbose)
    return OPS


def build(verbose: bool = False) -> None:
    build_library(verbose)
    build_ops(verbose)


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
    if "--ptxas" in sys.argv:
        build_library(verbose=False, ptxas_verbose=True)
