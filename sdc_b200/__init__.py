"""sdc_b200 — B200-native (sm_100a) ABFT FP8/NVFP4 GEMM path of meiyou666/SDC.

The native libraries built in-tree by ``sdc_b200._build`` are loaded on first
use of ``sdc_b200.ops`` or ``require_device`` (the ``gemm`` and ``abft``
modules use them at import): ``libsdc_b200.so`` (kernels + C ABI,
include/sdc_b200.h) and ``_sdc_ops.so`` (the ``torch.ops.sdc_cutlass``
operator library with the reference's schemas). There is no CPU or
pure-PyTorch fallback: if the libraries are missing, that first use raises
with the build command to run.

Subpackages mirror the reference's Python API for this path:
  sdc_b200.gemm   <- src/cutlass_gemm (quantize, dequantize, backend.gemm)
  sdc_b200.abft   <- src/abft         (AbftConfig, execute, execute_prepared,
                                       PreparedGemm, Classic/Sum methods)
"""
from __future__ import annotations

from pathlib import Path

import torch

__all__ = ["LIB_PATH", "OPS_PATH", "load", "require_device", "ops"]

_HERE = Path(__file__).resolve().parent
LIB_PATH = _HERE / "libsdc_b200.so"
OPS_PATH = _HERE / "_sdc_ops.so"
_loaded = False


def load() -> None:
    """Registers torch.ops.sdc_cutlass from the in-tree operator library."""
    global _loaded
    if _loaded:
        return
    if not OPS_PATH.exists() or not LIB_PATH.exists():
        raise RuntimeError(
            "sdc_b200 native libraries are not built; run `python -m sdc_b200._build` "
            f"(expected {LIB_PATH.name} and {OPS_PATH.name} in {_HERE})")
    torch.ops.load_library(str(OPS_PATH))
    _loaded = True


def require_device(device) -> None:
    """Raises unless ``device`` is a CUDA sm_100 (B200) device."""
    device = torch.device(device)
    if device.type != "cuda" or not torch.cuda.is_available():
        raise RuntimeError("sdc_b200 kernels require an NVIDIA CUDA device")
    index = device.index if device.index is not None else torch.cuda.current_device()
    if torch.cuda.get_device_capability(index) != (10, 0):
        raise RuntimeError("sdc_b200 kernels are built for sm_100a (B200)")
    load()


def __getattr__(name):
    # ``sdc_b200.ops`` loads the libraries on first use (and raises with the
    # build command if they are missing); importing the package alone does
    # not, so ``python -m sdc_b200._build`` works on a fresh checkout.
    if name == "ops":
        load()
        return torch.ops.sdc_cutlass
    raise AttributeError(f"module 'sdc_b200' has no attribute {name!r}")
