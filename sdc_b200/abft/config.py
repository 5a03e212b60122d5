"""ABFT configuration dataclasses.

Mirrors src/abft/config.py of the reference: the same fields, defaults,
validation rules and strict unknown-key rejection, so YAML/dict configs
written for the reference parse unchanged. Extensions (all defaulted to the
reference's behaviour):

* ``reference_layout``: ``"tile"`` (the reference's per-M-tile predicted
  partials, bit-identical) or ``"kslice"`` (same totals, computed inside the
  GEMM; see the K-slice layout in include/sdc_b200.h).
* ``locate``: run the device Classic locator on native executions (the
  reference's native finalizer never localises).
* ``recovery="correct"``: recompute only the located output element, falling
  back to the reference's full recompute when no single element is located.
"""
from __future__ import annotations

import json
import math
from collections.abc import Mapping
from dataclasses import dataclass, field, fields


def _json_safe(value):
    if isinstance(value, dict):
        if not all(isinstance(key, str) for key in value):
            raise ValueError("ABFT parameters require string dictionary keys")
        for child in value.values():
            _json_safe(child)
    elif isinstance(value, (list, tuple)):
        for child in value:
            _json_safe(child)


@dataclass(frozen=True)
class AbftConfig:
    method: str = "none"
    atol: float = 1e-4
    rtol: float = 1e-4
    recovery: str = "none"
    on_error: str = "raise"
    reference_block_k: int = 256
    diagnostics: bool = False
    timing: bool = False
    reference_mode: str = "separate"
    threshold_scale: str = "input"
    implementation: str = "reference"
    parameters: dict = field(default_factory=dict)
    reference_layout: str = "tile"
    locate: bool = False
    row_checksums: bool = False

    def __post_init__(self):
        if not isinstance(self.parameters, dict):
            raise ValueError("ABFT parameters must be a string-key dictionary")
        try:
            json.dumps(self.parameters, allow_nan=False)
            _json_safe(self.parameters)
        except (TypeError, ValueError, OverflowError, RecursionError) as error:
            raise ValueError("ABFT parameters must contain finite JSON-serializable values and string keys") from error
        if self.reference_mode not in {"separate", "input_fused", "augmented"}:
            raise ValueError("reference_mode must be separate, input_fused or augmented")
        if self.reference_mode in {"input_fused", "augmented"} and self.method == "none":
            raise ValueError("input_fused/augmented requires an ABFT method")
        needed = "output" if self.reference_mode == "augmented" else "input"
        if self.threshold_scale != needed:
            raise ValueError(f"{self.reference_mode} requires threshold_scale={needed}")
        if self.implementation not in {"reference", "native"}:
            raise ValueError("implementation must be reference or native")
        if self.implementation == "native" and self.method == "none":
            raise ValueError("native implementation requires an ABFT method")
        if not isinstance(self.method, str) or not self.method:
            raise ValueError("ABFT method must be a nonempty registered name")
        for value in (self.atol, self.rtol):
            if isinstance(value, bool) or not isinstance(value, (int, float)) or not math.isfinite(value) or value < 0:
                raise ValueError("ABFT tolerances must be finite and nonnegative")
        if self.recovery not in {"none", "recompute", "correct"} or self.on_error not in {"raise", "report"}:
            raise ValueError("Invalid ABFT recovery/on_error policy")
        if type(self.reference_block_k) is not int or self.reference_block_k <= 0 or self.reference_block_k % 16:
            raise ValueError("reference_block_k must be a positive multiple of 16")
        for name in ("diagnostics", "timing", "locate", "row_checksums"):
            if type(getattr(self, name)) is not bool:
                raise ValueError(f"{name} must be boolean")
        if self.row_checksums and (self.implementation != "native" or self.reference_mode != "input_fused"):
            raise ValueError("row_checksums needs the native input_fused execution")
        if self.reference_layout not in {"tile", "kslice"}:
            raise ValueError("reference_layout must be tile or kslice")


@dataclass(frozen=True)
class FaultConfig:
    location: str = "none"
    row: int = 0
    col: int = 0
    bit: int = 0
    call_index: int = 1
    layer: str | None = None
    role: str | None = None

    def __post_init__(self):
        if self.location not in {"none", "a", "b", "accumulator"}:
            raise ValueError("Invalid fault location")
        for name in ("row", "col", "bit", "call_index"):
            value = getattr(self, name)
            if type(value) is not int or value < (1 if name == "call_index" else 0):
                raise ValueError(f"Invalid fault {name}")
        for name in ("layer", "role"):
            if getattr(self, name) is not None and not isinstance(getattr(self, name), str):
                raise ValueError(f"fault {name} must be a string or None")
        if self.role is not None and self.role not in {"forward", "dgrad", "wgrad"}:
            raise ValueError("fault role must be forward, dgrad, wgrad, or None")


def _parse(value, cls):
    if isinstance(value, cls):
        return value
    if value is None or value == "none":
        return cls()
    if isinstance(value, str) and cls is AbftConfig:
        return cls(method=value)
    if not isinstance(value, Mapping):
        raise ValueError(f"{cls.__name__} must be a mapping")
    unknown = set(value) - {f.name for f in fields(cls)}
    if unknown:
        raise ValueError(f"Unknown {cls.__name__} fields: {sorted(unknown)}")
    return cls(**value)


def parse_abft_config(value=None):
    return _parse(value, AbftConfig)


def parse_fault_config(value=None):
    return _parse(value, FaultConfig)
