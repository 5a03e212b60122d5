"""Checksum methods: what a protected GEMM projects and how it decides.

A method answers three questions for the engine, through the plugin hooks of
``AbftMethod`` (the hook names and their arguments are the reference's plugin
interface, src/abft/methods.py, so methods written for it keep working):

* which row weights W [C, M] the column checksums use (``prepare*``);
* how per-tile partial sums become per-column totals (``propagate``);
* how observed totals are judged against the expected ones (``verify``).

The builtin methods are two parameterisations of one projection checksum:
``classic`` (C = 2: all-ones and row index + 1, which also locates a single
faulty element from the ratio of its two residuals) and ``sum`` (C = 1,
detection only). Each builtin names its compiled device policy, so native
executions run the same decision in the finalize kernel instead of Python.
"""
from __future__ import annotations

from abc import ABC, abstractmethod
from contextlib import nullcontext
from dataclasses import dataclass

import torch

PRECISIONS = frozenset({"fp32", "bf16", "fp8", "nvfp4"})
# The (policy id, channel count) pairs compiled into the finalize kernel.
INSTALLED_POLICIES = {0: 2, 1: 1}
REFERENCE_FORMATS = (("input_fused", "fp32_projection_fp32_accumulation"),
                     ("augmented", "bf16_encoding_fp32_accumulation"))


@dataclass(frozen=True)
class CompiledPolicy:
    """A device decision policy: its id in the finalize kernel and channels."""

    algorithm: int
    channels: int

    def __post_init__(self):
        exact_ints = type(self.algorithm) is int and type(self.channels) is int
        if not exact_ints or INSTALLED_POLICIES.get(self.algorithm) != self.channels:
            raise ValueError("Compiled ABFT policy must match an installed CUDA algorithm/channels pair")

    @property
    def reference_formats(self):
        return REFERENCE_FORMATS

    def metadata(self):
        return {"id": self.algorithm, "channels": self.channels, "reference_formats": dict(REFERENCE_FORMATS),
                "native_localization": self.algorithm == 0}


class AbftMethod(ABC):
    """Plugin interface of a checksum method (see the module docstring)."""

    stateful: bool = False
    needs_diagnostics: bool = False
    state_schema_version: int = 1
    compiled_policy = None
    supported_references = {"separate": PRECISIONS}
    _profile_scope = staticmethod(nullcontext)

    # --- checks ------------------------------------------------------------
    def validate_config(self, config):
        """Method-specific parameter checks (before any evidence is built)."""

    def validate_execution(self, operands, config):
        """Rejects unsupported combinations; returns the compiled policy the
        native path must run (None for the Python implementation)."""
        if type(self.needs_diagnostics) is not bool:
            raise TypeError("ABFT method needs_diagnostics must be a bool")
        self.validate_config(config)
        mode = config.reference_mode
        if mode not in self.supported_references:
            raise NotImplementedError(f"{config.method} does not support {mode}")
        if operands.precision not in self.supported_references[mode]:
            raise ValueError(f"{config.method} does not support {mode} with {operands.precision}")
        if config.implementation != "native":
            return self.compiled_policy
        # A native policy must be declared by the method's own class: a
        # subclass that overrides verify() must not silently inherit one.
        declared = type(self).__dict__.get("compiled_policy")
        if not isinstance(declared, CompiledPolicy) or "compiled_policy" in vars(self):
            raise ValueError(f"{config.method} has no explicit compiled CUDA policy for native implementation")
        if mode not in dict(declared.reference_formats):
            raise ValueError(f"{config.method} native implementation does not support {mode}")
        return declared

    # --- evidence hooks ------------------------------------------------------
    def prepare_fused(self, operands, config):
        raise NotImplementedError("Method does not support input_fused reference")

    def prepare_augmented(self, operands, config):
        raise NotImplementedError("Method does not support augmented GEMM")

    def bind_reference(self, predicted_partials, magnitude_partials, state):
        raise NotImplementedError("Method does not support input_fused reference")

    @abstractmethod
    def prepare(self, operands, config, mm=None):
        """Clean-input evidence for the separate reference mode."""

    @abstractmethod
    def propagate(self, partials, state):
        """Reduce per-tile partial projections to per-column totals."""

    @abstractmethod
    def verify(self, observed, output, state, config):
        """Device tensors describing anomalies (and candidate locations)."""

    def recover(self, operands, state):
        """A fresh observed evidence of the clean operands (full recompute)."""
        policy = self.compiled_policy
        return operands.collected_native(state["weights"], algorithm=policy.algorithm if policy else 0)

    # --- adaptive state ------------------------------------------------------
    def commit(self, state, decision, context):
        """Called once per transaction, after any retry (stateless: no-op)."""

    def state_dict(self):
        return {}

    def load_state_dict(self, state):
        if state:
            raise ValueError("This method has no persistent state")


# --- registry -------------------------------------------------------------------
# name -> zero-argument factory. Kept as a module attribute so that a caller
# (or a test) can swap in a private copy.
_METHODS = {}


def register_method(name, factory):
    if not name or name == "none" or name in _METHODS:
        raise ValueError(f"Invalid or duplicate ABFT method: {name}")
    _METHODS[name] = factory


def get_method(name):
    factory = _METHODS.get(name)
    if factory is None:
        raise ValueError(f"ABFT method is not implemented: {name}")
    instance = factory()
    if not isinstance(instance, AbftMethod):
        raise TypeError("ABFT factories must return an AbftMethod")
    instance._registered_name = name
    return instance


def validate_method_instance(name, method):
    """A caller-retained instance must have come from the configured method."""
    if not isinstance(method, AbftMethod):
        raise TypeError("method_instance must be an AbftMethod")
    origin = getattr(method, "_registered_name", None)
    if origin is None and _METHODS.get(name) is not type(method):
        raise ValueError("Create this method_instance with get_method for the configured method")
    if origin is not None and origin != name:
        raise ValueError("method_instance does not match the configured ABFT method")
    return method


# --- the projection checksum ----------------------------------------------------

def locate_single_error(residual, threshold, detected, nonfinite, m):
    """Ratio locator of the two-channel (ones, row + 1) checksum: a single
    faulty element at (r, c) changes channel 0 of column c by d and channel 1
    by (r + 1) d, so r = d1 / d0 - 1. The candidate is accepted only when
    exactly one column failed, d0 clears its threshold, the row is in range,
    d1 agrees with (r + 1) d0 within the combined thresholds, and the ratio's
    uncertainty keeps it within half a row. Op-for-op the arithmetic of the
    reference's verify (src/abft/methods.py:218-235) and of the device
    locator, so host and device decisions agree. Device tensors in and out."""
    above = residual.abs() > threshold
    failing_columns = above.any(dim=0)
    col = failing_columns.to(torch.int64).argmax()
    d0, d1 = residual[:, col].unbind()
    t0, t1 = threshold[0, col], threshold[1, col]
    ratio = d1 / torch.where(d0 == 0, torch.ones_like(d0), d0)
    row = ratio.round().to(torch.int64) - 1
    rows_p1 = (row + 1).float()
    consistent = (d1 - rows_p1 * d0).abs() <= t1 + (row + 1).abs().float() * t0
    spread = (t1 + ratio.abs() * t0) / (d0.abs() - t0).clamp_min(torch.finfo(torch.float32).tiny)
    sharp = (ratio - (row + 1)).abs() + spread < 0.5
    single = (failing_columns.sum() == 1) & (d0.abs() > t0)
    located = detected & ~nonfinite & single & (row >= 0) & (row < m) & consistent & sharp
    never = torch.full_like(row, -1)
    return located, torch.stack((torch.where(located, row, never), torch.where(located, col, never)))


class ProjectionChecksum(AbftMethod):
    """Weighted column checksums w_c^T C against the input-side w_c^T A B.

    Subclasses choose the channels (``weight_rows``) and whether the method
    locates single errors. Residual = observed - expected; threshold =
    atol + rtol * |w|^T |A| |B|; any non-finite value is a detection."""

    channels = 0
    localises = False
    parameter_free = True

    def weight_rows(self, m, device):
        raise NotImplementedError

    def projection_weights(self, operands):
        return self.weight_rows(operands.m, operands.a.device)

    def validate_config(self, config):
        if self.parameter_free and config.parameters:
            raise ValueError(f"{config.method} does not accept method parameters")

    # evidence
    def _fresh_state(self, operands, **extra):
        return {"weights": self.projection_weights(operands), "m": operands.m, "n": operands.n, **extra}

    def prepare_fused(self, operands, config):
        return self._fresh_state(operands)

    def prepare_augmented(self, operands, config):
        """Encoding weights in the BF16 input format shared with A and the
        checksum rows (rounded row numbers above 256 are not all distinct)."""
        if operands.precision != "bf16":
            raise ValueError("augmented currently requires BF16 GEMM")
        state = self._fresh_state(operands, augmented=True)
        state["weights"] = state["weights"].to(torch.bfloat16).contiguous()
        return state

    def bind_reference(self, predicted_partials, magnitude_partials, state):
        return {**state, "expected": self.propagate(predicted_partials, state),
                "magnitude": self.propagate(magnitude_partials, state)}

    def prepare(self, operands, config, mm=None):
        """Expected checksums w^T A B and magnitudes |w|^T |A| |B| from the
        decoded operands, one ``reference_block_k`` slice of K at a time."""
        if mm is None:
            from ..gemm import backend
            mm = backend.mm
        weights = self.projection_weights(operands)
        totals = torch.zeros((2, self.channels, operands.n), device=operands.a.device, dtype=torch.float32)
        step = config.reference_block_k
        for k0 in range(0, operands.k, step):
            a, b = (block.contiguous() for block in operands.decode_block(k0, min(operands.k, k0 + step)))
            totals[0] += mm(mm(weights, a).contiguous(), b)
            totals[1] += mm(mm(weights.abs(), a.abs()).contiguous(), b.abs().contiguous())
        return {"weights": weights, "expected": totals[0], "magnitude": totals[1], "m": operands.m,
                "n": operands.n}

    def propagate(self, partials, state):
        return partials.sum(dim=1)[:, :state["n"]]

    # decision
    def verify(self, observed, output, state, config):
        with self._profile_scope("abft.detect"):
            expected = state["expected"]
            residual = observed - expected
            threshold = config.atol + config.rtol * state["magnitude"]
            nonfinite = torch.stack([(~torch.isfinite(t)).any()
                                     for t in (observed, expected, threshold, output, residual)]).any()
            detected = nonfinite | (residual.abs() > threshold).any()
        with self._profile_scope("abft.locate"):
            if self.localises and not state.get("augmented", False):
                located, location = locate_single_error(residual, threshold, detected, nonfinite, state["m"])
            else:
                located = torch.zeros((), device=output.device, dtype=torch.bool)
                location = torch.full((2,), -1, device=output.device, dtype=torch.int64)
        return {"detected": detected, "nonfinite": nonfinite, "located": located, "location": location,
                "residual": residual, "threshold": threshold}


class Classic(ProjectionChecksum):
    """Two channels (ones, row + 1): detection and single-element location."""

    compiled_policy = CompiledPolicy(0, 2)
    supported_references = {"separate": PRECISIONS, "input_fused": PRECISIONS, "augmented": frozenset({"bf16"})}
    channels = 2
    localises = True

    def weight_rows(self, m, device):
        rows = torch.arange(1, m + 1, device=device, dtype=torch.float32)
        return torch.stack((torch.ones_like(rows), rows))


class Sum(ProjectionChecksum):
    """One all-ones channel: detection only."""

    compiled_policy = CompiledPolicy(1, 1)
    supported_references = Classic.supported_references
    channels = 1

    def weight_rows(self, m, device):
        return torch.ones((1, m), device=device, dtype=torch.float32)


register_method("classic", Classic)
register_method("sum", Sum)
