"""ABFT method registry and the compiled-policy contract.

Mirrors src/abft/methods.py of the reference: ``register_method`` /
``get_method`` / ``validate_method_instance``, the ``AbftMethod`` hooks used by
the engine, and the two builtin methods with compiled device policies —
``classic`` (two projections: ones and row index + 1; detection and
ratio-based localisation of a single output error) and ``sum`` (one all-ones
projection; detection only). The Python ``verify`` implementations are the
"reference" implementation path (and the CPU test seam); native executions use
the device finalize (and, when requested, the device locator) instead.
"""
from __future__ import annotations

from abc import ABC, abstractmethod
from contextlib import nullcontext
from dataclasses import dataclass

import torch

PRECISIONS = frozenset({"fp32", "bf16", "fp8", "nvfp4"})


@dataclass(frozen=True)
class CompiledPolicy:
    """Device policy id and its checksum channel count (policy ids 0 and 1)."""

    algorithm: int
    channels: int

    @property
    def reference_formats(self):
        return (("input_fused", "fp32_projection_fp32_accumulation"),
                ("augmented", "bf16_encoding_fp32_accumulation"))

    def __post_init__(self):
        if type(self.algorithm) is not int or type(self.channels) is not int or (
                self.algorithm, self.channels) not in {(0, 2), (1, 1)}:
            raise ValueError("Compiled ABFT policy must match an installed CUDA algorithm/channels pair")

    def metadata(self):
        return {"id": self.algorithm, "channels": self.channels,
                "reference_formats": dict(self.reference_formats), "native_localization": self.algorithm == 0}


class AbftMethod(ABC):
    stateful: bool = False
    needs_diagnostics: bool = False
    state_schema_version: int = 1
    compiled_policy = None
    supported_references = {"separate": PRECISIONS}
    _profile_scope = staticmethod(nullcontext)

    def validate_config(self, config):
        """Method-specific parameter checks (before any evidence is built)."""

    def validate_execution(self, operands, config):
        if type(self.needs_diagnostics) is not bool:
            raise TypeError("ABFT method needs_diagnostics must be a bool")
        self.validate_config(config)
        if config.reference_mode not in self.supported_references:
            raise NotImplementedError(f"{config.method} does not support {config.reference_mode}")
        if operands.precision not in self.supported_references[config.reference_mode]:
            raise ValueError(f"{config.method} does not support {config.reference_mode} with {operands.precision}")
        if config.implementation == "native":
            # A subclass must opt in to a compiled policy explicitly; inheriting
            # Classic's must not silently bypass an overridden verify().
            policy = type(self).__dict__.get("compiled_policy")
            if "compiled_policy" in vars(self) or not isinstance(policy, CompiledPolicy):
                raise ValueError(f"{config.method} has no explicit compiled CUDA policy for native implementation")
            if config.reference_mode not in dict(policy.reference_formats):
                raise ValueError(f"{config.method} native implementation does not support {config.reference_mode}")
            return policy
        return self.compiled_policy

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
        policy = self.compiled_policy
        algorithm = 0 if policy is None else policy.algorithm
        return operands.collected_native(state["weights"], algorithm=algorithm)

    def commit(self, state, decision, context):
        """Publish history once per transaction (stateless builtins: no-op)."""

    def state_dict(self):
        return {}

    def load_state_dict(self, state):
        if state:
            raise ValueError("This method has no persistent state")


_METHODS = {}


def register_method(name, factory):
    if not name or name == "none" or name in _METHODS:
        raise ValueError(f"Invalid or duplicate ABFT method: {name}")
    _METHODS[name] = factory


def get_method(name):
    if name not in _METHODS:
        raise ValueError(f"ABFT method is not implemented: {name}")
    method = _METHODS[name]()
    if not isinstance(method, AbftMethod):
        raise TypeError("ABFT factories must return an AbftMethod")
    method._registered_name = name
    return method


def validate_method_instance(name, method):
    if not isinstance(method, AbftMethod):
        raise TypeError("method_instance must be an AbftMethod")
    registered = getattr(method, "_registered_name", None)
    if registered is not None:
        if registered != name:
            raise ValueError("method_instance does not match the configured ABFT method")
    elif _METHODS.get(name) is not type(method):
        raise ValueError("Create this method_instance with get_method for the configured method")
    return method


def locate_single_error(residual, threshold, detected, nonfinite, m):
    """Classic two-channel ratio locator (src/abft/methods.py:525-542 of the
    reference): candidate (row, col) under a single-output-error assumption,
    rejected when ambiguous. Device tensors in, device tensors out."""
    failed = residual.abs() > threshold
    columns = failed.any(dim=0)
    col = columns.to(torch.int64).argmax()
    d0, d1 = residual[:, col].unbind()
    ratio = d1 / torch.where(d0 == 0, torch.ones_like(d0), d0)
    row = ratio.round().to(torch.int64) - 1
    consistency = (d1 - (row + 1).float() * d0).abs()
    allowance = threshold[1, col] + (row + 1).abs().float() * threshold[0, col]
    located = detected & ~nonfinite & (columns.sum() == 1) & (d0.abs() > threshold[0, col])
    located = located & (row >= 0) & (row < m) & (consistency <= allowance)
    uncertainty = (threshold[1, col] + ratio.abs() * threshold[0, col]) / (
        d0.abs() - threshold[0, col]).clamp_min(torch.finfo(torch.float32).tiny)
    located = located & ((ratio - (row + 1)).abs() + uncertainty < 0.5)
    location = torch.stack((torch.where(located, row, -1), torch.where(located, col, -1)))
    return located, location


class Classic(AbftMethod):
    compiled_policy = CompiledPolicy(0, 2)
    supported_references = {"separate": PRECISIONS, "input_fused": PRECISIONS, "augmented": frozenset({"bf16"})}
    channels = 2

    def validate_config(self, config):
        if config.parameters:
            raise ValueError("classic does not accept method parameters")

    def projection_weights(self, operands):
        device = operands.a.device
        return torch.stack((torch.ones(operands.m, device=device, dtype=torch.float32),
                            torch.arange(1, operands.m + 1, device=device, dtype=torch.float32)))

    def prepare_fused(self, operands, config):
        return {"weights": self.projection_weights(operands), "m": operands.m, "n": operands.n}

    def bind_reference(self, predicted_partials, magnitude_partials, state):
        return {**state, "expected": self.propagate(predicted_partials, state),
                "magnitude": self.propagate(magnitude_partials, state)}

    def prepare(self, operands, config, mm=None):
        if mm is None:
            from ..gemm import backend
            mm = backend.mm
        weights = self.projection_weights(operands)
        expected = torch.zeros((self.channels, operands.n), device=operands.a.device, dtype=torch.float32)
        magnitude = torch.zeros_like(expected)
        for start in range(0, operands.k, config.reference_block_k):
            end = min(operands.k, start + config.reference_block_k)
            a, b = (x.contiguous() for x in operands.decode_block(start, end))
            expected += mm(mm(weights, a).contiguous(), b)
            magnitude += mm(mm(weights.abs(), a.abs()).contiguous(), b.abs().contiguous())
        return {"weights": weights, "expected": expected, "magnitude": magnitude, "m": operands.m, "n": operands.n}

    def propagate(self, partials, state):
        return partials.sum(dim=1)[:, :state["n"]]

    def _detect(self, observed, output, state, config):
        residual = observed - state["expected"]
        threshold = config.atol + config.rtol * state["magnitude"]
        nonfinite = (~torch.isfinite(observed)).any() | (~torch.isfinite(state["expected"])).any()
        nonfinite = nonfinite | (~torch.isfinite(threshold)).any() | (~torch.isfinite(output)).any()
        nonfinite = nonfinite | (~torch.isfinite(residual)).any()
        return residual, threshold, nonfinite

    def verify(self, observed, output, state, config):
        with self._profile_scope("abft.detect"):
            residual, threshold, nonfinite = self._detect(observed, output, state, config)
            detected = (residual.abs() > threshold).any() | nonfinite
        with self._profile_scope("abft.locate"):
            if state.get("augmented", False):
                located = torch.zeros((), device=output.device, dtype=torch.bool)
                location = torch.full((2,), -1, device=output.device, dtype=torch.int64)
            else:
                located, location = locate_single_error(residual, threshold, detected, nonfinite, state["m"])
        return {"detected": detected, "nonfinite": nonfinite, "located": located, "location": location,
                "residual": residual, "threshold": threshold}


register_method("classic", Classic)


class Sum(Classic):
    """One all-ones column projection: detection only, no localisation."""

    compiled_policy = CompiledPolicy(1, 1)
    channels = 1

    def validate_config(self, config):
        if config.parameters:
            raise ValueError("sum does not accept method parameters")

    def projection_weights(self, operands):
        return torch.ones((1, operands.m), device=operands.a.device, dtype=torch.float32)

    def verify(self, observed, output, state, config):
        with self._profile_scope("abft.detect"):
            residual, threshold, nonfinite = self._detect(observed, output, state, config)
            detected = (residual.abs() > threshold).any() | nonfinite
        return {"detected": detected, "nonfinite": nonfinite,
                "located": torch.zeros((), device=output.device, dtype=torch.bool),
                "location": torch.full((2,), -1, device=output.device, dtype=torch.int64),
                "residual": residual, "threshold": threshold}


register_method("sum", Sum)
