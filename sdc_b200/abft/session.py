"""Caller-owned ABFT method instances, the physical call counter, checkpoints.

Mirrors src/abft/session.py of the reference (``MethodSession``): every
product request reserves a new ``call_index`` (activation-checkpoint replay
included); stateless methods (Classic, Sum) share one instance with no scope
bookkeeping, stream queries or locks on the hot path; stateful methods get one
instance per execution profile (layer, role, precision, device, m, n, k and
scale profile), reject concurrent entry, stream changes and CUDA-graph
capture, and snapshot / restore their history through ``state_dict`` /
``load_state_dict`` with the same checkpoint schema and validation rules.
"""
from __future__ import annotations

import hashlib
import json
import math
from contextlib import contextmanager, nullcontext
from dataclasses import asdict
from threading import Lock

import torch

from .config import parse_abft_config, parse_fault_config
from .methods import get_method

SCHEMA_VERSION = 1
CONFIG_VERSION = 1
_SCOPE_FIELDS = frozenset({"layer", "role", "precision", "device", "m", "n", "k", "scale_profile"})
_SCALING = {"fp32": "none", "bf16": "none", "fp8": "tensorwise", "nvfp4": "block16"}
_CHECKPOINT_FIELDS = frozenset({"schema_version", "config_version", "config_signature", "method_metadata",
                                "call_index", "instances", "pending_state"})


def _canonical(value):
    return json.dumps(value, sort_keys=True, separators=(",", ":"), allow_nan=False)


def _frozen(value, seen=None):
    """Detached copy of checkpointable state: dicts with str keys, lists,
    tuples, scalars and plain tensors only; no cycles."""
    if isinstance(value, torch.Tensor):
        copy = value.detach().clone()
        if type(copy) is not torch.Tensor:
            raise ValueError("ABFT state must use ordinary tensors, not tensor subclasses")
        return copy
    if value is None or type(value) in (bool, int, float, str):
        return value
    if type(value) not in (dict, list, tuple):
        raise ValueError("ABFT state must contain only dictionaries, lists, tuples, scalars and tensors; "
                         "save generator.get_state(), not a generator object")
    seen = set() if seen is None else seen
    if id(value) in seen:
        raise ValueError("ABFT state must not contain cycles")
    seen.add(id(value))
    try:
        if type(value) is dict:
            if not all(type(key) is str for key in value):
                raise ValueError("ABFT state dictionary keys must be strings")
            return {key: _frozen(item, seen) for key, item in value.items()}
        items = [_frozen(item, seen) for item in value]
        return items if type(value) is list else tuple(items)
    finally:
        seen.discard(id(value))


def _metadata(method, name):
    if method is None:
        return {"name": name, "class": None, "stateful": False, "state_schema_version": 1}
    stateful = getattr(method, "stateful", False)
    version = getattr(method, "state_schema_version", 1)
    if type(stateful) is not bool or type(version) is not int or version < 1:
        raise ValueError("ABFT method stateful/state_schema_version metadata is invalid")
    kind = type(method)
    return {"name": name, "class": f"{kind.__module__}.{kind.__qualname__}", "stateful": stateful,
            "state_schema_version": version}


def _scope_key(scope):
    """Validated hashable key of an execution profile."""
    if type(scope) is not dict or set(scope) != _SCOPE_FIELDS:
        raise ValueError("ABFT method scope metadata is invalid")
    if not isinstance(scope["layer"], str) or scope["role"] not in {"forward", "dgrad", "wgrad"}:
        raise ValueError("ABFT method layer/role scope is invalid")
    if scope["precision"] not in _SCALING:
        raise ValueError("ABFT method precision scope is invalid")
    if not all(type(scope[d]) is int and scope[d] > 0 for d in ("m", "n", "k")):
        raise ValueError("ABFT method shape scope is invalid")
    if not isinstance(scope["device"], str) or str(torch.device(scope["device"])) != scope["device"]:
        raise ValueError("ABFT method device scope is invalid")
    profile = scope["scale_profile"]
    if type(profile) is not dict or set(profile) != {"scaling", "global_scale", "input_dtypes"}:
        raise ValueError("ABFT scale profile metadata is invalid")
    if profile["scaling"] != _SCALING[scope["precision"]] and (scope["precision"], profile["scaling"]) != (
            "fp8", "blockwise"):
        raise ValueError("ABFT precision/scale profile mismatch")
    scale = profile["global_scale"]
    if scale != "amax" and (type(scale) not in (int, float) or not math.isfinite(scale) or scale <= 0):
        raise ValueError("ABFT global scale profile is invalid")
    dtypes = profile["input_dtypes"]
    if not isinstance(dtypes, list) or len(dtypes) != 2 or not all(isinstance(d, str) for d in dtypes):
        raise ValueError("ABFT input dtype profile is invalid")
    return (scope["layer"], scope["role"], scope["precision"], scope["device"], scope["m"], scope["n"],
            scope["k"], profile["scaling"], scale, *dtypes)


def _call_context(layer, role, index, profile):
    return {"layer": layer, "role": role, "call_index": index,
            "execution_kind": "forward_or_recompute" if role == "forward" else "backward", "retry": 0,
            "scale_profile": profile}


class MethodSession:
    """Retains method instances across calls of one configuration."""

    def __init__(self, config=None, fault=None):
        # Normalise through canonical JSON so the signature is stable.
        self.config = parse_abft_config(json.loads(_canonical(asdict(parse_abft_config(config)))))
        self.fault = parse_fault_config(json.loads(_canonical(asdict(parse_fault_config(fault)))))
        payload = {"version": CONFIG_VERSION, "abft": asdict(self.config), "fault": asdict(self.fault)}
        self.config_signature = hashlib.sha256(_canonical(payload).encode()).hexdigest()
        self._pending = get_method(self.config.method) if self.config.method != "none" else None
        self.metadata = _metadata(self._pending, self.config.method)
        self.stateful = self.metadata["stateful"]
        self.call_index = 0
        self._entries = {}
        self._streams = {}
        self._lock = Lock() if self.stateful else None

    @contextmanager
    def _exclusive(self):
        if self._lock is None:
            yield
            return
        if not self._lock.acquire(blocking=False):
            raise RuntimeError("Stateful ABFT session does not support concurrent calls or snapshots")
        try:
            yield
        finally:
            self._lock.release()

    def _bind_stream(self, device):
        if device.type == "cpu":
            return
        if device.type != "cuda":
            raise RuntimeError("Stateful ABFT sessions currently support CPU or one CUDA stream per device")
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("Stateful ABFT history cannot be advanced by CUDA Graph replay")
        stream = torch.cuda.current_stream(device)
        bound = self._streams.setdefault(str(device), stream)
        if bound.cuda_stream != stream.cuda_stream:
            raise RuntimeError("Stateful ABFT history cannot be shared across CUDA streams")

    @contextmanager
    def call(self, a, b, precision, scaling, global_scale, layer, role):
        """Reserve one physical call; yields (method instance, engine context)."""
        profile = {"scaling": scaling, "global_scale": global_scale, "input_dtypes": [str(a.dtype), str(b.dtype)]}
        if not self.stateful:
            self.call_index += 1
            yield self._pending, _call_context(layer, role, self.call_index, profile)
            return
        with self._exclusive():
            if a.ndim != 2 or b.ndim != 2 or a.shape[1] != b.shape[0] or a.device != b.device:
                raise ValueError("ABFT session requires compatible matrices on one device")
            scope = {"layer": layer, "role": role, "precision": precision, "device": str(a.device),
                     "m": int(a.shape[0]), "n": int(b.shape[1]), "k": int(a.shape[1]),
                     "scale_profile": profile}
            key = _scope_key(scope)
            self._bind_stream(a.device)
            entry = self._entries.get(key)
            if entry is None:
                method = self._pending if self._pending is not None else get_method(self.config.method)
                if _metadata(method, self.config.method) != self.metadata:
                    raise ValueError("ABFT method factory changed its state metadata")
                # The stored scope is a private copy: consumers may mutate the context.
                entry = self._entries[key] = (json.loads(_canonical(scope)), method)
                self._pending = None
            self.call_index += 1
            context_profile = {**profile, "input_dtypes": list(profile["input_dtypes"])}
            yield entry[1], _call_context(layer, role, self.call_index, context_profile)

    def state_dict(self):
        with self._exclusive():
            instances = []
            pending = None
            if self.stateful:
                for scope, method in self._entries.values():
                    stream = self._streams.get(scope["device"])
                    with torch.cuda.stream(stream) if stream is not None else nullcontext():
                        state = method.state_dict()
                    if type(state) is not dict:
                        raise ValueError("ABFT method state_dict must return a dictionary")
                    instances.append({"scope": json.loads(_canonical(scope)), "state": _frozen(state)})
                # Device clones finish before a caller serialises them.
                for stream in self._streams.values():
                    stream.synchronize()
                if self._pending is not None:
                    pending = self._pending.state_dict()
                    if type(pending) is not dict:
                        raise ValueError("ABFT method state_dict must return a dictionary")
                    pending = _frozen(pending)
            return {"schema_version": SCHEMA_VERSION, "config_version": CONFIG_VERSION,
                    "config_signature": self.config_signature, "method_metadata": dict(self.metadata),
                    "call_index": self.call_index, "instances": instances, "pending_state": pending}

    def load_state_dict(self, payload, *, device=None):
        with self._exclusive():
            self._check_header(payload)
            wanted = None if device is None else str(torch.device(device))
            entries = {}
            for item in payload["instances"]:
                if type(item) is not dict or set(item) != {"scope", "state"} or type(item["state"]) is not dict:
                    raise ValueError("ABFT method checkpoint entry is invalid")
                scope = json.loads(_canonical(item["scope"]))
                key = _scope_key(scope)
                if key in entries or (wanted is not None and scope["device"] != wanted):
                    raise ValueError("ABFT checkpoint has duplicate or mismatched device scopes")
                entries[key] = (scope, self._restored(item["state"]))
            pending = None if self.stateful else self._pending
            if self.stateful and not entries:
                if type(payload["pending_state"]) is not dict:
                    raise ValueError("Unused stateful ABFT method is missing its initial RNG/state")
                pending = self._restored(payload["pending_state"])
            elif payload["pending_state"] is not None:
                raise ValueError("ABFT checkpoint contains incompatible pending method state")
            if self.stateful:
                for stream in self._streams.values():
                    stream.synchronize()
                for name in {scope["device"] for scope, _ in entries.values()}:
                    if torch.device(name).type == "cuda":
                        torch.cuda.current_stream(torch.device(name)).synchronize()
            # Only now does the live state change: a rejected checkpoint leaves it intact.
            self._entries, self._pending, self._streams = entries, pending, {}
            self.call_index = payload["call_index"]

    def _check_header(self, payload):
        if type(payload) is not dict or set(payload) != _CHECKPOINT_FIELDS:
            raise ValueError("ABFT session checkpoint schema is invalid")
        metadata = payload["method_metadata"]
        if (type(metadata) is not dict or set(metadata) != set(self.metadata) or
                type(metadata["stateful"]) is not bool or type(metadata["state_schema_version"]) is not int):
            raise ValueError("ABFT method/state schema does not match checkpoint")
        if (type(payload["schema_version"]) is not int or type(payload["config_version"]) is not int or
                payload["schema_version"] != SCHEMA_VERSION or payload["config_version"] != CONFIG_VERSION or
                payload["config_signature"] != self.config_signature or metadata != self.metadata):
            raise ValueError("ABFT session configuration/method/state schema does not match checkpoint")
        if (type(payload["call_index"]) is not int or payload["call_index"] < 0 or
                type(payload["instances"]) is not list):
            raise ValueError("ABFT session call counter/instances are invalid")
        if not self.stateful and (payload["instances"] or payload["pending_state"] is not None):
            raise ValueError("Stateless ABFT methods must not restore adaptive history")

    def _restored(self, state):
        method = get_method(self.config.method)
        if _metadata(method, self.config.method) != self.metadata:
            raise ValueError("ABFT method factory changed its state metadata")
        method.load_state_dict(_frozen(state))
        return method
