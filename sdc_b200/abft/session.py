"""Method instances retained across the GEMM calls of one protected model.

A ``MethodSession`` does two jobs for the Linear bridge:

* it numbers every physical GEMM call (forward, dgrad, wgrad, and forwards
  replayed by activation checkpointing), which is what a fault's
  ``call_index`` refers to;
* it hands the engine the method instance a call must use. Stateless methods
  (classic, sum) share one instance and take no locks or stream queries on
  the hot path. Stateful methods get one instance per execution profile
  (layer, role, precision, device, shape, scale profile), are bound to one
  CUDA stream per device, refuse concurrent entry and CUDA-graph capture, and
  can be checkpointed with ``state_dict`` / ``load_state_dict``.

The checkpoint dictionary uses the reference's schema (src/abft/session.py)
so that checkpoints move between the two implementations: schema and config
versions, a SHA-256 signature of the canonical configuration, the method's
state metadata, the call counter, per-profile states and the state of a
not-yet-used stateful instance.
"""
from __future__ import annotations

import hashlib
import json
import math
from contextlib import contextmanager, nullcontext
from dataclasses import asdict, dataclass
from threading import Lock

import torch

from .config import parse_abft_config, parse_fault_config
from .methods import get_method

SCHEMA_VERSION = 1
CONFIG_VERSION = 1
CHECKPOINT_KEYS = frozenset({"schema_version", "config_version", "config_signature", "method_metadata",
                             "call_index", "instances", "pending_state"})
ROLES = frozenset({"forward", "dgrad", "wgrad"})
DEFAULT_SCALING = {"fp32": "none", "bf16": "none", "fp8": "tensorwise", "nvfp4": "block16"}


def _json(value):
    return json.dumps(value, sort_keys=True, separators=(",", ":"), allow_nan=False)


def _roundtrip(value):
    return json.loads(_json(value))


def _detached(value, _path=()):
    """A checkpoint-safe deep copy: string-key dictionaries, lists, tuples,
    scalars and plain tensors (cloned), without cycles."""
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
    if any(item is value for item in _path):
        raise ValueError("ABFT state must not contain cycles")
    path = _path + (value,)
    if type(value) is dict:
        if any(type(key) is not str for key in value):
            raise ValueError("ABFT state dictionary keys must be strings")
        return {key: _detached(item, path) for key, item in value.items()}
    items = [_detached(item, path) for item in value]
    return items if type(value) is list else tuple(items)


def _method_metadata(method, name):
    if method is None:
        return {"name": name, "class": None, "stateful": False, "state_schema_version": 1}
    stateful, version = getattr(method, "stateful", False), getattr(method, "state_schema_version", 1)
    if type(stateful) is not bool or type(version) is not int or version < 1:
        raise ValueError("ABFT method stateful/state_schema_version metadata is invalid")
    kind = type(method)
    return {"name": name, "class": f"{kind.__module__}.{kind.__qualname__}", "stateful": stateful,
            "state_schema_version": version}


@dataclass(frozen=True)
class _Scope:
    """One execution profile of a stateful method (hashable)."""

    layer: str
    role: str
    precision: str
    device: str
    m: int
    n: int
    k: int
    scaling: str
    global_scale: object
    dtypes: tuple

    def record(self):
        return {"layer": self.layer, "role": self.role, "precision": self.precision, "device": self.device,
                "m": self.m, "n": self.n, "k": self.k,
                "scale_profile": {"scaling": self.scaling, "global_scale": self.global_scale,
                                  "input_dtypes": list(self.dtypes)}}

    @classmethod
    def parse(cls, record):
        """Validated scope of a checkpoint (or freshly built) record."""
        fields = {"layer", "role", "precision", "device", "m", "n", "k", "scale_profile"}
        if type(record) is not dict or set(record) != fields:
            raise ValueError("ABFT method scope metadata is invalid")
        if not isinstance(record["layer"], str) or record["role"] not in ROLES:
            raise ValueError("ABFT method layer/role scope is invalid")
        precision = record["precision"]
        if precision not in DEFAULT_SCALING:
            raise ValueError("ABFT method precision scope is invalid")
        if any(type(record[d]) is not int or record[d] <= 0 for d in ("m", "n", "k")):
            raise ValueError("ABFT method shape scope is invalid")
        device = record["device"]
        if not isinstance(device, str) or str(torch.device(device)) != device:
            raise ValueError("ABFT method device scope is invalid")
        profile = record["scale_profile"]
        if type(profile) is not dict or set(profile) != {"scaling", "global_scale", "input_dtypes"}:
            raise ValueError("ABFT scale profile metadata is invalid")
        scaling = profile["scaling"]
        if scaling != DEFAULT_SCALING[precision] and (precision, scaling) != ("fp8", "blockwise"):
            raise ValueError("ABFT precision/scale profile mismatch")
        scale = profile["global_scale"]
        if scale != "amax" and (type(scale) not in (int, float) or not math.isfinite(scale) or scale <= 0):
            raise ValueError("ABFT global scale profile is invalid")
        dtypes = profile["input_dtypes"]
        if not isinstance(dtypes, list) or len(dtypes) != 2 or not all(isinstance(d, str) for d in dtypes):
            raise ValueError("ABFT input dtype profile is invalid")
        return cls(record["layer"], record["role"], precision, device, record["m"], record["n"], record["k"],
                   scaling, scale, tuple(dtypes))


def _engine_context(layer, role, index, profile):
    """The context the engine receives for one physical call."""
    kind = "forward_or_recompute" if role == "forward" else "backward"
    return {"layer": layer, "role": role, "call_index": index, "execution_kind": kind, "retry": 0,
            "scale_profile": profile}


class MethodSession:
    """Retains method instances across the calls of one configuration."""

    def __init__(self, config=None, fault=None):
        # Canonical JSON round trip: the signature depends on values only.
        self.config = parse_abft_config(_roundtrip(asdict(parse_abft_config(config))))
        self.fault = parse_fault_config(_roundtrip(asdict(parse_fault_config(fault))))
        signed = {"version": CONFIG_VERSION, "abft": asdict(self.config), "fault": asdict(self.fault)}
        self.config_signature = hashlib.sha256(_json(signed).encode()).hexdigest()
        self._spare = None if self.config.method == "none" else get_method(self.config.method)
        self.metadata = _method_metadata(self._spare, self.config.method)
        self.stateful = self.metadata["stateful"]
        self.call_index = 0
        self._by_scope = {}   # _Scope -> method instance (stateful only)
        self._streams = {}    # device name -> the one stream its history advances on
        self._guard = Lock() if self.stateful else None

    # --- calls ---------------------------------------------------------------
    @contextmanager
    def call(self, a, b, precision, scaling, global_scale, layer, role):
        """Reserve one physical call; yields (method instance, engine context)."""
        profile = {"scaling": scaling, "global_scale": global_scale, "input_dtypes": [str(a.dtype), str(b.dtype)]}
        if not self.stateful:
            self.call_index += 1
            yield self._spare, _engine_context(layer, role, self.call_index, profile)
            return
        with self._exclusive():
            if a.ndim != 2 or b.ndim != 2 or a.shape[1] != b.shape[0] or a.device != b.device:
                raise ValueError("ABFT session requires compatible matrices on one device")
            scope = _Scope.parse({"layer": layer, "role": role, "precision": precision, "device": str(a.device),
                                  "m": int(a.shape[0]), "n": int(b.shape[1]), "k": int(a.shape[1]),
                                  "scale_profile": _roundtrip(profile)})
            self._bind_stream(a.device)
            method = self._by_scope.get(scope)
            if method is None:
                method = self._spare if self._spare is not None else self._new_method()
                self._spare = None
                self._by_scope[scope] = method
            self.call_index += 1
            yield method, _engine_context(layer, role, self.call_index, _roundtrip(profile))

    @contextmanager
    def _exclusive(self):
        if self._guard is None:
            yield
            return
        if not self._guard.acquire(blocking=False):
            raise RuntimeError("Stateful ABFT session does not support concurrent calls or snapshots")
        try:
            yield
        finally:
            self._guard.release()

    def _bind_stream(self, device):
        if device.type == "cpu":
            return
        if device.type != "cuda":
            raise RuntimeError("Stateful ABFT sessions currently support CPU or one CUDA stream per device")
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("Stateful ABFT history cannot be advanced by CUDA Graph replay")
        stream = torch.cuda.current_stream(device)
        if self._streams.setdefault(str(device), stream).cuda_stream != stream.cuda_stream:
            raise RuntimeError("Stateful ABFT history cannot be shared across CUDA streams")

    def _new_method(self, state=None):
        method = get_method(self.config.method)
        if _method_metadata(method, self.config.method) != self.metadata:
            raise ValueError("ABFT method factory changed its state metadata")
        if state is not None:
            method.load_state_dict(_detached(state))
        return method

    # --- checkpoints -----------------------------------------------------------
    def state_dict(self):
        with self._exclusive():
            instances, pending = [], None
            if self.stateful:
                for scope, method in self._by_scope.items():
                    stream = self._streams.get(scope.device)
                    with torch.cuda.stream(stream) if stream is not None else nullcontext():
                        instances.append({"scope": scope.record(), "state": _detached(_own_state(method))})
                for stream in self._streams.values():  # clones complete before the caller serialises
                    stream.synchronize()
                if self._spare is not None:
                    pending = _detached(_own_state(self._spare))
            return {"schema_version": SCHEMA_VERSION, "config_version": CONFIG_VERSION,
                    "config_signature": self.config_signature, "method_metadata": dict(self.metadata),
                    "call_index": self.call_index, "instances": instances, "pending_state": pending}

    def load_state_dict(self, payload, *, device=None):
        """Restore a checkpoint; on any error the live state is untouched."""
        with self._exclusive():
            self._check_header(payload)
            wanted = None if device is None else str(torch.device(device))
            restored = {}
            for entry in payload["instances"]:
                if type(entry) is not dict or set(entry) != {"scope", "state"} or type(entry["state"]) is not dict:
                    raise ValueError("ABFT method checkpoint entry is invalid")
                scope = _Scope.parse(_roundtrip(entry["scope"]))
                if scope in restored or (wanted is not None and scope.device != wanted):
                    raise ValueError("ABFT checkpoint has duplicate or mismatched device scopes")
                restored[scope] = self._new_method(entry["state"])
            spare = self._spare if not self.stateful else None
            if self.stateful and not restored:
                if type(payload["pending_state"]) is not dict:
                    raise ValueError("Unused stateful ABFT method is missing its initial RNG/state")
                spare = self._new_method(payload["pending_state"])
            elif payload["pending_state"] is not None:
                raise ValueError("ABFT checkpoint contains incompatible pending method state")
            if self.stateful:
                for stream in self._streams.values():
                    stream.synchronize()
                for name in {scope.device for scope in restored}:
                    if torch.device(name).type == "cuda":
                        torch.cuda.current_stream(torch.device(name)).synchronize()
            self._by_scope, self._spare, self._streams = restored, spare, {}
            self.call_index = payload["call_index"]

    def _check_header(self, payload):
        if type(payload) is not dict or set(payload) != CHECKPOINT_KEYS:
            raise ValueError("ABFT session checkpoint schema is invalid")
        meta = payload["method_metadata"]
        if (type(meta) is not dict or set(meta) != set(self.metadata) or type(meta["stateful"]) is not bool
                or type(meta["state_schema_version"]) is not int):
            raise ValueError("ABFT method/state schema does not match checkpoint")
        versions = (payload["schema_version"], payload["config_version"])
        if (any(type(v) is not int for v in versions) or versions != (SCHEMA_VERSION, CONFIG_VERSION)
                or payload["config_signature"] != self.config_signature or meta != self.metadata):
            raise ValueError("ABFT session configuration/method/state schema does not match checkpoint")
        if type(payload["call_index"]) is not int or payload["call_index"] < 0 or type(payload["instances"]) is not list:
            raise ValueError("ABFT session call counter/instances are invalid")
        if not self.stateful and (payload["instances"] or payload["pending_state"] is not None):
            raise ValueError("Stateless ABFT methods must not restore adaptive history")


def _own_state(method):
    state = method.state_dict()
    if type(state) is not dict:
        raise ValueError("ABFT method state_dict must return a dictionary")
    return state
