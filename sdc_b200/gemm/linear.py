"""nn.Linear on the protected sm_100a GEMMs: forward, dgrad and wgrad.

``install(model, ...)`` swaps every ``nn.Linear`` of a model for a
``ProtectedLinear`` that keeps the same parameter objects (shared modules,
tied weights and train/eval mode survive), so optimisers, checkpoints and
DDP see an unchanged model. A linear layer is three GEMMs:

    forward  Y  = X W^T        (role "forward")
    dgrad    dX = dY W         (role "dgrad")
    wgrad    dW = dY^T X       (role "wgrad")

Each runs through ``backend.gemm`` or, when the model is protected, through
the ABFT engine (``sdc_b200.abft.execute``) with one ``MethodSession`` per
model that numbers the physical calls (activation-checkpoint replays
included). Reports go to a bounded in-memory deque and, optionally, to a
JSONL file (which reads them back to the host, so it is opt-in).

The public names and arguments are those of the reference's Linear bridge
(src/cutlass_gemm/linear.py; its ``CutlassLinear`` is an alias of
``ProtectedLinear`` here).
"""
from __future__ import annotations

import json
from collections import deque
from dataclasses import dataclass
from pathlib import Path

import torch
from torch import nn
from torch.autograd.function import once_differentiable

from ..abft.config import parse_abft_config, parse_fault_config
from ..abft.session import MethodSession
from . import backend

QUANTISED = frozenset({"fp8", "nvfp4"})


class Protection:
    """The model-wide ABFT state of an installed model: the session (call
    counter and method instances), the fault to inject and the reports."""

    def __init__(self, abft, fault, report_max_records=0, report_path=None):
        self.session = MethodSession(abft, fault)
        self.abft, self.fault = self.session.config, self.session.fault
        self.reports = deque(maxlen=report_max_records)
        self.report_path = Path(report_path) if report_path else None

    @property
    def call_index(self):
        return self.session.call_index

    def record(self, report):
        if report is None:
            return
        if self.reports.maxlen:
            self.reports.append(report)
        if self.report_path is not None:
            self.report_path.parent.mkdir(parents=True, exist_ok=True)
            with self.report_path.open("a", encoding="utf-8") as log:
                log.write(json.dumps(report.to_record()) + "\n")

    def product(self, a, b, precision, scaling, global_scale, layer, role):
        """a @ b as one protected physical call; its report is recorded even
        when the engine raises (it travels on the exception)."""
        from .. import abft

        with self.session.call(a, b, precision, scaling, global_scale, layer, role) as (method, context):
            try:
                output, report = abft.execute(a, b, precision, scaling, global_scale, self.abft, self.fault,
                                              context, method_instance=method)
            except Exception as error:
                self.record(getattr(error, "report", None))
                raise
            self.record(report)
            return output


def packed(matrix):
    """``matrix`` if it or its transpose is contiguous (a GEMM operand needs
    one of the two), else a contiguous copy (e.g. an expanded gradient)."""
    return matrix if matrix.is_contiguous() or matrix.T.is_contiguous() else matrix.contiguous()


@dataclass(frozen=True)
class _Route:
    """How one layer's GEMMs run: compute dtype and quantisation, and the
    protection (None: plain backend GEMMs) with the layer's name."""

    dtype: torch.dtype
    precision: str
    scaling: str
    global_scale: object
    protection: object = None
    layer: str = ""

    def product(self, left, right, role):
        if self.protection is None:
            return backend.gemm(left, right, self.precision, self.scaling, self.global_scale)
        return self.protection.product(left, right, self.precision, self.scaling, self.global_scale, self.layer,
                                       role)

    def operand(self, tensor):
        """Quantised precisions take the master values; others the compute dtype."""
        return packed(tensor if self.precision in QUANTISED else tensor.to(self.dtype))


class _LinearGemms(torch.autograd.Function):
    """Y = X W^T + b whose forward, dgrad and wgrad GEMMs all take the route."""

    @staticmethod
    def forward(ctx, x, weight, bias, route):
        with torch.autocast(device_type=x.device.type, enabled=False):
            rows = route.operand(x.reshape(-1, x.shape[-1]))
            w = route.operand(weight)
            ctx.save_for_backward(rows, w)
            ctx.route = route
            ctx.shapes = (x.shape, x.dtype, weight.dtype, None if bias is None else bias.dtype)
            y = route.product(rows, w.T, "forward").to(route.dtype)
            if bias is not None:
                y = y + bias.to(route.dtype)
            return y.reshape(*x.shape[:-1], weight.shape[0])

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_y):
        rows, w = ctx.saved_tensors
        route = ctx.route
        x_shape, x_dtype, w_dtype, b_dtype = ctx.shapes
        needs_x, needs_w, needs_b = ctx.needs_input_grad[:3]
        dx = dw = db = None
        with torch.autocast(device_type=grad_y.device.type, enabled=False):
            dy = packed(grad_y.reshape(-1, grad_y.shape[-1]).to(rows.dtype))
            if needs_x:
                dx = route.product(dy, w, "dgrad").reshape(x_shape).to(x_dtype)
            if needs_w:
                dw = route.product(dy.T, rows, "wgrad").to(w_dtype)
            if b_dtype is not None and needs_b:
                db = dy.sum(0).to(b_dtype)
        return dx, dw, db, None


class ProtectedLinear(nn.Linear):
    """An ``nn.Linear`` whose GEMMs run through this library (same parameters).

    ``precision`` None follows the input (FP32, or BF16 under autocast);
    "fp32" forces FP32; "bf16", "fp8" and "nvfp4" compute in BF16 with the
    quantised precisions quantising both operands of every GEMM."""

    def __init__(self, original, precision=None, scaling="none", global_scale="amax", protection=None, layer=""):
        nn.Module.__init__(self)
        self.in_features, self.out_features = original.in_features, original.out_features
        self.weight, self.bias = original.weight, original.bias
        self.precision, self.scaling, self.global_scale = precision, scaling, global_scale
        self.protection, self.layer_name = protection, layer
        self.train(original.training)

    def _compute_dtype(self, x):
        if self.precision == "fp32":
            return torch.float32
        if self.precision in {"bf16", "fp8", "nvfp4"}:
            return torch.bfloat16
        device = x.device.type
        dtype = torch.get_autocast_dtype(device) if torch.is_autocast_enabled(device) else x.dtype
        if dtype not in {torch.float32, torch.bfloat16}:
            raise ValueError("ProtectedLinear computes in BF16 or FP32")
        return dtype

    def forward(self, x):
        dtype = self._compute_dtype(x)
        precision = self.precision or ("bf16" if dtype == torch.bfloat16 else "fp32")
        route = _Route(dtype, precision, self.scaling, self.global_scale, self.protection,
                       self.layer_name if self.protection is not None else "")
        return _LinearGemms.apply(x, self.weight, self.bias, route)


CutlassLinear = ProtectedLinear


def protection_sessions(model):
    """One entry per distinct protection of ``model``: its session and the
    sorted paths of the layers that use it (tied aliases included)."""
    sessions = {}
    for path, module in model.named_modules(remove_duplicate=False):
        if isinstance(module, ProtectedLinear) and module.protection is not None:
            entry = sessions.setdefault(id(module.protection), {"layers": [], "session": module.protection.session})
            entry["layers"].append(path)
    for entry in sessions.values():
        entry["layers"].sort()
    return sorted(sessions.values(), key=lambda entry: entry["layers"])


def install(model, precision=None, scaling="none", global_scale="amax", *, abft_config=None, fault_config=None,
            report_max_records=0, report_path=None):
    """Replace every ``nn.Linear`` of ``model`` (or ``model`` itself) with a
    ``ProtectedLinear``, preserving parameter identity and module sharing."""
    abft_config, fault_config = parse_abft_config(abft_config), parse_fault_config(fault_config)
    protection = None
    if abft_config.method != "none" or fault_config.location != "none":
        protection = Protection(abft_config, fault_config, report_max_records, report_path)
    if isinstance(model, nn.Linear) and not isinstance(model, ProtectedLinear):
        return ProtectedLinear(model, precision, scaling, global_scale, protection)
    targets = [(path, module) for path, module in model.named_modules(remove_duplicate=False)
               if isinstance(module, nn.Linear) and not isinstance(module, ProtectedLinear)]
    if not targets:
        raise ValueError("the model has no nn.Linear to replace")
    swapped = {}
    for path, module in targets:
        # A shared module is replaced once; every path to it gets the same
        # replacement, named after the first path.
        replacement = swapped.get(id(module))
        if replacement is None:
            replacement = swapped[id(module)] = ProtectedLinear(module, precision, scaling, global_scale,
                                                                protection, path)
        parent, _, name = path.rpartition(".")
        setattr(model.get_submodule(parent) if parent else model, name, replacement)
    return model
