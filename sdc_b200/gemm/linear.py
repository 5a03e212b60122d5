"""nn.Linear forward / dgrad / wgrad through the protected sm_100a GEMMs.

Mirrors src/cutlass_gemm/linear.py of the reference: ``install`` replaces
every ``nn.Linear`` of a model (parameter identity, shared modules, tied
weights and train/eval mode preserved) with ``ProtectedLinear`` (the
reference's ``CutlassLinear``; that name is kept as an alias), whose autograd
function routes the three GEMMs of a linear layer — forward ``X W^T``, dgrad
``dY W`` and wgrad ``dY^T X`` — through ``backend.gemm`` or, when a
protection is installed, through the ABFT engine with one ``MethodSession``
counting physical calls per model. Reports are kept in a bounded deque and
optionally appended to a JSONL file (an explicit host sync, opt-in).
"""
from __future__ import annotations

import json
from collections import deque
from pathlib import Path

import torch
from torch import nn
from torch.autograd.function import once_differentiable

from ..abft.config import parse_abft_config, parse_fault_config
from ..abft.session import MethodSession
from . import backend


class _Protection:
    """Bounded reports and the model-wide physical GEMM call counter."""

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
            with self.report_path.open("a", encoding="utf-8") as stream:
                stream.write(json.dumps(report.to_record()) + "\n")

    def product(self, a, b, precision, scaling, global_scale, layer, role):
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
    """Keep a packed matrix or its plain transpose; copy any other strides
    (e.g. the expanded gradient of ``output.sum().backward()``)."""
    if matrix.is_contiguous() or matrix.T.is_contiguous():
        return matrix
    return matrix.contiguous()


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, dtype, precision, scaling, global_scale, protection=None, layer=""):
        with torch.autocast(device_type=x.device.type, enabled=False):
            quantised = precision in {"fp8", "nvfp4"}
            rows = x.reshape(-1, x.shape[-1])
            a = packed(rows if quantised else rows.to(dtype))
            w = packed(weight if quantised else weight.to(dtype))
            ctx.save_for_backward(a, w)
            ctx.input_shape, ctx.input_dtype, ctx.weight_dtype = x.shape, x.dtype, weight.dtype
            ctx.bias_dtype = None if bias is None else bias.dtype
            ctx.precision, ctx.scaling, ctx.global_scale = precision, scaling, global_scale
            ctx.protection, ctx.layer = protection, layer
            if protection is None:
                out = backend.gemm(a, w.T, precision, scaling, global_scale)
            else:
                out = protection.product(a, w.T, precision, scaling, global_scale, layer, "forward")
            out = out.to(dtype)
            if bias is not None:
                out = out + bias.to(dtype)
            return out.reshape(*x.shape[:-1], weight.shape[0])

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_output):
        a, w = ctx.saved_tensors
        with torch.autocast(device_type=grad_output.device.type, enabled=False):
            dy = packed(grad_output.reshape(-1, grad_output.shape[-1]).to(a.dtype))

            def product(left, right, role):
                if ctx.protection is None:
                    return backend.gemm(left, right, ctx.precision, ctx.scaling, ctx.global_scale)
                return ctx.protection.product(left, right, ctx.precision, ctx.scaling, ctx.global_scale,
                                              ctx.layer, role)

            dx = dw = db = None
            if ctx.needs_input_grad[0]:
                dx = product(dy, w, "dgrad").reshape(ctx.input_shape).to(ctx.input_dtype)
            if ctx.needs_input_grad[1]:
                dw = product(dy.T, a, "wgrad").to(ctx.weight_dtype)
            if ctx.bias_dtype is not None and ctx.needs_input_grad[2]:
                db = dy.sum(0).to(ctx.bias_dtype)
        return (dx, dw, db, None, None, None, None, None, None)[:len(ctx.needs_input_grad)]


class ProtectedLinear(nn.Linear):
    """An ``nn.Linear`` whose GEMMs run through this library (same parameters)."""

    def __init__(self, original, precision=None, scaling="none", global_scale="amax", protection=None, layer=""):
        nn.Module.__init__(self)
        self.in_features, self.out_features = original.in_features, original.out_features
        self.weight, self.bias = original.weight, original.bias
        self.precision, self.scaling, self.global_scale = precision, scaling, global_scale
        self.protection, self.layer_name = protection, layer
        self.train(original.training)

    def forward(self, x):
        autocast = torch.is_autocast_enabled(x.device.type)
        dtype = torch.get_autocast_dtype(x.device.type) if autocast else x.dtype
        if self.precision == "fp32":
            dtype = torch.float32
        elif self.precision in {"bf16", "fp8", "nvfp4"}:
            dtype = torch.bfloat16
        if dtype not in {torch.float32, torch.bfloat16}:
            raise ValueError("ProtectedLinear computes in BF16 or FP32")
        precision = self.precision or ("bf16" if dtype == torch.bfloat16 else "fp32")
        args = (x, self.weight, self.bias, dtype, precision, self.scaling, self.global_scale)
        if self.protection is None:
            return _Linear.apply(*args)
        return _Linear.apply(*args, self.protection, self.layer_name)


CutlassLinear = ProtectedLinear


def protection_sessions(model):
    """Distinct protection sessions with their sorted layer paths (tied
    aliases included), sorted by layer list."""
    groups = {}
    for name, module in model.named_modules(remove_duplicate=False):
        if isinstance(module, ProtectedLinear) and module.protection is not None:
            group = groups.setdefault(id(module.protection), {"layers": [], "session": module.protection.session})
            group["layers"].append(name)
    for group in groups.values():
        group["layers"].sort()
    return sorted(groups.values(), key=lambda group: group["layers"])


def install(model, precision=None, scaling="none", global_scale="amax", *, abft_config=None, fault_config=None,
            report_max_records=0, report_path=None):
    """Replace every nn.Linear, preserving parameter identity and sharing."""
    abft_config, fault_config = parse_abft_config(abft_config), parse_fault_config(fault_config)
    protection = None
    if abft_config.method != "none" or fault_config.location != "none":
        protection = _Protection(abft_config, fault_config, report_max_records, report_path)
    if isinstance(model, nn.Linear) and not isinstance(model, ProtectedLinear):
        return ProtectedLinear(model, precision, scaling, global_scale, protection)
    found = [(name, module) for name, module in model.named_modules(remove_duplicate=False)
             if isinstance(module, nn.Linear) and not isinstance(module, ProtectedLinear)]
    if not found:
        raise ValueError("the model has no nn.Linear to replace")
    replaced = {}
    for name, module in found:
        if id(module) not in replaced:
            replaced[id(module)] = ProtectedLinear(module, precision, scaling, global_scale, protection, name)
        parent, _, attribute = name.rpartition(".")
        setattr(model.get_submodule(parent) if parent else model, attribute, replaced[id(module)])
    return model
