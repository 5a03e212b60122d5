"""Multi-GPU ABFT: row-sharded protected GEMMs with one status exchange.

The path partitions along M: every rank holds its own rows of A and the whole
of B, runs the protected GEMM of its shard on its own GPU and keeps its rows
of the output. The only data that crosses ranks is

* the operand multiplier of A (``"amax"`` policy): one fp32 MAX all-reduce at
  prepare time, so each shard is quantised with exactly the multiplier the
  unsharded matrix would get and the shard's output rows are bit-identical to
  the same rows of the unsharded GEMM;
* the verdict: one SUM all-reduce of an int64[8] status vector per GEMM
  (detected, nonfinite, located, fault hit, recovered, recheck failed, global
  row, column), from which every rank derives the same global decision. A
  single located error is located globally only when exactly one shard
  located one.

Every rank takes the same collective steps in the same order, faults or
not; ``on_error="raise"`` is applied after the exchange on every rank, so a
detection on one shard never leaves the others waiting in a collective.

Works with NCCL (CUDA tensors) and with gloo (CPU tensors; the engine's
reference implementation and collector seams), which is how the host logic is
tested without GPUs.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .config import parse_abft_config, parse_fault_config
from .engine import AbftError
from .operands import PreparedGemm

_LIMIT = {"fp8": 448.0, "nvfp4": 6.0 * 448.0}
STATUS_FIELDS = ("detected", "nonfinite", "located", "fault_hit", "recovered", "recheck_failed", "row", "col")


def shard_rows(m, world, rank, align=128):
    """[start, stop) of rank's rows: contiguous, multiples of ``align`` (one
    GEMM M tile) except the last, as even as that allows. Empty shards are
    allowed when m is small."""
    if m < 0 or world <= 0 or not 0 <= rank < world or align <= 0:
        raise ValueError("shard_rows needs m >= 0, world > 0, 0 <= rank < world, align > 0")
    tiles = -(-m // align)
    base, extra = divmod(tiles, world)
    first = rank * base + min(rank, extra)
    count = base + (1 if rank < extra else 0)
    return min(m, first * align), min(m, (first + count) * align)


def _device(group):
    if dist.get_backend(group) == "nccl":
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def row_offsets(rows, group=None):
    """All ranks' shard row counts -> (this rank's first global row, total m)."""
    world = dist.get_world_size(group)
    local = torch.tensor([rows], dtype=torch.int64, device=_device(group))
    gathered = [torch.zeros_like(local) for _ in range(world)]
    dist.all_gather(gathered, local, group=group)
    counts = [int(t.item()) for t in gathered]
    rank = dist.get_rank(group)
    return sum(counts[:rank]), sum(counts)


def global_multiplier(shard, precision, group=None):
    """The ``"amax"`` multiplier of the unsharded matrix (limit / max |x| in
    fp32, 1 when the maximum is 0), from one MAX all-reduce. Returns "amax"
    (each shard on its own) when the maximum is not finite, so the nonfinite
    input is still quantised and detected where it lives."""
    amax = shard.detach().abs().amax().float() if shard.numel() else torch.zeros((), device=shard.device)
    value = amax.reshape(1).to(_device(group))
    dist.all_reduce(value, op=dist.ReduceOp.MAX, group=group)
    maximum = float(value.item())
    if maximum != maximum or maximum in (float("inf"), -float("inf")):
        return "amax"
    if maximum == 0.0:
        return 1.0
    # Quotient of two fp32 values rounded once to fp32 (the f64 quotient is
    # exact enough that rounding it to fp32 is the correctly rounded fp32 one).
    return float(torch.tensor(_LIMIT[precision], dtype=torch.float32) / torch.tensor(maximum, dtype=torch.float32))


def allreduce_status(tensors, row_offset, group=None):
    """One SUM all-reduce of the verdict; returns the global verdict tensors
    (on the exchange device) in the engine's report vocabulary."""
    device = _device(group)

    def flag(name):
        value = tensors.get(name)
        if value is None:
            return torch.zeros((), dtype=torch.int64, device=device)
        return value.reshape(-1)[:1].to(device=device, dtype=torch.int64).reshape(()).clamp(0, 1)

    located = flag("located")
    location = tensors.get("location")
    if location is None:
        location = torch.full((2,), -1, dtype=torch.int64)
    location = location.to(device=device, dtype=torch.int64)
    status = torch.stack((flag("detected"), flag("nonfinite"), located, flag("fault_hit"), flag("recovered"),
                          flag("recheck_failed"), located * (location[0] + row_offset), located * location[1]))
    dist.all_reduce(status, op=dist.ReduceOp.SUM, group=group)
    single = status[2] == 1
    return {"detected": status[0] > 0, "nonfinite": status[1] > 0, "located": single,
            "location": torch.where(single, status[6:8], torch.full_like(status[6:8], -1)),
            "fault_hit": status[3], "shards_detected": status[0], "shards_located": status[2],
            "recovered": (status[0] > 0) & (status[4] == status[0]), "recheck_failed": status[5] > 0}


class ShardedReport:
    """A rank's local engine report plus the global verdict."""

    def __init__(self, local, verdict, context):
        self.local = local
        self.tensors = verdict
        self.context = context

    def __getattr__(self, name):
        tensors = self.__dict__.get("tensors", {})
        if name in tensors:
            return tensors[name]
        raise AttributeError(name)

    def to_record(self):
        record = {name: value.detach().cpu().tolist() for name, value in self.tensors.items()}
        record["context"] = self.context
        record["local"] = self.local.to_record() if self.local is not None else None
        return record


class ShardedAbftError(AbftError):
    pass


@torch.no_grad()
def execute_sharded(a_rows, b, precision, scaling, abft_config=None, fault_config=None, context=None, *,
                    group=None, global_scale="amax", **engine_kwargs):
    """Protected GEMM of this rank's rows ``a_rows`` (local [m_i, K]) times the
    replicated ``b`` ([K, N]). ``fault_config`` rows are GLOBAL rows; the fault
    fires on the rank that owns that row. Returns (local output rows,
    ShardedReport). ``engine_kwargs`` are passed to the engine (the reference
    implementation's collector seams)."""
    from .engine import execute_prepared

    cfg, fault = parse_abft_config(abft_config), parse_fault_config(fault_config)
    offset, total = row_offsets(a_rows.shape[0], group)
    if precision in _LIMIT and global_scale == "amax" and scaling != "blockwise":
        scale_a = global_multiplier(a_rows, precision, group)
    else:
        scale_a = global_scale
    local_fault = fault
    if fault.location in {"accumulator", "a"}:
        inside = offset <= fault.row < offset + a_rows.shape[0]
        local_fault = parse_fault_config({**vars(fault), "row": fault.row - offset} if inside else None)
    report_cfg = cfg if cfg.method == "none" else parse_abft_config({**vars(cfg), "on_error": "report"})
    output, report = None, None
    if a_rows.shape[0] > 0:
        if precision in _LIMIT and scaling != "blockwise":
            # Block scales are per row (A) and per 128 x 128 block of B, so a
            # row shard quantises exactly like the same rows of the whole A.
            prepared = _prepare_split(a_rows, b, precision, scaling, scale_a, global_scale)
        else:
            prepared = PreparedGemm.prepare(a_rows, b, precision, scaling, global_scale)
        output, report = execute_prepared(prepared, report_cfg, local_fault, context, **engine_kwargs)
    tensors = report.tensors if report is not None else {}
    verdict = allreduce_status(tensors, offset, group)
    ctx = {"rank": dist.get_rank(group), "world_size": dist.get_world_size(group), "row_offset": offset,
           "m": total, "rows": a_rows.shape[0], "a_multiplier": scale_a, "exchange": "sum_allreduce_int64x8"}
    sharded = ShardedReport(report, verdict, ctx)
    if cfg.method != "none" and cfg.on_error == "raise" and bool(
            (verdict["detected"] & ~verdict["recovered"]).item()):
        raise ShardedAbftError(sharded)
    return output, sharded


def _prepare_split(a_rows, b, precision, scaling, scale_a, scale_b):
    """PreparedGemm with A quantised at the global multiplier and B at its own."""
    from .. import require_device
    from ..gemm.quantization import quantize

    if scaling != {"fp8": "tensorwise", "nvfp4": "block16"}[precision]:
        raise ValueError("Incompatible precision/scaling")
    if a_rows.ndim != 2 or b.ndim != 2 or a_rows.shape[1] != b.shape[0]:
        raise ValueError("GEMM requires compatible matrices on one device")
    require_device(a_rows.device)
    qa = quantize(a_rows.contiguous(), precision, scale_a)
    qb = quantize(b.T.contiguous(), precision, scale_b)
    alpha = (qa.multiplier * qb.multiplier).reciprocal()
    prepared = PreparedGemm(qa.codes, qb.codes, precision, a_rows.shape[0], b.shape[1], a_rows.shape[1], qa, qb,
                            alpha)
    if precision == "nvfp4":
        prepared.sfa, prepared.sfb = qa.scales_mma, qb.scales_mma
    return prepared
