"""Multi-GPU ABFT: row-sharded protected GEMMs with one status exchange.

The path partitions along M: every rank holds its own rows of A and the whole
of B, runs the protected GEMM of its shard on its own GPU and keeps its rows
of the output. What crosses ranks:

* the maximum |A| (``"amax"`` policy, FP8 tensorwise and NVFP4): one fp32
  MAX all-reduce at prepare time whose result stays on the device and feeds
  the quantizer directly, so each shard is quantised with exactly the
  multiplier of the unsharded matrix (its output rows are bit-identical to
  the same rows of the unsharded GEMM) and nothing is read back to the host;
* the verdict: one all-gather of a float64[10] vector per GEMM (detected,
  nonfinite, located, fault hit, recovered, recheck failed, global row,
  column, max |residual| / threshold, max |residual|), from which every
  rank derives the same global decision (sums of the flags, maxima of the
  residual norms). A single located error is located globally only when
  exactly one shard located one.

Every rank takes the same collective steps in the same order, faults or
not; ``on_error="raise"`` is applied after the exchange on every rank, so a
detection on one shard never leaves the others waiting in a collective.
Passing ``row_offset`` and ``total_rows`` (known when the shards come from
``shard_rows``) skips the one collective that reads shard sizes to the host.

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
    """All ranks' shard row counts -> (this rank's first global row, total m).
    One all-gather; the counts are read to the host once."""
    world = dist.get_world_size(group)
    local = torch.tensor([rows], dtype=torch.int64, device=_device(group))
    gathered = [torch.zeros_like(local) for _ in range(world)]
    dist.all_gather(gathered, local, group=group)
    counts = torch.cat(gathered).tolist()
    rank = dist.get_rank(group)
    return sum(counts[:rank]), sum(counts)


def global_amax(shard, group=None):
    """max |x| over every rank's shard, as a device fp32 scalar (one MAX
    all-reduce; nothing is read to the host). NaN propagates like torch.amax."""
    amax = shard.detach().abs().amax().float() if shard.numel() else torch.zeros((), device=shard.device)
    value = amax.reshape(1).to(_device(group))
    dist.all_reduce(value, op=dist.ReduceOp.MAX, group=group)
    return value.reshape(())


def global_multiplier(shard, precision, group=None):
    """The ``"amax"`` multiplier of the unsharded matrix as a host float
    (limit / max |x| in fp32, 1 when the maximum is 0; "amax" when it is not
    finite). Reads the maximum to the host; the sharded executor itself uses
    ``global_amax`` and never does."""
    maximum = float(global_amax(shard, group).item())
    if maximum != maximum or maximum in (float("inf"), -float("inf")):
        return "amax"
    if maximum == 0.0:
        return 1.0
    return float(torch.tensor(_LIMIT[precision], dtype=torch.float32) / torch.tensor(maximum, dtype=torch.float32))


EXCHANGE_FIELDS = ("detected", "nonfinite", "located", "fault_hit", "recovered", "recheck_failed", "row", "col",
                   "max_residual_over_threshold", "max_abs_residual")


def _status_vector(tensors, row_offset, device):
    """This rank's float64[10] verdict (see EXCHANGE_FIELDS); residual norms
    are -1 when the call kept no residuals (diagnostics off)."""
    def flag(name):
        value = tensors.get(name)
        if value is None:
            return torch.zeros((), dtype=torch.float64, device=device)
        return value.reshape(-1)[:1].to(device=device, dtype=torch.float64).reshape(()).clamp(0, 1)

    located = flag("located")
    location = tensors.get("location")
    location = (torch.full((2,), -1.0, dtype=torch.float64, device=device) if location is None
                else location.to(device=device, dtype=torch.float64))
    residual, threshold = tensors.get("residual"), tensors.get("threshold")
    if residual is None or threshold is None or residual.numel() == 0:
        norms = torch.full((2,), -1.0, dtype=torch.float64, device=device)
    else:
        res = residual.detach().abs().to(device=device, dtype=torch.float64)
        norms = torch.stack(((res / threshold.detach().to(device=device, dtype=torch.float64)).amax(), res.amax()))
    return torch.cat((torch.stack((flag("detected"), flag("nonfinite"), located, flag("fault_hit"),
                                   flag("recovered"), flag("recheck_failed"), located * (location[0] + row_offset),
                                   located * location[1])), norms))


def allreduce_status(tensors, row_offset, group=None):
    """One all-gather of the verdict vectors; returns the global verdict
    tensors (on the exchange device) in the engine's report vocabulary."""
    device = _device(group)
    local = _status_vector(tensors, row_offset, device)
    gathered = [torch.empty_like(local) for _ in range(dist.get_world_size(group))]
    dist.all_gather(gathered, local, group=group)
    table = torch.stack(gathered)
    sums, norms = table[:, :8].sum(dim=0), table[:, 8:].amax(dim=0)
    single = sums[2] == 1
    location = torch.where(single, sums[6:8], torch.full_like(sums[6:8], -1)).to(torch.int64)
    return {"detected": sums[0] > 0, "nonfinite": sums[1] > 0, "located": single, "location": location,
            "fault_hit": sums[3].to(torch.int64), "shards_detected": sums[0].to(torch.int64),
            "shards_located": sums[2].to(torch.int64), "recovered": (sums[0] > 0) & (sums[4] == sums[0]),
            "recheck_failed": sums[5] > 0, "max_residual_over_threshold": norms[0], "max_abs_residual": norms[1]}


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
                    group=None, global_scale="amax", row_offset=None, total_rows=None, **engine_kwargs):
    """Protected GEMM of this rank's rows ``a_rows`` (local [m_i, K]) times the
    replicated ``b`` ([K, N]). ``fault_config`` rows are GLOBAL rows; the fault
    fires on the rank that owns that row. ``row_offset``/``total_rows`` may
    be given to skip the shard-size exchange. Returns (local output rows,
    ShardedReport). ``engine_kwargs`` are passed to the engine (the reference
    implementation's collector seams)."""
    from .engine import execute_prepared

    cfg, fault = parse_abft_config(abft_config), parse_fault_config(fault_config)
    if (row_offset is None) != (total_rows is None):
        raise ValueError("row_offset and total_rows are given together or not at all")
    offset, total = (row_offset, total_rows) if row_offset is not None else row_offsets(a_rows.shape[0], group)
    shared_amax = precision in _LIMIT and global_scale == "amax" and scaling != "blockwise"
    amax = global_amax(a_rows, group) if shared_amax else None
    local_fault = fault
    if fault.location in {"accumulator", "a"}:
        inside = offset <= fault.row < offset + a_rows.shape[0]
        local_fault = parse_fault_config({**vars(fault), "row": fault.row - offset} if inside else None)
    report_cfg = cfg if cfg.method == "none" else parse_abft_config({**vars(cfg), "on_error": "report"})
    output, report = None, None
    if a_rows.shape[0] > 0:
        if shared_amax:
            prepared = _prepare_split(a_rows, b, precision, scaling, amax, global_scale)
        else:
            # Block scales are per row (A) and per 128 x 128 block of B, so a
            # row shard quantises exactly like the same rows of the whole A.
            prepared = PreparedGemm.prepare(a_rows, b, precision, scaling, global_scale)
        output, report = execute_prepared(prepared, report_cfg, local_fault, context, **engine_kwargs)
    verdict = allreduce_status(report.tensors if report is not None else {}, offset, group)
    if shared_amax and report is not None:
        verdict["a_multiplier"] = prepared.qa.multiplier  # device scalar, read only by to_record
    ctx = {"rank": dist.get_rank(group), "world_size": dist.get_world_size(group), "row_offset": offset,
           "m": total, "rows": a_rows.shape[0], "a_multiplier": "global_amax" if shared_amax else global_scale,
           "exchange": "all_gather_float64x10"}
    sharded = ShardedReport(report, verdict, ctx)
    if cfg.method != "none" and cfg.on_error == "raise" and bool(
            (verdict["detected"] & ~verdict["recovered"]).item()):
        raise ShardedAbftError(sharded)
    return output, sharded


def _prepare_split(a_rows, b, precision, scaling, amax, scale_b):
    """PreparedGemm with A quantised at the whole matrix's multiplier (from
    the device ``amax``) and B at its own."""
    from .. import require_device
    from ..gemm.quantization import quantize

    if scaling != {"fp8": "tensorwise", "nvfp4": "block16"}[precision]:
        raise ValueError("Incompatible precision/scaling")
    if a_rows.ndim != 2 or b.ndim != 2 or a_rows.shape[1] != b.shape[0]:
        raise ValueError("GEMM requires compatible matrices on one device")
    require_device(a_rows.device)
    qa = quantize(a_rows.contiguous(), precision, "amax", amax=amax)
    qb = quantize(b.T.contiguous(), precision, scale_b)
    alpha = (qa.multiplier * qb.multiplier).reciprocal()
    prepared = PreparedGemm(qa.codes, qb.codes, precision, a_rows.shape[0], b.shape[1], a_rows.shape[1], qa, qb,
                            alpha)
    if precision == "nvfp4":
        prepared.sfa, prepared.sfb = qa.scales_mma, qb.scales_mma
    return prepared
