"""Row-sharded ABFT over torch.distributed, tested as gloo ranks on the CPU.

Two processes (world size 2, rendezvous on 127.0.0.1) run the engine's
reference implementation through the fp32 collector seam on their row shards;
the verdict exchange, global location, fault ownership, raise-on-every-rank
and the global amax multiplier are the host logic under test.
"""
import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from sdc_b200.abft.distributed import (ShardedAbftError, allreduce_status, execute_sharded, global_multiplier,
                                       shard_rows)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def collect(operands, weights, fault):
    a, b = operands.decode_block(0, operands.k)
    output = a @ b
    row, col, bit = fault
    if row >= 0:
        output.view(torch.int32)[row, col] ^= (1 << bit) if bit < 31 else -(1 << 31)
    return output, (weights @ output).unsqueeze(1), torch.tensor([int(row >= 0)])


def _operands():
    g = torch.Generator().manual_seed(42)
    return torch.randn(300, 64, generator=g), torch.randn(64, 40, generator=g)


def _scenario(name, rank, world):
    a, b = _operands()
    start, stop = shard_rows(a.shape[0], world, rank)
    rows = a[start:stop]
    kwargs = dict(reference_mm=torch.mm, collector_fn=collect)
    if name == "clean":
        out, report = execute_sharded(rows, b, "fp32", "none", {"method": "classic", "on_error": "report"}, **kwargs)
        return {"rows": (start, stop), "out": out, "record": report.to_record()}
    if name == "fault":
        cfg = {"method": "classic", "on_error": "report", "recovery": "recompute", "rtol": 1e-6}
        fault = {"location": "accumulator", "row": 201, "col": 34, "bit": 24}
        out, report = execute_sharded(rows, b, "fp32", "none", cfg, fault, **kwargs)
        return {"rows": (start, stop), "out": out, "record": report.to_record()}
    if name == "raise":
        fault = {"location": "accumulator", "row": 5, "col": 3, "bit": 30}
        try:
            execute_sharded(rows, b, "fp32", "none", {"method": "classic"}, fault, **kwargs)
        except ShardedAbftError as error:
            return {"raised": True, "detected": bool(error.report.detected)}
        return {"raised": False}
    if name == "ambiguous":
        tensors = {"detected": torch.tensor(True), "located": torch.tensor(True),
                   "location": torch.tensor([3, 7]), "fault_hit": torch.tensor([1])}
        both = allreduce_status(tensors, 128 * rank)
        one = allreduce_status(tensors if rank == 1 else {}, 128 * rank)
        return {"both": [bool(both["located"]), both["location"].tolist()],
                "one": [bool(one["located"]), one["location"].tolist(), bool(one["detected"])]}
    if name == "norms":
        residual = torch.tensor([[1.0, -4.0 * (rank + 1)], [0.5, 2.0]])
        threshold = torch.tensor([[8.0, 8.0], [1.0, 64.0]])
        verdict = allreduce_status({"detected": torch.tensor(False), "residual": residual,
                                    "threshold": threshold}, 128 * rank)
        quiet = allreduce_status({"detected": torch.tensor(rank == 0)}, 128 * rank)
        return {"norms": [float(verdict["max_residual_over_threshold"]), float(verdict["max_abs_residual"])],
                "quiet": [float(quiet["max_residual_over_threshold"]), bool(quiet["detected"]),
                          int(quiet["shards_detected"])]}
    if name == "explicit_offsets":
        out, report = execute_sharded(rows, b, "fp32", "none", {"method": "classic", "on_error": "report"},
                                      row_offset=start, total_rows=a.shape[0], **kwargs)
        return {"rows": (start, stop), "out": out, "record": report.to_record()}
    if name == "multiplier":
        x = torch.randn(stop - start, 32, generator=torch.Generator().manual_seed(rank)) * (rank + 1)
        return {"st": global_multiplier(x, "fp8"), "local_amax": float(x.abs().amax()),
                "st4": global_multiplier(x, "nvfp4")}
    raise ValueError(name)


def _worker(rank, world, port, name, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, init_method=f"tcp://127.0.0.1:{port}")
        results[rank] = _scenario(name, rank, world)
    except Exception:  # reported to the parent, which fails the test
        results[rank] = {"error": traceback.format_exc()}
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _run(name, world=2):
    with mp.get_context("spawn").Manager() as manager:
        results = manager.dict()
        mp.start_processes(_worker, args=(world, _free_port(), name, results), nprocs=world, join=True,
                           start_method="spawn")
        out = [results[r] for r in range(world)]
    for r in out:
        assert "error" not in r, r.get("error")
    return out


def test_shard_rows_cover_m_in_tile_multiples():
    for m in (1, 127, 128, 300, 1024, 8192, 8193):
        for world in (1, 2, 3, 4, 8):
            ranges = [shard_rows(m, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == m
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            assert all(start % 128 == 0 for start, stop in ranges if stop > start)
            tiles = [-(-(stop - start) // 128) for start, stop in ranges]
            assert max(tiles) - min(tiles) <= 1
    with pytest.raises(ValueError):
        shard_rows(10, 2, 2)


def test_clean_sharded_run_matches_unsharded_rows():
    a, b = _operands()
    results = _run("clean")
    full = a @ b
    for r in results:
        start, stop = r["rows"]
        assert torch.equal(r["out"], full[start:stop])
        assert r["record"]["detected"] is False and r["record"]["located"] is False
        assert r["record"]["context"]["row_offset"] == start and r["record"]["context"]["m"] == 300


def test_fault_on_one_shard_is_seen_located_and_recovered_by_all():
    a, b = _operands()
    results = _run("fault")
    for r in results:
        rec = r["record"]
        assert rec["detected"] is True and rec["located"] is True
        assert rec["location"] == [201, 34]
        assert rec["fault_hit"] == 1 and rec["recovered"] is True
        start, stop = r["rows"]
        assert torch.equal(r["out"], (a @ b)[start:stop])
    owner = [r for r in results if r["rows"][0] <= 201 < r["rows"][1]]
    assert len(owner) == 1 and owner[0]["record"]["local"]["detected"] is True


def test_unrecovered_detection_raises_on_every_rank():
    results = _run("raise")
    assert all(r["raised"] and r["detected"] for r in results)


def test_two_located_shards_are_ambiguous():
    results = _run("ambiguous")
    for r in results:
        assert r["both"] == [False, [-1, -1]]
        assert r["one"] == [True, [131, 7], True]


def test_global_multiplier_is_the_unsharded_amax_policy():
    results = _run("multiplier")
    amax = max(r["local_amax"] for r in results)
    expected = float(torch.tensor(448.0) / torch.tensor(amax))
    assert all(r["st"] == expected for r in results)
    assert all(r["st4"] == float(torch.tensor(2688.0) / torch.tensor(amax)) for r in results)


def test_exchange_carries_residual_norms():
    results = _run("norms")
    for r in results:
        # Rank 1's column 1: |res| 8 against threshold 8 (ratio 1); the largest |res| is 8.
        assert r["norms"] == [1.0, 8.0]
        # Without residuals the norms are reported as -1; flags still sum.
        assert r["quiet"] == [-1.0, True, 1]


def test_explicit_offsets_skip_the_size_exchange():
    a, b = _operands()
    for r in _run("explicit_offsets"):
        start, stop = r["rows"]
        assert torch.equal(r["out"], (a @ b)[start:stop])
        assert r["record"]["context"]["row_offset"] == start and r["record"]["context"]["m"] == 300
        assert r["record"]["detected"] is False
