"""Row-sharded native ABFT over NCCL on two GPUs (skipped with fewer).

Each rank protects its 128-aligned row shard of A on its own GPU with the
fused FP8/NVFP4/block-scaled FP8 kernels; its output rows must equal the same
rows of the unsharded protected GEMM bit for bit (the A multiplier is the
global amax one; block scales are per row), and a fault on one shard must be
detected and located by every rank.
NVLS is off (NCCL_NVLS_ENABLE=0): the exchange is one tiny all-reduce.
"""
import os
import socket
import traceback

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, precision, results):
    precision, scaling = {"fp8": ("fp8", "tensorwise"), "nvfp4": ("nvfp4", "block16"),
                          "fp8_block": ("fp8", "blockwise")}[precision]
    import datetime

    import torch.distributed as dist

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        torch.cuda.set_device(rank)
        device = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, init_method=f"tcp://127.0.0.1:{port}",
                                timeout=datetime.timedelta(seconds=60), device_id=device)
        from sdc_b200.abft import execute
        from sdc_b200.abft.distributed import execute_sharded, shard_rows

        g = torch.Generator(device=device).manual_seed(21)
        m, n, k = 640, 384, 512
        a = torch.randn(m, k, device=device, generator=g)
        b = torch.randn(k, n, device=device, generator=g)
        cfg = {"method": "classic", "implementation": "native", "reference_mode": "input_fused",
               "on_error": "report", "atol": 1e-3, "rtol": 1e-4, "locate": True,
               "reference_layout": "kslice" if scaling == "blockwise" else "tile"}
        full, _ = execute(a, b, precision, scaling, abft_config=cfg)
        start, stop = shard_rows(m, world, rank)
        out, report = execute_sharded(a[start:stop], b, precision, scaling, cfg)
        same = bool(torch.equal(out, full[start:stop]))
        clean = report.to_record()
        # First element at or after (600, 77) with 4 <= |v| < 256: flipping
        # exponent bit 27 scales it by 2^16 (large, finite, locatable).
        flat = full.float().reshape(-1)[600 * n + 77:]
        index = 600 * n + 77 + int(((flat.abs() >= 4) & (flat.abs() < 256)).nonzero()[0, 0])
        row, col, bit = index // n, index % n, 27
        _, faulty = execute_sharded(a[start:stop], b, precision, scaling, cfg,
                                    {"location": "accumulator", "row": row, "col": col, "bit": bit})
        results[rank] = {"same": same, "clean_detected": clean["detected"], "record": faulty.to_record(),
                         "rows": (start, stop), "fault": [row, col]}
    except Exception:
        results[rank] = {"error": traceback.format_exc()}
    finally:
        import torch.distributed as dist
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("precision", ["fp8", "nvfp4", "fp8_block"])
def test_sharded_native_rows_bit_exact_and_verdict_global(precision):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        mp.start_processes(_worker, args=(2, _free_port(), precision, results), nprocs=2, join=True,
                           start_method="spawn")
        out = [results[r] for r in range(2)]
    for r in out:
        assert "error" not in r, r.get("error")
        assert r["same"] and r["clean_detected"] is False
        rec = r["record"]
        assert rec["detected"] is True and rec["located"] is True and rec["location"] == r["fault"]
