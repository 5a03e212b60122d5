"""Allocation-free finalize entry point (sdc_abft_finalize_noalloc).

Callers that cannot allocate device memory (a plain C/FFI host with no device
allocator of its own) use this entry point; its scratch lives in a fixed
device array inside the library. Checked through the C ABI against the
regular entry point, bit for bit (the finalize bar), on two calls in a row.
Collected last so a failure here never hides the other tests.
"""
import ctypes

import numpy as np
import pytest
import torch

import sdc_b200  # noqa: F401
from sdc_b200 import capi

pytestmark = pytest.mark.gpu


def _partials(tiles, n, seed):
    padded = ((n + 63) // 64) * 64
    g = torch.Generator().manual_seed(seed)
    p = torch.randn(3, 2, tiles, padded, generator=g)
    p[2].abs_()
    p[0, 1, tiles - 1, n - 1] += 50.0  # one detected column
    return p.cuda()


def _run(entry, p, n, use_workspace):
    lib = capi.lib()
    tiles, padded = p.shape[2], p.shape[3]
    obs, pred, mag = (p[i].contiguous() for i in range(3))
    hit = torch.ones(1, dtype=torch.int32, device="cuda")
    nonfinite = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = {"ref": torch.empty(2, 2, n, device="cuda"), "res": torch.empty(2, n, device="cuda"),
           "thr": torch.empty(2, n, device="cuda"), "flags": torch.empty(5, dtype=torch.uint8, device="cuda"),
           "hit": torch.empty(1, dtype=torch.int32, device="cuda"),
           "loc": torch.empty(2, dtype=torch.int64, device="cuda")}
    stream = torch.cuda.current_stream().cuda_stream
    args = [0, obs.data_ptr(), pred.data_ptr(), mag.data_ptr(), tiles, padded, n, None, 0, hit.data_ptr(),
            nonfinite.data_ptr(), 0.125, 0.25, out["ref"].data_ptr(), 0, 1, out["res"].data_ptr(),
            out["thr"].data_ptr(), None, 0, out["flags"].data_ptr(), out["hit"].data_ptr(), out["loc"].data_ptr()]
    if use_workspace:
        ws_bytes = lib.sdc_abft_finalize_workspace_bytes(0, n, tiles)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
        capi.check(entry(*args, ws.data_ptr(), ws_bytes, stream))
    else:
        capi.check(entry(*args, stream))
    torch.cuda.synchronize()
    return {k: v.cpu() for k, v in out.items()}


def test_noalloc_finalize_matches_workspace_entry_on_two_calls():
    lib = capi.lib()
    for call, (tiles, n) in enumerate([(9, 1025), (33, 257)]):
        p = _partials(tiles, n, seed=100 + call)
        expected = _run(lib.sdc_abft_finalize, p, n, use_workspace=True)
        actual = _run(lib.sdc_abft_finalize_noalloc, p, n, use_workspace=False)
        for key in expected:
            assert np.array_equal(actual[key].numpy().view(np.uint8), expected[key].numpy().view(np.uint8)), key
        assert actual["flags"].tolist() == [1, 0, 0, 0, 0] and actual["hit"].item() == 1


def test_noalloc_finalize_rejects_sizes_beyond_its_array():
    lib = capi.lib()
    # Every buffer is null: should the size check ever stop running first, the
    # regular argument checks still reject the call (with another message, so
    # the assertion fails) and nothing is launched.
    rc = lib.sdc_abft_finalize_noalloc(0, None, None, None, 1, 600000, 600000, None, 0, None, None, 0.0, 0.0,
                                       None, 0, 0, None, None, None, 0, None, None, None,
                                       torch.cuda.current_stream().cuda_stream)
    assert rc == capi.SDC_ERR_INVALID and "16384" in capi.last_error()
