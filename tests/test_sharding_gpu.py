"""Row-sharded quantisation on one GPU: a shard quantised with the whole
matrix's maximum (a device scalar, as the NCCL MAX all-reduce of the shards'
maxima leaves it) gives exactly the rows of the unsharded quantisation, with
no host read of the maximum; the multi-GPU exchange itself is covered by the
gloo tests on the CPU and the two-GPU NCCL test."""
import pytest
import torch

import sdc_b200  # noqa: F401
from sdc_b200.abft.distributed import shard_rows
from sdc_b200.gemm.quantization import quantize

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("precision", ["fp8", "nvfp4"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_shard_with_global_amax_equals_unsharded_rows(precision, dtype):
    g = torch.Generator(device=DEV).manual_seed(7)
    x = (torch.randn(1000, 512, device=DEV, generator=g) * 3).to(dtype)
    x[937, 5] = 90.0  # the maximum lives in the last shard
    whole = quantize(x, precision)
    amax = x.abs().amax().float()
    for rank in range(4):
        start, stop = shard_rows(x.shape[0], 4, rank)
        shard = quantize(x[start:stop], precision, amax=amax)
        assert torch.equal(shard.multiplier, whole.multiplier)
        assert torch.equal(shard.codes, whole.codes[start:stop])
        if precision == "nvfp4":
            assert torch.equal(shard.scales, whole.scales[start:stop])
    with pytest.raises(ValueError, match="amax policy"):
        quantize(x, precision, 2.0, amax=amax)
