"""ckb200.hostpipe.RowPipeline: pinned host batches through an op with overlapped copies give exactly the op's own
result (the same kernels on the same rows), call after call, for chunk counts that do and do not divide the rows."""

import pytest
import torch

from ckb200 import hostpipe, rmsnorm, softmax

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,chunks", [(1000, 8), (1024, 8), (7, 3), (5, 16), (1, 1)])
def test_rmsnorm_matches_direct_call(rows, chunks):
    g = torch.Generator().manual_seed(rows)
    cols = 4096
    w = torch.randn(cols, generator=g).cuda()
    pipe = hostpipe.RowPipeline(lambda x, y: rmsnorm.rmsnorm(x, w, out=y), rows, cols, torch.bfloat16, chunks=chunks)
    for call in range(3):  # the slots are reused across calls
        hx = torch.randn(rows, cols, generator=g).to(torch.bfloat16).pin_memory()
        hy = torch.empty_like(hx).pin_memory()
        pipe(hx, hy)
        pipe.synchronize()
        want = rmsnorm.rmsnorm(hx.cuda(), w).cpu()
        assert torch.equal(hy.view(torch.int16), want.view(torch.int16)), f"call {call}"


def test_softmax_through_the_pipeline():
    rows, cols = 300, 8192
    x = torch.randn(rows, cols, generator=torch.Generator().manual_seed(3))
    pipe = hostpipe.RowPipeline(lambda a, b: softmax.softmax(a, out=b), rows, cols, torch.float32, chunks=4)
    hx, hy = x.pin_memory(), torch.empty_like(x).pin_memory()
    pipe(hx, hy)
    pipe.synchronize()
    assert torch.equal(hy, softmax.softmax(x.cuda()).cpu())


def test_rejects_unpinned_or_misshapen_host_tensors():
    pipe = hostpipe.RowPipeline(lambda a, b: b.copy_(a), 4, 8, torch.float32)
    good = torch.zeros(4, 8).pin_memory()
    with pytest.raises(ValueError, match="pinned"):
        pipe(torch.zeros(4, 8), good)
    with pytest.raises(ValueError, match="contiguous host tensor"):
        pipe(torch.zeros(4, 9).pin_memory(), good)
