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


def test_multi_tensor_pipeline_rope_and_topk():
    """Pipeline with several inputs and outputs along one leading dim: RoPE (q, k, position ids -> q_out, k_out) and
    top-k (x -> values, indices) give exactly the direct calls' results."""
    from ckb200 import rope, topk, workloads

    g = torch.Generator().manual_seed(4)
    tokens = 1000
    hq = torch.randn(tokens, 32, 128, generator=g).to(torch.bfloat16).pin_memory()
    hk = torch.randn(tokens, 8, 128, generator=g).to(torch.bfloat16).pin_memory()
    hids = torch.randint(0, 4096, (tokens,), generator=g).pin_memory()
    c, s = workloads._rope_cache(10000.0, 128, 4096, torch.float32)
    cos, sin = c.cuda(), s.cuda()

    def rope_op(ins, outs):
        rope.rope(ins[0][None], ins[1][None], ins[2][None], cos, sin, out=(outs[0][None], outs[1][None]))

    pipe = hostpipe.Pipeline(rope_op, [((tokens, 32, 128), torch.bfloat16), ((tokens, 8, 128), torch.bfloat16),
                                       ((tokens,), torch.int64)],
                             [((tokens, 32, 128), torch.bfloat16), ((tokens, 8, 128), torch.bfloat16)], chunks=3)
    oq, ok = torch.empty_like(hq).pin_memory(), torch.empty_like(hk).pin_memory()
    pipe([hq, hk, hids], [oq, ok])
    pipe.synchronize()
    wq, wk = rope.rope(hq[None].cuda(), hk[None].cuda(), hids[None].cuda(), cos, sin)
    assert torch.equal(oq.view(torch.int16), wq[0].cpu().view(torch.int16))
    assert torch.equal(ok.view(torch.int16), wk[0].cpu().view(torch.int16))
    assert pipe.bytes_per_call() == (hq.numel() * 2 + hk.numel() * 2 + tokens * 8, hq.numel() * 2 + hk.numel() * 2)

    hx = (torch.randn(300, 50000, generator=g) * 3).pin_memory()
    pipe = hostpipe.Pipeline(lambda ins, outs: topk.topk(ins[0], 50, out=(outs[0], outs[1])),
                             [((300, 50000), torch.float32)], [((300, 50), torch.float32), ((300, 50), torch.int64)],
                             chunks=4)
    hv, hi = torch.empty(300, 50).pin_memory(), torch.empty(300, 50, dtype=torch.int64).pin_memory()
    pipe([hx], [hv, hi])
    pipe.synchronize()
    wv, wi = topk.topk(hx.cuda(), 50)
    assert torch.equal(hi, wi.cpu()) and torch.equal(hv, wv.cpu())


def test_pipeline_waits_for_the_callers_stream():
    """A weight the op reads, written on the caller's stream just before the call (behind a long kernel), is seen:
    the pipeline's streams wait for the caller's stream at each call."""
    rows, cols = 64, 4096
    g = torch.Generator().manual_seed(8)
    w = torch.zeros(cols, device="cuda")
    pipe = hostpipe.RowPipeline(lambda x, y: rmsnorm.rmsnorm(x, w, out=y), rows, cols, torch.bfloat16, chunks=2)
    hx = torch.randn(rows, cols, generator=g).to(torch.bfloat16).pin_memory()
    hy = torch.empty_like(hx).pin_memory()
    big = torch.randn(8192, 8192, device="cuda")
    big = big @ big  # keeps the caller's stream busy for a while
    w.fill_(1.0)  # queued on the caller's stream after the matmul
    pipe(hx, hy)
    pipe.synchronize()
    want = rmsnorm.rmsnorm(hx.cuda(), torch.ones(cols, device="cuda")).cpu()
    assert torch.equal(hy.view(torch.int16), want.view(torch.int16))
