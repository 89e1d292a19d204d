"""The peer-memory vocab-sharded top-k kernels on one GPU: W ranks emulated in one process, every rank's exchange
buffer on this GPU, every push queued before any merge (so no kernel waits on one that has not run; the fused
push-and-merge kernel, which waits inside, is only run here with one rank). Each rank's
merge must give the single-GPU top-k of the full rows bit for bit, over several epochs (both parity halves).
The bounded wait: a merge whose flags nothing sets gives up after its limit and reports through the status word."""

import ctypes

import pytest
import torch

from ckb200 import _native, sharded
from ckb200 import topk as tk
from oracle import topk as otk

pytestmark = pytest.mark.gpu


class _Buffers:
    def __init__(self, world, rows, k):
        self.lib = _native.load("topk")
        self.half, self.lo, self.fo = sharded.exchange_layout(world, rows, k)
        self.bases = []
        for _ in range(world):
            p = ctypes.c_void_p()
            assert self.lib.ckb_p2p_alloc(ctypes.byref(p), 2 * self.half) == 0
            self.bases.append(p.value)

    def ptrs(self, epoch):
        par = (epoch & 1) * self.half
        return [b + par + self.lo for b in self.bases], [b + par + self.fo for b in self.bases]

    def free(self):
        for b in self.bases:
            self.lib.ckb_p2p_free(ctypes.c_void_p(b))


@pytest.mark.parametrize("world", [1, 2, 3, 8])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_emulated_ranks_match_the_single_gpu_topk(world, dtype):
    rows, cols, k = 96, 40001, 50
    g = torch.Generator().manual_seed(world)
    buf = _Buffers(world, rows, k)
    try:
        epoch = 0
        for call in range(3):
            epoch = sharded.next_epoch(epoch)
            x = (torch.randn(rows, cols, generator=g) * 3).to(dtype)
            x[call, :] = 1.0  # a row of ties
            lists, flags = buf.ptrs(epoch)
            for r in range(world):
                lo, hi = sharded.col_range(cols, r, world)
                tk.shard_push(x[:, lo:hi].contiguous().cuda(), lo, k, lists, flags, r, epoch)
            want_v, want_i = otk.topk(x, k)
            for r in range(world):
                v, i = tk.merge_wait(lists[r], flags[r], world, epoch, rows, k, dtype, torch.device("cuda"))
                assert torch.equal(i.cpu(), want_i), f"rank {r} call {call}: indices"
                assert torch.equal(v.cpu(), want_v), f"rank {r} call {call}: values"
        assert _native.load("topk").ckb_topk_status(1) == 0
    finally:
        torch.cuda.synchronize()
        buf.free()


def test_single_rank_class_repeated_calls():
    x = torch.randn(64, 20000, generator=torch.Generator().manual_seed(5))
    op = sharded.PeerVocabShardedTopK(64, 50)
    try:
        for _ in range(4):
            v, i = op(x.cuda(), 0)
            wv, wi = otk.topk(x, 50)
            assert torch.equal(i.cpu(), wi) and torch.equal(v.cpu(), wv)
    finally:
        op.close()


def test_single_rank_fused_kernel_and_graph_replays():
    """One rank: the shard kernel merges in place (it waits only on its own flags); four captured graphs replayed in
    rotation keep giving the same answer."""
    x = torch.randn(512, 30011, generator=torch.Generator().manual_seed(6))
    xd = x.cuda()
    op = sharded.PeerVocabShardedTopK(512, 50)
    try:
        step = op.graphed(xd, 0)
        wv, wi = otk.topk(x, 50)
        for _ in range(9):
            v, i = step()
            torch.cuda.synchronize()
            assert torch.equal(i.cpu(), wi) and torch.equal(v.cpu(), wv)
        assert _native.load("topk").ckb_topk_status(1) == 0
    finally:
        op.close()


def test_merge_wait_that_nothing_releases_reports_a_timeout():
    lib = _native.load("topk")
    lib.ckb_topk_status(1)
    buf = _Buffers(2, 1, 8)
    try:
        lists, flags = buf.ptrs(1)
        # Rank 0 publishes its list; rank 1 never does, so the merge's wait on rank 1's flag runs out.
        x = torch.randn(1, 4096, generator=torch.Generator().manual_seed(9))
        tk.shard_push(x.cuda(), 0, 8, lists, flags, 0, 1)
        tk.merge_wait(lists[0], flags[0], 2, 1, 1, 8, torch.float32, torch.device("cuda"))
        torch.cuda.synchronize()
        assert lib.ckb_topk_status(1) == 1
        assert lib.ckb_topk_status(0) == 0
    finally:
        buf.free()


def test_class_check_raises_after_a_timed_out_wait_and_refuses_further_calls():
    """A timed-out peer wait is never silent: check() raises, and the object refuses calls until rebuilt. The timeout
    is made as above (a merge whose peer flag nothing sets), after the object exists, on the same device."""
    x = torch.randn(16, 4096, generator=torch.Generator().manual_seed(10))
    op = sharded.PeerVocabShardedTopK(16, 8)
    buf = _Buffers(2, 1, 8)
    try:
        op(x.cuda(), 0)
        op.check()  # fine so far
        lists, flags = buf.ptrs(1)
        tk.merge_wait(lists[0], flags[0], 2, 1, 1, 8, torch.float32, torch.device("cuda"))
        with pytest.raises(RuntimeError, match="ran out"):
            op.check()
        with pytest.raises(RuntimeError, match="rebuild"):
            op(x.cuda(), 0)
        assert _native.load("topk").ckb_topk_status(0) == 0  # check() cleared the word
    finally:
        torch.cuda.synchronize()
        buf.free()
        op.close()
