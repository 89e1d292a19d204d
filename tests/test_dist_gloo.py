"""The multi-GPU host path with world_size 2 on the CPU (gloo): the exchange of the vocab-sharded top-k, row
sharding and RoPE token sharding. The kernels' CPU stand-ins here are the oracle's (test infrastructure); the exchange code is the product's
(ckb200.sharded.gather_lists)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gather_tokens(t, sizes):
    """All-gather of every rank's [1, n_r, ...] token shard (n_r from sizes, which may differ by one): padded to the
    largest shard for the collective, trimmed after, concatenated along the tokens."""
    import torch.distributed as dist

    most = max(b - a for a, b in sizes)
    pad = torch.zeros((1, most, *t.shape[2:]), dtype=t.dtype, device=t.device)
    pad[:, :t.shape[1]] = t
    parts = [torch.empty_like(pad) for _ in sizes]
    dist.all_gather(parts, pad)
    return torch.cat([p[:, :b - a] for p, (a, b) in zip(parts, sizes)], 1)


def _worker(rank, world, port, q):
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    sys.path[:0] = [root, os.path.join(root, "cuda-kernels-optimized-for-rtx5090_b200")]
    from ckb200 import sharded
    from oracle import topk as otk

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(60))
        g = torch.Generator().manual_seed(11)
        x = (torch.randn(16, 3001, generator=g) * 3)
        x[:, 100:200] = 2.5  # ties across a shard boundary
        a, b = sharded.col_range(x.shape[1], rank, world)
        lists = otk.shard_lists(x[:, a:b], a, 50)
        gathered = sharded.gather_lists(lists)
        v, i = otk.merge_lists(gathered, torch.float32, 50)
        wv, wi = otk.topk(x, 50)
        ok_topk = torch.equal(i, wi) and torch.equal(v, wv)
        # row sharding: every rank's rows, gathered, cover the global rows once
        r0, r1 = sharded.row_range(16384, rank, world)
        span = torch.tensor([r0, r1])
        spans = [torch.zeros(2, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(spans, span)
        ok_rows = spans[0][0] == 0 and spans[-1][1] == 16384 and all(
            spans[j][1] == spans[j + 1][0] for j in range(world - 1))
        # token sharding of RoPE: every rank rotates its own tokens (the oracle stands in for the kernel here);
        # gathered over the ranks they equal the whole batch's rotation
        from ckb200 import workloads
        from oracle import rope as orope
        rp = workloads.rope_8x4096(integer=True, batch=3, seq=101)
        tq = sharded.token_shard(rp["q"], rank, world)
        tk = sharded.token_shard(rp["k"], rank, world)
        ids = sharded.token_shard(rp["position_ids"], rank, world)
        mq, _ = orope.rope(tq, tk, rp["cos"], rp["sin"], ids)
        sizes = [sharded.token_range(303, r, world) for r in range(world)]
        gathered = _gather_tokens(mq.contiguous().view(torch.float16), sizes)  # moved as raw 16-bit words
        wq, _ = orope.rope(rp["q"], rp["k"], rp["cos"], rp["sin"], rp["position_ids"])
        ok_rows = ok_rows and torch.equal(gathered.view(torch.int16), wq.view(1, -1, 32, 128).view(torch.int16))
        q.put((rank, bool(ok_topk), bool(ok_rows)))
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e), False))


def test_vocab_sharded_topk_exchange_and_row_sharding_world2():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, ok_topk, ok_rows in results:
        assert ok_topk is True, f"rank {rank}: {ok_topk}"
        assert ok_rows is True, f"rank {rank}"
