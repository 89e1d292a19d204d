"""Multi-GPU paths over NCCL with one process per GPU (skipped with fewer than 2 GPUs):
  * the vocab-sharded top-k (local shard kernel -> all_gather_into_tensor -> merge kernel) gives every rank the
    single-GPU answer, bit for bit, and so does its peer-memory form (PeerVocabShardedTopK: NVLink stores and
    per-row flags instead of the collective), call after call (both parity halves, fp32 and bf16);
  * row sharding: each rank normalises its own rows; gathered, they equal the oracle;
  * token sharding: each rank rotates its own tokens of an integer-valued RoPE batch in place (sharded.token_shard,
    the cos/sin cache replicated); gathered, they equal the oracle bit for bit.
Ranks are spawned processes with a short process-group timeout, so a stuck collective ends the test with an error."""

import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


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
    sys.path[:0] = [here, root, os.path.join(root, "cuda-kernels-optimized-for-rtx5090_b200")]
    import torch.distributed as dist

    from ckb200 import rmsnorm, rope, sharded, workloads
    from oracle import rmsnorm as orms
    from oracle import rope as orope
    from oracle import topk as otk
    from oracle.numerics import to_f32, ulp_distance

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        x = workloads.topk_512x151936(scale=4)["x"]
        lo, hi = sharded.col_range(x.shape[1], rank, world)
        values, indices = sharded.topk_vocab_sharded(x[:, lo:hi].contiguous().to(dev), lo, 50)
        op = sharded.VocabShardedTopK(x.shape[0], 50, device=dev)
        v2, i2 = op(x[:, lo:hi].contiguous().to(dev), lo)
        wv, wi = otk.topk(x, 50)
        ok_topk = (torch.equal(indices.cpu(), wi) and torch.equal(values.cpu(), wv) and
                   torch.equal(i2.cpu(), wi) and torch.equal(v2.cpu(), wv))
        peer = sharded.PeerVocabShardedTopK(x.shape[0], 50, device=dev)
        for call in range(5):
            xs = x if call % 2 == 0 else x.to(torch.bfloat16)
            pv, pi = peer(xs[:, lo:hi].contiguous().to(dev), lo)
            bv, bi = otk.topk(xs, 50)
            ok_topk = ok_topk and torch.equal(pi.cpu(), bi) and torch.equal(pv.cpu(), bv)
        step = peer.graphed(x[:, lo:hi].contiguous().to(dev), lo)
        for call in range(6):
            gv, gi = step()
            torch.cuda.synchronize()
            ok_topk = ok_topk and torch.equal(gi.cpu(), wi) and torch.equal(gv.cpu(), wv)
        peer.check()  # raises if any peer wait ran out
        peer.close()
        inp = workloads.rmsnorm_16384x4096(scale=64)
        r0, r1 = sharded.row_range(inp["x"].shape[0], rank, world)
        mine = rmsnorm.rmsnorm(inp["x"][r0:r1].contiguous().to(dev), inp["weight"].to(dev))
        parts = [torch.empty((sharded.row_range(inp["x"].shape[0], r, world)[1] -
                              sharded.row_range(inp["x"].shape[0], r, world)[0], 4096),
                             dtype=torch.bfloat16, device=dev) for r in range(world)]
        dist.all_gather(parts, mine)
        full = torch.cat(parts).cpu()
        ok_rows = int(ulp_distance(to_f32(full), to_f32(orms.rmsnorm(inp["x"], inp["weight"])),
                                   torch.bfloat16).max()) <= 1
        # token-sharded RoPE: uneven shards (3 x 999 tokens do not divide by most world sizes)
        rp = workloads.rope_8x4096(integer=True, batch=3, seq=999)
        tq = sharded.token_shard(rp["q"], rank, world).to(dev)
        tk = sharded.token_shard(rp["k"], rank, world).to(dev)
        ids = sharded.token_shard(rp["position_ids"], rank, world).to(dev)
        rope.rope(tq, tk, ids, rp["cos"].to(dev), rp["sin"].to(dev), inplace=True)
        sizes = [sharded.token_range(3 * 999, r, world) for r in range(world)]
        gq = _gather_tokens(tq, sizes).cpu().view(torch.int16)
        gk = _gather_tokens(tk, sizes).cpu().view(torch.int16)
        wq, wk = orope.rope(rp["q"], rp["k"], rp["cos"], rp["sin"], rp["position_ids"])
        ok_rows = ok_rows and torch.equal(gq, wq.view(1, -1, 32, 128).view(torch.int16)) and \
            torch.equal(gk, wk.view(1, -1, 8, 128).view(torch.int16))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, bool(ok_topk), bool(ok_rows)))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e), False))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_vocab_sharded_topk_and_row_shards_over_nccl():
    world = min(torch.cuda.device_count(), 8)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        results = [q.get(timeout=300) for _ in range(world)]
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank, ok_topk, ok_rows in results:
        assert ok_topk is True, f"rank {rank}: {ok_topk}"
        assert ok_rows is True, f"rank {rank}"
