"""Host-side logic of the Python entry points, on the CPU: argument validation mirrors the reference wrappers'
(ValueError with the op's name), CPU tensors are refused (no CPU path), sharding arithmetic, workload shapes."""

import pytest
import torch

from ckb200 import rmsnorm, rope, sharded, softmax, topk, workloads


def test_cpu_tensors_are_refused_not_computed():
    x = torch.zeros(4, 128)
    with pytest.raises(ValueError, match="CUDA"):
        softmax.run({"x": x})
    with pytest.raises(ValueError, match="CUDA"):
        rmsnorm.run({"x": x.to(torch.bfloat16)})
    with pytest.raises(ValueError, match="CUDA"):
        topk.run({"x": x})
    q = torch.zeros(1, 2, 4, 8, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        rope.rope(q, q, torch.zeros(1, 2, dtype=torch.int64), theta=1e4)


def test_validation_messages_follow_the_reference():
    with pytest.raises(ValueError, match="^rmsnorm candidate: dtype"):
        rmsnorm.run({"x": torch.zeros(4, 8)})
    with pytest.raises(ValueError, match="^rmsnorm candidate: shape"):
        rmsnorm.run({"x": torch.zeros(4, dtype=torch.bfloat16)})
    with pytest.raises(ValueError, match="^topk candidate takes a 2-D fp32 or bf16 tensor with at least 50"):
        topk.run({"x": torch.zeros(4, 49)})
    q = torch.zeros(1, 2, 4, 8, dtype=torch.bfloat16)
    ids = torch.zeros(1, 2, dtype=torch.int64)
    cos = torch.zeros(4, 8)
    with pytest.raises(ValueError, match="^rope candidate: dtypes"):
        rope.run({"q": q.float(), "k": q, "cos": cos, "sin": cos, "position_ids": ids})
    with pytest.raises(ValueError, match="^rope candidate: shapes"):
        rope.run({"q": q, "k": q, "cos": torch.zeros(4, 6), "sin": torch.zeros(4, 6), "position_ids": ids})
    with pytest.raises(ValueError, match="^softmax: dtype"):
        softmax.run({"x": torch.zeros(4, 8, dtype=torch.float16)})


@pytest.mark.parametrize("n,world", [(16384, 1), (16384, 8), (10, 3), (3, 8), (0, 2), (151936, 8)])
def test_split_range_partitions(n, world):
    parts = [sharded.split_range(n, r, world) for r in range(world)]
    assert parts[0][0] == 0 and parts[-1][1] == n
    for (a, b), (c, d) in zip(parts, parts[1:]):
        assert b == c
    sizes = [b - a for a, b in parts]
    assert max(sizes) - min(sizes) <= 1


def test_split_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        sharded.split_range(10, 2, 2)


def test_workload_shapes_and_bytes():
    x = workloads.softmax_4096x8192(scale=64)["x"]
    assert x.shape == (64, 8192) and x.dtype == torch.float32
    r = workloads.rmsnorm_16384x4096(scale=256)
    assert r["x"].shape == (64, 4096) and r["weight"].shape == (4096,)
    p = workloads.rope_8x4096(scale=8, seq=16)
    assert p["q"].shape == (1, 16, 32, 128) and p["k"].shape == (1, 16, 8, 128) and p["cos"].shape == (4096, 128)
    s = workloads.softmax_256x262144(scale=128)["x"]
    assert s.shape == (2, 262144) and (s.max(dim=1).values > 15).all()
    assert workloads.ALGORITHMIC_BYTES["rmsnorm_16384x4096"] == 268443648
    assert workloads.ALGORITHMIC_BYTES["softmax_4096x8192"] == 268435456
    assert workloads.ALGORITHMIC_BYTES["topk_512x151936"] == 311164928 + 307200


def test_rope_inv_freq_is_the_cache_builders():
    from oracle.rope import cos_sin_cache

    f = rope.inv_freq(10000.0, 128, "cpu")
    cos, sin = cos_sin_cache(10000.0, 128, 4096)
    ang = (torch.arange(4096).float()[:, None] * f[None, :])
    assert torch.equal(torch.cat([ang, ang], -1).cos(), cos)


def test_row_pipeline_rejects_empty_shapes_before_touching_the_gpu():
    from ckb200 import hostpipe

    with pytest.raises(ValueError, match="shape"):
        hostpipe.RowPipeline(lambda a, b: None, 0, 8, torch.float32)
    with pytest.raises(ValueError, match="chunks"):
        hostpipe.RowPipeline(lambda a, b: None, 4, 8, torch.float32, chunks=0)


def test_exchange_layout_and_epochs():
    half, lists_off, flags_off = sharded.exchange_layout(8, 512, 50)
    assert lists_off == 0 and flags_off == 8 * 512 * 50 * 8
    assert half % 256 == 0 and half >= flags_off + 8 * 512 * 4
    assert sharded.next_epoch(0) == 1 and sharded.next_epoch(1) == 2
    e = 0xFFFFFFFF
    assert sharded.next_epoch(e) == 2 and (sharded.next_epoch(e) & 1) != (e & 1)  # parity keeps alternating


@pytest.mark.parametrize("start", [0, 5, 0xFFFFFFFA, 0xFFFFFFFD])
def test_graph_epoch_rotation_alternates_parity_and_never_repeats_two_apart(start):
    warm, captured = sharded.graph_epochs(start)
    seq = [start] + warm + captured * 4
    assert 0 not in seq[1:]
    assert all((a & 1) != (b & 1) for a, b in zip(seq, seq[1:]))
    assert all(a != c for a, c in zip(seq[1:], seq[3:]))
