"""Top-k parity on the GPU against the exact CPU oracle (composite order of topk/kernel.cu:1-3,56-60): values bit
for bit and indices equal, descending, ties by lower index."""

import ctypes

import numpy as np
import pytest
import torch

from ckb200 import topk, workloads
from helpers import bits_equal, misaligned_copy, ref_lib
from oracle import topk as orc

pytestmark = pytest.mark.gpu


def _check(x, k, values, indices, what=""):
    wv, wi = orc.topk(x.cpu(), k)
    assert torch.equal(indices.cpu(), wi), f"{what}: indices differ"
    assert bits_equal(values, wv), f"{what}: values differ"


def test_config_512x151936():
    x = workloads.topk_512x151936()["x"]
    out = topk.run({"x": x.cuda()})
    _check(x, 50, out["values"], out["indices"], "config")


def test_config_bf16():
    x = workloads.topk_512x151936(scale=4)["x"].to(torch.bfloat16)
    out = topk.run({"x": x.cuda()})
    _check(x, 50, out["values"], out["indices"], "config bf16")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("rows,cols,k", [(1, 128256, 50), (64, 151936, 50), (512, 32000, 50), (3, 50, 50),
                                         (5, 1000, 1), (2, 4096, 512), (7, 2049, 64), (1, 1000003, 50),
                                         (4, 33, 33), (300, 2048, 17), (2, 262144, 512)])
def test_shapes(dtype, rows, cols, k):
    g = torch.Generator().manual_seed(rows * 7 + cols)
    x = (torch.randn(rows, cols, generator=g) * 3).to(dtype)
    vv, ii = topk.topk(x.cuda(), k)
    _check(x, k, vv, ii, f"{rows}x{cols} k={k} {dtype}")


@pytest.mark.parametrize("cols", [151936, 5000, 1999])
def test_ties_take_lower_index(cols):
    """Few distinct values: every selection boundary is a tie (torch.topk on CPU would not break these by index)."""
    g = torch.Generator().manual_seed(cols)
    x = torch.randint(-3, 4, (6, cols), generator=g).float()
    vv, ii = topk.topk(x.cuda(), 50)
    _check(x, 50, vv, ii, "ties")


def test_all_equal_rows():
    x = torch.full((3, 100000), 1.5)
    x[1] = -0.0
    x[2, ::2] = 0.0  # +0 and -0 are different keys: +0 ranks above -0
    vv, ii = topk.topk(x.cuda(), 50)
    _check(x, 50, vv, ii, "equal")


def test_special_values():
    g = torch.Generator().manual_seed(9)
    x = torch.randn(4, 20000, generator=g)
    x[0, 100] = float("inf")
    x[0, 200] = float("-inf")
    x[1, 5] = float("nan")
    x[1, 6] = -float("nan")
    x[2, :] = float("-inf")
    x[3, 1000:1060] = float("inf")
    vv, ii = topk.topk(x.cuda(), 50)
    _check(x, 50, vv, ii, "special")


def test_misaligned_and_odd_cols_use_scalar_staging():
    x = torch.randn(9, 30001, generator=torch.Generator().manual_seed(3))
    xd = misaligned_copy(x.cuda())
    vv, ii = topk.topk(xd, 50)
    _check(x, 50, vv, ii, "misaligned")


def _launch_with_chunk(x, k, chunk):
    lib = topk._native.load("topk")
    rows, cols = x.shape
    nseg = -(-cols // chunk)
    work = torch.empty(max(1, rows * nseg * k), dtype=torch.int64, device=x.device)
    counters = torch.zeros(rows, dtype=torch.int32, device=x.device)
    v = torch.empty(rows, k, dtype=x.dtype, device=x.device)
    i = torch.empty(rows, k, dtype=torch.int64, device=x.device)
    dt = 0 if x.dtype == torch.float32 else 1
    assert lib.launch(x.data_ptr(), v.data_ptr(), i.data_ptr(), work.data_ptr(), counters.data_ptr(), rows, cols, k,
                      dt, 256, 4, chunk, torch.cuda.current_stream().cuda_stream) == 0
    return v, i, counters


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("k", [50, 512])
def test_every_segment_count(dtype, k):
    """Rows split into 1..12 segments (odd counts pass a list through a merge round unpaired) give the same answer,
    and every split leaves the row counters at zero."""
    g = torch.Generator().manual_seed(k)
    x = (torch.randn(3, 100003, generator=g) * 3).to(dtype)
    xd = x.cuda()
    for nseg in range(1, 13):
        chunk = -(-x.shape[1] // nseg)
        v, i, counters = _launch_with_chunk(xd, k, chunk)
        _check(x, k, v, i, f"{nseg} segments")
        assert int(counters.abs().sum()) == 0


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_increasing_rows_overflow_every_tile(dtype):
    """Rising values: every tile beats the running top k with all of its elements, so every tile overflows the
    candidate buffer and takes the radix-select path; falling values never get past the first tile's bound."""
    cols = 200000 if dtype == torch.float32 else 100000
    up = torch.arange(cols, dtype=torch.float32)
    if dtype == torch.bfloat16:
        up = up / 64.0  # many exact ties in bf16
    x = torch.stack([up, up.flip(0), -up]).to(dtype)
    for k in (50, 512):
        vv, ii = topk.topk(x.cuda(), k)
        _check(x, k, vv, ii, f"monotone k={k}")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("nseg", [1, 2, 3, 5])
def test_wide_batch_segments(dtype, nseg):
    """A batch with at least two rows per SM (the 256-thread shape) with rows kept whole or split into nseg segments
    that the row's last finisher merges. Odd columns make every row's alignment differ."""
    g = torch.Generator().manual_seed(nseg)
    x = (torch.randn(400, 40001, generator=g) * 3).to(dtype)
    xd = x.cuda()
    v, i, counters = _launch_with_chunk(xd, 50, -(-x.shape[1] // nseg))
    _check(x, 50, v, i, f"{nseg} segments")
    assert int(counters.abs().sum()) == 0


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("k", [50, 64, 65, 200, 256])
def test_many_rows_edge_cases(dtype, k):
    """300 rows (at least two per SM: the 256-thread shape, and for k <= 64 its warp-local variant) mixing random
    rows, few-valued rows (ties everywhere), rising and falling rows (a tile overflowing a warp's slots; a speculative
    bound above the final k-th), constant rows and rows with infinities and NaN: every one bit-exact."""
    g = torch.Generator().manual_seed(k)
    cols = 20001
    x = torch.randn(300, cols, generator=g) * 3
    up = torch.arange(cols, dtype=torch.float32)
    for r in range(0, 300, 10):
        x[r + 1] = torch.randint(-3, 4, (cols,), generator=g).float()
        x[r + 2] = up
        x[r + 3] = up.flip(0)
        x[r + 4] = 1.5
        x[r + 5, r] = float("inf")
        x[r + 5, r + 7] = float("-inf")
        x[r + 6, 100 + r] = float("nan")
    x = x.to(dtype)
    vv, ii = topk.topk(x.cuda(), k)
    _check(x, k, vv, ii, f"many rows k={k}")


@pytest.mark.parametrize("k", [1, 50, 256])
def test_long_rows_one_wave_with_ties_and_rising_rows(k):
    """The config's shape class (at least two rows per SM, rows long enough to count as long segments): random,
    few-valued, rising and falling rows side by side, fp32, every row bit-exact for k up to the 256-thread bound."""
    g = torch.Generator().manual_seed(1000 + k)
    rows, cols = 304, 98305
    x = torch.randn(rows, cols, generator=g) * 3
    up = torch.arange(cols, dtype=torch.float32)
    for r in range(0, rows, 8):
        x[r + 1] = torch.randint(0, 8, (cols,), generator=g).float()
        x[r + 2] = up
        x[r + 3] = up.flip(0)
    vv, ii = topk.topk(x.cuda(), k)
    _check(x, k, vv, ii, f"long rows k={k}")


def test_repeated_calls_reuse_workspace_and_counters():
    x = workloads.topk_512x151936(scale=8)["x"].cuda()
    first = topk.topk(x, 50)
    for _ in range(3):
        again = topk.topk(x, 50)
        assert torch.equal(first[1], again[1]) and bits_equal(first[0], again[0])
    assert int(topk._row_counters(x.device, x.shape[0])[: x.shape[0]].abs().sum()) == 0


def test_shard_and_merge_equal_full_topk():
    """The vocab-sharded variant's two kernels on one GPU: 8 column shards -> lists -> merge == top-k of the row."""
    x = workloads.topk_512x151936(scale=4)["x"]
    xd = x.cuda()
    shards = 8
    bounds = np.linspace(0, x.shape[1], shards + 1).astype(int)
    lists = torch.stack([topk.shard_lists(xd[:, a:b].contiguous(), int(a), 50) for a, b in zip(bounds, bounds[1:])])
    want_lists = torch.stack([orc.shard_lists(x[:, a:b], int(a), 50) for a, b in zip(bounds, bounds[1:])])
    assert torch.equal(lists.cpu(), want_lists)
    vv, ii = topk.merge_lists(lists, torch.float32, 50)
    _check(x, 50, vv, ii, "shard+merge")


def test_no_bulk_wait_timed_out():
    lib = ctypes.CDLL(topk._native._build.lib_path("topk"))
    assert lib.ckb_topk_status(1) == 0


def test_matches_reference_kernel():
    lib = ref_lib("topk")
    if lib is None:
        pytest.skip("oracle/_ref not built")
    lib.plan.argtypes = [ctypes.c_longlong, ctypes.c_longlong, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    lib.plan.restype = ctypes.c_longlong
    lib.launch.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_longlong, ctypes.c_longlong, ctypes.c_int, ctypes.c_int,
                                                   ctypes.c_int, ctypes.c_int, ctypes.c_longlong, ctypes.c_void_p]
    x = workloads.topk_512x151936(scale=8)["x"].cuda()
    rows, cols = x.shape
    chunk = lib.plan(rows, cols, 0, 256, 4, 2048)
    nch = -(-cols // chunk)
    work = torch.empty(max(1, rows * nch * 50), dtype=torch.int64, device="cuda")
    counters = torch.zeros(4096, dtype=torch.int32, device="cuda")
    rv = torch.empty(rows, 50, device="cuda")
    ri = torch.empty(rows, 50, dtype=torch.int64, device="cuda")
    assert lib.launch(x.data_ptr(), rv.data_ptr(), ri.data_ptr(), work.data_ptr(), counters.data_ptr(), rows, cols,
                      50, 0, 256, 4, chunk, torch.cuda.current_stream().cuda_stream) == 0
    vv, ii = topk.topk(x, 50)
    assert torch.equal(ii, ri) and bits_equal(vv, rv)


def test_bad_arguments_raise():
    with pytest.raises(ValueError):
        topk.run({"x": torch.zeros(2, 49, device="cuda")})
    with pytest.raises(ValueError):
        topk.run({"x": torch.zeros(2, 100, dtype=torch.float16, device="cuda")})
