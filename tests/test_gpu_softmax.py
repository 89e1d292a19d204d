"""Softmax parity on the GPU against the fp64 oracle (the reference's torch.softmax, softmax/baseline.py:5-6,13).

Tolerance: fp32 outputs within 1e-6 relative of fp64 elementwise, and outputs below FLT_MIN (where fp32's spacing
is 2^-149, so no 1e-6 relative bound is representable) within two subnormal steps, 2^-148, of the fp64 value: they
are kept as subnormals, never flushed to zero. bf16 outputs within 1 bf16 ulp of the fp64 result rounded to bf16.
NaN exactly where the oracle has NaN (a row with +inf or NaN is all NaN, as in torch).
"""

import ctypes

import numpy as np
import pytest
import torch

from ckb200 import softmax, workloads
from helpers import assert_rel, assert_ulp, guarded_empty, misaligned_copy, ref_lib
from oracle import softmax as orc

pytestmark = pytest.mark.gpu
REL = 1e-6


def _check(x, y, what):
    want = orc.softmax_f64(x)
    if x.dtype == torch.float32:
        assert_rel(y, want, REL, what)
    else:
        assert_ulp(y.cpu(), want.to(torch.bfloat16), torch.bfloat16, 1, what)


def test_config1_4096x8192():
    x = workloads.softmax_4096x8192()["x"]
    _check(x, softmax.run({"x": x.cuda()})["y"], "4096x8192")


def test_config4_long_rows_cluster_path():
    x = workloads.softmax_256x262144()["x"]
    _check(x, softmax.run({"x": x.cuda()})["y"], "256x262144")


def test_config4_short_rows():
    x = workloads.softmax_262144x128()["x"]
    _check(x, softmax.run({"x": x.cuda()})["y"], "262144x128")


# Column counts that reach every path: group (G = 4, 8, 16, 32), block, cluster (several cluster sizes), and the
# stream fallback (cols not a multiple of the vector).
COLS = [1, 4, 12, 16, 32, 100, 128, 256, 512, 1024, 2048, 8192, 16384, 20000, 32768, 65536, 100000, 131072, 262144,
        524288, 1048576, 4194304,
        13, 1001, 40001]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("cols", COLS)
def test_shapes(dtype, cols):
    rows = 3 if cols >= 65536 else 37
    g = torch.Generator().manual_seed(cols)
    x = (torch.randn(rows, cols, generator=g) * 3).to(dtype)
    y, check = guarded_empty((rows, cols), dtype)
    softmax.softmax(x.cuda(), out=y)
    torch.cuda.synchronize()
    check()
    _check(x, y, f"{rows}x{cols} {dtype}")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_rows_beyond_the_grid_limit(dtype):
    """More rows than the cluster grid's y limit: resident clusters loop over the rows with a ring of slice buffers
    (each slice partly staged, partly in registers). Rows spread over the batch are checked against the oracle."""
    rows, cols = 65536 + 77, 16400 if dtype == torch.float32 else 32800
    g = torch.Generator(device="cuda").manual_seed(11)
    x = (torch.randn(rows, cols, generator=g, device="cuda") * 3).to(dtype)
    y = softmax.softmax(x)
    torch.cuda.synchronize()
    pick = torch.tensor([0, 1, 2, 4095, 32768, 65534, 65535, 65536, rows - 2, rows - 1])
    _check(x[pick].cpu(), y[pick], f"{rows}x{cols} {dtype} (ring)")
    del x, y


@pytest.mark.parametrize("cols", [128, 8192, 262144])
def test_misaligned(cols):
    x = torch.randn(3, cols, generator=torch.Generator().manual_seed(1))
    xd = misaligned_copy(x.cuda())
    _check(x, softmax.softmax(xd), f"misaligned {cols}")


@pytest.mark.parametrize("cols", [128, 8192, 262144, 4194304])
def test_special_values(cols):
    x = torch.randn(6, cols, generator=torch.Generator().manual_seed(2))
    x[0, 3] = float("-inf")
    x[1, :] = float("-inf")
    x[2, 5] = float("inf")
    x[3, 9] = float("nan")
    x[4, :] = 0.0
    x[5, : cols // 2] = float("-inf")  # whole cluster slices of -inf beside finite ones
    _check(x, softmax.softmax(x.cuda()), f"special {cols}")


def test_three_dims():
    x = torch.randn(4, 5, 96, generator=torch.Generator().manual_seed(3))
    _check(x, softmax.run({"x": x.cuda()})["y"], "3-D")


def test_no_bulk_wait_timed_out():
    lib = ctypes.CDLL(softmax._native._build.lib_path("softmax"))
    assert lib.ckb_softmax_status(1) == 0


def test_matches_reference_kernel():
    lib = ref_lib("softmax")
    if lib is None:
        pytest.skip("oracle/_ref not built")
    lib.launch.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_longlong, ctypes.c_int,
                           ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    for rows, cols in ((64, 8192), (8, 262144), (1024, 128)):
        x = (torch.randn(rows, cols, generator=torch.Generator().manual_seed(rows)) * 2).cuda()
        ref = torch.empty_like(x)
        assert lib.launch(x.data_ptr(), ref.data_ptr(), rows, cols, 0, 256, 1024,
                          torch.cuda.current_stream().cuda_stream) == 0
        got = softmax.softmax(x)
        want = orc.softmax_f64(x.cpu())
        assert_rel(got, want, REL, "ours")
        # the reference kernel against the same oracle, for the record (its division-based path is as accurate)
        assert_rel(ref, want, 2 * REL, "reference kernel")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("cols", [128, 8192, 262144, 4194304, 1001])
def test_wide_dynamic_range(cols, dtype):
    """Rows spanning 0 .. -120 below their max (every path: group, block, cluster, streaming cluster, stream): the
    true outputs run from near 1 down through the subnormal range to below 2^-149. Outputs of at least FLT_MIN keep
    1e-6 relative, smaller ones lie within two subnormal steps (bf16: 1 ulp), so none of the subnormals is lost."""
    g = torch.Generator().manual_seed(cols)
    x = (-torch.rand(3, cols, generator=g) * 120.0).to(dtype)
    x[:, 0] = 0.0
    y = softmax.softmax(x.cuda())
    _check(x, y, f"wide range {cols} {dtype}")
    want = orc.softmax_f64(x).numpy()
    tiny = np.finfo(np.float32).tiny
    smallest = 2.0 ** -149 if dtype == torch.float32 else 2.0 ** -133  # the dtype's smallest subnormal
    sub = (want < tiny) & (want >= smallest)
    assert sub.sum() > 0 and (want >= tiny).sum() > 0
    assert (y.cpu().double().numpy()[sub] > 0).all(), "a subnormal output was flushed to zero"


@pytest.mark.parametrize("cols", [8192, 262144])
def test_slice_far_below_the_row_max(cols):
    """A row whose max sits in one place and whose other values lie 60..100 below it: in the cluster path whole
    slices have maxima far below the row's, so their scale factor exp(m_c - M) / S is below FLT_MIN and is applied
    in two factors; their normal outputs keep 1e-6 relative and the subnormal ones stay within 2^-148."""
    g = torch.Generator().manual_seed(cols + 1)
    x = -60.0 - torch.rand(4, cols, generator=g) * 40.0
    x[:, cols // 3] = 0.0
    _check(x, softmax.softmax(x.cuda()), f"far slices {cols}")
