"""RMSNorm parity on the GPU: the CUDA kernels against the CPU oracle (and the reference's own kernel).

Tolerance: within 1 ulp of the output dtype (bf16 / fp16) of the fp32-accumulated oracle. The unweighted form rounds
the inverse RMS to the dtype as the reference does (rmsnorm/kernel.cu:46), so a last-bit difference in the fp32 sum
can move a result by one ulp; every other bit agrees.
"""

import ctypes

import numpy as np
import pytest
import torch

from ckb200 import rmsnorm, workloads
from helpers import assert_ulp, guarded_empty, misaligned_copy, ref_lib
from oracle import rmsnorm as orc

pytestmark = pytest.mark.gpu


def _x(rows, cols, dtype, seed=0, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(rows, cols, generator=g) * scale).to(dtype)


def test_config_weighted_bf16():
    """x bf16 [16384, 4096] ~ N(0,1), weight ~ N(1, 0.1^2), eps 1e-6."""
    inp = workloads.rmsnorm_16384x4096()
    want = orc.rmsnorm(inp["x"], inp["weight"])
    got = rmsnorm.run({k: v.cuda() for k, v in inp.items()})["y"]
    d = assert_ulp(got, want, torch.bfloat16, 1, "rmsnorm weighted config")
    assert (d == 0).mean() > 0.999


def test_config_unweighted_bf16():
    inp = workloads.rmsnorm_16384x4096()
    want = orc.rmsnorm(inp["x"])
    got = rmsnorm.run({"x": inp["x"].cuda()})["y"]
    d = assert_ulp(got, want, torch.bfloat16, 1, "rmsnorm config")
    assert (d == 0).mean() > 0.999


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("cols", [8, 64, 256, 1000, 1024, 4096, 8192, 32768, 40000])
@pytest.mark.parametrize("rows", [1, 7, 33])
def test_shapes(dtype, cols, rows):
    x = _x(rows, cols, dtype, seed=cols + rows)
    want = orc.rmsnorm(x)
    y, check = guarded_empty((rows, cols), dtype)
    rmsnorm.rmsnorm(x.cuda(), out=y)
    torch.cuda.synchronize()
    check()
    assert_ulp(y, want, dtype, 1, f"rmsnorm {rows}x{cols} {dtype}")


@pytest.mark.parametrize("wdtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("cols", [128, 1000, 4096, 40000])
def test_weighted(dtype, wdtype, cols):
    x = _x(9, cols, dtype, seed=3)
    w = (1 + 0.1 * torch.randn(cols, generator=torch.Generator().manual_seed(4))).to(wdtype)
    want = orc.rmsnorm(x, w)
    got = rmsnorm.rmsnorm(x.cuda(), w.cuda())
    assert_ulp(got, want, dtype, 1, f"weighted {cols} {dtype} w {wdtype}")


def test_misaligned_pointer_takes_scalar_path():
    x = _x(5, 4096, torch.bfloat16, seed=5)
    xd = misaligned_copy(x.cuda())
    assert xd.data_ptr() % 16 != 0
    got = rmsnorm.rmsnorm(xd)
    assert_ulp(got, orc.rmsnorm(x), torch.bfloat16, 1, "misaligned")


@pytest.mark.parametrize("cols", [512, 4096, 1001])
def test_nan_and_overflow_rows(cols):
    """A NaN makes its row NaN; a sum of squares that overflows fp32 gives inv = 0 (rmsnorm/kernel.cu:4-6)."""
    x = _x(4, cols, torch.bfloat16, seed=6)
    x[1, 7] = float("nan")
    x[2, :] = 1e30  # squares overflow: y = x * 0 = 0
    x[3, 3] = float("inf")  # inf * 0 = NaN there, 0 elsewhere
    got = rmsnorm.rmsnorm(x.cuda()).cpu().float()
    want = orc.rmsnorm(x).float()
    assert torch.isnan(got[1]).all() and torch.isnan(want[1]).all()
    assert torch.equal(torch.isnan(got), torch.isnan(want))
    fin = ~torch.isnan(want)
    assert torch.equal(got[fin], want[fin])


def test_zero_rows_is_noop():
    x = torch.empty(0, 4096, dtype=torch.bfloat16, device="cuda")
    assert rmsnorm.rmsnorm(x).shape == (0, 4096)


def test_matches_reference_kernel():
    """The reference's own rmsnorm kernel (rebuilt for sm_100a) on the same input: within 1 ulp, nearly all equal."""
    lib = ref_lib("rmsnorm")
    if lib is None:
        pytest.skip("oracle/_ref not built")
    x = _x(2048, 4096, torch.bfloat16, seed=7).cuda()
    ref = torch.empty_like(x)
    lib.launch.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_int,
                           ctypes.c_float, ctypes.c_int, ctypes.c_void_p]
    err = lib.launch(x.data_ptr(), ref.data_ptr(), 2048, 4096, 1, 1e-6, 256, torch.cuda.current_stream().cuda_stream)
    assert err == 0
    got = rmsnorm.rmsnorm(x)
    d = assert_ulp(got.cpu(), ref.cpu(), torch.bfloat16, 1, "vs reference kernel")
    assert (d == 0).mean() > 0.999


def test_bad_arguments_raise():
    with pytest.raises(ValueError):
        rmsnorm.run({"x": torch.zeros(4, 8, dtype=torch.float32, device="cuda")})
    with pytest.raises(ValueError):
        rmsnorm.run({"x": torch.zeros(2, 4, 8, dtype=torch.bfloat16, device="cuda")})
