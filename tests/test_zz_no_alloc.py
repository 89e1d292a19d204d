"""ckb_topk_launch_noalloc: top-k for callers that cannot allocate device memory.

Such callers (code inside a host framework that hands out a fixed device-memory budget through its own allocator,
or a latency-critical path that cannot take cudaMalloc's device synchronisation) cannot provide the workspace and
counters that `launch` needs; this entry point takes only the input and the outputs and uses a scratch array
compiled into the library. It must give exactly what `launch` gives (top-k parity is bit-exact), call after call,
since the scratch keeps the previous call's contents. This file sorts last so a run stopping at the first failure
has already run every other test; it also passes alone in a fresh process.
"""

import ctypes

import pytest
import torch

from ckb200 import build, topk, workloads
from helpers import bits_equal

pytestmark = pytest.mark.gpu


def _noalloc():
    lib = ctypes.CDLL(build.lib_path("topk"))
    fn = lib.ckb_topk_launch_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_longlong,
                   ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    return fn


@pytest.mark.parametrize("dtype,scale", [(torch.float32, 1), (torch.bfloat16, 4)])
def test_matches_launch_on_two_calls_in_a_row(dtype, scale):
    fn = _noalloc()
    x = workloads.topk_512x151936(scale=scale)["x"].to(dtype).cuda()
    rows, cols = x.shape
    want_v, want_i = topk.topk(x, 50)  # the existing entry point, with its own workspace and counters
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        v = torch.empty(rows, 50, dtype=dtype, device="cuda")
        i = torch.empty(rows, 50, dtype=torch.int64, device="cuda")
        assert fn(x.data_ptr(), v.data_ptr(), i.data_ptr(), rows, cols, 50, 0 if dtype == torch.float32 else 1,
                  stream) == 0
        torch.cuda.synchronize()
        assert torch.equal(i, want_i), f"call {call}: indices differ"
        assert bits_equal(v, want_v), f"call {call}: values differ"


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_split_rows_merge_through_the_scratch_call_after_call(dtype):
    """A small batch of long rows is split into several segments per row, so the call merges through the scratch
    workspace and its per-row counters (which must be left reusable): two calls in a row equal launch()."""
    fn = _noalloc()
    g = torch.Generator().manual_seed(5)
    x = (torch.randn(2, 1 << 20, generator=g) * 3).to(dtype).cuda()
    plan = ctypes.CDLL(build.lib_path("topk")).plan
    plan.restype = ctypes.c_longlong
    plan.argtypes = [ctypes.c_longlong, ctypes.c_longlong, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    dt = 0 if dtype == torch.float32 else 1
    assert -(-x.shape[1] // plan(2, x.shape[1], dt, 256, 4, 2048)) > 1
    want_v, want_i = topk.topk(x, 50)
    for call in range(2):
        v = torch.empty(2, 50, dtype=dtype, device="cuda")
        i = torch.empty(2, 50, dtype=torch.int64, device="cuda")
        assert fn(x.data_ptr(), v.data_ptr(), i.data_ptr(), 2, x.shape[1], 50, dt,
                  torch.cuda.current_stream().cuda_stream) == 0
        torch.cuda.synchronize()
        assert torch.equal(i, want_i), f"call {call}: indices differ"
        assert bits_equal(v, want_v), f"call {call}: values differ"


def test_large_batch_keeps_rows_whole_within_the_scratch():
    """4096 rows (a batch of many short rows, one CTA each, no workspace): equals launch()."""
    fn = _noalloc()
    g = torch.Generator().manual_seed(11)
    x = (torch.randn(4096, 8192, generator=g) * 3).cuda()
    want_v, want_i = topk.topk(x, 50)
    v = torch.empty(4096, 50, device="cuda")
    i = torch.empty(4096, 50, dtype=torch.int64, device="cuda")
    assert fn(x.data_ptr(), v.data_ptr(), i.data_ptr(), 4096, 8192, 50, 0, torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert torch.equal(i, want_i) and bits_equal(v, want_v)
