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


def test_rejects_plans_beyond_the_scratch():
    """600 rows x 1M columns with k = 512: more rows than one wave of CTAs holds, so the plan splits each row into
    several segments, and 600 * segments * 512 composites of workspace is more than the scratch holds (launch() with a
    caller's workspace serves it). Real buffers are passed so that even a planner change could not make the call touch
    memory it does not own."""
    fn = _noalloc()
    rows, cols, k = 600, 1 << 20, 512
    x = torch.empty(rows, cols, device="cuda")
    v = torch.empty(rows, k, device="cuda")
    i = torch.empty(rows, k, dtype=torch.int64, device="cuda")
    plan = ctypes.CDLL(build.lib_path("topk")).plan
    plan.restype = ctypes.c_longlong
    plan.argtypes = [ctypes.c_longlong, ctypes.c_longlong, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    nseg = -(-cols // plan(rows, cols, 0, 256, 4, 2048))
    assert nseg > 1 and rows * nseg * k > 491520
    assert fn(x.data_ptr(), v.data_ptr(), i.data_ptr(), rows, cols, k, 0, torch.cuda.current_stream().cuda_stream) == -2
    torch.cuda.synchronize()
