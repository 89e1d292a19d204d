"""The drop-in claim, checked with the reference's own, unchanged Python wrappers (rmsnorm, rope and top-k
`candidate.py`): pointed at this repository's libraries through CKOPT_BUILD_DIR (the variable they read), they bind
their `launch` / `plan` with their own ctypes signatures and drive these libraries through their own argument
packing and error convention (rmsnorm/candidate.py:25-28,40-52, rope/candidate.py:27-29,44-57,
topk/candidate.py:30-36,66-81).

Runs on the CPU where the reference checkout is present (it does not travel to the GPU box), so it calls only what
returns before any CUDA work: empty batches (a successful no-op in the reference's ABI) and arguments the ABI
rejects (-1, which the wrappers turn into RuntimeError("kernel launch failed: CUDA error -1")). The GPU tests drive
the same entry points with the same ctypes signatures (ckb200/_native.py) and check the results.
"""

import importlib.util
import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import __graft_entry__  # noqa: E402
from ckb200 import build  # noqa: E402

REF = __graft_entry__.reference_root()
pytestmark = pytest.mark.skipif(REF is None, reason="no reference checkout on this machine")


class _Stream:
    cuda_stream = None  # the default stream; never reached by these calls


@pytest.fixture(autouse=True)
def no_device_stream(monkeypatch):
    """The wrappers ask torch for the current CUDA stream; on a machine without a GPU hand them the default one."""
    monkeypatch.setattr(torch.cuda, "current_stream", lambda *a, **k: _Stream())


def _candidate(op, monkeypatch):
    build.build(ops=(op,))
    monkeypatch.setenv("CKOPT_BUILD_DIR", os.path.dirname(build.lib_path(op)))
    spec = importlib.util.spec_from_file_location(f"reference_{op}_candidate", os.path.join(REF, op, "candidate.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    assert os.path.samefile(mod._lib._name, build.lib_path(op)), "the wrapper did not load this repository's library"
    return mod


def test_rmsnorm_wrapper_binds_and_runs_an_empty_batch(monkeypatch):
    mod = _candidate("rmsnorm", monkeypatch)
    for dtype in (torch.bfloat16, torch.float16):
        out = mod.run({"x": torch.empty(0, 4096, dtype=dtype)})
        assert out["y"].shape == (0, 4096) and out["y"].dtype == dtype
    with pytest.raises(ValueError, match="rmsnorm candidate"):
        mod.run({"x": torch.empty(4, 4096, dtype=torch.float32)})  # the wrapper's own check


def test_rope_wrapper_binds_and_runs_an_empty_batch(monkeypatch):
    mod = _candidate("rope", monkeypatch)
    q = torch.empty(0, 4096, 32, 128, dtype=torch.bfloat16)
    k = torch.empty(0, 4096, 8, 128, dtype=torch.bfloat16)
    cache = torch.empty(4096, 128, dtype=torch.float32)
    out = mod.run({"q": q, "k": k, "cos": cache, "sin": cache, "position_ids": torch.empty(0, 4096,
                                                                                           dtype=torch.int64)})
    assert out["q_out"].shape == q.shape and out["k_out"].shape == k.shape


def test_topk_wrapper_plans_runs_an_empty_batch_and_reports_rejections(monkeypatch):
    mod = _candidate("topk", monkeypatch)
    out = mod.run({"x": torch.empty(0, 151936)})
    assert out["values"].shape == (0, 50) and out["indices"].dtype == torch.int64
    # More rows than the ABI serves: this library's launch returns -1 before any CUDA work, and the reference's
    # wrapper reports it with its own message.
    with pytest.raises(RuntimeError, match=r"kernel launch failed: CUDA error -1"):
        mod.run({"x": torch.empty(70000, 64)})
