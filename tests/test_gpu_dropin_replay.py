"""The reference's own wrappers, replayed on the GPU: every C-ABI call that the unchanged rmsnorm/, rope/ and
topk/candidate.py make (recorded where the reference checkout is present, tests/golden/make_dropin_calls.py ->
tests/golden/dropin_calls.json: symbol, the ctypes argument and result types the wrapper declares, and each argument)
is made again here against this repository's libraries, with the same inputs, buffers of the recorded shapes and the
recorded knob values (threads, depth, min_chunk, eps, dtype codes, the chunk its plan() call returned). The outputs
must equal this library's own Python entry points bit for bit and the oracle within the suite's tolerances: top-k
and cache-mode RoPE bit-exact, RMSNorm within 1 bf16 ulp.
"""

import ctypes
import json
import os

import pytest
import torch

from ckb200 import build, rmsnorm, rope, topk
from dropin_inputs import CASES, OUTPUTS, make_inputs
from helpers import assert_ulp, bits_equal
from oracle import rmsnorm as ormsnorm
from oracle import rope as orope
from oracle import topk as otopk

pytestmark = pytest.mark.gpu
FIXTURE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "dropin_calls.json")
DTYPES = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32, "int32": torch.int32,
          "int64": torch.int64}


def _replay(op, case):
    rec = json.load(open(FIXTURE))[op][case]
    inputs = {k: v.cuda() for k, v in make_inputs(op, case).items()}
    outputs = {k: torch.empty(s["shape"], dtype=DTYPES[s["dtype"]], device="cuda") for k, s in rec["outputs"].items()}
    allocs = {k: (torch.zeros if s["zero"] else torch.empty)(s["shape"], dtype=DTYPES[s["dtype"]], device="cuda")
              for k, s in rec["allocs"].items()}
    tensors = {**{f"in:{k}": v for k, v in inputs.items()}, **{f"out:{k}": v for k, v in outputs.items()}, **allocs}
    lib = ctypes.CDLL(build.lib_path(op))
    for call in rec["calls"]:
        fn = getattr(lib, call["fn"])
        fn.argtypes = [getattr(ctypes, t) for t in call["argtypes"]]
        fn.restype = getattr(ctypes, call["restype"]) if call["restype"] else None
        args = []
        for a in call["args"]:
            if "ptr" in a:
                t = tensors[a["ptr"]]
                args.append(t.data_ptr())
            elif "stream" in a:
                args.append(torch.cuda.current_stream().cuda_stream)
            else:
                args.append(a["value"])
        rc = fn(*args)
        if call["fn"] == "launch":
            assert rc == 0, f"{op}: launch returned {rc}"
    torch.cuda.synchronize()
    assert sorted(outputs) == sorted(OUTPUTS[op])
    return make_inputs(op, case), inputs, outputs


@pytest.mark.parametrize("case", CASES["rmsnorm"])
def test_rmsnorm_wrapper_calls(case):
    host, dev, out = _replay("rmsnorm", case)
    ours = rmsnorm.run(dev)["y"]
    assert bits_equal(out["y"], ours)
    assert_ulp(out["y"], ormsnorm.rmsnorm(host["x"]), host["x"].dtype, 1, f"replayed rmsnorm {case}")


@pytest.mark.parametrize("case", CASES["rope"])
def test_rope_wrapper_calls(case):
    host, dev, out = _replay("rope", case)
    ours = rope.run(dev)
    wq, wk = orope.rope(host["q"], host["k"], host["cos"], host["sin"], host["position_ids"])
    assert bits_equal(out["q_out"], ours["q_out"]) and bits_equal(out["k_out"], ours["k_out"])
    assert bits_equal(out["q_out"], wq) and bits_equal(out["k_out"], wk)


@pytest.mark.parametrize("case", CASES["topk"])
def test_topk_wrapper_calls(case):
    host, dev, out = _replay("topk", case)
    ours = topk.run(dev)
    assert torch.equal(out["indices"], ours["indices"]) and bits_equal(out["values"], ours["values"])
    wv, wi = otopk.topk(host["x"], 50)
    assert torch.equal(out["indices"].cpu(), wi) and bits_equal(out["values"], wv)
