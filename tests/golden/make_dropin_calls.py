"""Records the C-ABI calls the reference's own, unchanged Python wrappers make into a fixture the GPU suite replays.

    python tests/golden/make_dropin_calls.py --ref <reference checkout>   ->  tests/golden/dropin_calls.json

Runs on the CPU where the reference checkout is present. Each wrapper (rmsnorm/, rope/ and topk/candidate.py) is
loaded with CKOPT_BUILD_DIR pointing at this repository's library, exactly as a user of the reference would; its
library handle is then swapped for a recorder, and `run()` is called on the seeded inputs of
tests/dropin_inputs.py. The recorder keeps every call the wrapper makes: the symbol, the ctypes argument and result
types the wrapper declared, and each argument, with pointers named by what they point at (an input, an output, or a
buffer the wrapper allocated itself, with its shape, dtype and whether it was zeroed) and the stream marked as such.
`plan` is answered by this library's own plan (on the CPU it plans one segment per row, which is valid on any GPU).
The checkout cannot travel to the GPU box; the fixture can, and tests/test_gpu_dropin_replay.py replays it there.
"""

import argparse
import ctypes
import importlib.util
import json
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [ROOT, os.path.join(ROOT, "tests"), os.path.join(ROOT, "cuda-kernels-optimized-for-rtx5090_b200")]

from dropin_inputs import CASES, OUTPUTS, make_inputs  # noqa: E402


class _Stream:
    cuda_stream = None


class _Recorder:
    """Stands in for the wrapper's ctypes library: records calls, answers `plan` with the real library."""

    def __init__(self, real, log):
        self._real, self._log = real, log

    def __getattr__(self, name):
        fn = getattr(self._real, name)

        def call(*args):
            self._log.append({"fn": name, "argtypes": [t.__name__ for t in (fn.argtypes or [])],
                              "restype": fn.restype.__name__ if fn.restype is not None else None,
                              "args": list(args)})
            return fn(*args) if name == "plan" else 0

        return call


def _tensors(obj, prefix, out):
    if isinstance(obj, torch.Tensor):
        out.setdefault(obj.data_ptr(), (prefix, obj))
    elif isinstance(obj, dict):
        for k, v in obj.items():
            _tensors(v, f"{prefix}{k}", out)
    elif isinstance(obj, (list, tuple)):
        for i, v in enumerate(obj):
            _tensors(v, f"{prefix}{i}", out)


def record(op, case, ref, lib_dir):
    os.environ["CKOPT_BUILD_DIR"] = lib_dir
    spec = importlib.util.spec_from_file_location(f"reference_{op}_candidate", os.path.join(ref, op, "candidate.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    log = []
    mod._lib = _Recorder(mod._lib, log)
    real_stream = torch.cuda.current_stream
    torch.cuda.current_stream = lambda *a, **k: _Stream()
    try:
        inputs = make_inputs(op, case)
        outputs = mod.run(inputs)
    finally:
        torch.cuda.current_stream = real_stream
    assert sorted(outputs) == sorted(OUTPUTS[op]), f"{op}: outputs {sorted(outputs)}"
    known = {}
    _tensors(inputs, "in:", known)
    _tensors(outputs, "out:", known)
    # Buffers the wrapper keeps at module level (the top-k workspace and row counters).
    allocs = {}
    for name in dir(mod):
        val = getattr(mod, name)
        found = {}
        _tensors(val, "", found)
        for ptr, (_, t) in found.items():
            if ptr not in known:
                label = f"alloc:{len(allocs)}"
                allocs[label] = {"shape": list(t.shape), "dtype": str(t.dtype).replace("torch.", ""),
                                 "zero": bool((t == 0).all())}
                known[ptr] = (label, t)
    calls = []
    for c in log:
        args = []
        for t, v in zip(c["argtypes"], c["args"]):
            if t == "c_void_p":
                if v is None:
                    args.append({"stream": True})
                else:
                    assert v in known, f"{op}: pointer argument not traced to a tensor"
                    args.append({"ptr": known[v][0]})
            else:
                args.append({"value": v})
        calls.append({"fn": c["fn"], "argtypes": c["argtypes"], "restype": c["restype"], "args": args})
    return {"outputs": {k: {"shape": list(v.shape), "dtype": str(v.dtype).replace("torch.", "")}
                        for k, v in outputs.items()},
            "allocs": allocs, "calls": calls}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("CKB_REFERENCE"), help="the reference checkout")
    ap.add_argument("--out", default=os.path.join(HERE, "dropin_calls.json"))
    a = ap.parse_args()
    if not a.ref:
        ap.error("--ref (or CKB_REFERENCE) is required")
    from ckb200 import build
    fixture = {}
    for op in ("rmsnorm", "rope", "topk"):
        build.build(ops=(op,))
        fixture[op] = {case: record(op, case, a.ref, os.path.dirname(build.lib_path(op))) for case in CASES[op]}
    with open(a.out, "w") as f:
        json.dump(fixture, f, indent=1)
        f.write("\n")
    print(f"wrote {a.out}")


if __name__ == "__main__":
    main()
