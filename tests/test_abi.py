"""The C-ABI boundary on the CPU: every library builds, loads, and exports exactly what include/*.h declares, with
the Python bindings matching; argument checks that return before any CUDA call behave as the reference's do."""

import ctypes
import os
import re

import pytest

from ckb200 import _native, build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INCLUDE = os.path.join(ROOT, "include")
DECL = re.compile(r"^(?:int|long long)\s+(\w+)\(", re.M)


def declared(op):
    with open(os.path.join(INCLUDE, f"ckb200_{op}.h")) as f:
        return set(DECL.findall(f.read()))


@pytest.fixture(scope="module", autouse=True)
def libs():
    build.build()


@pytest.mark.parametrize("op", build.OPS)
def test_library_exports_every_declared_symbol(op):
    names = declared(op)
    assert names, f"no declarations parsed from ckb200_{op}.h"
    lib = ctypes.CDLL(build.lib_path(op))
    for name in names:
        assert hasattr(lib, name), f"{op}: {name} declared but not exported"
    assert names == set(_native.SIGNATURES[op]), f"{op}: Python bindings and header disagree"


@pytest.mark.parametrize("op", build.OPS)
def test_reference_symbols_kept(op):
    """The reference's ctypes wrappers bind `launch` (and top-k's `plan`) on $CKOPT_BUILD_DIR/libkernel.so."""
    lib = ctypes.CDLL(build.lib_path(op))
    assert hasattr(lib, "launch")
    if op == "topk":
        assert hasattr(lib, "plan")
    assert os.path.basename(build.lib_path(op)) == "libkernel.so"


def test_no_rows_is_a_successful_noop():
    assert _native.load("softmax").launch(None, None, 0, 128, 0, 256, 1024, None) == 0
    assert _native.load("softmax").launch(None, None, 4, 0, 0, 256, 1024, None) == 0
    assert _native.load("rmsnorm").launch(None, None, 0, 128, 1, 1e-6, 256, None) == 0
    assert _native.load("rope").launch(*([None] * 7), 0, 32, 8, 128, 1, 0, 40, 1, None) == 0
    assert _native.load("topk").launch(*([None] * 5), 0, 1000, 50, 0, 256, 4, 1000, None) == 0


def test_rejected_arguments_return_minus_one():
    sm, rms, rope, tk = (_native.load(op) for op in build.OPS)
    assert sm.launch(None, None, 4, 128, 7, 256, 1024, None) == -1  # dtype
    assert rms.launch(None, None, 4, 128, 0, 1e-6, 256, None) == -1  # fp32 is not served (reference: bf16/fp16)
    assert rms.launch(None, None, 4, 128, 1, 1e-6, 100, None) == -1  # threads not a multiple of 32
    assert rms.launch(None, None, 4, 0, 1, 1e-6, 256, None) == -1  # cols
    assert rms.ckb_rmsnorm_weighted_launch(None, None, None, 4, 128, 1, 0, 1e-6, None) == -1  # no weight
    assert rope.launch(*([None] * 7), 4, 32, 8, 127, 1, 0, 40, 1, None) == -1  # odd head_dim
    assert rope.launch(*([None] * 7), 4, 32, 8, 128, 1, 0, 0, 1, None) == -1  # rows < 1
    assert rope.launch(*([None] * 7), 4, 32, 8, 128, 1, 0, 40, 70000, None) == -1  # splits
    assert rope.ckb_rope_sincos_launch(*([None] * 6), 4, 32, 8, 128, 1, None) == -1  # no inv_freq
    assert tk.launch(*([None] * 5), 4, 40, 50, 0, 256, 4, 40, None) == -1  # k > cols
    assert tk.launch(*([None] * 5), 4, 1000, 513, 0, 256, 4, 1000, None) == -1  # k > 512
    assert tk.launch(*([None] * 5), 70000, 1000, 50, 0, 256, 4, 1000, None) == -1  # rows > 65535
    assert tk.launch(*([None] * 5), 4, 1000, 50, 0, 300, 4, 1000, None) == -1  # threads
    assert tk.launch(*([None] * 5), 4, 1000, 50, 0, 256, 3, 1000, None) == -1  # depth
    assert tk.launch(*([None] * 5), 4, 100000, 50, 0, 256, 4, 0, None) == -1  # chunk
    assert tk.launch(*([None] * 5), 4, 100000, 50, 0, 256, 4, 10, None) == -1  # segments * k beyond the merge
    assert tk.ckb_topk_merge_launch(None, 0, None, None, 4, 50, 0, None) == -1  # no lists
    # the no-allocation entry rejects what launch() rejects, before it looks up its scratch or touches the GPU
    assert tk.ckb_topk_launch_noalloc(None, None, None, 65536, 1000, 50, 0, None) == -1  # rows > 65535
    assert tk.ckb_topk_launch_noalloc(None, None, None, 4, 40, 50, 0, None) == -1  # k > cols
    assert tk.ckb_topk_launch_noalloc(None, None, None, 4, 1000, 50, 2, None) == -1  # dtype
    assert tk.ckb_topk_launch_noalloc(None, None, None, 0, 1000, 50, 0, None) == 0  # no rows


def test_topk_plan_host_logic():
    """plan() needs no GPU: a row splits into at most 12 segments (so any k <= 512 fits the last CTA's merge), each at
    least min_chunk columns. The headline batch (512 rows, at least two per SM) runs one CTA per row; a small batch
    splits its rows to fill the GPU."""
    tk = _native.load("topk")
    for rows, cols, dt in ((512, 151936, 0), (64, 151936, 0), (1, 128256, 0), (512, 32000, 1), (3, 50, 0)):
        chunk = tk.plan(rows, cols, dt, 256, 4, 2048)
        nseg = -(-cols // chunk)
        assert 1 <= chunk <= cols
        assert nseg <= 12
        if nseg > 1:
            assert chunk >= 2048
    assert tk.plan(512, 151936, 0, 256, 4, 2048) == 151936  # one CTA per row
    assert -(-151936 // tk.plan(64, 151936, 0, 256, 4, 2048)) > 1
    assert tk.plan(3, 50, 0, 256, 4, 2048) == 50


def test_noalloc_split_plans_stay_small():
    """Below two rows per SM a row is split into about one CTA per SM in all, so rows * segments * k stays within the
    no-allocation entry's 491,520-composite scratch for every k <= 512; larger batches keep rows whole."""
    tk = _native.load("topk")
    for rows in (1, 2, 3, 7, 64, 100, 147, 148, 200, 295):
        for cols in (1000, 4096, 151936, 1 << 20, 1 << 26):
            for dt in (0, 1):
                chunk = tk.plan(rows, cols, dt, 256, 4, 2048)
                nseg = -(-cols // chunk)
                assert nseg == 1 or rows * nseg * 512 <= 491520, (rows, cols, nseg)
    for rows in (296, 512, 1000, 65535):
        assert tk.plan(rows, 151936, 0, 256, 4, 2048) == 151936


def test_recorded_wrapper_calls_match_the_declared_signatures():
    """The fixture of the reference wrappers' calls (tests/golden/dropin_calls.json, replayed on the GPU by
    test_gpu_dropin_replay.py) binds exactly the argument and result types this library declares for each symbol."""
    import json

    from ckb200 import _native

    fixture = json.load(open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "dropin_calls.json")))
    for op, cases in fixture.items():
        for case, rec in cases.items():
            assert rec["calls"], (op, case)
            for call in rec["calls"]:
                res, args = _native.SIGNATURES[op][call["fn"]]
                assert [t.__name__ for t in args] == call["argtypes"], (op, case, call["fn"])
                assert res.__name__ == call["restype"], (op, case, call["fn"])
                assert len(call["args"]) == len(args), (op, case, call["fn"])
