"""RoPE parity on the GPU against the CPU oracle (the reference's rotation, rope/kernel.cu:5-8).

Cache mode uses the same cos/sin bits and the same roundings as the oracle, so it must match bit for bit on every
input (the integer-valued config is the north star's exact-match case). Sincos mode computes cos/sin on the device
with sincosf: 1 ulp of the output dtype wherever the rotation does not cancel, else 1e-6 * (|x_i| + |x_{i+h}|) for
the cos/sin difference.
"""

import ctypes

import numpy as np
import pytest
import torch

from ckb200 import rope, workloads
from helpers import bits_equal, misaligned_copy, ref_lib
from oracle import rope as orc
from oracle.numerics import to_f32, ulp_distance

pytestmark = pytest.mark.gpu


def _run_cache(inp, inplace=False, dev_inputs=None):
    d = dev_inputs or {k: (v.cuda() if torch.is_tensor(v) else v) for k, v in inp.items()}
    d = dict(d)
    d.pop("theta", None)
    d["inplace"] = inplace
    return rope.run(d)


@pytest.mark.parametrize("integer", [True, False])
def test_config_cache_exact(integer):
    """BASELINE config 3 (8 x 4096 tokens, 32 + 8 heads of 128), fp32 cache, in place."""
    inp = workloads.rope_8x4096(integer=integer)
    wq, wk = orc.rope(inp["q"], inp["k"], inp["cos"], inp["sin"], inp["position_ids"])
    out = _run_cache(inp, inplace=True)
    assert bits_equal(out["q_out"], wq) and bits_equal(out["k_out"], wk)


@pytest.mark.parametrize("cache_dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("qk_dtype", [torch.bfloat16, torch.float16])
def test_dtypes_out_of_place(cache_dtype, qk_dtype):
    inp = workloads.rope_8x4096(scale=8, cache_dtype=cache_dtype, seq=512)
    inp["q"], inp["k"] = inp["q"].to(qk_dtype), inp["k"].to(qk_dtype)
    wq, wk = orc.rope(inp["q"], inp["k"], inp["cos"], inp["sin"], inp["position_ids"])
    dq = inp["q"].cuda()
    out = _run_cache(inp, inplace=False, dev_inputs={**{k: (v.cuda() if torch.is_tensor(v) else v)
                                                        for k, v in inp.items()}, "q": dq})
    assert bits_equal(out["q_out"], wq) and bits_equal(out["k_out"], wk)
    assert bits_equal(dq, inp["q"].cuda())  # out of place leaves q alone


@pytest.mark.parametrize("head_dim,q_heads,kv_heads", [(64, 4, 1), (128, 32, 8), (256, 8, 8), (32, 3, 5),
                                                        (10, 2, 2), (48, 40, 1)])
def test_head_shapes(head_dim, q_heads, kv_heads):
    g = torch.Generator().manual_seed(head_dim)
    b, s = 2, 37
    q = torch.randn(b, s, q_heads, head_dim, generator=g).to(torch.bfloat16)
    k = torch.randn(b, s, kv_heads, head_dim, generator=g).to(torch.bfloat16)
    cos, sin = orc.cos_sin_cache(500.0, head_dim, 64)
    ids = torch.randint(0, 64, (b, s), generator=g)
    wq, wk = orc.rope(q, k, cos, sin, ids)
    qo, ko = rope.rope(q.cuda(), k.cuda(), ids.cuda(), cos.cuda(), sin.cuda())
    assert bits_equal(qo, wq) and bits_equal(ko, wk)


def test_misaligned_scalar_path_in_place():
    inp = workloads.rope_8x4096(scale=8, seq=64)
    wq, wk = orc.rope(inp["q"], inp["k"], inp["cos"], inp["sin"], inp["position_ids"])
    q = misaligned_copy(inp["q"].cuda())
    k = misaligned_copy(inp["k"].cuda())
    rope.rope(q, k, inp["position_ids"].cuda(), inp["cos"].cuda(), inp["sin"].cuda(), inplace=True)
    assert bits_equal(q, wq) and bits_equal(k, wk)


def _sincos_check(got, x, want):
    g = to_f32(got)
    w = to_f32(want)
    xf = to_f32(x)
    h = xf.shape[-1] // 2
    mag = np.abs(xf[..., :h]) + np.abs(xf[..., h:])
    mag = np.concatenate([mag, mag], axis=-1)
    d = ulp_distance(g, w, got.dtype)
    # Within 1 ulp of the dtype wherever the rotation does not cancel (|out| >= (|x_i| + |x_{i+h}|) / 64). Under
    # deep cancellation a cos/sin that differs from the cached value by an fp32 ulp moves the tiny result by many of
    # its own ulps; there the bound is absolute: 1e-6 * (|x_i| + |x_{i+h}|) (measured on the full config: 160 of
    # 167.8 M outputs beyond 1 ulp, all with |out| <= 2e-5 * (|x_i| + |x_{i+h}|)).
    cancels = np.abs(w) < mag / 64
    ok = (d <= 1) | (cancels & (np.abs(g - w) <= 1e-6 * mag + 2 ** -24))
    assert ok.all(), f"{(~ok).sum()} elements beyond tolerance"
    return (d == 0).mean()


def test_sincos_mode_config():
    inp = workloads.rope_8x4096(scale=4)
    wq, wk = orc.rope(inp["q"], inp["k"], inp["cos"], inp["sin"], inp["position_ids"])
    qo, ko = rope.rope(inp["q"].cuda(), inp["k"].cuda(), inp["position_ids"].cuda(), theta=10000.0)
    assert _sincos_check(qo, inp["q"], wq) > 0.99
    assert _sincos_check(ko, inp["k"], wk) > 0.99


def test_sincos_mode_in_place_matches_out_of_place():
    inp = workloads.rope_8x4096(scale=8, seq=256)
    q, k, ids = inp["q"].cuda(), inp["k"].cuda(), inp["position_ids"].cuda()
    qo, ko = rope.rope(q, k, ids, theta=10000.0)
    rope.run({"q": q, "k": k, "position_ids": ids, "theta": 10000.0, "inplace": True})
    assert bits_equal(q, qo) and bits_equal(k, ko)


def test_matches_reference_kernel():
    lib = ref_lib("rope")
    if lib is None:
        pytest.skip("oracle/_ref not built")
    lib.launch.argtypes = [ctypes.c_void_p] * 7 + [ctypes.c_longlong] + [ctypes.c_int] * 7 + [ctypes.c_void_p]
    inp = workloads.rope_8x4096(scale=8, seq=1024)
    d = {k: (v.cuda() if torch.is_tensor(v) else v) for k, v in inp.items()}
    qo, ko = torch.empty_like(d["q"]), torch.empty_like(d["k"])
    b, s, hq, hd = d["q"].shape
    err = lib.launch(d["q"].data_ptr(), d["k"].data_ptr(), d["cos"].data_ptr(), d["sin"].data_ptr(),
                     d["position_ids"].data_ptr(), qo.data_ptr(), ko.data_ptr(), b * s, hq, d["k"].shape[2], hd, 1, 0,
                     40, 1, torch.cuda.current_stream().cuda_stream)
    assert err == 0
    gq, gk = rope.rope(d["q"], d["k"], d["position_ids"], d["cos"], d["sin"])
    assert bits_equal(gq, qo) and bits_equal(gk, ko)


def test_bad_arguments_raise():
    q = torch.zeros(1, 2, 2, 8, dtype=torch.bfloat16, device="cuda")
    ids = torch.zeros(1, 2, dtype=torch.int64, device="cuda")
    with pytest.raises(ValueError):
        rope.rope(q, q, ids)  # neither a cache nor theta
    with pytest.raises(ValueError):
        rope.rope(q.float(), q.float(), ids, theta=1e4)
    with pytest.raises(ValueError):
        rope.rope(q, q[:, :1], ids, theta=1e4)
