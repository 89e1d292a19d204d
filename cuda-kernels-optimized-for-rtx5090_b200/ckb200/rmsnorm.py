"""RMSNorm on B200: run({"x"[, "weight"]}) -> {"y"}.

Without a weight this is the reference's rmsnorm/candidate.py:40-52: y = x * rsqrt(mean(x^2, -1) + 1e-6) with the
rsqrt rounded to x's dtype before the product, for 2-D bf16 or fp16 x, through the reference's C ABI
(rmsnorm/kernel.cu:132). With inputs["weight"] (cols values, fp32 or x's dtype) it is the weighted form
y = x * rsqrt(mean(x^2) + eps) * weight in fp32 with one rounding at the end (ckb_rmsnorm_weighted_launch).
params.json beside this module may set "threads" (a multiple of 32 from 32 to 1024, default 256) as the reference's
does; it sizes the scalar fallback's blocks.
"""

import json
import os

import torch

from . import _native

_HERE = os.path.dirname(os.path.abspath(__file__))
_PARAMS_PATH = os.path.join(_HERE, "params.json")
_params = {}
if os.path.exists(_PARAMS_PATH):
    with open(_PARAMS_PATH) as _handle:
        _params = json.load(_handle)
_THREADS = int(_params.get("threads", 256))
_EPS = 1e-6
_DTYPES = {torch.bfloat16: 1, torch.float16: 2}
_W_DTYPES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}


def _problem(x, weight):
    """Why these inputs are not an RMSNorm these kernels serve, or None."""
    if x.dtype not in _DTYPES:
        return f"dtype {x.dtype}"
    if x.dim() != 2 or x.shape[1] < 1:
        return f"shape {tuple(x.shape)}"
    if weight is not None:
        if weight.dtype not in _W_DTYPES or weight.dim() != 1 or weight.shape[0] != x.shape[1]:
            return f"weight {weight.dtype} {tuple(weight.shape)} for x {tuple(x.shape)}"
    return None


def rmsnorm(x, weight=None, eps=_EPS, out=None):
    """RMSNorm of 2-D x over its last dim (weighted when weight is given) into `out`; returns it."""
    problem = _problem(x, weight)
    if problem:
        raise ValueError(f"rmsnorm candidate: {problem}")
    _native.require_cuda("rmsnorm", x, *(() if weight is None else (weight,)))
    x = x.contiguous()
    y = torch.empty_like(x) if out is None else out
    if y.shape != x.shape or y.dtype != x.dtype or not y.is_contiguous() or y.device != x.device:
        raise ValueError("rmsnorm: out must be a contiguous tensor of x's shape, dtype and device")
    rows, cols = x.shape
    lib = _native.load("rmsnorm")
    with torch.cuda.device(x.device):
        stream = _native.stream_of(x)
        if weight is None:
            err = lib.launch(x.data_ptr(), y.data_ptr(), rows, cols, _DTYPES[x.dtype], eps, _THREADS, stream)
        else:
            weight = weight.contiguous()
            err = lib.ckb_rmsnorm_weighted_launch(x.data_ptr(), weight.data_ptr(), y.data_ptr(), rows, cols,
                                                  _DTYPES[x.dtype], _W_DTYPES[weight.dtype], eps, stream)
    _native.check(err)
    return y


def run(inputs):
    return {"y": rmsnorm(inputs["x"], inputs.get("weight"))}
