"""Softmax over the last dim on B200: run({"x"}) -> {"y"}.

Keeps the entry signature of the reference's softmax/baseline.py:12-13 (`run(inputs) -> {"y": softmax(x, -1)}`) and
drives the sm_100a kernels through the reference's softmax C ABI (softmax/kernel.cu:520). fp32 and bf16 inputs of
any rank (the leading dims are flattened into rows); the output is a new tensor of x's shape and dtype.
"""

import torch

from . import _native

_DTYPES = {torch.float32: 0, torch.bfloat16: 1}


def _problem(x):
    """Why x is not an input these kernels serve, or None."""
    if x.dtype not in _DTYPES:
        return f"dtype {x.dtype}"
    if x.dim() < 1:
        return f"shape {tuple(x.shape)}"
    return None


def softmax(x, out=None):
    """softmax(x, dim=-1) into `out` (allocated when None); returns it."""
    problem = _problem(x)
    if problem:
        raise ValueError(f"softmax: {problem}")
    _native.require_cuda("softmax", x)
    x = x.contiguous()
    y = torch.empty_like(x) if out is None else out
    if y.shape != x.shape or y.dtype != x.dtype or not y.is_contiguous() or y.device != x.device:
        raise ValueError("softmax: out must be a contiguous tensor of x's shape, dtype and device")
    cols = x.shape[-1] if x.dim() else 1
    rows = x.numel() // cols if cols else 0
    lib = _native.load("softmax")
    with torch.cuda.device(x.device):
        _native.check(lib.launch(x.data_ptr(), y.data_ptr(), rows, cols, _DTYPES[x.dtype], 256, 1024,
                                 _native.stream_of(x)))
    return y


def run(inputs):
    return {"y": softmax(inputs["x"])}
