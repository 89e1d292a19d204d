"""RMSNorm oracle (test infrastructure only), numpy fp32 with explicit roundings.

Unweighted: the reference's y = x * rsqrt(mean(x^2) + eps).to(x.dtype) (rmsnorm/candidate.py:3-5,
rmsnorm/kernel.cu:1-6): the sum of squares in fp32 accumulation (exact squares, rmsnorm/kernel.cu:58,80), the mean
sum / cols in fp32 (rmsnorm/kernel.cu:46), inv = rsqrt rounded to x's dtype (rmsnorm/kernel.cu:46), and
y = (x * inv) rounded to x's dtype (rmsnorm/kernel.cu:93). The sum is taken in fp64 and rounded once to fp32, the
most accurate fp32-accumulated value; kernels that sum in another order differ in its last bits.
Weighted (the BASELINE config; the reference has no weight): y = ((x * inv) * w) in fp32 with inv not rounded,
one rounding to x's dtype.
"""

import numpy as np
import torch

from .numerics import from_f32, round_to, to_f32


def inv_rms(xf, eps):
    """fp32 inverse RMS per row of float32 array xf [rows, cols]."""
    cols = xf.shape[1]
    ss = np.float32((xf.astype(np.float64) ** 2).sum(axis=1))
    mean = ss / np.float32(cols)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        return (np.float32(1.0) / np.sqrt(mean + np.float32(eps))).astype(np.float32)


def rmsnorm(x, weight=None, eps=1e-6):
    """Oracle RMSNorm of 2-D CPU tensor x (bf16 / fp16); returns a tensor of x's dtype."""
    xf = to_f32(x)
    inv = inv_rms(xf, eps)[:, None]
    with np.errstate(invalid="ignore", over="ignore"):
        if weight is None:
            y = xf * round_to(inv, x.dtype)
        else:
            y = (xf * inv) * to_f32(weight)[None, :]
    return from_f32(y.astype(np.float32), x.dtype)


def rmsnorm_cpu(x, weight=None, eps=1e-6):
    """Multi-threaded torch CPU restatement of the same semantics, the timed CPU baseline (no reference CPU code
    exists for RMSNorm): fp32 math, inv rounded to x's dtype without a weight."""
    xf = x.float()
    inv = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    if weight is None:
        return (xf * inv.to(x.dtype).float()).to(x.dtype)
    return (xf * inv * weight.float()).to(x.dtype)
