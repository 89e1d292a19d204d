"""Bit-level helpers of the oracle (test infrastructure only): bf16/fp16 <-> fp32 and ulp distances, in numpy.

bf16 is the high half of an fp32; fp32 -> bf16 rounds to nearest even (CUDA's __float2bfloat16_rn, used by the
reference at rmsnorm/kernel.cu:22, rope/kernel.cu:24, softmax/kernel.cu:30).
"""

import numpy as np
import torch


def bf16_bits_to_f32(bits):
    """uint16 bf16 bit patterns -> float32 values (exact)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(f):
    """float32 -> uint16 bf16 bit patterns, round to nearest even; NaN stays NaN (quiet)."""
    f = np.ascontiguousarray(f, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint32)
    nan = np.isnan(f)
    r[nan] = ((u[nan] >> 16).astype(np.uint32)) | 0x40
    return r.astype(np.uint16)


def round_to(f, dtype):
    """float32 values rounded to torch dtype (bf16 / fp16 / fp32), returned as float32."""
    f = np.asarray(f, dtype=np.float32)
    if dtype == torch.bfloat16:
        return bf16_bits_to_f32(f32_to_bf16_bits(f))
    if dtype == torch.float16:
        return f.astype(np.float16).astype(np.float32)
    if dtype == torch.float32:
        return f
    raise ValueError(f"dtype {dtype}")


def to_f32(t):
    """A CPU torch tensor (fp32 / bf16 / fp16 / fp64) as a float32 numpy array holding exactly its values."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return bf16_bits_to_f32(t.view(torch.int16).numpy().view(np.uint16))
    if t.dtype in (torch.float16, torch.float32):
        return t.numpy().astype(np.float32)
    raise ValueError(f"dtype {t.dtype}")


def from_f32(f, dtype):
    """float32 numpy values (already representable in dtype, or rounded to nearest even) -> CPU torch tensor."""
    f = np.ascontiguousarray(f, dtype=np.float32)
    if dtype == torch.bfloat16:
        return torch.from_numpy(f32_to_bf16_bits(f).view(np.int16)).view(torch.bfloat16)
    if dtype == torch.float16:
        return torch.from_numpy(f.astype(np.float16))
    if dtype == torch.float32:
        return torch.from_numpy(f.copy())
    raise ValueError(f"dtype {dtype}")


def ordered(f, dtype):
    """Monotone integer image of the values of `dtype` (adjacent representable values differ by 1)."""
    f = np.asarray(f, dtype=np.float32)
    if dtype == torch.bfloat16:
        b = f32_to_bf16_bits(f).astype(np.int64)
        sign = 0x8000
    elif dtype == torch.float16:
        b = f.astype(np.float16).view(np.uint16).astype(np.int64)
        sign = 0x8000
    else:
        b = f.view(np.uint32).astype(np.int64)
        sign = 0x80000000
    return np.where(b & sign, -(b & (sign - 1)), b)


def ulp_distance(a, b, dtype):
    """|steps| between a and b in dtype's representable values (NaN vs NaN = 0, NaN vs number = huge)."""
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    d = np.abs(ordered(a, dtype) - ordered(b, dtype))
    na, nb = np.isnan(a), np.isnan(b)
    d = np.where(na & nb, 0, d)
    return np.where(na ^ nb, np.iinfo(np.int64).max, d)
