"""Shared test helpers: device tensors with guard bands, the reference's own kernels (oracle/_ref) via ctypes, and
the tolerance checks the parity tests use."""

import ctypes
import os

import numpy as np
import torch

from oracle.numerics import to_f32, ulp_distance

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_DIR = os.path.join(ROOT, "oracle", "_ref")
CANARY = {torch.float32: 12345.678, torch.bfloat16: 12345.678, torch.float16: 1234.5, torch.int64: -77}


def guarded_empty(shape, dtype, device="cuda", pad=64):
    """A contiguous tensor of `shape` inside a larger buffer whose guard bands hold a canary; returns
    (tensor, check) where check() asserts the bands are untouched."""
    n = int(np.prod(shape)) if len(shape) else 1
    buf = torch.full((n + 2 * pad,), CANARY[dtype], dtype=dtype, device=device)
    view = buf[pad:pad + n].view(shape)

    def check():
        bands = torch.cat([buf[:pad], buf[pad + n:]]).cpu()
        want = torch.full_like(bands, CANARY[dtype])
        assert torch.equal(bands, want), "kernel wrote outside its output"

    return view, check


def misaligned_copy(t, offset_elems=1):
    """A contiguous device copy of t whose data pointer is offset_elems elements past a 16-byte boundary."""
    n = t.numel()
    buf = torch.empty(n + offset_elems, dtype=t.dtype, device=t.device)
    view = buf[offset_elems:offset_elems + n].view(t.shape)
    view.copy_(t)
    return view


def ref_lib(op):
    """The reference's own kernel library rebuilt for sm_100a (oracle/build_ref.sh), or None when not built."""
    path = os.path.join(REF_DIR, op, "libkernel.so")
    if not os.path.exists(path):
        return None
    return ctypes.CDLL(path)


def assert_ulp(got, want, dtype, max_ulp=1, what=""):
    d = ulp_distance(to_f32(got), to_f32(want), dtype)
    worst = int(d.max()) if d.size else 0
    assert worst <= max_ulp, f"{what}: {worst} ulp apart (allowed {max_ulp}); {(d > max_ulp).sum()} elements"
    return d


SUBNORMAL_FLOOR = 2.0 ** -148  # two steps of fp32's subnormal spacing (2^-149)


def assert_rel(got, want64, rel, what="", floor=SUBNORMAL_FLOOR):
    """|got - want| <= max(rel * |want|, floor) elementwise (want in fp64); NaN exactly where want is NaN. The floor
    only matters below fp32's FLT_MIN, where the format's own spacing (2^-149) is coarser than any relative bound
    near 1e-6: there an output must be within two subnormal steps, so a flushed-to-zero result fails."""
    g = got.detach().cpu().double().numpy()
    w = want64.detach().cpu().numpy()
    assert np.array_equal(np.isnan(g), np.isnan(w)), f"{what}: NaN pattern differs"
    ok = ~np.isnan(w)
    err = np.abs(g[ok] - w[ok])
    bound = np.maximum(rel * np.abs(w[ok]), floor)
    bad = err > bound
    assert not bad.any(), (f"{what}: {bad.sum()} elements beyond {rel} relative; worst "
                           f"{(err / np.maximum(np.abs(w[ok]), 1e-300)).max():.3e}")


def bits_equal(a, b):
    a = a.detach().cpu().contiguous()
    b = b.detach().cpu().contiguous()
    if a.dtype in (torch.bfloat16, torch.float16):
        return torch.equal(a.view(torch.int16), b.view(torch.int16))
    if a.dtype == torch.float32:
        return torch.equal(a.view(torch.int32), b.view(torch.int32))
    return torch.equal(a, b)
