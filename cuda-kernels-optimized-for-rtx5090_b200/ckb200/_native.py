"""ctypes bindings of the four kernel libraries (the reference's own FFI style, e.g. rmsnorm/candidate.py:25-28).

A library that is missing raises at first use: there is no CPU or PyTorch fallback for any op. Every binding takes
plain pointers, sizes and the caller's CUDA stream, exactly as declared in include/ckb200_<op>.h.
"""

import ctypes
import os
import threading

import torch

from . import build as _build

_VP, _LL, _INT, _FLT = ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_float
_UINT, _PVP = ctypes.c_uint, ctypes.POINTER(ctypes.c_void_p)

# Symbol -> (restype, argtypes), per op; mirrors include/ckb200_<op>.h.
SIGNATURES = {
    "softmax": {
        "launch": (_INT, [_VP, _VP, _LL, _LL, _INT, _INT, _INT, _VP]),
        "ckb_softmax_status": (_INT, [_INT]),
    },
    "rmsnorm": {
        "launch": (_INT, [_VP, _VP, _LL, _INT, _INT, _FLT, _INT, _VP]),
        "ckb_rmsnorm_weighted_launch": (_INT, [_VP, _VP, _VP, _LL, _INT, _INT, _INT, _FLT, _VP]),
    },
    "rope": {
        "launch": (_INT, [_VP] * 7 + [_LL] + [_INT] * 7 + [_VP]),
        "ckb_rope_sincos_launch": (_INT, [_VP] * 6 + [_LL] + [_INT] * 4 + [_VP]),
        "ckb_rope_kv_cache_launch": (_INT, [_VP] * 11 + [_LL] + [_INT] * 5 + [_VP]),
    },
    "topk": {
        "plan": (_LL, [_LL, _LL, _INT, _INT, _INT, _INT]),
        "launch": (_INT, [_VP] * 5 + [_LL, _LL, _INT, _INT, _INT, _INT, _LL, _VP]),
        "ckb_topk_shard_launch": (_INT, [_VP] * 4 + [_LL, _LL, _LL, _INT, _INT, _LL, _VP]),
        "ckb_topk_softmax_launch": (_INT, [_VP] * 5 + [_LL, _LL, _INT, _INT, _LL, _FLT, _VP, _VP, _VP]),
        "ckb_topk_merge_launch": (_INT, [_VP, _INT, _VP, _VP, _LL, _INT, _INT, _VP]),
        "ckb_topk_launch_noalloc": (_INT, [_VP, _VP, _VP, _LL, _LL, _INT, _INT, _VP]),
        "ckb_topk_shard_push_launch": (_INT, [_VP] * 5 + [_LL, _LL, _LL, _INT, _INT, _LL, _PVP, _PVP, _INT, _INT,
                                                           _UINT, _VP]),
        "ckb_topk_merge_wait_launch": (_INT, [_VP, _VP, _INT, _UINT, _VP, _VP, _LL, _INT, _INT, _VP]),
        "ckb_p2p_alloc": (_INT, [_PVP, ctypes.c_ulonglong]),
        "ckb_p2p_free": (_INT, [_VP]),
        "ckb_p2p_export": (_INT, [_VP, _VP]),
        "ckb_p2p_import": (_INT, [_VP, _PVP]),
        "ckb_p2p_close": (_INT, [_VP]),
        "ckb_topk_status": (_INT, [_INT]),
    },
}

_libs = {}
_lock = threading.Lock()


def load(op):
    """The op's library with typed entry points; raises if it has not been built."""
    lib = _libs.get(op)
    if lib is not None:
        return lib
    with _lock:
        lib = _libs.get(op)
        if lib is None:
            path = _build.lib_path(op)
            if not os.path.exists(path):
                raise RuntimeError(f"ckb200: the {op} CUDA library is not built ({path}); run "
                                   f"`python -m ckb200.build` or __graft_entry__.build() first")
            lib = ctypes.CDLL(path)
            for name, (res, args) in SIGNATURES[op].items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _libs[op] = lib
    return lib


def stream_of(t):
    """The current torch stream of t's device, as the cudaStream_t handle the C ABI takes."""
    return torch.cuda.current_stream(t.device).cuda_stream


def check(err):
    """The reference wrappers' error convention (rmsnorm/candidate.py:50-51, rope/candidate.py:55-56,
    topk/candidate.py:79-80): any non-zero return, -1 for rejected arguments included, raises RuntimeError."""
    if err:
        raise RuntimeError(f"kernel launch failed: CUDA error {err}")


def require_cuda(op, *tensors):
    for t in tensors:
        if not t.is_cuda:
            raise ValueError(f"{op}: tensors must be on a CUDA device (there is no CPU path), got {t.device}")
    dev = tensors[0].device
    for t in tensors[1:]:
        if t.device != dev:
            raise ValueError(f"{op}: tensors on different devices: {dev} and {t.device}")
