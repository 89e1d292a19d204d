"""RoPE on B200: run({"q", "k", "cos", "sin", "position_ids"}) -> {"q_out", "k_out"}.

The reference's rope/candidate.py:44-57: q [B, S, Hq, D] and k [B, S, Hkv, D] in bf16 or fp16 are rotated by the
cos/sin cache rows [max_position, D] (fp32, bf16 or fp16) that position_ids [B, S] (int64) pick, half-split pairing,
fp32 math with each product and the sum rounded, one rounding to the output dtype (rope/kernel.cu:1-8).
Extensions, both through this module's inputs:
  * inputs["inplace"] = True rotates q and k in place (they must be contiguous) and returns them as q_out / k_out;
  * no "cos"/"sin" but inputs["theta"] computes cos/sin in registers by sincosf(position * inv_freq) with
    inv_freq = 1 / theta^(2i / D) (the cat(freqs, freqs) cache layout), so no cache is read.
params.json beside this module may set "rows" and "splits" as the reference's does; they are validated by the C ABI
and do not change the B200 launch shape.
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
_ROWS = int(_params.get("rows", 40))
_SPLITS = int(_params.get("splits", 1))
_QK = {torch.bfloat16: 1, torch.float16: 2}
_CACHE = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}

_inv_freq_cache = {}


def inv_freq(theta, head_dim, device):
    """fp32 [head_dim / 2] inverse frequencies 1 / theta^(2i / head_dim), computed as the usual rotary-embedding
    cache builder does (fp32 arange / head_dim, fp32 power, fp32 reciprocal) so sincos mode sees the same angles."""
    key = (float(theta), int(head_dim), torch.device(device))
    t = _inv_freq_cache.get(key)
    if t is None:
        exps = torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim
        t = (1.0 / (float(theta) ** exps)).to(torch.float32).to(device)
        _inv_freq_cache[key] = t
    return t


def _problem(q, k, cos, sin, ids):
    """Why these inputs are not a rope call these kernels serve, or None (rope/candidate.py:32-41)."""
    if q.dtype not in _QK or k.dtype != q.dtype:
        return f"dtypes q {q.dtype}, k {k.dtype}"
    if cos is not None and (cos.dtype not in _CACHE or sin is None or sin.dtype != cos.dtype):
        return f"dtypes cos {cos.dtype}, sin {None if sin is None else sin.dtype}"
    if ids.dtype != torch.int64 or q.dim() != 4 or k.dim() != 4 or ids.dim() != 2 or \
            (cos is not None and cos.dim() != 2):
        return f"position_ids {ids.dtype} {tuple(ids.shape)}, q {tuple(q.shape)}, k {tuple(k.shape)}"
    if tuple(q.shape[:2]) != tuple(ids.shape) or tuple(k.shape[:2]) != tuple(ids.shape) or \
            q.shape[3] != k.shape[3] or q.shape[3] % 2 or \
            (cos is not None and (tuple(sin.shape) != tuple(cos.shape) or cos.shape[1] != q.shape[3])):
        return f"shapes q {tuple(q.shape)}, k {tuple(k.shape)}, position_ids {tuple(ids.shape)}" + \
            ("" if cos is None else f", cos {tuple(cos.shape)}")
    return None


def rope(q, k, position_ids, cos=None, sin=None, theta=None, inplace=False, out=None):
    """Rotates q and k; returns (q_out, k_out). Cache mode with cos/sin, sincos mode with theta. out = (q_out,
    k_out) gives the output tensors (contiguous, q's and k's shapes and dtype) instead of new ones."""
    if cos is None and sin is None and theta is None:
        raise ValueError("rope candidate: give the cos/sin cache or theta")
    if (cos is None) != (sin is None):
        raise ValueError("rope candidate: give both cos and sin")
    problem = _problem(q, k, cos, sin, position_ids)
    if problem:
        raise ValueError(f"rope candidate: {problem}")
    _native.require_cuda("rope", q, k, position_ids, *(() if cos is None else (cos, sin)))
    if inplace:
        if not (q.is_contiguous() and k.is_contiguous()):
            raise ValueError("rope candidate: in-place rotation needs contiguous q and k")
        q_out, k_out = q, k
    else:
        q, k = q.contiguous(), k.contiguous()
        if out is None:
            q_out, k_out = torch.empty_like(q), torch.empty_like(k)
        else:
            q_out, k_out = out
            for o, t in ((q_out, q), (k_out, k)):
                if o.shape != t.shape or o.dtype != t.dtype or not o.is_contiguous() or o.device != t.device:
                    raise ValueError("rope candidate: out must be contiguous tensors of q's and k's shapes, dtype "
                                     "and device")
    ids = position_ids.contiguous()
    batch, seq, q_heads, head_dim = q.shape
    lib = _native.load("rope")
    with torch.cuda.device(q.device):
        stream = _native.stream_of(q)
        if cos is not None:
            cos, sin = cos.contiguous(), sin.contiguous()
            err = lib.launch(q.data_ptr(), k.data_ptr(), cos.data_ptr(), sin.data_ptr(), ids.data_ptr(),
                             q_out.data_ptr(), k_out.data_ptr(), batch * seq, q_heads, k.shape[2], head_dim,
                             _QK[q.dtype], _CACHE[cos.dtype], _ROWS, _SPLITS, stream)
        else:
            freqs = inv_freq(theta, head_dim, q.device)
            err = lib.ckb_rope_sincos_launch(q.data_ptr(), k.data_ptr(), freqs.data_ptr(), ids.data_ptr(),
                                             q_out.data_ptr(), k_out.data_ptr(), batch * seq, q_heads, k.shape[2],
                                             head_dim, _QK[q.dtype], stream)
    _native.check(err)
    return q_out, k_out


def run(inputs):
    q_out, k_out = rope(inputs["q"], inputs["k"], inputs["position_ids"], inputs.get("cos"), inputs.get("sin"),
                        inputs.get("theta"), bool(inputs.get("inplace", False)))
    return {"q_out": q_out, "k_out": k_out}


def rope_kv_cache(q, k, v, position_ids, cos, sin, key_cache, value_cache, slot_mapping, inplace=True,
                  write_k=True):
    """RoPE fused with the paged KV-cache write, one kernel: q [B, S, Hq, D] and k [B, S, Hkv, D] are rotated by the
    cos/sin rows that position_ids [B, S] pick (in place when inplace, else into new tensors; k is not written back
    when write_k is False), and the rotated k and the unrotated v [B, S, Hkv, D] of token (b, s) are stored into
    key_cache / value_cache [num_blocks, block_size, Hkv, D] (q's dtype) at slot slot_mapping[b, s] (int64,
    block * block_size + offset; negative: padding, not written). Returns (q_out, k_out or None)."""
    problem = _problem(q, k, cos, sin, position_ids)
    if problem:
        raise ValueError(f"rope candidate: {problem}")
    if v.shape != k.shape or v.dtype != k.dtype:
        raise ValueError(f"rope candidate: v {v.dtype} {tuple(v.shape)} must match k {k.dtype} {tuple(k.shape)}")
    for name, c in (("key_cache", key_cache), ("value_cache", value_cache)):
        if c.dtype != q.dtype or c.dim() != 4 or tuple(c.shape[2:]) != tuple(k.shape[2:]) or not c.is_contiguous():
            raise ValueError(f"rope candidate: {name} must be a contiguous [blocks, block_size, {k.shape[2]}, "
                             f"{k.shape[3]}] tensor of {q.dtype}, got {c.dtype} {tuple(c.shape)}")
    if slot_mapping.dtype != torch.int64 or tuple(slot_mapping.shape) != tuple(position_ids.shape):
        raise ValueError(f"rope candidate: slot_mapping must be int64 {tuple(position_ids.shape)}")
    _native.require_cuda("rope", q, k, v, position_ids, cos, sin, key_cache, value_cache, slot_mapping)
    if inplace:
        if not (q.is_contiguous() and k.is_contiguous()):
            raise ValueError("rope candidate: in-place rotation needs contiguous q and k")
        q_out, k_out = q, (k if write_k else None)
    else:
        q, k = q.contiguous(), k.contiguous()
        q_out, k_out = torch.empty_like(q), (torch.empty_like(k) if write_k else None)
    v, ids, slots = v.contiguous(), position_ids.contiguous(), slot_mapping.contiguous()
    cos, sin = cos.contiguous(), sin.contiguous()
    batch, seq, q_heads, head_dim = q.shape
    lib = _native.load("rope")
    with torch.cuda.device(q.device):
        err = lib.ckb_rope_kv_cache_launch(q.data_ptr(), k.data_ptr(), v.data_ptr(), cos.data_ptr(), sin.data_ptr(),
                                           ids.data_ptr(), slots.data_ptr(), q_out.data_ptr(),
                                           None if k_out is None else k_out.data_ptr(), key_cache.data_ptr(),
                                           value_cache.data_ptr(), batch * seq, q_heads, k.shape[2], head_dim,
                                           _QK[q.dtype], _CACHE[cos.dtype], _native.stream_of(q))
    _native.check(err)
    return q_out, k_out
