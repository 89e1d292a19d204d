"""RoPE oracle (test infrastructure only), numpy fp32 with each product and sum rounded.

The reference's rotation (rope/kernel.cu:5-8,73-79,120-126): for i < h = head_dim / 2
  out[i]     = rn(rn(x[i] * cos[i]) - rn(x[i + h] * sin[i]))
  out[i + h] = rn(rn(x[i + h] * cos[i + h]) + rn(x[i] * sin[i + h]))
with cos/sin rows [max_position, head_dim] picked by position_ids (rope/kernel.cu:102-107), then one
round-to-nearest-even conversion to the q/k dtype. numpy float32 ufuncs round every operation and never contract
into an FMA, so these are the same bits.
"""

import numpy as np
import torch

from .numerics import from_f32, to_f32


def rotate(xf, cf, sf):
    """Rotated float32 values of xf [..., D] with per-row cos/sin cf, sf [..., D] (broadcast over heads)."""
    h = xf.shape[-1] // 2
    a, b = xf[..., :h], xf[..., h:]
    lo = (a * cf[..., :h]).astype(np.float32) - (b * sf[..., :h]).astype(np.float32)
    hi = (b * cf[..., h:]).astype(np.float32) + (a * sf[..., h:]).astype(np.float32)
    return np.concatenate([lo, hi], axis=-1).astype(np.float32)


def rope(q, k, cos, sin, position_ids):
    """Oracle RoPE of CPU tensors q [B,S,Hq,D], k [B,S,Hkv,D] with the cache rows cos/sin[position_ids]."""
    ids = position_ids.cpu().numpy()
    cf = to_f32(cos)[ids][:, :, None, :]
    sf = to_f32(sin)[ids][:, :, None, :]
    with np.errstate(invalid="ignore", over="ignore"):
        qo = rotate(to_f32(q), cf, sf)
        ko = rotate(to_f32(k), cf, sf)
    return from_f32(qo, q.dtype), from_f32(ko, k.dtype)


def cos_sin_cache(theta, head_dim, max_position, dtype=torch.float32):
    """The usual rotary cache: inv_freq = 1 / theta^(arange(0, D, 2) / D) in fp32, freqs = positions x inv_freq in
    fp32, emb = cat(freqs, freqs), cos/sin of emb in fp32, cast to dtype. Returns (cos, sin) [max_position, D]."""
    inv_freq = 1.0 / (float(theta) ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    t = torch.arange(max_position, dtype=torch.int64).float()
    freqs = torch.outer(t, inv_freq)
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def rope_cpu(q, k, cos, sin, position_ids):
    """Multi-threaded torch CPU restatement (the timed CPU baseline; the reference ships no CPU RoPE):
    x * cos + rotate_half(x) * sin in fp32, one rounding."""
    c = cos[position_ids].unsqueeze(2).float()
    s = sin[position_ids].unsqueeze(2).float()

    def rot(x):
        xf = x.float()
        h = xf.shape[-1] // 2
        rh = torch.cat([-xf[..., h:], xf[..., :h]], dim=-1)
        return (xf * c + rh * s).to(x.dtype)

    return rot(q), rot(k)


def rope_kv_cache(q, k, v, cos, sin, position_ids, key_cache, value_cache, slot_mapping):
    """Oracle of the fused RoPE + paged KV-cache write (no reference counterpart; its rotation is rope() above):
    (q_rot, k_rot, key_cache', value_cache') with the rotated k and the unrotated v of token t stored into row
    slot_mapping[t] of the caches viewed [slots, Hkv, D] (negative slots skipped; other rows unchanged)."""
    qo, ko = rope(q, k, cos, sin, position_ids)
    kc = key_cache.detach().cpu().clone()
    vc = value_cache.detach().cpu().clone()
    hkv, d = k.shape[2], k.shape[3]
    kc_rows, vc_rows = kc.view(-1, hkv, d), vc.view(-1, hkv, d)
    slots = slot_mapping.cpu().reshape(-1)
    kf, vf = ko.reshape(-1, hkv, d), v.detach().cpu().reshape(-1, hkv, d)
    for t, sl in enumerate(slots.tolist()):
        if sl >= 0:
            kc_rows[sl] = kf[t]
            vc_rows[sl] = vf[t]
    return qo, ko, kc, vc
