"""Top-k oracle (test infrastructure only), exact integer arithmetic in numpy.

The reference orders elements by a 64-bit composite (order-preserving key of the float bits << 32 | ~index),
topk/kernel.cu:1-3,56-60: larger value first, equal values by lower index; values decode bit-exactly from the key
(topk/kernel.cu:63-81), indices are int64. A bf16 element's key is that of the fp32 it widens to
(topk/kernel.cu:130-131). torch.topk is not used: on CPU it does not break ties by the lower index.
"""

import numpy as np
import torch


def keys(x):
    """uint32 order-preserving keys of CPU tensor x (fp32 or bf16)."""
    x = x.detach().cpu().contiguous()
    if x.dtype == torch.bfloat16:
        bits = x.view(torch.int16).numpy().view(np.uint16).astype(np.uint32) << 16
    elif x.dtype == torch.float32:
        bits = x.numpy().view(np.uint32)
    else:
        raise ValueError(f"dtype {x.dtype}")
    return np.where(bits & 0x80000000, ~bits, bits | 0x80000000).astype(np.uint32)


def composites(x, col_offset=0):
    """uint64 composites [rows, cols] of x with global column indices col_offset + j."""
    key = keys(x).astype(np.uint64)
    idx = (np.arange(x.shape[1], dtype=np.uint64) + np.uint64(col_offset)).astype(np.uint32)
    return (key << np.uint64(32)) | (~idx).astype(np.uint64)[None, :]


def top_composites(c, k):
    """The k largest composites of each row, descending (zero padded when a row has fewer than k)."""
    rows, cols = c.shape
    if cols > k:
        c = np.partition(c, cols - k, axis=1)[:, cols - k:]
    out = np.sort(c, axis=1)[:, ::-1]
    if out.shape[1] < k:
        out = np.concatenate([out, np.zeros((rows, k - out.shape[1]), dtype=np.uint64)], axis=1)
    return np.ascontiguousarray(out)


def decode(c, dtype):
    """(values tensor in dtype, int64 indices tensor) of composites c."""
    key = (c >> np.uint64(32)).astype(np.uint32)
    bits = np.where(key & 0x80000000, key & 0x7FFFFFFF, ~key).astype(np.uint32)
    idx = (~(c & np.uint64(0xFFFFFFFF)).astype(np.uint32)).astype(np.int64)
    if dtype == torch.bfloat16:
        values = torch.from_numpy((bits >> 16).astype(np.uint16).view(np.int16)).view(torch.bfloat16)
    else:
        values = torch.from_numpy(bits.view(np.float32).copy())
    return values, torch.from_numpy(idx)


def topk(x, k):
    """Oracle top-k of 2-D CPU tensor x: (values, indices), the reference's order and bits."""
    return decode(top_composites(composites(x), k), x.dtype)


def shard_lists(x_shard, col_offset, k):
    """A column shard's sorted top-k composites [rows, k] as int64 bits (what ckb200.topk.shard_lists returns)."""
    return torch.from_numpy(top_composites(composites(x_shard, col_offset), k).view(np.int64))


def merge_lists(lists, dtype, k):
    """Final (values, indices) from gathered shard lists [nlists, rows, k] (int64 bits of composites)."""
    c = lists.detach().cpu().numpy().view(np.uint64)
    nlists, rows, kk = c.shape
    allc = np.transpose(c, (1, 0, 2)).reshape(rows, nlists * kk)
    return decode(top_composites(allc, k), dtype)


def topk_cpu(x, k):
    """Multi-threaded torch CPU top-k with the same tie rule (stable descending sort), the timed CPU baseline."""
    v, i = torch.sort(x, dim=-1, descending=True, stable=True)
    return v[:, :k], i[:, :k]


def topk_softmax(x, k, temperature=1.0, uniforms=None):
    """Oracle of top-k sampling (no reference counterpart; its top-k is topk() above): the exact top k, then the
    softmax of those k logits / temperature in fp64, and for each uniform u the first index whose cumulative
    probability exceeds u. Returns (probs float64 [rows, k], indices int64 [rows, k], samples int64 [rows] or None,
    margin: the distance of each u from the nearest cumulative boundary)."""
    values, indices = topk(x, k)
    v = values.to(torch.float64) / float(temperature)
    p = torch.softmax(v, dim=-1)
    if uniforms is None:
        return p, indices, None, None
    cum = torch.cumsum(p, dim=-1)
    u = uniforms.detach().cpu().to(torch.float64)[:, None]
    pick = torch.clamp((cum <= u).sum(dim=-1), max=k - 1)
    samples = indices.gather(1, pick[:, None])[:, 0]
    margin = (cum - u).abs().min(dim=-1).values
    return p, indices, samples, margin
