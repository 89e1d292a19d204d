"""Top-k on B200: run({"x"}) -> {"values", "indices"}, K = 50.

The reference's topk/candidate.py:66-81: the K largest entries of each row of 2-D x (fp32 or bf16), in descending
order with ties broken by the lower index, values in x's dtype (bit-exact) and int64 indices, through the reference's
C ABI (plan + launch, topk/kernel.cu:520,549). plan() is cached per (device, shape, dtype); rows split into several
chunks merge through an int64 workspace and per-row int32 counters (zeroed once, left zeroed by the kernel), as the
reference does. Launches of one shape on one stream are serialised, so the cached workspace is reused.
params.json beside this module may set "log2_threads" (7..9), "log2_depth" (1..3) and "min_chunk" as the reference's
does; the first two are validated by the C ABI only, min_chunk bounds the plan's chunk from below.

Also here: topk(x, k) for any k <= 512, and the two halves of the vocab-sharded variant, shard_lists (local top-k of a
column shard as sorted 64-bit composites with global column indices) and merge_lists (the final merge after those
lists were gathered from every shard).
"""

import json
import os

import torch

from . import _native

K = 50
MAX_K = 512
_HERE = os.path.dirname(os.path.abspath(__file__))
_PARAMS_PATH = os.path.join(_HERE, "params.json")
_params = {}
if os.path.exists(_PARAMS_PATH):
    with open(_PARAMS_PATH) as _handle:
        _params = json.load(_handle)
_THREADS = 1 << int(_params.get("log2_threads", 8))
_DEPTH = 1 << int(_params.get("log2_depth", 2))
_MIN_CHUNK = int(_params.get("min_chunk", 2048))
_DTYPES = {torch.float32: 0, torch.bfloat16: 1}

_counters = {}
_plans = {}  # (device, rows, cols, dtype, k) -> (chunk, workspace)


def _row_counters(device, rows):
    counters = _counters.get(device)
    if counters is None or counters.numel() < rows:
        counters = torch.zeros(rows if rows > 4096 else 4096, dtype=torch.int32, device=device)
        _counters[device] = counters
    return counters


def _plan(x, rows, cols, dtype, k):
    key = (x.device, rows, cols, dtype, k)
    hit = _plans.get(key)
    if hit is not None:
        return hit
    lib = _native.load("topk")
    with torch.cuda.device(x.device):
        chunk = lib.plan(rows, cols, dtype, _THREADS, _DEPTH, _MIN_CHUNK)
    nchunks = -(-cols // chunk)
    work = torch.empty(rows * nchunks * k if nchunks > 1 else 1, dtype=torch.int64, device=x.device)
    if len(_plans) > 16:
        _plans.clear()
    _plans[key] = (chunk, work)
    return chunk, work


def _check_x(x, k):
    dtype = _DTYPES.get(x.dtype)
    if dtype is None or x.dim() != 2 or x.shape[1] < k:
        raise ValueError(f"topk candidate takes a 2-D fp32 or bf16 tensor with at least {k} columns, "
                         f"got {x.dtype} with shape {tuple(x.shape)}")
    if not 1 <= k <= MAX_K:
        raise ValueError(f"topk candidate: k must be in [1, {MAX_K}], got {k}")
    _native.require_cuda("topk", x)
    return dtype


def topk(x, k=K, out=None):
    """The k largest entries of each row of x, descending, ties by lower index: (values, int64 indices), written
    into out = (values, indices) when given (contiguous [rows, k] tensors of x's dtype and int64)."""
    dtype = _check_x(x, k)
    x = x.contiguous()
    rows, cols = x.shape
    chunk, work = _plan(x, rows, cols, dtype, k)
    counters = _row_counters(x.device, rows)
    if out is None:
        values = torch.empty((rows, k), dtype=x.dtype, device=x.device)
        indices = torch.empty((rows, k), dtype=torch.int64, device=x.device)
    else:
        values, indices = out
        for t, dt in ((values, x.dtype), (indices, torch.int64)):
            if tuple(t.shape) != (rows, k) or t.dtype != dt or not t.is_contiguous() or t.device != x.device:
                raise ValueError(f"topk candidate: out must be contiguous [rows, k] tensors of {x.dtype} and "
                                 f"int64 on x's device")
    lib = _native.load("topk")
    with torch.cuda.device(x.device):
        err = lib.launch(x.data_ptr(), values.data_ptr(), indices.data_ptr(), work.data_ptr(), counters.data_ptr(),
                         rows, cols, k, dtype, _THREADS, _DEPTH, chunk, _native.stream_of(x))
    _native.check(err)
    return values, indices


def run(inputs):
    values, indices = topk(inputs["x"], K)
    return {"values": values, "indices": indices}


def topk_softmax(x, k=K, temperature=1.0, uniforms=None):
    """Top-k sampling over each row of x (fp32 or bf16 logits): (probs, indices, samples). probs [rows, k] float is
    the softmax over the row's k largest logits divided by temperature, in descending order, with their int64
    indices; with uniforms (float [rows] in [0, 1), on x's device) samples [rows] int64 holds each row's sampled
    token (the first entry whose cumulative probability exceeds the uniform), else None. One kernel: the softmax
    runs in the top-k epilogue, so the row is read once."""
    dtype = _check_x(x, k)
    if not (float(temperature) > 0.0 and float(temperature) < float("inf")):
        raise ValueError(f"topk_softmax: temperature must be a positive finite number, got {temperature}")
    x = x.contiguous()
    rows, cols = x.shape
    chunk, work = _plan(x, rows, cols, dtype, k)
    counters = _row_counters(x.device, rows)
    probs = torch.empty((rows, k), dtype=torch.float32, device=x.device)
    indices = torch.empty((rows, k), dtype=torch.int64, device=x.device)
    samples = None
    if uniforms is not None:
        if uniforms.dtype != torch.float32 or uniforms.shape != (rows,) or uniforms.device != x.device:
            raise ValueError("topk_softmax: uniforms must be float32 [rows] on x's device")
        uniforms = uniforms.contiguous()
        samples = torch.empty(rows, dtype=torch.int64, device=x.device)
    lib = _native.load("topk")
    with torch.cuda.device(x.device):
        err = lib.ckb_topk_softmax_launch(x.data_ptr(), probs.data_ptr(), indices.data_ptr(), work.data_ptr(),
                                          counters.data_ptr(), rows, cols, k, dtype, chunk, float(temperature),
                                          None if uniforms is None else uniforms.data_ptr(),
                                          None if samples is None else samples.data_ptr(), _native.stream_of(x))
    _native.check(err)
    return probs, indices, samples


def shard_lists(x, col_offset, k=K, out=None):
    """Local top-k of a column shard x [rows, cols] holding global columns [col_offset, col_offset + cols): returns
    [rows, k] int64 tensor whose bits are the sorted 64-bit composites (key << 32 | ~global_index), zero padded."""
    dtype = _check_x(x, k)
    x = x.contiguous()
    rows, cols = x.shape
    chunk, work = _plan(x, rows, cols, dtype, k)
    counters = _row_counters(x.device, rows)
    lists = torch.empty((rows, k), dtype=torch.int64, device=x.device) if out is None else out
    if lists.shape != (rows, k) or lists.dtype != torch.int64 or not lists.is_contiguous():
        raise ValueError("topk shard: out must be a contiguous int64 [rows, k] tensor")
    lib = _native.load("topk")
    with torch.cuda.device(x.device):
        err = lib.ckb_topk_shard_launch(x.data_ptr(), lists.data_ptr(), work.data_ptr(), counters.data_ptr(),
                                        rows, cols, int(col_offset), k, dtype, chunk, _native.stream_of(x))
    _native.check(err)
    return lists


def merge_lists(lists, dtype, k=K):
    """Final top-k from gathered shard lists [nlists, rows, k] (int64 composites): (values in dtype, indices)."""
    if dtype not in _DTYPES:
        raise ValueError(f"topk merge: dtype {dtype}")
    if lists.dtype != torch.int64 or lists.dim() != 3 or lists.shape[2] != k:
        raise ValueError(f"topk merge: lists must be int64 [nlists, rows, {k}], got {lists.dtype} "
                         f"{tuple(lists.shape)}")
    _native.require_cuda("topk merge", lists)
    lists = lists.contiguous()
    nlists, rows, _ = lists.shape
    values = torch.empty((rows, k), dtype=dtype, device=lists.device)
    indices = torch.empty((rows, k), dtype=torch.int64, device=lists.device)
    lib = _native.load("topk")
    with torch.cuda.device(lists.device):
        err = lib.ckb_topk_merge_launch(lists.data_ptr(), nlists, values.data_ptr(), indices.data_ptr(), rows, k,
                                        _DTYPES[dtype], _native.stream_of(lists))
    _native.check(err)
    return values, indices


def shard_push(x, col_offset, k, lists_ptrs, flags_ptrs, rank, epoch, values=None, indices=None):
    """Local half of the vocab-sharded top-k over peer memory: the shard's row lists go to slot `rank` of every
    rank's exchange buffer (lists_ptrs / flags_ptrs: one device address per rank, this call's parity) and each row's
    flag is set to `epoch` there (ckb_topk_shard_push_launch). With values / indices ([rows, k] in x's dtype and
    int64) the final top k of the full rows is written too (in the same kernel when its CTAs fit the GPU at once)."""
    import ctypes

    dtype = _check_x(x, k)
    x = x.contiguous()
    rows, cols = x.shape
    if (values is None) != (indices is None):
        raise ValueError("topk shard push: give both values and indices, or neither")
    chunk, work = _plan(x, rows, cols, dtype, k)
    counters = _row_counters(x.device, rows)
    world = len(lists_ptrs)
    lists_arr = (ctypes.c_void_p * world)(*lists_ptrs)
    flags_arr = (ctypes.c_void_p * world)(*flags_ptrs)
    lib = _native.load("topk")
    with torch.cuda.device(x.device):
        err = lib.ckb_topk_shard_push_launch(x.data_ptr(), None if values is None else values.data_ptr(),
                                             None if indices is None else indices.data_ptr(), work.data_ptr(),
                                             counters.data_ptr(), rows, cols, int(col_offset), k, dtype, chunk,
                                             lists_arr, flags_arr, world, rank, epoch, _native.stream_of(x))
    _native.check(err)


def merge_wait(lists_ptr, flags_ptr, world, epoch, rows, k, dtype, device, values=None, indices=None):
    """Merge half over peer memory (ckb_topk_merge_wait_launch): waits per row for every rank's list of this epoch
    in this rank's exchange buffer, then (values in dtype, int64 indices) [rows, k]."""
    if dtype not in _DTYPES:
        raise ValueError(f"topk merge: dtype {dtype}")
    values = torch.empty((rows, k), dtype=dtype, device=device) if values is None else values
    indices = torch.empty((rows, k), dtype=torch.int64, device=device) if indices is None else indices
    lib = _native.load("topk")
    with torch.cuda.device(device):
        err = lib.ckb_topk_merge_wait_launch(lists_ptr, flags_ptr, world, epoch, values.data_ptr(),
                                             indices.data_ptr(), rows, k, _DTYPES[dtype],
                                             torch.cuda.current_stream(device).cuda_stream)
    _native.check(err)
    return values, indices
