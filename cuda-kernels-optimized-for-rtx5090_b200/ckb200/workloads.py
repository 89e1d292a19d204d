"""Seeded synthetic inputs of the benchmark configurations (CPU tensors; move them to the device to use them).

The reference measures no public dataset; these stand in for its workloads with the stated shapes, dtypes and value
distributions (the softmax shape 4096 x 8192 is the reference's s4096x8192 workload, softmax/README.md:8):
  softmax_4096x8192    fp32 [4096, 8192] ~ N(0, 2^2), seed 0
  rmsnorm_16384x4096   bf16 x [16384, 4096] ~ N(0, 1), weight [4096] ~ N(1, 0.1^2) (bf16), eps 1e-6, seed 1
  rope_8x4096          bf16 q [8, 4096, 32, 128], k [8, 4096, 8, 128] ~ N(0, 1), positions 0..4095 per batch,
                       theta 1e4, fp32 cos/sin cache [4096, 128], seed 2 (integer=True: values in [-8, 8])
  softmax_256x262144   fp32 [256, 262144] ~ N(0, 4^2) plus +20 at one seeded column per row, seed 3
  softmax_262144x128   fp32 [262144, 128] ~ N(0, 1), seed 3
  topk_512x151936      fp32 [512, 151936] ~ N(0, 3^2), k = 50, seed 4
Each generator takes a `scale` that divides the row count (rows never below 1) for smaller runs.
"""

import torch


def _gen(seed):
    return torch.Generator().manual_seed(seed)


def softmax_4096x8192(scale=1):
    g = _gen(0)
    return {"x": torch.randn(max(1, 4096 // scale), 8192, generator=g) * 2.0}


def rmsnorm_16384x4096(scale=1, weight_dtype=torch.bfloat16):
    g = _gen(1)
    x = torch.randn(max(1, 16384 // scale), 4096, generator=g).to(torch.bfloat16)
    w = (1.0 + 0.1 * torch.randn(4096, generator=g)).to(weight_dtype)
    return {"x": x, "weight": w}


def rope_8x4096(scale=1, integer=False, cache_dtype=torch.float32, batch=8, seq=4096):
    from_cache = _rope_cache(10000.0, 128, 4096, cache_dtype)
    g = _gen(2)
    b = max(1, batch // scale)
    if integer:
        q = torch.randint(-8, 9, (b, seq, 32, 128), generator=g).to(torch.bfloat16)
        k = torch.randint(-8, 9, (b, seq, 8, 128), generator=g).to(torch.bfloat16)
    else:
        q = torch.randn(b, seq, 32, 128, generator=g).to(torch.bfloat16)
        k = torch.randn(b, seq, 8, 128, generator=g).to(torch.bfloat16)
    ids = torch.arange(seq, dtype=torch.int64).repeat(b, 1)
    return {"q": q, "k": k, "cos": from_cache[0], "sin": from_cache[1], "position_ids": ids, "theta": 10000.0}


def softmax_256x262144(scale=1):
    g = _gen(3)
    rows = max(1, 256 // scale)
    x = torch.randn(rows, 262144, generator=g) * 4.0
    spike = torch.randint(0, 262144, (rows,), generator=g)
    x[torch.arange(rows), spike] += 20.0
    return {"x": x}


def softmax_262144x128(scale=1):
    g = _gen(3)
    return {"x": torch.randn(max(1, 262144 // scale), 128, generator=g)}


def topk_512x151936(scale=1):
    g = _gen(4)
    return {"x": torch.randn(max(1, 512 // scale), 151936, generator=g) * 3.0}


def _rope_cache(theta, head_dim, max_position, dtype):
    """The usual rotary cache builder: inv_freq = 1 / theta^(arange(0, D, 2) / D) (fp32), freqs = positions x
    inv_freq (fp32), emb = cat(freqs, freqs), cos/sin in fp32, cast to dtype."""
    inv_freq = 1.0 / (float(theta) ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    t = torch.arange(max_position, dtype=torch.int64).float()
    emb = torch.cat([torch.outer(t, inv_freq)] * 2, dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


# Algorithmic HBM bytes of one call at the full configuration (read + write each element once; RoPE in place over
# q and k, plus the cos/sin rows it reads; top-k reads x and writes values + indices).
ALGORITHMIC_BYTES = {
    "softmax_4096x8192": 2 * 4096 * 8192 * 4,
    "rmsnorm_16384x4096": 2 * 16384 * 4096 * 2 + 4096 * 2,
    "rope_8x4096": 2 * (8 * 4096 * 32 * 128 + 8 * 4096 * 8 * 128) * 2 + 2 * 4096 * 128 * 4 + 8 * 4096 * 8,
    "softmax_256x262144": 2 * 256 * 262144 * 4,
    "softmax_262144x128": 2 * 262144 * 128 * 4,
    "topk_512x151936": 512 * 151936 * 4 + 512 * 50 * (4 + 8),
}

ROWS = {
    "softmax_4096x8192": 4096,
    "rmsnorm_16384x4096": 16384,
    "rope_8x4096": 8 * 4096,
    "softmax_256x262144": 256,
    "softmax_262144x128": 262144,
    "topk_512x151936": 512,
}
