"""The two fusions with the neighbouring steps, against the oracle:
  * RoPE fused with the paged KV-cache write (ckb_rope_kv_cache_launch): rotated q (and k), and the cache rows of
    every non-padding token, bit for bit; cache rows no token maps to stay as they were;
  * top-k sampling (ckb_topk_softmax_launch): indices bit-exact, probabilities (the softmax over the k largest
    logits / temperature) within 1e-6 relative of fp64, and the sampled token equal to the oracle's wherever the
    uniform is not within 1e-5 of a cumulative boundary (fp32 rounding could legitimately move it there).
"""

import pytest
import torch

from ckb200 import rope, topk, workloads
from helpers import assert_rel
from oracle import rope as orope
from oracle import topk as otk

pytestmark = pytest.mark.gpu


def _bits(t):
    return t.detach().cpu().contiguous().view(torch.int16)


@pytest.mark.parametrize("inplace,write_k", [(True, True), (False, True), (False, False)])
@pytest.mark.parametrize("qk_dtype,cache_dtype,head_dim", [(torch.bfloat16, torch.float32, 128),
                                                           (torch.float16, torch.bfloat16, 64),
                                                           (torch.bfloat16, torch.float32, 40)])
def test_rope_kv_cache_matches_the_oracle(inplace, write_k, qk_dtype, cache_dtype, head_dim):
    g = torch.Generator().manual_seed(head_dim)
    batch, seq, hq, hkv, blocks, block_size = 3, 37, 8, 2, 16, 16
    q = torch.randn(batch, seq, hq, head_dim, generator=g).to(qk_dtype)
    k = torch.randn(batch, seq, hkv, head_dim, generator=g).to(qk_dtype)
    v = torch.randn(batch, seq, hkv, head_dim, generator=g).to(qk_dtype)
    cos, sin = orope.cos_sin_cache(10000.0, head_dim, 4096, cache_dtype)
    ids = torch.randint(0, 4096, (batch, seq), generator=g)
    slots = torch.randperm(blocks * block_size, generator=g)[:batch * seq].view(batch, seq)
    slots[0, :5] = -1  # padding tokens write no cache row
    kc0 = torch.randn(blocks, block_size, hkv, head_dim, generator=g).to(qk_dtype)
    vc0 = torch.randn(blocks, block_size, hkv, head_dim, generator=g).to(qk_dtype)
    wq, wk, wkc, wvc = orope.rope_kv_cache(q, k, v, cos, sin, ids, kc0, vc0, slots)

    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    kc, vc = kc0.cuda(), vc0.cuda()
    q_out, k_out = rope.rope_kv_cache(qd, kd, vd, ids.cuda(), cos.cuda(), sin.cuda(), kc, vc, slots.cuda(),
                                      inplace=inplace, write_k=write_k)
    torch.cuda.synchronize()
    assert torch.equal(_bits(q_out), _bits(wq)), "q"
    assert torch.equal(_bits(kc), _bits(wkc)), "key cache"
    assert torch.equal(_bits(vc), _bits(wvc)), "value cache"
    if write_k:
        assert torch.equal(_bits(k_out), _bits(wk)), "k"
    else:
        assert k_out is None and torch.equal(_bits(kd), _bits(k)), "k left untouched"
    if not inplace:
        assert torch.equal(_bits(qd), _bits(q)), "q input left untouched"


def test_rope_kv_cache_decode_batch_equals_rope_then_scatter():
    """Decode-shaped (64 sequences, one token each) on the BASELINE RoPE model shape: the fused kernel equals the
    unfused path (this library's RoPE, then the rows copied into the cache by indexing)."""
    g = torch.Generator().manual_seed(7)
    base = workloads.rope_8x4096(scale=1, batch=64, seq=1)
    q, k = base["q"].cuda(), base["k"].cuda()
    v = torch.randn(64, 1, 8, 128, generator=g).to(torch.bfloat16).cuda()
    ids = torch.randint(0, 4096, (64, 1), generator=g).cuda()
    slots = torch.randperm(4096, generator=g)[:64].view(64, 1).cuda()
    kc = torch.zeros(256, 16, 8, 128, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    cos, sin = base["cos"].cuda(), base["sin"].cuda()
    q_f, k_f = rope.rope_kv_cache(q.clone(), k.clone(), v, ids, cos, sin, kc, vc, slots)
    q_u, k_u = rope.rope(q.clone(), k.clone(), ids, cos, sin)
    kc_u, vc_u = torch.zeros_like(kc), torch.zeros_like(vc)
    kc_u.view(-1, 8, 128)[slots.view(-1)] = k_u.view(-1, 8, 128)
    vc_u.view(-1, 8, 128)[slots.view(-1)] = v.view(-1, 8, 128)
    torch.cuda.synchronize()
    assert torch.equal(_bits(q_f), _bits(q_u)) and torch.equal(_bits(k_f), _bits(k_u))
    assert torch.equal(_bits(kc), _bits(kc_u)) and torch.equal(_bits(vc), _bits(vc_u))


@pytest.mark.parametrize("rows,cols,k,dtype", [(64, 50000, 50, torch.float32), (64, 50000, 50, torch.bfloat16),
                                               (512, 32000, 1, torch.float32), (8, 20000, 300, torch.float32),
                                               (1, 128256, 50, torch.float32)])
def test_topk_softmax_matches_the_oracle(rows, cols, k, dtype):
    g = torch.Generator().manual_seed(rows * 7 + k)
    x = (torch.randn(rows, cols, generator=g) * 3).to(dtype)
    u = torch.rand(rows, generator=g)
    probs, idx, samples = topk.topk_softmax(x.cuda(), k, temperature=0.7, uniforms=u.cuda())
    wp, wi, ws, margin = otk.topk_softmax(x, k, temperature=0.7, uniforms=u)
    assert torch.equal(idx.cpu(), wi), "indices"
    assert_rel(probs, wp, 1e-6, "probabilities")
    clear = margin > 1e-5
    assert clear.sum() > 0
    assert torch.equal(samples.cpu()[clear], ws[clear]), "sampled tokens"
    assert torch.isin(samples.cpu(), wi).all() if rows == 1 else True


def test_topk_softmax_without_uniforms_and_rejections():
    x = torch.randn(16, 4096, generator=torch.Generator().manual_seed(3)).cuda()
    probs, idx, samples = topk.topk_softmax(x, 50)
    assert samples is None
    torch.testing.assert_close(probs.sum(-1), torch.ones(16, device="cuda"), rtol=1e-6, atol=1e-6)
    with pytest.raises(ValueError, match="temperature"):
        topk.topk_softmax(x, 50, temperature=0.0)
