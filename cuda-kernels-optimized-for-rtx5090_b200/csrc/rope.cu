// Rotary position embedding of q [tokens, q_heads, head_dim] and k [tokens, kv_heads, head_dim], half-split pairing
// (element i with i + h, h = head_dim / 2), full rotary, fp32 math with both products and the sum rounded separately,
// then one round-to-nearest-even conversion to the q/k dtype -- the reference's rotation (rope/kernel.cu:1-8,73-79):
//   out[i]     = x[i]     * cos[i]     - x[i + h] * sin[i]
//   out[i + h] = x[i + h] * cos[i + h] + x[i]     * sin[i + h]
// cos/sin come from a cache [max_position, head_dim] picked by position_ids (the reference's ABI), or, in sincos mode,
// from sincosf(position * inv_freq[i]) in registers with cos[i + h] = cos[i] (the cat(freqs, freqs) cache layout).
// q/k dtypes bf16 (1) and fp16 (2); cache dtypes fp32 (0), bf16 (1), fp16 (2). In place when the output pointers equal
// the inputs (each thread reads its elements before it writes them).
//
// B200 mapping (HBM bound: q and k are streamed once; cos/sin rows are L2/L1 hits): thread (c, r, z) of a block owns
// the 8 pairs 8c..8c+7 of head_dim in heads r, r + R, r + 2R, ... of token blockIdx.x * Z + z, so the cos/sin of its
// pairs are loaded (or computed) once and reused over its heads; up to 5 heads (10 16-byte loads) are in flight per
// thread. head_dim % 16 != 0 or an unaligned pointer falls back to a scalar kernel (one pair per thread).
#include "ckb200_rope.h"
#include "common.cuh"

#include <climits>

namespace ckb {
namespace {

#ifndef CKB_ROPE_HEADS_IN_FLIGHT
#define CKB_ROPE_HEADS_IN_FLIGHT 5
#endif
#ifndef CKB_ROPE_MIN_BLOCKS
#define CKB_ROPE_MIN_BLOCKS 1
#endif
constexpr int kHeadsInFlight = CKB_ROPE_HEADS_IN_FLIGHT;  // heads whose q/k loads one thread keeps in flight

// 8 consecutive cache values as fp32 (i a multiple of 8; the row start 16-byte aligned).
__device__ __forceinline__ void ld8(const float* p, long long i, float (&v)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p + i));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p + i) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void ld8(const __nv_bfloat16* p, long long i, float (&v)[8]) {
  unpack16(__ldg(reinterpret_cast<const uint4*>(p + i)), v, p);
}
__device__ __forceinline__ void ld8(const __half* p, long long i, float (&v)[8]) {
  unpack16(__ldg(reinterpret_cast<const uint4*>(p + i)), v, p);
}

// Offset of head `h` of `token` (q heads first, then k heads) in its tensor.
__device__ __forceinline__ long long head_offset(long long token, int h, int q_heads, int kv_heads, int head_dim) {
  return h < q_heads ? (token * q_heads + h) * head_dim : (token * kv_heads + (h - q_heads)) * head_dim;
}

template <bool kInPlace>
__device__ __forceinline__ uint4 ld_x(const void* p) {
  return kInPlace ? ld_inplace(p) : ld_stream(p);
}

// kCache: cos/sin from the cache (C its dtype); otherwise sincosf(pos * inv_freq[i]).
template <typename T, typename C, bool kCache, bool kInPlace>
__global__ void __launch_bounds__(256, CKB_ROPE_MIN_BLOCKS) rope_tokens(const T* q, const T* k, const C* __restrict__ cos_rows,
                                                const C* __restrict__ sin_rows, const float* __restrict__ inv_freq,
                                                const long long* __restrict__ ids, T* q_out, T* k_out,
                                                long long tokens, int q_heads, int kv_heads, int head_dim) {
  pdl_wait();
  pdl_trigger();
  const long long token = (long long)blockIdx.x * blockDim.z + threadIdx.z;
  if (token >= tokens) return;
  const int half = head_dim >> 1;
  const int c = threadIdx.x * 8;
  const int heads = q_heads + kv_heads;
  const int R = blockDim.y;

  // The first batch of heads is in flight before the position id -> cos/sin chain.
  uint4 ra[kHeadsInFlight], rb[kHeadsInFlight];
  long long off[kHeadsInFlight];
  int h0 = threadIdx.y;
#pragma unroll
  for (int j = 0; j < kHeadsInFlight; ++j) {
    const int h = h0 + j * R;
    off[j] = h < heads ? head_offset(token, h, q_heads, kv_heads, head_dim) + c : 0;
    if (h < heads) {
      const T* xs = h < q_heads ? q : k;
      ra[j] = ld_x<kInPlace>(xs + off[j]);
      rb[j] = ld_x<kInPlace>(xs + off[j] + half);
    }
  }
  const long long pos = __ldg(ids + token);
  float c1[8], s1[8], c2[8], s2[8];
  if constexpr (kCache) {
    const long long row = pos * head_dim;
    ld8(cos_rows, row + c, c1);
    ld8(sin_rows, row + c, s1);
    ld8(cos_rows, row + c + half, c2);
    ld8(sin_rows, row + c + half, s2);
  } else {
    const float p = (float)pos;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      sincosf(p * __ldg(inv_freq + c + j), &s1[j], &c1[j]);
      c2[j] = c1[j];
      s2[j] = s1[j];
    }
  }
  while (true) {
#pragma unroll
    for (int j = 0; j < kHeadsInFlight; ++j) {
      const int h = h0 + j * R;
      if (h < heads) {
        float a[8], b[8];
        unpack16(ra[j], a, q);
        unpack16(rb[j], b, q);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float lo = __fadd_rn(__fmul_rn(a[e], c1[e]), -__fmul_rn(b[e], s1[e]));
          const float hi = __fadd_rn(__fmul_rn(b[e], c2[e]), __fmul_rn(a[e], s2[e]));
          a[e] = lo;
          b[e] = hi;
        }
        T* out = h < q_heads ? q_out : k_out;
        st_stream(out + off[j], pack16(a, q));
        st_stream(out + off[j] + half, pack16(b, q));
      }
    }
    h0 += kHeadsInFlight * R;
    if (h0 >= heads) break;
#pragma unroll
    for (int j = 0; j < kHeadsInFlight; ++j) {
      const int h = h0 + j * R;
      off[j] = h < heads ? head_offset(token, h, q_heads, kv_heads, head_dim) + c : 0;
      if (h < heads) {
        const T* xs = h < q_heads ? q : k;
        ra[j] = ld_x<kInPlace>(xs + off[j]);
        rb[j] = ld_x<kInPlace>(xs + off[j] + half);
      }
    }
  }
}

__device__ __forceinline__ float ld1(const float* p, long long i) { return p[i]; }
__device__ __forceinline__ float ld1(const __nv_bfloat16* p, long long i) { return __bfloat162float(p[i]); }
__device__ __forceinline__ float ld1(const __half* p, long long i) { return __half2float(p[i]); }

// Scalar fallback: block (64, R) per token, thread (i, r) rotates pair i of heads r, r + R, ...
template <typename T, typename C, bool kCache>
__global__ void __launch_bounds__(1024) rope_scalar(const T* q, const T* k, const C* __restrict__ cos_rows,
                                                    const C* __restrict__ sin_rows,
                                                    const float* __restrict__ inv_freq,
                                                    const long long* __restrict__ ids, T* q_out, T* k_out,
                                                    int q_heads, int kv_heads, int head_dim) {
  pdl_wait();
  pdl_trigger();
  const long long token = blockIdx.x;
  const int half = head_dim >> 1;
  const long long pos = ids[token];
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    float c1, s1, c2, s2;
    if constexpr (kCache) {
      c1 = ld1(cos_rows, pos * head_dim + i);
      s1 = ld1(sin_rows, pos * head_dim + i);
      c2 = ld1(cos_rows, pos * head_dim + i + half);
      s2 = ld1(sin_rows, pos * head_dim + i + half);
    } else {
      sincosf((float)pos * inv_freq[i], &s1, &c1);
      c2 = c1;
      s2 = s1;
    }
    for (int h = threadIdx.y; h < q_heads + kv_heads; h += blockDim.y) {
      const long long o = head_offset(token, h, q_heads, kv_heads, head_dim);
      const T* xs = h < q_heads ? q : k;
      T* out = h < q_heads ? q_out : k_out;
      const float a = ld1(xs, o + i), b = ld1(xs, o + i + half);
      out[o + i] = from_f32<T>(__fadd_rn(__fmul_rn(a, c1), -__fmul_rn(b, s1)));
      out[o + i + half] = from_f32<T>(__fadd_rn(__fmul_rn(b, c2), __fmul_rn(a, s2)));
    }
  }
}

struct Args {
  const void *q, *k, *cos_rows, *sin_rows;
  const float* inv_freq;
  const long long* ids;
  void *q_out, *k_out;
  long long tokens;
  int q_heads, kv_heads, head_dim;
};

template <typename T, typename C, bool kCache>
int start(const Args& a, cudaStream_t s) {
  const int heads = a.q_heads + a.kv_heads;
  const int lanes = a.head_dim / 16;
  const bool in_place = a.q_out == a.q || a.k_out == a.k;
  const bool vec = a.head_dim % 16 == 0 && lanes <= 256 && aligned16(a.q) && aligned16(a.k) &&
                   aligned16(a.q_out) && aligned16(a.k_out) &&
                   (kCache ? aligned16(a.cos_rows) && aligned16(a.sin_rows) : aligned16(a.inv_freq));
  if (vec) {
    int r = (heads + kHeadsInFlight - 1) / kHeadsInFlight;
    if (r * lanes > 256) r = 256 / lanes;
    int z = 256 / (r * lanes);
    if (z < 1) z = 1;
    if (z > 64) z = 64;
    const long long grid = (a.tokens + z - 1) / z;
    if (grid > INT_MAX) return -1;
    const dim3 block(lanes, r, z);
    if (in_place) {
      launch_pdl(rope_tokens<T, C, kCache, true>, dim3((unsigned)grid), block, 0, s, (const T*)a.q, (const T*)a.k,
                 (const C*)a.cos_rows, (const C*)a.sin_rows, a.inv_freq, a.ids, (T*)a.q_out, (T*)a.k_out, a.tokens,
                 a.q_heads, a.kv_heads, a.head_dim);
    } else {
      launch_pdl(rope_tokens<T, C, kCache, false>, dim3((unsigned)grid), block, 0, s, (const T*)a.q, (const T*)a.k,
                 (const C*)a.cos_rows, (const C*)a.sin_rows, a.inv_freq, a.ids, (T*)a.q_out, (T*)a.k_out, a.tokens,
                 a.q_heads, a.kv_heads, a.head_dim);
    }
  } else {
    if (a.tokens > INT_MAX) return -1;
    const dim3 block(64, heads < 16 ? heads : 16);
    launch_pdl(rope_scalar<T, C, kCache>, dim3((unsigned)a.tokens), block, 0, s, (const T*)a.q, (const T*)a.k,
               (const C*)a.cos_rows, (const C*)a.sin_rows, a.inv_freq, a.ids, (T*)a.q_out, (T*)a.k_out, a.q_heads,
               a.kv_heads, a.head_dim);
  }
  return (int)cudaGetLastError();
}

template <typename T>
int start_cache(int cache_dtype, const Args& a, cudaStream_t s) {
  switch (cache_dtype) {
    case kF32: return start<T, float, true>(a, s);
    case kBF16: return start<T, __nv_bfloat16, true>(a, s);
    case kF16: return start<T, __half, true>(a, s);
    default: return -1;
  }
}

// ------------------------------------------------------------------------------ RoPE fused with the KV-cache write ---
// q [tokens, q_heads, D] and k [tokens, kv_heads, D] are rotated as above; the rotated k and the (unrotated) v
// [tokens, kv_heads, D] of token t are also stored into a paged cache at slot s = slots[t]: key_cache / value_cache
// [num_blocks, block_size, kv_heads, D], slot s = block * block_size + offset, so its row starts at s * kv_heads * D
// (a negative slot, a padding token, writes no cache row). k_out may be null (the rotated k goes to the cache only).
// Thread mapping as rope_tokens over q_heads + 2 kv_heads "heads" (q, then k, then v): every element is read once and
// written once or twice, with no second kernel re-reading k and v to fill the cache.
template <typename T, typename C, bool kInPlace>
__global__ void __launch_bounds__(256) rope_kv_tokens(const T* q, const T* k, const T* __restrict__ v,
                                                      const C* __restrict__ cos_rows, const C* __restrict__ sin_rows,
                                                      const long long* __restrict__ ids,
                                                      const long long* __restrict__ slots, T* q_out, T* k_out,
                                                      T* __restrict__ key_cache, T* __restrict__ value_cache,
                                                      long long tokens, int q_heads, int kv_heads, int head_dim) {
  pdl_wait();
  pdl_trigger();
  const long long token = (long long)blockIdx.x * blockDim.z + threadIdx.z;
  if (token >= tokens) return;
  const int half = head_dim >> 1;
  const int c = threadIdx.x * 8;
  const int heads = q_heads + 2 * kv_heads;
  const int R = blockDim.y;
  const long long slot = __ldg(slots + token);
  const long long pos = __ldg(ids + token);
  float c1[8], s1[8], c2[8], s2[8];
  ld8(cos_rows, pos * head_dim + c, c1);
  ld8(sin_rows, pos * head_dim + c, s1);
  ld8(cos_rows, pos * head_dim + c + half, c2);
  ld8(sin_rows, pos * head_dim + c + half, s2);
  for (int h0 = threadIdx.y; h0 < heads; h0 += kHeadsInFlight * R) {
    uint4 ra[kHeadsInFlight], rb[kHeadsInFlight];
#pragma unroll
    for (int j = 0; j < kHeadsInFlight; ++j) {  // every load of the group before any use
      const int h = h0 + j * R;
      if (h < q_heads) {
        const T* p = q + (token * q_heads + h) * head_dim + c;
        ra[j] = ld_x<kInPlace>(p);
        rb[j] = ld_x<kInPlace>(p + half);
      } else if (h < q_heads + kv_heads) {
        const T* p = k + (token * kv_heads + (h - q_heads)) * head_dim + c;
        ra[j] = ld_x<kInPlace>(p);
        rb[j] = ld_x<kInPlace>(p + half);
      } else if (h < heads) {
        const T* p = v + (token * kv_heads + (h - q_heads - kv_heads)) * head_dim + c;
        ra[j] = ld_stream(p);
        rb[j] = ld_stream(p + half);
      }
    }
#pragma unroll
    for (int j = 0; j < kHeadsInFlight; ++j) {
      const int h = h0 + j * R;
      if (h >= heads) continue;
      if (h >= q_heads + kv_heads) {  // v: straight into its cache row
        if (slot >= 0) {
          T* dst = value_cache + (slot * kv_heads + (h - q_heads - kv_heads)) * head_dim + c;
          st_stream(dst, ra[j]);
          st_stream(dst + half, rb[j]);
        }
        continue;
      }
      float a[8], b[8];
      unpack16(ra[j], a, q);
      unpack16(rb[j], b, q);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float lo = __fadd_rn(__fmul_rn(a[e], c1[e]), -__fmul_rn(b[e], s1[e]));
        const float hi = __fadd_rn(__fmul_rn(b[e], c2[e]), __fmul_rn(a[e], s2[e]));
        a[e] = lo;
        b[e] = hi;
      }
      const uint4 pa = pack16(a, q), pb = pack16(b, q);
      if (h < q_heads) {
        T* dst = q_out + (token * q_heads + h) * head_dim + c;
        st_stream(dst, pa);
        st_stream(dst + half, pb);
      } else {
        const int hk = h - q_heads;
        if (k_out != nullptr) {
          T* dst = k_out + (token * kv_heads + hk) * head_dim + c;
          st_stream(dst, pa);
          st_stream(dst + half, pb);
        }
        if (slot >= 0) {
          T* dst = key_cache + (slot * kv_heads + hk) * head_dim + c;
          st_stream(dst, pa);
          st_stream(dst + half, pb);
        }
      }
    }
  }
}

// Scalar form of rope_kv_tokens for any head_dim and alignment: block (64, R) per token.
template <typename T, typename C>
__global__ void __launch_bounds__(1024) rope_kv_scalar(const T* q, const T* k, const T* __restrict__ v,
                                                       const C* __restrict__ cos_rows, const C* __restrict__ sin_rows,
                                                       const long long* __restrict__ ids,
                                                       const long long* __restrict__ slots, T* q_out, T* k_out,
                                                       T* __restrict__ key_cache, T* __restrict__ value_cache,
                                                       int q_heads, int kv_heads, int head_dim) {
  pdl_wait();
  pdl_trigger();
  const long long token = blockIdx.x;
  const int half = head_dim >> 1;
  const long long pos = ids[token], slot = slots[token];
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const float c1 = ld1(cos_rows, pos * head_dim + i), s1 = ld1(sin_rows, pos * head_dim + i);
    const float c2 = ld1(cos_rows, pos * head_dim + i + half), s2 = ld1(sin_rows, pos * head_dim + i + half);
    for (int h = threadIdx.y; h < q_heads + 2 * kv_heads; h += blockDim.y) {
      if (h >= q_heads + kv_heads) {
        if (slot >= 0) {
          const int hv = h - q_heads - kv_heads;
          value_cache[(slot * kv_heads + hv) * head_dim + i] = v[(token * kv_heads + hv) * head_dim + i];
          value_cache[(slot * kv_heads + hv) * head_dim + i + half] = v[(token * kv_heads + hv) * head_dim + i + half];
        }
        continue;
      }
      const bool isq = h < q_heads;
      const int hh = isq ? h : h - q_heads;
      const long long o = (token * (isq ? q_heads : kv_heads) + hh) * head_dim;
      const T* xs = isq ? q : k;
      const float a = ld1(xs, o + i), b = ld1(xs, o + i + half);
      const T lo = from_f32<T>(__fadd_rn(__fmul_rn(a, c1), -__fmul_rn(b, s1)));
      const T hi = from_f32<T>(__fadd_rn(__fmul_rn(b, c2), __fmul_rn(a, s2)));
      if (isq) {
        q_out[o + i] = lo;
        q_out[o + i + half] = hi;
      } else {
        if (k_out != nullptr) {
          k_out[o + i] = lo;
          k_out[o + i + half] = hi;
        }
        if (slot >= 0) {
          key_cache[(slot * kv_heads + hh) * head_dim + i] = lo;
          key_cache[(slot * kv_heads + hh) * head_dim + i + half] = hi;
        }
      }
    }
  }
}

struct KvArgs {
  const void *q, *k, *v, *cos_rows, *sin_rows;
  const long long *ids, *slots;
  void *q_out, *k_out, *key_cache, *value_cache;
  long long tokens;
  int q_heads, kv_heads, head_dim;
};

template <typename T, typename C>
int start_kv(const KvArgs& a, cudaStream_t s) {
  const int heads = a.q_heads + 2 * a.kv_heads;
  const int lanes = a.head_dim / 16;
  const bool in_place = a.q_out == a.q || a.k_out == a.k;
  const bool vec = a.head_dim % 16 == 0 && lanes <= 256 && aligned16(a.q) && aligned16(a.k) && aligned16(a.v) &&
                   aligned16(a.q_out) && aligned16(a.k_out) && aligned16(a.key_cache) &&
                   aligned16(a.value_cache) && aligned16(a.cos_rows) && aligned16(a.sin_rows);
  if (vec) {
    int r = (heads + kHeadsInFlight - 1) / kHeadsInFlight;
    if (r * lanes > 256) r = 256 / lanes;
    int z = 256 / (r * lanes);
    if (z < 1) z = 1;
    if (z > 64) z = 64;
    const long long grid = (a.tokens + z - 1) / z;
    if (grid > INT_MAX) return -1;
    const dim3 block(lanes, r, z);
    if (in_place)
      launch_pdl(rope_kv_tokens<T, C, true>, dim3((unsigned)grid), block, 0, s, (const T*)a.q, (const T*)a.k,
                 (const T*)a.v, (const C*)a.cos_rows, (const C*)a.sin_rows, a.ids, a.slots, (T*)a.q_out,
                 (T*)a.k_out, (T*)a.key_cache, (T*)a.value_cache, a.tokens, a.q_heads, a.kv_heads, a.head_dim);
    else
      launch_pdl(rope_kv_tokens<T, C, false>, dim3((unsigned)grid), block, 0, s, (const T*)a.q, (const T*)a.k,
                 (const T*)a.v, (const C*)a.cos_rows, (const C*)a.sin_rows, a.ids, a.slots, (T*)a.q_out,
                 (T*)a.k_out, (T*)a.key_cache, (T*)a.value_cache, a.tokens, a.q_heads, a.kv_heads, a.head_dim);
  } else {
    if (a.tokens > INT_MAX) return -1;
    const dim3 block(64, heads < 16 ? heads : 16);
    launch_pdl(rope_kv_scalar<T, C>, dim3((unsigned)a.tokens), block, 0, s, (const T*)a.q, (const T*)a.k,
               (const T*)a.v, (const C*)a.cos_rows, (const C*)a.sin_rows, a.ids, a.slots, (T*)a.q_out, (T*)a.k_out,
               (T*)a.key_cache, (T*)a.value_cache, a.q_heads, a.kv_heads, a.head_dim);
  }
  return (int)cudaGetLastError();
}

template <typename T>
int start_kv_cache(int cache_dtype, const KvArgs& a, cudaStream_t s) {
  switch (cache_dtype) {
    case kF32: return start_kv<T, float>(a, s);
    case kBF16: return start_kv<T, __nv_bfloat16>(a, s);
    case kF16: return start_kv<T, __half>(a, s);
    default: return -1;
  }
}

bool bad_shape(long long tokens, int q_heads, int kv_heads, int head_dim) {
  return tokens > INT_MAX || head_dim <= 0 || head_dim % 2 || q_heads <= 0 || kv_heads <= 0 ||
         (long long)q_heads + kv_heads > INT_MAX;
}

}  // namespace
}  // namespace ckb

using namespace ckb;

// Replaces the reference's rope `launch` (rope/kernel.cu:201-215): same arguments, checks and return codes. `rows` and
// `splits` are the reference's block-shape knobs, validated as there but not needed by the B200 dispatcher. Passing
// q_out == q and k_out == k rotates in place.
CKB_EXPORT int launch(const void* q, const void* k, const void* cos_rows, const void* sin_rows, const void* ids,
                      void* q_out, void* k_out, long long tokens, int q_heads, int kv_heads, int head_dim,
                      int qk_dtype, int cache_dtype, int rows, int splits, cudaStream_t stream) {
  if (tokens <= 0) return 0;
  if (bad_shape(tokens, q_heads, kv_heads, head_dim) || rows < 1 || splits < 1 || splits > 65535) return -1;
  const Args a{q, k, cos_rows, sin_rows, nullptr, (const long long*)ids, q_out, k_out, tokens, q_heads, kv_heads,
               head_dim};
  if (qk_dtype == kBF16) return start_cache<__nv_bfloat16>(cache_dtype, a, stream);
  if (qk_dtype == kF16) return start_cache<__half>(cache_dtype, a, stream);
  return -1;
}

// RoPE with cos/sin computed in registers (no counterpart in the reference's ABI): angle_i = float(position) *
// inv_freq[i] for i < head_dim / 2, cos/sin by sincosf, the same rotation and rounding as `launch`. inv_freq is fp32
// [head_dim / 2] on the device (the caller computes it, e.g. 1 / theta^(2i / head_dim)). In place when q_out == q and
// k_out == k.
CKB_EXPORT int ckb_rope_sincos_launch(const void* q, const void* k, const float* inv_freq, const long long* ids,
                                      void* q_out, void* k_out, long long tokens, int q_heads, int kv_heads,
                                      int head_dim, int qk_dtype, cudaStream_t stream) {
  if (tokens <= 0) return 0;
  if (bad_shape(tokens, q_heads, kv_heads, head_dim) || inv_freq == nullptr) return -1;
  const Args a{q, k, nullptr, nullptr, inv_freq, ids, q_out, k_out, tokens, q_heads, kv_heads, head_dim};
  if (qk_dtype == kBF16) return start<__nv_bfloat16, float, false>(a, stream);
  if (qk_dtype == kF16) return start<__half, float, false>(a, stream);
  return -1;
}

// RoPE fused with the paged KV-cache write (no counterpart in the reference, which rotates q and k only,
// rope/kernel.cu:1-13): q and k rotated as launch() does (q_out == q rotates q in place; k_out == k rotates k in
// place, k_out null leaves k untouched), and for each token t with slots[t] >= 0 the rotated k and the unrotated v
// [tokens, kv_heads, head_dim] stored into key_cache / value_cache [num_blocks, block_size, kv_heads, head_dim] at
// row slots[t] (= block * block_size + offset). Caches have the q/k dtype. Returns 0, -1 for a rejected argument, or
// the launch's cudaError_t.
CKB_EXPORT int ckb_rope_kv_cache_launch(const void* q, const void* k, const void* v, const void* cos_rows,
                                        const void* sin_rows, const void* ids, const void* slots, void* q_out,
                                        void* k_out, void* key_cache, void* value_cache, long long tokens,
                                        int q_heads, int kv_heads, int head_dim, int qk_dtype, int cache_dtype,
                                        cudaStream_t stream) {
  if (tokens <= 0) return 0;
  if (bad_shape(tokens, q_heads, kv_heads, head_dim) || v == nullptr || slots == nullptr || key_cache == nullptr ||
      value_cache == nullptr || ids == nullptr || cos_rows == nullptr || sin_rows == nullptr || q_out == nullptr)
    return -1;
  const KvArgs a{q, k, v, cos_rows, sin_rows, (const long long*)ids, (const long long*)slots, q_out, k_out,
                 key_cache, value_cache, tokens, q_heads, kv_heads, head_dim};
  if (qk_dtype == kBF16) return start_kv_cache<__nv_bfloat16>(cache_dtype, a, stream);
  if (qk_dtype == kF16) return start_kv_cache<__half>(cache_dtype, a, stream);
  return -1;
}
