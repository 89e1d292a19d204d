// Row-wise top-k (largest k, sorted descending, ties broken by the lower index) of x[rows, cols], fp32 (dtype 0) or
// bf16 (dtype 1), values bit-exact in x's dtype and int64 indices -- the reference's output contract
// (topk/kernel.cu:1-3,436-441, topk/candidate.py:66-81).
//
// Order. Every element becomes a distinct 64-bit composite (order-preserving key of its float bits << 32 | ~index),
// the same total order as the reference's pack() (topk/kernel.cu:56-60): larger value first, equal values by lower
// index, NaN above +inf, -NaN below -inf. The top k of a row are its k largest composites.
//
// Algorithm (one CTA per chunk of a row, 512 threads):
//   1. the chunk is pulled into shared memory by bulk copies (cp.async.bulk, several pieces on their own mbarriers);
//   2. a lower bound: each thread keeps the max of its numbers (one fmax per element as the pieces land); the k-th
//      largest of those maxima has at least k elements at or above it, so the lower edge of its bin in a 2048-bin
//      histogram of the maxima's top 11 key bits (found by a block suffix scan) bounds the chunk's k-th largest key
//      from below;
//   3. one pass collects the composites at or above that edge (typically k + a few dozen): a float compare per
//      element, and the composite only for the few that pass, appended by each warp into its own slots of the
//      candidate buffer (a warp prefix sum places them; no shared atomics). If a warp's slots overflow (heavy ties),
//      a radix select over the composites narrows the edge first: the digit bin holding the k-th largest, refined
//      digit by digit (11/11/10 bits of the key, 11/11/10 of the index, so value ties resolve by index) until the
//      composites at or above it fit the 1024-entry buffer;
//   4. a block rank count (several lanes per candidate) leaves the chunk's top k sorted;
//   5. a row split over several chunks writes each chunk's sorted top k to the workspace; the row's last CTA to finish
//      (per-row counter, reset by that CTA) merges the sorted lists by rank (binary search of every candidate in the
//      other lists) and decodes values and indices from the composites (x is not read again).
// The vocab-sharded variant runs steps 1-5 on a column shard with a global column offset and stops at the sorted
// composites; after an all-gather across GPUs the merge kernel ranks the per-GPU lists the same way.
#include "ckb200_topk.h"
#include "common.cuh"

#include <math_constants.h>

#include <climits>

namespace ckb {

__device__ unsigned int g_topk_status = 0u;

namespace {

typedef unsigned long long u64;

#ifndef CKB_TOPK_THREADS
#define CKB_TOPK_THREADS 512
#endif
constexpr int kThreads = CKB_TOPK_THREADS;
constexpr int kWarps = kThreads / 32;
constexpr int kBins = 2048;            // largest digit: 11 bits
constexpr int kCap = 1024;             // candidate buffer (aliases the histogram)
constexpr int kWarpSlots = kCap / kWarps;  // each warp appends into its own slice of the candidate buffer
constexpr int kMaxK = 512;
constexpr int kPieces = 4;
constexpr int kLevels = 6;
#ifndef CKB_TOPK_CHUNK_BYTES
#define CKB_TOPK_CHUNK_BYTES (96 * 1024)
#endif
constexpr int kChunkBytes = CKB_TOPK_CHUNK_BYTES;  // staged bytes per CTA: chunk + histogram keep 2 CTAs per SM
constexpr int kMaxDataBytes = 160 * 1024;

// Radix digits over the 64-bit composite, most significant first: 11/11/10 bits of the key, then 11/11/10 of ~index.
__device__ __forceinline__ int level_shift(int L) {
  return L == 0 ? 53 : L == 1 ? 42 : L == 2 ? 32 : L == 3 ? 21 : L == 4 ? 10 : 0;
}
__device__ __forceinline__ int level_width(int L) { return (L == 2 || L == 5) ? 10 : 11; }

__device__ __forceinline__ unsigned order_key(unsigned bits) {
  return (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
}
__device__ __forceinline__ unsigned key_bits(unsigned key) {  // inverse of order_key
  return (key & 0x80000000u) ? (key & 0x7fffffffu) : ~key;
}
__device__ __forceinline__ u64 composite(unsigned key, unsigned idx) { return ((u64)key << 32) | (u64)(~idx); }

// Keys of the elements in one 16-byte vector of staged data.
__device__ __forceinline__ void keys16(const uint4& r, unsigned (&k)[4], const float*) {
  k[0] = order_key(r.x); k[1] = order_key(r.y); k[2] = order_key(r.z); k[3] = order_key(r.w);
}
__device__ __forceinline__ void keys16(const uint4& r, unsigned (&k)[8], const __nv_bfloat16*) {
  const unsigned w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    k[2 * j] = order_key(w[j] << 16);
    k[2 * j + 1] = order_key(w[j] & 0xffff0000u);
  }
}

// The largest non-NaN value of one staged 16-byte vector folded into a running max (NaN inputs are skipped, so a
// running max that is still NaN has seen no number).
// Three-input max of sm_100 (max.f32 with three sources): NaN operands are skipped. max3_nan propagates NaN.
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float max3_nan(float a, float b, float c) {
  float d;
  asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ unsigned max_bf16x2(unsigned a, unsigned b) {
  unsigned d;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ unsigned max_nan_bf16x2(unsigned a, unsigned b) {
  unsigned d;
  asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ float vec_max(const uint4& r, float m, const float*) {
  return max3(max3(m, __uint_as_float(r.x), __uint_as_float(r.y)), __uint_as_float(r.z), __uint_as_float(r.w));
}
__device__ __forceinline__ float vec_max(const uint4& r, float m, const __nv_bfloat16*) {
  const unsigned c = max_bf16x2(max_bf16x2(r.x, r.y), max_bf16x2(r.z, r.w));
  return max3(m, __uint_as_float(c << 16), __uint_as_float(c & 0xffff0000u));
}

// The largest value of one staged vector with NaN propagating (so a NaN element never hides behind the pre-filter).
__device__ __forceinline__ float vec_max_nan(const uint4& r, const float*) {
  return max3_nan(max3_nan(__uint_as_float(r.x), __uint_as_float(r.y), __uint_as_float(r.z)), __uint_as_float(r.w),
                  __uint_as_float(r.w));
}
__device__ __forceinline__ float vec_max_nan(const uint4& r, const __nv_bfloat16*) {
  const unsigned c = max_nan_bf16x2(max_nan_bf16x2(r.x, r.y), max_nan_bf16x2(r.z, r.w));
  const float lo = __uint_as_float(c << 16), hi = __uint_as_float(c & 0xffff0000u);
  return max3_nan(lo, hi, hi);
}

// The fp32 bits of element e of one staged vector (a bf16 element widened).
__device__ __forceinline__ unsigned word_of(const uint4& r, int j) {
  return j < 2 ? (j == 0 ? r.x : r.y) : (j == 2 ? r.z : r.w);
}
__device__ __forceinline__ unsigned elem_bits(const uint4& r, int e, const float*) { return word_of(r, e); }
__device__ __forceinline__ unsigned elem_bits(const uint4& r, int e, const __nv_bfloat16*) {
  const unsigned w = word_of(r, e >> 1);
  return (e & 1) ? (w & 0xffff0000u) : (w << 16);
}

// Bit mask (bit e) of the elements of one staged vector that are not below f_lo as floats, NaN included: a superset
// of the elements whose order key is >= the key of f_lo.
__device__ __forceinline__ unsigned vec_not_below(const uint4& r, float f_lo, const float*) {
  return (unsigned)!(__uint_as_float(r.x) < f_lo) | ((unsigned)!(__uint_as_float(r.y) < f_lo) << 1) |
         ((unsigned)!(__uint_as_float(r.z) < f_lo) << 2) | ((unsigned)!(__uint_as_float(r.w) < f_lo) << 3);
}
__device__ __forceinline__ unsigned vec_not_below(const uint4& r, float f_lo, const __nv_bfloat16*) {
  const unsigned w[4] = {r.x, r.y, r.z, r.w};
  unsigned m = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    m |= (unsigned)!(__uint_as_float(w[j] << 16) < f_lo) << (2 * j);
    m |= (unsigned)!(__uint_as_float(w[j] & 0xffff0000u) < f_lo) << (2 * j + 1);
  }
  return m;
}

template <typename T>
__device__ __forceinline__ T decode_value(u64 c);
template <>
__device__ __forceinline__ float decode_value<float>(u64 c) { return __uint_as_float(key_bits((unsigned)(c >> 32))); }
template <>
__device__ __forceinline__ __nv_bfloat16 decode_value<__nv_bfloat16>(u64 c) {
  return __ushort_as_bfloat16((unsigned short)(key_bits((unsigned)(c >> 32)) >> 16));
}
__device__ __forceinline__ long long decode_index(u64 c) { return (long long)(~(unsigned)c); }

// Number of entries greater than c in a descending list of n composites.
__device__ __forceinline__ int count_greater(const u64* list, int n, u64 c) {
  int lo = 0, hi = n;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (list[mid] > c) lo = mid + 1;
    else hi = mid;
  }
  return lo;
}

// Sum of v over the threads with a higher threadIdx.x (all threads call it; two barriers).
__device__ __forceinline__ unsigned block_suffix_excl(unsigned v, unsigned* warp_tot) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned y = __shfl_down_sync(0xffffffffu, x, o);
    if (lane + o < 32) x += y;
  }
  if (lane == 0) warp_tot[warp] = x;
  __syncthreads();
  // The warps' totals, suffix-summed across lanes: lane l holds the sum over warps >= l.
  unsigned t = lane < kWarps ? warp_tot[lane] : 0u;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned y = __shfl_down_sync(0xffffffffu, t, o);
    if (lane + o < 32) t += y;
  }
  const unsigned higher = __shfl_sync(0xffffffffu, t, (warp + 1) & 31) * (warp + 1 < 32 ? 1u : 0u);
  __syncthreads();
  return higher + x - v;
}

// The bin of a 2^w-bin histogram (w = 10 or 11) that holds the kk-th largest counted item, scanning from the top:
// thread t owns bins [t * per, (t + 1) * per). Writes *s_bin and *s_above (the items in higher bins); *s_bin keeps
// its previous value when fewer than kk items were counted. All threads call it; it ends with a barrier.
__device__ __forceinline__ void find_bin(const unsigned* hist, int w, unsigned kk, unsigned* warp_tot, int* s_bin,
                                         unsigned* s_above) {
  const int per = (1 << w) / kThreads;
  unsigned mine = 0;
  for (int b = 0; b < per; ++b) mine += hist[threadIdx.x * per + b];
  unsigned run = block_suffix_excl(mine, warp_tot);
  for (int b = per - 1; b >= 0; --b) {
    const unsigned h = hist[threadIdx.x * per + b];
    if (run < kk && run + h >= kk) {
      *s_bin = threadIdx.x * per + b;
      *s_above = run;
    }
    run += h;
  }
  __syncthreads();
}

// Appends every staged composite >= lo to cand (at most kCap stored, *s_cnt counts them all). A float compare finds
// the few elements that may qualify; only those build their composite and take a slot with a shared atomic.
template <typename T>
__device__ __forceinline__ void collect(const uint4* data, int nv, int n, unsigned base_idx, u64 lo, u64* cand,
                                        int* s_cnt) {
  constexpr int V = VecN<T>::N;
  const T* tag = nullptr;
  const float f_lo = __uint_as_float(key_bits((unsigned)(lo >> 32)));
  for (int i = threadIdx.x; i < nv; i += kThreads) {
    const uint4 r = data[i];
    unsigned mask = vec_not_below(r, f_lo, tag);
    if (mask == 0u) continue;
    unsigned take = 0u;
    for (unsigned m = mask; m; m &= m - 1u) {
      const int e = __ffs(m) - 1;
      const int idx = i * V + e;
      if (idx < n && composite(order_key(elem_bits(r, e, tag)), base_idx + (unsigned)idx) >= lo) take |= 1u << e;
    }
    if (take == 0u) continue;
    int pos = atomicAdd(s_cnt, __popc(take));
    for (; take; take &= take - 1u, ++pos) {
      const int e = __ffs(take) - 1;
      if (pos < kCap) cand[pos] = composite(order_key(elem_bits(r, e, tag)), base_idx + (unsigned)(i * V + e));
    }
  }
}

// The same selection into this warp's own slots of the candidate buffer. Two vectors per thread per step; a thread
// whose vectors all stay below lo (nearly every one) only loads and compares them: no vote, no shuffle. The rare
// thread holding a candidate reserves its slots with a shared atomic on its warp's own counter (no contention across
// warps). The counter may pass `slots` (the entries past it are dropped; the caller falls back).
template <typename T>
__device__ __forceinline__ void collect_warp(const uint4* data, int nv, int n, unsigned base_idx, u64 lo, u64* region,
                                             int slots, int* wcount) {
  constexpr int V = VecN<T>::N;
  const T* tag = nullptr;
  const float f_lo = __uint_as_float(key_bits((unsigned)(lo >> 32)));
  for (int i = threadIdx.x; i < nv; i += 2 * kThreads) {
    const int i1 = i + kThreads;
    const uint4 r0 = data[i];
    const uint4 r1 = i1 < nv ? data[i1] : make_uint4(0xffffffffu, 0xffffffffu, 0xffffffffu, 0xffffffffu);
    const float m0 = vec_max_nan(r0, tag), m1 = i1 < nv ? vec_max_nan(r1, tag) : -CUDART_INF_F;
    if (m0 < f_lo && m1 < f_lo) continue;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint4 r = h ? r1 : r0;
      const int iv = h ? i1 : i;
      if ((h ? m1 : m0) < f_lo) continue;
      unsigned take = 0u;
      for (unsigned m = vec_not_below(r, f_lo, tag); m; m &= m - 1u) {
        const int e = __ffs(m) - 1;
        const int idx = iv * V + e;
        if (idx < n && composite(order_key(elem_bits(r, e, tag)), base_idx + (unsigned)idx) >= lo) take |= 1u << e;
      }
      if (take == 0u) continue;
      int pos = atomicAdd(wcount, __popc(take));
      for (; take; take &= take - 1u, ++pos) {
        const int e = __ffs(take) - 1;
        if (pos < slots) region[pos] = composite(order_key(elem_bits(r, e, tag)), base_idx + (unsigned)(iv * V + e));
      }
    }
  }
}

// The top k of the cnt distinct composites in cand, sorted, into top[0, k) (zero padded when cnt < k): a rank count,
// G lanes per candidate (G the largest power of two <= 32 with cnt * G <= kThreads), each lane comparing against
// every G-th candidate, the partial counts summed by xor shuffles. Ends with a barrier.
__device__ __forceinline__ void select_top(const u64* cand, int cnt, int k, u64* top) {
  int g = 32;
  while (g > 1 && cnt * g > kThreads) g >>= 1;
  const int sub = threadIdx.x & (g - 1);
  for (int base = 0; base < cnt; base += kThreads / g) {  // uniform trip count: every lane joins the shuffles
    const int item = base + (int)threadIdx.x / g;
    u64 c = 0ull;
    int rank = 0;
    if (item < cnt) {
      c = cand[item];
      for (int j = sub; j < cnt; j += g) rank += cand[j] > c;
    }
    for (int o = g >> 1; o > 0; o >>= 1) rank += __shfl_xor_sync(0xffffffffu, rank, o);
    if (item < cnt && sub == 0 && rank < k) top[rank] = c;
  }
  for (int e = cnt + threadIdx.x; e < k; e += kThreads) top[e] = 0ull;
  __syncthreads();
}

// Radix select over all staged composites: the lower edge `lo` of the digit bin holding the kk-th largest, refined
// digit by digit (11/11/10 bits of the key, then 11/11/10 of the index) until the composites >= lo fit kCap. Every
// level zeroes and rebuilds the histogram. All threads call it, after a barrier that ends all use of `hist`.
template <typename T>
__device__ u64 radix_select(const uint4* data, int nv, int n, unsigned base_idx, unsigned kk0, unsigned* hist,
                            unsigned* warp_tot, int* s_bin, unsigned* s_above) {
  constexpr int V = VecN<T>::N;
  const T* tag = nullptr;
  u64 prefix = 0, lo = 0;
  unsigned kk = kk0, above_total = 0;
  for (int L = 0; L < kLevels; ++L) {
    const int sh = level_shift(L), w = level_width(L);
    const unsigned mask = (1u << w) - 1u;
    for (int i = threadIdx.x; i < kBins; i += kThreads) hist[i] = 0u;
    __syncthreads();
    for (int i = threadIdx.x; i < nv; i += kThreads) {
      unsigned key[V];
      keys16(data[i], key, tag);
#pragma unroll
      for (int e = 0; e < V; ++e) {
        const int idx = i * V + e;
        if (idx < n) {
          const u64 c = composite(key[e], base_idx + (unsigned)idx);
          if (L == 0 || (c >> (sh + w)) == prefix) atomicAdd(&hist[(unsigned)(c >> sh) & mask], 1u);
        }
      }
    }
    __syncthreads();
    find_bin(hist, w, kk, warp_tot, s_bin, s_above);
    const int bin = *s_bin;
    const unsigned above = *s_above, inbin = hist[bin];
    const u64 next = (prefix << w) | (u64)bin;
    lo = next << sh;
    if (above_total + above + inbin <= (unsigned)kCap || L == kLevels - 1) break;
    above_total += above;
    kk -= above;
    prefix = next;
    __syncthreads();  // every thread has read hist[bin] and the bin before the next level rewrites them
  }
  return lo;
}

struct ChunkArgs {
  const void* x;
  void* values;          // mode 0: [rows, k] in x's dtype
  long long* indices;    // mode 0: [rows, k]
  u64* lists;            // mode 1: [rows, k] sorted composites, zero padded
  u64* work;             // [rows, nchunks, k] when a row has several chunks
  unsigned* counters;    // [rows], zero on entry, left zero
  long long col_offset;  // added to every column index
  int cols, chunk, k, data_bytes, mode;
};

// Writes the row's final top k (sorted composites top[0, k)) in the requested form.
template <typename T>
__device__ __forceinline__ void emit(const ChunkArgs& a, long long row, int j, u64 c) {
  if (a.mode == 0) {
    reinterpret_cast<T*>(a.values)[row * a.k + j] = decode_value<T>(c);
    a.indices[row * a.k + j] = decode_index(c);
  } else {
    a.lists[row * a.k + j] = c;
  }
}

// Grid (nchunks, rows). kBulk: the chunk's rows are 16-byte aligned and sized, so bulk copies stage it; otherwise the
// threads copy it element by element.
template <typename T, bool kBulk>
__global__ void __launch_bounds__(kThreads) topk_chunk(const ChunkArgs a) {
  constexpr int V = VecN<T>::N;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t bars[kPieces];
  __shared__ unsigned warp_tot[kWarps];
  __shared__ int s_bin;
  __shared__ unsigned s_above;
  __shared__ int s_cnt;
  __shared__ int s_last;
  __shared__ int s_wcnt[kWarps];

  const T* tag = nullptr;
  uint4* data = reinterpret_cast<uint4*>(smem_raw);
  unsigned* hist = reinterpret_cast<unsigned*>(smem_raw + a.data_bytes);
  u64* cand = reinterpret_cast<u64*>(hist);  // used only after the last histogram has been read

  const long long row = blockIdx.y;
  const int nchunks = gridDim.x;
  const long long begin = (long long)blockIdx.x * a.chunk;
  const int n = (int)min((long long)a.chunk, (long long)a.cols - begin);
  const T* src = reinterpret_cast<const T*>(a.x) + row * a.cols + begin;
  const int nv = (n + V - 1) / V;  // staged 16-byte vectors
  const int pv = (nv + kPieces - 1) / kPieces;
  const unsigned base_idx = (unsigned)(a.col_offset + begin);

  // 1. Stage the chunk; zero the histogram meanwhile.
  if constexpr (kBulk) {
    if (threadIdx.x == 0) {
#pragma unroll
      for (int p = 0; p < kPieces; ++p) mbar_init(&bars[p], 1);
      mbar_fence_init();
#pragma unroll
      for (int p = 0; p < kPieces; ++p) {
        const int v0 = p * pv, v1 = min(nv, v0 + pv);
        if (v1 > v0) {
          mbar_arrive_expect_tx(&bars[p], (unsigned)(v1 - v0) * 16u);
          bulk_load(data + v0, reinterpret_cast<const uint4*>(src) + v0, (unsigned)(v1 - v0) * 16u, &bars[p]);
        }
      }
    }
  } else {
    T* d = reinterpret_cast<T*>(data);
    for (int i = threadIdx.x; i < n; i += kThreads) d[i] = src[i];
    // Pad the last vector with NaN: the max pass skips it and the collect pass rejects it by index.
    for (int i = n + threadIdx.x; i < nv * V; i += kThreads) d[i] = from_f32<T>(__int_as_float(0x7fc00000));
  }
  for (int i = threadIdx.x; i < kBins / 4; i += kThreads) reinterpret_cast<uint4*>(hist)[i] = make_uint4(0u, 0u, 0u, 0u);
  if (threadIdx.x == 0) {
    s_bin = -1;
    s_above = 0u;
    s_cnt = 0;
  }
  if (threadIdx.x < kWarps) s_wcnt[threadIdx.x] = 0;
  __syncthreads();

  // 2. A lower bound from the per-thread maxima: the k-th largest of them has at least k elements at or above it, so
  //    the lower edge of its histogram bin bounds the chunk's k-th largest key from below. Only 512 maxima touch the
  //    histogram; the one pass over the chunk is a max.
  bool ok = true;
  float fmax = __int_as_float(0x7fc00000);  // NaN: no number seen yet
  for (int p = 0; p < kPieces; ++p) {
    const int v0 = p * pv, v1 = min(nv, v0 + pv);
    if (v1 <= v0) continue;
    if constexpr (kBulk) ok = mbar_wait(&bars[p], 0) && ok;
    int i = v0 + threadIdx.x;
    for (; i + kThreads < v1; i += 2 * kThreads) fmax = vec_max(data[i + kThreads], vec_max(data[i], fmax, tag), tag);
    if (i < v1) fmax = vec_max(data[i], fmax, tag);
  }
  if (!ok) atomicOr(&g_topk_status, CKB_STATUS_TIMEOUT);
  const unsigned kk0 = (unsigned)min(a.k, n);
  u64 lo = 0;
  if (n > kCap) {
    // fmax is one of this thread's elements (or NaN when it has no number): the maxima counted are real elements.
    if (fmax == fmax) atomicAdd(&hist[order_key(__float_as_uint(fmax)) >> 21], 1u);
    __syncthreads();
    find_bin(hist, 11, kk0, warp_tot, &s_bin, &s_above);
    if (s_bin >= 0) lo = (u64)s_bin << 53;
  }
  __syncthreads();  // the histogram is dead from here: the candidate buffer reuses it

  // 3. Collect the composites >= lo, each warp into its own kWarpSlots slots (no shared atomics). If a warp's slots
  //    overflow (heavy ties, or too few maxima), a radix select over the chunk's composites narrows `lo` until they
  //    fit the whole buffer, and they are collected again.
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  collect_warp<T>(data, nv, n, base_idx, lo, cand + warp * kWarpSlots, kWarpSlots, &s_wcnt[warp]);
  __syncthreads();
  const int wcnt = s_wcnt[warp];
  // Every warp scans the 16 counts across its lanes: the total, this warp's start, any overflow.
  int wc = lane < kWarps ? s_wcnt[lane] : 0;
  const bool over = __any_sync(0xffffffffu, wc > kWarpSlots);
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, wc, o);
    if (lane >= o) wc += y;
  }
  const int cnt = __shfl_sync(0xffffffffu, wc, 31);
  const int start = warp ? __shfl_sync(0xffffffffu, wc, (warp - 1) & 31) : 0;

  // 4. The chunk's top k, sorted, into top[0, k) (zero padded when the chunk has fewer than k elements); the chunk's
  //    staging area is dead from here and holds the packed candidates and top.
  u64* packed = reinterpret_cast<u64*>(smem_raw);
  u64* top = packed + kCap;
  if (!over) {
    for (int j = lane; j < wcnt; j += 32) packed[start + j] = cand[warp * kWarpSlots + j];
    __syncthreads();
    select_top(packed, cnt, a.k, top);
  } else {
    lo = radix_select<T>(data, nv, n, base_idx, kk0, hist, warp_tot, &s_bin, &s_above);
    if (threadIdx.x == 0) s_cnt = 0;
    __syncthreads();
    collect<T>(data, nv, n, base_idx, lo, cand, &s_cnt);
    __syncthreads();
    select_top(cand, min(s_cnt, kCap), a.k, top);
  }

  // 5. Output, or the multi-chunk merge by the row's last CTA.
  if (nchunks == 1) {
    for (int j = threadIdx.x; j < a.k; j += kThreads) emit<T>(a, row, j, top[j]);
    return;
  }
  u64* wr = a.work + row * (long long)nchunks * a.k;
  // The writers (threads below k <= kThreads) fence their own stores before the row counter moves.
  if ((int)threadIdx.x < a.k) {
    wr[(long long)blockIdx.x * a.k + threadIdx.x] = top[threadIdx.x];
    __threadfence();
  }
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(&a.counters[row], 1u) == (unsigned)nchunks - 1u;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const int total = nchunks * a.k;
  u64* lists = reinterpret_cast<u64*>(smem_raw);
  for (int i = threadIdx.x; i < total; i += kThreads) lists[i] = __ldcg(wr + i);
  __syncthreads();
  for (int i = threadIdx.x; i < total; i += kThreads) {
    const u64 c = lists[i];
    if (c == 0ull) continue;
    const int own = i / a.k;
    int rank = i - own * a.k;
    for (int l = 0; l < nchunks && rank < a.k; ++l)
      if (l != own) rank += count_greater(lists + l * a.k, a.k, c);
    if (rank < a.k) emit<T>(a, row, rank, c);
  }
  if (threadIdx.x == 0) a.counters[row] = 0u;
}

// Merge of nlists sorted composite lists per row, lists laid out [nlists][rows][k] (an all-gather's output); one
// CTA per row writes the top k values and indices.
template <typename T>
__global__ void __launch_bounds__(256) topk_merge(const u64* __restrict__ lists, int nlists, long long rows, int k,
                                                  T* __restrict__ values, long long* __restrict__ indices) {
  extern __shared__ __align__(16) u64 sl[];
  const long long row = blockIdx.x;
  const int total = nlists * k;
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int l = i / k, j = i - l * k;
    sl[i] = __ldg(lists + ((long long)l * rows + row) * k + j);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const u64 c = sl[i];
    if (c == 0ull) continue;
    const int own = i / k;
    int rank = i - own * k;
    for (int l = 0; l < nlists && rank < k; ++l)
      if (l != own) rank += count_greater(sl + l * k, k, c);
    if (rank < k) {
      values[row * k + rank] = decode_value<T>(c);
      indices[row * k + rank] = decode_index(c);
    }
  }
}

// Columns per CTA: the fewest chunks whose staged bytes fit kChunkBytes, raised (down to min_chunk columns, up to
// kGrowChunks chunks so the last CTA's merge stays short) until the grid holds at least three CTAs per SM; a multiple
// of 16 columns so every chunk starts 16-byte aligned.
constexpr long long kGrowChunks = 32;

long long plan_chunk(long long rows, long long cols, int elem, int min_chunk) {
  if (rows <= 0 || cols <= 0) return cols > 0 ? cols : 1;
  const long long max_elems = kChunkBytes / elem;
  long long nchunks = (cols + max_elems - 1) / max_elems;
  const long long target = 3LL * device_sm_count();
  if (min_chunk < 1024) min_chunk = 1024;
  while (rows * nchunks < target && nchunks < kGrowChunks && (cols + nchunks) / (nchunks + 1) >= min_chunk)
    ++nchunks;
  if (nchunks <= 1) return cols;
  long long chunk = (cols + nchunks - 1) / nchunks;
  chunk = (chunk + 15) / 16 * 16;
  return chunk;
}

int data_bytes_for(long long chunk, int elem, int nchunks, int k) {
  long long b = chunk * elem;
  if (b < (long long)(kCap + k) * 8) b = (long long)(kCap + k) * 8;  // packed candidates + top, after the chunk
  if (nchunks > 1 && b < (long long)nchunks * k * 8) b = (long long)nchunks * k * 8;
  return (int)((b + 127) / 128 * 128);
}

template <typename T>
int start_chunk(const ChunkArgs& base, long long rows, long long cols, long long chunk, cudaStream_t s) {
  const int elem = (int)sizeof(T);
  const long long nchunks = (cols + chunk - 1) / chunk;
  ChunkArgs a = base;
  a.cols = (int)cols;
  a.chunk = (int)chunk;
  a.data_bytes = data_bytes_for(chunk, elem, (int)nchunks, a.k);
  if (a.data_bytes > kMaxDataBytes) return -1;
  const int smem = a.data_bytes + kBins * 4;
  const bool bulk = aligned16(a.x) && (cols * elem) % 16 == 0 && (chunk * elem) % 16 == 0;
  const dim3 grid((unsigned)nchunks, (unsigned)rows);
  if (bulk) {
    auto kern = topk_chunk<T, true>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return (int)cudaGetLastError();
    kern<<<grid, kThreads, smem, s>>>(a);
  } else {
    auto kern = topk_chunk<T, false>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return (int)cudaGetLastError();
    kern<<<grid, kThreads, smem, s>>>(a);
  }
  return (int)cudaGetLastError();
}

// The reference's argument checks (topk/kernel.cu:551-554) plus this library's chunk staging limit.
bool bad_args(long long rows, long long cols, int k, long long chunk, int elem) {
  if (k > cols || k > kMaxK || cols > INT_MAX / 2 || rows > 65535 || chunk <= 0) return true;
  const long long nchunks = (cols + chunk - 1) / chunk;
  if (nchunks > 1 && (chunk % 4 || nchunks * k > INT_MAX / 2)) return true;
  if (chunk > cols) chunk = cols;
  return data_bytes_for(chunk, elem, (int)nchunks, k) > kMaxDataBytes;
}

}  // namespace
}  // namespace ckb

using namespace ckb;

// Replaces the reference's top-k `plan` (topk/kernel.cu:520-547): the columns per CTA for a rows x cols launch
// (dtype 0 fp32, 1 bf16). `threads` and `depth` are the reference's kernel knobs and do not change the B200 plan;
// min_chunk is a lower bound on the chunk when a row is split to fill the GPU. A row's chunk count is
// ceil(cols / chunk); the workspace launch() needs is rows * chunks * k int64 values.
CKB_EXPORT long long plan(long long rows, long long cols, int dtype, int threads, int depth, int min_chunk) {
  (void)threads;
  (void)depth;
  return plan_chunk(rows, cols, dtype == kBF16 ? 2 : 4, min_chunk);
}

// Replaces the reference's top-k `launch` (topk/kernel.cu:549-570): same arguments, checks and return codes. work is
// int64 [rows * nchunks * k] (unused with one chunk), counters int32 [rows] zeroed once and left zeroed by the kernel.
// `chunk` must come from plan() (or be small enough for the shared-memory staging; larger gives -1).
CKB_EXPORT int launch(const void* x, void* values, void* indices, void* work, void* counters, long long rows,
                      long long cols, int k, int dtype, int threads, int depth, long long chunk,
                      cudaStream_t stream) {
  if (rows <= 0 || k <= 0) return 0;
  if (threads != 128 && threads != 256 && threads != 512) return -1;
  if (depth != 2 && depth != 4 && depth != 8) return -1;
  const int elem = dtype == kBF16 ? 2 : 4;
  if (bad_args(rows, cols, k, chunk, elem)) return -1;
  if (chunk > cols) chunk = cols;
  ChunkArgs a{x, values, (long long*)indices, nullptr, (u64*)work, (unsigned*)counters, 0, 0, 0, k, 0, 0};
  if (dtype == kF32) return start_chunk<float>(a, rows, cols, chunk, stream);
  if (dtype == kBF16) return start_chunk<__nv_bfloat16>(a, rows, cols, chunk, stream);
  return -1;
}

// Top-k of a column shard for the vocab-sharded variant (no counterpart in the reference): x is [rows, cols] holding
// global columns [col_offset, col_offset + cols); lists receives [rows, k] sorted composites (uint64, zero padded)
// carrying global indices, ready for an all-gather and ckb_topk_merge_launch. work/counters/chunk as in launch().
CKB_EXPORT int ckb_topk_shard_launch(const void* x, unsigned long long* lists, void* work, void* counters,
                                     long long rows, long long cols, long long col_offset, int k, int dtype,
                                     long long chunk, cudaStream_t stream) {
  if (rows <= 0 || k <= 0) return 0;
  const int elem = dtype == kBF16 ? 2 : 4;
  if (col_offset < 0 || col_offset + cols > INT_MAX / 2 || bad_args(rows, cols, k, chunk, elem)) return -1;
  if (chunk > cols) chunk = cols;
  ChunkArgs a{x, nullptr, nullptr, lists, (u64*)work, (unsigned*)counters, col_offset, 0, 0, k, 0, 1};
  if (dtype == kF32) return start_chunk<float>(a, rows, cols, chunk, stream);
  if (dtype == kBF16) return start_chunk<__nv_bfloat16>(a, rows, cols, chunk, stream);
  return -1;
}

// Final merge of the vocab-sharded variant (no counterpart in the reference): lists [nlists][rows][k] of sorted
// composites (one list per shard) -> values [rows, k] in the dtype (0 fp32, 1 bf16) and int64 indices [rows, k].
CKB_EXPORT int ckb_topk_merge_launch(const unsigned long long* lists, int nlists, void* values, void* indices,
                                     long long rows, int k, int dtype, cudaStream_t stream) {
  if (rows <= 0 || k <= 0) return 0;
  if (nlists <= 0 || k > kMaxK || rows > INT_MAX) return -1;
  const long long smem = (long long)nlists * k * 8;
  if (smem > kMaxDataBytes) return -1;
  if (dtype == kF32) {
    if (cudaFuncSetAttribute(topk_merge<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
      return (int)cudaGetLastError();
    topk_merge<float><<<(unsigned)rows, 256, (size_t)smem, stream>>>((const u64*)lists, nlists, rows, k,
                                                                     (float*)values, (long long*)indices);
  } else if (dtype == kBF16) {
    if (cudaFuncSetAttribute(topk_merge<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
      return (int)cudaGetLastError();
    topk_merge<__nv_bfloat16><<<(unsigned)rows, 256, (size_t)smem, stream>>>(
        (const u64*)lists, nlists, rows, k, (__nv_bfloat16*)values, (long long*)indices);
  } else {
    return -1;
  }
  return (int)cudaGetLastError();
}

// Status of the bounded waits in this library's kernels since the last reset: 0, or 1 when a bulk-copy wait gave up.
// Synchronises with the device; reset != 0 clears the word.
CKB_EXPORT int ckb_topk_status(int reset) {
  unsigned v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_topk_status, sizeof(v));
  if (e != cudaSuccess) return -(int)e;
  if (reset) {
    const unsigned zero = 0;
    e = cudaMemcpyToSymbol(g_topk_status, &zero, sizeof(zero));
    if (e != cudaSuccess) return -(int)e;
  }
  return (int)v;
}

// ------------------------------------------------------------------------------------------ no-allocation entry ---
// Some callers cannot allocate device memory for the workspace and counters that launch() takes: code living inside
// a host framework that hands out a fixed budget through its own allocator (and may have reserved nearly all of the
// GPU up front), or a latency-critical path where cudaMalloc's implicit device synchronisation is not acceptable.
// ckb_topk_launch_noalloc serves them from a scratch array compiled into this library instead: 4 MiB of device
// memory that every GPU which loads the library holds until the process exits. The first 256 KiB are the per-row
// counters (up to 65536 rows), the rest the chunk workspace (491,520 composites, i.e. rows * chunks * k at most that).
constexpr size_t kNoAllocBytes = size_t(4) << 20;
static __device__ __align__(256) unsigned long long g_noalloc_scratch[kNoAllocBytes / 8];

namespace ckb {
namespace {

constexpr long long kNoAllocCounterWords = 32768;  // 65536 uint32 counters in the first 256 KiB
constexpr long long kNoAllocWorkWords = (long long)(kNoAllocBytes / 8) - kNoAllocCounterWords;

// The scratch array's device address on the current device. In host code g_noalloc_scratch names a host-side
// stand-in, not device memory, so the address is looked up once per device (with that device current) and cached.
cudaError_t noalloc_scratch(void** out) {
  static std::atomic<void*> cache[64];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  void* p = cache[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    cache[dev].store(p, std::memory_order_release);
  }
  *out = p;
  return cudaSuccess;
}

}  // namespace
}  // namespace ckb

// The top-k of launch() without any caller-provided workspace or counters (no counterpart in the reference): values
// [rows, k] in x's dtype and int64 indices [rows, k] of x [rows, cols], dtype 0 (fp32) or 1 (bf16), planned as plan()
// would with min_chunk 2048. Allocates nothing. Returns 0, -1 for arguments launch() would also reject, -2 when the
// plan needs more than the static scratch holds (rows * chunks * k > 491,520 or rows > 65,536), or a cudaError_t.
// The first call on a device looks up the scratch address (make it before any stream capture). Every call shares the
// one scratch array, so calls that overlap on the GPU (different streams, no ordering between them) race; calls on
// one stream are ordered. The counters are cleared on the caller's stream at each call.
CKB_EXPORT int ckb_topk_launch_noalloc(const void* x, void* values, void* indices, long long rows, long long cols,
                                       int k, int dtype, cudaStream_t stream) {
  if (rows <= 0 || k <= 0) return 0;
  if (dtype != kF32 && dtype != kBF16) return -1;
  const int elem = dtype == kBF16 ? 2 : 4;
  long long chunk = plan_chunk(rows, cols, elem, 2048);
  if (bad_args(rows, cols, k, chunk, elem)) return -1;
  if (chunk > cols) chunk = cols;
  const long long nchunks = (cols + chunk - 1) / chunk;
  if (rows > 2 * kNoAllocCounterWords || (nchunks > 1 && rows * nchunks * k > kNoAllocWorkWords)) return -2;
  void* base = nullptr;
  cudaError_t e = noalloc_scratch(&base);
  if (e != cudaSuccess) return (int)e;
  unsigned* counters = reinterpret_cast<unsigned*>(base);
  u64* work = reinterpret_cast<u64*>(base) + kNoAllocCounterWords;
  if (nchunks > 1) {
    e = cudaMemsetAsync(counters, 0, (size_t)rows * sizeof(unsigned), stream);
    if (e != cudaSuccess) return (int)e;
  }
  ChunkArgs a{x, values, (long long*)indices, nullptr, work, counters, 0, 0, 0, k, 0, 0};
  if (dtype == kF32) return start_chunk<float>(a, rows, cols, chunk, stream);
  return start_chunk<__nv_bfloat16>(a, rows, cols, chunk, stream);
}
