// Row-wise top-k (largest k, sorted descending, ties broken by the lower index) of x[rows, cols], fp32 (dtype 0) or
// bf16 (dtype 1), values bit-exact in x's dtype and int64 indices -- the reference's output contract
// (topk/kernel.cu:1-3,436-441, topk/candidate.py:66-81).
//
// Order. Every element becomes a distinct 64-bit composite (order-preserving key of its float bits << 32 | ~index),
// the same total order as the reference's pack() (topk/kernel.cu:56-60): larger value first, equal values by lower
// index, NaN above +inf, -NaN below -inf. The top k of a row are its k largest composites.
//
// Algorithm (grid: segments x rows, 512 threads per CTA, one pass over HBM):
//   1. each CTA streams its segment of the row through a ring of shared-memory stages that its threads fill with
//      16-byte asynchronous copies (cp.async); a thread reads back only the vectors it copied itself, so the ring
//      needs no block barrier and keeps several tiles (512 x U vectors each) in flight;
//   2. first tile, a lower bound: every thread takes the max of its numbers; in each warp the c-th largest of the 32
//      maxima (c = ceil(k / 16)) has c distinct elements at or above it, so the smallest of the 16 warps' values has
//      at least k elements at or above it and bounds the segment's k-th largest composite from below;
//   3. every tile: the composites at or above the running bound are appended (a float pre-filter per vector, the
//      composite only for the few that pass) behind the running top k in a candidate buffer; a block rank count leaves
//      the new running top k and the bound rises to one above its k-th entry, so a later tile passes only elements
//      that enter the top k (about k / tile number of them). A tile that overflows the buffer (heavy ties) first
//      raises the bound by a radix select over its composites, still in registers (11/11/10 bits of the key, then
//      11/11/10 of the index, so value ties resolve by index);
//   4. a row split over several segments writes each segment's sorted top k to the workspace; the row's last CTA to
//      finish (per-row counter, reset by that CTA) merges the lists pairwise (each entry's rank in the partner list by
//      binary search) and decodes values and indices from the composites (x is not read again).
// The vocab-sharded variant runs steps 1-4 on a column shard with a global column offset and stops at the sorted
// composites; after an all-gather across GPUs the merge kernel ranks the per-GPU lists the same way.
#include "ckb200_topk.h"
#include "common.cuh"

#include <math_constants.h>

#include <climits>
#include <cstring>

namespace ckb {

__device__ unsigned int g_topk_status = 0u;

namespace {

typedef unsigned long long u64;

// Two CTA shapes. 256 threads (8 warps, 4 CTAs per SM) serve k <= 256: a GPU's worth of CTAs holds 592 rows'
// streams at once, so a batch of a few hundred long rows runs in one wave without splitting rows. 512 threads (16
// warps, 2 CTAs per SM) serve k <= 512. The first tile's bound needs c = ceil(k / warps) <= 32 maxima per warp.
#ifndef CKB_TOPK_STAGES
#define CKB_TOPK_STAGES 3
#endif
#ifndef CKB_TOPK_UNROLL
#define CKB_TOPK_UNROLL 4
#endif
// fp32 rows: 20 KB tiles in a 2-stage ring (one tile in flight while one is filtered). Measured on B200 at 512 x
// 151936: 16 KB x 3 stages 60.8 us, 20 KB x 2 58.6, 24 KB x 2 58.5 (spills), 12 KB x 4 61.8; fewer barriers per
// byte outweigh the shallower ring at four CTAs per SM.
#ifndef CKB_TOPK_STAGES_256
#define CKB_TOPK_STAGES_256 2
#endif
#ifndef CKB_TOPK_UNROLL_256
#define CKB_TOPK_UNROLL_256 5
#endif
#ifndef CKB_TOPK_SLOTS_256
#define CKB_TOPK_SLOTS_256 32
#endif
// Candidate buffer of the 256-thread shape (the running top k and the survivors behind it). 1280 lets every warp's
// 32 slots expand in one pass (k + 8 warps x 32 vectors x 4 composites fits with room to spare) and a tile of heavy
// ties collect without the overflow path. Measured on B200, fp32 512 x 151936: 512 entries 58.9 us, 1024 58.9, 1280
// 56.7, 1536 56.6; few-valued rows 137.2 -> 113.1 us, ascending rows 551 -> 380 us.
#ifndef CKB_TOPK_CAND_256
#define CKB_TOPK_CAND_256 1280
#endif
// The 256-thread shape for 2-byte elements: 20 KB tiles (10240 elements) in a 2-stage ring as for fp32 (measured at
// 512 x 151936 bf16: 16 KB tiles 44.9 us, 20 KB 43.9 us, 12 KB x 3 stages 45.7 us).
#ifndef CKB_TOPK_STAGES_256H
#define CKB_TOPK_STAGES_256H 2
#endif
#ifndef CKB_TOPK_UNROLL_256H
#define CKB_TOPK_UNROLL_256H 5
#endif
#ifndef CKB_TOPK_SLOTS_256H
#define CKB_TOPK_SLOTS_256H 32
#endif
#ifndef CKB_TOPK_STRICT
#define CKB_TOPK_STRICT 1
#endif
// 0: a survivor slot holds the recorded vector's index only, and the vector is read again (from L2, where the
// streamed tile still is) when the slots are expanded, so a warp holds 32 slots in the shared memory that 10 slots
// of vector + index took (1: vector and index; measured on B200, fp32 512 x 151936: 63.2 us with 10 such slots, 60.9
// us with 32 index slots; 512 x 18992, a vocab shard at 8 GPUs: 27.1 -> 24.1 us).
#ifndef CKB_TOPK_SLOT_DATA
#define CKB_TOPK_SLOT_DATA 0
#endif
constexpr bool kSlotData = CKB_TOPK_SLOT_DATA != 0;
// Segments of at least this many elements ask for a compaction once a warp holds CKB_TOPK_SLOTS_FULL_LONG records
// (the earlier raise of the bound pays over the long rest); shorter ones only when the slots are nearly full.
#ifndef CKB_TOPK_LONG_ELEMS
#define CKB_TOPK_LONG_ELEMS 65536
#endif
#ifndef CKB_TOPK_SLOTS_FULL_LONG
#define CKB_TOPK_SLOTS_FULL_LONG 12
#endif
#ifndef CKB_TOPK_SLOTS_FULL_LONG_H
#define CKB_TOPK_SLOTS_FULL_LONG_H 20  // 2-byte elements: a vector holds 8, so more vectors pass per survivor
#endif
#ifndef CKB_TOPK_OVF_BOUND
#define CKB_TOPK_OVF_BOUND 1
#endif
#ifndef CKB_TOPK_WIDE_ONLY
#define CKB_TOPK_WIDE_ONLY 0
#endif
#ifndef CKB_TOPK_SPEC_Z
#define CKB_TOPK_SPEC_Z 4.5f
#endif
#ifndef CKB_TOPK_SPEC_MARGIN
#define CKB_TOPK_SPEC_MARGIN 3.0f
#endif
// Speculative bound after a compaction: the m-th largest composite seen so far. The bound is too high only when the
// seen part (a fraction f of the segment) holds m or more of the segment's top k elements; with values in random
// order that count is about Poisson(k f), so m = ceil(k f + z sqrt(k f) + margin) makes a miss rare (the kernel
// checks for it and then streams the segment again with guaranteed bounds).
constexpr float kSpecZ = CKB_TOPK_SPEC_Z;
constexpr float kSpecMargin = CKB_TOPK_SPEC_MARGIN;
__device__ __forceinline__ int spec_rank(int k, float seen) {
  const float kf = (float)k * fminf(fmaxf(seen, 0.0f), 1.0f);
  return min(k, (int)ceilf(kf + kSpecZ * sqrtf(kf) + kSpecMargin));
}
constexpr int kMaxK = 512;
constexpr int kDirectSelect = 192;                // compactions of more candidates narrow them by radix first
constexpr int kSmPerSmBytes = 233472;             // shared memory per SM (228 KB)

// Per shape: the ring, the candidate buffer (the running top k and the survivors behind it, so at least 2 kMaxK), the
// compaction scratch (select output, packing, or the radix histogram of kDigit-bit digits) and the warps' survivor
// slots. The 256-thread shape keeps all of it within a quarter of an SM's shared memory.
template <int NT, int EB = 4>  // EB: element bytes (the ring and slots differ; the rest is the same for both)
struct Cfg {
  static constexpr int kWarps = NT / 32;
  static constexpr int kMaxK = NT == 512 ? 512 : 256;              // c = ceil(k / kWarps) <= 32
  static constexpr int kStages =                                    // ring depth
      NT == 512 ? CKB_TOPK_STAGES : EB == 4 ? CKB_TOPK_STAGES_256 : CKB_TOPK_STAGES_256H;
  static constexpr int kU =                                         // vectors per thread per tile
      NT == 512 ? CKB_TOPK_UNROLL : EB == 4 ? CKB_TOPK_UNROLL_256 : CKB_TOPK_UNROLL_256H;
  static constexpr int kTileVecs = NT * kU;       // thread t holds vectors u * NT + t of a tile
  static constexpr int kRingBytes = kStages * kTileVecs * 16;
  static constexpr int kCand = NT == 512 ? 2 * kMaxK : CKB_TOPK_CAND_256;  // running top k + survivors since the
                                                                              // last compaction
  static constexpr int kPack = kMaxK;             // compaction scratch entries
  static constexpr int kDigit = NT == 512 ? 10 : 9;
  static constexpr int kRadixBins = 1 << kDigit;
  static constexpr int kLevels = (64 + kDigit - 1) / kDigit;
  static constexpr int kSlots =  // vectors a warp records between compactions
      NT == 512 ? 12 : EB == 4 ? CKB_TOPK_SLOTS_256 : CKB_TOPK_SLOTS_256H;
  static constexpr int kSlotsFull = kSlots - 4;       // a warp holding this many asks for a compaction
  static constexpr int kSlotBytes = kWarps * kSlots * (kSlotData ? 20 : 4);  // recorded vectors (16 B), indices (4 B)
  static constexpr int kSmemBytes = kRingBytes + kCand * 8 + kPack * 8 + kSlotBytes;
  static constexpr int kMergeEntries = kRingBytes / 16;    // nseg * k: the merge ping-pongs between ring halves
  static constexpr int kMinBlocks = NT == 512 ? 2 : 4;
  // Each CTA also holds 1 KB the hardware reserves and a few hundred bytes of static shared memory.
  static constexpr int kCtasPerSm =
      kSmPerSmBytes / (kSmemBytes + 1280) < kMinBlocks ? kSmPerSmBytes / (kSmemBytes + 1280) : kMinBlocks;
  static_assert(kMaxK <= 32 * kWarps, "the first tile's bound needs ceil(k / warps) <= 32");
  static_assert(kCand - kMaxK >= kMaxK, "after a compaction a radix select must leave room for k survivors");
  static_assert(kMergeEntries >= kMaxK, "the ring must hold one list per segment");
  static_assert(kRadixBins % NT == 0, "histogram bins split evenly over the threads");
  static_assert(kRadixBins * 4 <= kPack * 8, "the radix histogram lives in the compaction scratch");
  static_assert(kSlots <= 32, "a warp expands its slots one per lane");
  static_assert(kCtasPerSm >= 1, "one CTA's shared memory fits an SM");
};
// Segments per row that every k fits in every shape's merge, and at most 8 (measured on B200 at 1 x 128256: 8
// segments 14.0 us fp32 / 11.2 us bf16, 10 segments 14.3 / 11.6 us: the last CTA's merge grows with the lists).
template <int NT, int EB>
constexpr int seg_cap() { return Cfg<NT, EB>::kMergeEntries / Cfg<NT, EB>::kMaxK; }
constexpr int min2(int a, int b) { return a < b ? a : b; }
#ifndef CKB_TOPK_MAX_SEG
#define CKB_TOPK_MAX_SEG \
  min2(8, min2(min2(seg_cap<256, 4>(), seg_cap<256, 2>()), min2(seg_cap<512, 4>(), seg_cap<512, 2>())))
#endif
constexpr int kMaxSeg = CKB_TOPK_MAX_SEG;

// Radix digits of D bits over the 64-bit composite, most significant first (the last digit takes what is left).
template <int D>
__device__ __forceinline__ int level_shift(int L) { return 64 - D * (L + 1) > 0 ? 64 - D * (L + 1) : 0; }
template <int D>
__device__ __forceinline__ int level_width(int L) { return 64 - D * L < D ? 64 - D * L : D; }

__device__ __forceinline__ unsigned order_key(unsigned bits) {
  return (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
}
__device__ __forceinline__ unsigned key_bits(unsigned key) {  // inverse of order_key
  return (key & 0x80000000u) ? (key & 0x7fffffffu) : ~key;
}
__device__ __forceinline__ u64 composite(unsigned key, unsigned idx) { return ((u64)key << 32) | (u64)(~idx); }

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

// The largest non-NaN value of one 16-byte vector folded into a running max (NaN inputs are skipped, so a running
// max that is still NaN has seen no number). The result is always one of the inputs.
__device__ __forceinline__ float vec_max(const uint4& r, float m, const float*) {
  return max3(max3(m, __uint_as_float(r.x), __uint_as_float(r.y)), __uint_as_float(r.z), __uint_as_float(r.w));
}
__device__ __forceinline__ float vec_max(const uint4& r, float m, const __nv_bfloat16*) {
  const unsigned c = max_bf16x2(max_bf16x2(r.x, r.y), max_bf16x2(r.z, r.w));
  return max3(m, __uint_as_float(c << 16), __uint_as_float(c & 0xffff0000u));
}

// The largest value of one vector with NaN propagating (so a NaN element never hides behind the pre-filter).
__device__ __forceinline__ float vec_max_nan(const uint4& r, const float*) {
  return max3_nan(max3_nan(__uint_as_float(r.x), __uint_as_float(r.y), __uint_as_float(r.z)), __uint_as_float(r.w),
                  __uint_as_float(r.w));
}
__device__ __forceinline__ float vec_max_nan(const uint4& r, const __nv_bfloat16*) {
  const unsigned c = max_nan_bf16x2(max_nan_bf16x2(r.x, r.y), max_nan_bf16x2(r.z, r.w));
  const float lo = __uint_as_float(c << 16), hi = __uint_as_float(c & 0xffff0000u);
  return max3_nan(lo, hi, hi);
}

// The fp32 bits of element e of one vector (a bf16 element widened). Selects, not an indexed array, so the vector
// stays in registers.
__device__ __forceinline__ unsigned word_of(const uint4& r, int j) {
  return j < 2 ? (j == 0 ? r.x : r.y) : (j == 2 ? r.z : r.w);
}
__device__ __forceinline__ unsigned elem_bits(const uint4& r, int e, const float*) { return word_of(r, e); }
__device__ __forceinline__ unsigned elem_bits(const uint4& r, int e, const __nv_bfloat16*) {
  const unsigned w = word_of(r, e >> 1);
  return (e & 1) ? (w & 0xffff0000u) : (w << 16);
}
__device__ __forceinline__ unsigned scalar_bits(float v) { return __float_as_uint(v); }
__device__ __forceinline__ unsigned scalar_bits(__nv_bfloat16 v) { return (unsigned)__bfloat16_as_ushort(v) << 16; }

// Bit mask (bit e) of the elements of one vector that are not below f_lo as floats, NaN included: a superset of the
// elements whose order key is >= the key of f_lo.
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

// ------------------------------------------------------------------------------------ asynchronous 16-byte copies ---
__device__ __forceinline__ void cp_async16(void* dst_smem, const void* src) {
  asm volatile("cp.async.cg.shared.global.L2::256B [%0], [%1], 16;" ::"r"(smem_u32(dst_smem)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Sum of v over the threads with a higher threadIdx.x (all NT threads call it; two barriers).
template <int NT>
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
  unsigned t = lane < NT / 32 ? warp_tot[lane] : 0u;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned y = __shfl_down_sync(0xffffffffu, t, o);
    if (lane + o < 32) t += y;
  }
  const unsigned higher = __shfl_sync(0xffffffffu, t, (warp + 1) & 31) * (warp + 1 < 32 ? 1u : 0u);
  __syncthreads();
  return higher + x - v;
}

// The bin of an nb-bin histogram (nb a power of two <= 1024) that holds the kk-th largest counted item, scanning
// from the top: thread t owns bins [t * per, (t + 1) * per). Writes *s_bin and *s_above (the items in higher bins);
// *s_bin keeps its previous value when fewer than kk items were counted. All threads call it; it ends with a barrier.
template <int NT>
__device__ __forceinline__ void find_bin(const unsigned* hist, int nb, unsigned kk, unsigned* warp_tot, int* s_bin,
                                         unsigned* s_above) {
  const int per = nb > NT ? nb / NT : 1;
  const int b0 = threadIdx.x * per;
  unsigned mine = 0;
  for (int b = 0; b < per; ++b)
    if (b0 + b < nb) mine += hist[b0 + b];
  unsigned run = block_suffix_excl<NT>(mine, warp_tot);
  for (int b = per - 1; b >= 0; --b) {
    if (b0 + b >= nb) continue;
    const unsigned h = hist[b0 + b];
    if (run < kk && run + h >= kk) {
      *s_bin = b0 + b;
      *s_above = run;
    }
    run += h;
  }
  __syncthreads();
}

// Reserves n consecutive slots for each lane of the warp: an exclusive scan of n over the lanes and one shared
// atomic on *counter for the whole warp. Every lane of the warp calls it; returns this lane's first slot.
__device__ __forceinline__ int warp_reserve(int n, int* counter) {
  const int lane = threadIdx.x & 31;
  int incl = n;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  int base = 0;
  if (lane == 31 && incl > 0) base = atomicAdd(counter, incl);
  base = __shfl_sync(0xffffffffu, base, 31);
  return base + incl - n;
}

// One tile of the stream as this thread holds it: U vectors (vector u is the segment's vector vb + u * NT, present
// when below nv) and, on the first tile only, one element outside the aligned body.
template <typename T, int NT, int U>
struct TileRegs {
  uint4 r[U];
  int vb, nv;
  unsigned base_idx;  // column index of the segment's first body element
  bool has_x;
  unsigned xbits, xidx;
};

// Calls f(c) for every composite >= lo of this thread's tile.
template <typename T, int NT, int U, typename F>
__device__ __forceinline__ void for_each_at_least(const TileRegs<T, NT, U>& t, u64 lo, F&& f) {
  constexpr int V = VecN<T>::N;
  const T* tag = nullptr;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int v = t.vb + u * NT;
    if (v >= t.nv) continue;
    const unsigned idx0 = t.base_idx + (unsigned)(v * V);
#pragma unroll
    for (int e = 0; e < V; ++e) {
      const u64 c = composite(order_key(elem_bits(t.r[u], e, tag)), idx0 + (unsigned)e);
      if (c >= lo) f(c);
    }
  }
  if (t.has_x) {
    const u64 c = composite(order_key(t.xbits), t.xidx);
    if (c >= lo) f(c);
  }
}

// Appends the tile's composites >= lo to buf[off + ...] (entries past cap are dropped; *counter counts them all).
// A float compare per vector finds the few that may qualify; only those build their composites, and a warp that has
// any reserves its slots with one shared atomic. Every lane of every warp calls it.
template <typename T, int NT, int U>
__device__ __forceinline__ void collect(const TileRegs<T, NT, U>& t, u64 lo, u64* buf, int off, int* counter) {
  constexpr int cap = Cfg<NT>::kCand;
  constexpr int V = VecN<T>::N;
  const T* tag = nullptr;
  const float f_lo = __uint_as_float(key_bits((unsigned)(lo >> 32)));
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int v = t.vb + u * NT;
    const bool maybe = v < t.nv && !(vec_max_nan(t.r[u], tag) < f_lo);
    if (!__any_sync(0xffffffffu, maybe)) continue;
    const unsigned idx0 = t.base_idx + (unsigned)(v * V);
    unsigned take = 0u;
    if (maybe)
      for (unsigned m = vec_not_below(t.r[u], f_lo, tag); m; m &= m - 1u) {
        const int e = __ffs(m) - 1;
        if (composite(order_key(elem_bits(t.r[u], e, tag)), idx0 + (unsigned)e) >= lo) take |= 1u << e;
      }
    int pos = off + warp_reserve(__popc(take), counter);
    for (; take; take &= take - 1u, ++pos) {
      const int e = __ffs(take) - 1;
      if (pos < cap) buf[pos] = composite(order_key(elem_bits(t.r[u], e, tag)), idx0 + (unsigned)e);
    }
  }
  if (__any_sync(0xffffffffu, t.has_x)) {
    const u64 c = composite(order_key(t.xbits), t.xidx);
    const bool keep = t.has_x && c >= lo;
    const int pos = off + warp_reserve(keep ? 1 : 0, counter);
    if (keep && pos < cap) buf[pos] = c;
  }
}

// Records, for tiles after the first, each of this thread's vectors that may hold a composite >= lo (its largest value
// not below f_lo, NaN included) in its warp's slots: the vector and its index within the segment, at a place found
// by a ballot (no atomics, no composites; those are built when the slots are expanded). Returns the warp's new count;
// slots past the shape's kSlots are not written (the caller sees the count exceed them). Every lane of the warp calls
// it.
template <bool kFull, typename T, int NT, int U>
__device__ __forceinline__ int record(const TileRegs<T, NT, U>& t, float f_lo, uint4* wslot, unsigned* widx,
                                      int wcnt) {
  const T* tag = nullptr;
  const unsigned below = (1u << (threadIdx.x & 31)) - 1u;
  // The U tests and ballots are independent; one branch skips the (common) tile slice with nothing to record.
  bool maybe[U];
  unsigned bal[U], any = 0u;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int v = t.vb + u * NT;
    maybe[u] = (kFull || v < t.nv) && !(vec_max_nan(t.r[u], tag) < f_lo);
  }
#pragma unroll
  for (int u = 0; u < U; ++u) {
    bal[u] = __ballot_sync(0xffffffffu, maybe[u]);
    any |= bal[u];
  }
  if (any == 0u) return wcnt;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    if (maybe[u]) {
      const int pos = wcnt + __popc(bal[u] & below);
      if (pos < Cfg<NT, sizeof(T)>::kSlots) {
        if (kSlotData) wslot[pos] = t.r[u];
        widx[pos] = (unsigned)(t.vb + u * NT);
      }
    }
    wcnt += __popc(bal[u]);
  }
  return wcnt;
}

// Appends the composites >= lo of this warp's n recorded vectors (n <= kSlots, one per lane) to buf[off + ...]
// (entries past cap are dropped; *counter counts them all); with buf null it only counts them. Every lane of the
// warp calls it.
template <typename T, int cap>
__device__ __forceinline__ void expand(const uint4* wslot, const unsigned* widx, int n, unsigned base_idx, u64 lo,
                                       u64* buf, int off, int* counter) {
  constexpr int V = VecN<T>::N;
  const T* tag = nullptr;
  const int lane = threadIdx.x & 31;
  uint4 r = make_uint4(0u, 0u, 0u, 0u);
  unsigned idx0 = 0u, take = 0u;
  if (lane < n) {
    r = kSlotData ? wslot[lane] : __ldcg(wslot + widx[lane]);
    idx0 = base_idx + widx[lane] * (unsigned)V;
#pragma unroll
    for (int e = 0; e < V; ++e)
      if (composite(order_key(elem_bits(r, e, tag)), idx0 + (unsigned)e) >= lo) take |= 1u << e;
  }
  if (buf == nullptr) {
    const int sum = __reduce_add_sync(0xffffffffu, __popc(take));
    if (lane == 0 && sum > 0) atomicAdd(counter, sum);
    return;
  }
  int pos = off + warp_reserve(__popc(take), counter);
  for (; take; take &= take - 1u, ++pos) {
    const int e = __ffs(take) - 1;
    if (pos < cap) buf[pos] = composite(order_key(elem_bits(r, e, tag)), idx0 + (unsigned)e);
  }
}

// Calls f(c) for every composite >= lo of this warp's n recorded vectors (one per lane).
template <typename T, typename F>
__device__ __forceinline__ void for_each_recorded(const uint4* wslot, const unsigned* widx, int n, unsigned base_idx,
                                                  u64 lo, F&& f) {
  constexpr int V = VecN<T>::N;
  const T* tag = nullptr;
  const int lane = threadIdx.x & 31;
  if (lane >= n) return;
  const uint4 r = kSlotData ? wslot[lane] : __ldcg(wslot + widx[lane]);
  const unsigned idx0 = base_idx + widx[lane] * (unsigned)V;
#pragma unroll
  for (int e = 0; e < V; ++e) {
    const u64 c = composite(order_key(elem_bits(r, e, tag)), idx0 + (unsigned)e);
    if (c >= lo) f(c);
  }
}

// Radix select: the lower edge of the digit bin holding the kk-th largest of the items that each thread's
// items(f) visits, refined digit by digit (10 bits at a time from the top of the composite, so value ties resolve by
// index) until the items >= edge number at most cap (cap >= kk: the last digit leaves exactly kk). Every level
// rebuilds the histogram `hist` (the shape's kRadixBins words). All threads call it; it ends with a barrier.
template <int NT, typename Items>
__device__ u64 radix_edge(Items&& items, unsigned kk, int cap, unsigned* hist, unsigned* warp_tot, int* s_bin,
                          unsigned* s_above) {
  u64 prefix = 0, edge = 0;
  unsigned above_total = 0;
  using C = Cfg<NT>;
  for (int L = 0; L < C::kLevels; ++L) {
    const int sh = level_shift<C::kDigit>(L), w = level_width<C::kDigit>(L);
    const unsigned mask = (1u << w) - 1u;
    for (int i = threadIdx.x; i < C::kRadixBins; i += NT) hist[i] = 0u;
    if (threadIdx.x == 0) *s_bin = 0;
    __syncthreads();
    items([&](u64 c) {
      if (L == 0 || (c >> (sh + w)) == prefix) atomicAdd(&hist[(unsigned)(c >> sh) & mask], 1u);
    });
    __syncthreads();
    find_bin<NT>(hist, 1 << w, kk, warp_tot, s_bin, s_above);
    const int bin = *s_bin;
    const unsigned above = *s_above, inbin = hist[bin];
    const u64 next = (prefix << w) | (u64)bin;
    edge = next << sh;
    if (above_total + above + inbin <= (unsigned)cap || L == C::kLevels - 1) break;
    above_total += above;
    kk -= above;
    prefix = next;
    __syncthreads();  // every thread has read hist[bin] and the bin before the next level rewrites them
  }
  __syncthreads();  // the histogram is dead before the caller reuses its buffer
  return edge;
}

// The top k of the cnt distinct composites in cand, sorted, into top[0, k) (zero padded when cnt < k): a rank count,
// G lanes per candidate (G the largest power of two <= 32 with cnt * G <= kThreads), each lane comparing against
// every G-th candidate, the partial counts summed by xor shuffles. Ends with a barrier.
template <int NT>
__device__ __forceinline__ void select_top(const u64* cand, int cnt, int k, u64* top) {
  int g = 32;
  while (g > 1 && cnt * g > NT) g >>= 1;
  const int sub = threadIdx.x & (g - 1);
  for (int base = 0; base < cnt; base += NT / g) {  // uniform trip count: every lane joins the shuffles
    const int item = base + (int)threadIdx.x / g;
    u64 c = 0ull;
    int rank = 0;
    if (item < cnt) {
      c = cand[item];
#pragma unroll 4
      for (int j = sub; j < cnt; j += g) rank += cand[j] > c;
    }
    for (int o = g >> 1; o > 0; o >>= 1) rank += __shfl_xor_sync(0xffffffffu, rank, o);
    if (item < cnt && sub == 0 && rank < k) top[rank] = c;
  }
  for (int e = cnt + threadIdx.x; e < k; e += NT) top[e] = 0ull;
  __syncthreads();
}

// select_top when cand[0, np) is already sorted descending (the running top of the last compaction) and only
// cand[np, cnt) is new: an entry of the sorted prefix ranks at its index plus the new entries above it; a new entry
// at the prefix entries above it (binary search) plus the other new entries above it. Each rank counts cnt - np
// entries instead of cnt.
template <int NT>
__device__ __forceinline__ void select_top_sorted_prefix(const u64* cand, int np, int cnt, int k, u64* top) {
  int g = 32;
  while (g > 1 && cnt * g > NT) g >>= 1;
  const int sub = threadIdx.x & (g - 1);
  for (int base = 0; base < cnt; base += NT / g) {  // uniform trip count: every lane joins the shuffles
    const int item = base + (int)threadIdx.x / g;
    u64 c = 0ull;
    int rank = 0;
    if (item < cnt) {
      c = cand[item];
#pragma unroll 4
      for (int j = np + sub; j < cnt; j += g) rank += cand[j] > c;
      if (sub == 0) rank += item < np ? item : count_greater(cand, np, c);
    }
    for (int o = g >> 1; o > 0; o >>= 1) rank += __shfl_xor_sync(0xffffffffu, rank, o);
    if (item < cnt && sub == 0 && rank < k) top[rank] = c;
  }
  for (int e = cnt + threadIdx.x; e < k; e += NT) top[e] = 0ull;
  __syncthreads();
}

// Compaction: the top k of the n distinct composites in cand[0, n), sorted, into cand[0, k) (zero padded when
// n < k); returns min(k, n). cand[0, np) must be sorted descending (np = 0: no such prefix). Up to cap = max(k + 32, kDirectSelect) candidates (at most kPack) go straight to the
// rank count, whose cost grows with the square of the count; more are first narrowed by a radix select to at most
// cap, packed into tmp. tmp (kPack entries) is scratch. All threads call it; ends with a barrier.
template <int NT>
__device__ int compact(u64* cand, int np, int n, int k, u64* tmp, unsigned* warp_tot, int* s_bin,
                       unsigned* s_above, int* s_pack) {
  constexpr int kPack = Cfg<NT>::kPack;
  const int cap = min(kPack, max(kDirectSelect, k + 32));
  if (n <= cap) {
    if (np > 0) select_top_sorted_prefix<NT>(cand, np, n, k, tmp);
    else select_top<NT>(cand, n, k, tmp);
    for (int i = threadIdx.x; i < k; i += NT) cand[i] = tmp[i];
    __syncthreads();
    return min(k, n);
  }
  const u64 edge = radix_edge<NT>(
      [&](auto&& f) {
        for (int i = threadIdx.x; i < n; i += NT) f(cand[i]);
      },
      (unsigned)k, cap, reinterpret_cast<unsigned*>(tmp), warp_tot, s_bin, s_above);
  if (threadIdx.x == 0) *s_pack = 0;
  __syncthreads();
  for (int base = 0; base < n; base += NT) {  // uniform trip count: every lane joins warp_reserve
    const int i = base + threadIdx.x;
    const u64 c = i < n ? cand[i] : 0ull;
    const bool keep = i < n && c >= edge;
    const int pos = warp_reserve(keep ? 1 : 0, s_pack);
    if (keep && pos < kPack) tmp[pos] = c;
  }
  __syncthreads();
  select_top<NT>(tmp, min(*s_pack, kPack), k, cand);
  return min(k, n);
}

constexpr int kMaxPeers = 8;

// Modes 2 and 3 (vocab-sharded top-k over peer memory): each rank's exchange buffer holds, for the current call's
// parity, lists [world][rows][k] and flags [world][rows]; this rank writes its row lists into slot `rank` of every
// rank's buffer and then sets flag [rank][row] = epoch there. Mode 3 then also waits, per row, for every rank's list
// of the row in its own buffer and writes the merged top k (values / indices as mode 0). Flags are compared for
// equality: consecutive calls alternate parity, and any two calls on one parity carry different epochs.
struct PushArgs {
  u64* lists[kMaxPeers];        // every rank's lists base for this parity (this rank's own included)
  unsigned* flags[kMaxPeers];   // every rank's flags base for this parity
  int world, rank;
  unsigned epoch;
  long long rows;
};

struct SegArgs {
  const void* x;
  void* values;          // mode 0: [rows, k] in x's dtype
  long long* indices;    // mode 0: [rows, k]
  u64* lists;            // mode 1: [rows, k] sorted composites, zero padded
  u64* work;             // [rows, nseg, k] when a row has several segments
  unsigned* counters;    // [rows], zero on entry, left zero
  long long col_offset;  // added to every column index
  int cols, k, mode;
  PushArgs push;         // mode 2
  // Mode 4 (top-k sampling): values is float [rows, k] and receives softmax(top-k values * inv_temp) in rank order;
  // with uniforms (float [rows], in [0, 1)), samples[row] (int64) is the index of the first entry whose cumulative
  // probability exceeds uniforms[row].
  float inv_temp;
  const float* uniforms;
  long long* samples;
};

#ifdef CKB_TOPK_TRACE
// Measurement build only: per row, the global timer at the kernel's start, the end of the stream, the row's lists
// published (fence and flags), the peers' lists seen, and the row's end.
__device__ unsigned long long g_trace[65536][5];
#define TOPK_TRACE(row, i) \
  do { if (threadIdx.x == 0 && blockIdx.x == 0 && (row) < 65536) g_trace[row][i] = global_ns(); } while (0)
#else
#define TOPK_TRACE(row, i) ((void)0)
#endif

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Writes entry j of the row's final top k in the requested form.
template <typename T>
__device__ __forceinline__ void emit(const SegArgs& a, long long row, int j, u64 c) {
  if (a.mode == 0) {
    reinterpret_cast<T*>(a.values)[row * a.k + j] = decode_value<T>(c);
    a.indices[row * a.k + j] = decode_index(c);
  } else if (a.mode == 1) {
    a.lists[row * a.k + j] = c;
  } else {
    const long long at = ((long long)a.push.rank * a.push.rows + row) * a.k + j;
    for (int p = 0; p < a.push.world; ++p) a.push.lists[p][at] = c;  // NVLink stores to every rank (and itself)
  }
}

// Mode 4: the row's final top k (sorted composites in shared memory) as probabilities softmax(v * inv_temp) over the
// k values (fp32, the exponentials taken against the largest, their sum in fp64) with the int64 indices, and the
// sampled index when the launch has uniforms. The first warp does it (k <= 512: 16 entries per lane at most); an
// entry past the row's elements (zero padding) has probability 0 and is never sampled.
template <typename T>
__device__ void emit_probs(const SegArgs& a, long long row, const u64* list) {
  if (threadIdx.x >= 32) return;
  const int lane = threadIdx.x, k = a.k;
  float* probs = reinterpret_cast<float*>(a.values);
  const u64 c0 = list[0];
  const float v0 = to_f32(decode_value<T>(c0)) * a.inv_temp;
  double sum = 0.0;
  for (int i = lane; i < k; i += 32) {
    const u64 c = list[i];
    if (c != 0ull) sum += (double)expf(to_f32(decode_value<T>(c)) * a.inv_temp - v0);
  }
  sum = warp_sum(sum);
  const float inv = (float)(1.0 / sum);
  for (int i = lane; i < k; i += 32) {
    const u64 c = list[i];
    probs[row * k + i] = c != 0ull ? expf(to_f32(decode_value<T>(c)) * a.inv_temp - v0) * inv : 0.0f;
    a.indices[row * k + i] = c != 0ull ? decode_index(c) : -1;
  }
  if (a.uniforms == nullptr || a.samples == nullptr) return;
  // The first entry whose cumulative probability exceeds u (the last real entry when rounding leaves u above them
  // all), by a running scan over the lanes' chunks of 32 entries.
  const double u = (double)a.uniforms[row] * sum;
  double base = 0.0;
  long long pick = -1;
  for (int i0 = 0; i0 < k && pick < 0; i0 += 32) {
    const int i = i0 + lane;
    const u64 c = i < k ? list[i] : 0ull;
    double e = c != 0ull ? (double)expf(to_f32(decode_value<T>(c)) * a.inv_temp - v0) : 0.0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {  // inclusive scan
      const double y = __shfl_up_sync(0xffffffffu, e, o);
      if (lane >= o) e += y;
    }
    const unsigned hit = __ballot_sync(0xffffffffu, c != 0ull && base + e > u);
    if (hit) pick = decode_index(list[i0 + __ffs(hit) - 1]);
    base += __shfl_sync(0xffffffffu, e, 31);
  }
  if (pick < 0) {  // u at or above the total after rounding: the last real entry
    int last = k - 1;
    while (last > 0 && list[last] == 0ull) --last;
    pick = decode_index(list[last]);
  }
  if (lane == 0) a.samples[row] = pick;
}

// Mode 3, once the row is published: thread p < world waits (bounded) until rank p's list of the row is in this
// rank's buffer, then the block ranks the world lists in shared memory `sl` (world * k entries) and writes the row's
// final top k. The lists are read through L2: peers wrote them during this kernel's life.
template <typename T>
__device__ void merge_published(const SegArgs& a, long long row, int tid, int nthreads, u64* sl, int* s_timeout) {
  const int world = a.push.world, k = a.k;
  const long long rows = a.push.rows;
  if (tid < world) {
    const unsigned* f = a.push.flags[a.push.rank] + (long long)tid * rows + row;
    if (ld_acquire_sys(f) != a.push.epoch) {
      const unsigned long long start = global_ns();
      while (ld_acquire_sys(f) != a.push.epoch) {
        if (global_ns() - start > kWaitLimitNs) {
          *s_timeout = 1;
          break;
        }
        __nanosleep(64);
      }
    }
  }
  __syncthreads();
  TOPK_TRACE(row, 3);
  if (*s_timeout && tid == 0) atomicOr(&g_topk_status, CKB_STATUS_TIMEOUT);
  const u64* own = a.push.lists[a.push.rank];
  for (int i = tid; i < world * k; i += nthreads) {
    const int l = i / k, j = i - l * k;
    sl[i] = __ldcg(own + ((long long)l * rows + row) * k + j);
  }
  __syncthreads();
  for (int i = tid; i < world * k; i += nthreads) {
    const u64 c = sl[i];
    if (c == 0ull) continue;
    const int mine = i / k;
    int rank = i - mine * k;
    for (int l = 0; l < world && rank < k; ++l)
      if (l != mine) rank += count_greater(sl + l * k, k, c);
    if (rank < k) {
      reinterpret_cast<T*>(a.values)[row * k + rank] = decode_value<T>(c);
      a.indices[row * k + rank] = decode_index(c);
    }
  }
}

// Modes 2 and 3, after every emit of the row: the row's flag moves on each rank once every writer's stores (threads
// below k) are visible there. The block barrier orders the writers' stores before the flag stores, and each flag
// store is a release at system scope, which is cumulative: it makes every store it is ordered after (the other
// threads' included) visible to a peer that acquires the flag. One release per rank, not a system-scope fence per
// writer (the same pattern NCCL's proxies use: the data's threads meet at a barrier, one release publishes). Per-row
// timestamps on two B200s (-DCKB_TOPK_TRACE): publishing took 16.8 us per row with a fence per writer, 7 us with
// this.
__device__ __forceinline__ void publish_row(const SegArgs& a, long long row, int tid) {
  __syncthreads();
  if (tid < a.push.world) st_release_sys(a.push.flags[tid] + (long long)a.push.rank * a.push.rows + row, a.push.epoch);
  TOPK_TRACE(row, 2);
}

// The end of a segment: its sorted top k (cand[0, k), zero padded) becomes the row's output in the launch's mode, or,
// for a row split into several segments, goes to the workspace, and the row's last CTA (per-row counter, reset by it)
// merges the segments' lists in `scratch` (two halves of merge_entries composites, idle shared memory) and writes
// the output. All threads of the CTA call it.
template <typename T>
__device__ void finish_segment(const SegArgs& a, long long row, int seg, int nseg, const u64* cand, int k,
                               unsigned char* scratch, int merge_entries, int* s_last, int* s_timeout) {
  const int tid = threadIdx.x, nthreads = blockDim.x;
  if (nseg == 1) {
    if (a.mode == 4) {
      emit_probs<T>(a, row, cand);
      return;
    }
    for (int i = tid; i < k; i += nthreads) emit<T>(a, row, i, cand[i]);
    if (a.mode >= 2) publish_row(a, row, tid);
    if (a.mode == 3) merge_published<T>(a, row, tid, nthreads, reinterpret_cast<u64*>(scratch), s_timeout);
    return;
  }
  u64* wr = a.work + ((long long)row * nseg + seg) * k;
  // The writers (threads below k <= nthreads) fence their own stores before the row counter moves.
  if (tid < k) {
    wr[tid] = cand[tid];
    __threadfence();
  }
  __syncthreads();
  if (tid == 0) *s_last = atomicAdd(&a.counters[row], 1u) == (unsigned)nseg - 1u;
  __syncthreads();
  if (!*s_last) return;
  __threadfence();
  u64* la = reinterpret_cast<u64*>(scratch);  // the ring is idle: two halves of nseg * k <= merge_entries each
  u64* lb = la + merge_entries;
  const u64* rw = a.work + (long long)row * nseg * k;
  for (int i = tid; i < nseg * k; i += nthreads) la[i] = __ldcg(rw + i);
  __syncthreads();
  // Pairwise rounds: lists 2p and 2p + 1 become list p (an odd last list moves on as it is). An entry's place in the
  // merged list is its place in its own list plus the entries of the partner list above it; zero padding lands
  // behind every real entry.
  for (int n = nseg; n > 1; n = (n + 1) / 2) {
    for (int i = tid; i < n * k; i += nthreads) {
      const int l = i / k, e = i - l * k;
      const u64 c = la[i];
      int rank = e;
      if (!((n & 1) && l == n - 1)) rank += count_greater(la + (l ^ 1) * k, k, c);
      if (rank < k) lb[(l >> 1) * k + rank] = c;
    }
    __syncthreads();
    u64* sw = la;
    la = lb;
    lb = sw;
  }
  if (a.mode == 4) emit_probs<T>(a, row, la);
  else
    for (int i = tid; i < k; i += nthreads) emit<T>(a, row, i, la[i]);
  if (tid == 0) a.counters[row] = 0u;
  if (a.mode >= 2) publish_row(a, row, tid);  // its barrier also ends every read of la / lb in the ring
  if (a.mode == 3) merge_published<T>(a, row, tid, nthreads, reinterpret_cast<u64*>(scratch), s_timeout);
}

// Grid (nseg, rows). A row's 16-byte aligned body is split evenly into nseg segments of vectors; the elements before
// the body's first aligned address go with segment 0, those after its end with the last segment.
template <typename T, int NT>
__global__ void __launch_bounds__(NT, Cfg<NT>::kMinBlocks) topk_stream(const SegArgs a) {
  pdl_wait();
  pdl_trigger();
  TOPK_TRACE(blockIdx.y, 0);
  using C = Cfg<NT, sizeof(T)>;
  constexpr int V = VecN<T>::N;
  constexpr int kThreads = NT, kWarps = C::kWarps, kU = C::kU, kStages = C::kStages, kTileVecs = C::kTileVecs;
  constexpr int kRingBytes = C::kRingBytes, kMergeEntries = C::kMergeEntries;
  constexpr int kCand = C::kCand, kPack = C::kPack, kSlots = C::kSlots, kSlotsFull = C::kSlotsFull;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ unsigned warp_tot[kWarps];
  __shared__ unsigned warp_key[kWarps];
  __shared__ int s_bin;
  __shared__ unsigned s_above;
  __shared__ int s_cnt;     // appends of the current collect or expansion
  __shared__ int s_flag[3];  // tile j >= 1: bit 0 some warp's slots are half full, bit 1 some warp's overflowed
  __shared__ int s_pack;
  __shared__ int s_last;
  __shared__ int s_timeout;  // mode 3: a wait for a peer's list ran out

  if (threadIdx.x == 0) s_timeout = 0;
  const T* tag = nullptr;
  uint4* ring = reinterpret_cast<uint4*>(smem_raw);
  u64* cand = reinterpret_cast<u64*>(smem_raw + kRingBytes);  // running top at [0, ntop), survivors behind it
  u64* tmp = cand + kCand;  // compaction scratch: kPack composites or the radix histogram
  unsigned char* slots = smem_raw + kRingBytes + (kCand + kPack) * 8;
  uint4* wslot = reinterpret_cast<uint4*>(slots) + (threadIdx.x >> 5) * kSlots;  // this warp's recorded vectors
  unsigned* widx = reinterpret_cast<unsigned*>(slots + (kSlotData ? kWarps * kSlots * 16 : 0)) +
                   (threadIdx.x >> 5) * kSlots;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long row = blockIdx.y;
  const int seg = blockIdx.x, nseg = gridDim.x, k = a.k;
  const T* rowp = reinterpret_cast<const T*>(a.x) + row * (long long)a.cols;

  // The row's aligned body [head, tail0) in vectors, and this segment's share [v0, v0 + nv).
  const int mis = (int)((reinterpret_cast<uintptr_t>(rowp) & 15u) / sizeof(T));
  const int head = mis ? min(a.cols, V - mis) : 0;
  const int nvr = (a.cols - head) / V;
  const int tail0 = head + nvr * V;
  const int segv = (nvr + nseg - 1) / nseg;
  const int v0 = min(nvr, seg * segv);
  const int nv = min(nvr, v0 + segv) - v0;
  const uint4* body = reinterpret_cast<const uint4*>(rowp + head) + v0;
  const uint4* const rec_src = kSlotData ? wslot : body;  // where an expansion reads a recorded vector

  TileRegs<T, NT, kU> t;
  t.nv = nv;
  t.base_idx = (unsigned)(a.col_offset + head) + (unsigned)v0 * (unsigned)V;
  const int nhead = seg == 0 ? head : 0;
  const int nextra = nhead + (seg == nseg - 1 ? a.cols - tail0 : 0);  // at most 2 (V - 1)
  const bool mine_x = tid < nextra;
  t.xbits = 0u;
  t.xidx = 0u;
  if (mine_x) {
    const int col = tid < nhead ? tid : tail0 + (tid - nhead);
    t.xbits = scalar_bits(rowp[col]);
    t.xidx = (unsigned)(a.col_offset + col);
  }

  const int ntiles = max(1, (nv + kTileVecs - 1) / kTileVecs);
  const int full_tiles = nv / kTileVecs;  // tiles whose every vector lies in the segment
  constexpr int kFullLong = sizeof(T) == 2 ? CKB_TOPK_SLOTS_FULL_LONG_H : CKB_TOPK_SLOTS_FULL_LONG;
  const int slots_full =
      (long long)nv * V >= CKB_TOPK_LONG_ELEMS && kFullLong < kSlotsFull ? kFullLong : kSlotsFull;
  // Tile j's vectors of this thread into ring stage `stage`; one commit group per tile (empty past the last tile).
  auto issue = [&](int j, int stage) {
    if (j < ntiles) {
      const uint4* src = body + j * kTileVecs + tid;
      uint4* dst = ring + stage * kTileVecs + tid;
      if (j < full_tiles) {
#pragma unroll
        for (int u = 0; u < kU; ++u) cp_async16(dst + u * kThreads, src + u * kThreads);
      } else {
#pragma unroll
        for (int u = 0; u < kU; ++u)
          if (j * kTileVecs + u * kThreads + tid < nv) cp_async16(dst + u * kThreads, src + u * kThreads);
      }
    }
    cp_async_commit();
  };
  // This thread's vectors of tile j (landed in ring stage `stage`) into t; vectors past the segment read as NaN.
  auto load = [&](int j, int stage) {
    const uint4* st = ring + stage * kTileVecs + tid;
    t.vb = j * kTileVecs + tid;
    if (j < full_tiles) {
#pragma unroll
      for (int u = 0; u < kU; ++u) t.r[u] = st[u * kThreads];
    } else {
#pragma unroll
      for (int u = 0; u < kU; ++u)
        t.r[u] = t.vb + u * kThreads < nv ? st[u * kThreads]
                                           : make_uint4(0x7fc07fc0u, 0x7fc07fc0u, 0x7fc07fc0u, 0x7fc07fc0u);
    }
  };
  // The fraction of the segment in tiles 0..j.
  const float seg_elems = (float)nv * V + (float)nextra;
  auto seen_after = [&](int j) {
    return seg_elems > 0.0f ? ((float)min(nv, (j + 1) * kTileVecs) * V + (float)nextra) / seg_elems : 1.0f;
  };

  // Pass 0 speculates: the bound rises to the m-th largest composite seen so far (m sized so that the whole segment
  // almost surely holds k composites above it). The answer is exact when the final k-th composite reaches every
  // speculative bound used (then no element left out can rank in the top k); otherwise pass 1 streams the segment
  // again with guaranteed bounds only.
  int ntop = 0;    // entries of the running top in cand[0, ntop), sorted
  int filled = 0;  // survivors appended behind it since the last compaction
  u64 lo = 0;      // every composite that can still enter the top k (or, speculating, pass the check) is >= lo
  u64 spec = 0;    // the highest speculative bound used
  bool speculate = true;
  // lo is an element's own composite (or one above it, within the same key): an element not yet streamed has a larger
  // index, so one of equal value falls below lo and the float pre-filter of later tiles may drop equal values.
  bool lo_strict = false;
  auto set_lo = [&](u64 v, bool strict) {
    if (v > lo) {
      lo = v;
      lo_strict = strict;
    } else if (v == lo && strict) {
      lo_strict = true;
    }
  };
  // The bound after a compaction that left a full top k: one above its k-th entry (strict unless the +1 carries into
  // the key, which happens only for index 0).
  auto raise_to = [&](u64 kth) {
    if (kth != ~0ull) set_lo(kth + 1ull, (unsigned)kth != 0xffffffffu);
  };

  // Appends the current collect's or expansion's count (all threads call it, after the appends and a barrier).
  auto take_count = [&]() {
    filled = min(filled + s_cnt, kCand - ntop);
    __syncthreads();  // every thread has read s_cnt before the next reset
  };
  // The top k of cand, a guaranteed bound from its k-th entry and, speculating, a speculative one from its m-th
  // (after `seen` elements of the segment).
  auto compact_all = [&](float seen) {  // seen < 0: no speculative bound
    ntop = compact<NT>(cand, ntop, ntop + filled, k, tmp, warp_tot, &s_bin, &s_above, &s_pack);
    filled = 0;
    if (ntop == k) {
      raise_to(cand[k - 1]);
      if (speculate && seen >= 0.0f) {
        const int m = spec_rank(k, seen);
        if (m < k) {
          const u64 s_m = cand[m - 1];
          spec = s_m > spec ? s_m : spec;
          set_lo(s_m, true);
        }
      }
    }
  };
  // The composites >= lo of the tile held in registers into cand; a tile that overflows the buffer (heavy ties, rising
  // values) first compacts what is there and raises lo until its composites fit.
  auto collect_tile = [&]() {
    if (tid == 0) s_cnt = 0;
    __syncthreads();
    collect(t, lo, cand, ntop + filled, &s_cnt);
    __syncthreads();
    if (ntop + filled + s_cnt > kCand) {
      __syncthreads();  // every thread has read s_cnt
      ntop = compact<NT>(cand, ntop, ntop + filled, k, tmp, warp_tot, &s_bin, &s_above, &s_pack);
      filled = 0;
      if (ntop == k) raise_to(cand[k - 1]);
      const u64 edge = radix_edge<NT>([&](auto&& f) { for_each_at_least(t, lo, f); }, (unsigned)k, kCand - ntop,
                                  reinterpret_cast<unsigned*>(tmp), warp_tot, &s_bin, &s_above);
      set_lo(edge, false);
      if (tid == 0) s_cnt = 0;
      __syncthreads();
      collect(t, lo, cand, ntop, &s_cnt);
      __syncthreads();
    }
    take_count();
  };
  // Every warp's first n recorded vectors (n per warp) into cand. Their composites >= lo are counted first; when they
  // do not fit, cand is compacted, and if they still do not fit (heavy ties) lo rises by a radix select over them.
  auto expand_all = [&](int n) {
    n = min(n, kSlots);
    if (ntop + filled + kWarps * kSlots * V <= kCand) {  // every composite of every slot fits: no count needed
      if (tid == 0) s_cnt = 0;
      __syncthreads();
      expand<T, kCand>(rec_src, widx, n, t.base_idx, lo, cand, ntop + filled, &s_cnt);
      __syncthreads();
      take_count();
      return;
    }
    if (tid == 0) s_cnt = 0;
    __syncthreads();
    expand<T, kCand>(rec_src, widx, n, t.base_idx, lo, nullptr, 0, &s_cnt);
    __syncthreads();
    const int need = s_cnt;
    __syncthreads();
    if (need == 0) return;
    if (ntop + filled + need > kCand) compact_all(-1.0f);
    if (ntop + filled + need > kCand) {
      const u64 edge = radix_edge<NT>(
          [&](auto&& f) { for_each_recorded<T>(rec_src, widx, n, t.base_idx, lo, f); }, (unsigned)k, kCand - ntop,
          reinterpret_cast<unsigned*>(tmp), warp_tot, &s_bin, &s_above);
      set_lo(edge, false);
    }
    if (tid == 0) s_cnt = 0;
    __syncthreads();
    expand<T, kCand>(rec_src, widx, n, t.base_idx, lo, cand, ntop + filled, &s_cnt);
    __syncthreads();
    take_count();
  };

  // The c-th largest per-thread maximum of each warp over the tile in registers (and the extra element), smallest over
  // the warps, as a key: c * warps elements of the tile are at or above it. Key 0 (no number's key) when a warp holds
  // fewer than c numbers: no bound. All threads call it; it ends with a barrier.
  auto tile_bound = [&](int c) -> unsigned {
    float fm = __int_as_float(0x7fc00000);
#pragma unroll
    for (int u = 0; u < kU; ++u) fm = vec_max(t.r[u], fm, tag);
    if (t.has_x) fm = max3(fm, __uint_as_float(t.xbits), __uint_as_float(t.xbits));
    // A bitonic sort of the 32 keys across the lanes, descending: lane l ends with the (l + 1)-th largest.
    unsigned key = fm == fm ? order_key(__float_as_uint(fm)) : 0u;
#pragma unroll
    for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        const unsigned o = __shfl_xor_sync(0xffffffffu, key, stride);
        const bool keep_max = ((lane & stride) == 0) == ((lane & size) == 0);
        key = keep_max ? max(key, o) : min(key, o);
      }
    }
    const unsigned wk = __shfl_sync(0xffffffffu, key, c - 1);
    if (lane == 0) warp_key[warp] = wk;
    __syncthreads();
    unsigned b = warp_key[0];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) b = min(b, warp_key[w]);
    return b;
  };
  // The float pre-filter of later tiles for the bound lo: the value of lo's key, or, when lo is strict, the next float
  // above it (equal values cannot pass; -0 keeps the plain form, since +0 compares equal to it as a float but ranks
  // above it).
  auto prefilter = [&]() {
    const unsigned kb = key_bits((unsigned)(lo >> 32));
    float f = __uint_as_float(kb);
    if (CKB_TOPK_STRICT && lo_strict && kb != 0x80000000u && f == f && f != CUDART_INF_F)
      f = __uint_as_float((kb & 0x80000000u) ? kb - 1u : kb + 1u);
    return f;
  };

  for (int pass = 0; pass < 2; ++pass) {
    speculate = pass == 0;
#pragma unroll
    for (int j = 0; j < kStages - 1; ++j) issue(j, j);
    for (int i = tid; i < k; i += kThreads) cand[i] = 0ull;
    if (tid < 3) s_flag[tid] = 0;
    ntop = 0;
    filled = 0;
    lo = 0;
    spec = 0;

    // Tile 0: the bound, every composite at or above it, and a first compaction that sets the running bounds.
    const int c_full = (k + kWarps - 1) / kWarps;
    issue(kStages - 1, kStages - 1);
    cp_async_wait<kStages - 1>();
    load(0, 0);
    t.has_x = mine_x;
    lo = (u64)tile_bound(c_full) << 32;
    lo_strict = false;
    collect_tile();
    compact_all(seen_after(0));
    t.has_x = false;

    // Later tiles: record the vectors that may hold a survivor; expand and compact only when a warp's slots fill.
    int wcnt = 0;                           // this warp's recorded vectors
    int rs = kStages > 1 ? 1 % kStages : 0;  // ring stage of tile j
    int fs = 1;                             // s_flag word of tile j
    float f_lo = prefilter();
    for (int j = 1; j < ntiles; ++j) {
      issue(j + kStages - 1, rs == 0 ? kStages - 1 : rs - 1);  // into the stage tile j - 1 left
      cp_async_wait<kStages - 1>();                            // this thread's copies of tile j have landed
      load(j, rs);
      const int before = wcnt;
      wcnt = j < full_tiles ? record<true>(t, f_lo, wslot, widx, wcnt) : record<false>(t, f_lo, wslot, widx, wcnt);
      if (lane == 0 && wcnt >= slots_full) atomicOr(&s_flag[fs], wcnt > kSlots ? 3 : 1);
      const int fnext = fs == 2 ? 0 : fs + 1;
      if (tid == 0) s_flag[fnext] = 0;  // its last reads came before the barrier of tile j - 1
      __syncthreads();
      const int flag = s_flag[fs];
      if (flag & 2) {
        // Some warp overflowed: keep every warp's records from earlier tiles, take this tile from registers, after
        // raising the bound to the tile's own guaranteed bound (k of its elements are at or above it), so a tile of
        // rising values collects about k composites instead of all of them.
        expand_all(before);
        wcnt = 0;
        if (CKB_TOPK_OVF_BOUND) set_lo((u64)tile_bound(c_full) << 32, false);
        collect_tile();
        compact_all(seen_after(j));
        f_lo = prefilter();
      } else if (flag & 1) {
        expand_all(wcnt);
        wcnt = 0;
        if (filled > 0) compact_all(seen_after(j));
        f_lo = prefilter();
      }
      rs = rs + 1 == kStages ? 0 : rs + 1;
      fs = fnext;
    }
    expand_all(wcnt);
    if (filled > 0) ntop = compact<NT>(cand, ntop, ntop + filled, k, tmp, warp_tot, &s_bin, &s_above, &s_pack);
    cp_async_wait<0>();
    if (spec == 0ull || (ntop == k && cand[k - 1] >= spec)) break;
    __syncthreads();  // every thread has read cand[k - 1] before the second pass clears the buffer
  }

  TOPK_TRACE(row, 1);
  finish_segment<T>(a, row, seg, nseg, cand, k, smem_raw, kMergeEntries, &s_last, &s_timeout);
  TOPK_TRACE(row, 4);
}


// Merge of nlists sorted composite lists per row, lists laid out [nlists][rows][k] (an all-gather's output); one
// CTA per row writes the top k values and indices.
template <typename T>
__global__ void __launch_bounds__(256) topk_merge(const u64* __restrict__ lists, int nlists, long long rows, int k,
                                                  T* __restrict__ values, long long* __restrict__ indices) {
  pdl_wait();
  pdl_trigger();
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

// Merge of the vocab-sharded variant over peer memory: lists [world][rows][k] and flags [world][rows] in this rank's
// exchange buffer (this call's parity). Thread p < world of row `row`'s CTA waits (bounded) until rank p has
// published the row for this epoch; the lists are then read through L2 (peers wrote them during this kernel's life,
// so not through the read-only path) and ranked as in topk_merge. A wait that runs out sets the status word.
template <typename T>
__global__ void __launch_bounds__(256) topk_merge_wait(const u64* lists, const unsigned* flags, int world,
                                                       unsigned epoch, long long rows, int k, T* __restrict__ values,
                                                       long long* __restrict__ indices) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) u64 sl[];
  __shared__ int s_timeout;
  const long long row = blockIdx.x;
  if (threadIdx.x == 0) s_timeout = 0;
  __syncthreads();
  if (threadIdx.x < world) {
    const unsigned* f = flags + (long long)threadIdx.x * rows + row;
    if (ld_acquire_sys(f) != epoch) {
      const unsigned long long start = global_ns();
      while (ld_acquire_sys(f) != epoch) {
        if (global_ns() - start > kWaitLimitNs) {
          s_timeout = 1;
          break;
        }
        __nanosleep(64);
      }
    }
  }
  __syncthreads();
  if (s_timeout && threadIdx.x == 0) atomicOr(&g_topk_status, CKB_STATUS_TIMEOUT);
  const int total = world * k;
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int l = i / k, j = i - l * k;
    sl[i] = __ldcg(lists + ((long long)l * rows + row) * k + j);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const u64 c = sl[i];
    if (c == 0ull) continue;
    const int own = i / k;
    int rank = i - own * k;
    for (int l = 0; l < world && rank < k; ++l)
      if (l != own) rank += count_greater(sl + l * k, k, c);
    if (rank < k) {
      values[row * k + rank] = decode_value<T>(c);
      indices[row * k + rank] = decode_index(c);
    }
  }
}

// The CTA shape. 256 threads (4 CTAs per SM) when k fits its bound and the batch has at least two rows per SM:
// every row streams in its own CTA, all in one wave. Smaller batches (and k > 256) take 512 threads (2 per SM), the
// deeper ring per CTA, and split rows to fill the GPU.
inline bool narrow_for(long long rows, int k) {
  return !CKB_TOPK_WIDE_ONLY && k <= Cfg<256>::kMaxK && rows >= 2LL * device_sm_count();
}

// Segments per row (each at least min_chunk columns, at most kMaxSeg): one row per CTA once the batch fills the GPU,
// otherwise about one CTA per SM in all (measured on B200: more CTAs of the 512-thread shape gain nothing, and each
// split adds a merge).
long long plan_seg(long long rows, long long cols, int elem, int min_chunk) {
  (void)elem;
  if (rows <= 0 || cols <= 0) return cols > 0 ? cols : 1;
  if (min_chunk < 1024) min_chunk = 1024;
  long long n = 1;
  if (rows < 2LL * device_sm_count()) {
    n = device_sm_count() / rows;
    if (n > kMaxSeg) n = kMaxSeg;
    if (n > cols / min_chunk) n = cols / min_chunk;
    if (n < 1) n = 1;
  }
  return (cols + n - 1) / n;
}

// Sets the kernel's shared-memory limit once per device.
template <typename T, int NT>
cudaError_t prepare_stream_kernel() {
  static std::atomic<unsigned long long> done{0ull};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = 1ull << (dev & 63);
  if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
  e = cudaFuncSetAttribute(topk_stream<T, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           Cfg<NT, sizeof(T)>::kSmemBytes);
  if (e != cudaSuccess) return e;
  done.fetch_or(bit, std::memory_order_acq_rel);
  return cudaSuccess;
}

template <typename T, int NT>
int start_shape(const SegArgs& a, long long rows, long long nseg, cudaStream_t s) {
  const cudaError_t e = prepare_stream_kernel<T, NT>();
  if (e != cudaSuccess) {
    cudaGetLastError();
    return (int)e;
  }
  launch_pdl(topk_stream<T, NT>, dim3((unsigned)nseg, (unsigned)rows), dim3(NT), Cfg<NT, sizeof(T)>::kSmemBytes, s,
             a);
  return (int)cudaGetLastError();
}

template <typename T>
int start_seg(const SegArgs& a, long long rows, long long nseg, cudaStream_t s) {
  return narrow_for(rows, a.k) ? start_shape<T, 256>(a, rows, nseg, s) : start_shape<T, 512>(a, rows, nseg, s);
}

long long segments(long long cols, long long chunk) { return (cols + chunk - 1) / chunk; }

// CTAs of the shape start_seg picks that the GPU holds at once (0 on error).
template <typename T, int NT>
long long resident_ctas() {
  if (prepare_stream_kernel<T, NT>() != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, topk_stream<T, NT>, NT, Cfg<NT, sizeof(T)>::kSmemBytes) !=
      cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return (long long)per_sm * device_sm_count();
}
template <typename T>
long long resident_for(long long rows, int k) {
  return narrow_for(rows, k) ? resident_ctas<T, 256>() : resident_ctas<T, 512>();
}

// The reference's argument checks (topk/kernel.cu:551-554) plus this library's limits: an element-aligned x and
// at most the shape's merge capacity (segments x k composites) for a split row.
bool bad_args(const void* x, long long rows, long long cols, int k, long long chunk, int elem) {
  if (k > cols || k > kMaxK || cols > INT_MAX / 2 || rows > 65535 || chunk <= 0) return true;
  if (reinterpret_cast<uintptr_t>(x) % (uintptr_t)elem) return true;
  if (chunk > cols) chunk = cols;
  const long long cap = narrow_for(rows, k) ? (elem == 4 ? Cfg<256, 4>::kMergeEntries : Cfg<256, 2>::kMergeEntries)
                                            : (elem == 4 ? Cfg<512, 4>::kMergeEntries : Cfg<512, 2>::kMergeEntries);
  return segments(cols, chunk) * k > cap;
}

}  // namespace
}  // namespace ckb

using namespace ckb;

// Replaces the reference's top-k `plan` (topk/kernel.cu:520-547): the columns per CTA for a rows x cols launch
// (dtype 0 fp32, 1 bf16). `threads` and `depth` are the reference's kernel knobs and do not change the B200 plan;
// min_chunk is a lower bound on the columns per CTA when a row is split. A row's segment count is
// ceil(cols / chunk); the workspace launch() needs is rows * segments * k int64 values.
CKB_EXPORT long long plan(long long rows, long long cols, int dtype, int threads, int depth, int min_chunk) {
  (void)threads;
  (void)depth;
  return plan_seg(rows, cols, dtype == kBF16 ? 2 : 4, min_chunk);
}

// Replaces the reference's top-k `launch` (topk/kernel.cu:549-570): same arguments, checks and return codes. work is
// int64 [rows * segments * k] (unused with one segment), counters int32 [rows] zeroed once and left zeroed by the
// kernel. Any chunk >= 1 is served while segments * k fits the last CTA's merge (2048 to 6144 composites by launch
// shape and dtype; beyond it -1); plan() gives the fastest.
CKB_EXPORT int launch(const void* x, void* values, void* indices, void* work, void* counters, long long rows,
                      long long cols, int k, int dtype, int threads, int depth, long long chunk,
                      cudaStream_t stream) {
  if (rows <= 0 || k <= 0) return 0;
  if (threads != 128 && threads != 256 && threads != 512) return -1;
  if (depth != 2 && depth != 4 && depth != 8) return -1;
  if (dtype != kF32 && dtype != kBF16) return -1;
  const int elem = dtype == kBF16 ? 2 : 4;
  if (bad_args(x, rows, cols, k, chunk, elem)) return -1;
  if (chunk > cols) chunk = cols;
  const SegArgs a{x, values, (long long*)indices, nullptr, (u64*)work, (unsigned*)counters, 0, (int)cols, k, 0};
  if (dtype == kF32) return start_seg<float>(a, rows, segments(cols, chunk), stream);
  return start_seg<__nv_bfloat16>(a, rows, segments(cols, chunk), stream);
}

// Top-k sampling (no counterpart in the reference): the top k of each row as launch() finds them, then the softmax
// over those k logits divided by `temperature` (probs float [rows, k], rank order) with their int64 indices, and with
// uniforms (float [rows], each in [0, 1)) the sampled token of each row into samples (int64 [rows]). work, counters
// and chunk as in launch() (chunk from plan()). Returns 0, -1 for a rejected argument (launch()'s, a temperature
// that is not a positive finite number, or only one of uniforms / samples), or the launch's cudaError_t.
CKB_EXPORT int ckb_topk_softmax_launch(const void* x, float* probs, long long* indices, void* work, void* counters,
                                       long long rows, long long cols, int k, int dtype, long long chunk,
                                       float temperature, const float* uniforms, long long* samples,
                                       cudaStream_t stream) {
  if (rows <= 0 || k <= 0) return 0;
  if (dtype != kF32 && dtype != kBF16) return -1;
  if (!(temperature > 0.0f) || !(temperature < INFINITY) || (uniforms == nullptr) != (samples == nullptr)) return -1;
  if (probs == nullptr || indices == nullptr) return -1;
  const int elem = dtype == kBF16 ? 2 : 4;
  if (bad_args(x, rows, cols, k, chunk, elem)) return -1;
  if (chunk > cols) chunk = cols;
  SegArgs a{x, probs, indices, nullptr, (u64*)work, (unsigned*)counters, 0, (int)cols, k, 4};
  a.inv_temp = 1.0f / temperature;
  a.uniforms = uniforms;
  a.samples = samples;
  if (dtype == kF32) return start_seg<float>(a, rows, segments(cols, chunk), stream);
  return start_seg<__nv_bfloat16>(a, rows, segments(cols, chunk), stream);
}

// Top-k of a column shard for the vocab-sharded variant (no counterpart in the reference): x is [rows, cols] holding
// global columns [col_offset, col_offset + cols); lists receives [rows, k] sorted composites (uint64, zero padded)
// carrying global indices, ready for an all-gather and ckb_topk_merge_launch. work/counters/chunk as in launch().
CKB_EXPORT int ckb_topk_shard_launch(const void* x, unsigned long long* lists, void* work, void* counters,
                                     long long rows, long long cols, long long col_offset, int k, int dtype,
                                     long long chunk, cudaStream_t stream) {
  if (rows <= 0 || k <= 0) return 0;
  if (dtype != kF32 && dtype != kBF16) return -1;
  const int elem = dtype == kBF16 ? 2 : 4;
  if (col_offset < 0 || col_offset + cols > INT_MAX / 2 || bad_args(x, rows, cols, k, chunk, elem)) return -1;
  if (chunk > cols) chunk = cols;
  const SegArgs a{x, nullptr, nullptr, lists, (u64*)work, (unsigned*)counters, col_offset, (int)cols, k, 1};
  if (dtype == kF32) return start_seg<float>(a, rows, segments(cols, chunk), stream);
  return start_seg<__nv_bfloat16>(a, rows, segments(cols, chunk), stream);
}

// Final merge of the vocab-sharded variant (no counterpart in the reference): lists [nlists][rows][k] of sorted
// composites (one list per shard) -> values [rows, k] in the dtype (0 fp32, 1 bf16) and int64 indices [rows, k].
CKB_EXPORT int ckb_topk_merge_launch(const unsigned long long* lists, int nlists, void* values, void* indices,
                                     long long rows, int k, int dtype, cudaStream_t stream) {
  if (rows <= 0 || k <= 0) return 0;
  if (nlists <= 0 || k > kMaxK || rows > INT_MAX) return -1;
  const long long smem = (long long)nlists * k * 8;
  if (smem > 96 * 1024) return -1;
  if (dtype == kF32) {
    if (cudaFuncSetAttribute(topk_merge<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
      return (int)cudaGetLastError();
    launch_pdl(topk_merge<float>, dim3((unsigned)rows), dim3(256), (size_t)smem, stream, (const u64*)lists, nlists,
               rows, k, (float*)values, (long long*)indices);
  } else if (dtype == kBF16) {
    if (cudaFuncSetAttribute(topk_merge<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
      return (int)cudaGetLastError();
    launch_pdl(topk_merge<__nv_bfloat16>, dim3((unsigned)rows), dim3(256), (size_t)smem, stream, (const u64*)lists,
               nlists, rows, k, (__nv_bfloat16*)values, (long long*)indices);
  } else {
    return -1;
  }
  return (int)cudaGetLastError();
}

// Vocab-sharded variant over peer memory (no counterpart in the reference): as ckb_topk_shard_launch, but each row's
// sorted list goes to slot `rank` of every rank's exchange buffer (lists[p] + (rank * rows + row) * k for p < world,
// NVLink stores) and flags[p][rank * rows + row] is then set to `epoch` (release, system scope). lists / flags are
// host arrays of `world` device pointers (this call's parity of each rank's buffer, this rank's own included).
// With values / indices null that is all (ckb_topk_merge_wait_launch merges later). With them, the final top k of
// the full rows is written too: by the same kernel when all of its CTAs fit on the GPU at once (each row's CTA waits
// for the other ranks' lists of its row, then merges), otherwise by a merge-wait launch behind it on `stream`.
// 1 <= world <= 8, 0 <= rank < world, epoch != 0.
CKB_EXPORT int ckb_topk_shard_push_launch(const void* x, void* values, void* indices, void* work, void* counters,
                                          long long rows, long long cols, long long col_offset, int k, int dtype,
                                          long long chunk, unsigned long long* const* lists, unsigned* const* flags,
                                          int world, int rank, unsigned epoch, cudaStream_t stream) {
  if (rows <= 0 || k <= 0) return 0;
  if (dtype != kF32 && dtype != kBF16) return -1;
  if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world || epoch == 0u || !lists || !flags) return -1;
  if ((values == nullptr) != (indices == nullptr)) return -1;
  const int elem = dtype == kBF16 ? 2 : 4;
  if (col_offset < 0 || col_offset + cols > INT_MAX / 2 || bad_args(x, rows, cols, k, chunk, elem)) return -1;
  if (chunk > cols) chunk = cols;
  SegArgs a{x, values, (long long*)indices, nullptr, (u64*)work, (unsigned*)counters, col_offset, (int)cols, k, 2, {}};
  for (int p = 0; p < world; ++p) {
    if (!lists[p] || !flags[p]) return -1;
    a.push.lists[p] = (u64*)lists[p];
    a.push.flags[p] = flags[p];
  }
  a.push.world = world;
  a.push.rank = rank;
  a.push.epoch = epoch;
  a.push.rows = rows;
  const long long nseg = segments(cols, chunk);
  if (values) {
    const long long cap = dtype == kF32 ? resident_for<float>(rows, k) : resident_for<__nv_bfloat16>(rows, k);
    if (rows * nseg <= cap) a.mode = 3;
  }
  const int err = dtype == kF32 ? start_seg<float>(a, rows, nseg, stream) : start_seg<__nv_bfloat16>(a, rows, nseg, stream);
  if (err || !values || a.mode == 3) return err;
  return ckb_topk_merge_wait_launch(lists[rank], flags[rank], world, epoch, values, indices, rows, k, dtype, stream);
}

// Vocab-sharded variant over peer memory, merge half (no counterpart in the reference): lists [world][rows][k] and
// flags [world][rows] are this rank's exchange buffer (this call's parity). Each row waits until every rank has
// published it for `epoch` (at most 2 s; then the status word records the timeout and the row is merged from
// whatever is there), then values [rows, k] (dtype 0 / 1) and int64 indices [rows, k] as ckb_topk_merge_launch.
CKB_EXPORT int ckb_topk_merge_wait_launch(const unsigned long long* lists, const unsigned* flags, int world,
                                          unsigned epoch, void* values, void* indices, long long rows, int k,
                                          int dtype, cudaStream_t stream) {
  if (rows <= 0 || k <= 0) return 0;
  if (world < 1 || world > kMaxPeers || epoch == 0u || k > kMaxK || rows > INT_MAX || !lists || !flags) return -1;
  const int smem = world * k * 8;
  if (dtype == kF32) {
    if (cudaFuncSetAttribute(topk_merge_wait<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
        cudaSuccess)
      return (int)cudaGetLastError();
    launch_pdl(topk_merge_wait<float>, dim3((unsigned)rows), dim3(256), (size_t)smem, stream, (const u64*)lists,
               flags, world, epoch, rows, k, (float*)values, (long long*)indices);
  } else if (dtype == kBF16) {
    if (cudaFuncSetAttribute(topk_merge_wait<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
        cudaSuccess)
      return (int)cudaGetLastError();
    launch_pdl(topk_merge_wait<__nv_bfloat16>, dim3((unsigned)rows), dim3(256), (size_t)smem, stream,
               (const u64*)lists, flags, world, epoch, rows, k, (__nv_bfloat16*)values, (long long*)indices);
  } else {
    return -1;
  }
  return (int)cudaGetLastError();
}

// Exchange buffers for the peer-memory variant: device memory of `bytes` (zeroed) that other processes can map
// through a 64-byte CUDA IPC handle. alloc/free on the owning process; export gives the handle of an alloc'd base
// pointer; import maps a peer's handle (peer access enabled lazily) and close unmaps it. Each returns 0 or the
// cudaError_t.
CKB_EXPORT int ckb_p2p_alloc(void** ptr, unsigned long long bytes) {
  if (!ptr || bytes == 0) return -1;
  cudaError_t e = cudaMalloc(ptr, (size_t)bytes);
  if (e != cudaSuccess) return (int)e;
  e = cudaMemset(*ptr, 0, (size_t)bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  return (int)e;
}
CKB_EXPORT int ckb_p2p_free(void* ptr) { return (int)cudaFree(ptr); }
CKB_EXPORT int ckb_p2p_export(const void* ptr, void* handle) {
  if (!ptr || !handle) return -1;
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
  if (e != cudaSuccess) return (int)e;
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  memcpy(handle, &h, sizeof(h));
  return 0;
}
CKB_EXPORT int ckb_p2p_import(const void* handle, void** ptr) {
  if (!handle || !ptr) return -1;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return (int)cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
}
CKB_EXPORT int ckb_p2p_close(void* ptr) { return (int)cudaIpcCloseMemHandle(ptr); }

#ifdef CKB_TOPK_TRACE
CKB_EXPORT int ckb_topk_trace(void* out, int rows) {
  if (rows < 0 || rows > 65536) return -1;
  return (int)cudaMemcpyFromSymbol(out, g_trace, (size_t)rows * 5 * 8);
}
#endif

// Status word of this library's kernels since the last reset: 0 fine, 1 when a wait on a peer's per-row flag (the
// vocab-sharded variant over peer memory) ran out. Synchronises with the device; reset != 0 clears the word.
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
// counters (up to 65536 rows), the rest the segment workspace (491,520 composites: rows * segments * k at most that).
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
// would with min_chunk 2048, except that a plan whose split rows would need more than the scratch's 491,520
// composites of workspace runs each row in one piece. Allocates nothing. Returns 0, -1 for arguments launch() would
// also reject (more than 65,535 rows among them, so the scratch's 65,536 counters always suffice), or a cudaError_t.
// The first call on a device looks up the scratch address (make it before any stream capture) and caches it for the
// life of the process: after a cudaDeviceReset the cached address is stale, so a device reset is not supported once
// this entry point has been called on that device. Every call shares the one scratch array, so calls that overlap on
// the GPU (different streams, no ordering between them) race; calls on one stream are ordered. The counters are
// cleared on the caller's stream at each call.
CKB_EXPORT int ckb_topk_launch_noalloc(const void* x, void* values, void* indices, long long rows, long long cols,
                                       int k, int dtype, cudaStream_t stream) {
  if (rows <= 0 || k <= 0) return 0;
  if (dtype != kF32 && dtype != kBF16) return -1;
  const int elem = dtype == kBF16 ? 2 : 4;
  long long chunk = plan_seg(rows, cols, elem, 2048);
  if (bad_args(x, rows, cols, k, chunk, elem)) return -1;
  if (chunk > cols) chunk = cols;
  long long nseg = segments(cols, chunk);
  if (nseg > 1 && rows * nseg * k > kNoAllocWorkWords) nseg = 1;  // whole rows: no workspace at all
  static_assert(2 * kNoAllocCounterWords > 65535, "bad_args() bounds rows by the scratch's counters");
  void* base = nullptr;
  cudaError_t e = noalloc_scratch(&base);
  if (e != cudaSuccess) return (int)e;
  unsigned* counters = reinterpret_cast<unsigned*>(base);
  u64* work = reinterpret_cast<u64*>(base) + kNoAllocCounterWords;
  if (nseg > 1) {
    e = cudaMemsetAsync(counters, 0, (size_t)rows * sizeof(unsigned), stream);
    if (e != cudaSuccess) return (int)e;
  }
  const SegArgs a{x, values, (long long*)indices, nullptr, work, counters, 0, (int)cols, k, 0};
  if (dtype == kF32) return start_seg<float>(a, rows, nseg, stream);
  return start_seg<__nv_bfloat16>(a, rows, nseg, stream);
}
