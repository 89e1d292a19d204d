// Row-wise softmax over the last dim: y = exp(x - max) / sum(exp(x - max)), fp32 (dtype 0) and bf16 (dtype 1) rows,
// every value computed in fp32. Semantics follow the reference's torch.softmax(x, dim=-1) (softmax/baseline.py:12-13);
// the C entry keeps the reference's ABI (softmax/kernel.cu:520-527).
//
// Paths, chosen by row length (all read each element once from HBM and write it once):
//   * group path, rows of at most 256 16-byte vectors: G = 4..32 lanes per row, so one warp holds 32 / G rows and
//     every lane keeps NV vectors of its row in registers; group-local shuffles, no barrier;
//   * block path, rows of at most 32768 fp32 / bf16 values: one block per row, 32 values per thread in
//     registers, two barriers per row;
//   * cluster path, longer rows: a row is split over a thread-block cluster of CL CTAs (2..16), one row per cluster
//     (a resident set of clusters loops over the rows only beyond the grid's y limit). Every CTA pulls its own slice
//     of the row into its own shared memory with a bulk copy (cp.async.bulk on an mbarrier), takes the slice's max
//     and exp(x - max) in place, and the CTAs exchange one (max, sum) pair each through distributed shared memory;
//     each CTA scales from shared memory. No copy is multicast;
//   * streaming cluster path, rows whose slices exceed shared memory: the same split and single exchange, each CTA
//     reading its slice twice from global memory (a running max and sum per warp, then exp(x - M) / S; the second
//     read comes from L2);
//   * stream path (unaligned pointers, cols not a multiple of the vector): one block per row reading the row three
//     times (max, sum, normalise; the later reads mostly from L2).
// Accuracy (fp32 outputs within 1e-6 relative of an fp64 softmax, elementwise; outputs below FLT_MIN within two
// subnormal steps): every path takes 2^64 * exp(x - max) with exp_pair below (relative error within about 2.1e-7);
// bf16 rows, whose outputs hold 8 bits, take the uncompensated exp_pair_fast (within about 1e-5).
// Each thread sums its exponentials pairwise per 16-byte vector into an fp64 accumulator, cross-thread and cross-CTA
// reductions run in fp64, and the output is e * (float)(1 / sum) (or e * (float)(exp(m_c - M) / S) per cluster
// slice, in two factors when that is below FLT_MIN) with one rounding, so outputs below FLT_MIN are kept as
// subnormals. Maxima propagate NaN, so a row holding a NaN (or +inf, or only -inf) comes out all NaN, as in torch.
#include "ckb200_softmax.h"
#include "common.cuh"

#include <cooperative_groups.h>
#include <math_constants.h>

#include <climits>
#include <mutex>

namespace cg = cooperative_groups;

namespace ckb {

__device__ unsigned int g_softmax_status = 0u;

namespace {

template <typename T>
__device__ __forceinline__ void store16(T* p, const float (&f)[VecN<T>::N]) {
  st_stream(p, pack16(f, p));
}

// ---------------------------------------------------------------------------------------------------------------
// Packed exponentials: 2^64 * exp(x - M) for two values at a time on the fp32x2 pipe (sm_100); every path uses them.
// Method (from the mathematics; no library routine is restated): TwoSum (Knuth) splits x - M into s + lo exactly;
// tb = s * log2(e) + 384 rounded to fp32 puts th = tb - 384 (exact) on the grid of 2^-15 for every s in the range
// used (s >= -150 after the clamp below), so th + 64 is exact too; E = 2^(th + 64) by the ex2.approx instruction,
// which is 2^64 * 2^th without overflow (th <= 0) and normal for th >= -190; the residual r = (s + lo) - th * ln 2,
// with ln 2 as a float pair so that r is exact to far below an ulp of E and |r| < 1.1e-5, is folded in as E * (1 + r)
// (the dropped r^2 / 2 term is below 1e-10). The relative error is that of ex2.approx plus one rounding.
// The 2^64 scale rides through every sum (S' = 2^64 S, so 1 / S' stays a normal float for any row length) and leaves
// with the final multiplication: each output is E * (1 / S') with one rounding, so results below FLT_MIN come out as
// subnormals instead of zero. Before the split x is raised to `lowc`, a value below M whose exponential is zero, so
// that x = -inf gives 0 instead of the inf - inf of the split; a NaN or +inf max makes lowc NaN and every result NaN.
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ float max_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
template <int WIDTH = 32>
__device__ __forceinline__ float warp_max_nan(float v) {
#pragma unroll
  for (int o = WIDTH / 2; o > 0; o >>= 1) v = max_nan(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float ex2_ftz(float a) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(a));
  return r;
}

struct ExpShift {
  float2 nm;   // (-M, -M)
  float lowc;  // every x below it has exp(x - M) == 0 in fp32
  __device__ __forceinline__ explicit ExpShift(float M) {
    nm = make_float2(-M, -M);
    lowc = M - fmaxf(150.0f, fabsf(M) * 0x1p-20f);
  }
};

__device__ __forceinline__ float2 exp_pair(float2 x, const ExpShift& e) {
  const float2 kNeg1 = make_float2(-1.0f, -1.0f);
  const float2 kL2E = make_float2(1.44269502162933349609375f, 1.44269502162933349609375f);  // fp32(log2 e)
  const float2 kNLn2Hi = make_float2(-0.693147182464599609375f, -0.693147182464599609375f);  // -fp32(ln 2)
  const float2 kNLn2Lo = make_float2(1.904654323148236e-09f, 1.904654323148236e-09f);       // -(ln 2 - fp32(ln 2))
  const float2 kGrid = make_float2(384.0f, 384.0f);     // 1.5 * 2^8: th lands on the 2^-15 grid
  const float2 kNGrid = make_float2(-384.0f, -384.0f);
  const float2 kNGridS = make_float2(-320.0f, -320.0f);  // -384 + 64: the 2^64 scale
  x.x = fmaxf(x.x, e.lowc);
  x.y = fmaxf(x.y, e.lowc);
  const float2 s = __fadd2_rn(x, e.nm);
  const float2 xb = __ffma2_rn(e.nm, kNeg1, s);  // s - (-M): x as rounded into s
  const float2 mb = __ffma2_rn(xb, kNeg1, s);    // s - xb: -M as rounded into s
  const float2 dx = __ffma2_rn(xb, kNeg1, x);    // x - xb
  const float2 dm = __ffma2_rn(mb, kNeg1, e.nm); // -M - mb
  const float2 lo = __fadd2_rn(dx, dm);          // s + lo == x - M exactly
  const float2 tb = __ffma2_rn(s, kL2E, kGrid);  // s * log2 e + 384, in [167, 384]
  const float2 th = __fadd2_rn(tb, kNGrid);      // exact
  const float2 ts = __fadd2_rn(tb, kNGridS);     // th + 64, exact
  const float2 E = make_float2(ex2_ftz(ts.x), ex2_ftz(ts.y));
  float2 r = __ffma2_rn(th, kNLn2Hi, s);          // s - th * ln2_hi, exact but for one tiny rounding
  r = __fadd2_rn(r, __ffma2_rn(th, kNLn2Lo, lo)); // + lo - th * ln2_lo
  return __ffma2_rn(E, r, E);
}

// The same scaled exponential for rows of 16-bit values, whose outputs need about 9 good bits, not 24:
// 2^(s * log2 e + 64) by one ex2.approx (relative error within about 1e-5 for the s of the clamped range: the
// rounding of the exponent, |s * log2 e| <= 217, dominates), with no compensation. Same 2^64 scale and clamp.
__device__ __forceinline__ float2 exp_pair_fast(float2 x, const ExpShift& e) {
  const float2 kL2E = make_float2(1.44269502162933349609375f, 1.44269502162933349609375f);
  const float2 k64 = make_float2(64.0f, 64.0f);
  x.x = fmaxf(x.x, e.lowc);
  x.y = fmaxf(x.y, e.lowc);
  const float2 t = __ffma2_rn(__fadd2_rn(x, e.nm), kL2E, k64);
  return make_float2(ex2_ftz(t.x), ex2_ftz(t.y));
}

// The exponential a row of T takes: compensated for fp32 outputs, plain for 16-bit ones.
template <typename T>
__device__ __forceinline__ float2 exp2v(float2 x, const ExpShift& e) {
  if constexpr (sizeof(T) == 4) return exp_pair(x, e);
  else return exp_pair_fast(x, e);
}

// One value (the unaligned stream path): the pair routine with the value in both halves.
template <typename T>
__device__ __forceinline__ float exp_one(float x, const ExpShift& es) { return exp2v<T>(make_float2(x, x), es).x; }

// In place: f = exp(f - M) by pairs; returns their pairwise sum.
template <typename T, int V>
__device__ __forceinline__ float exp_vec2(float (&f)[V], const ExpShift& es) {
  float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
  for (int j = 0; j < V; j += 2) {
    const float2 e = exp2v<T>(make_float2(f[j], f[j + 1]), es);
    f[j] = e.x;
    f[j + 1] = e.y;
    acc = j == 0 ? e : __fadd2_rn(acc, e);
  }
  return acc.x + acc.y;
}

// ------------------------------------------------------------------------------------------------ group path ----
// G lanes per row (4..32), NV vectors per lane, 256 threads = 8 warps = 8 * 32 / G rows per block.
template <typename T, int G, int NV>
__global__ void __launch_bounds__(256) sm_group(const T* __restrict__ x, T* __restrict__ y, long long rows, int cols) {
  pdl_wait();
  pdl_trigger();
  constexpr int V = VecN<T>::N;
  constexpr int RPW = 32 / G;
  const int lane = threadIdx.x & 31;
  const int sub = lane % G;
  const long long row = ((long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * RPW + lane / G;
  const bool live = row < rows;  // dead groups still join the shuffles
  const int nvec = cols / V;
  const T* xr = x + (live ? row : 0) * (long long)cols;
  T* yr = y + (live ? row : 0) * (long long)cols;
  float v[NV][V];
  bool in[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int i = sub + k * G;
    in[k] = live && i < nvec;
    uint4 r = in[k] ? ld_stream(xr + (long long)i * V) : make_uint4(0u, 0u, 0u, 0u);
    unpack16(r, v[k], x);
  }
  float m = -CUDART_INF_F;
#pragma unroll
  for (int k = 0; k < NV; ++k)
    if (in[k]) {
#pragma unroll
      for (int j = 0; j < V; ++j) m = max_nan(m, v[k][j]);
    }
  m = warp_max_nan<G>(m);
  const ExpShift es(m);
  double s = 0.0;
#pragma unroll
  for (int k = 0; k < NV; ++k)
    if (in[k]) s += (double)exp_vec2<T>(v[k], es);
  s = warp_sum<G>(s);
  const float inv = (float)(1.0 / s);
#pragma unroll
  for (int k = 0; k < NV; ++k)
    if (in[k]) {
#pragma unroll
      for (int j = 0; j < V; ++j) v[k][j] *= inv;
      store16(yr + (long long)(sub + k * G) * V, v[k]);
    }
}

// ------------------------------------------------------------------------------------------------ block path ----
// One block per row; thread t keeps vectors t, t + B, ..., t + B (NV - 1).
template <typename T, int NV, int MAXT>
__global__ void __launch_bounds__(MAXT) sm_block(const T* __restrict__ x, T* __restrict__ y, int cols) {
  pdl_wait();
  pdl_trigger();
  constexpr int V = VecN<T>::N;
  __shared__ float red_m[32];
  __shared__ double red_s[32];
  const int nvec = cols / V;
  const T* xr = x + (long long)blockIdx.x * cols;
  T* yr = y + (long long)blockIdx.x * cols;
  float v[NV][V];
  bool in[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    in[k] = i < nvec;
    uint4 r = in[k] ? ld_stream(xr + (long long)i * V) : make_uint4(0u, 0u, 0u, 0u);
    unpack16(r, v[k], x);
  }
  const int warps = blockDim.x >> 5, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float m = -CUDART_INF_F;
#pragma unroll
  for (int k = 0; k < NV; ++k)
    if (in[k]) {
#pragma unroll
      for (int j = 0; j < V; ++j) m = max_nan(m, v[k][j]);
    }
  m = warp_max_nan(m);
  if (lane == 0) red_m[warp] = m;
  __syncthreads();
  m = warp_max_nan(lane < warps ? red_m[lane] : -CUDART_INF_F);
  const ExpShift es(m);
  double s = 0.0;
#pragma unroll
  for (int k = 0; k < NV; ++k)
    if (in[k]) s += (double)exp_vec2<T>(v[k], es);
  s = warp_sum(s);
  if (lane == 0) red_s[warp] = s;
  __syncthreads();
  s = warp_sum(lane < warps ? red_s[lane] : 0.0);
  const float inv = (float)(1.0 / s);
#pragma unroll
  for (int k = 0; k < NV; ++k)
    if (in[k]) {
#pragma unroll
      for (int j = 0; j < V; ++j) v[k][j] *= inv;
      store16(yr + (long long)(threadIdx.x + k * blockDim.x) * V, v[k]);
    }
}

// ---------------------------------------------------------------------------------------------- cluster path ----
constexpr int kClusterThreads = 256;
constexpr int kClusterMinBlocks = 4;  // registers for four CTAs per SM (64 per thread)
constexpr int kTailVecs = 4;          // tail vectors per thread: a slice may keep 16 KB out of shared memory
constexpr int kMaxStages = 4;

// The start-up handshake: the initialising thread's fence.mbarrier_init (release, cluster scope) already publishes the
// mbarrier initialisation, so the arrive is relaxed (a release arrive would make every warp wait on a memory fence).
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

// Block-wide max (NaN-propagating) / sum of one value per thread through `red` (32 slots); every thread gets the same
// result.
__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max_nan(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  const int warps = blockDim.x >> 5;
  float r = red[0];
  for (int i = 1; i < warps; ++i) r = max_nan(r, red[i]);
  return r;
}
__device__ __forceinline__ double block_sum(double v, double* red) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  const int warps = blockDim.x >> 5;
  double r = red[0];
  for (int i = 1; i < warps; ++i) r += red[i];
  return r;
}

// DSMEM exchange: st.async writes a value into a peer CTA's shared memory and completes its bytes on the peer's
// mbarrier, so a CTA learns its peers' partials by waiting on its own mbarrier; no cluster-wide barrier (and no release
// of this CTA's outstanding global stores) sits on a row's critical path.
__device__ __forceinline__ unsigned mapa_u32(unsigned local_addr, unsigned rank) {
  unsigned r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_async_u32(unsigned raddr, unsigned v, unsigned rbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(raddr), "r"(v),
               "r"(rbar)
               : "memory");
}
__device__ __forceinline__ void st_async_u64(unsigned raddr, unsigned long long v, unsigned rbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b64 [%0], %1, [%2];" ::"r"(raddr), "l"(v),
               "r"(rbar)
               : "memory");
}

constexpr int kMaxCluster = 16;

// Pass 3 of the cluster path: y = E * s1 (* s2) for the staged part of the slice (fp32: the exponentials in place;
// bf16: the raw values, whose exponentials are taken again), streamed to HBM.
template <typename T, bool kTwo>
__device__ __forceinline__ void cluster_store(const uint4* buf, uint4* dst, int ns, float s1, float s2,
                                              const ExpShift& es) {
  constexpr int V = VecN<T>::N;
  const float2 m1 = make_float2(s1, s1), m2 = make_float2(s2, s2);
#pragma unroll 4
  for (int i = threadIdx.x; i < ns; i += kClusterThreads) {
    const uint4 raw = buf[i];
    if constexpr (V == 4) {
      float2 a = __fmul2_rn(make_float2(__uint_as_float(raw.x), __uint_as_float(raw.y)), m1);
      float2 b = __fmul2_rn(make_float2(__uint_as_float(raw.z), __uint_as_float(raw.w)), m1);
      if (kTwo) {
        a = __fmul2_rn(a, m2);
        b = __fmul2_rn(b, m2);
      }
      st_stream(dst + i, make_uint4(__float_as_uint(a.x), __float_as_uint(a.y), __float_as_uint(b.x),
                                    __float_as_uint(b.y)));
    } else {
      float f[V];
      unpack16(raw, f, (const T*)nullptr);
#pragma unroll
      for (int j = 0; j < V / 2; ++j) {
        float2 e = __fmul2_rn(exp2v<T>(make_float2(f[2 * j], f[2 * j + 1]), es), m1);
        if (kTwo) e = __fmul2_rn(e, m2);
        f[2 * j] = e.x;
        f[2 * j + 1] = e.y;
      }
      store16(reinterpret_cast<T*>(dst + i), f);
    }
  }
}

// The slice's tail, vectors [ns, nv) held in registers: thread t owns vectors ns + t + j * kClusterThreads.
__device__ __forceinline__ uint4 neg_inf16(const float*) {
  return make_uint4(0xff800000u, 0xff800000u, 0xff800000u, 0xff800000u);
}
__device__ __forceinline__ uint4 neg_inf16(const __nv_bfloat16*) {
  return make_uint4(0xff80ff80u, 0xff80ff80u, 0xff80ff80u, 0xff80ff80u);
}
template <typename T>
__device__ __forceinline__ void tail_load(uint4 (&tv)[kTailVecs], const uint4* src, int ns, int nv) {
#pragma unroll
  for (int j = 0; j < kTailVecs; ++j) {
    const int i = ns + (int)threadIdx.x + j * kClusterThreads;
    tv[j] = i < nv ? __ldcg(src + i) : neg_inf16((const T*)nullptr);
  }
}

// Grid (CL, G), cluster (CL, 1, 1): cluster g handles rows g, g + G, g + 2G, ... and CTA `rank` owns elements
// [rank * slice, min((rank + 1) * slice, cols)) of each (slice and cols multiples of the 16-byte vector). Of its nv
// vectors, the first ns = min(nv, ns_cap) are staged in shared memory by one bulk copy and the rest (at most
// kClusterThreads * kTailVecs, the tail) are read into registers beside it: a 64 KB slice fits four CTAs per SM that
// way, where staging all of it fits three. A CTA cycles its rows through `stages` slice buffers in dynamic shared
// memory (stride `stage_vec` 16-byte vectors): the bulk copy of a row is issued `stages` rows ahead. Per row: the
// slice's max m_c -> exp(x - m_c) (in place for the staged fp32 part) and their sum s_c -> warp 0 st.asyncs (m_c, s_c)
// to every peer -> warp 0 combines the cluster's pairs in fp64 into the row max M, the row sum S = sum of
// s_l * exp(m_l - M) and this slice's scale exp(m_c - M) / S, broadcast through shared memory -> every thread scales
// and stores. One exchange per row, and no thread waits for the row max before its exponentials. The exchange slots
// and their mbarrier are double buffered by row parity, so a fast CTA's next row never lands in a slot a slow peer
// still reads.
// kRing false: one row per cluster (grid y = rows), one buffer, no refills.
template <typename T, bool kRing>
__global__ void __launch_bounds__(kClusterThreads, kClusterMinBlocks) sm_cluster(const T* __restrict__ x,
                                                                             T* __restrict__ y, long long rows,
                                                                             long long cols, int slice, int ns_cap,
                                                                             int stages_arg, int stage_vec) {
  pdl_wait();
  pdl_trigger();
  constexpr int V = VecN<T>::N;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t bars[kMaxStages];
  __shared__ __align__(8) uint64_t bar_pair[2];
  __shared__ float xmax[2][kMaxCluster];
  __shared__ double xsum[2][kMaxCluster];
  __shared__ float red[32];
  __shared__ double red_d[32];
  __shared__ float scale, scale_lo;

  cg::cluster_group cluster = cg::this_cluster();
  const unsigned rank = cluster.block_rank();
  const unsigned csize = cluster.num_blocks();
  const long long beg = (long long)rank * slice;
  long long n = cols - beg;
  n = n < 0 ? 0 : (n > slice ? slice : n);
  const int nv = (int)(n / V);                 // vectors of this CTA's slice (the same for every row)
  const int ns = nv < ns_cap ? nv : ns_cap;    // of which staged in shared memory; [ns, nv) is the tail
  const unsigned bytes = (unsigned)ns * 16u;
  uint4* const buf0 = reinterpret_cast<uint4*>(smem_raw);
  const long long first = blockIdx.y, step = gridDim.y;
  const int stages = kRing ? stages_arg : 1;

  if (threadIdx.x == 0) {
    for (int st = 0; st < stages; ++st) mbar_init(&bars[st], 1);
    mbar_init(&bar_pair[0], 1);
    mbar_init(&bar_pair[1], 1);
    mbar_fence_init();
    if (bytes)
      for (int st = 0; st < stages; ++st) {
        const long long r = first + st * step;
        if (r < rows) {
          mbar_arrive_expect_tx(&bars[st], bytes);
          bulk_load(buf0 + (size_t)st * stage_vec, x + r * cols + beg, bytes, &bars[st]);
        }
      }
  }
  // The first row's tail goes out beside its bulk copy; each later row's is loaded at the end of the row before.
  uint4 tv[kTailVecs];
  if (first < rows) tail_load<T>(tv, reinterpret_cast<const uint4*>(x + first * cols + beg), ns, nv);
  // No thread polls a copy mbarrier before thread 0 has initialised it (shared memory still holds whatever the SM's
  // previous CTA left at these addresses, possibly a completed mbarrier of the same layout).
  __syncthreads();
  // Every CTA's exchange mbarriers are initialised before any peer sends to them: every thread arrives here, and
  // warp 0, the only one that touches peers, waits for the whole cluster before its first send.
  cluster_arrive();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = blockDim.x >> 5;
  // The peer addresses lane l of warp 0 sends to (lanes 0 .. csize-1 each serve one peer).
  unsigned peer_max[2] = {0u, 0u}, peer_sum[2] = {0u, 0u}, peer_bar[2] = {0u, 0u};
  if (threadIdx.x < csize) {
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      peer_max[p] = mapa_u32(smem_u32(&xmax[p][rank]), threadIdx.x);
      peer_sum[p] = mapa_u32(smem_u32(&xsum[p][rank]), threadIdx.x);
      peer_bar[p] = mapa_u32(smem_u32(&bar_pair[p]), threadIdx.x);
    }
  }

  bool ok = true;
  int t = 0;
  for (long long row = first; row < rows; row += step, ++t) {
    const int st = kRing ? t % stages : 0;
    const int p = kRing ? t & 1 : 0;
    uint4* const buf = buf0 + (size_t)st * stage_vec;
    if (threadIdx.x == 0) mbar_arrive_expect_tx(&bar_pair[p], csize * 12u);

    // Pass 1: the slice's max m_c (NaN-propagating), folded by every warp from the per-warp maxima; the tail (whose
    // loads usually land first) before the wait for the staged part.
    float m = -CUDART_INF_F;
#pragma unroll
    for (int j = 0; j < kTailVecs; ++j) {
      float f[V];
      unpack16(tv[j], f, x);
#pragma unroll
      for (int q = 0; q < V; ++q) m = max_nan(m, f[q]);
    }
    if (bytes) ok = mbar_wait(&bars[st], (unsigned)(t / stages) & 1u) && ok;
#pragma unroll 4
    for (int i = threadIdx.x; i < ns; i += kClusterThreads) {
      float f[V];
      unpack16(buf[i], f, x);
#pragma unroll
      for (int j = 0; j < V; ++j) m = max_nan(m, f[j]);
    }
    m = warp_max_nan(m);
    if (lane == 0) red[warp] = m;
    __syncthreads();
    const float mc = warp_max_nan(lane < warps ? red[lane] : -CUDART_INF_F);
    // A slice of -inf only takes its (zero) exponentials against 0; its pair still reports m_c = -inf.
    const ExpShift es(mc == -CUDART_INF_F ? 0.0f : mc);

    // Pass 2: exp(x - m_c), summed pairwise per vector into fp64; the staged fp32 part keeps its exponentials in
    // place, the tail keeps its raw values (its exponentials are taken again in pass 3).
    double sum = 0.0;
#pragma unroll 4
    for (int i = threadIdx.x; i < ns; i += kClusterThreads) {
      const uint4 raw = buf[i];
      if constexpr (V == 4) {
        const float2 a = exp_pair(make_float2(__uint_as_float(raw.x), __uint_as_float(raw.y)), es);
        const float2 b = exp_pair(make_float2(__uint_as_float(raw.z), __uint_as_float(raw.w)), es);
        const float2 ab = __fadd2_rn(a, b);
        sum += (double)(ab.x + ab.y);
        buf[i] = make_uint4(__float_as_uint(a.x), __float_as_uint(a.y), __float_as_uint(b.x), __float_as_uint(b.y));
      } else {
        float f[V];
        unpack16(raw, f, x);
        float2 e[V / 2];
#pragma unroll
        for (int j = 0; j < V / 2; ++j) e[j] = exp2v<T>(make_float2(f[2 * j], f[2 * j + 1]), es);
        const float2 s01 = __fadd2_rn(e[0], e[1]), s23 = __fadd2_rn(e[2], e[3]);
        const float2 s03 = __fadd2_rn(s01, s23);
        sum += (double)(s03.x + s03.y);
      }
    }
#pragma unroll
    for (int j = 0; j < kTailVecs; ++j) {
      if (ns + (int)threadIdx.x + j * kClusterThreads < nv) {
        float f[V];
        unpack16(tv[j], f, x);
        float2 e[V / 2];
#pragma unroll
        for (int q = 0; q < V / 2; ++q) e[q] = exp2v<T>(make_float2(f[2 * q], f[2 * q + 1]), es);
        float2 acc = __fadd2_rn(e[0], e[1]);
#pragma unroll
        for (int q = 2; q < V / 2; q += 2) acc = __fadd2_rn(acc, __fadd2_rn(e[q], e[q + 1]));
        sum += (double)(acc.x + acc.y);
      }
    }
    sum = warp_sum(sum);
    if (lane == 0) red_d[warp] = sum;
    __syncthreads();

    // Exchange and combine (warp 0): M = max m_l, S = sum s_l * exp(m_l - M) in fp64, scale = exp(m_c - M) / S.
    // A NaN or +inf anywhere in the row, or a row of -inf, makes M, S or the scale NaN, so the row is all NaN.
    if (warp == 0) {
      const double sc = warp_sum(lane < warps ? red_d[lane] : 0.0);
      if (t == 0) cluster_wait();
      if (lane < (int)csize) {
        st_async_u32(p ? peer_max[1] : peer_max[0], __float_as_uint(mc), p ? peer_bar[1] : peer_bar[0]);
        st_async_u64(p ? peer_sum[1] : peer_sum[0], (unsigned long long)__double_as_longlong(sc),
                     p ? peer_bar[1] : peer_bar[0]);
      }
      ok = mbar_wait(&bar_pair[p], (unsigned)(t >> 1) & 1u) && ok;
      const float ml = lane < (int)csize ? xmax[p][lane] : -CUDART_INF_F;
      const float M = warp_max_nan(ml);
      const double w = lane < (int)csize ? exp((double)ml - (double)M) : 0.0;
      const double S = warp_sum(lane < (int)csize ? xsum[p][lane] * w : 0.0);
      const double wc = __shfl_sync(0xffffffffu, w, (int)rank);
      if (lane == 0) {
        // Outputs are E * f with E up to 2^64 (exp_pair's scale). A factor f below FLT_MIN would drop bits of normal
        // outputs, so it is applied as (E * (f * 2^100)) * 2^-100, both factors normal; f below 2^-226 only has
        // outputs that round to 0. A NaN factor passes through.
        const double f = wc / S;
        float hi = (float)f, lo_f = 1.0f;
        if (f < 0x1p-126) {
          hi = f >= 0x1p-226 ? (float)(f * 0x1p100) : 0.0f;
          lo_f = f >= 0x1p-226 ? 0x1p-100f : 1.0f;
        }
        scale = hi;
        scale_lo = lo_f;
      }
    }
    __syncthreads();

    // Pass 3: scale from shared memory, stream to HBM (the two-factor form only when the factor needs it): the tail
    // from its registers, then the staged part.
    uint4* const dst = reinterpret_cast<uint4*>(y + row * cols + beg);
    const float s1 = scale, s2 = scale_lo;
#pragma unroll
    for (int j = 0; j < kTailVecs; ++j) {
      const int i = ns + (int)threadIdx.x + j * kClusterThreads;
      if (i < nv) {
        float f[V];
        unpack16(tv[j], f, x);
#pragma unroll
        for (int q = 0; q < V / 2; ++q) {
          float2 e = __fmul2_rn(exp2v<T>(make_float2(f[2 * q], f[2 * q + 1]), es), make_float2(s1, s1));
          if (s2 != 1.0f) e = __fmul2_rn(e, make_float2(s2, s2));
          f[2 * q] = e.x;
          f[2 * q + 1] = e.y;
        }
        st_stream(dst + i, pack16(f, x));
      }
    }
    if (s2 == 1.0f) cluster_store<T, false>(buf, dst, ns, s1, 1.0f, es);
    else cluster_store<T, true>(buf, dst, ns, s1, s2, es);
    // Refill this buffer `stages` rows ahead once every thread is done with it (the exponentials written into it by
    // the generic proxy are ordered before the bulk copy's writes by the proxy fence). With no row left for the
    // buffer, the CTA just finishes. The barrier also keeps `scale` and `red` from being rewritten while read.
    if (!kRing) break;
    const long long next = row + (long long)stages * step;
    if (next < rows) {
      if (bytes) fence_proxy_async();
      __syncthreads();
      if (threadIdx.x == 0 && bytes) {
        mbar_arrive_expect_tx(&bars[st], bytes);
        bulk_load(buf, x + next * cols + beg, bytes, &bars[st]);
      }
    }
    if (row + step < rows) tail_load<T>(tv, reinterpret_cast<const uint4*>(x + (row + step) * cols + beg), ns, nv);
  }
  if (!ok) atomicOr(&g_softmax_status, CKB_STATUS_TIMEOUT);
}

// ------------------------------------------------------------------------------------ streaming cluster path ----
// One row per cluster of CL CTAs (2..16) of 512 threads; CTA `rank` owns the 16-byte vectors [rank * sv, (rank + 1) *
// sv) of the row. Nothing is staged in shared memory: pass A streams the slice from HBM, U vectors per thread in
// flight, with a running max per warp and exp(x - max) summed per thread (a larger max rescales the sum in fp64);
// the warps' pairs fold into the CTA's (m_c, s_c), warp 0 st.asyncs it to every peer and combines the cluster's
// pairs in fp64 into the row max M and sum S; pass B re-reads the slice (from L2: every resident cluster's slices
// together are a fraction of it) and writes exp(x - M) * (1 / S).
constexpr int kStreamThreads = 512;
constexpr int kStreamMaxCluster = 8;  // measured best for 4 MB rows (16-CTA clusters at 2 CTAs/SM pack worse)


template <typename T, int U>
__global__ void __launch_bounds__(kStreamThreads, 2) sm_cluster_stream(const T* __restrict__ x, T* __restrict__ y,
                                                                      long long rows, long long cols, long long sv) {
  pdl_wait();
  pdl_trigger();
  constexpr int V = VecN<T>::N;
  constexpr int kWarps = kStreamThreads / 32;
  constexpr long long kStep = (long long)kStreamThreads * U;
  __shared__ __align__(8) uint64_t bar_pair[2];
  __shared__ float xmax[2][kMaxCluster];
  __shared__ double xsum[2][kMaxCluster];
  __shared__ float wmax[kWarps];
  __shared__ double wsum[kWarps];
  __shared__ float row_m, row_inv;

  cg::cluster_group cluster = cg::this_cluster();
  const unsigned rank = cluster.block_rank();
  const unsigned csize = cluster.num_blocks();
  const long long nvec = cols / V;
  const long long vb = (long long)rank * sv < nvec ? (long long)rank * sv : nvec;
  const long long ve = vb + sv < nvec ? vb + sv : nvec;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint4 fill = neg_inf16(x);

  if (threadIdx.x == 0) {
    mbar_init(&bar_pair[0], 1);
    mbar_init(&bar_pair[1], 1);
    mbar_fence_init();
  }
  // Every thread arrives; warp 0, the only one that touches peers, waits before its first send.
  cluster_arrive();
  unsigned peer_max[2] = {0u, 0u}, peer_sum[2] = {0u, 0u}, peer_bar[2] = {0u, 0u};
  if (threadIdx.x < csize) {
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      peer_max[p] = mapa_u32(smem_u32(&xmax[p][rank]), threadIdx.x);
      peer_sum[p] = mapa_u32(smem_u32(&xsum[p][rank]), threadIdx.x);
      peer_bar[p] = mapa_u32(smem_u32(&bar_pair[p]), threadIdx.x);
    }
  }

  bool ok = true;
  int t = 0;
  for (long long row = blockIdx.y; row < rows; row += gridDim.y, ++t) {
    const int p = t & 1;
    if (threadIdx.x == 0) mbar_arrive_expect_tx(&bar_pair[p], csize * 12u);
    const uint4* src = reinterpret_cast<const uint4*>(x + row * cols);

    // Pass A: a running max per warp (mw, the same in every lane) and this thread's sum of exp(x - mw).
    float mw = -CUDART_INF_F;
    double s = 0.0;
    for (long long i0 = vb + threadIdx.x; i0 < ve; i0 += kStep) {
      uint4 r[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const long long i = i0 + (long long)u * kStreamThreads;
        r[u] = i < ve ? __ldg(src + i) : fill;  // -inf past the slice: no effect on the max, exp 0
      }
      float cm = -CUDART_INF_F;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        float f[V];
        unpack16(r[u], f, x);
#pragma unroll
        for (int j = 0; j < V; ++j) cm = max_nan(cm, f[j]);
      }
      cm = warp_max_nan(cm);
      if (!(cm <= mw)) {  // a larger (or NaN) max: rescale the sum so far (warp-uniform branch)
        if (s != 0.0) s *= exp((double)mw - (double)cm);
        mw = cm;
      }
      const ExpShift es(mw == -CUDART_INF_F ? 0.0f : mw);  // all -inf so far: exponentials are 0 against any value
#pragma unroll
      for (int u = 0; u < U; ++u) {
        float f[V];
        unpack16(r[u], f, x);
        float2 acc = exp2v<T>(make_float2(f[0], f[1]), es);
#pragma unroll
        for (int j = 2; j < V; j += 2) acc = __fadd2_rn(acc, exp2v<T>(make_float2(f[j], f[j + 1]), es));
        s += (double)(acc.x + acc.y);
      }
    }
    s = warp_sum(s);
    if (lane == 0) {
      wmax[warp] = mw;
      wsum[warp] = s;
    }
    __syncthreads();

    // Warp 0: this CTA's pair (a slice of -inf contributes m_c = -inf, s_c = 0), the exchange, the row's M and S.
    // A NaN or +inf anywhere in the row, or a row of -inf, makes M or S NaN, so the row is all NaN.
    if (warp == 0) {
      const float ml = lane < kWarps ? wmax[lane] : -CUDART_INF_F;
      const float mc = warp_max_nan(ml);
      double sc = 0.0;
      if (mc != -CUDART_INF_F) sc = warp_sum(lane < kWarps ? wsum[lane] * exp((double)ml - (double)mc) : 0.0);
      if (t == 0) cluster_wait();
      if (lane < (int)csize) {
        st_async_u32(p ? peer_max[1] : peer_max[0], __float_as_uint(mc), p ? peer_bar[1] : peer_bar[0]);
        st_async_u64(p ? peer_sum[1] : peer_sum[0], (unsigned long long)__double_as_longlong(sc),
                     p ? peer_bar[1] : peer_bar[0]);
      }
      ok = mbar_wait(&bar_pair[p], (unsigned)(t >> 1) & 1u) && ok;
      const float pm = lane < (int)csize ? xmax[p][lane] : -CUDART_INF_F;
      const float M = warp_max_nan(pm);
      const double S = warp_sum(lane < (int)csize ? xsum[p][lane] * exp((double)pm - (double)M) : 0.0);
      if (lane == 0) {
        row_m = M;
        row_inv = (float)(1.0 / S);
      }
    }
    __syncthreads();

    // Pass B: re-read (last use), exp(x - M) * inv, stream out.
    const ExpShift es(row_m);
    const float2 inv2 = make_float2(row_inv, row_inv);
    uint4* dst = reinterpret_cast<uint4*>(y + row * cols);
    for (long long i0 = vb + threadIdx.x; i0 < ve; i0 += kStep) {
      uint4 r[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const long long i = i0 + (long long)u * kStreamThreads;
        r[u] = i < ve ? __ldcs(src + i) : fill;
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const long long i = i0 + (long long)u * kStreamThreads;
        float f[V];
        unpack16(r[u], f, x);
#pragma unroll
        for (int j = 0; j < V; j += 2) {
          const float2 e = __fmul2_rn(exp2v<T>(make_float2(f[j], f[j + 1]), es), inv2);
          f[j] = e.x;
          f[j + 1] = e.y;
        }
        if (i < ve) store16(reinterpret_cast<T*>(dst + i), f);
      }
    }
  }
  if (!ok) atomicOr(&g_softmax_status, CKB_STATUS_TIMEOUT);
}

// ----------------------------------------------------------------------------------------------- stream path ----
// One block per row, any alignment: a pass for the max, one for the sum (fp64 per thread), one to write; the second
// and third reads of a row mostly hit L2.
template <typename T>
__global__ void __launch_bounds__(1024) sm_stream(const T* __restrict__ x, T* __restrict__ y, long long cols) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[32];
  __shared__ double red_d[32];
  const T* xr = x + (long long)blockIdx.x * cols;
  T* yr = y + (long long)blockIdx.x * cols;
  float m = -CUDART_INF_F;
  for (long long i = threadIdx.x; i < cols; i += blockDim.x) m = max_nan(m, to_f32(xr[i]));
  const ExpShift es(block_max(m, red));
  double s = 0.0;
  for (long long i = threadIdx.x; i < cols; i += blockDim.x) s += (double)exp_one<T>(to_f32(xr[i]), es);
  s = block_sum(s, red_d);
  const float inv = (float)(1.0 / s);
  for (long long i = threadIdx.x; i < cols; i += blockDim.x) yr[i] = from_f32<T>(exp_one<T>(to_f32(xr[i]), es) * inv);
}

// ------------------------------------------------------------------------------------------------- dispatch -----
template <typename T, int G, int NV>
int start_group(const T* x, T* y, long long rows, int cols, cudaStream_t s) {
  constexpr long long rows_per_block = 8 * (32 / G);
  const long long grid = (rows + rows_per_block - 1) / rows_per_block;
  if (grid > INT_MAX) return -1;
  launch_pdl(sm_group<T, G, NV>, dim3((unsigned)grid), dim3(256), 0, s, x, y, rows, cols);
  return (int)cudaGetLastError();
}

// Rows that need at most 512 threads run the 512-thread instantiation (more registers per thread).
template <typename T, int NV>
int start_block(const T* x, T* y, long long rows, int cols, int threads, cudaStream_t s) {
  if (rows > INT_MAX) return -1;
  if (threads <= 512) launch_pdl(sm_block<T, NV, 512>, dim3((unsigned)rows), dim3(threads), 0, s, x, y, cols);
  else launch_pdl(sm_block<T, NV, 1024>, dim3((unsigned)rows), dim3(threads), 0, s, x, y, cols);
  return (int)cudaGetLastError();
}

constexpr long long kMaxRingBytes = 200 * 1024;
// Shared memory a slice stages before the rest goes to the register tail: 52 KB keeps four CTAs per SM (measured on
// 64 KB slices: 48 KB staged + 16 KB tail 91.6 us, 52 + 12 89.6 us, 55 + 9 91.2 us, all 64 KB staged at three CTAs
// per SM 104.6 us).
#ifndef CKB_SOFTMAX_STAGE_TARGET
#define CKB_SOFTMAX_STAGE_TARGET (52 * 1024)
#endif
constexpr long long kStageTargetVec = CKB_SOFTMAX_STAGE_TARGET / 16;
constexpr long long kTailCapVec = (long long)kClusterThreads * kTailVecs;

struct ClusterPlan {
  int cl = 0;         // 0: no cluster configuration fits
  int slice = 0;      // elements per CTA
  int ns_cap = 0;     // vectors of a slice staged in shared memory (the rest, at most kTailCapVec, in registers)
  int stages = 0;     // slice buffers per CTA
  int stage_vec = 0;  // 16-byte vectors between buffers
  int active = 0;     // co-resident clusters
  bool ring = false;  // persistent clusters looping over rows (rows beyond the grid's y limit)
};

cudaLaunchConfig_t cluster_config(int cl, unsigned grid_y, int smem, cudaStream_t s, cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)cl;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see launch_pdl
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3((unsigned)cl, grid_y, 1);
  cfg.blockDim = dim3(kClusterThreads, 1, 1);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = CKB_PDL ? 2 : 1;
  return cfg;
}

// The cluster shape for rows of `cols` elements. For each cluster size CL in 16, 8, 4, 2 the slice is cols / CL; a CTA
// stages min(slice, 52 KB) of it in shared memory (more when the rest would exceed the register tail's 16 KB) in one
// buffer (or, for the persistent ring, the whole slice in as many buffers as fit in 200 KB, at most 4), and
// cudaOccupancyMaxActiveClusters says
// how many such clusters stay resident. The score is resident CTAs, doubled for a ring of two or more buffers; a tie
// goes to the smaller cluster (fewer CTAs exchange per row). Cached per (device, cols, ring); the cache holds the last
// shape asked for.
template <typename T>
ClusterPlan plan_cluster(long long cols, bool ring) {
  constexpr int V = VecN<T>::N;
  static std::mutex mu;
  static int last_dev = -1;
  static long long last_cols = -1;
  static bool last_ring = false;
  static ClusterPlan last;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev == last_dev && cols == last_cols && ring == last_ring) return last;
  }
  ClusterPlan best;
  best.ring = ring;
  long long best_score = 0;
  auto kern = ring ? sm_cluster<T, true> : sm_cluster<T, false>;
  for (int cl = 16; cl >= 2; cl /= 2) {
    const long long slice = ((cols + cl - 1) / cl + V - 1) / V * V;
    const long long slice_vec = slice / V;
    long long ns_cap = slice_vec < kStageTargetVec ? slice_vec : kStageTargetVec;
    if (slice_vec - ns_cap > kTailCapVec || ring) ns_cap = slice_vec - (ring ? 0 : kTailCapVec);
    const long long stage_bytes = (ns_cap * 16 + 127) / 128 * 128;
    long long stages = stage_bytes > 0 ? kMaxRingBytes / stage_bytes : 1;
    if (stages > kMaxStages) stages = kMaxStages;
    if (!ring && stages > 1) stages = 1;
    if (stages < 1) continue;
    const int smem = (int)(stages * stage_bytes);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess ||
        (cl > 8 && cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)) {
      cudaGetLastError();
      continue;
    }
    cudaLaunchAttribute attr[2];
    cudaLaunchConfig_t cfg = cluster_config(cl, 1, smem, nullptr, attr);
    cfg.numAttrs = 1;  // the cluster shape alone for the occupancy query
    int active = 0;
    if (cudaOccupancyMaxActiveClusters(&active, kern, &cfg) != cudaSuccess) {
      cudaGetLastError();
      continue;
    }
    const long long score = (long long)active * cl * (stages >= 2 ? 2 : 1);
    if (active > 0 && score >= best_score) {
      best_score = score;
      best.cl = cl;
      best.slice = (int)slice;
      best.ns_cap = (int)ns_cap;
      best.stages = (int)stages;
      best.stage_vec = (int)(stage_bytes / 16);
      best.active = active;
    }
  }
  std::lock_guard<std::mutex> lock(mu);
  last_dev = dev;
  last_cols = cols;
  last_ring = ring;
  last = best;
  return best;
}

template <typename T>
int start_cluster(const ClusterPlan& p, const T* x, T* y, long long rows, long long cols, cudaStream_t s) {
  auto kern = p.ring ? sm_cluster<T, true> : sm_cluster<T, false>;
  const int smem = p.stages * p.stage_vec * 16;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
    cudaGetLastError();
    return -2;
  }
  if (p.cl > 8) cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  // One row per cluster (measured best: the whole row set in flight, four CTAs per SM), unless the rows exceed the
  // grid's y limit: then as many clusters as stay resident loop over the rows with a ring of slice buffers.
  const long long g = p.ring ? (rows < p.active ? rows : p.active) : rows;
  if (g > 65535) return -2;  // grid.y limit: the caller falls back
  cudaLaunchAttribute attr[2];
  cudaLaunchConfig_t cfg = cluster_config(p.cl, (unsigned)g, smem, s, attr);
  const cudaError_t err = cudaLaunchKernelEx(&cfg, kern, x, y, rows, cols, p.slice, p.ns_cap, p.stages, p.stage_vec);
  if (err != cudaSuccess) return (int)err;
  return (int)cudaGetLastError();
}

// Streaming cluster path: the smallest cluster (2..8) whose slices are at most 64 KB (8 for longer rows); one row per
// cluster, rows above the grid's y limit loop.
template <typename T>
int start_cluster_stream(const T* x, T* y, long long rows, long long cols, cudaStream_t s) {
  constexpr int V = VecN<T>::N;
  constexpr int U = V == 4 ? 8 : 4;
  auto kern = sm_cluster_stream<T, U>;
  const long long nvec = cols / V;
  int cl = 2;
  while (cl < kStreamMaxCluster && (nvec + cl - 1) / cl * 16 > 64 * 1024) cl *= 2;
  if (cl > 8 && cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
    cudaGetLastError();
    return -2;
  }
  const long long sv = (nvec + cl - 1) / cl;
  const unsigned gy = (unsigned)(rows < 65535 ? rows : 65535);
  cudaLaunchAttribute attr[2];
  cudaLaunchConfig_t cfg = cluster_config(cl, 1, 0, s, attr);
  cfg.blockDim = dim3(kStreamThreads, 1, 1);
  const unsigned launch_attrs = cfg.numAttrs;
  cfg.numAttrs = 1;  // the cluster shape alone for the occupancy query
  int active = 0;
  if (cudaOccupancyMaxActiveClusters(&active, kern, &cfg) != cudaSuccess || active <= 0) {
    cudaGetLastError();
    return -2;
  }
  cfg.gridDim = dim3((unsigned)cl, gy, 1);
  cfg.numAttrs = launch_attrs;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, kern, x, y, rows, cols, sv);
  if (err != cudaSuccess) return (int)err;
  return (int)cudaGetLastError();
}

#ifndef CKB_SOFTMAX_BLOCK_MAX_THREADS
#define CKB_SOFTMAX_BLOCK_MAX_THREADS 512
#endif
constexpr int kBlockMaxThreads = CKB_SOFTMAX_BLOCK_MAX_THREADS;  // longer rows go to the cluster path

template <typename T>
int dispatch(const T* x, T* y, long long rows, long long cols, cudaStream_t s) {
  constexpr int V = VecN<T>::N;
  constexpr int kMaxNV = 32 / V;  // at most 32 fp32 values cached per thread
  const bool vec = cols % V == 0 && aligned16(x) && aligned16(y) && cols <= INT_MAX;
  if (vec) {
    const long long nvec = cols / V;
    const int c = (int)cols;
    // Group path: the narrowest group that keeps at most kMaxNV vectors per lane (fewer for tiny rows).
    if (nvec <= 4) return start_group<T, 4, 1>(x, y, rows, c, s);
    if (nvec <= 8) return start_group<T, 4, 2>(x, y, rows, c, s);
    if (nvec <= 4LL * kMaxNV) return start_group<T, 4, kMaxNV>(x, y, rows, c, s);
    if (nvec <= 8LL * kMaxNV) return start_group<T, 8, kMaxNV>(x, y, rows, c, s);
    if (nvec <= 16LL * kMaxNV) return start_group<T, 16, kMaxNV>(x, y, rows, c, s);
    if (nvec <= 32LL * kMaxNV) return start_group<T, 32, kMaxNV>(x, y, rows, c, s);
    // Block path: NV = kMaxNV with the fewest threads, up to kBlockMaxThreads.
    if (nvec <= (long long)kBlockMaxThreads * kMaxNV) {
      const int threads = (int)((nvec + kMaxNV - 1) / kMaxNV + 31) / 32 * 32;
      return start_block<T, kMaxNV>(x, y, rows, c, threads, s);
    }
  }
#ifndef CKB_SOFTMAX_FORCE_STREAM
#define CKB_SOFTMAX_FORCE_STREAM 0  // 1: every vectorised row of the cluster sizes takes the streaming cluster path
#endif
  if (vec && CKB_SOFTMAX_FORCE_STREAM) {
    const int err = start_cluster_stream<T>(x, y, rows, cols, s);
    if (err != -2) return err;
  }
  if (vec) {
    const ClusterPlan p = plan_cluster<T>(cols, rows > 65535);
    if (p.cl > 0) {
      const int err = start_cluster<T>(p, x, y, rows, cols, s);
      if (err != -2) return err;
    } else {
      const int err = start_cluster_stream<T>(x, y, rows, cols, s);
      if (err != -2) return err;
    }
  }
  if (rows > INT_MAX) return -1;
  launch_pdl(sm_stream<T>, dim3((unsigned)rows), dim3(1024), 0, s, x, y, cols);
  return (int)cudaGetLastError();
}

}  // namespace
}  // namespace ckb

using namespace ckb;

// Replaces the reference's softmax `launch` (softmax/kernel.cu:520-527): x, y row-major [rows, cols]; dtype 0 fp32,
// 1 bf16; `threads` and `aux` are the reference's block-size hints and are accepted but not needed here (the B200
// dispatcher picks its own shapes). Returns 0 (also for rows <= 0 or cols <= 0), -1 for an unknown dtype or a shape
// no path serves, or the CUDA error of the launch.
CKB_EXPORT int launch(const void* x, void* y, long long rows, long long cols, int dtype, int threads, int aux,
                      cudaStream_t stream) {
  (void)threads;
  (void)aux;
  if (rows <= 0 || cols <= 0) return 0;
  if (dtype == kF32) return dispatch<float>((const float*)x, (float*)y, rows, cols, stream);
  if (dtype == kBF16)
    return dispatch<__nv_bfloat16>((const __nv_bfloat16*)x, (__nv_bfloat16*)y, rows, cols, stream);
  return -1;
}

// Status of the bounded waits in this library's kernels since the last reset: 0, or 1 when a bulk-copy wait gave up
// (the launch then produced garbage instead of hanging). Synchronises with the device; reset != 0 clears the word.
CKB_EXPORT int ckb_softmax_status(int reset) {
  unsigned v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_softmax_status, sizeof(v));
  if (e != cudaSuccess) return -(int)e;
  if (reset) {
    const unsigned zero = 0;
    e = cudaMemcpyToSymbol(g_softmax_status, &zero, sizeof(zero));
    if (e != cudaSuccess) return -(int)e;
  }
  return (int)v;
}
