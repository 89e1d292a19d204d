// Row-wise softmax over the last dim: y = exp(x - max) / sum(exp(x - max)), fp32 (dtype 0) and bf16 (dtype 1) rows,
// every value computed in fp32. Semantics follow the reference's torch.softmax(x, dim=-1) (softmax/baseline.py:12-13);
// the C entry keeps the reference's ABI (softmax/kernel.cu:520-527).
//
// Paths, chosen by row length (all read each element once from HBM and write it once):
//   * group path, rows of at most 256 16-byte vectors: G = 4..32 lanes per row, so one warp holds 32 / G rows and
//     every lane keeps NV vectors of its row in registers; group-local shuffles, no barrier;
//   * block path, rows of at most 32768 fp32 / bf16 values: one block per row, 32 values per thread in
//     registers, two barriers per row;
//   * cluster path, longer rows: a row is split over a thread-block cluster of CL CTAs (2..16); the grid holds as many
//     clusters as stay resident and each loops over its rows. Every CTA pulls its own slice of a row into its own
//     shared memory with a bulk copy (cp.async.bulk on an mbarrier) issued up to 4 rows ahead (a ring of slice
//     buffers), the CTAs exchange the max and then the sum through distributed shared memory, and each CTA
//     normalises from shared memory. No copy is multicast;
//   * wide cluster path, rows whose slices exceed shared memory: the same split and exchange, each CTA reading its
//     slice twice from global memory (online max/sum, then normalise; the second read mostly from L2);
//   * stream path (unaligned pointers, cols not a multiple of the vector): one block per row reading the row three
//     times (max, sum, normalise; the later reads mostly from L2).
// Accuracy (fp32 outputs within 1e-6 relative of an fp64 softmax, elementwise): exp(x - max) uses CUDA's expf on the
// fp32 difference and folds the difference's rounding error back in (TwoSum), each thread sums its exponentials
// pairwise per 16-byte vector into an fp64 accumulator and the cross-thread reductions run in fp64; the output is
// e * (float)(1 / sum).
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

// exp(x - m) for m >= x. The fp32 difference d carries a rounding error of up to half an ulp of |d| (relative error
// |d| * 2^-25 after exp, over 1e-6 once |d| > 32); TwoSum recovers that error lo exactly and exp(d + lo) is taken
// as exp(d) * (1 + lo). A zero or NaN exponential (x = -inf, or an inf/NaN row) is left as it is.
__device__ __forceinline__ float exp_shifted(float x, float m) {
  const float d = x - m;
  const float bv = d - x;
  const float lo = (x - (d - bv)) + (-m - bv);
  const float e = expf(d);
  return e > 0.0f ? fmaf(e, lo, e) : e;
}

// Pairwise sum of the values of one 16-byte vector.
__device__ __forceinline__ float vec_sum(const float (&f)[4]) { return (f[0] + f[1]) + (f[2] + f[3]); }
__device__ __forceinline__ float vec_sum(const float (&f)[8]) {
  return ((f[0] + f[1]) + (f[2] + f[3])) + ((f[4] + f[5]) + (f[6] + f[7]));
}

// In place: f = exp(f - m); returns their pairwise sum.
template <int V>
__device__ __forceinline__ float exp_vec(float (&f)[V], float m) {
#pragma unroll
  for (int j = 0; j < V; ++j) f[j] = exp_shifted(f[j], m);
  return vec_sum(f);
}

// ------------------------------------------------------------------------------------------------ group path ----
// G lanes per row (4..32), NV vectors per lane, 256 threads = 8 warps = 8 * 32 / G rows per block.
template <typename T, int G, int NV>
__global__ void __launch_bounds__(256) sm_group(const T* __restrict__ x, T* __restrict__ y, long long rows, int cols) {
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
      for (int j = 0; j < V; ++j) m = fmaxf(m, v[k][j]);
    }
  m = warp_max<G>(m);
  double s = 0.0;
#pragma unroll
  for (int k = 0; k < NV; ++k)
    if (in[k]) s += (double)exp_vec(v[k], m);
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
      for (int j = 0; j < V; ++j) m = fmaxf(m, v[k][j]);
    }
  m = warp_max(m);
  if (lane == 0) red_m[warp] = m;
  __syncthreads();
  m = red_m[0];
  for (int i = 1; i < warps; ++i) m = fmaxf(m, red_m[i]);
  double s = 0.0;
#pragma unroll
  for (int k = 0; k < NV; ++k)
    if (in[k]) s += (double)exp_vec(v[k], m);
  s = warp_sum(s);
  if (lane == 0) red_s[warp] = s;
  __syncthreads();
  s = 0.0;
  for (int i = 0; i < warps; ++i) s += red_s[i];
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
constexpr int kClusterThreads = 512;
constexpr int kMaxStages = 4;

__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

// Block-wide max / sum of one value per thread through `red` (32 slots); every thread gets the same result.
__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  const int warps = blockDim.x >> 5;
  float r = red[0];
  for (int i = 1; i < warps; ++i) r = fmaxf(r, red[i]);
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

// Grid (CL, G), cluster (CL, 1, 1): cluster g handles rows g, g + G, g + 2G, ... and CTA `rank` owns elements
// [rank * slice, min((rank + 1) * slice, cols)) of each (slice and cols multiples of the 16-byte vector). A CTA cycles
// its rows through `stages` slice buffers in dynamic shared memory (stride `stage_vec` 16-byte vectors): the bulk copy
// of a row is issued `stages` rows ahead. Per row: max over the slice -> every CTA st.asyncs its max to every peer ->
// exp and sum -> the same for the sums -> normalise and store. The exchange slots and their mbarriers are double
// buffered by row parity, so a fast CTA's next row never lands in a slot a slow peer still reads.
template <typename T>
__global__ void __launch_bounds__(kClusterThreads) sm_cluster(const T* __restrict__ x, T* __restrict__ y,
                                                              long long rows, long long cols, int slice,
                                                              int stages, int stage_vec) {
  constexpr int V = VecN<T>::N;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t bars[kMaxStages];
  __shared__ __align__(8) uint64_t bar_max[2], bar_sum[2];
  __shared__ float xmax[2][kMaxCluster];
  __shared__ double xsum[2][kMaxCluster];
  __shared__ float red[32];
  __shared__ double red_d[32];

  cg::cluster_group cluster = cg::this_cluster();
  const unsigned rank = cluster.block_rank();
  const unsigned csize = cluster.num_blocks();
  const long long beg = (long long)rank * slice;
  long long n = cols - beg;
  n = n < 0 ? 0 : (n > slice ? slice : n);
  const int nv = (int)(n / V);  // vectors of this CTA's slice (the same for every row)
  const unsigned bytes = (unsigned)nv * 16u;
  uint4* const buf0 = reinterpret_cast<uint4*>(smem_raw);
  const long long first = blockIdx.y, step = gridDim.y;

  if (threadIdx.x == 0) {
    for (int st = 0; st < stages; ++st) mbar_init(&bars[st], 1);
    for (int p = 0; p < 2; ++p) {
      mbar_init(&bar_max[p], 1);
      mbar_init(&bar_sum[p], 1);
    }
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
  // Every CTA's exchange mbarriers are initialised before any peer sends to them.
  cluster_arrive();
  cluster_wait();

  // The peer addresses this thread sends to (threads 0 .. csize-1 each serve one peer).
  unsigned peer_max[2] = {0u, 0u}, peer_sum[2] = {0u, 0u}, peer_bmax[2] = {0u, 0u}, peer_bsum[2] = {0u, 0u};
  if (threadIdx.x < csize) {
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      peer_max[p] = mapa_u32(smem_u32(&xmax[p][rank]), threadIdx.x);
      peer_sum[p] = mapa_u32(smem_u32(&xsum[p][rank]), threadIdx.x);
      peer_bmax[p] = mapa_u32(smem_u32(&bar_max[p]), threadIdx.x);
      peer_bsum[p] = mapa_u32(smem_u32(&bar_sum[p]), threadIdx.x);
    }
  }

  bool ok = true;
  int t = 0;
  for (long long row = first; row < rows; row += step, ++t) {
    const int st = t % stages;
    const int p = t & 1;
    const unsigned xphase = (unsigned)(t >> 1) & 1u;
    uint4* const buf = buf0 + (size_t)st * stage_vec;
    if (threadIdx.x == 0) {
      mbar_arrive_expect_tx(&bar_max[p], csize * 4u);
      mbar_arrive_expect_tx(&bar_sum[p], csize * 8u);
    }
    if (bytes) ok = mbar_wait(&bars[st], (unsigned)(t / stages) & 1u) && ok;

    // Pass 1: this slice's max, sent to every CTA of the cluster; the row's max from the cluster's.
    float m = -CUDART_INF_F;
    for (int i = threadIdx.x; i < nv; i += blockDim.x) {
      float f[V];
      unpack16(buf[i], f, x);
#pragma unroll
      for (int j = 0; j < V; ++j) m = fmaxf(m, f[j]);
    }
    m = block_max(m, red);
    if (threadIdx.x < csize)
      st_async_u32(p ? peer_max[1] : peer_max[0], __float_as_uint(m), p ? peer_bmax[1] : peer_bmax[0]);
    ok = mbar_wait(&bar_max[p], xphase) && ok;
    m = xmax[p][0];
    for (unsigned r = 1; r < csize; ++r) m = fmaxf(m, xmax[p][r]);

    // Pass 2: sum of exp(x - max); fp32 slices keep the exponentials in place for pass 3.
    double sum = 0.0;
    for (int i = threadIdx.x; i < nv; i += blockDim.x) {
      float f[V];
      unpack16(buf[i], f, x);
      sum += (double)exp_vec(f, m);
      if constexpr (V == 4) buf[i] = pack16(f, x);
    }
    sum = block_sum(sum, red_d);
    if (threadIdx.x < csize)
      st_async_u64(p ? peer_sum[1] : peer_sum[0], (unsigned long long)__double_as_longlong(sum),
                   p ? peer_bsum[1] : peer_bsum[0]);
    ok = mbar_wait(&bar_sum[p], xphase) && ok;
    double total = 0.0;
    for (unsigned r = 0; r < csize; ++r) total += xsum[p][r];
    const float inv = (float)(1.0 / total);

    // Pass 3: normalise from shared memory, stream to HBM.
    T* dst = y + row * cols + beg;
    for (int i = threadIdx.x; i < nv; i += blockDim.x) {
      float f[V];
      unpack16(buf[i], f, x);
      if constexpr (V == 4) {
#pragma unroll
        for (int j = 0; j < V; ++j) f[j] *= inv;
      } else {
#pragma unroll
        for (int j = 0; j < V; ++j) f[j] = exp_shifted(f[j], m) * inv;
      }
      store16(reinterpret_cast<T*>(reinterpret_cast<uint4*>(dst) + i), f);
    }
    // Every thread is done with this buffer (and with red / red_d): refill it `stages` rows ahead.
    fence_proxy_async();
    __syncthreads();
    if (threadIdx.x == 0 && bytes) {
      const long long r = row + (long long)stages * step;
      if (r < rows) {
        mbar_arrive_expect_tx(&bars[st], bytes);
        bulk_load(buf, x + r * cols + beg, bytes, &bars[st]);
      }
    }
  }
  if (!ok) atomicOr(&g_softmax_status, CKB_STATUS_TIMEOUT);
}

// Rows whose slices do not fit shared memory: the same cluster split and st.async exchange, but each CTA reads its
// slice from global memory twice -- an online (max, sum) pass, then the normalising pass, whose reads mostly hit L2
// (the resident CTAs' slices fit in it). The per-thread running sum is fp64 and is rescaled in fp64 when the running
// max grows; the CTAs' (max, sum) pairs combine in fp64.
template <typename T>
__global__ void __launch_bounds__(kClusterThreads) sm_cluster_wide(const T* __restrict__ x, T* __restrict__ y,
                                                                   long long rows, long long cols, long long slice) {
  constexpr int V = VecN<T>::N;
  __shared__ __align__(8) uint64_t bar_pair[2];
  __shared__ float xmax[2][kMaxCluster];
  __shared__ double xsum[2][kMaxCluster];
  __shared__ float red[32];
  __shared__ double red_d[32];
  __shared__ float row_max;

  cg::cluster_group cluster = cg::this_cluster();
  const unsigned rank = cluster.block_rank();
  const unsigned csize = cluster.num_blocks();
  const long long beg = rank * slice;
  long long n = cols - beg;
  n = n < 0 ? 0 : (n > slice ? slice : n);
  const long long nv = n / V;
  if (threadIdx.x == 0) {
    mbar_init(&bar_pair[0], 1);
    mbar_init(&bar_pair[1], 1);
    mbar_fence_init();
  }
  cluster_arrive();
  cluster_wait();
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
    const uint4* src = reinterpret_cast<const uint4*>(x + row * cols + beg);
    // Online (max, sum) of this thread's elements.
    float m = -CUDART_INF_F;
    double s = 0.0;
    for (long long i = threadIdx.x; i < nv; i += blockDim.x) {
      float f[V];
      unpack16(__ldg(src + i), f, x);
      float vm = f[0];
#pragma unroll
      for (int j = 1; j < V; ++j) vm = fmaxf(vm, f[j]);
      if (vm > m) {
        if (s != 0.0) s *= exp((double)m - (double)vm);
        m = vm;
      }
      if (m != -CUDART_INF_F) {
        s += (double)exp_vec(f, m);  // -inf elements add 0, NaN (and inf - inf) poison the sum
      } else {
#pragma unroll
        for (int j = 0; j < V; ++j)
          if (f[j] != f[j]) s = __longlong_as_double(0x7ff8000000000000ll);  // only -inf and NaN seen so far
      }
    }
    // Block combine: the block max, then every thread rescales its sum to it.
    const float bm = block_max(m, red);
    s = (s != 0.0) ? s * exp((double)m - (double)bm) : 0.0;
    s = block_sum(s, red_d);
    if (threadIdx.x < csize) {
      const unsigned pm = p ? peer_max[1] : peer_max[0];
      const unsigned ps = p ? peer_sum[1] : peer_sum[0];
      const unsigned pb = p ? peer_bar[1] : peer_bar[0];
      st_async_u32(pm, __float_as_uint(bm), pb);
      st_async_u64(ps, (unsigned long long)__double_as_longlong(s), pb);
    }
    ok = mbar_wait(&bar_pair[p], (unsigned)(t >> 1) & 1u) && ok;
    float M = xmax[p][0];
    for (unsigned r = 1; r < csize; ++r) M = fmaxf(M, xmax[p][r]);
    double total = 0.0;
    for (unsigned r = 0; r < csize; ++r) {
      const double sr = xsum[p][r];
      if (sr != 0.0) total += sr * exp((double)xmax[p][r] - (double)M);
    }
    if (M == -CUDART_INF_F || M != M) total = __longlong_as_double(0x7ff8000000000000ll);  // all -inf / NaN row
    const float inv = (float)(1.0 / total);
    // Normalising pass (second read).
    uint4* dst = reinterpret_cast<uint4*>(y + row * cols + beg);
    for (long long i = threadIdx.x; i < nv; i += blockDim.x) {
      float f[V];
      unpack16(__ldg(src + i), f, x);
#pragma unroll
      for (int j = 0; j < V; ++j) f[j] = exp_shifted(f[j], M) * inv;
      store16(reinterpret_cast<T*>(dst + i), f);
    }
    __syncthreads();  // red / red_d are reused by the next row
  }
  if (!ok) atomicOr(&g_softmax_status, CKB_STATUS_TIMEOUT);
  (void)row_max;
}

// ----------------------------------------------------------------------------------------------- stream path ----
// One block per row, any alignment: a pass for the max, one for the sum (fp64 per thread), one to write; the second
// and third reads of a row mostly hit L2.
template <typename T>
__global__ void __launch_bounds__(1024) sm_stream(const T* __restrict__ x, T* __restrict__ y, long long cols) {
  __shared__ float red[32];
  __shared__ double red_d[32];
  const T* xr = x + (long long)blockIdx.x * cols;
  T* yr = y + (long long)blockIdx.x * cols;
  float m = -CUDART_INF_F;
  for (long long i = threadIdx.x; i < cols; i += blockDim.x) m = fmaxf(m, to_f32(xr[i]));
  m = block_max(m, red);
  double s = 0.0;
  for (long long i = threadIdx.x; i < cols; i += blockDim.x) s += (double)exp_shifted(to_f32(xr[i]), m);
  s = block_sum(s, red_d);
  const float inv = (float)(1.0 / s);
  for (long long i = threadIdx.x; i < cols; i += blockDim.x) yr[i] = from_f32<T>(exp_shifted(to_f32(xr[i]), m) * inv);
}

// ------------------------------------------------------------------------------------------------- dispatch -----
template <typename T, int G, int NV>
int start_group(const T* x, T* y, long long rows, int cols, cudaStream_t s) {
  constexpr long long rows_per_block = 8 * (32 / G);
  const long long grid = (rows + rows_per_block - 1) / rows_per_block;
  if (grid > INT_MAX) return -1;
  sm_group<T, G, NV><<<(unsigned)grid, 256, 0, s>>>(x, y, rows, cols);
  return (int)cudaGetLastError();
}

// Rows that need at most 512 threads run the 512-thread instantiation (more registers per thread).
template <typename T, int NV>
int start_block(const T* x, T* y, long long rows, int cols, int threads, cudaStream_t s) {
  if (rows > INT_MAX) return -1;
  if (threads <= 512) sm_block<T, NV, 512><<<(unsigned)rows, threads, 0, s>>>(x, y, cols);
  else sm_block<T, NV, 1024><<<(unsigned)rows, threads, 0, s>>>(x, y, cols);
  return (int)cudaGetLastError();
}

constexpr long long kMaxRingBytes = 200 * 1024;
constexpr long long kSliceTarget = 64 * 1024;

struct ClusterPlan {
  int cl = 0;         // 0: no cluster configuration fits
  int slice = 0;      // elements per CTA
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
  cfg.gridDim = dim3((unsigned)cl, grid_y, 1);
  cfg.blockDim = dim3(kClusterThreads, 1, 1);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

// The cluster shape for rows of `cols` elements. For each cluster size CL in 16, 8, 4, 2 the slice is cols / CL; a CTA
// holds one slice buffer (or, for the persistent ring, as many as fit in 200 KB, at most 4) and
// cudaOccupancyMaxActiveClusters says how many such clusters stay resident; the score is resident CTAs, doubled for
// a ring of two or more buffers. Cached per (device, cols, ring); the cache holds the last shape asked for.
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
  auto kern = sm_cluster<T>;
  for (int cl = 16; cl >= 2; cl /= 2) {
    const long long slice = ((cols + cl - 1) / cl + V - 1) / V * V;
    const long long stage_bytes = (slice * (long long)sizeof(T) + 127) / 128 * 128;
    long long stages = kMaxRingBytes / stage_bytes;
    if (stages > kMaxStages) stages = kMaxStages;
    if (!ring && stages > 1) stages = 1;
    if (stages < 1) continue;
    const int smem = (int)(stages * stage_bytes);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess ||
        (cl > 8 && cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)) {
      cudaGetLastError();
      continue;
    }
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = cluster_config(cl, 1, smem, nullptr, attr);
    int active = 0;
    if (cudaOccupancyMaxActiveClusters(&active, kern, &cfg) != cudaSuccess) {
      cudaGetLastError();
      continue;
    }
    // Score: resident CTAs (x2 for a ring of two or more buffers), and the smallest cluster whose slice is at most
    // kSliceTarget bytes wins outright (fewer CTAs per row exchange less, three such slices fit an SM).
    long long score = (long long)active * cl * (stages >= 2 ? 2 : 1);
    if (stage_bytes <= kSliceTarget) score = (1LL << 40) + (kMaxCluster - cl);
    if (active > 0 && score > best_score) {
      best_score = score;
      best.cl = cl;
      best.slice = (int)slice;
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
  auto kern = sm_cluster<T>;
  const int smem = p.stages * p.stage_vec * 16;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
    cudaGetLastError();
    return -2;
  }
  if (p.cl > 8) cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  // One row per cluster (measured best: the whole row set in flight, three CTAs per SM), unless the rows exceed the
  // grid's y limit: then as many clusters as stay resident loop over the rows with a ring of slice buffers.
  const long long g = p.ring ? (rows < p.active ? rows : p.active) : rows;
  if (g > 65535) return -2;  // grid.y limit: the caller falls back
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = cluster_config(p.cl, (unsigned)g, smem, s, attr);
  const cudaError_t err = cudaLaunchKernelEx(&cfg, kern, x, y, rows, cols, p.slice, p.stages, p.stage_vec);
  if (err != cudaSuccess) return (int)err;
  return (int)cudaGetLastError();
}

// Rows too long for shared-memory slices: clusters of 16 CTAs (8 if 16 cannot be resident), one row each (rows above
// the grid's y limit loop).
template <typename T>
int start_cluster_wide(const T* x, T* y, long long rows, long long cols, cudaStream_t s) {
  constexpr int V = VecN<T>::N;
  auto kern = sm_cluster_wide<T>;
  for (int cl = 16; cl >= 8; cl /= 2) {
    if (cl > 8 && cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
      cudaGetLastError();
      continue;
    }
    const long long slice = ((cols + cl - 1) / cl + V - 1) / V * V;
    const unsigned gy = (unsigned)(rows < 65535 ? rows : 65535);
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = cluster_config(cl, 1, 0, s, attr);
    int active = 0;
    if (cudaOccupancyMaxActiveClusters(&active, kern, &cfg) != cudaSuccess || active <= 0) {
      cudaGetLastError();
      continue;
    }
    cfg.gridDim = dim3((unsigned)cl, gy, 1);
    const cudaError_t err = cudaLaunchKernelEx(&cfg, kern, x, y, rows, cols, slice);
    if (err != cudaSuccess) return (int)err;
    return (int)cudaGetLastError();
  }
  return -2;
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
#ifndef CKB_SOFTMAX_FORCE_WIDE
#define CKB_SOFTMAX_FORCE_WIDE 0
#endif
  if (vec && CKB_SOFTMAX_FORCE_WIDE) {
    const int err = start_cluster_wide<T>(x, y, rows, cols, s);
    if (err != -2) return err;
  }
  if (vec) {
    const ClusterPlan p = plan_cluster<T>(cols, rows > 65535);
    if (p.cl > 0) {
      const int err = start_cluster<T>(p, x, y, rows, cols, s);
      if (err != -2) return err;
    } else {
      const int err = start_cluster_wide<T>(x, y, rows, cols, s);
      if (err != -2) return err;
    }
  }
  if (rows > INT_MAX) return -1;
  sm_stream<T><<<(unsigned)rows, 1024, 0, s>>>(x, y, cols);
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
