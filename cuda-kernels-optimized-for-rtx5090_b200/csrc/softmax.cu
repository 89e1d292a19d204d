// Row-wise softmax over the last dim: y = exp(x - max) / sum(exp(x - max)), fp32 (dtype 0) and bf16 (dtype 1) rows,
// every value computed in fp32. Semantics follow the reference's torch.softmax(x, dim=-1) (softmax/baseline.py:12-13);
// the C entry keeps the reference's ABI (softmax/kernel.cu:520-527).
//
// Paths, chosen by row length (all read each element once from HBM and write it once):
//   * group path, rows of at most 256 16-byte vectors: G = 4..32 lanes per row, so one warp holds 32 / G rows and
//     every lane keeps NV vectors of its row in registers; group-local shuffles, no barrier;
//   * block path, rows of at most 2048 vectors: one block per row, NV vectors per thread in registers,
//     two barriers per row;
//   * cluster path, longer rows: the row is split over a thread-block cluster of CL CTAs (2..16). Each CTA pulls
//     its own slice into its own shared memory with bulk copies (cp.async.bulk, several pieces on separate
//     mbarriers so the max can start on the first piece), the CTAs exchange the max and then the sum through
//     distributed shared memory, and each CTA normalises from shared memory. No copy is multicast;
//   * stream path (unaligned pointers, cols not a multiple of the vector, or rows too long for the cluster slices):
//     one block per row reading the row three times (max, sum, normalise; the later reads mostly from L2).
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
template <typename T, int NV>
__global__ void __launch_bounds__(NV >= 8 ? 512 : 1024) sm_block(const T* __restrict__ x, T* __restrict__ y, int cols) {
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
constexpr int kPieces = 4;  // bulk copies (and mbarriers) per slice

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

// Grid (CL, rows), cluster (CL, 1, 1). CTA `rank` owns elements [rank * slice, min((rank + 1) * slice, cols)) of row
// blockIdx.y, staged in dynamic shared memory. slice and cols are multiples of the 16-byte vector.
template <typename T>
__global__ void __launch_bounds__(kClusterThreads) sm_cluster(const T* __restrict__ x, T* __restrict__ y,
                                                              long long cols, int slice) {
  constexpr int V = VecN<T>::N;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t bars[kPieces];
  __shared__ float red[32];
  __shared__ double red_d[32];
  __shared__ float part_max;   // this CTA's max, read by the peers
  __shared__ double part_sum;  // this CTA's sum, read by the peers
  __shared__ float row_max;
  __shared__ double row_sum;

  cg::cluster_group cluster = cg::this_cluster();
  const unsigned rank = cluster.block_rank();
  const unsigned csize = cluster.num_blocks();
  const long long row = blockIdx.y;
  const long long beg = (long long)rank * slice;
  long long n = cols - beg;
  n = n < 0 ? 0 : (n > slice ? slice : n);
  const int nv = (int)(n / V);                        // vectors in this slice
  const int pv = (nv + kPieces - 1) / kPieces;        // vectors per piece
  const T* src = x + row * cols + beg;
  T* dst = y + row * cols + beg;
  uint4* buf = reinterpret_cast<uint4*>(smem_raw);

  if (threadIdx.x == 0) {
#pragma unroll
    for (int p = 0; p < kPieces; ++p) mbar_init(&bars[p], 1);
    mbar_fence_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
#pragma unroll
    for (int p = 0; p < kPieces; ++p) {
      const int v0 = p * pv, v1 = min(nv, v0 + pv);
      if (v1 > v0) {
        const unsigned bytes = (unsigned)(v1 - v0) * 16u;
        mbar_arrive_expect_tx(&bars[p], bytes);
        bulk_load(buf + v0, reinterpret_cast<const uint4*>(src) + v0, bytes, &bars[p]);
      }
    }
  }

  // Pass 1: max over the slice as each piece lands.
  bool ok = true;
  float m = -CUDART_INF_F;
#pragma unroll
  for (int p = 0; p < kPieces; ++p) {
    const int v0 = p * pv, v1 = min(nv, v0 + pv);
    if (v1 <= v0) continue;
    ok = mbar_wait(&bars[p], 0) && ok;
    for (int i = v0 + threadIdx.x; i < v1; i += blockDim.x) {
      float f[V];
      unpack16(buf[i], f, x);
#pragma unroll
      for (int j = 0; j < V; ++j) m = fmaxf(m, f[j]);
    }
  }
  if (!ok) atomicOr(&g_softmax_status, CKB_STATUS_TIMEOUT);
  m = block_max(m, red);
  if (threadIdx.x == 0) part_max = m;
  cluster_arrive();
  cluster_wait();
  if (threadIdx.x < 32) {
    float pm = threadIdx.x < csize ? *cluster.map_shared_rank(&part_max, threadIdx.x) : -CUDART_INF_F;
    pm = warp_max(pm);
    if (threadIdx.x == 0) row_max = pm;
  }
  __syncthreads();
  m = row_max;

  // Pass 2: sum of exp(x - max); fp32 slices keep the exponentials in place for pass 3.
  double s = 0.0;
  for (int i = threadIdx.x; i < nv; i += blockDim.x) {
    float f[V];
    unpack16(buf[i], f, x);
    s += (double)exp_vec(f, m);
    if constexpr (V == 4) buf[i] = pack16(f, x);
  }
  s = block_sum(s, red_d);
  if (threadIdx.x == 0) part_sum = s;
  cluster_arrive();
  cluster_wait();
  if (threadIdx.x < 32) {
    double ps = threadIdx.x < csize ? *cluster.map_shared_rank(&part_sum, threadIdx.x) : 0.0;
    ps = warp_sum(ps);
    if (threadIdx.x == 0) row_sum = ps;
  }
  // Peers may still read this CTA's part_sum until they pass the next cluster barrier; arrive now, wait at the end.
  cluster_arrive();
  __syncthreads();
  const float inv = (float)(1.0 / row_sum);

  // Pass 3: normalise from shared memory, stream to HBM.
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
  cluster_wait();
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

template <typename T, int NV>
int start_block(const T* x, T* y, long long rows, int cols, int threads, cudaStream_t s) {
  if (rows > INT_MAX) return -1;
  sm_block<T, NV><<<(unsigned)rows, threads, 0, s>>>(x, y, cols);
  return (int)cudaGetLastError();
}

constexpr int kMaxSliceBytes = 200 * 1024;

struct ClusterPlan {
  int cl = 0;     // 0: no cluster configuration fits
  int slice = 0;  // elements per CTA
  int smem = 0;   // dynamic shared memory bytes per CTA
};

// The cluster shape for rows of `cols` elements: for each cluster size whose slice fits in shared memory, the number
// of CTAs the device keeps resident (cudaOccupancyMaxActiveClusters x size); the size with the most resident CTAs
// wins, the smaller size on a tie. Cached per (device, dtype, cols); the cache holds the last shape asked for.
template <typename T>
ClusterPlan plan_cluster(long long cols) {
  constexpr int V = VecN<T>::N;
  static std::mutex mu;
  static int last_dev = -1;
  static long long last_cols = -1;
  static ClusterPlan last;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev == last_dev && cols == last_cols) return last;
  }
  ClusterPlan best;
  long long best_ctas = 0;
  for (int cl = 2; cl <= 16; cl *= 2) {
    long long slice = ((cols + cl - 1) / cl + V - 1) / V * V;
    const long long bytes = slice * (long long)sizeof(T);
    if (bytes > kMaxSliceBytes) continue;
    const int smem = (int)((bytes + 127) / 128 * 128);
    auto kern = sm_cluster<T>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess ||
        (cl > 8 && cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)) {
      cudaGetLastError();
      continue;
    }
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)cl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3((unsigned)cl, 1, 1);
    cfg.blockDim = dim3(kClusterThreads, 1, 1);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int active = 0;
    if (cudaOccupancyMaxActiveClusters(&active, kern, &cfg) != cudaSuccess) {
      cudaGetLastError();
      continue;
    }
    const long long ctas = (long long)active * cl;
    if (ctas > best_ctas) {
      best_ctas = ctas;
      best.cl = cl;
      best.slice = (int)slice;
      best.smem = smem;
    }
  }
  std::lock_guard<std::mutex> lock(mu);
  last_dev = dev;
  last_cols = cols;
  last = best;
  return best;
}

template <typename T>
int start_cluster(const ClusterPlan& p, const T* x, T* y, long long rows, long long cols, cudaStream_t s) {
  if (rows > 65535) return -2;  // grid.y limit: the caller falls back
  auto kern = sm_cluster<T>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, p.smem) != cudaSuccess) {
    cudaGetLastError();
    return -2;
  }
  if (p.cl > 8) cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)p.cl;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3((unsigned)p.cl, (unsigned)rows, 1);
  cfg.blockDim = dim3(kClusterThreads, 1, 1);
  cfg.dynamicSmemBytes = (size_t)p.smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, kern, x, y, cols, p.slice);
  if (err != cudaSuccess) return (int)err;
  return (int)cudaGetLastError();
}

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
    // Block path: NV = kMaxNV with the fewest threads, up to 512.
    if (nvec <= 512LL * kMaxNV) {
      const int threads = (int)((nvec + kMaxNV - 1) / kMaxNV + 31) / 32 * 32;
      return start_block<T, kMaxNV>(x, y, rows, c, threads, s);
    }
  }
  if (vec) {
    const ClusterPlan p = plan_cluster<T>(cols);
    if (p.cl > 0) {
      const int err = start_cluster<T>(p, x, y, rows, cols, s);
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
