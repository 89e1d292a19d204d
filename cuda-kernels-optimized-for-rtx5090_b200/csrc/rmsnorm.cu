// RMSNorm of x[rows, cols] over the last dim, bf16 (dtype 1) or fp16 (dtype 2) rows, fp32 accumulation.
//
// Two entry points:
//   launch(...)                      the reference's ABI and semantics (rmsnorm/kernel.cu:1-8,132-139): no weight,
//                                    y = T(x * T(rsqrt(sum(x^2) / cols + eps))) -- the inverse is rounded to the
//                                    row dtype before the product (rmsnorm/kernel.cu:46,93);
//   ckb_rmsnorm_weighted_launch(...) the weighted form y = T((x * rsqrt(sum(x^2) / cols + eps)) * w) with the inverse
//                                    and both products in fp32 and one rounding at the end; w is fp32, bf16 or fp16.
// A NaN in a row makes the row NaN; a sum that overflows gives an inverse of 0 (as the reference).
//
// B200 mapping (HBM bound: 2 bytes read + 2 written per element, the weight stays in L1/L2):
//   * rows of at most 128 16-byte vectors: one warp per row, 8 rows per 256-thread block, no block barrier;
//   * rows of at most 4096 vectors: one block per row, each thread keeps VPT 16-byte vectors in registers
//     (VPT = 1..8, chosen so a block has about 256 threads, 128 with a weight) and the weight's vectors for the same
//     columns, fetched with the row's loads so no weight load waits behind the reduction; one barrier per row;
//   * anything else (cols % 8 != 0, a pointer not 16-byte aligned, longer rows): a scalar block-per-row kernel that
//     reads the row twice.
#include "ckb200_rmsnorm.h"
#include "common.cuh"

#include <climits>
#include <type_traits>

namespace ckb {
namespace {

struct NoWeight {};

// The weight of 8 consecutive columns starting at element i (a multiple of 8, w 16-byte aligned), fetched raw so the
// load can be issued with the row's own loads and widened to fp32 only where it is used.
struct NoW8 {};
struct W8x16 { uint4 r; };
struct W8x32 { float4 a, b; };
template <typename WT> struct WRaw { using type = W8x16; };
template <> struct WRaw<NoWeight> { using type = NoW8; };
template <> struct WRaw<float> { using type = W8x32; };

__device__ __forceinline__ NoW8 fetch_w8(const NoWeight*, long long) { return {}; }
__device__ __forceinline__ W8x32 fetch_w8(const float* w, long long i) {
  return {__ldg(reinterpret_cast<const float4*>(w + i)), __ldg(reinterpret_cast<const float4*>(w + i) + 1)};
}
template <typename W>
__device__ __forceinline__ W8x16 fetch_w8(const W* w, long long i) {
  return {__ldg(reinterpret_cast<const uint4*>(w + i))};
}
__device__ __forceinline__ void widen_w8(const NoW8&, const NoWeight*, float (&)[8]) {}
__device__ __forceinline__ void widen_w8(const W8x32& r, const float*, float (&f)[8]) {
  f[0] = r.a.x; f[1] = r.a.y; f[2] = r.a.z; f[3] = r.a.w;
  f[4] = r.b.x; f[5] = r.b.y; f[6] = r.b.z; f[7] = r.b.w;
}
template <typename W>
__device__ __forceinline__ void widen_w8(const W8x16& r, const W* w, float (&f)[8]) {
  unpack16(r.r, f, w);
}

__device__ __forceinline__ float load_w1(const NoWeight*, long long) { return 1.0f; }
template <typename W>
__device__ __forceinline__ float load_w1(const W* w, long long i) { return to_f32(w[i]); }

// The row's inverse RMS from the fp32 sum of squares: rounded to T without a weight (the reference's semantics),
// kept in fp32 with one.
template <typename T, bool kWeighted>
__device__ __forceinline__ float row_inv(float total, int cols, float eps) {
  const float inv = rsqrtf(total / (float)cols + eps);
  return kWeighted ? inv : round_through<T>(inv);
}

// Normalises the 8 values of one vector in place: f = f * inv (* w).
template <bool kWeighted>
__device__ __forceinline__ void scale8(float (&f)[8], float inv, const float (&w)[8]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) f[j] = kWeighted ? (f[j] * inv) * w[j] : f[j] * inv;
}

// One warp per row, lane l holding vectors l, l + 32, ..., l + 32 (VPT - 1).
template <typename T, typename WT, int VPT>
__global__ void __launch_bounds__(256) rms_warp_rows(const T* __restrict__ x, const WT* __restrict__ w,
                                                     T* __restrict__ y, long long rows, int cols, float eps) {
  constexpr bool kW = !std::is_same<WT, NoWeight>::value;
  pdl_wait();
  pdl_trigger();
  const long long row = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;  // whole warps leave together: no shuffle is left waiting
  const int lane = threadIdx.x & 31;
  const int nvec = cols >> 3;
  const T* xr = x + row * cols;
  T* yr = y + row * cols;
  uint4 v[VPT];
  typename WRaw<WT>::type wr[VPT];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int i = lane + 32 * k;
    v[k] = i < nvec ? ld_stream(xr + 8 * i) : make_uint4(0u, 0u, 0u, 0u);
  }
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int i = lane + 32 * k;
    if (i < nvec) wr[k] = fetch_w8(w, 8LL * i);
  }
  float ss = 0.0f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    float f[8];
    unpack16(v[k], f, x);
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = fmaf(f[j], f[j], ss);  // exact squares of 16-bit values
  }
  const float inv = row_inv<T, kW>(warp_sum(ss), cols, eps);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int i = lane + 32 * k;
    if (i < nvec) {
      float f[8], wf[8];
      unpack16(v[k], f, x);
      widen_w8(wr[k], w, wf);
      scale8<kW>(f, inv, wf);
      st_stream(yr + 8 * i, pack16(f, x));
    }
  }
}

// Block-size bound of rms_block_rows: fp32 weights hold twice the registers per vector, so their shapes stop at
// half the threads (the dispatcher sends longer fp32-weighted rows to rms_generic).
template <typename WT, int VPT>
constexpr int block_rows_bound() {
  return std::is_same<WT, float>::value ? (VPT >= 8 ? 256 : 512) : (VPT >= 8 ? 512 : 1024);
}

// One block per row, thread t holding vectors t, t + B, ..., t + B (VPT - 1) (B = blockDim.x).
template <typename T, typename WT, int VPT>
__global__ void __launch_bounds__(block_rows_bound<WT, VPT>()) rms_block_rows(const T* __restrict__ x, const WT* __restrict__ w,
                                                       T* __restrict__ y, int cols, float eps) {
  constexpr bool kW = !std::is_same<WT, NoWeight>::value;
  __shared__ float slots[32];
  pdl_wait();
  pdl_trigger();
  const int nvec = cols >> 3;
  const long long off = (long long)blockIdx.x * cols;
  const T* xr = x + off;
  T* yr = y + off;
  uint4 v[VPT];
  typename WRaw<WT>::type wr[VPT];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    v[k] = i < nvec ? ld_stream(xr + 8 * i) : make_uint4(0u, 0u, 0u, 0u);
  }
#pragma unroll
  for (int k = 0; k < VPT; ++k) {  // the weight's loads go out with the row's, off the row's critical path
    const int i = threadIdx.x + k * blockDim.x;
    if (i < nvec) wr[k] = fetch_w8(w, 8LL * i);
  }
  float ss = 0.0f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    float f[8];
    unpack16(v[k], f, x);
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = fmaf(f[j], f[j], ss);
  }
  // One barrier: each warp posts its sum, then every thread folds the posts in the same order.
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) slots[threadIdx.x >> 5] = ss;
  __syncthreads();
  const int warps = blockDim.x >> 5;
  float total = 0.0f;
  for (int i = 0; i < warps; ++i) total += slots[i];
  const float inv = row_inv<T, kW>(total, cols, eps);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    if (i < nvec) {
      float f[8], wf[8];
      unpack16(v[k], f, x);
      widen_w8(wr[k], w, wf);
      scale8<kW>(f, inv, wf);
      st_stream(yr + 8 * i, pack16(f, x));
    }
  }
}

// Any shape and alignment: scalar loads, the row read twice (the second time mostly from L2).
template <typename T, typename WT>
__global__ void __launch_bounds__(1024) rms_generic(const T* __restrict__ x, const WT* __restrict__ w,
                                                    T* __restrict__ y, int cols, float eps) {
  pdl_wait();
  pdl_trigger();
  constexpr bool kW = !std::is_same<WT, NoWeight>::value;
  __shared__ float slots[32];
  const long long off = (long long)blockIdx.x * cols;
  float ss = 0.0f;
  for (int i = threadIdx.x; i < cols; i += blockDim.x) {
    const float f = to_f32(x[off + i]);
    ss = fmaf(f, f, ss);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) slots[threadIdx.x >> 5] = ss;
  __syncthreads();
  const int warps = blockDim.x >> 5;
  float total = 0.0f;
  for (int i = 0; i < warps; ++i) total += slots[i];
  const float inv = row_inv<T, kW>(total, cols, eps);
  for (int i = threadIdx.x; i < cols; i += blockDim.x) {
    const float f = to_f32(x[off + i]);
    y[off + i] = from_f32<T>(kW ? (f * inv) * load_w1(w, i) : f * inv);
  }
}

constexpr int kWarpRowsMaxVec = 128;      // warp path: at most 4 vectors per lane
constexpr int kBlockRowsMaxVec = 4096;    // block path: at most 512 threads x 8 vectors
// Block path: VPT grows until a row needs at most this many threads. Measured on B200 at 16384 x 4096 bf16 (and
// 2048 rows): without a weight 256 threads (2 vectors each) are fastest, with one 128 threads (4 vectors and the
// weight's 4, more registers per thread but fewer, fuller CTAs).
#ifndef CKB_RMSNORM_TARGET_THREADS
#define CKB_RMSNORM_TARGET_THREADS 256
#endif
#ifndef CKB_RMSNORM_TARGET_THREADS_W
#define CKB_RMSNORM_TARGET_THREADS_W 128
#endif

template <typename T, typename WT, int VPT>
void start_warp(const void* x, const void* w, void* y, long long rows, int cols, float eps, cudaStream_t s) {
  const unsigned grid = (unsigned)((rows + 7) / 8);
  launch_pdl(rms_warp_rows<T, WT, VPT>, dim3(grid), dim3(256), 0, s, (const T*)x, (const WT*)w, (T*)y, rows, cols,
             eps);
}

template <typename T, typename WT, int VPT>
void start_block(const void* x, const void* w, void* y, long long rows, int cols, int threads, float eps,
                 cudaStream_t s) {
  launch_pdl(rms_block_rows<T, WT, VPT>, dim3((unsigned)rows), dim3(threads), 0, s, (const T*)x, (const WT*)w,
             (T*)y, cols, eps);
}

template <typename T, typename WT>
int dispatch(const void* x, const void* w, void* y, long long rows, int cols, float eps, int generic_threads,
             cudaStream_t s) {
  const bool vec = cols % 8 == 0 && aligned16(x) && aligned16(y) && (w == nullptr || aligned16(w));
  const int nvec = cols / 8;
  if (vec && nvec <= kWarpRowsMaxVec) {
    if (nvec <= 32) start_warp<T, WT, 1>(x, w, y, rows, cols, eps, s);
    else if (nvec <= 64) start_warp<T, WT, 2>(x, w, y, rows, cols, eps, s);
    else start_warp<T, WT, 4>(x, w, y, rows, cols, eps, s);
    return (int)cudaGetLastError();
  }
  if (vec && nvec <= (std::is_same<WT, float>::value ? kBlockRowsMaxVec / 2 : kBlockRowsMaxVec)) {
    constexpr int target = std::is_same<WT, NoWeight>::value ? CKB_RMSNORM_TARGET_THREADS
                                                             : CKB_RMSNORM_TARGET_THREADS_W;
    int vpt = 1;
    while (vpt < 8 && (nvec + vpt - 1) / vpt > target) vpt *= 2;
    const int threads = ((nvec + vpt - 1) / vpt + 31) / 32 * 32;
    switch (vpt) {
      case 1: start_block<T, WT, 1>(x, w, y, rows, cols, threads, eps, s); break;
      case 2: start_block<T, WT, 2>(x, w, y, rows, cols, threads, eps, s); break;
      case 4: start_block<T, WT, 4>(x, w, y, rows, cols, threads, eps, s); break;
      default: start_block<T, WT, 8>(x, w, y, rows, cols, threads, eps, s); break;
    }
    return (int)cudaGetLastError();
  }
  launch_pdl(rms_generic<T, WT>, dim3((unsigned)rows), dim3(generic_threads), 0, s, (const T*)x, (const WT*)w, (T*)y,
             cols, eps);
  return (int)cudaGetLastError();
}

template <typename T>
int dispatch_weight(int w_dtype, const void* x, const void* w, void* y, long long rows, int cols, float eps,
                    cudaStream_t s) {
  switch (w_dtype) {
    case kF32: return dispatch<T, float>(x, w, y, rows, cols, eps, 256, s);
    case kBF16: return dispatch<T, __nv_bfloat16>(x, w, y, rows, cols, eps, 256, s);
    case kF16: return dispatch<T, __half>(x, w, y, rows, cols, eps, 256, s);
    default: return -1;
  }
}

}  // namespace
}  // namespace ckb

using namespace ckb;

// Replaces the reference's rmsnorm `launch` (rmsnorm/kernel.cu:132-139): same arguments, checks and return codes.
// `threads` is validated as the reference does and used as the block size of the scalar fallback; the vectorised
// paths choose their own block shape for B200.
CKB_EXPORT int launch(const void* x, void* y, long long rows, int cols, int dtype, float eps, int threads,
                      cudaStream_t stream) {
  if (rows <= 0) return 0;
  if (rows > INT_MAX || cols <= 0 || threads < kWarp || threads > 1024 || threads % kWarp) return -1;
  if (dtype == kBF16) return dispatch<__nv_bfloat16, NoWeight>(x, nullptr, y, rows, cols, eps, threads, stream);
  if (dtype == kF16) return dispatch<__half, NoWeight>(x, nullptr, y, rows, cols, eps, threads, stream);
  return -1;
}

// Weighted RMSNorm (no counterpart in the reference): y = T((x * rsqrt(mean(x^2) + eps)) * w), fp32 throughout,
// one rounding. dtype 1 (bf16) or 2 (fp16) rows; w_dtype 0 (fp32), 1 (bf16) or 2 (fp16), w holds cols values.
CKB_EXPORT int ckb_rmsnorm_weighted_launch(const void* x, const void* w, void* y, long long rows, int cols,
                                           int dtype, int w_dtype, float eps, cudaStream_t stream) {
  if (rows <= 0) return 0;
  if (rows > INT_MAX || cols <= 0 || w == nullptr) return -1;
  if (dtype == kBF16) return dispatch_weight<__nv_bfloat16>(w_dtype, x, w, y, rows, cols, eps, stream);
  if (dtype == kF16) return dispatch_weight<__half>(w_dtype, x, w, y, rows, cols, eps, stream);
  return -1;
}
