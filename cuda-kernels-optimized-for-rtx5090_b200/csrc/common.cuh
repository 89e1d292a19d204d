// Shared device and host helpers for the four row-wise kernels (softmax, RMSNorm, RoPE, top-k) built for sm_100a.
//
// Conventions every library in this directory follows (the reference's C ABI, e.g. rmsnorm/kernel.cu:132-139):
//   * dtype codes: 0 = fp32, 1 = bf16, 2 = fp16;
//   * return 0 on success (a call with no rows is a successful no-op), -1 for an argument the kernels do not serve,
//     otherwise the cudaError_t of the launch;
//   * launches are asynchronous on the caller's stream and the caller's current device; nothing allocates memory.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <atomic>

namespace ckb {

enum DType : int { kF32 = 0, kBF16 = 1, kF16 = 2 };

constexpr int kWarp = 32;

// ---------------------------------------------------------------------------------------------------------------
// Element conversions. bf16 -> fp32 is exact (the high half of the float); fp32 -> bf16/fp16 is round to nearest even.
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }

// A value rounded to T and widened back to fp32 (identity for fp32).
template <typename T>
__device__ __forceinline__ float round_through(float v) { return to_f32(from_f32<T>(v)); }

// Elements of T in one 16-byte vector.
template <typename T>
struct VecN { static constexpr int N = 16 / sizeof(T); };

// 16 bytes <-> VecN<T>::N floats.
__device__ __forceinline__ void unpack16(const uint4& r, float (&f)[4], const float*) {
  f[0] = __uint_as_float(r.x); f[1] = __uint_as_float(r.y); f[2] = __uint_as_float(r.z); f[3] = __uint_as_float(r.w);
}
__device__ __forceinline__ void unpack16(const uint4& r, float (&f)[8], const __nv_bfloat16*) {
  const unsigned w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    f[2 * j] = __uint_as_float(w[j] << 16);
    f[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
  }
}
__device__ __forceinline__ void unpack16(const uint4& r, float (&f)[8], const __half*) {
  const __half2* h = reinterpret_cast<const __half2*>(&r);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 p = __half22float2(h[j]);
    f[2 * j] = p.x;
    f[2 * j + 1] = p.y;
  }
}
__device__ __forceinline__ uint4 pack16(const float (&f)[4], const float*) {
  return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3]));
}
__device__ __forceinline__ uint4 pack16(const float (&f)[8], const __nv_bfloat16*) {
  uint4 r;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&r);
#pragma unroll
  for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(f[2 * j], f[2 * j + 1]);
  return r;
}
__device__ __forceinline__ uint4 pack16(const float (&f)[8], const __half*) {
  uint4 r;
  __half2* h = reinterpret_cast<__half2*>(&r);
#pragma unroll
  for (int j = 0; j < 4; ++j) h[j] = __floats2half2_rn(f[2 * j], f[2 * j + 1]);
  return r;
}

// ---------------------------------------------------------------------------------------------------------------
// Global memory access with cache policy. Streams read once go around L1 and are marked evict-first in L2; outputs
// are written evict-first (they are not read again by this kernel). In-place kernels read with ld.global.cs instead
// of the non-coherent path, because they write the same addresses later in the same launch.
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ uint4 ld_inplace(const void* p) { return __ldcs(reinterpret_cast<const uint4*>(p)); }
__device__ __forceinline__ void st_stream(void* p, const uint4& v) { __stcs(reinterpret_cast<uint4*>(p), v); }

// ---------------------------------------------------------------------------------------------------------------
// Warp reductions (butterfly: every lane ends with the same bits).
// ---------------------------------------------------------------------------------------------------------------
template <int WIDTH = 32, typename F = float>
__device__ __forceinline__ F warp_sum(F v) {
#pragma unroll
  for (int o = WIDTH / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
template <int WIDTH = 32>
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = WIDTH / 2; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---------------------------------------------------------------------------------------------------------------
// Shared-memory addresses, mbarriers and bulk (TMA) copies, written against the PTX ISA for sm_90+.
// Every wait is bounded by the global timer; a wait that runs out reports false and the caller records an error
// status instead of spinning forever.
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ unsigned smem_u32(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
// Makes mbarrier initialisation visible to the async proxy (bulk copies) and to the rest of the cluster.
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0u;
}

// try_wait that lets the hardware suspend the thread for up to kSuspendNs until the phase completes, so waiting
// warps sleep instead of spinning through the issue slots.
constexpr unsigned kSuspendNs = 100000u;
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendNs)
      : "memory");
  return ok != 0u;
}

constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s: far beyond any copy this library issues

// Waits for the phase with the given parity to complete; false when the wait ran out of time. The clock is read only
// every 64 tries.
#ifndef CKB_MBAR_SUSPEND
#define CKB_MBAR_SUSPEND 1
#endif
__device__ __forceinline__ bool mbar_poll(uint64_t* bar, unsigned parity) {
  return CKB_MBAR_SUSPEND ? mbar_try_wait_suspend(bar, parity) : mbar_try_wait(bar, parity);
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity) {
  if (mbar_poll(bar, parity)) return true;
  const unsigned long long start = global_ns();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_poll(bar, parity)) return true;
    if (global_ns() - start > kWaitLimitNs) return false;
  }
}

// One bulk copy global -> this CTA's shared memory, completing `bytes` of transaction on `bar`. Addresses 16-byte
// aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(void* dst_smem, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Orders this thread's generic-proxy shared-memory accesses before later bulk copies into the same bytes.
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Status word a kernel sets when a bounded wait gave up (0 = fine). One per library, read by <op>_status().
#define CKB_STATUS_TIMEOUT 1u

// ---------------------------------------------------------------------------------------------------------------
// Programmatic dependent launch. A kernel launched with the programmatic-serialisation attribute may be scheduled
// while the previous kernel on its stream is still finishing; pdl_wait() then blocks until that kernel has completed
// and its memory operations are visible (so every read of an input and every write of an output comes after it),
// and pdl_trigger() lets the next such kernel be scheduled once every CTA of this one has started. Both are no-ops
// for a kernel launched without the attribute.
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

}  // namespace ckb

// ---------------------------------------------------------------------------------------------------------------
// Host side: per-device SM count (cached for up to 64 devices; thread-safe, racing first calls store the same value).
// ---------------------------------------------------------------------------------------------------------------
namespace ckb {
inline int device_sm_count() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return 148;
  }
  if (dev < 0 || dev >= 64) dev = 0;
  int n = cache[dev].load(std::memory_order_relaxed);
  if (n > 0) return n;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = 148;
  }
  cache[dev].store(n, std::memory_order_relaxed);
  return n;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Launches kernel<<<grid, block, smem, stream>>>(args...) with programmatic stream serialisation allowed, so it can
// overlap the tail of the kernel before it on the stream (its pdl_wait() keeps every data dependency).
#ifndef CKB_PDL
#define CKB_PDL 1  // 0: launch without programmatic serialisation (measurements)
#endif
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = CKB_PDL ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}
}  // namespace ckb

#define CKB_EXPORT extern "C" __attribute__((visibility("default")))
