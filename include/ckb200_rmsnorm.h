/* RMSNorm library (lib/rmsnorm/libkernel.so) on B200 (sm_100a). Conventions as in ckb200_softmax.h. */
#ifndef CKB200_RMSNORM_H
#define CKB200_RMSNORM_H

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

/* y = x * T(rsqrt(mean(x^2) + eps)) rounded to T, x and y [rows, cols] of bf16 (dtype 1) or fp16 (dtype 2), no
 * weight. Replaces the reference's `launch` (rmsnorm/kernel.cu:132-139), same symbol, arguments, checks (rows <=
 * INT_MAX, cols > 0, threads a multiple of 32 in [32, 1024]) and return codes. */
int launch(const void* x, void* y, long long rows, int cols, int dtype, float eps, int threads, cudaStream_t stream);

/* Weighted RMSNorm: y = T((x * rsqrt(mean(x^2) + eps)) * w), fp32 math, one rounding; w [cols] of w_dtype 0 (fp32),
 * 1 (bf16) or 2 (fp16). No counterpart in the reference (its RMSNorm has no weight, rmsnorm/kernel.cu:1); the same
 * call shape as its `launch` with the weight pointer and dtype added. */
int ckb_rmsnorm_weighted_launch(const void* x, const void* w, void* y, long long rows, int cols, int dtype,
                                int w_dtype, float eps, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
#endif
