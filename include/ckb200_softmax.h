/* Softmax library (lib/softmax/libkernel.so): row-wise softmax over the last dim on B200 (sm_100a).
 *
 * Conventions shared by every ckb200 library: row-major contiguous buffers in device memory owned by the caller;
 * dtype codes 0 = fp32, 1 = bf16, 2 = fp16; return 0 on success (no rows is a successful no-op), -1 for arguments
 * the kernels do not serve, otherwise the cudaError_t of the launch; launches are asynchronous on `stream` and the
 * caller's current device; nothing allocates memory. */
#ifndef CKB200_SOFTMAX_H
#define CKB200_SOFTMAX_H

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

/* y[rows, cols] = softmax(x[rows, cols], dim = -1), fp32 (dtype 0) or bf16 (dtype 1), fp32 math.
 * Replaces the reference's `launch` (softmax/kernel.cu:520-527; also softmax/seed.cu:68-81), same symbol and
 * argument list. threads / aux are the reference's block-size hints: accepted, not needed on B200. */
int launch(const void* x, void* y, long long rows, long long cols, int dtype, int threads, int aux,
           cudaStream_t stream);

/* Bounded-wait status of the cluster kernel since the last reset: 0 fine, 1 a bulk-copy wait gave up (that launch's
 * output is invalid; no kernel hangs). Synchronous; reset != 0 clears it. Negative: -cudaError_t of the query.
 * No counterpart in the reference (its kernels never wait on a copy). */
int ckb_softmax_status(int reset);

#ifdef __cplusplus
}
#endif
#endif
