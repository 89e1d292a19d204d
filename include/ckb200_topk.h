/* Top-k library (lib/topk/libkernel.so) on B200 (sm_100a). Conventions as in ckb200_softmax.h. */
#ifndef CKB200_TOPK_H
#define CKB200_TOPK_H

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Columns per CTA for a rows x cols launch of dtype 0 (fp32) or 1 (bf16); ceil(cols / chunk) chunks per row.
 * Replaces the reference's `plan` (topk/kernel.cu:520-547), same symbol and arguments (threads and depth are the
 * reference's kernel knobs; min_chunk bounds the chunk from below). */
long long plan(long long rows, long long cols, int dtype, int threads, int depth, int min_chunk);

/* values [rows, k] (x's dtype) and indices [rows, k] (int64) = the k largest entries of each row of x [rows, cols],
 * descending, ties by lower index, values bit-exact. work: int64 [rows * chunks * k] when chunks > 1; counters:
 * int32 [rows], zero on entry, left zero. Replaces the reference's `launch` (topk/kernel.cu:549-570), same symbol,
 * arguments, checks (k <= cols, k <= 512, rows <= 65535, threads in {128, 256, 512}, depth in {2, 4, 8}) and
 * return codes; `chunk` must come from plan(). */
int launch(const void* x, void* values, void* indices, void* work, void* counters, long long rows, long long cols,
           int k, int dtype, int threads, int depth, long long chunk, cudaStream_t stream);

/* Vocab-sharded variant, local half: x [rows, cols] holds global columns [col_offset, col_offset + cols); lists
 * [rows, k] receives each row's top k as sorted 64-bit composites (order key << 32 | ~global_index), zero padded.
 * work / counters / chunk as in launch(). No counterpart in the reference (single GPU). */
int ckb_topk_shard_launch(const void* x, unsigned long long* lists, void* work, void* counters, long long rows,
                          long long cols, long long col_offset, int k, int dtype, long long chunk,
                          cudaStream_t stream);

/* Vocab-sharded variant, merge half: lists [nlists][rows][k] (the shards' lists after an all-gather) -> values
 * [rows, k] in dtype 0 / 1 and int64 indices [rows, k]. No counterpart in the reference. */
int ckb_topk_merge_launch(const unsigned long long* lists, int nlists, void* values, void* indices, long long rows,
                          int k, int dtype, cudaStream_t stream);

/* The top-k of launch() for callers that cannot allocate device memory (a host framework that owns the GPU's memory
 * through its own fixed-budget allocator, or a path that cannot afford cudaMalloc's device synchronisation): no
 * workspace or counters are passed; a 4 MiB scratch array compiled into this library (held on every GPU that loads
 * it, until exit) serves instead. No counterpart in the reference. dtype 0 fp32 / 1 bf16; returns -1 for arguments
 * launch() rejects, -2 for more than 65,536 rows (beyond the scratch's counters; launch() rejects those anyway). A
 * plan whose split rows would need more workspace than the scratch's 491,520 composites runs each row in one piece
 * instead. The first call on a device looks up the scratch address: make it before any stream capture. All calls
 * share the scratch, so calls that overlap on the GPU race; the counters are cleared on `stream` at every call. */
int ckb_topk_launch_noalloc(const void* x, void* values, void* indices, long long rows, long long cols, int k,
                            int dtype, cudaStream_t stream);

/* Status word of this library's kernels since the last reset (0 fine; the streaming kernel waits only on its own
 * asynchronous copies, which always complete, so nothing sets it today). Synchronous; reset != 0 clears it; negative:
 * -cudaError_t. No counterpart in the reference. */
int ckb_topk_status(int reset);

#ifdef __cplusplus
}
#endif
#endif
