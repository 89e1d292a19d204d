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

/* Top-k sampling: the top k of each row found as launch() does, then probs [rows, k] (float) = the softmax over those k
 * logits divided by temperature (> 0, finite), in rank order, with their int64 indices [rows, k]; with uniforms
 * (float [rows], each in [0, 1)) the sampled token of each row, the index of the first entry whose cumulative
 * probability exceeds the row's uniform, into samples (int64 [rows]); uniforms and samples are both null or both
 * set. work / counters / chunk as in launch(). No counterpart in the reference (its top-k stops at the values,
 * topk/kernel.cu:436-441): the softmax over the k survivors runs in the top-k kernel's epilogue, so the vocab row is
 * read once. */
int ckb_topk_softmax_launch(const void* x, float* probs, long long* indices, void* work, void* counters,
                            long long rows, long long cols, int k, int dtype, long long chunk, float temperature,
                            const float* uniforms, long long* samples, cudaStream_t stream);

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

/* Vocab-sharded variant over peer memory (one process per GPU; no counterpart in the reference, which is single-GPU).
 * Each rank owns an exchange buffer that every rank maps (ckb_p2p_*), double buffered by call parity; a parity half
 * holds lists [world][rows][k] (uint64 composites) and flags [world][rows] (uint32, zero at allocation).
 * Local half: as ckb_topk_shard_launch, but every row's sorted list is stored into slot `rank` of every rank's lists
 * (NVLink stores) and then flags[p][rank * rows + row] = epoch on every rank p (release, system scope). lists / flags:
 * host arrays of `world` device pointers to this parity's half of each rank's buffer (this rank's own included).
 * values / indices (both null, or both set): when set, the final top k of the full rows [rows, k] (x's dtype, int64)
 * is written too, by the same kernel when all of its CTAs fit on the GPU at once (each row waits for the other
 * ranks' lists of the row in this rank's buffer, then merges; waits bounded as below), otherwise by a
 * ckb_topk_merge_wait_launch queued behind it. 1 <= world <= 8, 0 <= rank < world, epoch != 0; flags are compared
 * for equality, so successive calls must alternate parity (half = epoch & 1) and two calls on one half must carry
 * different epochs (counting calls from 1 does both; so does cycling 1, 2, 3, 4). */
int ckb_topk_shard_push_launch(const void* x, void* values, void* indices, void* work, void* counters, long long rows,
                               long long cols, long long col_offset, int k, int dtype, long long chunk,
                               unsigned long long* const* lists, unsigned* const* flags, int world, int rank,
                               unsigned epoch, cudaStream_t stream);

/* Merge half: lists / flags = this rank's own buffer half for this parity. Row r waits until flags[p][r] equals
 * `epoch` for every rank p (at most 2 s; a wait that runs out sets ckb_topk_status() and the row is merged from
 * whatever is there), then writes values [rows, k] (dtype 0 fp32 / 1 bf16) and int64 indices [rows, k] as
 * ckb_topk_merge_launch. */
int ckb_topk_merge_wait_launch(const unsigned long long* lists, const unsigned* flags, int world, unsigned epoch,
                               void* values, void* indices, long long rows, int k, int dtype, cudaStream_t stream);

/* Exchange buffers: alloc gives `bytes` of zeroed device memory on the current device; export writes the 64-byte CUDA
 * IPC handle of an alloc'd pointer; import maps a peer's handle into this process (peer access enabled lazily);
 * close unmaps an imported pointer; free releases an alloc'd one. Each returns 0 or the cudaError_t (-1 for null
 * arguments). */
int ckb_p2p_alloc(void** ptr, unsigned long long bytes);
int ckb_p2p_free(void* ptr);
int ckb_p2p_export(const void* ptr, void* handle);
int ckb_p2p_import(const void* handle, void** ptr);
int ckb_p2p_close(void* ptr);

/* The top-k of launch() for callers that cannot allocate device memory (a host framework that owns the GPU's memory
 * through its own fixed-budget allocator, or a path that cannot afford cudaMalloc's device synchronisation): no
 * workspace or counters are passed; a 4 MiB scratch array compiled into this library (held on every GPU that loads
 * it, until exit) serves instead. No counterpart in the reference. dtype 0 fp32 / 1 bf16; returns -1 for arguments
 * launch() rejects (more than 65,535 rows among them; the scratch holds a counter for each of those). A plan whose
 * split rows would need more workspace than the scratch's 491,520 composites runs each row in one piece instead.
 * The first call on a device looks up the scratch address and keeps it for the life of the process: make that call
 * before any stream capture, and do not reset the device afterwards. All calls share the scratch, so calls that
 * overlap on the GPU race; the counters are cleared on `stream` at every call. */
int ckb_topk_launch_noalloc(const void* x, void* values, void* indices, long long rows, long long cols, int k,
                            int dtype, cudaStream_t stream);

/* Status word of this library's kernels since the last reset: 0 fine, 1 a peer-memory wait (the vocab-sharded
 * variant's per-row flags) ran out. Synchronous; reset != 0 clears it; negative: -cudaError_t. No counterpart in the
 * reference. */
int ckb_topk_status(int reset);

#ifdef __cplusplus
}
#endif
#endif
