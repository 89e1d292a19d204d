/* RoPE library (lib/rope/libkernel.so) on B200 (sm_100a). Conventions as in ckb200_softmax.h. */
#ifndef CKB200_ROPE_H
#define CKB200_ROPE_H

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Rotates q [tokens, q_heads, head_dim] and k [tokens, kv_heads, head_dim] (qk_dtype 1 bf16, 2 fp16) by the cos/sin
 * cache rows [*, head_dim] (cache_dtype 0 fp32, 1 bf16, 2 fp16) that ids (int64 [tokens], each in [0, rows of the
 * cache)) pick; half-split pairing, fp32 math with separately rounded products and sum. q_out == q and k_out == k
 * rotate in place. Replaces the reference's `launch` (rope/kernel.cu:201-215), same symbol, arguments, checks and
 * return codes; rows / splits are its block-shape knobs, validated, not needed on B200. */
int launch(const void* q, const void* k, const void* cos_rows, const void* sin_rows, const void* ids, void* q_out,
           void* k_out, long long tokens, int q_heads, int kv_heads, int head_dim, int qk_dtype, int cache_dtype,
           int rows, int splits, cudaStream_t stream);

/* The same rotation with cos/sin computed in registers: angle_i = (float)ids[t] * inv_freq[i] (inv_freq fp32
 * [head_dim / 2] in device memory), cos/sin by sincosf, cos[i + h] = cos[i]. No counterpart in the reference's ABI
 * (it always reads a cache, rope/kernel.cu:102-107). */
int ckb_rope_sincos_launch(const void* q, const void* k, const float* inv_freq, const long long* ids, void* q_out,
                           void* k_out, long long tokens, int q_heads, int kv_heads, int head_dim, int qk_dtype,
                           cudaStream_t stream);

/* RoPE fused with the paged KV-cache write: q and k rotated as launch() does (q_out == q rotates q in place; k_out == k
 * rotates k in place, k_out null leaves k untouched), and for each token t with slots[t] >= 0 the rotated k and the
 * unrotated v [tokens, kv_heads, head_dim] (qk_dtype) are stored into key_cache / value_cache [num_blocks,
 * block_size, kv_heads, head_dim] at row slots[t] (int64; slot = block * block_size + offset; negative: a padding
 * token, no cache row written). One pass: k and v are read once. No counterpart in the reference, whose RoPE rotates
 * q and k only (rope/kernel.cu:1-13); the cache layout is the usual paged one (flattened [slot, head, dim]). */
int ckb_rope_kv_cache_launch(const void* q, const void* k, const void* v, const void* cos_rows, const void* sin_rows,
                             const void* ids, const void* slots, void* q_out, void* k_out, void* key_cache,
                             void* value_cache, long long tokens, int q_heads, int kv_heads, int head_dim,
                             int qk_dtype, int cache_dtype, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
#endif
