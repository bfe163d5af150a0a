/*
 * mesh_noalloc.h - allocation-free C entry point for paged decode attention.
 *
 * Declaration: this entry point has no counterpart in the reference project (saint0x/mesh);
 * it is an addition of this library.
 *
 * Who needs it: callers that cannot allocate device memory while they run. Examples are a
 * runtime that has already reserved all GPU memory for its own pool, code that runs inside a
 * custom memory manager or a real-time loop where cudaMalloc/cudaFree (which may synchronise
 * the device) are not allowed, and plain C hosts without PyTorch's caching allocator. They pass
 * the inputs and the output buffer; the scratch space that split-KV attention needs (one
 * partial output and one log-sum-exp per query head and split) comes from a fixed array that is
 * part of this library's device image.
 *
 * Limit: B * num_q_heads * splits * (head_dim + 1) <= MESH_NOALLOC_SCRATCH_FLOATS (4 MiB of
 * fp32). Larger requests return MESH_NOALLOC_ERR_TOO_LARGE and launch nothing. Every GPU that
 * loads this library keeps the 4 MiB array until the process exits.
 */
#ifndef MESH_NOALLOC_H
#define MESH_NOALLOC_H

#ifdef __cplusplus
extern "C" {
#endif

#define MESH_NOALLOC_SCRATCH_FLOATS (1u << 20)

#define MESH_NOALLOC_OK 0
#define MESH_NOALLOC_ERR_ARGUMENT (-1)
#define MESH_NOALLOC_ERR_TOO_LARGE (-2)
#define MESH_NOALLOC_ERR_SETUP (-3)
#define MESH_NOALLOC_ERR_LAUNCH (-4)

/*
 * Split-KV paged GQA decode attention, one query token per sequence.
 *   q            [B, num_q_heads * head_dim] bf16
 *   k_cache      [num_pages, num_kv_heads, page_size, head_dim] bf16 (v_cache the same)
 *   block_tables [B, max_pages_per_seq] int32, seq_lens [B] int32 (keys per sequence)
 *   out          [B, num_q_heads * head_dim] bf16
 * head_dim 64 or 128; num_q_heads / num_kv_heads in {1, 2, 4, 8}; splits >= 1; window 0 for
 * full context, else the number of most recent keys attended. The work is enqueued on `stream`
 * (a cudaStream_t; NULL = legacy default stream) on the current device; the call returns
 * without waiting for it.
 *
 * The first call on a device looks up the device address of the scratch array there
 * (cudaGetSymbolAddress) and caches it; make that first call before any CUDA stream capture on
 * that device. All calls on a device share the one scratch array, which keeps the last call's
 * contents; nothing in it has to start at zero (every split writes all of its slot). Calls
 * whose executions overlap on the GPU (different streams without ordering) race on it.
 */
int mesh_attn_decode_noalloc(const void* q, const void* k_cache, const void* v_cache, const int* block_tables,
                             const int* seq_lens, void* out, int B, int num_q_heads, int num_kv_heads, int head_dim,
                             int page_size, int max_pages_per_seq, int splits, float scale, int window,
                             void* stream);

#ifdef __cplusplus
}
#endif
#endif
