/* Allocation-free C entry point of the paged decode attention.
 *
 * This entry point has no counterpart in the reference: it is an addition of this
 * library for callers that may not allocate device memory while they run.  Examples are
 * a serving runtime that owns all device memory through its own pool and forbids
 * allocation on its hot path, a plugin loaded into such a runtime, or C code with no
 * access to PyTorch's caching allocator.  The regular entry point (attn_decode, used by
 * the Python model) allocates its fp32 partial results per call; this one keeps them in
 * one fixed-size array compiled into the library instead.
 *
 * Scratch: a file-scope device array of QFC_NOALLOC_SCRATCH_BYTES (16 MiB).  Every GPU
 * that loads the library holds one such array until the process exits.  A call needs
 *     batch * num_q_heads * ceil(max_pages_per_seq * page_size / 256) * (head_dim + 2) * 4
 * bytes of it and returns QFC_NOALLOC_ERR_TOO_LARGE (doing nothing) above that.
 *
 * The first call on each device looks up the array's device address (with that device
 * current) and opts the kernels into their shared memory on that device.  Make that first
 * call before any CUDA stream capture begins.  One process may call it on several GPUs:
 * each device has its own copy of the array, address and opt-in.
 *
 * All calls share the one array and it keeps the last call's contents; every value a
 * call reads from it was written earlier in the same call, so nothing needs clearing.
 * Calls whose kernels overlap on the GPU (two streams, or two host threads) race on the
 * array and produce wrong results: serialise them.
 */
#pragma once

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QFC_NOALLOC_SCRATCH_BYTES (16u << 20)

enum {
  QFC_NOALLOC_OK = 0,
  QFC_NOALLOC_ERR_TOO_LARGE = 1, /* the call needs more scratch than QFC_NOALLOC_SCRATCH_BYTES */
  QFC_NOALLOC_ERR_BAD_ARGS = 2,  /* unsupported head_dim / GQA group / dtype, or a null pointer */
  QFC_NOALLOC_ERR_CUDA = 3       /* a CUDA runtime call failed (see cudaGetLastError) */
};

/* One query token per sequence attends over its paged KV cache.
 *   q            [batch, num_q_heads * head_dim]            (bf16 or fp16, dtype 0 / 1)
 *   k_cache/v_cache [pages, num_kv_heads, page_size, head_dim]
 *   block_table  [batch, max_pages_per_seq] int32 page indices
 *   seq_lens     [batch] int32, tokens in the cache per sequence
 *   out          [batch, num_q_heads * head_dim]
 * head_dim is 64 or 128; num_q_heads / num_kv_heads is 1, 2, 4 or 8.  The kernels run on
 * `stream` of the current device; the call returns without synchronising. */
__attribute__((visibility("default"))) int qfc_attn_decode_noalloc(
    const void* q, const void* k_cache, const void* v_cache, const int* block_table, const int* seq_lens, void* out,
    int batch, int num_q_heads, int num_kv_heads, int head_dim, int page_size, int max_pages_per_seq, float scale,
    int dtype, cudaStream_t stream);

/* Scratch bytes a call with these sizes needs. */
__attribute__((visibility("default"))) unsigned long long qfc_attn_decode_noalloc_scratch_bytes(
    int batch, int num_q_heads, int head_dim, int page_size, int max_pages_per_seq);

/* A short description of a return code. */
__attribute__((visibility("default"))) const char* qfc_noalloc_error_string(int code);

#ifdef __cplusplus
}
#endif
