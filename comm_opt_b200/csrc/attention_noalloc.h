// Allocation-free C entry point of the paged GQA decode attention.
//
// This entry point has no counterpart in the reference (allennnnnz/comm_opt); it is an addition of
// this library.
//
// Who it is for: callers that cannot allocate device memory when they run attention - code that
// links this library from C or another language runtime without PyTorch's caching allocator, where
// a cudaMalloc would synchronize the whole device in the middle of a decode step, and serving
// engines that reserve all device memory up front for weights and KV cache and do not allow a
// library to take more. Those callers pass only their inputs and outputs; the split-KV partial
// results live in a fixed array compiled into the library instead of a buffer they must provide.
//
// Limits and behaviour:
//   * the scratch array holds COB_NOALLOC_SCRATCH_BYTES (8 MiB) per GPU and stays resident on
//     every GPU that loads the library until the process exits;
//   * a geometry whose split-KV scratch would exceed it is rejected (cudaErrorInvalidValue, message
//     from cob_noalloc_last_error()), and so is a split plan that does not cover the block table
//     (splits * pages_per_split < max_blocks_per_seq), which would silently drop tokens;
//   * the caches are declared to the copy engine as exactly num_blocks pages, so a block-table entry
//     past the end of the cache reads zeros instead of memory the caller does not own;
//   * the first call on each device looks up the array's device address with that device current;
//     make that first call before any stream capture;
//   * every call on a device shares the one array and finds the previous call's partial results
//     in it; the call clears the per-(sequence, head) counters it needs before launching, and calls
//     that overlap on the GPU (different streams without ordering) race on the array.
#pragma once

#include <stddef.h>
#include <stdint.h>

#define COB_NOALLOC_SCRATCH_BYTES (8u << 20)

#ifdef __cplusplus
extern "C" {
#endif

// Same math and layouts as the regular entry point (q [B, nq, D], caches [num_blocks, nkv, 16, D],
// block_tables [B, max_blocks_per_seq], seq_lens [B], out [B, nq, D]); head_dim 64 or 128, block_size
// 16, dtype: 1 = fp16, 2 = bf16. Split s of a sequence covers block-table columns
// [s * pages_per_split, (s + 1) * pages_per_split). `stream` is a cudaStream_t (0 = legacy default
// stream). Returns 0 or a cudaError_t code.
int cob_decode_attention_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                 const int32_t* block_tables, const int32_t* seq_lens, void* out, int batch,
                                 int nq, int nkv, int head_dim, int block_size, int max_blocks_per_seq,
                                 int num_blocks, int splits, int pages_per_split, float scale, int dtype,
                                 void* stream);

// Bytes of the built-in scratch array (the limit checked by the entry point).
size_t cob_noalloc_scratch_capacity(void);

// Text of the last error reported by the entry point on this host thread ("" if none).
const char* cob_noalloc_last_error(void);

#ifdef __cplusplus
}
#endif
