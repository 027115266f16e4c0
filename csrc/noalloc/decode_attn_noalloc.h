// Allocation-free split-KV decode attention: the one exported C entry point of
// lib/libfoundry_noalloc.so.
//
// This header has no counterpart in the reference (foundry-org/foundry ships
// no attention kernels). The entry point exists for callers that cannot
// allocate device memory:
//   * code running inside an active deterministic allocation region, where
//     any allocation advances the region cursor and shifts every later
//     address away from the layout that restored graphs were saved with;
//   * an out-of-memory handler that still needs one attention result;
//   * a plain C or C++ host that has no caching allocator to borrow scratch
//     memory from.
// Its per-split partials live in a fixed file-scope device array of
// 8,519,680 bytes (16,384 partial rows of 128 + 2 floats) that every GPU
// which loads the library holds until the process exits.
#pragma once

#ifdef __cplusplus
extern "C" {
#endif

// Maximum number of (sequence, query head, split) partial rows that fit the
// library's static scratch; requests with splits > 1 that need more are
// refused with return code 1.
#define FB_NOALLOC_MAX_PARTIAL_ROWS 16384

// out[b, h, :] = softmax(q[b, h] . K^T * scale) V over the first seq_lens[b]
// tokens of sequence b's pages.
//   q            [batch, n_q, 128] bf16
//   k_cache      [blocks, n_kv, 64, 128] bf16 (64-token pages)
//   v_cache      [blocks, n_kv, 64, 128] bf16
//   block_tables [batch, max_blocks] int32
//   seq_lens     [batch] int32
//   out          [batch, n_q, 128] bf16
// n_q / n_kv must be 4 or 8; splits * pages_per_split must cover max_blocks.
// stream is a cudaStream_t (0 = the legacy default stream).
//
// Returns 0 on success, 1 when the partials do not fit the static scratch,
// 2 for an invalid argument, 3 for a CUDA error; a message goes to err when
// err is not null.
//
// The first call in each CUDA context does a one-time set-up (it resolves the
// scratch array's device address and loads the kernels); make that first call
// before any stream capture. All calls in a process share the one scratch
// array: calls that overlap on the GPU race on it. Calls on one stream are
// ordered and safe.
int fb_decode_attention_noalloc(const void* q, const void* k_cache, const void* v_cache, const int* block_tables,
                                int max_blocks, const int* seq_lens, void* out, int batch, int n_q, int n_kv,
                                int splits, int pages_per_split, float scale, void* stream, char* err,
                                int err_len);

#ifdef __cplusplus
}
#endif
