// phx_noalloc.h — allocation-free C entry point of the cascade (shared-prefix) paged attention.
//
// This entry point has no counterpart in the reference: the reference's cascade attention runs inside
// SGLang on tensors that the engine allocates. It exists for callers that cannot call cudaMalloc (or any
// allocating routine) at the point where they run attention: code running inside a host allocator hook
// or a memory-pool callback, runtimes that forbid device allocation after start-up (fixed memory
// budgets on shared GPUs), and plain C hosts without a caching allocator, which would otherwise pay a
// cudaMalloc/cudaFree pair per call. The caller passes inputs and outputs; the two-pass cascade keeps its
// (O, LSE) partials in a file-scope device array instead of a temporary buffer.
//
// Limits and behaviour:
//   * The partial buffer holds at most PHX_NOALLOC_MAX_ROWS (token, query-head) rows: T * Hq must not
//     exceed it (32768 rows = 8 MiB of bf16 partials + 128 KiB of fp32 LSE). Every GPU that loads the
//     library holds this array until the process exits. Larger calls return PHX_NOALLOC_ERR_TOO_LARGE.
//   * head_dim must be 128 and the KV page size 64 (the kernel's tile shape); the work lists must be
//     built with 64 query rows per tile (tile_row0 multiples of 64).
//   * Runs on the current device and on `stream`, which must belong to it. The first call on a device
//     sets it up: it looks up the device address of the array (cudaGetSymbolAddress) and opts the
//     attention kernel into its dynamic shared memory (cudaFuncSetAttribute); make that first call before
//     any stream capture. Later calls read the cached address and launch kernels (up to three).
//   * A pass with tiles needs its whole work list: num_tiles1 > 0 (or num_tiles2 > 0) with a NULL
//     items/tile_item/tile_row0 pointer of that pass returns PHX_NOALLOC_ERR_BAD_ARGS without launching.
//   * All calls share the array and each call overwrites it (the LSE rows are reset at the start of
//     every call). Calls that overlap on the GPU — on different streams, or from several host threads
//     without ordering — race on it; order them on one stream.
//   * Calls no cudaMalloc, cudaFree or allocating library routine.
#pragma once
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PHX_NOALLOC_MAX_ROWS 32768

#define PHX_NOALLOC_OK 0
#define PHX_NOALLOC_ERR_TOO_LARGE 1
#define PHX_NOALLOC_ERR_BAD_ARGS 2
#define PHX_NOALLOC_ERR_CUDA 3

// q        bf16 [T, Hq, 128] (roped queries)
// k_cache, v_cache  bf16 [pages, Hkv, 64, 128]
// pages, page_indptr, prefix_len, q_start: the paged-attention metadata (int32)
// tree     int64 [T] ancestor bitmasks (causal == 0), or NULL (causal == 1)
// items1/tile_item1/tile_row0_1/num_tiles1: prefix-pass work list (num_tiles1 == 0: no shared prefix)
// items2/tile_item2/tile_row0_2/num_tiles2: per-request pass work list
// out_bf16 bf16 [T, Hq*128] or NULL; out_q fp8 e4m3 [T, Hq*128] and out_qs fp32 [Hq, T], or NULL
// Returns PHX_NOALLOC_OK or an error code (see phx_noalloc_strerror).
int phx_cascade_attention_noalloc(const void* q, const void* k_cache, const void* v_cache, const int32_t* pages,
                                  const int32_t* page_indptr, const int32_t* prefix_len, const int32_t* q_start,
                                  const int64_t* tree, const int32_t* items1, const int32_t* tile_item1,
                                  const int32_t* tile_row0_1, int32_t num_tiles1, const int32_t* items2,
                                  const int32_t* tile_item2, const int32_t* tile_row0_2, int32_t num_tiles2,
                                  int32_t T, int32_t Hq, int32_t Hkv, int32_t causal, float softmax_scale,
                                  void* out_bf16, void* out_q, float* out_qs, void* stream);

const char* phx_noalloc_strerror(int code);

#ifdef __cplusplus
}
#endif
