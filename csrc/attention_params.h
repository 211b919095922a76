// Parameter block of the paged attention kernel (csrc/attention.cu), shared with entry points that
// launch it on raw pointers.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace phx {

struct AttnParams {
  const __nv_bfloat16* q;   // [T, Hq, D]
  const __nv_bfloat16* kc;  // [P, Hkv, 64, D]
  const __nv_bfloat16* vc;
  const int* pages;
  const int* page_indptr;
  const int* prefix_len;    // [R]
  const int* q_start;       // [R]
  const uint64_t* tree;     // [T] or null
  const int* items;         // [W, 6]
  const int* tile_item;     // [tiles]
  const int* tile_row0;     // [tiles]
  const __nv_bfloat16* o_in;  // seed partial [T, Hq, D] or null
  const float* lse_in;        // [T, Hq]
  __nv_bfloat16* o_part;      // partial out [T, Hq, D] or null
  float* lse_part;
  __nv_bfloat16* out;         // final bf16 [T, Hq*D] or null
  uint8_t* out_q;             // final fp8 [T, Hq*D] or null
  float* out_qs;              // [Hq, T]
  int T, Hq, Hkv, causal, num_tiles;
  float scale_log2;
};

// One-time set-up of the raw launcher on the current device: opts the kernel into its dynamic shared
// memory. Call once per device (with that device current) before launch_paged_attention_raw.
cudaError_t paged_attention_raw_setup();

// Launch the paged attention kernel for `num_tiles` row tiles x p.Hkv KV heads on `stream`; returns the
// launch's error code. Sets no attribute and allocates nothing.
cudaError_t launch_paged_attention_raw(const AttnParams& p, int num_tiles, cudaStream_t stream);

}  // namespace phx
