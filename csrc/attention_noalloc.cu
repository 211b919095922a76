// Allocation-free cascade attention entry point; see phx_noalloc.h for the contract.
#include <cuda_runtime.h>
#include <math.h>

#include <atomic>
#include <mutex>

#include "attention_params.h"
#include "phx_noalloc.h"

namespace {

constexpr long kRows = PHX_NOALLOC_MAX_ROWS;
constexpr long kPartBytes = kRows * 128 * 2;  // bf16 O partials
constexpr long kLseBytes = kRows * 4;         // fp32 LSE partials

// The scratch: every device that loads the library holds it until exit.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kPartBytes + kLseBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
// Per device: the scratch's device address, published once its set-up (symbol lookup + the kernel's
// shared-memory opt-in) has succeeded. Later calls read it without taking the lock.
std::atomic<void*> g_base[kMaxDevices];

// Device address of the scratch on the current device (host code may not use the symbol directly:
// on the host it names a stand-in, not device memory). The first call on a device also opts the
// attention kernel into its dynamic shared memory; both are done once per device.
int scratch_base(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return PHX_NOALLOC_ERR_CUDA;
  void* p = g_base[dev].load(std::memory_order_acquire);
  if (!p) {
    std::lock_guard<std::mutex> lk(g_mu);
    p = g_base[dev].load(std::memory_order_relaxed);
    if (!p) {
      if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return PHX_NOALLOC_ERR_CUDA;
      if (phx::paged_attention_raw_setup() != cudaSuccess) return PHX_NOALLOC_ERR_CUDA;
      g_base[dev].store(p, std::memory_order_release);
    }
  }
  *out = p;
  return PHX_NOALLOC_OK;
}

__global__ void fill_neg_inf(float* p, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) p[i] = -INFINITY;
}

}  // namespace

extern "C" const char* phx_noalloc_strerror(int code) {
  switch (code) {
    case PHX_NOALLOC_OK: return "ok";
    case PHX_NOALLOC_ERR_TOO_LARGE: return "T * Hq exceeds PHX_NOALLOC_MAX_ROWS (32768) partial rows";
    case PHX_NOALLOC_ERR_BAD_ARGS:
      return "bad arguments (null input or work list, Hq % Hkv != 0, or no output)";
    case PHX_NOALLOC_ERR_CUDA: return "CUDA error while resolving the scratch or launching";
    default: return "unknown error";
  }
}

extern "C" int phx_cascade_attention_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                             const int32_t* pages, const int32_t* page_indptr,
                                             const int32_t* prefix_len, const int32_t* q_start, const int64_t* tree,
                                             const int32_t* items1, const int32_t* tile_item1,
                                             const int32_t* tile_row0_1, int32_t num_tiles1, const int32_t* items2,
                                             const int32_t* tile_item2, const int32_t* tile_row0_2,
                                             int32_t num_tiles2, int32_t T, int32_t Hq, int32_t Hkv, int32_t causal,
                                             float softmax_scale, void* out_bf16, void* out_q, float* out_qs,
                                             void* stream) {
  if (!q || !k_cache || !v_cache || !pages || !page_indptr || !prefix_len || !q_start || Hkv <= 0 || Hq <= 0 ||
      Hq % Hkv != 0 || T < 0 || (!out_bf16 && !out_q) || (out_q && !out_qs) || (!causal && !tree))
    return PHX_NOALLOC_ERR_BAD_ARGS;
  // a pass with tiles needs its whole work list: a missing prefix list would silently drop the shared keys,
  // a missing suffix list would be dereferenced on the device
  if (num_tiles1 > 0 && (!items1 || !tile_item1 || !tile_row0_1)) return PHX_NOALLOC_ERR_BAD_ARGS;
  if (num_tiles2 > 0 && (!items2 || !tile_item2 || !tile_row0_2)) return PHX_NOALLOC_ERR_BAD_ARGS;
  if ((long)T * Hq > kRows) return PHX_NOALLOC_ERR_TOO_LARGE;
  if (T == 0 || num_tiles2 <= 0) return PHX_NOALLOC_OK;
  void* base = nullptr;
  int rc = scratch_base(&base);
  if (rc != PHX_NOALLOC_OK) return rc;
  auto* o_part = reinterpret_cast<__nv_bfloat16*>(base);
  auto* lse_part = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(base) + kPartBytes);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);

  phx::AttnParams p{};
  p.q = reinterpret_cast<const __nv_bfloat16*>(q);
  p.kc = reinterpret_cast<const __nv_bfloat16*>(k_cache);
  p.vc = reinterpret_cast<const __nv_bfloat16*>(v_cache);
  p.pages = pages;
  p.page_indptr = page_indptr;
  p.prefix_len = prefix_len;
  p.q_start = q_start;
  p.tree = reinterpret_cast<const uint64_t*>(tree);
  p.T = T;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.causal = causal ? 1 : 0;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;

  const bool cascade = num_tiles1 > 0;
  if (cascade) {
    // rows the prefix pass does not cover must read as "no prefix" (LSE = -inf) in the second pass
    const int n = T * Hq;
    fill_neg_inf<<<(n + 255) / 256 < 1024 ? (n + 255) / 256 : 1024, 256, 0, st>>>(lse_part, n);
    if (cudaGetLastError() != cudaSuccess) return PHX_NOALLOC_ERR_CUDA;
    phx::AttnParams p1 = p;
    p1.items = items1;
    p1.tile_item = tile_item1;
    p1.tile_row0 = tile_row0_1;
    p1.num_tiles = num_tiles1;
    p1.o_part = o_part;
    p1.lse_part = lse_part;
    if (phx::launch_paged_attention_raw(p1, num_tiles1, st) != cudaSuccess) return PHX_NOALLOC_ERR_CUDA;
  }
  phx::AttnParams p2 = p;
  p2.items = items2;
  p2.tile_item = tile_item2;
  p2.tile_row0 = tile_row0_2;
  p2.num_tiles = num_tiles2;
  p2.o_in = cascade ? o_part : nullptr;
  p2.lse_in = cascade ? lse_part : nullptr;
  p2.out = reinterpret_cast<__nv_bfloat16*>(out_bf16);
  p2.out_q = reinterpret_cast<uint8_t*>(out_q);
  p2.out_qs = out_qs;
  return phx::launch_paged_attention_raw(p2, num_tiles2, st) == cudaSuccess ? PHX_NOALLOC_OK : PHX_NOALLOC_ERR_CUDA;
}
