// Device-side speculative sampling over (vocab-sharded) bf16 verify logits, sm_100a. No host
// synchronisation anywhere: the whole path can be captured in a CUDA graph.
//
// 1. sample_candidates: for every logits row and every vocab chunk of up to 16384 columns (one CTA each),
//    the chunk's KC best values of x / T (T applied by IEEE division; greedy rows use T = 1) with their
//    global vocab indices. "Best" orders by value, ties toward the lower index, the order of a stable
//    descending sort. The chunk is staged in shared memory as 16-bit order-preserving keys of the bf16
//    logits (division by a positive T keeps the order of distinct bf16 values: fp32 has 16 more mantissa
//    bits); an exact two-level radix select (high byte, then low byte, warp-aggregated shared-memory
//    histograms) finds the KC-th key, and a pass in index order collects the keys above it plus the
//    lowest-index keys equal to it. Optionally also the chunk's (max, sum exp(x/T - max)).
//    Under tensor parallelism each rank runs this on its vocab shard; the [rows, chunks, KC] candidates
//    of all ranks are then exchanged (a few MB), so every rank holds every shard's candidates.
// 2. spec_accept: one CTA per request walks its verified tree. At the current node it merges the node's
//    candidates from every shard/chunk (bitonic sort in shared memory), keeps the request's top_k, takes
//    the softmax over them, applies the top-p cut (smallest prefix reaching top_p, first token always
//    kept) and renormalises; then, with the seeded coin of this depth, accepts the first child (node
//    order) whose cumulative target probability exceeds the coin; if none, it draws the bonus token by
//    inverse CDF in vocab-index order (double accumulation) from the target distribution with the
//    children's tokens removed (all of it if that leaves no mass), with the step's final coin.
//    Coins are MurmurHash3_x86_32 of (committed length lo, hi, column) seeded by the request seed,
//    mapped to [0, 1) as h / (2^32 - 1) in double rounded to fp32 and clamped below 1.
// The same definition in plain torch (dense target distribution) is engine/sampling.py; this path serves
// requests with temperature 0 or 1 <= top_k <= KC (the reference's sparse top-k target-probability path,
// docker/opt/v5/topkbf_normcfg/topkbf/kopt_topkbf.py:353-399, and its seeded verify coins,
// docker/opt/v3/seed/dflash_seed.patch:127-160).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <algorithm>
#include <type_traits>

#include "common.cuh"

namespace phx {

constexpr int kCandThreads = 512;
constexpr int kCandChunk = 16384;   // columns per CTA (32 KB of 16-bit keys in shared memory)

__device__ __forceinline__ uint32_t bf16_key(uint16_t b) { return (b & 0x8000u) ? (~b & 0xffffu) : (b | 0x8000u); }
__device__ __forceinline__ float key_value(uint32_t k) {
  const uint16_t b = (k & 0x8000u) ? (uint16_t)(k & 0x7fffu) : (uint16_t)(~k & 0xffffu);
  return __uint_as_float((uint32_t)b << 16);
}

// Warp 0 finds the bin where the count of keys in bins above it, plus the bin's own count, first reaches
// `need` (bins scanned from 255 down). Writes the bin and the count strictly above it.
__device__ __forceinline__ void find_crossing(const uint32_t* hist, uint32_t need, int* bin_out, uint32_t* above_out) {
  const int lane = threadIdx.x & 31;
  // lane l owns bins 255-8l .. 248-8l (descending)
  uint32_t c[8], tot = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    c[j] = hist[255 - 8 * lane - j];
    tot += c[j];
  }
  uint32_t incl = tot;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  const uint32_t excl = incl - tot;
  const unsigned hit = __ballot_sync(0xffffffffu, incl >= need && excl < need);
  const int src = hit ? __ffs(hit) - 1 : 31;
  if (lane == src) {
    uint32_t run = excl;
    int b = 255 - 8 * lane - 7;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (run + c[j] >= need) {
        b = 255 - 8 * lane - j;
        break;
      }
      run += c[j];
    }
    *bin_out = b;
    *above_out = run;
  }
}

// Exact fallback for the chunks where the fast kernel's candidate set overflowed (heavy ties at the
// threshold): the chunk is staged in shared memory and radix-selected. Only CTAs whose overflow flag is set
// do any work.
template <int KC, bool LSE>
__global__ void __launch_bounds__(kCandThreads) sample_candidates_exact_kernel(
    const __nv_bfloat16* __restrict__ logits, int V, int ld, int nchunks, int vocab_offset,
    const float* __restrict__ temp, int rows_per_temp, float* __restrict__ cv, int* __restrict__ ci,
    float* __restrict__ cms, const int* __restrict__ overflow, int items) {
  __shared__ __align__(16) uint16_t keys[kCandChunk];
  __shared__ uint32_t hist[256];
  __shared__ uint32_t wcnt[kCandThreads / 32];
  __shared__ int s_bin;
  __shared__ uint32_t s_above, s_gt;
  __shared__ float red[kCandThreads / 32];

  for (int item = blockIdx.x; item < items; item += gridDim.x) {
  if (!overflow[item]) continue;
  __syncthreads();   // the previous item's shared-memory readers are done
  const int row = item / nchunks, chunk = item % nchunks;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c0 = chunk * kCandChunk;
  const int n = min(kCandChunk, V - c0);
  const uint16_t* src = reinterpret_cast<const uint16_t*>(logits + (size_t)row * ld + c0);
  float T = temp ? temp[row / rows_per_temp] : 1.0f;
  if (!(T > 0.f)) T = 1.0f;   // greedy rows: argmax of the raw logits

  // ---- stage the chunk as order-preserving keys ----
  const bool vec = ((reinterpret_cast<uintptr_t>(src) & 15u) == 0);
  if (vec) {
    const int n8 = n / 8;
    for (int i = tid; i < n8; i += kCandThreads) {
      const uint4 v = reinterpret_cast<const uint4*>(src)[i];
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) o[e] = bf16_key(w[e] & 0xffffu) | (bf16_key(w[e] >> 16) << 16);
      reinterpret_cast<uint4*>(keys)[i] = make_uint4(o[0], o[1], o[2], o[3]);
    }
    for (int i = n8 * 8 + tid; i < n; i += kCandThreads) keys[i] = (uint16_t)bf16_key(src[i]);
  } else {
    for (int i = tid; i < n; i += kCandThreads) keys[i] = (uint16_t)bf16_key(src[i]);
  }
  for (int i = tid; i < 256; i += kCandThreads) hist[i] = 0;
  if (tid == 0) s_gt = 0;
  __syncthreads();

  const uint32_t need = (uint32_t)min(KC, n);
  const int rounds = (n + kCandThreads - 1) / kCandThreads;
  // ---- level 1: histogram of the high byte (one shared atomic per distinct bin per warp) ----
  for (int r = 0; r < rounds; ++r) {
    const int e = r * kCandThreads + tid;
    const bool valid = e < n;
    const uint32_t b = valid ? (uint32_t)(keys[e] >> 8) : 0x100u + lane;
    const unsigned peers = __match_any_sync(0xffffffffu, b);
    if (valid && lane == __ffs(peers) - 1) atomicAdd(&hist[b], (uint32_t)__popc(peers));
  }
  __syncthreads();
  if (warp == 0) find_crossing(hist, need, &s_bin, &s_above);
  __syncthreads();
  const uint32_t hi = (uint32_t)s_bin, above_hi = s_above;
  __syncthreads();
  for (int i = tid; i < 256; i += kCandThreads) hist[i] = 0;
  __syncthreads();
  // ---- level 2: histogram of the low byte among keys in the crossing high bin ----
  for (int r = 0; r < rounds; ++r) {
    const int e = r * kCandThreads + tid;
    const uint32_t k = e < n ? keys[e] : 0u;
    const bool valid = e < n && (k >> 8) == hi;
    const uint32_t b = valid ? (k & 0xffu) : 0x100u + lane;
    const unsigned peers = __match_any_sync(0xffffffffu, b);
    if (valid && lane == __ffs(peers) - 1) atomicAdd(&hist[b], (uint32_t)__popc(peers));
  }
  __syncthreads();
  if (warp == 0) find_crossing(hist, need - above_hi, &s_bin, &s_above);
  __syncthreads();
  const uint32_t thr = (hi << 8) | (uint32_t)s_bin;
  const uint32_t n_gt = above_hi + s_above;          // keys strictly above the threshold (< need)
  const uint32_t need_eq = need - n_gt;              // lowest-index keys equal to it
  const size_t obase = ((size_t)row * nchunks + chunk) * KC;

  // ---- collect, in index order ----
  uint32_t eq_base = 0;   // keys equal to the threshold seen in earlier rounds (same value in every thread)
  for (int r = 0; r < rounds; ++r) {
    const int e = r * kCandThreads + tid;
    const uint32_t k = e < n ? keys[e] : 0u;
    const bool gt = e < n && k > thr, eq = e < n && k == thr;
    int slot = -1;
    if (gt) slot = (int)atomicAdd(&s_gt, 1u);
    const unsigned bal = __ballot_sync(0xffffffffu, eq);
    if (lane == 0) wcnt[warp] = __popc(bal);
    __syncthreads();
    uint32_t before = 0, tot = 0;
#pragma unroll
    for (int w = 0; w < kCandThreads / 32; ++w) {
      const uint32_t c = wcnt[w];
      before += w < warp ? c : 0u;
      tot += c;
    }
    if (eq) {
      const uint32_t off = eq_base + before + __popc(bal & ((1u << lane) - 1u));
      if (off < need_eq) slot = (int)(n_gt + off);
    }
    if (slot >= 0) {
      const float x = key_value(k);
      cv[obase + slot] = T == 1.0f ? x : __fdiv_rn(x, T);
      ci[obase + slot] = vocab_offset + c0 + e;
    }
    eq_base += tot;
    __syncthreads();   // every thread has read wcnt before the next round overwrites it
  }
  // chunks narrower than KC: pad
  for (int j = (int)need + tid; j < KC; j += kCandThreads) {
    cv[obase + j] = -INFINITY;
    ci[obase + j] = 0x7fffffff;
  }
  if constexpr (LSE) {
    __syncthreads();
    // max of the chunk is the largest key; then sum exp(x/T - max)
    float m = -INFINITY;
    for (int i = tid; i < n; i += kCandThreads) m = fmaxf(m, key_value(keys[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = -INFINITY;
    for (int w = 0; w < kCandThreads / 32; ++w) m = fmaxf(m, red[w]);
    __syncthreads();
    const float mt = T == 1.0f ? m : __fdiv_rn(m, T);
    float s = 0.f;
    if (mt != -INFINITY)
      for (int i = tid; i < n; i += kCandThreads) {
        const float x = key_value(keys[i]);
        s += expf((T == 1.0f ? x : __fdiv_rn(x, T)) - mt);
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (tid == 0) {
      float tot = 0.f;
      for (int w = 0; w < kCandThreads / 32; ++w) tot += red[w];
      cms[((size_t)row * nchunks + chunk) * 2] = mt;
      cms[((size_t)row * nchunks + chunk) * 2 + 1] = tot;
    }
  }
}  // items
}

// Fast path. Each thread holds 32 keys of the chunk in registers (four 16-byte loads). The KC-th largest of
// the 512 per-thread maxima, tau, is a lower bound of the chunk's KC-th largest key (those KC maxima are KC
// distinct elements), so every top-KC element has key >= tau, and for realistic logits only a few hundred
// elements do. They are compacted into shared memory as 64-bit (key, ~index) words -- descending order of
// the word is value descending, index ascending -- and sorted there (bitonic). More than kCandCap of them
// (heavy ties at tau) sets the chunk's overflow flag and leaves it to the exact kernel.
constexpr int kCandCap = 2048;

// in-place bitonic sort, descending, of n (a power of two) 64-bit words in shared memory; all threads call it
__device__ __forceinline__ void bitonic_desc_u64(uint64_t* v, int n) {
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int j = threadIdx.x; j < n; j += blockDim.x) {
        const int o = j ^ stride;
        if (o > j) {
          const uint64_t x = v[j], y = v[o];
          const bool desc = (j & size) == 0;
          if (desc ? (y > x) : (x > y)) {
            v[j] = y;
            v[o] = x;
          }
        }
      }
      __syncthreads();
    }
  }
}

// Shared memory of the fast path: two 32 KB chunk buffers (the next chunk is fetched by a bulk copy while
// the current one is processed), the candidate words and small scratch.
struct CandSmem {
  uint16_t buf[2][kCandChunk];
  uint64_t cand[kCandCap];
  uint32_t hist[256];
  float red[kCandThreads / 32];
  uint64_t full[2];
  int bin;
  uint32_t above, cnt;
};

// One chunk (n columns at src: global or shared memory, 16-byte aligned when vec) -> its KC candidates.
template <int KC, bool LSE>
__device__ __forceinline__ void cand_chunk(CandSmem& sm, const uint16_t* src, int n, bool vec, float T, int gcol0,
                                           float* cvp, int* cip, float* cmsp, int* ovf) {
  constexpr int PER = kCandChunk / kCandThreads;   // 32 keys per thread
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t kp[PER / 2];
#pragma unroll
  for (int j = 0; j < PER / 8; ++j) {
    const int v = tid + j * kCandThreads;
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    if (vec) {
      if (v * 8 < n) {
        const uint4 q = reinterpret_cast<const uint4*>(src)[v];
        w[0] = q.x, w[1] = q.y, w[2] = q.z, w[3] = q.w;
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (v * 8 + e < n) w[e / 2] |= (uint32_t)src[v * 8 + e] << (16 * (e & 1));
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int el = v * 8 + 2 * e;
      const uint32_t lo = el < n ? bf16_key(w[e] & 0xffffu) : 0u;   // key 0 marks padding
      const uint32_t hi = el + 1 < n ? bf16_key(w[e] >> 16) : 0u;
      kp[j * 4 + e] = lo | (hi << 16);
    }
  }
  uint32_t tmax = 0;
#pragma unroll
  for (int j = 0; j < PER / 2; ++j) tmax = max(tmax, max(kp[j] & 0xffffu, kp[j] >> 16));

  // ---- tau = KC-th largest per-thread maximum (radix select over 512 values) ----
  for (int i = tid; i < 256; i += kCandThreads) sm.hist[i] = 0;
  if (tid == 0) sm.cnt = 0;
  __syncthreads();
  const uint32_t need = (uint32_t)min(KC, kCandThreads);
  {
    const uint32_t b = tmax >> 8;
    const unsigned peers = __match_any_sync(0xffffffffu, b);
    if (lane == __ffs(peers) - 1) atomicAdd(&sm.hist[b], (uint32_t)__popc(peers));
  }
  __syncthreads();
  if (warp == 0) find_crossing(sm.hist, need, &sm.bin, &sm.above);
  __syncthreads();
  const uint32_t hi_bin = (uint32_t)sm.bin, above_hi = sm.above;
  __syncthreads();
  for (int i = tid; i < 256; i += kCandThreads) sm.hist[i] = 0;
  __syncthreads();
  {
    const bool in = (tmax >> 8) == hi_bin;
    const uint32_t b = in ? (tmax & 0xffu) : 0x100u + lane;
    const unsigned peers = __match_any_sync(0xffffffffu, b);
    if (in && lane == __ffs(peers) - 1) atomicAdd(&sm.hist[b], (uint32_t)__popc(peers));
  }
  __syncthreads();
  if (warp == 0) find_crossing(sm.hist, need - above_hi, &sm.bin, &sm.above);
  __syncthreads();
  const uint32_t tau = max((hi_bin << 8) | (uint32_t)sm.bin, 1u);

  // ---- compact the keys >= tau (warp-aggregated slots) ----
#pragma unroll
  for (int j = 0; j < PER / 2; ++j) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t k = h ? (kp[j] >> 16) : (kp[j] & 0xffffu);
      const bool take = k >= tau;
      const unsigned m = __ballot_sync(0xffffffffu, take);
      if (m) {
        uint32_t base = 0;
        if (lane == __ffs(m) - 1) base = atomicAdd(&sm.cnt, (uint32_t)__popc(m));
        base = __shfl_sync(0xffffffffu, base, __ffs(m) - 1);
        if (take) {
          const uint32_t slot = base + __popc(m & ((1u << lane) - 1u));
          const int e = (tid + (j / 4) * kCandThreads) * 8 + (j % 4) * 2 + h;
          if (slot < (uint32_t)kCandCap) sm.cand[slot] = ((uint64_t)k << 32) | (uint64_t)(0xffffffffu - (uint32_t)e);
        }
      }
    }
  }
  __syncthreads();
  const uint32_t cnt = sm.cnt;
  if (tid == 0) *ovf = cnt > (uint32_t)kCandCap ? 1 : 0;
  if (cnt > (uint32_t)kCandCap) return;     // the exact kernel takes this chunk (uniform branch)
  auto emit = [&](int j, uint64_t w) {
    const float x = key_value((uint32_t)(w >> 32));
    cvp[j] = T == 1.0f ? x : __fdiv_rn(x, T);
    cip[j] = gcol0 + (int)(0xffffffffu - (uint32_t)(w & 0xffffffffu));
  };
  uint32_t top = 0;   // largest key (for the LSE)
  if (cnt <= 512) {
    // rank selection: each candidate counts the candidates above it (distinct words, no ties)
    for (int j = tid; j < (int)cnt; j += kCandThreads) {
      const uint64_t w = sm.cand[j];
      int rank = 0;
      for (int q = 0; q < (int)cnt; ++q) rank += sm.cand[q] > w;
      if (rank < KC) emit(rank, w);
    }
    if constexpr (LSE) {
      uint32_t mk = 0;
      for (int j = tid; j < (int)cnt; j += kCandThreads) mk = max(mk, (uint32_t)(sm.cand[j] >> 32));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mk = max(mk, __shfl_xor_sync(0xffffffffu, mk, o));
      if (lane == 0) sm.red[warp] = __uint_as_float(mk);
      __syncthreads();
      for (int w = 0; w < kCandThreads / 32; ++w) top = max(top, __float_as_uint(sm.red[w]));
      __syncthreads();
    }
  } else {
    int P = 1024;
    while (P < (int)cnt) P <<= 1;
    for (int j = (int)cnt + tid; j < P; j += kCandThreads) sm.cand[j] = 0ull;
    __syncthreads();
    bitonic_desc_u64(sm.cand, P);
    for (int j = tid; j < KC; j += kCandThreads) emit(j, sm.cand[j]);
    top = (uint32_t)(sm.cand[0] >> 32);
  }
  for (int j = (int)cnt + tid; j < KC; j += kCandThreads) {   // fewer than KC columns: pad
    cvp[j] = -INFINITY;
    cip[j] = 0x7fffffff;
  }
  if constexpr (LSE) {
    const float m0 = key_value(top);
    const float mt = T == 1.0f ? m0 : __fdiv_rn(m0, T);
    float ssum = 0.f;
    if (mt != -INFINITY) {
#pragma unroll
      for (int j = 0; j < PER / 2; ++j) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t k = h ? (kp[j] >> 16) : (kp[j] & 0xffffu);
          if (k) {
            const float x = key_value(k);
            ssum += expf((T == 1.0f ? x : __fdiv_rn(x, T)) - mt);
          }
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ssum += __shfl_xor_sync(0xffffffffu, ssum, o);
    if (lane == 0) sm.red[warp] = ssum;
    __syncthreads();
    if (tid == 0) {
      float tot = 0.f;
      for (int w = 0; w < kCandThreads / 32; ++w) tot += sm.red[w];
      cmsp[0] = mt;
      cmsp[1] = tot;
    }
  }
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// Persistent over (row, chunk) items. tma: rows are 16-byte aligned and chunk widths multiples of 8, so each
// chunk is fetched into shared memory by one bulk copy issued an item ahead; else keys are read directly.
template <int KC, bool LSE>
__global__ void __launch_bounds__(kCandThreads, 2) sample_candidates_kernel(
    const __nv_bfloat16* __restrict__ logits, int V, int ld, int nchunks, int items, int vocab_offset,
    const float* __restrict__ temp, int rows_per_temp, float* __restrict__ cv, int* __restrict__ ci,
    float* __restrict__ cms, int* __restrict__ overflow, int tma, int* status) {
  extern __shared__ __align__(16) uint8_t cand_smem_raw[];
  CandSmem& sm = *reinterpret_cast<CandSmem*>(cand_smem_raw);
  __shared__ int abort_flag;
  const int tid = threadIdx.x;
  auto src_of = [&](int item, int* n) {
    const int row = item / nchunks, chunk = item % nchunks;
    *n = min(kCandChunk, V - chunk * kCandChunk);
    return reinterpret_cast<const uint16_t*>(logits + (size_t)row * ld + (size_t)chunk * kCandChunk);
  };
  auto issue = [&](int item, int b) {
    int n;
    const uint16_t* src = src_of(item, &n);
    mbar_arrive_expect_tx(&sm.full[b], (uint32_t)n * 2u);
    bulk_load(sm.buf[b], src, (uint32_t)n * 2u, &sm.full[b]);
  };
  if (tid == 0) {
    abort_flag = 0;
    mbar_init(&sm.full[0], 1);
    mbar_init(&sm.full[1], 1);
    fence_mbar_init();
    if (tma && (int)blockIdx.x < items) issue(blockIdx.x, 0);
  }
  __syncthreads();
  int it = 0;
  for (int item = blockIdx.x; item < items; item += gridDim.x, ++it) {
    const int b = it & 1;
    if (tma && tid == 0 && item + (int)gridDim.x < items) issue(item + gridDim.x, b ^ 1);
    int n;
    const uint16_t* src = src_of(item, &n);
    if (tma) {
      if (!mbar_wait(&sm.full[b], (uint32_t)((it >> 1) & 1), status, kErrTimeoutProducer, &abort_flag)) {
        // a copy that never lands: report and stop (the other copy of this CTA has landed or was never issued)
        break;
      }
      src = sm.buf[b];
    }
    const int row = item / nchunks, chunk = item % nchunks;
    float T = temp ? temp[row / rows_per_temp] : 1.0f;
    if (!(T > 0.f)) T = 1.0f;   // greedy rows: argmax of the raw logits
    const bool vec = tma || (n % 8 == 0 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0);
    cand_chunk<KC, LSE>(sm, src, n, vec, T, vocab_offset + chunk * kCandChunk, cv + (size_t)item * KC,
                        ci + (size_t)item * KC, cms ? cms + (size_t)item * 2 : nullptr, overflow + item);
    __syncthreads();
  }
}

// ------------------------------------------------------------------------------------------------
// seeded coins (MurmurHash3_x86_32, Appleby, public domain)
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t rotl32(uint32_t x, int r) { return (x << r) | (x >> (32 - r)); }

__device__ __forceinline__ uint32_t murmur3_words(const uint32_t* w, int n, uint32_t seed) {
  uint32_t h = seed;
  for (int i = 0; i < n; ++i) {
    uint32_t k = w[i] * 0xCC9E2D51u;
    k = rotl32(k, 15);
    k *= 0x1B873593u;
    h ^= k;
    h = rotl32(h, 13);
    h = h * 5u + 0xE6546B64u;
  }
  h ^= (uint32_t)(4 * n);
  h ^= h >> 16;
  h *= 0x85EBCA6Bu;
  h ^= h >> 13;
  h *= 0xC2B2AE35u;
  h ^= h >> 16;
  return h;
}

__device__ __forceinline__ float seeded_coin(int64_t seed, int64_t prefix_len, int col) {
  const uint32_t w[3] = {(uint32_t)((uint64_t)prefix_len & 0xffffffffu), (uint32_t)((uint64_t)prefix_len >> 32),
                         (uint32_t)col};
  const uint32_t h = murmur3_words(w, 3, (uint32_t)((uint64_t)seed & 0xffffffffu));
  const float u = (float)((double)h / 4294967295.0);
  return fminf(u, 0.99999994f);   // the largest fp32 below 1
}

// ------------------------------------------------------------------------------------------------
// accept walk
// ------------------------------------------------------------------------------------------------
constexpr int kAcceptThreads = 256;
constexpr int kMaxCand = 1024;   // shards x chunks x KC per row
constexpr int kMaxNodes = 64;

struct AcceptArgs {
  // candidate values / vocab indices, [ranks][rows][nch][KC]: list s of a row is chunk s % nch of rank s / nch
  const float* cv;
  const int* ci;
  int64_t rank_stride, row_stride;
  int S, nch, KC;           // candidate lists per row (ranks x chunks), chunks per rank, entries per list
  const int64_t* tokens;    // [R, N]
  const int64_t* parent;    // [R, N] (-1 for the root)
  const float* temp;        // [R]
  const int* top_k;         // [R]
  const float* top_p;       // [R]
  const int64_t* seed;      // [R]
  const int64_t* committed; // [R]: coin key (committed length)
  int N, D;
  int64_t* acc;             // [R, D] accepted node ids, -1 padded
  int64_t* bonus;           // [R]
};

// order-preserving 32-bit image of an fp32 value
__device__ __forceinline__ uint32_t f32_key(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float f32_of_key(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

__global__ void __launch_bounds__(kAcceptThreads) spec_accept_kernel(const AcceptArgs a) {
  __shared__ uint64_t cand[kMaxCand];  // (value key, ~vocab index): descending = value desc, index asc
  __shared__ float pk[64];             // kept probabilities in sorted order (first k)
  __shared__ int tk[64];               // their vocab indices
  __shared__ int64_t s_tok[kMaxNodes];
  __shared__ int64_t s_par[kMaxNodes];
  __shared__ float kp[kMaxNodes];      // target probability of each child's token under the current node
  __shared__ int s_next, s_k, s_done;

  const int r = blockIdx.x, tid = threadIdx.x;
  const int N = a.N, D = a.D;
  const float T = a.temp[r];
  const bool greedy = !(T > 0.f);
  const int n_all = a.S * a.KC;
  int P = 1;
  while (P < n_all) P <<= 1;
  const float top_p = a.top_p[r];
  const int64_t seed = a.seed[r], committed = a.committed[r];
  for (int j = tid; j < N; j += kAcceptThreads) {
    s_tok[j] = a.tokens[(int64_t)r * N + j];
    s_par[j] = a.parent[(int64_t)r * N + j];
  }
  for (int j = tid; j < D; j += kAcceptThreads) a.acc[(int64_t)r * D + j] = -1;
  int cur = 0;
  for (int d = 1; d <= D + 1; ++d) {
    const int64_t row = (int64_t)r * N + cur;
    // ---- this node's candidates from every shard / chunk, sorted ----
    for (int j = tid; j < P; j += kAcceptThreads) {
      uint64_t w = 0ull;
      if (j < n_all) {
        const int s = j / a.KC, q = j % a.KC;
        const int64_t o = (int64_t)(s / a.nch) * a.rank_stride + row * a.row_stride + (s % a.nch) * a.KC + q;
        const int idx = a.ci[o];
        if (idx != 0x7fffffff) w = ((uint64_t)f32_key(a.cv[o]) << 32) | (uint64_t)(0xffffffffu - (uint32_t)idx);
      }
      cand[j] = w;
    }
    __syncthreads();
    bitonic_desc_u64(cand, P);
    // ---- target distribution over the kept tokens ----
    if (tid < 32) {
      const int k = greedy ? 1 : min(max(a.top_k[r], 1), min(a.KC, n_all));
      for (int i = tid; i < k; i += 32) tk[i] = (int)(0xffffffffu - (uint32_t)(cand[i] & 0xffffffffu));
      if (tid == 0) {
        const float m = f32_of_key((uint32_t)(cand[0] >> 32));
        float ssum = 0.f;
        for (int i = 0; i < k; ++i) {
          pk[i] = expf(f32_of_key((uint32_t)(cand[i] >> 32)) - m);
          ssum += pk[i];
        }
        for (int i = 0; i < k; ++i) pk[i] = pk[i] / ssum;
        if (!greedy && top_p < 1.0f) {
          float cum = 0.f, kept = 0.f;
          for (int i = 0; i < k; ++i) {
            cum += pk[i];
            if (!((cum - pk[i]) < top_p)) pk[i] = 0.f;
            kept += pk[i];
          }
          for (int i = 0; i < k; ++i) pk[i] = pk[i] / kept;
        }
        s_k = k;
      }
    }
    __syncthreads();
    const int k = s_k;
    // ---- probability of every child's token ----
    for (int j = tid; j < N; j += kAcceptThreads) {
      float p = 0.f;
      if (j > 0 && d <= D && s_par[j] == cur) {
        const int64_t tok = s_tok[j];
        for (int i = 0; i < k; ++i)
          if (tk[i] == tok) p = pk[i];
      }
      kp[j] = p;
    }
    __syncthreads();
    if (tid == 0) {
      const float u = seeded_coin(seed, committed, d - 1);
      int next = -1;
      float cum = 0.f;
      for (int j = 1; j < N && d <= D; ++j) {
        if (s_par[j] != cur) continue;
        cum += kp[j];
        if (u < cum) {
          next = j;
          break;
        }
      }
      s_done = next < 0;
      s_next = next;
      if (next >= 0) a.acc[(int64_t)r * D + (d - 1)] = next;
    }
    __syncthreads();
    if (s_done) {
      // bonus: the target distribution without the children's tokens (all of it if that leaves no mass),
      // inverse CDF in vocab-index order with the final coin
      if (tid < k) {          // zero the kept tokens that are children of cur (k <= 64 threads)
        bool child = false;
        for (int j = 1; j < N && d <= D; ++j) child |= (s_par[j] == cur && s_tok[j] == tk[tid]);
        kp[tid] = child ? 0.f : pk[tid];     // kp is free now: reuse it for q
      }
      __syncthreads();
      if (tid == 0) {
        int64_t tok;
        if (greedy) {
          tok = tk[0];
        } else {
          double tot = 0.0;
          for (int i = 0; i < k; ++i) tot += (double)kp[i];
          const bool empty = !(tot > 0.0);
          int ord[64];
          for (int i = 0; i < k; ++i) ord[i] = i;
          for (int i = 1; i < k; ++i) {          // kept tokens by vocab index
            const int x = ord[i];
            int j = i - 1;
            while (j >= 0 && tk[ord[j]] > tk[x]) {
              ord[j + 1] = ord[j];
              --j;
            }
            ord[j + 1] = x;
          }
          tot = 0.0;
          for (int i = 0; i < k; ++i) tot += (double)(empty ? pk[ord[i]] : kp[ord[i]]);
          const double target = (double)seeded_coin(seed, committed, D + 1) * tot;
          double c = 0.0;
          tok = tk[ord[k - 1]];
          for (int i = 0; i < k; ++i) {
            c += (double)(empty ? pk[ord[i]] : kp[ord[i]]);
            if (c > target) {
              tok = tk[ord[i]];
              break;
            }
          }
        }
        a.bonus[r] = tok;
      }
      break;
    }
    cur = s_next;
    __syncthreads();
  }
}

// ------------------------------------------------------------------------------------------------
// host entry points
// ------------------------------------------------------------------------------------------------

void sample_candidates(torch::Tensor logits, int64_t kc, c10::optional<torch::Tensor> temp, int64_t rows_per_temp,
                       int64_t vocab_offset, torch::Tensor cv, torch::Tensor ci, c10::optional<torch::Tensor> cms,
                       torch::Tensor status) {
  TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == at::kBFloat16 && logits.dim() == 2);
  TORCH_CHECK(logits.stride(1) == 1, "logits rows must be contiguous");
  const int rows = (int)logits.size(0), V = (int)logits.size(1);
  const int nchunks = (V + kCandChunk - 1) / kCandChunk;
  TORCH_CHECK(cv.is_cuda() && cv.scalar_type() == at::kFloat && cv.numel() == (int64_t)rows * nchunks * kc);
  TORCH_CHECK(ci.is_cuda() && ci.scalar_type() == at::kInt && ci.numel() == (int64_t)rows * nchunks * kc);
  if (temp) TORCH_CHECK(temp->is_cuda() && temp->scalar_type() == at::kFloat && rows_per_temp > 0);
  if (cms) TORCH_CHECK(cms->is_cuda() && cms->scalar_type() == at::kFloat && cms->numel() == (int64_t)rows * nchunks * 2);
  if (rows == 0) return;
  const at::cuda::CUDAGuard guard(logits.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const int items = rows * nchunks;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = std::min(items, 2 * sms);
  const int smem = (int)sizeof(CandSmem);
  const float* tp = temp ? temp->data_ptr<float>() : nullptr;
  auto* lp = reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr());
  float* cmsp = cms ? cms->data_ptr<float>() : nullptr;
  const int ld = (int)logits.stride(0);
  // bulk copies need 16-byte aligned rows and whole 16-byte chunk widths
  const int tma = ((reinterpret_cast<uintptr_t>(lp) & 15u) == 0 && (ld % 8) == 0 && (V % 8) == 0) ? 1 : 0;
  auto ovf = torch::empty({items}, logits.options().dtype(at::kInt));
  int* ovp = ovf.data_ptr<int>();
  int* st = status.data_ptr<int>();
  static bool attr[64][8] = {};   // per device and instantiation: the dynamic shared-memory opt-in
  TORCH_CHECK(dev < 64, "device index out of range");
  auto run = [&](auto kcv, auto lsev, int slot) {
    constexpr int KC = decltype(kcv)::value;
    constexpr bool LSE = decltype(lsev)::value;
    if (!attr[dev][slot]) {
      C10_CUDA_CHECK(cudaFuncSetAttribute(sample_candidates_kernel<KC, LSE>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      attr[dev][slot] = true;
    }
    sample_candidates_kernel<KC, LSE><<<grid, kCandThreads, smem, stream>>>(
        lp, V, ld, nchunks, items, (int)vocab_offset, tp, (int)rows_per_temp, cv.data_ptr<float>(),
        ci.data_ptr<int>(), cmsp, ovp, tma, st);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    sample_candidates_exact_kernel<KC, LSE><<<grid, kCandThreads, 0, stream>>>(
        lp, V, ld, nchunks, (int)vocab_offset, tp, (int)rows_per_temp, cv.data_ptr<float>(), ci.data_ptr<int>(),
        cmsp, ovp, items);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  };
  const bool l = cms.has_value();
  if (kc == 1) l ? run(std::integral_constant<int, 1>{}, std::true_type{}, 0)
                 : run(std::integral_constant<int, 1>{}, std::false_type{}, 1);
  else if (kc == 8) l ? run(std::integral_constant<int, 8>{}, std::true_type{}, 2)
                      : run(std::integral_constant<int, 8>{}, std::false_type{}, 3);
  else if (kc == 16) l ? run(std::integral_constant<int, 16>{}, std::true_type{}, 4)
                       : run(std::integral_constant<int, 16>{}, std::false_type{}, 5);
  else if (kc == 64) l ? run(std::integral_constant<int, 64>{}, std::true_type{}, 6)
                       : run(std::integral_constant<int, 64>{}, std::false_type{}, 7);
  else TORCH_CHECK(false, "candidate count must be 1, 8, 16 or 64");
}

int64_t sample_chunks(int64_t vocab) { return (vocab + kCandChunk - 1) / kCandChunk; }

void spec_accept(torch::Tensor cv, torch::Tensor ci, int64_t ranks, int64_t nch, int64_t kc,
                 torch::Tensor tokens, torch::Tensor parent, torch::Tensor temp, torch::Tensor top_k,
                 torch::Tensor top_p, torch::Tensor seed, torch::Tensor committed, int64_t D, torch::Tensor acc,
                 torch::Tensor bonus) {
  const int R = (int)tokens.size(0), N = (int)tokens.size(1);
  const int64_t S = ranks * nch;
  TORCH_CHECK(cv.is_cuda() && ci.is_cuda() && cv.scalar_type() == at::kFloat && ci.scalar_type() == at::kInt);
  // D = 0 with a one-node tree is a plain draw from the row's top-k / top-p distribution (the final coin)
  TORCH_CHECK(S * kc <= kMaxCand && kc <= 64 && N <= kMaxNodes && D >= 0, "spec_accept: sizes out of range");
  TORCH_CHECK(cv.numel() == ranks * (int64_t)R * N * nch * kc && ci.numel() == cv.numel(),
              "candidates must be [ranks, R * N, chunks, KC]");
  TORCH_CHECK(tokens.scalar_type() == at::kLong && parent.scalar_type() == at::kLong && tokens.is_contiguous() &&
              parent.is_contiguous() && parent.sizes() == tokens.sizes());
  TORCH_CHECK(temp.scalar_type() == at::kFloat && top_p.scalar_type() == at::kFloat && top_k.scalar_type() == at::kInt);
  TORCH_CHECK(seed.scalar_type() == at::kLong && committed.scalar_type() == at::kLong);
  TORCH_CHECK(acc.scalar_type() == at::kLong && acc.is_contiguous() && acc.size(0) == R && acc.size(1) == D);
  TORCH_CHECK(bonus.scalar_type() == at::kLong && bonus.numel() == R);
  if (R == 0) return;
  const at::cuda::CUDAGuard guard(cv.device());
  AcceptArgs a;
  a.cv = cv.data_ptr<float>();
  a.ci = ci.data_ptr<int>();
  a.row_stride = nch * kc;
  a.rank_stride = (int64_t)R * N * nch * kc;
  a.S = (int)S;
  a.nch = (int)nch;
  a.KC = (int)kc;
  a.tokens = tokens.data_ptr<int64_t>();
  a.parent = parent.data_ptr<int64_t>();
  a.temp = temp.data_ptr<float>();
  a.top_k = top_k.data_ptr<int>();
  a.top_p = top_p.data_ptr<float>();
  a.seed = seed.data_ptr<int64_t>();
  a.committed = committed.data_ptr<int64_t>();
  a.N = N;
  a.D = (int)D;
  a.acc = acc.data_ptr<int64_t>();
  a.bonus = bonus.data_ptr<int64_t>();
  spec_accept_kernel<<<R, kAcceptThreads, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace phx
