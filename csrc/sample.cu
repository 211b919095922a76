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

template <int KC, bool LSE>
__global__ void __launch_bounds__(kCandThreads) sample_candidates_kernel(
    const __nv_bfloat16* __restrict__ logits, int V, int ld, int nchunks, int vocab_offset,
    const float* __restrict__ temp, int rows_per_temp, float* __restrict__ cv, int* __restrict__ ci,
    float* __restrict__ cms) {
  __shared__ __align__(16) uint16_t keys[kCandChunk];
  __shared__ uint32_t hist[256];
  __shared__ uint32_t wcnt[kCandThreads / 32];
  __shared__ int s_bin;
  __shared__ uint32_t s_above, s_gt;
  __shared__ float red[kCandThreads / 32];

  const int row = blockIdx.x, chunk = blockIdx.y;
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

__device__ __forceinline__ bool cand_better(float a, int ia, float b, int ib) { return a > b || (a == b && ia < ib); }

__global__ void __launch_bounds__(kAcceptThreads) spec_accept_kernel(const AcceptArgs a) {
  __shared__ float sv[kMaxCand];
  __shared__ int si[kMaxCand];
  __shared__ float kp[kMaxNodes];      // target probability of each node's token under the current node
  __shared__ float pk[kMaxCand];       // kept probabilities (sorted order), first k entries
  __shared__ int s_next, s_k, s_done;

  const int r = blockIdx.x, tid = threadIdx.x;
  const int N = a.N, D = a.D;
  const float T = a.temp[r];
  const bool greedy = !(T > 0.f);
  const int n_all = a.S * a.KC;
  int P = 1;
  while (P < n_all) P <<= 1;
  const float top_p = a.top_p[r];
  int cur = 0;
  for (int j = tid; j < D; j += kAcceptThreads) a.acc[(int64_t)r * D + j] = -1;
  for (int d = 1; d <= D + 1; ++d) {
    const int64_t row = (int64_t)r * N + cur;
    // ---- gather this node's candidates and sort them (value desc, index asc) ----
    for (int j = tid; j < P; j += kAcceptThreads) {
      if (j < n_all) {
        const int s = j / a.KC, q = j % a.KC;
        const int64_t o = (int64_t)(s / a.nch) * a.rank_stride + row * a.row_stride + (s % a.nch) * a.KC + q;
        sv[j] = a.cv[o];
        si[j] = a.ci[o];
      } else {
        sv[j] = -INFINITY;
        si[j] = 0x7fffffff;
      }
    }
    __syncthreads();
    for (int size = 2; size <= P; size <<= 1) {
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        for (int j = tid; j < P; j += kAcceptThreads) {
          const int o = j ^ stride;
          if (o > j) {
            const bool desc = (j & size) == 0;   // overall descending
            const bool sw = desc ? cand_better(sv[o], si[o], sv[j], si[j]) : cand_better(sv[j], si[j], sv[o], si[o]);
            if (sw) {
              const float tv = sv[j];
              const int ti = si[j];
              sv[j] = sv[o];
              si[j] = si[o];
              sv[o] = tv;
              si[o] = ti;
            }
          }
        }
        __syncthreads();
      }
    }
    // ---- target distribution over the kept tokens ----
    if (tid == 0) {
      int k = greedy ? 1 : min(max(a.top_k[r], 1), min(a.KC, n_all));
      const float m = sv[0];
      float s = 0.f;
      for (int i = 0; i < k; ++i) {
        pk[i] = expf(sv[i] - m);
        s += pk[i];
      }
      for (int i = 0; i < k; ++i) pk[i] = pk[i] / s;
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
    __syncthreads();
    const int k = s_k;
    // ---- probability of every child's token (nodes whose parent is cur) ----
    for (int j = tid; j < N; j += kAcceptThreads) {
      float p = 0.f;
      if (j > 0 && d <= D && a.parent[(int64_t)r * N + j] == cur) {
        const int64_t tok = a.tokens[(int64_t)r * N + j];
        for (int i = 0; i < k; ++i)
          if (si[i] == tok) p = pk[i];
      }
      kp[j] = p;
    }
    __syncthreads();
    if (tid == 0) {
      const int64_t committed = a.committed[r];
      const float u = seeded_coin(a.seed[r], committed, d - 1);
      int next = -1;
      float cum = 0.f;
      for (int j = 1; j < N && d <= D; ++j) {
        if (a.parent[(int64_t)r * N + j] != cur) continue;
        cum += kp[j];
        if (u < cum) {
          next = j;
          break;
        }
      }
      s_done = 0;
      if (next >= 0) {
        a.acc[(int64_t)r * D + (d - 1)] = next;
        s_next = next;
      } else {
        // bonus: the target distribution without the children's tokens (all of it if that leaves no mass),
        // inverse CDF in vocab-index order with the final coin
        int64_t tok;
        if (greedy) {
          tok = si[0];
        } else {
          float q[64 + 1];   // k <= KC <= 64
          int ord[64 + 1];
          double tot = 0.0;
          for (int i = 0; i < k; ++i) {
            q[i] = pk[i];
            for (int j = 1; j < N && d <= D; ++j)
              if (a.parent[(int64_t)r * N + j] == cur && a.tokens[(int64_t)r * N + j] == si[i]) q[i] = 0.f;
            tot += q[i];
          }
          if (!(tot > 0.0))
            for (int i = 0; i < k; ++i) q[i] = pk[i];
          // order the kept tokens by vocab index
          for (int i = 0; i < k; ++i) ord[i] = i;
          for (int i = 1; i < k; ++i) {
            const int x = ord[i];
            int j = i - 1;
            while (j >= 0 && si[ord[j]] > si[x]) {
              ord[j + 1] = ord[j];
              --j;
            }
            ord[j + 1] = x;
          }
          double c = 0.0;
          tot = 0.0;
          for (int i = 0; i < k; ++i) tot += (double)q[ord[i]];
          const double target = (double)seeded_coin(a.seed[r], committed, D + 1) * tot;
          tok = si[ord[k - 1]];
          for (int i = 0; i < k; ++i) {
            c += (double)q[ord[i]];
            if (c > target) {
              tok = si[ord[i]];
              break;
            }
          }
        }
        a.bonus[r] = tok;
        s_done = 1;
      }
    }
    __syncthreads();
    if (s_done) break;
    cur = s_next;
    __syncthreads();
  }
}

// ------------------------------------------------------------------------------------------------
// host entry points
// ------------------------------------------------------------------------------------------------

void sample_candidates(torch::Tensor logits, int64_t kc, c10::optional<torch::Tensor> temp, int64_t rows_per_temp,
                       int64_t vocab_offset, torch::Tensor cv, torch::Tensor ci, c10::optional<torch::Tensor> cms) {
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
  dim3 grid(rows, nchunks);
  const float* tp = temp ? temp->data_ptr<float>() : nullptr;
  auto* lp = reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr());
  float* cmsp = cms ? cms->data_ptr<float>() : nullptr;
  const int ld = (int)logits.stride(0);
#define PHX_CAND(KC)                                                                                             \
  if (cms)                                                                                                       \
    sample_candidates_kernel<KC, true><<<grid, kCandThreads, 0, stream>>>(lp, V, ld, nchunks, (int)vocab_offset, \
                                                                          tp, (int)rows_per_temp,                 \
                                                                          cv.data_ptr<float>(),                   \
                                                                          ci.data_ptr<int>(), cmsp);              \
  else                                                                                                           \
    sample_candidates_kernel<KC, false><<<grid, kCandThreads, 0, stream>>>(lp, V, ld, nchunks, (int)vocab_offset, \
                                                                           tp, (int)rows_per_temp,                 \
                                                                           cv.data_ptr<float>(),                   \
                                                                           ci.data_ptr<int>(), nullptr);
  if (kc == 1) { PHX_CAND(1) }
  else if (kc == 8) { PHX_CAND(8) }
  else if (kc == 16) { PHX_CAND(16) }
  else if (kc == 64) { PHX_CAND(64) }
  else TORCH_CHECK(false, "candidate count must be 1, 8, 16 or 64");
#undef PHX_CAND
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

int64_t sample_chunks(int64_t vocab) { return (vocab + kCandChunk - 1) / kCandChunk; }

void spec_accept(torch::Tensor cv, torch::Tensor ci, int64_t ranks, int64_t nch, int64_t kc,
                 torch::Tensor tokens, torch::Tensor parent, torch::Tensor temp, torch::Tensor top_k,
                 torch::Tensor top_p, torch::Tensor seed, torch::Tensor committed, int64_t D, torch::Tensor acc,
                 torch::Tensor bonus) {
  const int R = (int)tokens.size(0), N = (int)tokens.size(1);
  const int64_t S = ranks * nch;
  TORCH_CHECK(cv.is_cuda() && ci.is_cuda() && cv.scalar_type() == at::kFloat && ci.scalar_type() == at::kInt);
  TORCH_CHECK(S * kc <= kMaxCand && kc <= 64 && N <= kMaxNodes && D >= 1, "spec_accept: sizes out of range");
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
