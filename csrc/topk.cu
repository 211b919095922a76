// Fused top-k + log-sum-exp over bf16 logits rows (vocab or vocab shard), sm_100a.
//
//   topk_logprobs(logits [R, V] bf16, k, temperature) -> (logprob [R, k] fp32, index [R, k] int64,
//                                                         lse [R] fp32)
// Without an lse output (argmax use) the kernel skips the exponentials and returns the raw x/T values.
// logprob = x/T - logsumexp(x/T) of the k largest x (ties toward the lower index), with T applied by
// IEEE division (the reference's verify top-k divides with div.rn.f32,
// docker/opt/v5/topkbf_normcfg/topkbf/kopt_topkbf.py:134-141). k = 1 is argmax.
//
// Stage 1: grid (rows x 16384-column chunks); a CTA holds its chunk in registers (eight 16-byte loads in
// flight per thread), reduces (max, sum exp), and selects its top-k through a threshold filter (the k-th
// largest per-thread maximum bounds the chunk's top k from below; see topk_stage1). Stage 2: one warp per row merges the splits' candidates
// and (max, sum) pairs. The per-split partials are also what a vocab-sharded tensor-parallel merge
// exchanges between ranks (values, global indices, log-sum-exp), a few hundred bytes per row.
// The reference's equivalent kernels are Triton (docker/opt/v4/topk20/topk20.py:124-253, kopt_topkbf).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace phx {

constexpr int kTopkThreads = 256;
constexpr int kTopkMaxK = 16;

template <int K>
struct TopK {
  float v[K];
  int i[K];
  __device__ __forceinline__ void init() {
#pragma unroll
    for (int k = 0; k < K; ++k) v[k] = -INFINITY, i[k] = 0x7fffffff;
  }
  __device__ __forceinline__ void push(float x, int idx) {
    if (!(x > v[K - 1] || (x == v[K - 1] && idx < i[K - 1]))) return;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const bool better = x > v[k] || (x == v[k] && idx < i[k]);
      if (better) {
        const float tv = v[k];
        const int ti = i[k];
        v[k] = x;
        i[k] = idx;
        x = tv;
        idx = ti;
      }
    }
  }
};

// (m, s) pairs over raw logits: s = sum 2^((x - m) * c2), c2 = log2(e) / T
__device__ __forceinline__ void ms_combine(float& m, float& s, float m2, float s2, float c2) {
  const float M = fmaxf(m, m2);
  if (M == -INFINITY) return;
  s = s * exp2f((m - M) * c2) + s2 * exp2f((m2 - M) * c2);
  m = M;
}

// Warp-cooperative selection of the best `k` of `n` candidates (vals/idxs in shared memory; consumed).
template <int K>
__device__ __forceinline__ void warp_select(float* vals, int* idxs, int n, float* out_v, int* out_i) {
  const int lane = threadIdx.x & 31;
  for (int r = 0; r < K; ++r) {
    float bv = -INFINITY;
    int bi = 0x7fffffff, bp = -1;
    for (int q = lane; q < n; q += 32) {
      const float x = vals[q];
      const int xi = idxs[q];
      if (x > bv || (x == bv && xi < bi)) bv = x, bi = xi, bp = q;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      const int op = __shfl_xor_sync(0xffffffffu, bp, o);
      if (ov > bv || (ov == bv && oi < bi)) bv = ov, bi = oi, bp = op;
    }
    if (lane == 0) {
      out_v[r] = bv;
      out_i[r] = bi;
      if (bp >= 0) vals[bp] = -INFINITY, idxs[bp] = 0x7fffffff;
    }
    __syncwarp();
  }
}

// The K best entries of a warp's 32 sorted register lists (value desc, index asc): K rounds of a warp-wide
// argmax over the list heads; the winning lane pops its head.
template <int K>
__device__ __forceinline__ void warp_merge_lists(TopK<K>& tk, float* out_v, int* out_i) {
  const int lane = threadIdx.x & 31;
  for (int r = 0; r < K; ++r) {
    float bv = tk.v[0];
    int bi = tk.i[0], bl = lane;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      const int ol = __shfl_xor_sync(0xffffffffu, bl, o);
      if (ov > bv || (ov == bv && oi < bi)) bv = ov, bi = oi, bl = ol;
    }
    if (lane == 0) out_v[r] = bv, out_i[r] = bi;
    if (lane == bl) {
#pragma unroll
      for (int k = 0; k + 1 < K; ++k) tk.v[k] = tk.v[k + 1], tk.i[k] = tk.i[k + 1];
      tk.v[K - 1] = -INFINITY;
      tk.i[K - 1] = 0x7fffffff;
    }
  }
}

constexpr int kTopkVec = 8;                                   // 16-byte vectors per thread
constexpr int kTopkChunk = kTopkThreads * kTopkVec * 8;        // columns per CTA (16384)
constexpr int kTopkCap = 1024;                                 // candidate buffer of the threshold filter
constexpr int kTopkCapW = kTopkCap / (kTopkThreads / 32);      // per warp

// 2^x by the MUFU instruction (ex2.approx.ftz: relative error about 2^-22; the log-sum-exp needs no more)
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Descending bitonic sort of one value per lane across a warp.
__device__ __forceinline__ float warp_sort_desc(float v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      const float o = __shfl_xor_sync(0xffffffffu, v, j);
      const bool keep_max = ((lane & j) == 0) == ((lane & k) == 0);
      v = keep_max ? fmaxf(v, o) : fminf(v, o);
    }
  }
  return v;
}

// Selection runs on the raw logits: x -> x / T (T > 0, IEEE division) keeps the order of distinct bf16 values
// (fp32 has 16 more mantissa bits than bf16), so the k largest x are the k largest x / T and only the winners
// are divided (in stage 2).
// One CTA per (row, 16384-column chunk); the chunk is read once, 64 values per thread held in registers
// (eight 16-byte loads in flight per thread). Each thread forms its maximum m_t and s_t = sum 2^((x - m_t) c2),
// c2 = log2(e) / T; the CTA combines them into the chunk's (max, sum). Each warp sorts its 32 thread maxima;
// tau is the largest of the warps' K-th values: K distinct elements reach it, so the chunk's top K are all
// >= tau. Every warp appends its elements >= tau to its own shared region (ballot order, no atomics; a few
// dozen on random rows), selects its top K from them, and warp 0 selects from the 8 x K by (value desc,
// index asc). If a warp has more than kTopkCapW elements at or above tau (a constant row, say), every thread
// builds a register top-K instead and the warps merge those lists: the same result, slower.
template <int K, bool LSE>
__global__ void __launch_bounds__(kTopkThreads, 3) topk_stage1(const __nv_bfloat16* __restrict__ logits, int V, int ld,
                                                            int splits, float c2, float* __restrict__ pv,
                                                            int* __restrict__ pi, float* __restrict__ pm,
                                                            float* __restrict__ ps) {
  __shared__ float cv[kTopkCap];
  __shared__ int ci[kTopkCap];
  __shared__ float wv[(kTopkThreads / 32) * K];
  __shared__ int wi[(kTopkThreads / 32) * K];
  __shared__ float red_m[kTopkThreads / 32], red_s[kTopkThreads / 32];
  __shared__ float wtau[kTopkThreads / 32];
  __shared__ int s_cnt;
  const int row = blockIdx.x / splits, sp = blockIdx.x % splits;
  const int v0 = sp * kTopkChunk, v1 = min(V, v0 + kTopkChunk);
  const __nv_bfloat16* x = logits + (size_t)row * ld;
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  if (tid == 0) s_cnt = 0;

  // ---- load: vector j of thread t covers columns v0 + (j * 256 + t) * 8 .. + 8 ----
  uint4 d[kTopkVec];
  const bool vec_ok = (ld % 8) == 0;
#pragma unroll
  for (int j = 0; j < kTopkVec; ++j) {
    const int c = v0 + (j * kTopkThreads + tid) * 8;
    if (vec_ok && c + 8 <= v1) {
      d[j] = __ldcs(reinterpret_cast<const uint4*>(x + c));
    } else {
      uint32_t h[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint16_t lo = c + 2 * e < v1 ? __bfloat16_as_ushort(x[c + 2 * e]) : (uint16_t)0xff80u;   // -inf
        const uint16_t hi = c + 2 * e + 1 < v1 ? __bfloat16_as_ushort(x[c + 2 * e + 1]) : (uint16_t)0xff80u;
        h[e] = (uint32_t)lo | ((uint32_t)hi << 16);
      }
      d[j] = make_uint4(h[0], h[1], h[2], h[3]);
    }
  }
  auto val = [&](int j, int e) -> float {   // element e (0..7) of vector j
    const uint32_t wd = e < 2 ? d[j].x : e < 4 ? d[j].y : e < 6 ? d[j].z : d[j].w;
    return __uint_as_float((e & 1) ? (wd & 0xffff0000u) : (wd << 16));
  };
  auto col = [&](int j, int e) { return v0 + (j * kTopkThreads + tid) * 8 + e; };

  // ---- thread max and sum exp (2^(x c2 - m c2): one FFMA and one ex2 per element) ----
  float vmax[kTopkVec];
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < kTopkVec; ++j) {
    float a = val(j, 0);
#pragma unroll
    for (int e = 1; e < 8; ++e) a = fmaxf(a, val(j, e));
    vmax[j] = a;
    m = fmaxf(m, a);
  }
  float s = 0.f;
  if constexpr (LSE) {
    if (m != -INFINITY) {
      const float mc = -m * c2;
#pragma unroll
      for (int j = 0; j < kTopkVec; ++j)
#pragma unroll
        for (int e = 0; e < 8; ++e) s += ex2_approx(fmaf(val(j, e), c2, mc));
    }
  }
  float bm = m, bs = s;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, bm, o), os = __shfl_xor_sync(0xffffffffu, bs, o);
    ms_combine(bm, bs, om, os, c2);
  }
  if (lane == 0) red_m[w] = bm, red_s[w] = bs;
  __syncthreads();

  // ---- threshold: tau = max over warps of the K-th largest thread maximum of the warp (a warp bitonic sort
  // of its 32 maxima); the warp reaching tau has K elements >= tau, so the CTA's top K are all >= tau ----
  {
    const float srt = warp_sort_desc(m);
    const float tw = __shfl_sync(0xffffffffu, srt, K - 1);
    if (lane == 0) wtau[w] = tw;
  }
  __syncthreads();
  float tau = wtau[0];
#pragma unroll
  for (int q = 1; q < kTopkThreads / 32; ++q) tau = fmaxf(tau, wtau[q]);

  // ---- filter: every warp appends its elements >= tau to its own region, in (vector, element, lane) order ----
  float* rv = cv + w * kTopkCapW;
  int* ri = ci + w * kTopkCapW;
  int cnt = 0;
  const unsigned lt = (1u << lane) - 1u;
#pragma unroll
  for (int j = 0; j < kTopkVec; ++j) {
    if (!__any_sync(0xffffffffu, vmax[j] >= tau && vmax[j] != -INFINITY)) continue;   // most vectors
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float f = val(j, e);
      const bool take = f >= tau && f != -INFINITY;
      const unsigned msk = __ballot_sync(0xffffffffu, take);
      if (take) {
        const int slot = cnt + __popc(msk & lt);
        if (slot < kTopkCapW) rv[slot] = f, ri[slot] = col(j, e);
      }
      cnt += __popc(msk);
    }
  }
  if (lane == 0 && cnt > kTopkCapW) s_cnt = 1;   // overflow flag
  __syncwarp();
  if (cnt <= kTopkCapW) warp_select<K>(rv, ri, cnt, wv + w * K, wi + w * K);
  __syncthreads();
  const size_t base = (size_t)blockIdx.x * K;
  if (!s_cnt) {
    if (w == 0) {
      warp_select<K>(wv, wi, (kTopkThreads / 32) * K, pv + base, pi + base);
      if (lane == 0) {
        float cm = red_m[0], cs = red_s[0];
        for (int q = 1; q < kTopkThreads / 32; ++q) ms_combine(cm, cs, red_m[q], red_s[q], c2);
        pm[blockIdx.x] = cm, ps[blockIdx.x] = cs;
      }
    }
    return;
  }
  __syncthreads();   // every warp's selection is done before the overflow path rewrites wv / wi
  // ---- overflow (heavy ties at the threshold): per-thread register top-K, then two warp-level merges ----
  // (re-reads the chunk from global memory, so the register copy is dead by now)
  TopK<K> tk;
  tk.init();
#pragma unroll 1
  for (int j = 0; j < kTopkVec; ++j)
#pragma unroll 1
    for (int e = 0; e < 8; ++e) {
      const int c = v0 + (j * kTopkThreads + tid) * 8 + e;
      const float f = c < v1 ? __bfloat162float(x[c]) : -INFINITY;
      if (f != -INFINITY) tk.push(f, c);
    }
  warp_merge_lists<K>(tk, wv + w * K, wi + w * K);
  __syncthreads();
  if (w == 0) {
    warp_select<K>(wv, wi, (kTopkThreads / 32) * K, pv + base, pi + base);
    if (lane == 0) {
      float cm = red_m[0], cs = red_s[0];
      for (int q = 1; q < kTopkThreads / 32; ++q) ms_combine(cm, cs, red_m[q], red_s[q], c2);
      pm[blockIdx.x] = cm, ps[blockIdx.x] = cs;
    }
  }
}

// K = 1 (argmax, greedy verify): a streaming scan with four 16-byte loads in flight per thread over a slice
// of about V * R / 592 columns per CTA; per 8-element vector one max (and, with LSE, one rescale check and
// eight exp2 terms); the thread keeps its first maximum (indices rise along its scan).
template <bool LSE>
__global__ void __launch_bounds__(kTopkThreads) argmax_stage1(const __nv_bfloat16* __restrict__ logits, int V, int ld,
                                                              int splits, int chunk, float c2,
                                                              float* __restrict__ pv, int* __restrict__ pi,
                                                              float* __restrict__ pm, float* __restrict__ ps) {
  __shared__ float wv[kTopkThreads / 32];
  __shared__ int wi[kTopkThreads / 32];
  __shared__ float red_m[kTopkThreads / 32], red_s[kTopkThreads / 32];
  const int row = blockIdx.x / splits, sp = blockIdx.x % splits;
  const int v0 = sp * chunk, v1 = min(V, v0 + chunk);
  const __nv_bfloat16* x = logits + (size_t)row * ld;
  float m = -INFINITY, s = 0.f, bv = -INFINITY;
  int bi = 0x7fffffff;
  auto take8 = [&](const float (&f)[8], int idx0) {
    float gmax = f[0];
#pragma unroll
    for (int e = 1; e < 8; ++e) gmax = fmaxf(gmax, f[e]);
    if (gmax == -INFINITY) return;
    if constexpr (LSE) {
      if (gmax > m) {
        s *= exp2f((m - gmax) * c2);
        m = gmax;
      }
      float acc = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc += exp2f((f[e] - m) * c2);
      s += acc;
    }
    if (gmax > bv) {
#pragma unroll
      for (int e = 7; e >= 0; --e)          // the lowest index of the vector's maximum
        if (f[e] == gmax) bi = idx0 + e;
      bv = gmax;
    }
  };
  auto take1 = [&](float f, int idx) {
    float g[8] = {f, -INFINITY, -INFINITY, -INFINITY, -INFINITY, -INFINITY, -INFINITY, -INFINITY};
    take8(g, idx);
  };
  if ((ld % 8) == 0) {
    const int vend = v0 + ((v1 - v0) / 8) * 8;
    constexpr int U = 4, STEP = kTopkThreads * 8;
    for (int vb = v0 + threadIdx.x * 8; vb < vend; vb += U * STEP) {
      uint4 d[U];
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (vb + u * STEP < vend) d[u] = __ldcs(reinterpret_cast<const uint4*>(x + vb + u * STEP));
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int v = vb + u * STEP;
        if (v >= vend) break;
        const uint32_t ww[4] = {d[u].x, d[u].y, d[u].z, d[u].w};
        float f[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 t = unpack_bf16x2(ww[e]);
          f[2 * e] = t.x;
          f[2 * e + 1] = t.y;
        }
        take8(f, v);
      }
    }
    for (int t = vend + threadIdx.x; t < v1; t += kTopkThreads) take1(__bfloat162float(x[t]), t);
  } else {
    for (int t = v0 + threadIdx.x; t < v1; t += kTopkThreads) take1(__bfloat162float(x[t]), t);
  }
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o), os = __shfl_xor_sync(0xffffffffu, s, o);
    ms_combine(m, s, om, os, c2);
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) bv = ov, bi = oi;
  }
  if (lane == 0) red_m[w] = m, red_s[w] = s, wv[w] = bv, wi[w] = bi;
  __syncthreads();
  if (threadIdx.x == 0) {
    float cm = red_m[0], cs = red_s[0], cv = wv[0];
    int cidx = wi[0];
    for (int q = 1; q < kTopkThreads / 32; ++q) {
      ms_combine(cm, cs, red_m[q], red_s[q], c2);
      if (wv[q] > cv || (wv[q] == cv && wi[q] < cidx)) cv = wv[q], cidx = wi[q];
    }
    pv[blockIdx.x] = cv, pi[blockIdx.x] = cidx, pm[blockIdx.x] = cm, ps[blockIdx.x] = cs;
  }
}

template <int K>
__global__ void topk_stage2(int rows, int splits, int k_out, const float* __restrict__ pv, const int* __restrict__ pi,
                            const float* __restrict__ pm, const float* __restrict__ ps, float* __restrict__ out_lp,
                            int64_t* __restrict__ out_idx, float* __restrict__ out_lse, int vocab_offset,
                            bool with_lse, float temp, float c2) {
  extern __shared__ uint8_t smem[];
  const int warps = blockDim.x >> 5;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * warps + w;
  if (row >= rows) return;
  float* vals = reinterpret_cast<float*>(smem) + (size_t)w * splits * K;
  int* idxs = reinterpret_cast<int*>(reinterpret_cast<float*>(smem) + (size_t)warps * splits * K) + (size_t)w * splits * K;
  float m = -INFINITY, s = 0.f;
  for (int q = lane; q < splits; q += 32)
    ms_combine(m, s, pm[(size_t)row * splits + q], ps[(size_t)row * splits + q], c2);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o), os = __shfl_xor_sync(0xffffffffu, s, o);
    ms_combine(m, s, om, os, c2);
  }
  for (int q = lane; q < splits * K; q += 32) {
    vals[q] = pv[(size_t)row * splits * K + q];
    idxs[q] = pi[(size_t)row * splits * K + q];
  }
  __syncwarp();
  __shared__ float ov[32][kTopkMaxK];
  __shared__ int oi[32][kTopkMaxK];
  warp_select<K>(vals, idxs, splits * K, ov[w], oi[w]);
  const bool scaled = temp != 1.0f;
  // log-sum-exp of x / T = m / T + ln(sum exp((x - m) / T)); the winners' x / T by IEEE division
  const float lse = with_lse ? (scaled ? __fdiv_rn(m, temp) : m) + logf(s) : 0.f;
  if (lane < k_out) {
    const float v = ov[w][lane];
    out_lp[(size_t)row * k_out + lane] = (scaled ? __fdiv_rn(v, temp) : v) - lse;
    out_idx[(size_t)row * k_out + lane] = (int64_t)oi[w][lane] + vocab_offset;
  }
  if (lane == 0 && out_lse) out_lse[row] = lse;
}

template <int K>
static void run_topk(const torch::Tensor& logits, int64_t k, double temperature, torch::Tensor& lp, torch::Tensor& idx,
                     c10::optional<torch::Tensor> lse, int64_t vocab_offset, cudaStream_t stream) {
  const int R = logits.size(0), V = logits.size(1), ld = logits.stride(0);
  int splits = (V + kTopkChunk - 1) / kTopkChunk, chunk = kTopkChunk;
  if (K == 1) {   // streaming argmax: about four CTAs per SM in total
    splits = std::max(1, std::min((V + 4095) / 4096, (148 * 4 + R - 1) / R));
    chunk = ((V + splits - 1) / splits + 7) / 8 * 8;
    splits = (V + chunk - 1) / chunk;
  }
  auto opts = logits.options().dtype(at::kFloat);
  auto pv = torch::empty({R * splits * K}, opts);
  auto pi = torch::empty({R * splits * K}, opts.dtype(at::kInt));
  auto pm = torch::empty({R * splits}, opts);
  auto ps = torch::empty({R * splits}, opts);
  const float c2 = (float)(1.4426950408889634 / temperature);   // log2(e) / T
  const auto* xp = reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr());
  if constexpr (K == 1) {
    auto a1 = lse ? argmax_stage1<true> : argmax_stage1<false>;
    a1<<<R * splits, kTopkThreads, 0, stream>>>(xp, V, ld, splits, chunk, c2, pv.data_ptr<float>(),
                                                 pi.data_ptr<int>(), pm.data_ptr<float>(), ps.data_ptr<float>());
  } else {
    auto stage1 = lse ? topk_stage1<K, true> : topk_stage1<K, false>;
    stage1<<<R * splits, kTopkThreads, 0, stream>>>(xp, V, ld, splits, c2, pv.data_ptr<float>(), pi.data_ptr<int>(),
                                                     pm.data_ptr<float>(), ps.data_ptr<float>());
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  const int warps = 4;
  const size_t smem = (size_t)warps * splits * K * 8;
  topk_stage2<K><<<(R + warps - 1) / warps, warps * 32, smem, stream>>>(
      R, splits, (int)k, pv.data_ptr<float>(), pi.data_ptr<int>(), pm.data_ptr<float>(), ps.data_ptr<float>(),
      lp.data_ptr<float>(), idx.data_ptr<int64_t>(), lse ? lse->data_ptr<float>() : nullptr, (int)vocab_offset,
      lse.has_value(), (float)temperature, c2);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void topk_logprobs(torch::Tensor logits, int64_t k, double temperature, torch::Tensor lp, torch::Tensor idx,
                   c10::optional<torch::Tensor> lse, int64_t vocab_offset) {
  TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == at::kBFloat16 && logits.dim() == 2 && logits.stride(1) == 1);
  TORCH_CHECK(k >= 1 && k <= kTopkMaxK && k <= logits.size(1), "1 <= k <= 16");
  TORCH_CHECK(temperature > 0, "temperature must be > 0 (use k = 1 for greedy)");
  TORCH_CHECK(logits.size(1) >= 1 && (size_t)logits.size(1) < (1ull << 31));
  if (logits.size(0) == 0) return;
  const at::cuda::CUDAGuard guard(logits.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  if (k == 1) run_topk<1>(logits, k, temperature, lp, idx, lse, vocab_offset, stream);
  else if (k <= 4) run_topk<4>(logits, k, temperature, lp, idx, lse, vocab_offset, stream);
  else if (k <= 8) run_topk<8>(logits, k, temperature, lp, idx, lse, vocab_offset, stream);
  else run_topk<16>(logits, k, temperature, lp, idx, lse, vocab_offset, stream);
}

}  // namespace phx
