// Fused top-k + log-sum-exp over bf16 logits rows (vocab or vocab shard), sm_100a.
//
//   topk_logprobs(logits [R, V] bf16, k, temperature) -> (logprob [R, k] fp32, index [R, k] int64,
//                                                         lse [R] fp32)
// Without an lse output (argmax use) the kernel skips the exponentials and returns the raw x/T values.
// logprob = x/T - logsumexp(x/T) of the k largest x (ties toward the lower index), with T applied by
// IEEE division (the reference's verify top-k divides with div.rn.f32,
// docker/opt/v5/topkbf_normcfg/topkbf/kopt_topkbf.py:134-141). k = 1 is argmax.
//
// Stage 1: grid (rows x splits); a CTA scans its vocab slice with 16-byte loads, every thread keeps an
// online (max, sum exp) and a sorted register top-k; the CTA reduces (max, sum) and selects its top-k
// from the per-thread lists in shared memory. Stage 2: one warp per row merges the splits' candidates
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

__device__ __forceinline__ void ms_combine(float& m, float& s, float m2, float s2) {
  const float M = fmaxf(m, m2);
  if (M == -INFINITY) return;
  s = s * expf(m - M) + s2 * expf(m2 - M);
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

template <int K, bool LSE>
__global__ void __launch_bounds__(kTopkThreads) topk_stage1(const __nv_bfloat16* __restrict__ logits, int V, int ld,
                                                            int splits, int chunk, float temp,
                                                            float* __restrict__ pv, int* __restrict__ pi,
                                                            float* __restrict__ pm, float* __restrict__ ps) {
  __shared__ float sv[kTopkThreads * K];
  __shared__ int si[kTopkThreads * K];
  __shared__ float wv[(kTopkThreads / 32) * K];
  __shared__ int wi[(kTopkThreads / 32) * K];
  __shared__ float red_m[kTopkThreads / 32], red_s[kTopkThreads / 32];
  const int row = blockIdx.x / splits, sp = blockIdx.x % splits;
  const int v0 = sp * chunk, v1 = min(V, v0 + chunk);
  const __nv_bfloat16* x = logits + (size_t)row * ld;
  const bool scaled = temp != 1.0f;
  TopK<K> tk;
  tk.init();
  float m = -INFINITY, s = 0.f;
  auto take = [&](float val, int idx) {
    if (scaled) val = __fdiv_rn(val, temp);
    if (val == -INFINITY) return;
    if constexpr (LSE) {
      if (val > m) {
        s = s * expf(m - val) + 1.f;
        m = val;
      } else {
        s += expf(val - m);
      }
    }
    tk.push(val, idx);
  };
  if ((ld % 8) == 0) {
    // 16-byte vector body over whole 8-element groups (v0 is a multiple of 8), then the < 8 tail
    const int vend = v0 + ((v1 - v0) / 8) * 8;
    // argmax (K = 1): four 16-byte loads in flight per thread before any is consumed, the scan is otherwise
    // latency-bound; K > 1 keeps one (measured faster there: the register top-k list competes for registers)
    constexpr int U = K == 1 ? 4 : 1, STEP = kTopkThreads * 8;
    for (int vb = v0 + threadIdx.x * 8; vb < vend; vb += U * STEP) {
      uint4 w[U];
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (vb + u * STEP < vend) w[u] = __ldcs(reinterpret_cast<const uint4*>(x + vb + u * STEP));
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int v = vb + u * STEP;
        if (v >= vend) break;
        const uint32_t ww[4] = {w[u].x, w[u].y, w[u].z, w[u].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = unpack_bf16x2(ww[e]);
          take(f.x, v + 2 * e);
          take(f.y, v + 2 * e + 1);
        }
      }
    }
    for (int t = vend + threadIdx.x; t < v1; t += kTopkThreads) take(__bfloat162float(x[t]), t);
  } else {
    for (int t = v0 + threadIdx.x; t < v1; t += kTopkThreads) take(__bfloat162float(x[t]), t);
  }
  // (max, sum) block reduction
  float bm = m, bs = s;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, bm, o), os = __shfl_xor_sync(0xffffffffu, bs, o);
    ms_combine(bm, bs, om, os);
  }
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red_m[w] = bm, red_s[w] = bs;
#pragma unroll
  for (int k = 0; k < K; ++k) sv[threadIdx.x * K + k] = tk.v[k], si[threadIdx.x * K + k] = tk.i[k];
  __syncwarp();
  // two-level selection: every warp reduces its 32 threads' lists to K, then warp 0 selects from 8 x K
  warp_select<K>(sv + w * 32 * K, si + w * 32 * K, 32 * K, wv + w * K, wi + w * K);
  __syncthreads();
  if (w == 0) {
    float cm = lane < kTopkThreads / 32 ? red_m[lane] : -INFINITY;
    float cs = lane < kTopkThreads / 32 ? red_s[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, cm, o), os = __shfl_xor_sync(0xffffffffu, cs, o);
      ms_combine(cm, cs, om, os);
    }
    const size_t base = (size_t)blockIdx.x * K;
    warp_select<K>(wv, wi, (kTopkThreads / 32) * K, pv + base, pi + base);
    if (lane == 0) pm[blockIdx.x] = cm, ps[blockIdx.x] = cs;
  }
}

template <int K>
__global__ void topk_stage2(int rows, int splits, int k_out, const float* __restrict__ pv, const int* __restrict__ pi,
                            const float* __restrict__ pm, const float* __restrict__ ps, float* __restrict__ out_lp,
                            int64_t* __restrict__ out_idx, float* __restrict__ out_lse, int vocab_offset,
                            bool with_lse) {
  extern __shared__ uint8_t smem[];
  const int warps = blockDim.x >> 5;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * warps + w;
  if (row >= rows) return;
  float* vals = reinterpret_cast<float*>(smem) + (size_t)w * splits * K;
  int* idxs = reinterpret_cast<int*>(reinterpret_cast<float*>(smem) + (size_t)warps * splits * K) + (size_t)w * splits * K;
  float m = -INFINITY, s = 0.f;
  for (int q = lane; q < splits; q += 32) ms_combine(m, s, pm[(size_t)row * splits + q], ps[(size_t)row * splits + q]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o), os = __shfl_xor_sync(0xffffffffu, s, o);
    ms_combine(m, s, om, os);
  }
  for (int q = lane; q < splits * K; q += 32) {
    vals[q] = pv[(size_t)row * splits * K + q];
    idxs[q] = pi[(size_t)row * splits * K + q];
  }
  __syncwarp();
  __shared__ float ov[32][kTopkMaxK];
  __shared__ int oi[32][kTopkMaxK];
  warp_select<K>(vals, idxs, splits * K, ov[w], oi[w]);
  const float lse = with_lse ? m + logf(s) : 0.f;
  if (lane < k_out) {
    out_lp[(size_t)row * k_out + lane] = ov[w][lane] - lse;
    out_idx[(size_t)row * k_out + lane] = (int64_t)oi[w][lane] + vocab_offset;
  }
  if (lane == 0 && out_lse) out_lse[row] = lse;
}

template <int K>
static void run_topk(const torch::Tensor& logits, int64_t k, double temperature, torch::Tensor& lp, torch::Tensor& idx,
                     c10::optional<torch::Tensor> lse, int64_t vocab_offset, cudaStream_t stream) {
  const int R = logits.size(0), V = logits.size(1), ld = logits.stride(0);
  const int target_ctas = 148 * 4;
  int splits = std::max(1, std::min((V + 4095) / 4096, (target_ctas + R - 1) / R));
  int chunk = ((V + splits - 1) / splits + 7) / 8 * 8;
  splits = (V + chunk - 1) / chunk;
  auto opts = logits.options().dtype(at::kFloat);
  auto pv = torch::empty({R * splits * K}, opts);
  auto pi = torch::empty({R * splits * K}, opts.dtype(at::kInt));
  auto pm = torch::empty({R * splits}, opts);
  auto ps = torch::empty({R * splits}, opts);
  auto stage1 = lse ? topk_stage1<K, true> : topk_stage1<K, false>;
  stage1<<<R * splits, kTopkThreads, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), V, ld, splits, chunk, (float)temperature,
      pv.data_ptr<float>(), pi.data_ptr<int>(), pm.data_ptr<float>(), ps.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  const int warps = 4;
  const size_t smem = (size_t)warps * splits * K * 8;
  topk_stage2<K><<<(R + warps - 1) / warps, warps * 32, smem, stream>>>(
      R, splits, (int)k, pv.data_ptr<float>(), pi.data_ptr<int>(), pm.data_ptr<float>(), ps.data_ptr<float>(),
      lp.data_ptr<float>(), idx.data_ptr<int64_t>(), lse ? lse->data_ptr<float>() : nullptr, (int)vocab_offset,
      lse.has_value());
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
