// Gated DeltaNet (linear attention) kernels for hybrid models, sm_100a.
//
// Per value head the recurrent state S is [K=128, V=128] fp32. One token t:
//   q, k <- L2-normalised (eps 1e-6 inside the sqrt), q <- q * scale
//   S <- exp(g_t) S;  v' = beta_t (v - S^T k);  S <- S + k v'^T;  o = S^T q
// (the reference's per-token rule, docker/opt/kern/a2/kernels.py:85-96, with g = -exp(A_log) *
// softplus(a + dt_bias) and beta = sigmoid(b) computed by gdn_gates below).
//
// Design: one CTA per (request, value head), 256 threads; a pair of threads owns the state column S[:, j] in
// registers (64 rows each), so S^T k and S^T q are pair-local dot products (one shuffle) and the rank-1
// update is thread-local; the L2 norms of a chunk of tokens' q and k are formed up front (one warp per
// token), so the token loop has no block barrier. The state is read once per launch.
//   gdn_verify: runs a request's T verify tokens from its committed state WITHOUT writing the state;
//               writes outputs and a stash (normalised k, v', g) per token — the reference's
//               "Track B" verify (docker/opt/kern/braw/kernels.py:69-280) without per-token states.
//   gdn_fold:   commits the first n_accept[r] stashed tokens into the state (S <- exp(g) S + k v'^T),
//               the reference's fold after acceptance (braw/kernels.py:283-332).
//   gdn_prefill: verify + fold of all tokens in one pass (prompt processing), state written.
//   causal_conv1d: depthwise causal conv (W taps) + SiLU over a request's tokens, conv window
//               [W-1, C] (C contiguous: the reference's p-major layout, docker/opt/v5/cf/kopt_convp.py),
//               and the window update for the first n_commit tokens.
//   gated_rmsnorm: y = rmsnorm(o) * w * silu(z) per head group (docker/opt/v5/topkbf_normcfg/normcfg).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace phx {

constexpr int kGdnK = 128;
constexpr int kGdnV = 128;

// q, k, v: [T, H*, 128] bf16 (rows = tokens of the batch); g, beta: [T, HV] fp32; state: [slots, HV, K, V] fp32
// (K-major rows: state[slot][h][i][j]). tok_start [R+1]; slot[R] = state slot of request r.
// GQA: value head h uses q/k head h / (HV / HK).
// 256 threads: the pair of threads (2j, 2j + 1) owns state column j, each half of its 128 rows in registers
// (64 floats), and the pair adds its two partial dot products with one shuffle; each dot product keeps four
// independent accumulators (one chain of 64 dependent FMAs would leave the schedulers waiting on FMA
// latency). Tokens are taken in chunks of kGdnChunk: the 8 warps first normalise the chunk's q and k rows into
// shared memory (one warp per token, warp-shuffle norms) with its decays and betas, then every thread runs the
// chunk's tokens back to back with no block barrier inside the chunk. Column j's update only reads column j.
constexpr int kGdnChunk = 16;
constexpr int kGdnHalf = kGdnK / 2;
constexpr int kGdnRowPad = kGdnK + 8;   // half 1 of a row starts 4 floats past 64: the two halves' float4 reads
                                        // of one step land in different banks
template <bool WRITE_STATE, bool STASH>
__global__ void __launch_bounds__(256) gdn_recurrent_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v,
    const float* __restrict__ g, const float* __restrict__ beta, float* __restrict__ state,
    const int* __restrict__ tok_start, const int* __restrict__ slot, int HK, int HV, float scale,
    __nv_bfloat16* __restrict__ out, float* __restrict__ st_k, float* __restrict__ st_v, float* __restrict__ st_g) {
  __shared__ __align__(16) float sq[kGdnChunk][kGdnRowPad], sk[kGdnChunk][kGdnRowPad];
  __shared__ float sdec[kGdnChunk], sbeta[kGdnChunk];
  const int r = blockIdx.x, h = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int j = tid >> 1, half = tid & 1;
  const int hk = h / (HV / HK);
  const int t0 = tok_start[r], t1 = tok_start[r + 1];
  float* S = state + ((size_t)slot[r] * HV + h) * kGdnK * kGdnV;
  float col[kGdnHalf];
#pragma unroll
  for (int i = 0; i < kGdnHalf; ++i) col[i] = S[(size_t)(half * kGdnHalf + i) * kGdnV + j];
  const int hoff = half * (kGdnHalf + 4);    // this thread's half inside a padded shared row
  for (int c0 = t0; c0 < t1; c0 += kGdnChunk) {
    const int n = min(kGdnChunk, t1 - c0);
    // ---- normalise the chunk's q and k rows (warp w: tokens w, w + 8) ----
    for (int u = warp; u < n; u += 8) {
      const int t = c0 + u;
      float qv[4], kv4[4], sqq = 0.f, skk = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = lane + 32 * e;
        qv[e] = __bfloat162float(q[((size_t)t * HK + hk) * kGdnK + i]);
        kv4[e] = __bfloat162float(k[((size_t)t * HK + hk) * kGdnK + i]);
        sqq += qv[e] * qv[e];
        skk += kv4[e] * kv4[e];
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        sqq += __shfl_xor_sync(0xffffffffu, sqq, o);
        skk += __shfl_xor_sync(0xffffffffu, skk, o);
      }
      const float qn = rsqrtf(sqq + 1e-6f) * scale, kn = rsqrtf(skk + 1e-6f);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = lane + 32 * e;
        const int pi = i < kGdnHalf ? i : i + 4;
        sq[u][pi] = qv[e] * qn;
        sk[u][pi] = kv4[e] * kn;
        if (STASH) st_k[((size_t)t * HV + h) * kGdnK + i] = kv4[e] * kn;
      }
      if (lane == 0) {
        const float gt = g[(size_t)t * HV + h];
        sdec[u] = expf(gt);
        sbeta[u] = beta[(size_t)t * HV + h];
        if (STASH) st_g[(size_t)t * HV + h] = gt;
      }
    }
    __syncthreads();
    // ---- the chunk's tokens: decay, S^T k, delta-rule update, S^T q ----
    for (int u = 0; u < n; ++u) {
      const int t = c0 + u;
      const float vj = __bfloat162float(v[((size_t)t * HV + h) * kGdnV + j]);
      const float decay = sdec[u];
      const float4* k4 = reinterpret_cast<const float4*>(&sk[u][hoff]);
      const float4* q4 = reinterpret_cast<const float4*>(&sq[u][hoff]);
      float4 a4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int i = 0; i < kGdnHalf / 4; ++i) {
        const float4 kk = k4[i];
        col[4 * i] *= decay;
        col[4 * i + 1] *= decay;
        col[4 * i + 2] *= decay;
        col[4 * i + 3] *= decay;
        a4.x = fmaf(col[4 * i], kk.x, a4.x);
        a4.y = fmaf(col[4 * i + 1], kk.y, a4.y);
        a4.z = fmaf(col[4 * i + 2], kk.z, a4.z);
        a4.w = fmaf(col[4 * i + 3], kk.w, a4.w);
      }
      float kv = (a4.x + a4.y) + (a4.z + a4.w);
      kv += __shfl_xor_sync(0xffffffffu, kv, 1);
      const float vp = (vj - kv) * sbeta[u];
      float4 o4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int i = 0; i < kGdnHalf / 4; ++i) {
        const float4 kk = k4[i], qq = q4[i];
        col[4 * i] = fmaf(kk.x, vp, col[4 * i]);
        col[4 * i + 1] = fmaf(kk.y, vp, col[4 * i + 1]);
        col[4 * i + 2] = fmaf(kk.z, vp, col[4 * i + 2]);
        col[4 * i + 3] = fmaf(kk.w, vp, col[4 * i + 3]);
        o4.x = fmaf(col[4 * i], qq.x, o4.x);
        o4.y = fmaf(col[4 * i + 1], qq.y, o4.y);
        o4.z = fmaf(col[4 * i + 2], qq.z, o4.z);
        o4.w = fmaf(col[4 * i + 3], qq.w, o4.w);
      }
      float o = (o4.x + o4.y) + (o4.z + o4.w);
      o += __shfl_xor_sync(0xffffffffu, o, 1);
      if (half == 0) {
        out[((size_t)t * HV + h) * kGdnV + j] = __float2bfloat16(o);
        if (STASH) st_v[((size_t)t * HV + h) * kGdnV + j] = vp;
      }
    }
    __syncthreads();   // the next chunk rewrites the shared rows
  }
  if (WRITE_STATE) {
#pragma unroll
    for (int i = 0; i < kGdnHalf; ++i) S[(size_t)(half * kGdnHalf + i) * kGdnV + j] = col[i];
  }
}

// commit the first n_accept[r] stashed tokens of request r into its state
__global__ void __launch_bounds__(128) gdn_fold_kernel(float* __restrict__ state, const int* __restrict__ tok_start,
                                                       const int* __restrict__ slot, const int* __restrict__ n_accept,
                                                       int HV, const float* __restrict__ st_k,
                                                       const float* __restrict__ st_v, const float* __restrict__ st_g) {
  __shared__ float sk[kGdnK];
  const int r = blockIdx.x, h = blockIdx.y, j = threadIdx.x;
  const int n = n_accept[r];
  if (n <= 0) return;
  const int t0 = tok_start[r];
  float* S = state + ((size_t)slot[r] * HV + h) * kGdnK * kGdnV;
  float col[kGdnK];
#pragma unroll
  for (int i = 0; i < kGdnK; ++i) col[i] = S[(size_t)i * kGdnV + j];
  for (int t = t0; t < t0 + n; ++t) {
    sk[j] = st_k[((size_t)t * HV + h) * kGdnK + j];
    __syncthreads();
    const float decay = expf(st_g[(size_t)t * HV + h]);
    const float vp = st_v[((size_t)t * HV + h) * kGdnV + j];
#pragma unroll
    for (int i = 0; i < kGdnK; ++i) col[i] = fmaf(sk[i], vp, col[i] * decay);
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < kGdnK; ++i) S[(size_t)i * kGdnV + j] = col[i];
}

// g = -exp(A_log[h]) * softplus(a + dt_bias[h]) (softplus linear above 20), beta = sigmoid(b)
__global__ void gdn_gates_kernel(const __nv_bfloat16* __restrict__ a, const __nv_bfloat16* __restrict__ b,
                                 const float* __restrict__ A_log, const float* __restrict__ dt_bias, int T, int HV,
                                 float* __restrict__ g, float* __restrict__ beta) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= T * HV) return;
  const int h = i % HV;
  const float x = __bfloat162float(a[i]) + dt_bias[h];
  const float sp = x > 20.f ? x : log1pf(expf(x));
  g[i] = -expf(A_log[h]) * sp;
  beta[i] = 1.f / (1.f + expf(-__bfloat162float(b[i])));
}

// x [T, C] bf16; window [slots, W-1, C] bf16 (oldest first); w [C, W]; bias [C] or null.
// y[t] = silu(bias + sum_j w[c][j] * seq[t + j]) where seq = window ++ x of the request.
// The window is updated with the first n_commit[r] tokens (all tokens when n_commit is null).
__global__ void causal_conv1d_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ window,
                                     const __nv_bfloat16* __restrict__ w, const __nv_bfloat16* __restrict__ bias,
                                     const int* __restrict__ tok_start, const int* __restrict__ slot,
                                     const int* __restrict__ n_commit, int C, int W, __nv_bfloat16* __restrict__ y) {
  const int r = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const int t0 = tok_start[r], t1 = tok_start[r + 1];
  __nv_bfloat16* win = window + (size_t)slot[r] * (W - 1) * C;
  float hist[8];
  for (int j = 0; j < W - 1; ++j) hist[j] = __bfloat162float(win[(size_t)j * C + c]);
  float wt[8];
  for (int j = 0; j < W; ++j) wt[j] = __bfloat162float(w[(size_t)c * W + j]);
  const float bb = bias ? __bfloat162float(bias[c]) : 0.f;
  const int ncommit = n_commit ? n_commit[r] : (t1 - t0);
  float keep[8];
  for (int j = 0; j < W - 1; ++j) keep[j] = hist[j];
  for (int t = t0; t < t1; ++t) {
    const float xt = __bfloat162float(x[(size_t)t * C + c]);
    float acc = bb;
    for (int j = 0; j < W - 1; ++j) acc = fmaf(wt[j], hist[j], acc);
    acc = fmaf(wt[W - 1], xt, acc);
    y[(size_t)t * C + c] = __float2bfloat16(acc / (1.f + expf(-acc)));
    for (int j = 0; j < W - 2; ++j) hist[j] = hist[j + 1];
    hist[W - 2] = xt;
    if (t - t0 + 1 == ncommit)
      for (int j = 0; j < W - 1; ++j) keep[j] = hist[j];
  }
  for (int j = 0; j < W - 1; ++j) win[(size_t)j * C + c] = __float2bfloat16(keep[j]);
}

// y = rmsnorm(o) * w * silu(z) over groups of D channels (one warp per (token, head))
__global__ void gated_rmsnorm_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ z,
                                     const __nv_bfloat16* __restrict__ w, int rows, int D, float eps,
                                     __nv_bfloat16* __restrict__ y) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const __nv_bfloat16* op = o + (size_t)row * D;
  float ss = 0.f;
  for (int d = lane; d < D; d += 32) {
    const float x = __bfloat162float(op[d]);
    ss += x * x;
  }
#pragma unroll
  for (int s = 16; s > 0; s >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, s);
  const float inv = rsqrtf(ss / D + eps);
  for (int d = lane; d < D; d += 32) {
    const float zz = __bfloat162float(z[(size_t)row * D + d]);
    const float val = __bfloat162float(op[d]) * inv * __bfloat162float(w[d]) * (zz / (1.f + expf(-zz)));
    y[(size_t)row * D + d] = __float2bfloat16(val);
  }
}

// ------------------------------------------------------------------------------------------------
void gdn_recurrent(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor g, torch::Tensor beta,
                   torch::Tensor state, torch::Tensor tok_start, torch::Tensor slot, double scale, torch::Tensor out,
                   bool write_state, c10::optional<torch::Tensor> st_k, c10::optional<torch::Tensor> st_v,
                   c10::optional<torch::Tensor> st_g) {
  TORCH_CHECK(q.size(-1) == kGdnK && v.size(-1) == kGdnV && state.size(-1) == kGdnV && state.size(-2) == kGdnK);
  TORCH_CHECK(state.scalar_type() == at::kFloat && g.scalar_type() == at::kFloat);
  const int R = tok_start.size(0) - 1, HK = q.size(1), HV = v.size(1);
  TORCH_CHECK(HV % HK == 0);
  if (R == 0) return;
  const at::cuda::CUDAGuard guard(q.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  auto P = [](const torch::Tensor& t) { return reinterpret_cast<const __nv_bfloat16*>(t.data_ptr()); };
  dim3 grid(R, HV);
  const bool stash = st_k.has_value();
  float* sk = stash ? st_k->data_ptr<float>() : nullptr;
  float* sv = stash ? st_v->data_ptr<float>() : nullptr;
  float* sg = stash ? st_g->data_ptr<float>() : nullptr;
  auto o = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  if (write_state && stash)
    gdn_recurrent_kernel<true, true><<<grid, 256, 0, stream>>>(P(q), P(k), P(v), g.data_ptr<float>(), beta.data_ptr<float>(),
        state.data_ptr<float>(), tok_start.data_ptr<int>(), slot.data_ptr<int>(), HK, HV, (float)scale, o, sk, sv, sg);
  else if (write_state)
    gdn_recurrent_kernel<true, false><<<grid, 256, 0, stream>>>(P(q), P(k), P(v), g.data_ptr<float>(), beta.data_ptr<float>(),
        state.data_ptr<float>(), tok_start.data_ptr<int>(), slot.data_ptr<int>(), HK, HV, (float)scale, o, sk, sv, sg);
  else
    gdn_recurrent_kernel<false, true><<<grid, 256, 0, stream>>>(P(q), P(k), P(v), g.data_ptr<float>(), beta.data_ptr<float>(),
        state.data_ptr<float>(), tok_start.data_ptr<int>(), slot.data_ptr<int>(), HK, HV, (float)scale, o, sk, sv, sg);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gdn_fold(torch::Tensor state, torch::Tensor tok_start, torch::Tensor slot, torch::Tensor n_accept,
              torch::Tensor st_k, torch::Tensor st_v, torch::Tensor st_g) {
  const int R = tok_start.size(0) - 1, HV = state.size(1);
  if (R == 0) return;
  const at::cuda::CUDAGuard guard(state.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  gdn_fold_kernel<<<dim3(R, HV), 128, 0, stream>>>(state.data_ptr<float>(), tok_start.data_ptr<int>(),
                                                   slot.data_ptr<int>(), n_accept.data_ptr<int>(), HV,
                                                   st_k.data_ptr<float>(), st_v.data_ptr<float>(), st_g.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gdn_gates(torch::Tensor a, torch::Tensor b, torch::Tensor A_log, torch::Tensor dt_bias, torch::Tensor g,
               torch::Tensor beta) {
  const int T = a.size(0), HV = a.size(1);
  if (T == 0) return;
  const at::cuda::CUDAGuard guard(a.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  gdn_gates_kernel<<<(T * HV + 255) / 256, 256, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(a.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(b.data_ptr()),
      A_log.data_ptr<float>(), dt_bias.data_ptr<float>(), T, HV, g.data_ptr<float>(), beta.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void causal_conv1d(torch::Tensor x, torch::Tensor window, torch::Tensor w, c10::optional<torch::Tensor> bias,
                   torch::Tensor tok_start, torch::Tensor slot, c10::optional<torch::Tensor> n_commit, torch::Tensor y) {
  const int C = x.size(1), W = w.size(1), R = tok_start.size(0) - 1;
  TORCH_CHECK(W >= 2 && W <= 8 && window.size(1) == W - 1 && window.size(2) == C);
  if (R == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  dim3 grid((C + 127) / 128, R);
  causal_conv1d_kernel<<<grid, 128, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), reinterpret_cast<__nv_bfloat16*>(window.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
      bias ? reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr()) : nullptr, tok_start.data_ptr<int>(),
      slot.data_ptr<int>(), n_commit ? n_commit->data_ptr<int>() : nullptr, C, W,
      reinterpret_cast<__nv_bfloat16*>(y.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gated_rmsnorm(torch::Tensor o, torch::Tensor z, torch::Tensor w, double eps, torch::Tensor y) {
  const int D = w.size(0);
  const int rows = o.numel() / D;
  if (rows == 0) return;
  const at::cuda::CUDAGuard guard(o.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  gated_rmsnorm_kernel<<<(rows + 7) / 8, 256, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(o.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(z.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), rows, D, (float)eps,
      reinterpret_cast<__nv_bfloat16*>(y.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace phx
