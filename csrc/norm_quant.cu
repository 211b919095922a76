// Memory-bound fused kernels (sm_100a):
//   add_rmsnorm_quant : h <- bf16(h + delta); y = rmsnorm(h) * w; emit y as block-scaled fp8
//                       (one fp32 scale per 128 channels, stored [H/128, M]) and/or bf16.
//                       Blackwell counterpart of the reference's fused add+RMSNorm+FP8 quant
//                       (docker/opt/v5/fusedq/gemma_quant.cuh:38-167, which quantizes per token).
//   silu_mul_quant    : a = bf16(silu(g) * u) from gu = [g | u]; emit a as block-scaled fp8.
//                       Counterpart of docker/opt/v5/fusedq/silu_quant.cuh:28-79 (per-token there).
//   act_quant         : bf16 [M, K] -> block-scaled fp8.
//   rope_kv_write     : rotate-half RoPE of q and k from the fused qkv projection, q to a packed
//                       [M, Hq, D] buffer, k and v into the paged cache [pages, Hkv, page, D].
// Scale = the smallest power of two >= amax / 448 per 128-block (1 for an all-zero block); q = v * (1 / scale),
// saturating to e4m3 (a power-of-two scale is exact in UE8M0, the scale format of the hardware-scaled GEMM).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace phx {

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  __syncthreads();
  const int nw = blockDim.x >> 5;
  float t = l < nw ? red[l] : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  __syncthreads();
  return t;
}

// amax over the 16 lanes of a half-warp holding one 128-element block (8 values per lane)
__device__ __forceinline__ float halfwarp_max(float v) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Called by all 32 lanes of a warp (the shuffles span the half-warp); lanes with valid == false
// contribute nothing and store nothing.
__device__ __forceinline__ void quant_store8(const float (&y)[8], int chunk, int row, int M, uint8_t* q, float* qs,
                                             int ld_q, bool valid = true) {
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(y[j]));
  amax = halfwarp_max(amax);
  if (!valid) return;
  float inv;
  const float scale = fp8_block_scale(amax, &inv);
  uint2 pk;
  pk.x = pack_fp8x4(y[0] * inv, y[1] * inv, y[2] * inv, y[3] * inv);
  pk.y = pack_fp8x4(y[4] * inv, y[5] * inv, y[6] * inv, y[7] * inv);
  *reinterpret_cast<uint2*>(q + (size_t)row * ld_q + chunk * 8) = pk;
  if ((chunk & 15) == 0) qs[(size_t)(chunk >> 4) * M + row] = scale;
}

// one CTA per row; thread t owns 8-element chunks t, t + blockDim, ...
template <int MAXC>
__global__ void add_rmsnorm_quant_kernel(__nv_bfloat16* __restrict__ h, const __nv_bfloat16* __restrict__ delta,
                                         const __nv_bfloat16* __restrict__ w, float eps, int H, int M,
                                         uint8_t* __restrict__ q, float* __restrict__ qs,
                                         __nv_bfloat16* __restrict__ out) {
  __shared__ float red[32];
  const int row = blockIdx.x;
  const int nch = H / 8;
  float x[MAXC][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    if (c < nch) {
      uint4 hv = *reinterpret_cast<const uint4*>(h + (size_t)row * H + c * 8);
      uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w};
      if (delta) {
        uint4 dv = *reinterpret_cast<const uint4*>(delta + (size_t)row * H + c * 8);
        uint32_t dw[4] = {dv.x, dv.y, dv.z, dv.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float2 a = unpack_bf16x2(hw[j]), b = unpack_bf16x2(dw[j]);
          hw[j] = pack_bf16x2(a.x + b.x, a.y + b.y);
        }
        *reinterpret_cast<uint4*>(h + (size_t)row * H + c * 8) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 a = unpack_bf16x2(hw[j]);
        x[i][2 * j] = a.x;
        x[i][2 * j + 1] = a.y;
        ss += a.x * a.x + a.y * a.y;
      }
    }
  }
  const float inv = rsqrtf(block_sum(ss, red) / (float)H + eps);
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    const bool valid = c < nch;
    float y[8];
    if (valid) {
      uint4 wv = *reinterpret_cast<const uint4*>(w + c * 8);
      uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 a = unpack_bf16x2(ww[j]);
        y[2 * j] = x[i][2 * j] * inv * a.x;
        y[2 * j + 1] = x[i][2 * j + 1] * inv * a.y;
      }
      if (out) {
        *reinterpret_cast<uint4*>(out + (size_t)row * H + c * 8) =
            make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]), pack_bf16x2(y[4], y[5]),
                       pack_bf16x2(y[6], y[7]));
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) y[j] = 0.f;
    }
    // warp-uniform: every warp with at least one valid lane runs the quant together
    if (q && __any_sync(0xffffffffu, valid)) quant_store8(y, c, row, M, q, qs, H, valid);
  }
}

// gu [M, 2F] -> a = bf16(silu(g) * u) -> fp8 [M, F] + scales [F/128, M]. One half-warp per 128-block.
__global__ void silu_mul_quant_kernel(const __nv_bfloat16* __restrict__ gu, int F, int M, int ld_gu,
                                      uint8_t* __restrict__ q, float* __restrict__ qs,
                                      __nv_bfloat16* __restrict__ out) {
  const int nblk = F / 128;
  const int warps_per_cta = blockDim.x / 32;
  const int sub = threadIdx.x & 15;
  const long total = (long)M * nblk;
  for (long wj = (long)blockIdx.x * warps_per_cta + threadIdx.x / 32; 2 * wj < total;
       wj += (long)gridDim.x * warps_per_cta) {
    const long job = 2 * wj + ((threadIdx.x >> 4) & 1);
    const bool valid = job < total;
    const int row = valid ? job / nblk : 0, blk = valid ? job % nblk : 0;
    const int chunk = blk * 16 + sub;
    float y[8];
    if (valid) {
      const __nv_bfloat16* gp = gu + (size_t)row * ld_gu + chunk * 8;
      uint4 gv = *reinterpret_cast<const uint4*>(gp);
      uint4 uv = *reinterpret_cast<const uint4*>(gp + F);
      uint32_t g4[4] = {gv.x, gv.y, gv.z, gv.w}, u4[4] = {uv.x, uv.y, uv.z, uv.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 g = unpack_bf16x2(g4[j]), u = unpack_bf16x2(u4[j]);
        float2 a = unpack_bf16x2(pack_bf16x2(g.x / (1.f + expf(-g.x)) * u.x, g.y / (1.f + expf(-g.y)) * u.y));
        y[2 * j] = a.x;
        y[2 * j + 1] = a.y;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) y[j] = 0.f;
    }
    if (out && valid) {
      *reinterpret_cast<uint4*>(out + (size_t)row * F + chunk * 8) =
          make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]), pack_bf16x2(y[4], y[5]),
                     pack_bf16x2(y[6], y[7]));
    }
    if (q) quant_store8(y, chunk, row, M, q, qs, F, valid);
  }
}

__global__ void act_quant_kernel(const __nv_bfloat16* __restrict__ x, int K, int M, int ld_x, uint8_t* __restrict__ q,
                                 float* __restrict__ qs) {
  const int nblk = K / 128;
  const int warps_per_cta = blockDim.x / 32;
  const int sub = threadIdx.x & 15;
  const long total = (long)M * nblk;
  for (long wj = (long)blockIdx.x * warps_per_cta + threadIdx.x / 32; 2 * wj < total;
       wj += (long)gridDim.x * warps_per_cta) {
    const long job = 2 * wj + ((threadIdx.x >> 4) & 1);
    const bool valid = job < total;
    const int row = valid ? job / nblk : 0, blk = valid ? job % nblk : 0;
    const int chunk = blk * 16 + sub;
    float y[8];
    if (valid) {
      uint4 v = *reinterpret_cast<const uint4*>(x + (size_t)row * ld_x + chunk * 8);
      uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 a = unpack_bf16x2(w4[j]);
        y[2 * j] = a.x;
        y[2 * j + 1] = a.y;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) y[j] = 0.f;
    }
    quant_store8(y, chunk, row, M, q, qs, K, valid);
  }
}

// qkv [M, (Hq + 2 Hkv) * D]; cos_sin [max_pos, D/2] float2; one warp per (token, head); D = 128 or 64.
__global__ void rope_kv_write_kernel(const __nv_bfloat16* __restrict__ qkv, int ld_qkv, const int* __restrict__ pos,
                                     const int64_t* __restrict__ slots, const float2* __restrict__ cos_sin,
                                     __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ k_cache,
                                     __nv_bfloat16* __restrict__ v_cache, int M, int Hq, int Hkv, int D,
                                     int page_size) {
  const int warps = blockDim.x >> 5;
  const int head = blockIdx.x * warps + (threadIdx.x >> 5);
  const int tok = blockIdx.y;
  const int lane = threadIdx.x & 31;
  const int nh = Hq + 2 * Hkv;
  if (head >= nh || tok >= M) return;
  const __nv_bfloat16* src = qkv + (size_t)tok * ld_qkv + (size_t)head * D;
  const int half = D / 2;
  const int p = pos[tok];
  const int64_t slot = slots ? slots[tok] : -1;
  __nv_bfloat16* dst;
  if (head < Hq) {
    dst = q_out + ((size_t)tok * Hq + head) * D;
  } else {
    if (slot < 0) return;
    const int kvh = head < Hq + Hkv ? head - Hq : head - Hq - Hkv;
    const int64_t page = slot / page_size, off = slot % page_size;
    __nv_bfloat16* base = head < Hq + Hkv ? k_cache : v_cache;
    dst = base + ((page * Hkv + kvh) * page_size + off) * D;
  }
  if (head >= Hq + Hkv) {  // v: plain copy
    for (int d = lane * 2; d < D; d += 64)
      *reinterpret_cast<uint32_t*>(dst + d) = *reinterpret_cast<const uint32_t*>(src + d);
    return;
  }
  for (int d = lane * 2; d < half; d += 64) {
    float2 x1 = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(src + d));
    float2 x2 = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(src + d + half));
    float2 cs0 = cos_sin[(size_t)p * half + d];
    float2 cs1 = cos_sin[(size_t)p * half + d + 1];
    float o1a = x1.x * cs0.x - x2.x * cs0.y, o1b = x1.y * cs1.x - x2.y * cs1.y;
    float o2a = x2.x * cs0.x + x1.x * cs0.y, o2b = x2.y * cs1.x + x1.y * cs1.y;
    *reinterpret_cast<uint32_t*>(dst + d) = pack_bf16x2(o1a, o1b);
    *reinterpret_cast<uint32_t*>(dst + d + half) = pack_bf16x2(o2a, o2b);
  }
}

// Wide variant (the hot path): two heads per warp (16 lanes each), four rotary pairs per lane with 8-byte q/k
// loads and 16-byte float4 cos/sin loads, v copied in 16-byte chunks, 32-bit slot arithmetic. The per-element
// arithmetic is the narrow kernel's, so the outputs are identical; the host checks the alignment it needs
// (D % 8 == 0, 16-byte-aligned rows) and otherwise launches the narrow kernel.
__global__ void rope_kv_write_wide_kernel(const __nv_bfloat16* __restrict__ qkv, int ld_qkv, const int* __restrict__ pos,
                                          const int64_t* __restrict__ slots, const float2* __restrict__ cos_sin,
                                          __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ k_cache,
                                          __nv_bfloat16* __restrict__ v_cache, int M, int Hq, int Hkv, int D,
                                          int page_size) {
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31, l16 = lane & 15;
  const int head = (blockIdx.x * warps + (threadIdx.x >> 5)) * 2 + (lane >> 4);
  const int tok = blockIdx.y;
  const int nh = Hq + 2 * Hkv;
  if (head >= nh || tok >= M) return;
  const __nv_bfloat16* src = qkv + (size_t)tok * ld_qkv + (size_t)head * D;
  const int half = D / 2;
  __nv_bfloat16* dst;
  if (head < Hq) {
    dst = q_out + ((size_t)tok * Hq + head) * D;
  } else {
    const int64_t slot = slots ? slots[tok] : -1;
    if (slot < 0) return;
    const int s = static_cast<int>(slot);                  // pool slots fit in 31 bits (host check)
    const int kvh = head < Hq + Hkv ? head - Hq : head - Hq - Hkv;
    const int page = s / page_size, off = s - page * page_size;
    __nv_bfloat16* base = head < Hq + Hkv ? k_cache : v_cache;
    dst = base + (((size_t)page * Hkv + kvh) * page_size + off) * D;
  }
  if (head >= Hq + Hkv) {  // v: plain copy
    for (int d = l16 * 8; d < D; d += 128)
      *reinterpret_cast<uint4*>(dst + d) = *reinterpret_cast<const uint4*>(src + d);
    return;
  }
  const float2* cs = cos_sin + (size_t)pos[tok] * half;
  for (int d = l16 * 4; d < half; d += 64) {
    const uint2 a = *reinterpret_cast<const uint2*>(src + d);
    const uint2 b = *reinterpret_cast<const uint2*>(src + d + half);
    const float4 c01 = *reinterpret_cast<const float4*>(cs + d);       // (cos, sin) of d and d + 1
    const float4 c23 = *reinterpret_cast<const float4*>(cs + d + 2);   // (cos, sin) of d + 2 and d + 3
    const float2 x1a = unpack_bf16x2(a.x), x1b = unpack_bf16x2(a.y);
    const float2 x2a = unpack_bf16x2(b.x), x2b = unpack_bf16x2(b.y);
    uint2 o1, o2;
    o1.x = pack_bf16x2(x1a.x * c01.x - x2a.x * c01.y, x1a.y * c01.z - x2a.y * c01.w);
    o1.y = pack_bf16x2(x1b.x * c23.x - x2b.x * c23.y, x1b.y * c23.z - x2b.y * c23.w);
    o2.x = pack_bf16x2(x2a.x * c01.x + x1a.x * c01.y, x2a.y * c01.z + x1a.y * c01.w);
    o2.y = pack_bf16x2(x2b.x * c23.x + x1b.x * c23.y, x2b.y * c23.z + x1b.y * c23.w);
    *reinterpret_cast<uint2*>(dst + d) = o1;
    *reinterpret_cast<uint2*>(dst + d + half) = o2;
  }
}

// ------------------------------------------------------------------------------------------------
// host wrappers
// ------------------------------------------------------------------------------------------------
// one CTA per row: up to 512 threads, so a thread holds at most two 8-element chunks of an 8192-wide row (more
// resident CTAs per SM than 256 threads x four chunks, whose registers limited occupancy to half the warps)
static int norm_threads(int H) {
  int nch = H / 8;
  int t = nch >= 512 ? 512 : nch >= 256 ? 256 : ((nch + 15) / 16) * 16;
  return std::max(32, ((t + 31) / 32) * 32);
}

void add_rmsnorm_quant(torch::Tensor h, c10::optional<torch::Tensor> delta, torch::Tensor w, double eps,
                       c10::optional<torch::Tensor> q, c10::optional<torch::Tensor> qs,
                       c10::optional<torch::Tensor> out) {
  TORCH_CHECK(h.is_cuda() && h.scalar_type() == at::kBFloat16 && h.is_contiguous());
  const int M = h.size(0), H = h.size(1);
  TORCH_CHECK(H % 8 == 0);
  if (q) TORCH_CHECK(H % 128 == 0 && q->scalar_type() == at::kFloat8_e4m3fn && qs->size(0) == H / 128 &&
                     qs->size(1) == M);
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(h.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const int threads = norm_threads(H);
  const int maxc = (H / 8 + threads - 1) / threads;
  auto hp = reinterpret_cast<__nv_bfloat16*>(h.data_ptr());
  auto dp = delta ? reinterpret_cast<const __nv_bfloat16*>(delta->data_ptr()) : nullptr;
  auto wp = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  auto qp = q ? reinterpret_cast<uint8_t*>(q->data_ptr()) : nullptr;
  auto sp = qs ? qs->data_ptr<float>() : nullptr;
  auto op = out ? reinterpret_cast<__nv_bfloat16*>(out->data_ptr()) : nullptr;
#define LAUNCH(C) add_rmsnorm_quant_kernel<C><<<M, threads, 0, stream>>>(hp, dp, wp, (float)eps, H, M, qp, sp, op)
  if (maxc <= 1) LAUNCH(1);
  else if (maxc <= 2) LAUNCH(2);
  else if (maxc <= 4) LAUNCH(4);
  else if (maxc <= 8) LAUNCH(8);
  else TORCH_CHECK(false, "hidden size too large");
#undef LAUNCH
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void silu_mul_quant(torch::Tensor gu, c10::optional<torch::Tensor> q, c10::optional<torch::Tensor> qs,
                    c10::optional<torch::Tensor> out) {
  TORCH_CHECK(gu.scalar_type() == at::kBFloat16 && gu.stride(1) == 1);
  const int M = gu.size(0), F = gu.size(1) / 2;
  TORCH_CHECK(F % 128 == 0);
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(gu.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const long jobs = (long)M * (F / 128);
  const int threads = 256;
  const int grid = (int)std::min<long>((jobs + 15) / 16, 148L * 16);  // 16 jobs per 256-thread CTA pass
  silu_mul_quant_kernel<<<grid, threads, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()), F, M, (int)gu.stride(0),
      q ? reinterpret_cast<uint8_t*>(q->data_ptr()) : nullptr, qs ? qs->data_ptr<float>() : nullptr,
      out ? reinterpret_cast<__nv_bfloat16*>(out->data_ptr()) : nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void act_quant(torch::Tensor x, torch::Tensor q, torch::Tensor qs) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.stride(1) == 1);
  const int M = x.size(0), K = x.size(1);
  TORCH_CHECK(K % 128 == 0);
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const long jobs = (long)M * (K / 128);
  const int grid = (int)std::min<long>((jobs + 15) / 16, 148L * 16);  // 16 jobs per 256-thread CTA pass
  act_quant_kernel<<<grid, 256, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), K, M,
                                             (int)x.stride(0), reinterpret_cast<uint8_t*>(q.data_ptr()),
                                             qs.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void rope_kv_write(torch::Tensor qkv, torch::Tensor pos, c10::optional<torch::Tensor> slots, torch::Tensor cos_sin,
                   torch::Tensor q_out, c10::optional<torch::Tensor> k_cache, c10::optional<torch::Tensor> v_cache,
                   int64_t Hq, int64_t Hkv, int64_t D, int64_t page_size) {
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16 && qkv.stride(1) == 1);
  TORCH_CHECK(pos.scalar_type() == at::kInt && cos_sin.scalar_type() == at::kFloat);
  TORCH_CHECK(D % 4 == 0 && D <= 256);
  const int M = qkv.size(0);
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(qkv.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const int nh = Hq + 2 * Hkv;
  const int warps = 8;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  const bool wide = D % 8 == 0 && qkv.stride(0) % 8 == 0 && al16(qkv.data_ptr()) && al16(q_out.data_ptr()) &&
                    cos_sin.is_contiguous() && al16(cos_sin.data_ptr()) &&
                    (!k_cache || (al16(k_cache->data_ptr()) && k_cache->size(0) * page_size < (1LL << 31))) &&
                    (!v_cache || al16(v_cache->data_ptr()));
  if (wide) {
    dim3 grid((nh + 2 * warps - 1) / (2 * warps), M);
    rope_kv_write_wide_kernel<<<grid, warps * 32, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), (int)qkv.stride(0), pos.data_ptr<int>(),
        slots ? slots->data_ptr<int64_t>() : nullptr, reinterpret_cast<const float2*>(cos_sin.data_ptr()),
        reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr()),
        k_cache ? reinterpret_cast<__nv_bfloat16*>(k_cache->data_ptr()) : nullptr,
        v_cache ? reinterpret_cast<__nv_bfloat16*>(v_cache->data_ptr()) : nullptr, M, (int)Hq, (int)Hkv, (int)D,
        (int)page_size);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  dim3 grid((nh + warps - 1) / warps, M);
  rope_kv_write_kernel<<<grid, warps * 32, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), (int)qkv.stride(0), pos.data_ptr<int>(),
      slots ? slots->data_ptr<int64_t>() : nullptr, reinterpret_cast<const float2*>(cos_sin.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr()),
      k_cache ? reinterpret_cast<__nv_bfloat16*>(k_cache->data_ptr()) : nullptr,
      v_cache ? reinterpret_cast<__nv_bfloat16*>(v_cache->data_ptr()) : nullptr, M, (int)Hq, (int)Hkv, (int)D,
      (int)page_size);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace phx
