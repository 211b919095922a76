// Mixture-of-experts combine (sm_100a).
//
// The expert-parallel MoE block (models/mixtral.py) runs the local experts' grouped GEMMs over the
// (token, slot) assignments sorted by expert. The combine turns the expert rows back into per-token
// outputs:
//   out[t, :] = sum_j local[t, j] * w[t, j] * y[pos[t, j], :]       (fp32 accumulate, bf16 out)
// where pos[t, j] is the permuted row of assignment (t, j). One CTA per token, 16-byte chunks per thread;
// non-local slots are skipped (their y row is never read, so rows the grouped GEMM did not write cannot
// leak). `out` may have a row stride (the fused tensor-parallel reduction's partial buffer), so the result
// lands where the cross-rank reduction reads it without another copy.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace phx {

template <int MAXK>
__global__ void moe_combine_kernel(const __nv_bfloat16* __restrict__ y, const int64_t* __restrict__ pos,
                                   const float* __restrict__ w, const bool* __restrict__ local, int K, int H,
                                   __nv_bfloat16* __restrict__ out, int ld_out) {
  const int t = blockIdx.x;
  int rows[MAXK];
  float ws[MAXK];
  bool ok[MAXK];
#pragma unroll
  for (int j = 0; j < MAXK; ++j) {
    ok[j] = j < K && local[(size_t)t * K + j];
    rows[j] = ok[j] ? static_cast<int>(pos[(size_t)t * K + j]) : 0;
    ws[j] = ok[j] ? w[(size_t)t * K + j] : 0.f;
  }
  for (int c = threadIdx.x; c < H / 8; c += blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    // every slot's row chunk is requested before any is used (the loads overlap); same summation order
    uint4 vr[MAXK];
#pragma unroll
    for (int j = 0; j < MAXK; ++j)
      vr[j] = ok[j] ? *reinterpret_cast<const uint4*>(y + (size_t)rows[j] * H + c * 8) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int j = 0; j < MAXK; ++j) {
      if (ok[j]) {
        const uint4 v = vr[j];
        const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = unpack_bf16x2(vv[e]);
          acc[2 * e] += ws[j] * f.x;
          acc[2 * e + 1] += ws[j] * f.y;
        }
      }
    }
    *reinterpret_cast<uint4*>(out + (size_t)t * ld_out + c * 8) =
        make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]), pack_bf16x2(acc[4], acc[5]),
                   pack_bf16x2(acc[6], acc[7]));
  }
}

void moe_combine(torch::Tensor y, torch::Tensor pos, torch::Tensor w, torch::Tensor local, torch::Tensor out) {
  TORCH_CHECK(y.is_cuda() && y.scalar_type() == at::kBFloat16 && y.is_contiguous());
  TORCH_CHECK(pos.scalar_type() == at::kLong && pos.is_contiguous() && pos.dim() == 2);
  TORCH_CHECK(w.scalar_type() == at::kFloat && w.is_contiguous() && local.scalar_type() == at::kBool &&
              local.is_contiguous());
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.stride(1) == 1 && out.stride(0) % 8 == 0);
  const int T = pos.size(0), K = pos.size(1), H = y.size(1);
  TORCH_CHECK(w.size(0) == T && w.size(1) == K && local.size(0) == T && local.size(1) == K);
  TORCH_CHECK(out.size(0) == T && out.size(1) == H && H % 8 == 0 && K <= 8, "moe_combine: top-k <= 8, H % 8 == 0");
  if (T == 0) return;
  const at::cuda::CUDAGuard guard(y.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const int threads = std::min(256, std::max(32, ((H / 8 + 31) / 32) * 32));
  auto* yp = reinterpret_cast<const __nv_bfloat16*>(y.data_ptr());
  auto* op = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  if (K <= 2)
    moe_combine_kernel<2><<<T, threads, 0, stream>>>(yp, pos.data_ptr<int64_t>(), w.data_ptr<float>(),
                                                     local.data_ptr<bool>(), K, H, op, (int)out.stride(0));
  else
    moe_combine_kernel<8><<<T, threads, 0, stream>>>(yp, pos.data_ptr<int64_t>(), w.data_ptr<float>(),
                                                     local.data_ptr<bool>(), K, H, op, (int)out.stride(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace phx
