// Paged attention for prefill, decode, chain/tree verification and cascade (shared-prefix) attention.
//
// One kernel, driven by a list of work items built on the host per step:
//   item = {q0, qn, table_req, kv_lo, kv_hi, mask_req}
//     queries: tokens [q0, q0+qn) of the batch (all heads of one KV head group per CTA row tile)
//     keys:    positions [kv_lo, kv_hi) of request `table_req`'s page table
//     mask:    mask_req < 0 -> every key in range is visible (cascade prefix pass over a shared prefix);
//              else request mask_req's rule: key j is visible to its token of local index i iff
//              j < prefix_len[r] or (causal: j - prefix_len[r] <= i) or (tree: bit (j - prefix_len[r])
//              of the token's 64-bit ancestor mask).
// Grouped-query heads are packed into the row dimension (row = token * G + g, G = Hq / Hkv), so a
// 64-row CTA tile shares each K/V page across its G heads.
//
// Cascade (shared prefix + per-request suffix), the Blackwell counterpart of the reference's
// FA3-based cascade verify (docker/opt/v5/casc/kopt_casc.py:175-202): pass 1 runs one item per prefix
// group over the shared pages with all member rows as one query block and writes (O, LSE) partials;
// pass 2 runs one item per request over its private keys, seeds its online-softmax state from the
// partial (m = LSE, l = 1, acc = O), and writes the final output — the LSE merge happens in registers,
// no separate merge kernel (the reference merges with merge_state_v2, kopt_casc.py:198).
//
// Output: bf16 [T, Hq*D] and/or block-scaled fp8 (D = 128 = one scale block per (token, head); scales
// stored [Hq, T] so they feed the o_proj GEMM directly).
//
// Compute: mma.sync m16n8k16 bf16 (4 warps x 16 rows), K/V pages double-buffered with cp.async.
// Requires head_dim 128 and page size 64 (one page per key tile).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "attention_params.h"
#include "common.cuh"

namespace phx {

constexpr int kAttD = 128;
constexpr int kAttRows = 64;
constexpr int kAttKeys = 64;
constexpr float kLog2e = 1.4426950408889634f;



__device__ __forceinline__ uint32_t swz(int row, int chunk) {  // byte offset in a [rows][256B] tile
  return row * 256 + ((chunk ^ (row & 7)) << 4);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
  const int n = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__global__ void __launch_bounds__(128, 2) paged_attention_kernel(const AttnParams p) {
  extern __shared__ __align__(128) uint8_t sm[];
  uint8_t* sQ = sm;                         // 64 x 256 B
  uint8_t* sK = sm + 64 * 256;              // 2 x 64 x 256 B
  uint8_t* sV = sm + 3 * 64 * 256;          // 2 x 64 x 256 B
  const int tile = blockIdx.x;
  if (tile >= p.num_tiles) return;
  const int item = p.tile_item[tile];
  if (item < 0) return;
  const int kvh = blockIdx.y;
  const int G = p.Hq / p.Hkv;
  const int* it = p.items + item * 6;
  const int q0 = it[0], qn = it[1], treq = it[2], kv_lo = it[3], kv_hi = it[4], mreq = it[5];
  const int row0 = p.tile_row0[tile];
  const int nrows = qn * G;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int* pg = p.pages + p.page_indptr[treq];

  // ---- load Q tile ----
  for (int i = tid; i < kAttRows * 16; i += 128) {
    const int r = i >> 4, c = i & 15;
    const int pr = row0 + r;
    const bool ok = pr < nrows;
    const int tok = q0 + (ok ? pr / G : 0), head = kvh * G + (ok ? pr % G : 0);
    cp_async16(smem_u32(sQ) + swz(r, c), p.q + ((size_t)tok * p.Hq + head) * kAttD + c * 8, ok);
  }
  cp_async_commit();

  auto load_kv = [&](int kt, int buf) {
    const int k0 = kv_lo + kt * kAttKeys;
    const int page = pg[k0 / kAttKeys];
    const size_t base = ((size_t)page * p.Hkv + kvh) * kAttKeys * kAttD;
    for (int i = tid; i < kAttKeys * 16; i += 128) {
      const int r = i >> 4, c = i & 15;
      const bool ok = k0 + r < kv_hi;
      cp_async16(smem_u32(sK + buf * 64 * 256) + swz(r, c), p.kc + base + (size_t)r * kAttD + c * 8, ok);
      cp_async16(smem_u32(sV + buf * 64 * 256) + swz(r, c), p.vc + base + (size_t)r * kAttD + c * 8, ok);
    }
    cp_async_commit();
  };

  const int ntiles = (kv_hi - kv_lo + kAttKeys - 1) / kAttKeys;
  if (ntiles > 0) load_kv(0, 0);

  // ---- per-thread row bookkeeping (rows r0 = lane/4, r1 = r0 + 8 of this warp's 16) ----
  int tok_r[2], li_r[2];
  bool ok_r[2];
  uint64_t tmask[2];
  int plen = 0;
  if (mreq >= 0) plen = p.prefix_len[mreq];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int pr = row0 + warp * 16 + (lane >> 2) + 8 * h;
    ok_r[h] = pr < nrows;
    tok_r[h] = q0 + (ok_r[h] ? pr / G : 0);
    li_r[h] = mreq >= 0 ? tok_r[h] - p.q_start[mreq] : 0;
    tmask[h] = (mreq >= 0 && p.tree && !p.causal) ? p.tree[tok_r[h]] : 0ull;
  }

  float o[16][4];
  float m[2], l[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) m[h] = -INFINITY, l[h] = 0.f;
#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;

  if (p.o_in) {  // seed from the prefix pass
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int pr = row0 + warp * 16 + (lane >> 2) + 8 * h;
      if (!ok_r[h]) continue;
      const int head = kvh * G + pr % G;
      const float lse = p.lse_in[(size_t)tok_r[h] * p.Hq + head];
      if (lse == -INFINITY) continue;
      m[h] = lse * kLog2e;
      l[h] = 1.f;
      const __nv_bfloat16* src = p.o_in + ((size_t)tok_r[h] * p.Hq + head) * kAttD + 2 * (lane & 3);
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        float2 v = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(src + n * 8));
        o[n][2 * h] = v.x;
        o[n][2 * h + 1] = v.y;
      }
    }
  }

  cp_async_wait<0>();
  __syncthreads();
  // Q fragments: 8 k-steps of 16 dims
  uint32_t qf[8][4];
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const int r = warp * 16 + (lane & 15);
    const int c = kk * 2 + (lane >> 4);
    ldsm_x4(smem_u32(sQ) + swz(r, c), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
  }

  for (int kt = 0; kt < ntiles; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < ntiles) {
      load_kv(kt + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint32_t kb = smem_u32(sK + buf * 64 * 256);
    const uint32_t vb = smem_u32(sV + buf * 64 * 256);
    const int k0 = kv_lo + kt * kAttKeys;

    float s[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int kk = 0; kk < 8; kk += 2) {
        uint32_t b0, b1, b2, b3;
        const int r = nt * 8 + (lane & 7);
        const int c = kk * 2 + (lane >> 3);
        ldsm_x4(kb + swz(r, c), b0, b1, b2, b3);
        mma16816(s[nt], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b0, b1);
        mma16816(s[nt], qf[kk + 1][0], qf[kk + 1][1], qf[kk + 1][2], qf[kk + 1][3], b2, b3);
      }
    }
    // scale + mask
    const bool full_tile = (k0 + kAttKeys <= kv_hi) && (mreq < 0 || k0 + kAttKeys <= plen);
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int h = e >> 1;
        const int j = k0 + nt * 8 + 2 * (lane & 3) + (e & 1);
        float v = s[nt][e] * p.scale_log2;
        if (!full_tile) {
          bool vis = j < kv_hi && ok_r[h];
          if (vis && mreq >= 0 && j >= plen) {
            const int rel = j - plen;
            vis = p.causal ? (rel <= li_r[h]) : (rel < 64 && ((tmask[h] >> rel) & 1ull));
          }
          if (!vis) v = -INFINITY;
        }
        s[nt][e] = v;
      }
    }
    // online softmax
    float alpha[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float mx = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) mx = fmaxf(mx, fmaxf(s[nt][2 * h], s[nt][2 * h + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mn = fmaxf(m[h], mx);
      const float msafe = mn == -INFINITY ? 0.f : mn;
      alpha[h] = exp2f(m[h] - msafe);
      m[h] = mn;
      float sum = 0.f;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        s[nt][2 * h] = exp2f(s[nt][2 * h] - msafe);
        s[nt][2 * h + 1] = exp2f(s[nt][2 * h + 1] - msafe);
        sum += s[nt][2 * h] + s[nt][2 * h + 1];
      }
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      l[h] = l[h] * alpha[h] + sum;
    }
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      o[n][0] *= alpha[0];
      o[n][1] *= alpha[0];
      o[n][2] *= alpha[1];
      o[n][3] *= alpha[1];
    }
    // O += P V
#pragma unroll
    for (int j = 0; j < 4; ++j) {  // 16-key steps
      const uint32_t a0 = pack_bf16x2(s[2 * j][0], s[2 * j][1]);
      const uint32_t a1 = pack_bf16x2(s[2 * j][2], s[2 * j][3]);
      const uint32_t a2 = pack_bf16x2(s[2 * j + 1][0], s[2 * j + 1][1]);
      const uint32_t a3 = pack_bf16x2(s[2 * j + 1][2], s[2 * j + 1][3]);
#pragma unroll
      for (int n = 0; n < 16; n += 2) {
        uint32_t b0, b1, b2, b3;
        const int r = j * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = n + (lane >> 4);
        ldsm_x4_t(vb + swz(r, c), b0, b1, b2, b3);
        mma16816(o[n], a0, a1, a2, a3, b0, b1);
        mma16816(o[n + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();
  }

  // ---- finalize ----
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int pr = row0 + warp * 16 + (lane >> 2) + 8 * h;
    const float inv = l[h] > 0.f ? 1.f / l[h] : 0.f;
    const float lse = l[h] > 0.f ? (m[h] + log2f(l[h])) / kLog2e : -INFINITY;
    float amax = 0.f;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      o[n][2 * h] *= inv;
      o[n][2 * h + 1] *= inv;
      amax = fmaxf(amax, fmaxf(fabsf(o[n][2 * h]), fabsf(o[n][2 * h + 1])));
    }
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    if (!ok_r[h]) continue;
    const int head = kvh * G + pr % G;
    const int tok = tok_r[h];
    const size_t obase = ((size_t)tok * p.Hq + head) * kAttD + 2 * (lane & 3);
    if (p.o_part) {
#pragma unroll
      for (int n = 0; n < 16; ++n)
        *reinterpret_cast<uint32_t*>(p.o_part + obase + n * 8) = pack_bf16x2(o[n][2 * h], o[n][2 * h + 1]);
      if ((lane & 3) == 0) p.lse_part[(size_t)tok * p.Hq + head] = lse;
    }
    if (p.out) {
#pragma unroll
      for (int n = 0; n < 16; ++n)
        *reinterpret_cast<uint32_t*>(p.out + obase + n * 8) = pack_bf16x2(o[n][2 * h], o[n][2 * h + 1]);
    }
    if (p.out_q) {
      float isc;
      const float sc = fp8_block_scale(amax, &isc);
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        __nv_fp8x2_storage_t v =
            __nv_cvt_float2_to_fp8x2(make_float2(o[n][2 * h] * isc, o[n][2 * h + 1] * isc), __NV_SATFINITE, __NV_E4M3);
        *reinterpret_cast<__nv_fp8x2_storage_t*>(p.out_q + obase + n * 8) = v;
      }
      if ((lane & 3) == 0) p.out_qs[(size_t)head * p.T + tok] = sc;
    }
  }
}

void paged_attention(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor pages,
                     torch::Tensor page_indptr, torch::Tensor prefix_len, torch::Tensor q_start,
                     c10::optional<torch::Tensor> tree, torch::Tensor items, torch::Tensor tile_item,
                     torch::Tensor tile_row0, int64_t num_tiles, bool causal, double softmax_scale,
                     c10::optional<torch::Tensor> o_in, c10::optional<torch::Tensor> lse_in,
                     c10::optional<torch::Tensor> o_part, c10::optional<torch::Tensor> lse_part,
                     c10::optional<torch::Tensor> out, c10::optional<torch::Tensor> out_q,
                     c10::optional<torch::Tensor> out_qs) {
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && q.is_contiguous() && q.dim() == 3 && q.size(2) == kAttD,
              "q must be contiguous bf16 [T, Hq, 128]");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(2) == kAttKeys && k_cache.size(3) == kAttD,
              "kv cache must be [pages, Hkv, 64, 128]");
  const int T = q.size(0), Hq = q.size(1), Hkv = k_cache.size(1);
  TORCH_CHECK(Hq % Hkv == 0);
  if (T == 0 || num_tiles == 0) return;
  const at::cuda::CUDAGuard guard(q.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  AttnParams p;
  p.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  p.kc = reinterpret_cast<const __nv_bfloat16*>(k_cache.data_ptr());
  p.vc = reinterpret_cast<const __nv_bfloat16*>(v_cache.data_ptr());
  p.pages = pages.data_ptr<int>();
  p.page_indptr = page_indptr.data_ptr<int>();
  p.prefix_len = prefix_len.data_ptr<int>();
  p.q_start = q_start.data_ptr<int>();
  p.tree = tree ? reinterpret_cast<const uint64_t*>(tree->data_ptr<int64_t>()) : nullptr;
  p.items = items.data_ptr<int>();
  p.tile_item = tile_item.data_ptr<int>();
  p.tile_row0 = tile_row0.data_ptr<int>();
  p.o_in = o_in ? reinterpret_cast<const __nv_bfloat16*>(o_in->data_ptr()) : nullptr;
  p.lse_in = lse_in ? lse_in->data_ptr<float>() : nullptr;
  p.o_part = o_part ? reinterpret_cast<__nv_bfloat16*>(o_part->data_ptr()) : nullptr;
  p.lse_part = lse_part ? lse_part->data_ptr<float>() : nullptr;
  p.out = out ? reinterpret_cast<__nv_bfloat16*>(out->data_ptr()) : nullptr;
  p.out_q = out_q ? reinterpret_cast<uint8_t*>(out_q->data_ptr()) : nullptr;
  p.out_qs = out_qs ? out_qs->data_ptr<float>() : nullptr;
  p.T = T;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.causal = causal ? 1 : 0;
  p.num_tiles = (int)num_tiles;
  p.scale_log2 = (float)softmax_scale * kLog2e;
  const int smem = 5 * 64 * 256;
  int dev = 0;
  cudaGetDevice(&dev);
  static bool attr[64] = {};   // the opt-in belongs to each device's context
  TORCH_CHECK(dev < 64, "device index out of range");
  if (!attr[dev]) {
    cudaFuncSetAttribute(paged_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    attr[dev] = true;
  }
  dim3 grid((unsigned)num_tiles, Hkv);
  paged_attention_kernel<<<grid, 128, smem, stream>>>(p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Launch on raw pointers (used by entry points that manage their own buffers).
cudaError_t paged_attention_raw_setup() {
  return cudaFuncSetAttribute(paged_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 5 * 64 * 256);
}

cudaError_t launch_paged_attention_raw(const AttnParams& p, int num_tiles, cudaStream_t stream) {
  dim3 grid((unsigned)num_tiles, p.Hkv);
  paged_attention_kernel<<<grid, 128, 5 * 64 * 256, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace phx
