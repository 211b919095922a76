// tcgen05 paged attention for sm_100a (same work-list semantics as csrc/attention.cu; 256-row tiles).
//
// CTA = two 128-row query tiles Q0, Q1 (packed grouped-query rows, row = token * G + g) x one KV head,
// walking 128-key tiles (two 64-key pages) of its item's key range. The two query tiles ping-pong:
// while softmax warpgroup 0 works on S0_j the tensor core computes PV1_{j-1} and S1_j, and the
// other way round, so the tensor pipe and the softmax overlap inside one CTA.
//   warp 0     TMA: Q0/Q1 once (3-D map over [T, Hq, 128], box {64, G, 128/G}); per key tile the K and
//              V pages (2-D map over the cache viewed as [pages*Hkv*64, 128], box {64, 64}); two K and
//              two V stages; a K stage is released as soon as both S MMAs of its tile complete.
//   warp 1     TMEM owner; lane 0 issues, per key tile j:  PV0_{j-1}, S0_j, PV1_{j-1}, S1_j
//              S = Q K^T (SS, M=N=128, 8 x K16); PV = P V (TS: P in TMEM aliasing S, V MN-major).
//   warps 2-5  softmax of Q0; warps 6-9 softmax of Q1; one thread per row: two passes over the S row in
//              TMEM (max, then exp2 / pack / store P), lazy rescale of O in TMEM only when the row max
//              grows by more than 8 (2^8), and the epilogue (O / l, cascade-seed merge, bf16 / fp8 /
//              partial outputs).
// TMEM: S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512).  All waits are bounded (status + abort).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "tmap.h"

namespace phx {

namespace attn_tc {

constexpr int kRows = 128;   // rows per query tile; a CTA holds two
constexpr int kKeys = 128;
constexpr int kD = 128;
constexpr int kThreads = 320;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;
constexpr uint32_t kTmemCols = 512;

struct Smem {
  uint8_t q[2][2][kRows * 128];       // [query tile][d-half], 16 KB each
  uint8_t k[2][2][kKeys * 128];       // [stage][d-half]
  uint8_t v[2][2][kKeys * 128];
  uint64_t q_full;
  uint64_t k_full[2], v_full[2], k_empty[2], v_empty[2];
  uint64_t s_full[2], p_full[2], o_done[2];   // per query tile
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
};

struct Params {
  const int* pages;
  const int* page_indptr;
  const int* prefix_len;
  const int* q_start;
  const uint64_t* tree;
  const int* items;
  const int* tile_item;
  const int* tile_row0;
  const __nv_bfloat16* o_in;
  const float* lse_in;
  __nv_bfloat16* o_part;
  float* lse_part;
  __nv_bfloat16* out;
  uint8_t* out_q;
  float* out_qs;
  int* status;
  int T, Hq, Hkv, causal, num_tiles;
  float scale_log2;
};

// MN-major SWIZZLE_128B descriptor (V as the B operand): LBO = byte stride between 64-element column
// blocks along N, SBO = byte stride between 8-row groups along K.
__device__ __forceinline__ uint64_t sdesc_mn_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFF) >> 4);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFF) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

__device__ __forceinline__ float exp2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void tmem_ld32x2(uint32_t taddr, uint32_t (&r)[64]) {
  tmem_ld32(taddr, *reinterpret_cast<uint32_t(*)[32]>(r));
  tmem_ld32(taddr + 32, *reinterpret_cast<uint32_t(*)[32]>(r + 32));
}

// Visibility of the 32 keys [kw, kw+32) for one query row, as a bitmask (bit e = key kw+e visible):
// keys below kv_hi, and (mreq >= 0) either committed (key < plen) or allowed by the causal / tree rule.
struct RowMask {
  int kv_hi, plen, li, mreq, causal;
  uint64_t tm;
  __device__ __forceinline__ static uint32_t low_bits(int n) {   // n low bits set, n clamped to [0, 32]
    return n <= 0 ? 0u : (n >= 32 ? 0xffffffffu : ((1u << n) - 1u));
  }
  __device__ __forceinline__ uint32_t word(int kw) const {
    uint32_t m = low_bits(kv_hi - kw);
    if (mreq < 0) return m;
    const uint32_t pre = low_bits(plen - kw);
    const int rel0 = kw - plen;                     // rel of bit 0
    uint32_t rule;
    if (causal) {
      // rel0 + e <= li  <=>  e <= li - rel0, and only for rel >= 0 (pre covers rel < 0)
      rule = low_bits(li - rel0 + 1);
    } else {
      uint64_t t;
      if (rel0 >= 64 || rel0 <= -32) t = 0;
      else t = rel0 >= 0 ? (tm >> rel0) : (tm << (-rel0));
      rule = static_cast<uint32_t>(t);
    }
    return m & (pre | (rule & ~pre));
  }
};

__global__ void __launch_bounds__(kThreads, 1)
    attn_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>(smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023));
  const int warp = warp_id(), lane = lane_id();
  const int tile = blockIdx.x;
  const int kvh = blockIdx.y;
  const int item = tile < p.num_tiles ? p.tile_item[tile] : -1;
  if (item < 0) return;  // uniform for the CTA, before any barrier or TMEM use
  const int G = p.Hq / p.Hkv;
  const int* it = p.items + item * 6;
  const int q0 = it[0], qn = it[1], treq = it[2], kv_lo = it[3], kv_hi = it[4], mreq = it[5];
  const int row0 = p.tile_row0[tile];
  const int nrows = qn * G;
  const int ntiles = kv_hi > kv_lo ? (kv_hi - kv_lo + kKeys - 1) / kKeys : 0;
  const int* pg = p.pages + p.page_indptr[treq];
  const int npages = p.page_indptr[treq + 1] - p.page_indptr[treq];

  if (threadIdx.x == 0) {
    mbar_init(&s.q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.k_full[i], 1);
      mbar_init(&s.v_full[i], 1);
      mbar_init(&s.k_empty[i], 1);
      mbar_init(&s.v_empty[i], 1);
      mbar_init(&s.s_full[i], 1);
      mbar_init(&s.p_full[i], 4);
      mbar_init(&s.o_done[i], 1);
    }
    mbar_init(&s.mma_done, 1);
    s.abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&s.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  volatile int* abort = &s.abort;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- loader ----------------
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      mbar_arrive_expect_tx(&s.q_full, 4 * kRows * 128);
      for (int qt = 0; qt < 2; ++qt) {
        const int tok0 = q0 + (row0 + qt * kRows) / G;
        tma_load_3d(&tmQ, &s.q_full, s.q[qt][0], 0, kvh * G, tok0);
        tma_load_3d(&tmQ, &s.q_full, s.q[qt][1], 64, kvh * G, tok0);
      }
      int issued = 0;
      for (int j = 0; j < ntiles && !*abort; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        const int k0 = kv_lo + j * kKeys;
        const int pi0 = k0 / 64;
        const int pi1 = pi0 + 1 < npages ? pi0 + 1 : pi0;  // past the last page: reload a valid one (masked)
        const int r0 = (pg[pi0] * p.Hkv + kvh) * 64, r1 = (pg[pi1] * p.Hkv + kvh) * 64;
        if (!mbar_wait(&s.k_empty[st], ph ^ 1, p.status, kErrTimeoutProducer, abort)) break;
        mbar_arrive_expect_tx(&s.k_full[st], 4 * 64 * 128);
        for (int h = 0; h < 2; ++h) {
          tma_load_2d(&tmK, &s.k_full[st], s.k[st][h], h * 64, r0);
          tma_load_2d(&tmK, &s.k_full[st], s.k[st][h] + 64 * 128, h * 64, r1);
        }
        if (!mbar_wait(&s.v_empty[st], ph ^ 1, p.status, kErrTimeoutProducer, abort)) {
          ++issued;
          break;
        }
        mbar_arrive_expect_tx(&s.v_full[st], 4 * 64 * 128);
        for (int h = 0; h < 2; ++h) {
          tma_load_2d(&tmV, &s.v_full[st], s.v[st][h], h * 64, r0);
          tma_load_2d(&tmV, &s.v_full[st], s.v[st][h] + 64 * 128, h * 64, r1);
        }
        ++issued;
      }
      // drain the copies in flight before the CTA may exit (bounded)
      volatile int never = 0;
      mbar_wait(&s.q_full, 0, nullptr, 0, &never);
      for (int j = issued - 2 < 0 ? 0 : issued - 2; j < issued; ++j) {
        mbar_wait(&s.k_full[j & 1], (j >> 1) & 1, nullptr, 0, &never);
        mbar_wait(&s.v_full[j & 1], (j >> 1) & 1, nullptr, 0, &never);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && ntiles > 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idS = idesc_make(128, 128, 1);
      constexpr uint32_t idPV = idesc_make(128, 128, 1) | (1u << 16);  // B (V) MN-major
      auto issue_s = [&](int qt, int j) {
        const int st = j & 1;
        const uint32_t dS = tmem + qt * 128;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint64_t da = sdesc_sw128(smem_u32(s.q[qt][k >> 2])) + 2 * (k & 3);
          const uint64_t db = sdesc_sw128(smem_u32(s.k[st][k >> 2])) + 2 * (k & 3);
          umma_f16(dS, da, db, idS, k > 0);
        }
        umma_commit(&s.s_full[qt]);
      };
      auto issue_pv = [&](int qt, int j) {
        const int st = j & 1;
#pragma unroll
        for (int k = 0; k < 8; ++k) {  // 16 keys per instruction: P columns k*8, V rows k*16
          const uint64_t db = sdesc_mn_sw128(smem_u32(s.v[st][0]) + k * 2048, kKeys * 128, 1024);
          umma_f16_ts(tmem + 256 + qt * 128, tmem + qt * 128 + k * 8, db, idPV, (j > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(&s.o_done[qt]);
      };
      if (!mbar_wait(&s.q_full, 0, p.status, kErrTimeoutMma, abort)) goto mma_out;
      if (!mbar_wait(&s.k_full[0], 0, p.status, kErrTimeoutMma, abort)) goto mma_out;
      tc_fence_after();
      issue_s(0, 0);
      issue_s(1, 0);
      umma_commit(&s.k_empty[0]);
      for (int j = 0; j < ntiles; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        const bool more = j + 1 < ntiles;
        if (!mbar_wait(&s.v_full[st], ph, p.status, kErrTimeoutMma, abort)) goto mma_out;
        if (!mbar_wait(&s.p_full[0], j & 1, p.status, kErrTimeoutMma, abort)) goto mma_out;
        tc_fence_after();
        issue_pv(0, j);
        if (more) {
          const int st1 = (j + 1) & 1;
          if (!mbar_wait(&s.k_full[st1], ((j + 1) >> 1) & 1, p.status, kErrTimeoutMma, abort)) goto mma_out;
          tc_fence_after();
          issue_s(0, j + 1);
        }
        if (!mbar_wait(&s.p_full[1], j & 1, p.status, kErrTimeoutMma, abort)) goto mma_out;
        tc_fence_after();
        issue_pv(1, j);
        umma_commit(&s.v_empty[st]);
        if (more) {
          issue_s(1, j + 1);
          umma_commit(&s.k_empty[(j + 1) & 1]);
        }
      }
    mma_out:
      umma_commit(&s.mma_done);
      volatile int never = 0;
      mbar_wait(&s.mma_done, 0, nullptr, 0, &never);
    }
  } else {
    // ---------------- softmax + epilogue (warps 2-5: Q0, warps 6-9: Q1) ----------------
    const int qt = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;             // row within the query tile == TMEM lane
    const int pr = row0 + qt * kRows + r;
    const bool row_ok = pr < nrows;
    const int tok = q0 + (row_ok ? pr / G : 0);
    const int head = kvh * G + (row_ok ? pr % G : 0);
    RowMask rm{kv_hi, 0, 0, mreq, p.causal, 0ull};
    if (mreq >= 0) {
      rm.plen = p.prefix_len[mreq];
      rm.li = tok - p.q_start[mreq];
      if (p.tree && !p.causal) rm.tm = p.tree[tok];
    }
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t colS = qt * 128, colO = 256 + qt * 128;
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      ok = mbar_wait(&s.s_full[qt], j & 1, p.status, kErrTimeoutEpilogue, abort);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      tc_fence_after();
      const int k0 = kv_lo + j * kKeys;
      uint32_t vis[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) vis[c] = rm.word(k0 + c * 32);
      // pass 1: row max of the visible raw scores
      float mx = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t rr[32];
        tmem_ld32(tmem + lane_addr + colS + c * 32, rr);
        tmem_wait_ld();
        const uint32_t vm = vis[c];
#pragma unroll
        for (int e = 0; e < 32; ++e) mx = fmaxf(mx, ((vm >> e) & 1u) ? __uint_as_float(rr[e]) : -INFINITY);
      }
      mx *= p.scale_log2;
      // lazy rescale: move the reference max only when it grows by more than 2^8
      const bool need = mx > m_ref + kRescaleThreshold;
      if (__any_sync(0xffffffffu, need)) {
        const float new_ref = need ? mx : m_ref;
        const float alpha = need ? exp2_approx(m_ref - new_ref) : 1.f;  // m_ref = -inf -> 0
        if (j > 0) {
          // O holds PV_0..PV_{j-1}; wait for PV_{j-1} before rescaling it in place
          ok = mbar_wait(&s.o_done[qt], (j - 1) & 1, p.status, kErrTimeoutEpilogue, abort);
          if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
          tc_fence_after();
          const float2 a2 = make_float2(alpha, alpha);
#pragma unroll 1
          for (int c = 0; c < 8; ++c) {
            uint32_t rr[16];
            tmem_ld16(tmem + lane_addr + colO + c * 16, rr);
            tmem_wait_ld();
#pragma unroll
            for (int x = 0; x < 16; x += 2) {
              const float2 v = __fmul2_rn(make_float2(__uint_as_float(rr[x]), __uint_as_float(rr[x + 1])), a2);
              rr[x] = __float_as_uint(v.x);
              rr[x + 1] = __float_as_uint(v.y);
            }
            tmem_st16(tmem + lane_addr + colO + c * 16, rr);
          }
          tmem_wait_st();
        }
        l *= alpha;
        m_ref = new_ref;
      }
      // pass 2: P = exp2(s * scale - m_ref) as bf16 over the first 64 columns of this S buffer. Every
      // chunk of S is read before the packed P that overwrites it is stored.
      const float mref_safe = m_ref == -INFINITY ? 0.f : m_ref;
      const float2 sc2 = make_float2(p.scale_log2, p.scale_log2), nm2 = make_float2(-mref_safe, -mref_safe);
      float2 rs2 = make_float2(0.f, 0.f);
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t rr[32];
        tmem_ld32(tmem + lane_addr + colS + c * 32, rr);
        tmem_wait_ld();
        const uint32_t vm = vis[c];
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float2 x = __ffma2_rn(make_float2(__uint_as_float(rr[2 * e]), __uint_as_float(rr[2 * e + 1])), sc2, nm2);
          const float a = ((vm >> (2 * e)) & 1u) ? exp2_approx(x.x) : 0.f;
          const float b = ((vm >> (2 * e + 1)) & 1u) ? exp2_approx(x.y) : 0.f;
          rs2 = __fadd2_rn(rs2, make_float2(a, b));
          pk[e] = pack_bf16x2(a, b);
        }
        tmem_st16(tmem + lane_addr + colS + c * 16, pk);
      }
      tmem_wait_st();
      l += rs2.x + rs2.y;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.p_full[qt]);
    }
    // ---- epilogue ----
    bool have_o = false;
    if (ok && ntiles > 0) {
      ok = mbar_wait(&s.o_done[qt], (ntiles - 1) & 1, p.status, kErrTimeoutEpilogue, abort);
      if (__all_sync(0xffffffffu, ok)) {
        tc_fence_after();
        have_o = true;
      } else {
        ok = false;
      }
    }
    if (ok) {
      // merge with the seed partial: acc (relative to m_ref) + O_in (relative to lse_in)
      float w_acc = l > 0.f ? 1.f : 0.f, w_seed = 0.f, m2 = m_ref;
      const __nv_bfloat16* seed = nullptr;
      if (p.o_in && row_ok) {
        const float lse2 = p.lse_in[(size_t)tok * p.Hq + head] * kLog2e;
        if (lse2 != -INFINITY) {
          seed = p.o_in + ((size_t)tok * p.Hq + head) * kD;
          const float M = fmaxf(m_ref, lse2);
          w_acc = l > 0.f ? exp2f(m_ref - M) : 0.f;
          w_seed = exp2f(lse2 - M);
          m2 = M;
        }
      }
      const float denom = w_acc * l + w_seed;
      const float inv = denom > 0.f ? 1.f / denom : 0.f;
      const float lse = denom > 0.f ? (m2 + log2f(denom)) / kLog2e : -INFINITY;
      const size_t ob = ((size_t)tok * p.Hq + head) * kD;
      // two passes over O in TMEM (32 columns at a time): amax for the fp8 scale, then convert and store
      auto chunk = [&](int c, float (&o)[32]) {
        uint32_t rr[32];
        if (have_o) {
          tmem_ld32(tmem + lane_addr + colO + c * 32, rr);
          tmem_wait_ld();
        }
#pragma unroll
        for (int e = 0; e < 32; ++e) o[e] = have_o ? w_acc * __uint_as_float(rr[e]) : 0.f;
        if (seed) {
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            const uint4 v = *reinterpret_cast<const uint4*>(seed + c * 32 + e);
            const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int x = 0; x < 4; ++x) {
              const float2 f = unpack_bf16x2(wv[x]);
              o[e + 2 * x] += w_seed * f.x;
              o[e + 2 * x + 1] += w_seed * f.y;
            }
          }
        }
#pragma unroll
        for (int e = 0; e < 32; ++e) o[e] *= inv;
      };
      float amax = 0.f;
      if (p.out_q) {
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          float o[32];
          chunk(c, o);
#pragma unroll
          for (int e = 0; e < 32; ++e) amax = fmaxf(amax, fabsf(o[e]));
        }
      }
      float isc;
      const float sc = fp8_block_scale(amax, &isc);
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float o[32];
        chunk(c, o);
        if (!row_ok) continue;
#pragma unroll
        for (int e = 0; e < 32; e += 8) {
          const size_t off = ob + c * 32 + e;
          const uint4 b16 = make_uint4(pack_bf16x2(o[e], o[e + 1]), pack_bf16x2(o[e + 2], o[e + 3]),
                                       pack_bf16x2(o[e + 4], o[e + 5]), pack_bf16x2(o[e + 6], o[e + 7]));
          if (p.o_part) *reinterpret_cast<uint4*>(p.o_part + off) = b16;
          if (p.out) *reinterpret_cast<uint4*>(p.out + off) = b16;
          if (p.out_q)
            *reinterpret_cast<uint2*>(p.out_q + off) =
                make_uint2(pack_fp8x4(o[e] * isc, o[e + 1] * isc, o[e + 2] * isc, o[e + 3] * isc),
                           pack_fp8x4(o[e + 4] * isc, o[e + 5] * isc, o[e + 6] * isc, o[e + 7] * isc));
        }
      }
      if (row_ok) {
        if (p.lse_part) p.lse_part[(size_t)tok * p.Hq + head] = lse;
        if (p.out_q) p.out_qs[(size_t)head * p.T + tok] = sc;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

}  // namespace attn_tc

void paged_attention_tc(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor pages,
                        torch::Tensor page_indptr, torch::Tensor prefix_len, torch::Tensor q_start,
                        c10::optional<torch::Tensor> tree, torch::Tensor items, torch::Tensor tile_item,
                        torch::Tensor tile_row0, int64_t num_tiles, bool causal, double softmax_scale,
                        c10::optional<torch::Tensor> o_in, c10::optional<torch::Tensor> lse_in,
                        c10::optional<torch::Tensor> o_part, c10::optional<torch::Tensor> lse_part,
                        c10::optional<torch::Tensor> out, c10::optional<torch::Tensor> out_q,
                        c10::optional<torch::Tensor> out_qs, torch::Tensor status) {
  using namespace attn_tc;
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && q.is_contiguous() && q.dim() == 3 && q.size(2) == kD,
              "q must be contiguous bf16 [T, Hq, 128]");
  TORCH_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous() && k_cache.dim() == 4 && k_cache.size(2) == 64 &&
                  k_cache.size(3) == kD,
              "kv cache must be contiguous [pages, Hkv, 64, 128]");
  const int T = q.size(0), Hq = q.size(1), Hkv = k_cache.size(1);
  TORCH_CHECK(Hq % Hkv == 0);
  const int G = Hq / Hkv;
  TORCH_CHECK(G <= 128 && 128 % G == 0, "group size must divide 128");
  if (T == 0 || num_tiles == 0) return;
  const at::cuda::CUDAGuard guard(q.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const uint64_t kv_rows = (uint64_t)k_cache.size(0) * Hkv * 64;
  CUtensorMap tq = make_tmap_3d(q.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, kD, Hq, T, kD * 2, (uint64_t)Hq * kD * 2,
                                64, G, 128 / G, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tk = make_tmap_2d(k_cache.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, kD, kv_rows, kD * 2, 64, 64,
                                CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tv = make_tmap_2d(v_cache.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, kD, kv_rows, kD * 2, 64, 64,
                                CU_TENSOR_MAP_SWIZZLE_128B);
  Params p{};
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
  p.status = status.data_ptr<int>();
  p.T = T;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.causal = causal ? 1 : 0;
  p.num_tiles = (int)num_tiles;
  p.scale_log2 = (float)softmax_scale * kLog2e;
  const size_t smem = sizeof(Smem) + 1024;
  int dev = 0;
  cudaGetDevice(&dev);
  static bool attr[64] = {};   // the opt-in belongs to each device's context
  TORCH_CHECK(dev < 64, "device index out of range");
  if (!attr[dev]) {
    cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attr[dev] = true;
  }
  dim3 grid((unsigned)num_tiles, Hkv);
  attn_kernel<<<grid, kThreads, smem, stream>>>(tq, tk, tv, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace phx
