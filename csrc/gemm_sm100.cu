// tcgen05 / TMEM / TMA GEMMs for sm_100a.
//
//   gemm_fp8_block: out[M,N] (bf16) = sum_kb xs[kb,m] * ws[n/128,kb] * (xq[m, kb*128:+128] . wq[n, kb*128:+128])
//     xq fp8 e4m3 [M,K] row-major, xs fp32 [K/128, M], wq fp8 [N,K] row-major, ws fp32 [ceil(N/128), K/128].
//     This is the block-scaled FP8 linear of DeepSeek/Qwen-style FP8 checkpoints (128x128 weight blocks,
//     1x128 activation blocks). The reference runs its FP8 linears through a CUTLASS sm90 wgmma tile table
//     (docker/opt/v5/wq/kopt_wq_gemm.cuh:47-221, per-token x per-channel scales); this kernel is the
//     Blackwell design for the block-scaled format.
//   gemm_bf16: out[M,N] (bf16) = x[M,K] . w[N,K]^T, fp32 accumulate (lm_head, bf16 models).
//   gemm_fp8_swiglu: the gate/up projection with SwiGLU + FP8 quant in the epilogue (SwigluArgs).
//   gemm_fp8_grouped / gemm_bf16_grouped: MoE experts over device-side row offsets; optional row gather
//     inside the A loads (TMA gather4).
//   gemm_scatter: row-parallel projection whose epilogue stores rows into their owner rank's receive slot.
//
// Design (one persistent CTA per SM, 320 threads):
//   warp 0      TMA producer: 128-byte-wide K slices of A (128 rows) and B (BN rows) into a STAGES-deep
//               ring of SWIZZLE_128B tiles, one mbarrier (full/empty) pair per stage.
//   warp 1      allocates TMEM; lane 0 issues tcgen05.mma (M=128, N=BN, K=32 fp8 or 16 bf16 per
//               instruction, 4 per stage) into one of two TMEM accumulators and commits to mbarriers.
//   warps 2-9   epilogue. bf16, and fp8 with hardware scaling (HWS, the default): the MMA accumulates the
//               whole K range in TMEM and the epilogue drains it once per tile into registers, frees the
//               accumulator, then converts and stores while the next tile's MMAs run.
//               fp8 with software promotion (HWS off): every 128-wide K block lands in a fresh TMEM
//               accumulator; the epilogue reads it with tcgen05.ld and adds it, scaled by
//               xs[kb,row]*ws[nblk,kb], into fp32 registers, while the MMA fills the other accumulator.
//   HWS: the block scales are powers of two (see fp8_block_scale), so they are exact UE8M0 values and the
//   tensor core applies them itself: tcgen05.mma kind::mxf8f6f4.block_scale reads one scale per A row and
//   per B column for each 32-deep K step from TMEM. Per stage the producer warp converts the stage's 128
//   activation scales and BN/128 weight scales to exponent bytes in shared memory, in the replicated
//   32-lane x 4-column layout, and the MMA thread moves them to TMEM with tcgen05.cp (.32x128b.warpx4)
//   right before the stage's four MMAs (cp -> mma from one thread runs in issue order). A scale that is
//   not a positive power of two sets kErrScaleNotPow2 in the status word. The producer loads the scales
//   four stages ahead of their stage (an L2 round trip outlasts a stage's MMAs).
//   Tiles are walked M-fastest so CTAs running together share weight (B) columns in L2.
//   PAIR (hardware-scaled fp8, BN = 256): clusters of two CTAs on neighbouring SMs run one 256 x 256 tile with
//   tcgen05.mma.cta_group::2 (M = 256): each CTA stages its own 128 rows of A and its own 128 rows of B,
//   and the pair leader's MMA reads both CTAs' halves, so a CTA moves 32 KB per 128-deep K block for a
//   128 x 256 x 128 product instead of 48 KB: 1.5x the FLOPs per byte of L2 -> shared-memory traffic, the
//   bound of the single-CTA tile. Each CTA's TMA counts its bytes on the leader's full barrier; the
//   non-leader also arrives there after staging its scale factors; the leader commits MMA completion to
//   both CTAs' empty / tfull barriers, and both CTAs' epilogues release the leader's accumulator.
//   Measured on B200 (Llama-3-70B verify shapes): with the cluster-scope release of the per-stage peer
//   arrive the pair runs at about half the single-CTA rate (the release waits out the peer's in-flight
//   copies, so the ring degenerates to one stage); with a relaxed arrive it reaches 0.85-1.0x of it.
//   Under the 1 kW power cap (about 1.35 GHz sustained) the tensor-pipe clock, not operand traffic, bounds
//   these GEMMs, so the pair is opt-in (PHX_GEMM_PAIR=1) and the single-CTA tile is the default.
//   No TMA multicast anywhere: every CTA loads its own tiles.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cudaTypedefs.h>
#include <torch/extension.h>

#include "common.cuh"
#include "tmap.h"

namespace phx {

constexpr int kBM = 128;
constexpr int kEpiWarps = 8;
constexpr int kGemmThreads = 64 + kEpiWarps * 32;  // producer warp, MMA warp, 8 epilogue warps

template <int BN, int STAGES, bool HWS = false, int BROWS = BN>
struct GemmSmem {
  uint8_t a[STAGES][kBM * 128];
  uint8_t b[STAGES][BROWS * 128];      // BROWS = BN, or BN/2 per CTA of a pair
  // HWS scale-factor staging, per stage: activation scales (32 lanes x 16 B: byte 4c of lane l = row 32c+l),
  // then BN/128 groups of weight scales in the same shape (column 32c+l of the group's 128)
  uint8_t sf[HWS ? STAGES : 1][HWS ? 512 * (1 + BN / 128) : 16];
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[512 / BN];
  uint64_t tempty[512 / BN];
  uint64_t done;
  uint64_t up_ready, up_free;   // SWIGLU epilogue: up-half warps -> gate-half warps hand-off of staged rows
  uint64_t split_bar;           // split-K epilogue: the epilogue warps' barrier (kEpiWarps arrivals a phase)
  uint32_t tmem_base;
  int abort;
  int split_ok;
};

// the scatter epilogue stages each warp's 32 output rows in shared memory (8 warps x 32 rows x (BN/2 + 8)
// bf16); BN = 256 gives up one operand stage for it
template <int BN, bool SCATTER = false, bool PAIR = false>
constexpr int gemm_stages() {
  return PAIR ? (SCATTER ? 4 : 6) : BN == 256 ? (SCATTER ? 3 : 4) : (SCATTER ? 5 : 6);
}

template <int BN>
constexpr int scatter_row_bytes() {
  return BN + 16;   // BN/2 bf16 columns per epilogue warp row, padded by 16 bytes against bank conflicts
}

// Output tile t -> rows [m0, m_end) of A / out, rows [b0, b0 + BN) of B, output columns [n0, n0 + BN),
// weight-scale row base. Plain GEMM: tiles walk M fastest. Grouped GEMM (grp_off != null, MoE experts):
// A rows are sorted by group, group e owns rows [grp_off[e], grp_off[e+1]) and B rows [e*N, (e+1)*N);
// tiles are enumerated group by group (M fastest inside a group) from the device-side offsets, so the
// tile list needs no host round trip; tiles past the last group are invalid.
struct TileInfo {
  int m0, m_end, b0, n0, sb_base;
  bool valid;
};

template <int BN, int BMT = kBM>
__device__ __forceinline__ TileInfo tile_info(int t, int M, int N, int m_tiles, int n_tiles, const int* grp_off,
                                              int groups) {
  TileInfo ti;
  if (!grp_off) {
    const int m_blk = t % m_tiles, n_blk = t / m_tiles;
    ti.m0 = m_blk * BMT;
    ti.m_end = M;
    ti.n0 = n_blk * BN;
    ti.b0 = ti.n0;
    ti.sb_base = 0;
    ti.valid = t < m_tiles * n_tiles;
    return ti;
  }
  ti.valid = false;
  for (int e = 0; e < groups; ++e) {
    const int lo = grp_off[e], hi = grp_off[e + 1];
    const int mt = (hi - lo + kBM - 1) / kBM;
    const int tiles = mt * n_tiles;
    if (t < tiles) {
      const int n_blk = t / mt, m_blk = t % mt;
      ti.m0 = lo + m_blk * kBM;
      ti.m_end = hi;
      ti.n0 = n_blk * BN;
      ti.b0 = e * N + ti.n0;
      ti.sb_base = e * ((N + 127) / 128);
      ti.valid = true;
      return ti;
    }
    t -= tiles;
  }
  return ti;
}

// Scatter epilogue of a row-parallel projection under tensor parallelism: output row r is stored, over
// NVLink, into rank owner(r) = r / rows_per's receive buffer at slot [rank][r - owner*rows_per] (each
// rank's workspace base in peer_base). The reduce-scatter then reads only local memory, and the transfer
// overlaps the remaining tiles' MMAs. peer_base == nullptr: plain stores to `out`.
struct ScatterArgs {
  const uint64_t* peer_base;
  uint64_t off_recv;
  int rows_per, rank;
  int bulk;          // 1: each staged row leaves as one TMA bulk copy; 0: row-contiguous 16-byte lane stores
};

// SwiGLU epilogue of the gate/up projection (hardware-scaled fp8, BN = 256). The weight rows are interleaved
// in 128-row blocks (gate block j, then up block j), so output tile n0 holds gate columns [n0/2, n0/2 + 128)
// in its first 128 columns and the matching up columns in the other 128. The epilogue writes
// a = bf16(silu(bf16(g)) * bf16(u)) quantized to e4m3 with one power-of-two scale per 128 columns:
// q [M, F] (row stride F) and qs [F/128, M] -- bitwise what the GEMM's bf16 [g | u] output followed by
// silu_mul_quant produces, without the [M, 2F] bf16 round trip through HBM.
struct SwigluArgs {
  uint8_t* q;
  float* qs;
  int F;
};

// Split-K tail of a plain GEMM whose tile count leaves the last wave of the persistent grid mostly idle
// (fewer tiles than SMs, or a few tiles past a whole number of waves: Llama-3-70B qkv at TP8 has 160 tiles of
// 128 x 256 for 148 SMs, the draft rounds' M = 512 GEMMs 20-40 tiles). Tiles [0, dp_tiles) run whole; each
// later tile is cut into `splits` contiguous K ranges, one work item each. dp_tiles is a multiple of the grid
// size and the split items number at most the grid size, so every CTA takes at most one split item and takes
// it in its last round: all parts of a split tile run at the same time (one CTA per SM, grid <= SMs). Each
// part stores its fp32 partial tile into a workspace slot in epilogue-thread order (coalesced), arrives on
// the tile's counter, waits (bounded) for the other parts, then sums one 1/splits share of the tile over all
// parts (L2-resident reads) and stores it as bf16. The last part to leave zeroes the tile's counters for the
// next launch. splits <= 1: every tile whole (the other epilogues always run that way).
struct SplitArgs {
  float* ws;        // [split tiles x splits][BN/8][256] float4 partials
  int* cnt;         // [2 x split tiles] arrive / depart counters, zero between launches
  int dp_tiles;
  int splits;
};

struct WorkItem {
  int t, kb0, kb1, part;   // tile, K-step range [kb0, kb1), part index (-1: whole tile)
};

__device__ __forceinline__ WorkItem work_item(int i, int ksteps, const SplitArgs& sk) {
  WorkItem w;
  if (sk.splits <= 1 || i < sk.dp_tiles) {
    w.t = i;
    w.kb0 = 0;
    w.kb1 = ksteps;
    w.part = -1;
    return w;
  }
  const int j = i - sk.dp_tiles;
  w.t = sk.dp_tiles + j / sk.splits;
  w.part = j % sk.splits;
  w.kb0 = (int)((long long)w.part * ksteps / sk.splits);
  w.kb1 = (int)((long long)(w.part + 1) * ksteps / sk.splits);
  return w;
}

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void epi_bar_sync() {   // the kEpiWarps epilogue warps only (named barrier 1)
  asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory");
}

// Workspace of the split-K tail: statically allocated device memory (no allocation at call time, so the
// split path is also safe inside CUDA-graph capture). kMaxSplitItems parts of up to 128 x 256 fp32.
constexpr int kMaxSplitItems = 160;
__device__ __align__(256) float g_split_ws[(size_t)kMaxSplitItems * kBM * 256];
__device__ __align__(16) int g_split_cnt[2 * kMaxSplitItems];

template <int BN, bool FP8, bool SCATTER, bool HWS, bool PAIR, bool SWIGLU = false>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_sm100_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      __nv_bfloat16* __restrict__ out, int M, int N, int K, int ldc, const float* __restrict__ sa,
                      const float* __restrict__ sb, int* status, const int* __restrict__ grp_off, int groups,
                      int max_tiles, const ScatterArgs sc, const int* __restrict__ a_rows, int sa_ld,
                      const SwigluArgs sw, const SplitArgs sk) {
  static_assert(!HWS || FP8, "hardware scaling is an fp8 mode");
  static_assert(!PAIR || (HWS && BN == 256), "CTA pairs run the hardware-scaled 256-wide tile");
  static_assert(!SWIGLU || (HWS && BN == 256 && !PAIR && !SCATTER), "SwiGLU epilogue: single-CTA hardware-scaled BN=256");
  constexpr int STAGES = gemm_stages<BN, SCATTER || SWIGLU, PAIR>();
  constexpr int BKE = FP8 ? 128 : 64;  // K elements per 128-byte stage row
  constexpr int BMT = PAIR ? 2 * kBM : kBM;   // output rows per tile (both CTAs of a pair)
  constexpr int BROWS = PAIR ? BN / 2 : BN;   // B rows staged by this CTA
  constexpr uint32_t IDESC = HWS ? idesc_make_bs(BMT, BN) : idesc_make(kBM, BN, FP8 ? 0 : 1);
  // TMEM accumulators: all 512 columns, except under HWS, where columns [256, 256 + STAGES * SF_COLS) hold
  // the stages' scale factors (BN = 256: one accumulator, freed as soon as the epilogue has drained it)
  constexpr int NBUF = HWS ? 256 / BN : 512 / BN;
  constexpr int SF_COLS = 4 + BN / 32;  // per stage: 4 columns of A scales, BN/32 of B scales
  static_assert(!HWS || 256 + STAGES * SF_COLS <= 512, "scale factors exceed TMEM");
  constexpr uint32_t TMEM_COLS = 512;
  constexpr int CPT = BN / 2;  // columns per epilogue thread
  constexpr bool PROMOTE = FP8 && !HWS;   // per-K-block software scale promotion
  using Smem = GemmSmem<BN, STAGES, HWS, BROWS>;

  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>(smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023));

  const int warp = warp_id();
  const int lane = lane_id();
  const uint32_t crank = PAIR ? cluster_ctarank() : 0u;   // 0 = pair leader
  const bool leader = crank == 0;
  const int unit = PAIR ? blockIdx.x / 2 : blockIdx.x;     // this CTA's pair (or CTA) index, and the count
  const int units = PAIR ? gridDim.x / 2 : gridDim.x;
  const int my_row0 = PAIR ? kBM * static_cast<int>(crank) : 0;   // this CTA's rows within a tile
  const int m_tiles = (M + BMT - 1) / BMT;
  const int n_tiles = (N + BN - 1) / BN;
  const int num_tiles = grp_off ? max_tiles : m_tiles * n_tiles;
  const int ksteps = K / BKE;          // smem stages per tile
  const int kblocks = K / 128;         // scale blocks (fp8)
  // work items: whole tiles, then the split tiles' K ranges (sk.splits <= 1: one item per tile)
  const int num_items = sk.splits > 1 ? sk.dp_tiles + (num_tiles - sk.dp_tiles) * sk.splits : num_tiles;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.full[i], PAIR ? 2 : 1);         // pair: the leader's expect_tx + the peer's arrive
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < NBUF; ++i) {
      mbar_init(&s.tfull[i], 1);
      mbar_init(&s.tempty[i], PAIR ? 2 * kEpiWarps : kEpiWarps);   // pair: both CTAs' epilogue warps
    }
    mbar_init(&s.done, 1);
    mbar_init(&s.up_ready, 4);   // the four up-half epilogue warps
    mbar_init(&s.up_free, 4);    // the four gate-half epilogue warps
    mbar_init(&s.split_bar, kEpiWarps);
    s.abort = 0;
    s.split_ok = 0;
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(&s.tmem_base, TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(&s.tmem_base, TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (PAIR) cluster_sync();   // both CTAs' barriers and TMEM exist before either CTA uses them
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = s.tmem_base;
  volatile int* abort = &s.abort;

  if (warp == 0 && HWS) {
    // ---------------- TMA producer + scale-factor staging (whole warp) ----------------
    int stage = 0;
    uint32_t phase = 0;
    int issued = 0;
    bool bad = false;
    // a_rows (dispatch fused into the A loads): A row r of the GEMM is row a_rows[r] of the activation
    // matrix, fetched with TMA gather4 (lane l: rows 4l..4l+3 of the tile) and scaled by that row's scales.
    auto src_row = [&](int r) { r = r < M ? r : M - 1; return a_rows ? a_rows[r] : r; };
    // Scale prefetch, LA stages ahead: an L2 round trip (~0.45 us) is longer than one stage's MMAs
    // (~0.3 us), so loading a stage's scales only one stage ahead left the producer waiting on them and
    // the ring under-filled (ncu: tensor pipe 41 % active, long-scoreboard stalls dominant). Slot 0 of the
    // ring is the current stage; a cursor (la_t, la_ks) walks the (tile, k block) sequence LA stages
    // ahead; srow are the cursor tile's scale rows for this lane.
    constexpr int LA = 4;
    float fa_r[LA][4], fb_r[LA][BN / 128];
    int la_i = unit, la_ks = -1;   // cursor: work item, K step (-1: item not started)
    WorkItem la_w{0, 0, 0, -1};
    int srow[4] = {0, 0, 0, 0};
    TileInfo la_ti;
    la_ti.valid = false;
    auto la_load = [&](float (&fa)[4], float (&fb)[BN / 128]) {
#pragma unroll
      for (int c = 0; c < 4; ++c) fa[c] = 1.f;
#pragma unroll
      for (int g = 0; g < BN / 128; ++g) fb[g] = 1.f;
      if (la_i >= num_items) return;
      if (la_ks < 0) {
        la_w = work_item(la_i, ksteps, sk);
        la_ks = la_w.kb0;
        la_ti = tile_info<BN, BMT>(la_w.t, M, N, m_tiles, n_tiles, grp_off, groups);
        if (la_ti.valid) {
#pragma unroll
          for (int c = 0; c < 4; ++c) srow[c] = src_row(la_ti.m0 + my_row0 + 32 * c + lane);
        }
      }
      if (la_ti.valid) {
#pragma unroll
        for (int c = 0; c < 4; ++c) fa[c] = sa[(size_t)la_ks * sa_ld + srow[c]];
        const int nb_last = la_ti.sb_base + (N + 127) / 128 - 1;
#pragma unroll
        for (int g = 0; g < BN / 128; ++g) {
          const int nb = la_ti.sb_base + (la_ti.n0 >> 7) + g;
          fb[g] = sb[(size_t)(nb < nb_last ? nb : nb_last) * kblocks + la_ks];
        }
      }
      if (++la_ks == la_w.kb1) la_ks = -1, la_i += units;
    };
    int g4[4] = {0, 0, 0, 0};
    auto ue8m0 = [&](float v) -> uint32_t {
      const uint32_t u = __float_as_uint(v);
      bad |= (u & 0x807FFFFFu) != 0u || (u >> 23) == 0u;
      return (u >> 23) & 0xFFu;
    };
#pragma unroll
    for (int j = 0; j < LA; ++j) la_load(fa_r[j], fb_r[j]);
    for (int it = unit; it < num_items && !*abort; it += units) {
      const WorkItem wi = work_item(it, ksteps, sk);
      const TileInfo ti = tile_info<BN, BMT>(wi.t, M, N, m_tiles, n_tiles, grp_off, groups);
      if (!ti.valid) break;
      if (a_rows) {
#pragma unroll
        for (int i = 0; i < 4; ++i) g4[i] = src_row(ti.m0 + 4 * lane + i);
      }
      bool ok = true;
      for (int ks = wi.kb0; ks < wi.kb1; ++ks) {
        const uint4 wa = make_uint4(ue8m0(fa_r[0][0]), ue8m0(fa_r[0][1]), ue8m0(fa_r[0][2]), ue8m0(fa_r[0][3]));
        uint32_t wb[BN / 128];
#pragma unroll
        for (int g = 0; g < BN / 128; ++g) wb[g] = ue8m0(fb_r[0][g]);
#pragma unroll
        for (int j = 0; j + 1 < LA; ++j) {
#pragma unroll
          for (int c = 0; c < 4; ++c) fa_r[j][c] = fa_r[j + 1][c];
#pragma unroll
          for (int g = 0; g < BN / 128; ++g) fb_r[j][g] = fb_r[j + 1][g];
        }
        la_load(fa_r[LA - 1], fb_r[LA - 1]);
        int got = 1;
        if (lane == 0) got = mbar_wait(&s.empty[stage], phase ^ 1, status, kErrTimeoutProducer, abort);
        if (!__shfl_sync(0xffffffffu, got, 0)) {
          ok = false;
          break;
        }
        uint8_t* sf = s.sf[stage];
        *reinterpret_cast<uint4*>(sf + 16 * lane) = wa;
#pragma unroll
        for (int g = 0; g < BN / 128; ++g)
          *reinterpret_cast<uint4*>(sf + 512 * (1 + g) + 16 * lane) = make_uint4(wb[g], wb[g], wb[g], wb[g]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if constexpr (PAIR) {
            // both halves count on the leader's barrier; the peer's arrive also publishes its scale factors
            const uint32_t fbar = mapa_shared(smem_u32(&s.full[stage]), 0);
            if (leader) mbar_arrive_expect_tx(&s.full[stage], 2 * (kBM + BROWS) * 128);
            tma_load_2d_pair(&tmA, fbar, s.a[stage], ks * BKE, ti.m0 + my_row0);
            tma_load_2d_pair(&tmB, fbar, s.b[stage], ks * BKE, ti.b0 + BROWS * static_cast<int>(crank));
            if (!leader) mbar_arrive_cluster(fbar);
          } else {
            mbar_arrive_expect_tx(&s.full[stage], (kBM + BN) * 128);
            if (!a_rows) tma_load_2d(&tmA, &s.full[stage], s.a[stage], ks * BKE, ti.m0);
            tma_load_2d(&tmB, &s.full[stage], s.b[stage], ks * BKE, ti.b0);
          }
        }
        if (!PAIR && a_rows) {
          __syncwarp();   // the stage's transaction count is armed before any gather lands
          tma_gather4(&tmA, &s.full[stage], s.a[stage] + lane * 4 * 128, ks * BKE, g4[0], g4[1], g4[2], g4[3]);
        }
        ++issued;
        if (++stage == STAGES) stage = 0, phase ^= 1;
      }
      if (!ok) break;
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) atomicCAS(status, 0, kErrScaleNotPow2);
    if (lane == 0 && leader) {   // a pair's copies all count on the leader's barriers
      volatile int never = 0;
      for (int i = 0; i < STAGES && i < issued; ++i) {
        if (--stage < 0) stage = STAGES - 1, phase ^= 1;
        mbar_wait(&s.full[stage], phase, nullptr, 0, &never);
      }
    }
  } else if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      for (int it = unit; it < num_items && !*abort; it += units) {
        const WorkItem wi = work_item(it, ksteps, sk);
        const TileInfo ti = tile_info<BN, BMT>(wi.t, M, N, m_tiles, n_tiles, grp_off, groups);
        if (!ti.valid) break;
        for (int ks = wi.kb0; ks < wi.kb1; ++ks) {
          if (!mbar_wait(&s.empty[stage], phase ^ 1, status, kErrTimeoutProducer, abort)) break;
          mbar_arrive_expect_tx(&s.full[stage], (kBM + BN) * 128);
          tma_load_2d(&tmA, &s.full[stage], s.a[stage], ks * BKE, ti.m0);
          tma_load_2d(&tmB, &s.full[stage], s.b[stage], ks * BKE, ti.b0);
          ++issued;
          if (++stage == STAGES) stage = 0, phase ^= 1;
        }
      }
      // drain: the copies of the last (up to STAGES) armed stages have landed before exit (bounded)
      volatile int never = 0;
      for (int i = 0; i < STAGES && i < issued; ++i) {
        if (--stage < 0) stage = STAGES - 1, phase ^= 1;
        mbar_wait(&s.full[stage], phase, nullptr, 0, &never);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------- MMA issuer (a pair's leader issues for both CTAs) ----------------
      int stage = 0;
      uint32_t phase = 0;
      int tb = 0;
      uint32_t tphase = 0;
      for (int it = unit; it < num_items && !*abort; it += units) {
        const WorkItem wi = work_item(it, ksteps, sk);
        if (grp_off && !tile_info<BN, BMT>(wi.t, M, N, m_tiles, n_tiles, grp_off, groups).valid) break;
        for (int ks = wi.kb0; ks < wi.kb1; ++ks) {
          const bool new_acc = PROMOTE || ks == wi.kb0;
          const bool end_acc = PROMOTE || ks == wi.kb1 - 1;
          if (new_acc) {
            if (!mbar_wait<PAIR>(&s.tempty[tb], tphase ^ 1, status, kErrTimeoutMma, abort)) goto mma_done;
            tc_fence_after();
          }
          if (!mbar_wait<PAIR>(&s.full[stage], phase, status, kErrTimeoutMma, abort)) goto mma_done;
          tc_fence_after();
          {
            const uint64_t da = sdesc_sw128(smem_u32(s.a[stage]));
            const uint64_t db = sdesc_sw128(smem_u32(s.b[stage]));
            const uint32_t dtm = tmem_base + tb * BN;
            const uint32_t tsf = tmem_base + 256 + stage * SF_COLS;   // HWS: this stage's scale columns
            if constexpr (PAIR) {
              const uint32_t sfs = smem_u32(s.sf[stage]);
              tmem_cp_32x128b_x4_pair(tsf, sdesc_plain(sfs));
#pragma unroll
              for (int g = 0; g < BN / 128; ++g)
                tmem_cp_32x128b_x4_pair(tsf + 4 + 4 * g, sdesc_plain(sfs + 512 * (1 + g)));
            } else if constexpr (HWS) {
              const uint32_t sfs = smem_u32(s.sf[stage]);
              tmem_cp_32x128b_x4(tsf, sdesc_plain(sfs));
#pragma unroll
              for (int g = 0; g < BN / 128; ++g) tmem_cp_32x128b_x4(tsf + 4 + 4 * g, sdesc_plain(sfs + 512 * (1 + g)));
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint32_t acc = new_acc ? (k > 0) : 1u;
              if constexpr (PAIR)
                umma_f8_bs_pair(dtm, da + 2 * k, db + 2 * k, IDESC, acc, tsf, tsf + 4);
              else if constexpr (HWS)
                umma_f8_bs(dtm, da + 2 * k, db + 2 * k, IDESC, acc, tsf, tsf + 4);
              else if constexpr (FP8)
                umma_f8(dtm, da + 2 * k, db + 2 * k, IDESC, acc);
              else
                umma_f16(dtm, da + 2 * k, db + 2 * k, IDESC, acc);
            }
            if constexpr (PAIR) {
              // release the stage in both CTAs (each producer waits on its own empty barrier), and hand a
              // finished accumulator to both CTAs' epilogues
              const uint32_t eb = smem_u32(&s.empty[stage]);
              umma_commit_pair(mapa_shared(eb, 0));
              umma_commit_pair(mapa_shared(eb, 1));
              if (end_acc) {
                const uint32_t fb = smem_u32(&s.tfull[tb]);
                umma_commit_pair(mapa_shared(fb, 0));
                umma_commit_pair(mapa_shared(fb, 1));
              }
            } else {
              umma_commit(&s.empty[stage]);
              if (end_acc) umma_commit(&s.tfull[tb]);
            }
          }
          if (++stage == STAGES) stage = 0, phase ^= 1;
          if (end_acc)
            if (++tb == NBUF) tb = 0, tphase ^= 1;
        }
      }
    mma_done:
      // all issued MMAs complete before teardown
      if constexpr (PAIR) umma_commit_pair(smem_u32(&s.done));
      else umma_commit(&s.done);
      volatile int never = 0;
      mbar_wait(&s.done, 0, nullptr, 0, &never);
    }
  } else {
    // ---------------- epilogue ----------------
    const int ew = warp - 2;
    const int sub = warp & 3;     // TMEM lane quarter this warp may access
    const int half = ew >> 2;     // column half of the tile
    int tb = 0;
    uint32_t tphase = 0;
    float2 acc[CPT / 2];          // packed pairs: the promotion uses the f32x2 FMA (half the issue slots)
    const int epi_blocks = PROMOTE ? kblocks : 1;
    // the scales of the next (tile, k block) are loaded one step ahead, so their latency overlaps the
    // current block's TMEM drain
    int t = unit;
    int swg_iter = 0;             // SWIGLU: tiles handed through the staging buffer so far (mbarrier phase)
    float sa_next = 0.f, sb_next = 0.f;
    auto load_scales = [&](int tt, int kb) {
      if (!PROMOTE || tt >= num_tiles) return;
      const TileInfo ti = tile_info<BN, BMT>(tt, M, N, m_tiles, n_tiles, grp_off, groups);
      if (!ti.valid) return;
      const int rr = ti.m0 + my_row0 + sub * 32 + lane;
      const int c0 = ti.n0 + half * CPT;
      sa_next = sa[(size_t)kb * M + (rr < M ? rr : M - 1)];
      sb_next = c0 < N ? sb[(size_t)(ti.sb_base + (c0 >> 7)) * kblocks + kb] : 0.f;
    };
    load_scales(t, 0);   // (software promotion never splits: items are tiles there)
    uint32_t split_phase = 0;
    for (; t < num_items && !*abort; t += units) {
      const WorkItem wi = work_item(t, ksteps, sk);
      const TileInfo ti = tile_info<BN, BMT>(wi.t, M, N, m_tiles, n_tiles, grp_off, groups);
      if (!ti.valid) break;
      const int row = ti.m0 + my_row0 + sub * 32 + lane;
      const int col0 = ti.n0 + half * CPT;
      const bool col_ok = col0 < N;
      for (int kb = 0; kb < epi_blocks; ++kb) {
        const float scale = PROMOTE ? sa_next * sb_next : 1.f;
        if (kb + 1 < epi_blocks) load_scales(t, kb + 1);
        else load_scales(t + units, 0);
        const bool ok = mbar_wait<PAIR>(&s.tfull[tb], tphase, status, kErrTimeoutEpilogue, abort);
        if (!__all_sync(0xffffffffu, ok)) goto epi_done;
        tc_fence_after();
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(sub * 32) << 16) + tb * BN + half * CPT;
        constexpr int BATCH = CPT >= 128 ? 16 : CPT;   // columns per tcgen05.wait::ld (register budget)
        const float2 s2 = make_float2(scale, scale);
#pragma unroll
        for (int c0 = 0; c0 < CPT; c0 += BATCH) {
          uint32_t r[BATCH];
#pragma unroll
          for (int q = 0; q < BATCH / 16; ++q)
            tmem_ld16(taddr + c0 + q * 16, *reinterpret_cast<uint32_t(*)[16]>(r + q * 16));
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < BATCH / 2; ++j) {
            const float2 v = make_float2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
            float2& a = acc[(c0 >> 1) + j];
            if (PROMOTE)
              a = kb == 0 ? __fmul2_rn(v, s2) : __ffma2_rn(v, s2, a);
            else
              a = v;
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if constexpr (PAIR) mbar_arrive_cluster(mapa_shared(smem_u32(&s.tempty[tb]), 0));   // the leader's
          else mbar_arrive(&s.tempty[tb]);
        }
        if (++tb == NBUF) tb = 0, tphase ^= 1;
      }
      if constexpr (!SCATTER && !SWIGLU && !PAIR && !PROMOTE) {
        if (wi.part >= 0) {
          // ---- split-K part: publish the fp32 partial, meet the tile's other parts, sum a share ----
          constexpr int ET = kEpiWarps * 32;            // epilogue threads
          constexpr int F4 = (CPT / 4) * ET;            // float4s per tile
          const int et = ew * 32 + lane;
          const int sti = wi.t - sk.dp_tiles;
          float4* wsb = reinterpret_cast<float4*>(sk.ws) + (size_t)sti * sk.splits * F4;
          float4* mine = wsb + (size_t)wi.part * F4;
#pragma unroll
          for (int c4 = 0; c4 < CPT / 4; ++c4)
            __stcg(mine + c4 * ET + et,
                   make_float4(acc[2 * c4].x, acc[2 * c4].y, acc[2 * c4 + 1].x, acc[2 * c4 + 1].y));
          __threadfence();
          auto epi_sync = [&]() -> bool {
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.split_bar);
            const bool ok = mbar_wait(&s.split_bar, split_phase, status, kErrTimeoutSplit, abort);
            split_phase ^= 1;
            return __all_sync(0xffffffffu, ok);
          };
          if (!epi_sync()) goto epi_done;
          if (et == 0) {
            int* arrive = sk.cnt + 2 * sti;
            __threadfence();
            atomicAdd(arrive, 1);
            bool ok = true;
            const uint64_t t0 = globaltimer();
            while (ld_acquire_gpu(arrive) < sk.splits) {
              if (*abort || globaltimer() - t0 > PHX_WAIT_TIMEOUT_NS) {
                ok = false;
                break;
              }
            }
            if (!ok) {
              atomicCAS(status, 0, kErrTimeoutSplit);
              *abort = 1;
            }
            s.split_ok = ok;
          }
          if (!epi_sync() || !s.split_ok) goto epi_done;
          __threadfence();
          const int lo = (int)((long long)wi.part * F4 / sk.splits);
          const int hi = (int)((long long)(wi.part + 1) * F4 / sk.splits);
          for (int f = lo + et; f < hi; f += ET) {
            float4 v = __ldcg(wsb + f);
            for (int q = 1; q < sk.splits; ++q) {
              const float4 u = __ldcg(wsb + (size_t)q * F4 + f);
              v.x += u.x;
              v.y += u.y;
              v.z += u.z;
              v.w += u.w;
            }
            const int e = f % ET, c4 = f / ET, eew = e >> 5;
            const int r = ti.m0 + ((eew + 2) & 3) * 32 + (e & 31);      // that thread's TMEM lane quarter
            const int c = ti.n0 + (eew >> 2) * CPT + 4 * c4;             // and column half
            if (r < M && c < N) {
              uint2 o;
              o.x = pack_bf16x2(v.x, v.y);
              o.y = pack_bf16x2(v.z, v.w);
              *reinterpret_cast<uint2*>(out + (size_t)r * ldc + c) = o;
            }
          }
          if (!epi_sync()) goto epi_done;   // this CTA's reads of the tile's partials are done
          if (et == 0) {
            __threadfence();
            if (atomicAdd(sk.cnt + 2 * sti + 1, 1) == sk.splits - 1) {   // last part out: reset for the next launch
              sk.cnt[2 * sti] = 0;
              sk.cnt[2 * sti + 1] = 0;
            }
          }
          continue;
        }
      }
      if constexpr (SWIGLU) {
        // up-half warps stage their rows' up values (bf16) in shared memory; gate-half warps combine them with
        // their gate values, quantize each row's 128 outputs and store them. Two mbarriers with bounded waits
        // hand the staging buffer back and forth (a timed-out wait abandons the tile loop, never hangs).
        constexpr int ROWB = scatter_row_bytes<BN>();
        uint8_t* st = reinterpret_cast<uint8_t*>(&s) + ((sizeof(Smem) + 127) & ~size_t(127));
        uint8_t* my_row = st + (size_t)(sub * 32 + lane) * ROWB;
        const uint32_t sphase = swg_iter & 1;
        if (half == 1) {
          // wait until the gate half has consumed the previous tile's rows
          const bool ok2 = swg_iter == 0 || mbar_wait(&s.up_free, sphase ^ 1, status, kErrTimeoutEpilogue, abort);
          if (!__all_sync(0xffffffffu, ok2)) goto epi_done;
#pragma unroll
          for (int c = 0; c < CPT / 8; ++c)
            *reinterpret_cast<uint4*>(my_row + c * 16) =
                make_uint4(pack_bf16x2(acc[4 * c + 0].x, acc[4 * c + 0].y), pack_bf16x2(acc[4 * c + 1].x, acc[4 * c + 1].y),
                           pack_bf16x2(acc[4 * c + 2].x, acc[4 * c + 2].y), pack_bf16x2(acc[4 * c + 3].x, acc[4 * c + 3].y));
          __syncwarp();
          if (lane == 0) mbar_arrive(&s.up_ready);
        } else {
          const bool ok2 = mbar_wait(&s.up_ready, sphase, status, kErrTimeoutEpilogue, abort);
          if (!__all_sync(0xffffffffu, ok2)) goto epi_done;
          float amax = 0.f;
#pragma unroll
          for (int c = 0; c < CPT / 8; ++c) {
            const uint4 uv = *reinterpret_cast<const uint4*>(my_row + c * 16);
            const uint32_t uw[4] = {uv.x, uv.y, uv.z, uv.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float2 g = unpack_bf16x2(pack_bf16x2(acc[4 * c + j].x, acc[4 * c + j].y));
              const float2 u = unpack_bf16x2(uw[j]);
              const float2 a = unpack_bf16x2(pack_bf16x2(g.x / (1.f + expf(-g.x)) * u.x, g.y / (1.f + expf(-g.y)) * u.y));
              acc[4 * c + j] = a;
              amax = fmaxf(amax, fmaxf(fabsf(a.x), fabsf(a.y)));
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&s.up_free);
          float inv;
          const float scale = fp8_block_scale(amax, &inv);
          if (row < ti.m_end && row < M) {
            const int oc = ti.n0 >> 1;   // output column block of this tile
            uint8_t* qrow = sw.q + (size_t)row * sw.F + oc;
#pragma unroll
            for (int c = 0; c < CPT / 16; ++c) {
              uint4 v;
              v.x = pack_fp8x4(acc[8 * c + 0].x * inv, acc[8 * c + 0].y * inv, acc[8 * c + 1].x * inv, acc[8 * c + 1].y * inv);
              v.y = pack_fp8x4(acc[8 * c + 2].x * inv, acc[8 * c + 2].y * inv, acc[8 * c + 3].x * inv, acc[8 * c + 3].y * inv);
              v.z = pack_fp8x4(acc[8 * c + 4].x * inv, acc[8 * c + 4].y * inv, acc[8 * c + 5].x * inv, acc[8 * c + 5].y * inv);
              v.w = pack_fp8x4(acc[8 * c + 6].x * inv, acc[8 * c + 6].y * inv, acc[8 * c + 7].x * inv, acc[8 * c + 7].y * inv);
              *reinterpret_cast<uint4*>(qrow + c * 16) = v;
            }
            sw.qs[(size_t)(oc >> 7) * M + row] = scale;
          }
        }
        ++swg_iter;
      } else if constexpr (SCATTER) {
        // each lane stages its row's BN/2 bf16 columns in shared memory and hands them to the TMA engine as one
        // bulk copy into the row's owner receive slot (over NVLink for a peer): the NVLink writes drain
        // asynchronously while the epilogue moves on to the next tile (lane-issued 16-byte peer stores kept
        // the epilogue warps waiting on remote-store issue). A lane rewrites its staging row only after its
        // previous copy has read it.
        constexpr int ROWB = scatter_row_bytes<BN>();
        uint8_t* st = reinterpret_cast<uint8_t*>(&s) + ((sizeof(Smem) + 127) & ~size_t(127)) + (size_t)ew * 32 * ROWB;
        uint8_t* my_st = st + (size_t)lane * ROWB;
        if (sc.bulk) bulk_wait_read0();
#pragma unroll
        for (int c = 0; c < CPT / 8; ++c) {
          uint4 v;
          v.x = pack_bf16x2(acc[4 * c + 0].x, acc[4 * c + 0].y);
          v.y = pack_bf16x2(acc[4 * c + 1].x, acc[4 * c + 1].y);
          v.z = pack_bf16x2(acc[4 * c + 2].x, acc[4 * c + 2].y);
          v.w = pack_bf16x2(acc[4 * c + 3].x, acc[4 * c + 3].y);
          *reinterpret_cast<uint4*>(my_st + c * 16) = v;
        }
        if (sc.bulk) {
          fence_proxy_async_smem();
          if (row < ti.m_end && row < M && col_ok) {
            const int owner = row / sc.rows_per;
            __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(sc.peer_base[owner] + sc.off_recv) +
                                 ((size_t)sc.rank * sc.rows_per + (row - owner * sc.rows_per)) * ldc + col0;
            const int ncols = N - col0 < CPT ? N - col0 : CPT;     // N % 8 == 0: a multiple of 16 bytes
            bulk_store(dst, my_st, (uint32_t)ncols * 2);
            bulk_commit();
          }
        } else {
          // the warp's 32 staged rows stored row-contiguously (2 or 4 rows per warp instruction)
          __syncwarp();
          constexpr int CH = CPT / 8;      // 16-byte chunks per staged row
          constexpr int RPI = 32 / CH;     // rows per warp instruction
#pragma unroll 4
          for (int it = 0; it < 32 / RPI; ++it) {
            const int rl = it * RPI + lane / CH, ch = lane % CH;
            const int grow = ti.m0 + my_row0 + sub * 32 + rl, gcol = col0 + ch * 8;
            if (grow < ti.m_end && grow < M && gcol < N) {
              const int owner = grow / sc.rows_per;
              __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(sc.peer_base[owner] + sc.off_recv) +
                                   ((size_t)sc.rank * sc.rows_per + (grow - owner * sc.rows_per)) * ldc + gcol;
              *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(st + rl * ROWB + ch * 16);
            }
          }
          __syncwarp();
        }
      } else if (row < ti.m_end && row < M && col_ok) {
        __nv_bfloat16* dst = out + (size_t)row * ldc + col0;
        const bool full_cols = col0 + CPT <= N;
#pragma unroll
        for (int c = 0; c < CPT / 8; ++c) {
          if (!full_cols && col0 + 8 * c >= N) break;
          uint4 v;
          v.x = pack_bf16x2(acc[4 * c + 0].x, acc[4 * c + 0].y);
          v.y = pack_bf16x2(acc[4 * c + 1].x, acc[4 * c + 1].y);
          v.z = pack_bf16x2(acc[4 * c + 2].x, acc[4 * c + 2].y);
          v.w = pack_bf16x2(acc[4 * c + 3].x, acc[4 * c + 3].y);
          *reinterpret_cast<uint4*>(dst + 8 * c) = v;
        }
      }
    }
  epi_done:;
    if (SCATTER) {
      if (sc.bulk) bulk_wait0();   // this lane's bulk copies have landed
      __threadfence_system();    // peer stores ordered before the reduction's release flags
    }
  }

  tc_fence_before();
  if constexpr (PAIR) cluster_sync();   // the leader's MMAs into the peer's TMEM and reads of its smem are done
  else __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    if constexpr (PAIR) tmem_dealloc_pair(tmem_base, TMEM_COLS);
    else tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------------------------------------
// host
// ------------------------------------------------------------------------------------------------
int num_sms() {
  static int n = 0;
  if (!n) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

// Parts per split tile of the split-K tail (1: no split). req: 0 = automatic, 1 = off, >= 2 = that many parts
// (clamped). Automatic: split when the last wave of tiles leaves at least half the SMs idle and the tile has
// at least 16 K steps (shorter tiles do not repay the partial-tile round trip through L2).
static int split_parts(int tiles, int ksteps, int P, int req) {
  const int rem = tiles % P;
  if (req == 1 || rem == 0) return 1;
  int parts = req >= 2 ? req : (ksteps >= 16 ? P / rem : 1);
  parts = std::min(parts, P / rem);                 // every split item in the grid's last round
  parts = std::min(parts, ksteps / 2);              // at least two K steps per part
  parts = std::min(parts, kMaxSplitItems / rem);    // workspace
  return parts >= 2 ? parts : 1;
}

// This device's copy of the split-K workspace (the device symbols' addresses in the current context).
static SplitArgs split_workspace(int dev) {
  static float* ws[64] = {};
  static int* cnt[64] = {};
  if (!ws[dev]) {
    void* a = nullptr;
    void* c = nullptr;
    C10_CUDA_CHECK(cudaGetSymbolAddress(&a, g_split_ws));
    C10_CUDA_CHECK(cudaGetSymbolAddress(&c, g_split_cnt));
    cnt[dev] = static_cast<int*>(c);
    ws[dev] = static_cast<float*>(a);
  }
  return SplitArgs{ws[dev], cnt[dev], 0, 1};
}

template <int BN, bool FP8, bool SCATTER = false, bool HWS = false, bool PAIR = false, bool SWIGLU = false>
void launch_gemm_ptr(const torch::Tensor& a, const torch::Tensor& b, __nv_bfloat16* out_ptr, int ldc, int n_out,
                     const float* sa, const float* sb, int* status, cudaStream_t stream, int max_ctas,
                     const int* grp_off, int groups, ScatterArgs sc, const int* a_rows = nullptr, int m_rows = 0,
                     SwigluArgs sw = SwigluArgs{nullptr, nullptr, 0}, int split = 1) {
  static_assert(!PAIR || HWS, "CTA pairs run the hardware-scaled kernel");
  // a_rows: GEMM row r reads activation row a_rows[r] (m_rows GEMM rows; `a` holds the activations and `sa`
  // their scales [K/128, a.size(0)]); A is fetched by TMA gather4 with a one-row box
  TORCH_CHECK(!a_rows || (HWS && !PAIR), "row-gathered A needs the hardware-scaled single-CTA kernel");
  const int M = a_rows ? m_rows : (int)a.size(0), K = a.size(1);
  const int sa_ld = (int)a.size(0);
  const int N = grp_off ? n_out : (int)b.size(0);   // grouped: b holds groups * N rows
  const CUtensorMapDataType dt = FP8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const int esz = FP8 ? 1 : 2;
  const uint32_t box_inner = 128 / esz;
  CUtensorMap ta = make_tmap_2d(a.data_ptr(), dt, K, a.size(0), (uint64_t)a.stride(0) * esz, box_inner,
                                a_rows ? 1 : kBM, CU_TENSOR_MAP_SWIZZLE_128B);
  constexpr int BROWS = PAIR ? BN / 2 : BN;
  CUtensorMap tb = make_tmap_2d(b.data_ptr(), dt, K, b.size(0), (uint64_t)b.stride(0) * esz, box_inner, BROWS,
                                CU_TENSOR_MAP_SWIZZLE_128B);
  constexpr int STAGES = gemm_stages<BN, SCATTER || SWIGLU, PAIR>();
  const size_t smem = ((sizeof(GemmSmem<BN, STAGES, HWS, BROWS>) + 127) & ~size_t(127)) + 1024 +
                      ((SCATTER || SWIGLU) ? (size_t)kEpiWarps * 32 * scatter_row_bytes<BN>() : 0);
  auto kern = gemm_sm100_kernel<BN, FP8, SCATTER, HWS, PAIR, SWIGLU>;
  // per device: a process may drive several GPUs (the attribute belongs to each device's context)
  int dev = 0;
  cudaGetDevice(&dev);
  static bool attr_set[64] = {};
  TORCH_CHECK(dev < 64, "device index out of range");
  if (!attr_set[dev]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attr_set[dev] = true;
  }
  constexpr int BMT = PAIR ? 2 * kBM : kBM;
  // grouped: at most M/128 + groups row tiles in total (one partial tile per group)
  const int m_tiles_bound = grp_off ? (M + BMT - 1) / BMT + groups : (M + BMT - 1) / BMT;
  const int tiles = m_tiles_bound * ((N + BN - 1) / BN);
  if constexpr (PAIR) {
    // clusters of two CTAs; as many pairs as can be resident at once (a GPC with an odd SM count leaves one
    // SM out), each walking tiles persistently
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    static int max_pairs_dev[64] = {};
    int& max_pairs = max_pairs_dev[dev];
    if (!max_pairs) {
      cfg.gridDim = dim3(2 * (num_sms() / 2));
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
        (void)cudaGetLastError();
        n = num_sms() / 2 - 4;
      }
      max_pairs = n;
    }
    int pairs = std::min(tiles, max_ctas > 0 ? std::max(1, max_ctas / 2) : max_pairs);
    cfg.gridDim = dim3(2 * pairs);
    C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, ta, tb, out_ptr, M, N, K, ldc, sa, sb, status, grp_off, groups,
                                      tiles, sc, a_rows, sa_ld, sw, SplitArgs{nullptr, nullptr, 0, 1}));
  } else {
    // split-K tail: plain GEMMs with bf16 output and the whole K range in TMEM (bf16, hardware-scaled fp8)
    SplitArgs sk{nullptr, nullptr, 0, 1};
    int items = tiles;
    constexpr bool kCanSplit = !SCATTER && !SWIGLU && (HWS || !FP8);
    if (kCanSplit && !grp_off && !a_rows && max_ctas <= 0 && split != 1) {
      const int P = num_sms();
      const int parts = split_parts(tiles, K / (FP8 ? 128 : 64), P, split);
      if (parts > 1) {
        const int rem = tiles % P;
        sk = split_workspace(dev);
        sk.dp_tiles = tiles - rem;
        sk.splits = parts;
        items = tiles - rem + rem * parts;
      }
    }
    int grid = std::min(items, max_ctas > 0 ? max_ctas : num_sms());
    kern<<<grid, kGemmThreads, smem, stream>>>(ta, tb, out_ptr, M, N, K, ldc, sa, sb, status, grp_off, groups, tiles,
                                               sc, a_rows, sa_ld, sw, sk);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
}

template <int BN, bool FP8, bool HWS = false, bool PAIR = false>
void launch_gemm(const torch::Tensor& a, const torch::Tensor& b, torch::Tensor& out, const float* sa,
                 const float* sb, int* status, cudaStream_t stream, int max_ctas, const int* grp_off = nullptr,
                 int groups = 0, int split = 1) {
  launch_gemm_ptr<BN, FP8, false, HWS, PAIR>(a, b, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), (int)out.stride(0),
                           (int)out.size(1), sa, sb, status, stream, max_ctas, grp_off, groups,
                           ScatterArgs{nullptr, 0, 1, 0, 0}, nullptr, 0, SwigluArgs{nullptr, nullptr, 0}, split);
}

// Hardware scaling with 256-wide tiles leaves TMEM room for one accumulator only, so the epilogue drain is
// not overlapped with the next tile; with at most 16 K blocks per tile that drain is a large share of the
// tile and the two-accumulator promotion path is faster (o_proj at TP8, K = 1024: 0.068 vs 0.072 ms).
static bool prefer_promote(int bn, int K) { return bn == 256 && K / 128 <= 16; }

static int pick_bn(int M, int N) {
  // BN=256 halves the A-operand shared-memory traffic per FLOP; use 128 when 256 leaves SMs idle or when
  // the padded columns of a partial last 256-wide tile exceed an eighth of N (a vocab shard of 16032
  // columns pads 96: 256 stays, measured 0.61 -> 0.39 ms at 4096 x 16032 x 4096).
  if (N <= 128 || (N % 256 != 0 && (256 - N % 256) * 8 > N)) return 128;
  const long tiles256 = (long)((M + 127) / 128) * ((N + 255) / 256);
  if (tiles256 < num_sms() && (long)((M + 127) / 128) * (N / 128) <= 2L * num_sms()) return 128;
  return 256;
}

// hws: the tensor core applies the (power-of-two) block scales; otherwise the epilogue promotes per K block.
// pair: run 256 x 256 tiles on CTA pairs (hardware scaling, BN = 256, more than one 128-row block)
// split: split-K tail parts (0 automatic, 1 off, >= 2 requested; hardware-scaled single-CTA tiles only)
void gemm_fp8_block(torch::Tensor xq, torch::Tensor xs, torch::Tensor wq, torch::Tensor ws, torch::Tensor out,
                    torch::Tensor status, int64_t bn, int64_t max_ctas, bool hws, bool pair, int64_t split) {
  TORCH_CHECK(xq.is_cuda() && wq.is_cuda() && out.is_cuda());
  TORCH_CHECK(xq.scalar_type() == at::kFloat8_e4m3fn && wq.scalar_type() == at::kFloat8_e4m3fn);
  TORCH_CHECK(out.scalar_type() == at::kBFloat16);
  TORCH_CHECK(xs.scalar_type() == at::kFloat && ws.scalar_type() == at::kFloat);
  const int M = xq.size(0), K = xq.size(1), N = wq.size(0);
  TORCH_CHECK(wq.size(1) == K && K % 128 == 0 && N % 8 == 0, "gemm_fp8_block: K % 128 and N % 8 must be 0");
  TORCH_CHECK(xq.stride(1) == 1 && wq.stride(1) == 1 && out.stride(1) == 1);
  TORCH_CHECK(xs.is_contiguous() && xs.size(0) == K / 128 && xs.size(1) == M, "xs must be [K/128, M]");
  TORCH_CHECK(ws.is_contiguous() && ws.size(0) == (N + 127) / 128 && ws.size(1) == K / 128,
              "ws must be [ceil(N/128), K/128]");
  TORCH_CHECK(out.size(0) == M && out.size(1) == N);
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(xq.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const int b = bn > 0 ? (int)bn : pick_bn(M, N);
  const float* sa = xs.data_ptr<float>();
  const float* sb = ws.data_ptr<float>();
  int* st = status.data_ptr<int>();
  if (hws && !pair && bn <= 0 && prefer_promote(b, K)) hws = false;
  if (hws) {
    if (b == 256 && pair && M > kBM) launch_gemm<256, true, true, true>(xq, wq, out, sa, sb, st, stream, (int)max_ctas);
    else if (b == 256) launch_gemm<256, true, true>(xq, wq, out, sa, sb, st, stream, (int)max_ctas, nullptr, 0, (int)split);
    else launch_gemm<128, true, true>(xq, wq, out, sa, sb, st, stream, (int)max_ctas, nullptr, 0, (int)split);
  } else {
    if (b == 256) launch_gemm<256, true>(xq, wq, out, sa, sb, st, stream, (int)max_ctas);
    else launch_gemm<128, true>(xq, wq, out, sa, sb, st, stream, (int)max_ctas);
  }
}

// Gate/up projection with the SwiGLU + FP8 quant epilogue (see SwigluArgs): wq / ws hold the gate and up
// weights interleaved in 128-row blocks ([2F, K] / [2F/128, K/128]); q [M, F] e4m3 and qs [F/128, M] fp32 out.
void gemm_fp8_swiglu(torch::Tensor xq, torch::Tensor xs, torch::Tensor wq, torch::Tensor ws, torch::Tensor q,
                     torch::Tensor qs, torch::Tensor status) {
  TORCH_CHECK(xq.is_cuda() && xq.scalar_type() == at::kFloat8_e4m3fn && wq.scalar_type() == at::kFloat8_e4m3fn);
  TORCH_CHECK(q.scalar_type() == at::kFloat8_e4m3fn && q.is_contiguous() && qs.scalar_type() == at::kFloat &&
              qs.is_contiguous());
  const int M = xq.size(0), K = xq.size(1), N = wq.size(0), F = N / 2;
  TORCH_CHECK(wq.size(1) == K && K % 128 == 0 && N % 256 == 0, "gemm_fp8_swiglu: K % 128 == 0, 2F % 256 == 0");
  TORCH_CHECK(xq.stride(1) == 1 && wq.stride(1) == 1 && xs.is_contiguous() && xs.size(0) == K / 128 && xs.size(1) == M);
  TORCH_CHECK(ws.is_contiguous() && ws.size(0) == N / 128 && ws.size(1) == K / 128);
  TORCH_CHECK(q.size(0) == M && q.size(1) == F && qs.size(0) == F / 128 && qs.size(1) == M);
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(xq.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  launch_gemm_ptr<256, true, false, true, false, true>(
      xq, wq, nullptr, N, N, xs.data_ptr<float>(), ws.data_ptr<float>(), status.data_ptr<int>(), stream, 0, nullptr,
      0, ScatterArgs{nullptr, 0, 1, 0, 0}, nullptr, 0,
      SwigluArgs{reinterpret_cast<uint8_t*>(q.data_ptr()), qs.data_ptr<float>(), F});
}

// Grouped block-scaled FP8 GEMM (MoE experts): GEMM rows sorted by group, group e = rows
// [offsets[e], offsets[e+1]) (device int32 [G+1]); wq [G*N, K]; ws [G*ceil(N/128), K/128]; out [Mtot, N].
// rows (optional, int32 [Mtot], hardware-scaled path): GEMM row r is xq row rows[r] and takes that row's
// scales from xs [K/128, xq.size(0)], so the expert dispatch (token gather) happens inside the A loads;
// without rows, xq [Mtot, K] is already in GEMM row order. Measured at Mixtral EP8 shapes (2048 rows per
// expert, N = 28672, K = 4096): 0.636 ms with rows vs 0.280 ms for a gather copy + the plain grouped GEMM --
// 32 gather4 TMA operations per stage (and per N tile) bound the producer -- so the MoE block gathers once.
void gemm_fp8_grouped(torch::Tensor xq, torch::Tensor xs, torch::Tensor wq, torch::Tensor ws, torch::Tensor offsets,
                      torch::Tensor out, torch::Tensor status, bool hws, c10::optional<torch::Tensor> rows) {
  TORCH_CHECK(xq.scalar_type() == at::kFloat8_e4m3fn && wq.scalar_type() == at::kFloat8_e4m3fn);
  TORCH_CHECK(offsets.scalar_type() == at::kInt && offsets.is_cuda() && offsets.dim() == 1);
  const int M = rows ? (int)rows->size(0) : (int)xq.size(0), K = xq.size(1), N = out.size(1), G = offsets.size(0) - 1;
  TORCH_CHECK(G >= 1 && wq.size(0) == (int64_t)G * N && wq.size(1) == K && K % 128 == 0 && N % 8 == 0);
  TORCH_CHECK(ws.size(0) == (int64_t)G * ((N + 127) / 128) && ws.size(1) == K / 128);
  TORCH_CHECK(xs.size(0) == K / 128 && xs.size(1) == xq.size(0) && out.size(0) == M);
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(xq.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  if (rows) {
    TORCH_CHECK(hws && rows->scalar_type() == at::kInt && rows->is_cuda() && rows->is_contiguous(),
                "row-gathered grouped GEMM: hardware scaling and int32 rows");
    TORCH_CHECK(xq.stride(1) == 1 && xs.is_contiguous());
    launch_gemm_ptr<256, true, false, true>(xq, wq, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
                                            (int)out.stride(0), N, xs.data_ptr<float>(), ws.data_ptr<float>(),
                                            status.data_ptr<int>(), stream, 0, offsets.data_ptr<int>(), G,
                                            ScatterArgs{nullptr, 0, 1, 0, 0}, rows->data_ptr<int>(), M);
  } else if (hws)
    launch_gemm<256, true, true>(xq, wq, out, xs.data_ptr<float>(), ws.data_ptr<float>(), status.data_ptr<int>(),
                                 stream, 0, offsets.data_ptr<int>(), G);
  else
    launch_gemm<256, true>(xq, wq, out, xs.data_ptr<float>(), ws.data_ptr<float>(), status.data_ptr<int>(), stream, 0,
                           offsets.data_ptr<int>(), G);
}

// Grouped bf16 GEMM (bf16 MoE experts); same layout as gemm_fp8_grouped without scales.
void gemm_bf16_grouped(torch::Tensor x, torch::Tensor w, torch::Tensor offsets, torch::Tensor out,
                       torch::Tensor status) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16);
  TORCH_CHECK(offsets.scalar_type() == at::kInt && offsets.is_cuda() && offsets.dim() == 1);
  const int M = x.size(0), K = x.size(1), N = out.size(1), G = offsets.size(0) - 1;
  TORCH_CHECK(G >= 1 && w.size(0) == (int64_t)G * N && w.size(1) == K && K % 64 == 0 && N % 8 == 0);
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  launch_gemm<256, false>(x, w, out, nullptr, nullptr, status.data_ptr<int>(), stream, 0, offsets.data_ptr<int>(), G);
}

void gemm_bf16(torch::Tensor x, torch::Tensor w, torch::Tensor out, torch::Tensor status, int64_t bn,
               int64_t max_ctas, int64_t split) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 &&
              out.scalar_type() == at::kBFloat16);
  const int M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K && K % 64 == 0 && N % 8 == 0, "gemm_bf16: K % 64 and N % 8 must be 0");
  TORCH_CHECK(x.stride(1) == 1 && w.stride(1) == 1 && out.stride(1) == 1);
  TORCH_CHECK(out.size(0) == M && out.size(1) == N);
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const int b = bn > 0 ? (int)bn : pick_bn(M, N);
  if (b == 256)
    launch_gemm<256, false>(x, w, out, nullptr, nullptr, status.data_ptr<int>(), stream, (int)max_ctas, nullptr, 0,
                            (int)split);
  else
    launch_gemm<128, false>(x, w, out, nullptr, nullptr, status.data_ptr<int>(), stream, (int)max_ctas, nullptr, 0,
                            (int)split);
}

// Row-parallel projection with the scatter epilogue (see ScatterArgs): fp8 (ws defined) or bf16 operands.
void gemm_scatter(torch::Tensor x, c10::optional<torch::Tensor> xs, torch::Tensor w, c10::optional<torch::Tensor> ws,
                  torch::Tensor peer_base, int64_t off_recv, int64_t rows_per, int64_t rank, torch::Tensor status,
                  bool hws, bool pair, int64_t bn, bool bulk) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && peer_base.is_cuda() && peer_base.scalar_type() == at::kLong);
  const int M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K && N % 8 == 0 && x.stride(1) == 1 && w.stride(1) == 1);
  TORCH_CHECK(rows_per > 0 && (int64_t)rows_per * peer_base.numel() >= M);
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(x.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const ScatterArgs sc{reinterpret_cast<const uint64_t*>(peer_base.data_ptr<int64_t>()), (uint64_t)off_recv,
                       (int)rows_per, (int)rank, bulk ? 1 : 0};
  const int b = bn > 0 ? (int)bn : pick_bn(M, N);
  if (ws.has_value()) {
    TORCH_CHECK(x.scalar_type() == at::kFloat8_e4m3fn && w.scalar_type() == at::kFloat8_e4m3fn && K % 128 == 0);
    TORCH_CHECK(xs->is_contiguous() && xs->size(0) == K / 128 && xs->size(1) == M);
    TORCH_CHECK(ws->is_contiguous() && ws->size(0) == (N + 127) / 128 && ws->size(1) == K / 128);
    const float* sa = xs->data_ptr<float>();
    const float* sb = ws->data_ptr<float>();
    int* st = status.data_ptr<int>();
    if (hws && !pair && bn <= 0 && prefer_promote(b, K)) hws = false;
    if (hws) {
      if (b == 256 && pair && M > kBM)
        launch_gemm_ptr<256, true, true, true, true>(x, w, nullptr, N, N, sa, sb, st, stream, 0, nullptr, 0, sc);
      else if (b == 256) launch_gemm_ptr<256, true, true, true>(x, w, nullptr, N, N, sa, sb, st, stream, 0, nullptr, 0, sc);
      else launch_gemm_ptr<128, true, true, true>(x, w, nullptr, N, N, sa, sb, st, stream, 0, nullptr, 0, sc);
    } else {
      if (b == 256) launch_gemm_ptr<256, true, true>(x, w, nullptr, N, N, sa, sb, st, stream, 0, nullptr, 0, sc);
      else launch_gemm_ptr<128, true, true>(x, w, nullptr, N, N, sa, sb, st, stream, 0, nullptr, 0, sc);
    }
  } else {
    TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 && K % 64 == 0);
    if (b == 256)
      launch_gemm_ptr<256, false, true>(x, w, nullptr, N, N, nullptr, nullptr, status.data_ptr<int>(), stream, 0, nullptr, 0,
                                  sc);
    else
      launch_gemm_ptr<128, false, true>(x, w, nullptr, N, N, nullptr, nullptr, status.data_ptr<int>(), stream, 0, nullptr, 0,
                                  sc);
  }
}

}  // namespace phx
