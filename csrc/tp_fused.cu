// Fused tensor-parallel reduction + residual add + RMSNorm + block-FP8 quantization over NVLink peer memory.
//
// After a row-parallel projection (o_proj, down_proj) every rank holds a bf16 partial sum [M, H] in its
// symmetric workspace. One launch of tp_ar_norm_kernel replaces "NCCL all-reduce, then add+RMSNorm+quant":
//   1. start barrier: each rank publishes `epoch` into slot [0][rank] of every peer's flag array
//      (st.release.sys) and waits until all peers' flags in its own array reach `epoch` (ld.acquire.sys);
//   2. rank r owns rows [r*ceil(M/W), ...): for each row, a CTA loads the W peers' partial rows (P2P loads,
//      16 bytes per thread per peer in flight), sums in fp32, rounds the sum to bf16 (as a bf16 all-reduce
//      result), adds the residual, RMSNorm (block reduction), and quantizes to e4m3 with one fp32 scale per
//      128 channels — or emits the normalized row in bf16 (final norm, bf16 models);
//   3. pushes the new residual row, the fp8 row and its scales (or the bf16 row) into EVERY rank's
//      workspace with P2P stores (a reduce-scatter + all-gather, fused with the normalization);
//   4. end barrier: the last CTA to finish (device atomic counter) publishes slot [1][rank] to all peers
//      and waits for theirs, so no rank's next GEMM overwrites a partial a peer is still reading, and
//      every rank's outputs are complete when the kernel retires.
// Every spin is bounded by a %globaltimer deadline; on expiry the kernel records kErrTimeoutPeer and
// skips its work instead of hanging.
// Epochs live on the device (a word next to the CTA counter): every CTA reads epoch = word + 1 at entry and
// the last CTA stores it after the end barrier, so launches captured in a CUDA graph advance the barrier
// protocol on every replay exactly as eager launches do.
// The residual h is only read by the rank that owns a row, so it is pushed to the peers only when asked
// (push_h: the last layer, when the caller needs the full pre-norm hidden state).
// tp_allgather_kernel uses the same barriers to copy a small staging block of every rank into slot
// [rank] of every peer's gather region (vocab-sharded top-k / argmax candidates).
// The reference has no tensor parallelism (configuration.yaml: tensor_parallel_size 1 everywhere); this is
// the fused "GEMM -> reduce-scatter -> +residual -> RMSNorm -> FP8 quant -> all-gather" path of the
// B200 design (the all-gather pushes the quantized rows the next GEMM consumes).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <map>
#include <mutex>
#include <type_traits>
#include <utility>

#include "common.cuh"

namespace phx {

struct TpArgs {
  const uint64_t* peer_base;  // [W] base address of every rank's workspace (device array)
  int rank, world, M, H;
  float eps;
  const __nv_bfloat16* w;     // norm weight [H], local
  int out_bf16;               // 0: fp8 q + scales, 1: bf16 y
  int push_h;                 // 1: store the new residual rows into every rank's h (else only locally)
  int recv;                   // 1: partials were pushed into this rank's receive slots (gemm_scatter); 0: pull
  uint64_t off_recv;          // receive buffer [W][rows_per][H] bf16
  int* status;
  // byte offsets inside the workspace
  uint64_t off_partial, off_h, off_y, off_q, off_s, off_flags, off_counter;
  int s_ld;                   // row stride (elements) of the scale matrix [H/128, s_ld]
  uint64_t mc_base;           // multicast (NVLS) address of the workspace, 0 = none: see tp_ar_norm_kernel
  // optional phase timer [4] (ns sums over launches): start-barrier wait and row work summed over CTAs, the
  // last CTA's end barrier, CTA count
  unsigned long long* phase_ns;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// NVLS (NVLink SHARP) multimem accesses through the workspace's multicast address: one load returns the
// sum of the W ranks' copies (reduced in the switch with fp32 accumulation, rounded once to bf16, as the
// peer-load path rounds its fp32 sum), one store writes every rank's copy.
__device__ __forceinline__ uint4 mm_ld_reduce_bf16x8(const void* mc) {
  uint4 r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(mc)
               : "memory");
  return r;
}
__device__ __forceinline__ void mm_st16(void* mc, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(mc), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void mm_st8(void* mc, uint2 v) {
  asm volatile("multimem.st.relaxed.sys.global.v2.f32 [%0], {%1,%2};" ::"l"(mc), "r"(v.x), "r"(v.y) : "memory");
}
__device__ __forceinline__ void mm_st4(void* mc, uint32_t v) {
  asm volatile("multimem.st.relaxed.sys.global.f32 [%0], %1;" ::"l"(mc), "r"(v) : "memory");
}

// wait until flags[slot0 + i] >= epoch for i < W (threads 0..W-1 each poll one); false on timeout
__device__ __forceinline__ bool wait_flags(const uint32_t* flags, int W, uint32_t epoch, int* status) {
  __shared__ int fail;
  if (threadIdx.x == 0) fail = 0;
  __syncthreads();
  if (threadIdx.x < W) {
    const uint64_t t0 = globaltimer();
    while ((int32_t)(ld_acquire_sys(flags + threadIdx.x) - epoch) < 0) {
      if (globaltimer() - t0 > PHX_WAIT_TIMEOUT_NS) {
        atomicCAS(status, 0, kErrTimeoutPeer);
        fail = 1;
        break;
      }
    }
  }
  __syncthreads();
  return fail == 0;
}

// end barrier: the last CTA of this rank's launch publishes slot [1][rank] to every peer, waits for all
// peers' slot [1], then stores the epoch for the next launch (all CTAs of this launch have read it).
__device__ __forceinline__ void end_barrier(uint8_t* mine, uint64_t off_flags, uint64_t off_counter, uint32_t epoch,
                                            int W, int rank, const uint64_t* peer_base, int* status,
                                            unsigned long long* phase_ns = nullptr) {
  __shared__ int is_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    unsigned int* cnt = reinterpret_cast<unsigned int*>(mine + off_counter);
    const unsigned int old = atomicAdd(cnt, 1u);
    is_last = old == gridDim.x - 1;
    if (is_last) *cnt = 0;  // the next launch starts after this one retires
  }
  __syncthreads();
  if (is_last) {
    const uint64_t t0 = phase_ns ? globaltimer() : 0;
    uint32_t* my_flags = reinterpret_cast<uint32_t*>(mine + off_flags);
    if (threadIdx.x < W) {
      __threadfence_system();
      st_release_sys(reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(peer_base[threadIdx.x]) + off_flags) +
                         W + rank,
                     epoch);
    }
    wait_flags(my_flags + W, W, epoch, status);
    if (threadIdx.x == 0) reinterpret_cast<volatile uint32_t*>(mine + off_counter)[1] = epoch;
    if (phase_ns && threadIdx.x == 0) atomicAdd(&phase_ns[2], (unsigned long long)(globaltimer() - t0));
  }
}

// WT: the world size as a compile-time constant (2, 4, 8) so the W peer loads of a 16-byte chunk are all
// issued before the first is consumed; 0 = runtime world size.
// NV: the reduce-scatter (pull mode) is one multimem.ld_reduce per 16 bytes (the switch sums the W partials in
// fp32 and rounds to bf16) and the all-gather of the results is one multimem.st per 16/8/4 bytes instead of W peer stores.
template <int MAXC, int WT, bool NV>
__global__ void __launch_bounds__(256) tp_ar_norm_kernel(const TpArgs a) {
  __shared__ float red[32];
  const int W = WT > 0 ? WT : a.world;
  auto base = [&](int p) { return reinterpret_cast<uint8_t*>(a.peer_base[p]); };
  uint8_t* const mc = reinterpret_cast<uint8_t*>(a.mc_base);
  uint8_t* mine = base(a.rank);
  uint32_t* my_flags = reinterpret_cast<uint32_t*>(mine + a.off_flags);
  uint32_t* epoch_word = reinterpret_cast<uint32_t*>(mine + a.off_counter) + 1;
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(epoch_word) + 1u;

  // ---- 1. start barrier ----
  const uint64_t t_entry = a.phase_ns ? globaltimer() : 0;
  if (blockIdx.x == 0 && threadIdx.x < W) {
    __threadfence_system();
    st_release_sys(reinterpret_cast<uint32_t*>(base(threadIdx.x) + a.off_flags) + a.rank, epoch);
  }
  const bool ok = wait_flags(my_flags, W, epoch, a.status);
  const uint64_t t_start = a.phase_ns ? globaltimer() : 0;

  // ---- 2./3. reduce my rows, normalize, push to every rank ----
  const int H = a.H, nch = H / 8;
  const int rows_per = (a.M + W - 1) / W;
  const int r0 = a.rank * rows_per, r1 = min(a.M, r0 + rows_per);
  for (int row = r0 + blockIdx.x; ok && row < r1; row += gridDim.x) {
    float x[MAXC][8];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int c = threadIdx.x + i * blockDim.x;
      if (c < nch) {
        float acc[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = 0.f;
        const size_t off = ((size_t)row * H + c * 8) * 2;
        auto add = [&](const uint4 v) {
          const uint32_t vw[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = unpack_bf16x2(vw[e]);
            acc[2 * e] += f.x;
            acc[2 * e + 1] += f.y;
          }
        };
        // source of rank p's partial of this row: its pushed copy in my receive slot p, or its partial buffer
        const size_t roff = ((size_t)(row - r0) * H + c * 8) * 2, rstride = (size_t)rows_per * H * 2;
        auto src = [&](int p) -> const uint4* {
          return a.recv ? reinterpret_cast<const uint4*>(mine + a.off_recv + p * rstride + roff)
                        : reinterpret_cast<const uint4*>(base(p) + a.off_partial + off);
        };
        if (NV && !a.recv) {
          add(mm_ld_reduce_bf16x8(mc + a.off_partial + off));
        } else if constexpr (WT > 0) {
          uint4 v[WT];
#pragma unroll
          for (int p = 0; p < WT; ++p) v[p] = *src(p);
#pragma unroll
          for (int p = 0; p < WT; ++p) add(v[p]);
        } else {
          for (int p = 0; p < W; ++p) add(*src(p));
        }
        const uint4 hv = *reinterpret_cast<const uint4*>(mine + a.off_h + off);
        const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w};
        uint32_t nh[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          // all-reduce result rounded to bf16, then the bf16 residual add (the unfused path's rounding)
          const float2 o = unpack_bf16x2(pack_bf16x2(acc[2 * e], acc[2 * e + 1]));
          const float2 h = unpack_bf16x2(hw[e]);
          nh[e] = pack_bf16x2(h.x + o.x, h.y + o.y);
          const float2 r = unpack_bf16x2(nh[e]);
          x[i][2 * e] = r.x;
          x[i][2 * e + 1] = r.y;
          ss += r.x * r.x + r.y * r.y;
        }
        const uint4 out = make_uint4(nh[0], nh[1], nh[2], nh[3]);
        if (a.push_h && NV)
          mm_st16(mc + a.off_h + off, out);
        else if (a.push_h)
          for (int p = 0; p < W; ++p) *reinterpret_cast<uint4*>(base(p) + a.off_h + off) = out;
        else
          *reinterpret_cast<uint4*>(mine + a.off_h + off) = out;
      }
    }
    // RMSNorm statistics
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += red[i];
    __syncthreads();
    const float inv = rsqrtf(tot / (float)H + a.eps);
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int c = threadIdx.x + i * blockDim.x;
      const bool valid = c < nch;
      float y[8];
      if (valid) {
        const uint4 wv = *reinterpret_cast<const uint4*>(a.w + c * 8);
        const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = unpack_bf16x2(ww[e]);
          y[2 * e] = x[i][2 * e] * inv * f.x;
          y[2 * e + 1] = x[i][2 * e + 1] * inv * f.y;
        }
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) y[e] = 0.f;
      }
      if (a.out_bf16) {
        if (valid) {
          const uint4 out = make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]), pack_bf16x2(y[4], y[5]),
                                       pack_bf16x2(y[6], y[7]));
          const size_t off = ((size_t)row * H + c * 8) * 2;
          if constexpr (NV)
            mm_st16(mc + a.off_y + off, out);
          else
            for (int p = 0; p < W; ++p) *reinterpret_cast<uint4*>(base(p) + a.off_y + off) = out;
        }
      } else if (__any_sync(0xffffffffu, valid)) {
        float amax = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(y[e]));
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        float isc = 0.f;
        const float sc = valid ? fp8_block_scale(amax, &isc) : 0.f;
        const uint2 q = make_uint2(pack_fp8x4(y[0] * isc, y[1] * isc, y[2] * isc, y[3] * isc),
                                   pack_fp8x4(y[4] * isc, y[5] * isc, y[6] * isc, y[7] * isc));
        // lane pairs hold adjacent chunks (c, c + 1): the even lane stores both as one 16-byte store
        const uint32_t nx = __shfl_down_sync(0xffffffffu, q.x, 1), ny = __shfl_down_sync(0xffffffffu, q.y, 1);
        const bool pair = c + 1 < nch && (threadIdx.x & 31) != 31;
        if (valid) {
          const size_t qoff = (size_t)row * H + c * 8;
          const size_t soff = ((size_t)(c >> 4) * a.s_ld + row) * 4;
          const bool even = (c & 1) == 0;
          const uint4 q2 = make_uint4(q.x, q.y, nx, ny);
          if constexpr (NV) {
            if (even && pair) mm_st16(mc + a.off_q + qoff, q2);
            else if (even) mm_st8(mc + a.off_q + qoff, q);
            if ((c & 15) == 0) mm_st4(mc + a.off_s + soff, __float_as_uint(sc));
          } else {
            for (int p = 0; p < W; ++p) {
              if (even && pair) *reinterpret_cast<uint4*>(base(p) + a.off_q + qoff) = q2;
              else if (even) *reinterpret_cast<uint2*>(base(p) + a.off_q + qoff) = q;
              if ((c & 15) == 0) *reinterpret_cast<float*>(base(p) + a.off_s + soff) = sc;
            }
          }
        }
      }
    }
  }

  if (a.phase_ns && threadIdx.x == 0) {
    atomicAdd(&a.phase_ns[0], (unsigned long long)(t_start - t_entry));
    atomicAdd(&a.phase_ns[1], (unsigned long long)(globaltimer() - t_start));
    atomicAdd(&a.phase_ns[3], 1ull);
  }
  end_barrier(mine, a.off_flags, a.off_counter, epoch, W, a.rank, a.peer_base, a.status, a.phase_ns);
}

// CTAs of `threads` threads of this kernel resident on the current device at once (SMs x CTAs per SM),
// queried once per kernel and device
static int resident_ctas(const void* kern, int threads) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find({kern, dev});
  if (it != cache.end()) return it->second;
  int per_sm = 0, sms = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, 0) != cudaSuccess || per_sm <= 0) {
    (void)cudaGetLastError();
    per_sm = 2;
  }
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int n = std::max(1, sms * per_sm);
  cache[{kern, dev}] = n;
  return n;
}

void tp_ar_norm(torch::Tensor peer_base, int64_t rank, int64_t world, int64_t M, int64_t H, double eps,
                torch::Tensor w, bool out_bf16, bool push_h, torch::Tensor status, std::vector<int64_t> offsets,
                int64_t s_ld, int64_t off_recv, int64_t mc_base, c10::optional<torch::Tensor> phase) {
  TORCH_CHECK(peer_base.is_cuda() && peer_base.scalar_type() == at::kLong && peer_base.numel() == world);
  TORCH_CHECK(H % 128 == 0 && world >= 1 && world <= 32 && offsets.size() == 7);
  if (M == 0) return;
  const at::cuda::CUDAGuard guard(w.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  TpArgs a;
  a.peer_base = reinterpret_cast<const uint64_t*>(peer_base.data_ptr<int64_t>());
  a.rank = (int)rank;
  a.world = (int)world;
  a.M = (int)M;
  a.H = (int)H;
  a.eps = (float)eps;
  a.w = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  a.out_bf16 = out_bf16 ? 1 : 0;
  a.push_h = push_h ? 1 : 0;
  a.recv = off_recv >= 0 ? 1 : 0;
  a.off_recv = off_recv >= 0 ? (uint64_t)off_recv : 0;
  a.status = status.data_ptr<int>();
  a.off_partial = offsets[0];
  a.off_h = offsets[1];
  a.off_y = offsets[2];
  a.off_q = offsets[3];
  a.off_s = offsets[4];
  a.off_flags = offsets[5];
  a.off_counter = offsets[6];
  a.s_ld = (int)s_ld;
  a.mc_base = (uint64_t)mc_base;
  a.phase_ns = nullptr;
  if (phase) {
    TORCH_CHECK(phase->scalar_type() == at::kLong && phase->numel() >= 4 && phase->is_cuda());
    a.phase_ns = reinterpret_cast<unsigned long long*>(phase->data_ptr<int64_t>());
  }
  const int rows_per = (int)((M + world - 1) / world);
  const int maxc = (int)((H / 8 + 255) / 256);
  // one wave: as many CTAs as are resident at once (every CTA of the launch spins at the start barrier, and
  // a second wave would serialise behind the first), each walking rows; the residency is queried once per
  // kernel instantiation and device
  auto go = [&](void (*kern)(const TpArgs)) {
    const int grid = std::max(1, std::min(rows_per, resident_ctas(reinterpret_cast<const void*>(kern), 256)));
    kern<<<grid, 256, 0, stream>>>(a);
  };
  auto launch_nv = [&](auto wt, auto nv) {
    constexpr int WT = decltype(wt)::value;
    constexpr bool NV = decltype(nv)::value;
    if (maxc <= 1) go(tp_ar_norm_kernel<1, WT, NV>);
    else if (maxc <= 2) go(tp_ar_norm_kernel<2, WT, NV>);
    else if (maxc <= 4) go(tp_ar_norm_kernel<4, WT, NV>);
    else if (maxc <= 8) go(tp_ar_norm_kernel<8, WT, NV>);
    else TORCH_CHECK(false, "hidden size too large");
  };
  auto launch = [&](auto wt) {
    if (mc_base != 0) launch_nv(wt, std::true_type{});
    else launch_nv(wt, std::false_type{});
  };
  if (world == 2) launch(std::integral_constant<int, 2>{});
  else if (world == 4) launch(std::integral_constant<int, 4>{});
  else if (world == 8) launch(std::integral_constant<int, 8>{});
  else launch(std::integral_constant<int, 0>{});
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

struct GatherArgs {
  const uint64_t* peer_base;
  int rank, world;
  int64_t n16;                // 16-byte words per rank
  uint64_t off_src, off_dst, off_flags, off_counter;
  int* status;
  uint64_t mc_base;           // multicast address of the workspace (0: peer stores)
};

// copy this rank's staging block [n16 x 16 B] into slot [rank] of every rank's gather region
__global__ void __launch_bounds__(256) tp_allgather_kernel(const GatherArgs a) {
  const int W = a.world;
  auto base = [&](int p) { return reinterpret_cast<uint8_t*>(a.peer_base[p]); };
  uint8_t* mine = base(a.rank);
  uint32_t* my_flags = reinterpret_cast<uint32_t*>(mine + a.off_flags);
  const uint32_t epoch = reinterpret_cast<volatile uint32_t*>(mine + a.off_counter)[1] + 1u;
  if (blockIdx.x == 0 && threadIdx.x < W) {
    __threadfence_system();
    st_release_sys(reinterpret_cast<uint32_t*>(base(threadIdx.x) + a.off_flags) + a.rank, epoch);
  }
  // start barrier: every peer has finished reading its gather region from the previous exchange
  const bool ok = wait_flags(my_flags, W, epoch, a.status);
  if (ok) {
    const uint4* src = reinterpret_cast<const uint4*>(mine + a.off_src);
    const uint64_t dst_off = a.off_dst + (uint64_t)a.rank * (uint64_t)a.n16 * 16u;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < a.n16; i += (int64_t)gridDim.x * blockDim.x) {
      const uint4 v = src[i];
      if (a.mc_base)
        mm_st16(reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(a.mc_base) + dst_off) + i, v);
      else
        for (int p = 0; p < W; ++p) reinterpret_cast<uint4*>(base(p) + dst_off)[i] = v;
    }
  }
  end_barrier(mine, a.off_flags, a.off_counter, epoch, W, a.rank, a.peer_base, a.status);
}

void tp_allgather(torch::Tensor peer_base, int64_t rank, int64_t world, int64_t nbytes, torch::Tensor status,
                  std::vector<int64_t> offsets, int64_t mc_base) {
  TORCH_CHECK(peer_base.is_cuda() && peer_base.numel() == world && offsets.size() == 4);
  TORCH_CHECK(nbytes > 0 && nbytes % 16 == 0, "gather block must be a positive multiple of 16 bytes");
  const at::cuda::CUDAGuard guard(peer_base.device());
  GatherArgs a;
  a.peer_base = reinterpret_cast<const uint64_t*>(peer_base.data_ptr<int64_t>());
  a.rank = (int)rank;
  a.world = (int)world;
  a.n16 = nbytes / 16;
  a.off_src = offsets[0];
  a.off_dst = offsets[1];
  a.off_flags = offsets[2];
  a.off_counter = offsets[3];
  a.status = status.data_ptr<int>();
  a.mc_base = (uint64_t)mc_base;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((a.n16 + 255) / 256, 148));
  tp_allgather_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace phx
