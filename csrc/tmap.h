// Host-side TMA tensor-map construction (cuTensorMapEncodeTiled through the runtime's driver
// entry-point query, so the extension does not link libcuda directly).
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

namespace phx {

inline PFN_cuTensorMapEncodeTiled_v12000 tmap_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    TORCH_CHECK(e == cudaSuccess && q == cudaDriverEntryPointSuccess && p, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 2-D tiled map over a row-major matrix: `inner` elements per row (contiguous), `outer` rows,
// `row_stride_bytes` between rows. The base must be 16-byte aligned and the stride a multiple of 16.
inline CUtensorMap make_tmap_2d(const void* base, CUtensorMapDataType dt, uint64_t inner, uint64_t outer,
                               uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                               CUtensorMapSwizzle sw) {
  TORCH_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK(row_stride_bytes % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = tmap_encode_fn()(&m, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                                CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", (int)r);
  return m;
}

// 3-D tiled map (dims innermost first), strides in bytes for dims 1 and 2.
inline CUtensorMap make_tmap_3d(const void* base, CUtensorMapDataType dt, uint64_t d0, uint64_t d1, uint64_t d2,
                               uint64_t stride1, uint64_t stride2, uint32_t b0, uint32_t b1, uint32_t b2,
                               CUtensorMapSwizzle sw) {
  TORCH_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK(stride1 % 16 == 0 && stride2 % 16 == 0, "TMA strides must be multiples of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1, stride2};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = tmap_encode_fn()(&m, dt, 3, const_cast<void*>(base), dims, strides, box, estr,
                                CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", (int)r);
  return m;
}

}  // namespace phx
