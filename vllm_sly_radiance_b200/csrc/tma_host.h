// Host-side TMA descriptor creation.  cuTensorMapEncodeTiled is fetched through the runtime's
// driver entry-point query so the extension needs no link-time dependency on libcuda.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

namespace rad {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn get_encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    TORCH_CHECK(e == cudaSuccess && q == cudaDriverEntryPointSuccess && p,
                "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D tiled map: `inner` elements per row (dim 0), `rows` rows (dim 1), row stride in bytes.
inline CUtensorMap make_tma_2d(void* base, CUtensorMapDataType dtype, uint64_t inner,
                               uint64_t rows, uint64_t row_stride_bytes, uint32_t box_inner,
                               uint32_t box_rows, CUtensorMapSwizzle swizzle,
                               CUtensorMapL2promotion promo = CU_TENSOR_MAP_L2_PROMOTION_L2_256B) {
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode_tiled()(&m, dtype, 2, base, dims, strides, box, estr,
                                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, promo,
                                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", (int)r,
              " (inner=", inner, " rows=", rows, " stride=", row_stride_bytes, " box=", box_inner,
              "x", box_rows, ")");
  return m;
}

// 3-D tiled map (dims innermost first), strides for dims 1 and 2 in bytes.
inline CUtensorMap make_tma_3d(void* base, CUtensorMapDataType dtype, uint64_t d0, uint64_t d1,
                               uint64_t d2, uint64_t s1, uint64_t s2, uint32_t b0, uint32_t b1,
                               uint32_t b2, CUtensorMapSwizzle swizzle) {
  CUtensorMap m;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {s1, s2};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = get_encode_tiled()(&m, dtype, 3, base, dims, strides, box, estr,
                                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (3d) failed with code ", (int)r);
  return m;
}

}  // namespace rad
