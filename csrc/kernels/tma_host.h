// Host-side construction of TMA tensor maps. The driver entry point is looked
// up at run time through the CUDA runtime, so the extension does not link
// against libcuda directly.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

namespace nk {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    TORCH_CHECK(e == cudaSuccess && q == cudaDriverEntryPointSuccess && p, "cuTensorMapEncodeTiled unavailable");
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

// 2-D bf16 tensor map over a row-major matrix with `outer` rows of `inner`
// elements (row stride `ld` elements), box = box_inner x box_outer, with the
// given swizzle (the inner box must span the swizzle width).
inline CUtensorMap make_tmap_bf16_2d_swz(const void* base, int64_t inner, int64_t outer, int64_t ld, int box_inner,
                                         int box_outer, CUtensorMapSwizzle swz) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK((ld * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {cuuint64_t(inner), cuuint64_t(outer)};
  cuuint64_t strides[1] = {cuuint64_t(ld * 2)};
  cuuint32_t box[2] = {cuuint32_t(box_inner), cuuint32_t(box_outer)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_tiled_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                                 estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", int(r));
  return m;
}

// 128-byte swizzled operand tiles (64-element inner box).
inline CUtensorMap make_tmap_bf16_2d(const void* base, int64_t inner, int64_t outer, int64_t ld, int box_inner,
                                     int box_outer) {
  TORCH_CHECK(box_inner * 2 == 128, "128B swizzle needs a 64-element inner box");
  return make_tmap_bf16_2d_swz(base, inner, outer, ld, box_inner, box_outer, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace nk
