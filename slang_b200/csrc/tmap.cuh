// Host helper: 2D TMA tensor maps (cuTensorMapEncodeTiled through the runtime's
// driver entry point, so the library links against cudart only).
#pragma once

#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace sb {

inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Row-major [outer][inner] tensor of `elt`-byte elements with rows
// `row_stride_elems` apart, copied in boxes of box_outer x box_inner.
inline int make_map(CUtensorMap* map, CUtensorMapDataType dt, int elt, const void* base, uint64_t inner,
                    uint64_t outer, uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer,
                    CUtensorMapSwizzle sw) {
  auto fn = encode_fn();
  if (!fn) return fail(SB_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * elt};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SB_ERR_ARG, "cuTensorMapEncodeTiled failed (CUresult %d)", static_cast<int>(r));
  return SB_OK;
}

}  // namespace sb
