// TMA tensor-map encoding through the driver entry point (no link-time
// dependency on libcuda).
#include <cstdio>

#include "vab_internal.h"

namespace vab {

namespace {

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
  static EncodeTiled fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(p);
    else
      fprintf(stderr, "vocalarc-b200: cuTensorMapEncodeTiled is unavailable\n");
  }
  return fn;
}

}  // namespace

bool make_tmap_2d(CUtensorMap* map, const void* base, int elem_bytes, uint64_t inner, uint64_t outer,
                  uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, int swizzle_bytes, bool bf16) {
  EncodeTiled fn = encoder();
  if (fn == nullptr || (elem_bytes != 2 && elem_bytes != 4)) return false;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_stride_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType type = elem_bytes == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                                   : (bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                           : CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
  const CUtensorMapSwizzle swz = swizzle_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                 : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                       : CU_TENSOR_MAP_SWIZZLE_NONE;
  const CUresult r = fn(map, type, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    fprintf(stderr, "vocalarc-b200: cuTensorMapEncodeTiled(2d) failed (%d)\n", static_cast<int>(r));
    return false;
  }
  return true;
}

bool make_tmap_4d(CUtensorMap* map, const void* base, int elem_bytes, const uint64_t dims_in[4],
                  const uint64_t strides_bytes[3], const uint32_t box_in[4], bool bf16) {
  EncodeTiled fn = encoder();
  if (fn == nullptr || elem_bytes != 2) return false;
  const cuuint64_t dims[4] = {dims_in[0], dims_in[1], dims_in[2], dims_in[3]};
  const cuuint64_t strides[3] = {strides_bytes[0], strides_bytes[1], strides_bytes[2]};
  const cuuint32_t box[4] = {box_in[0], box_in[1], box_in[2], box_in[3]};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                        const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    fprintf(stderr, "vocalarc-b200: cuTensorMapEncodeTiled(4d) failed (%d)\n", static_cast<int>(r));
    return false;
  }
  return true;
}

}  // namespace vab
