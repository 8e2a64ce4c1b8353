// Tensor maps (TMA descriptors) for the tensor-core kernels, encoded on the host
// through the driver's cuTensorMapEncodeTiled, looked up once via the runtime.
#include <cuda.h>

#include <mutex>

#include "bm_host.h"
#include "bm_tma.h"

namespace bm {

namespace {

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// The driver's tensor-map encoder, looked up once through the runtime.
EncodeTiled encoder() {
  static std::once_flag once;
  static EncodeTiled fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiled>(p);
    }
  });
  return fn;
}

}  // namespace

// A 2-D bf16 tensor map over [outer][inner] (row stride `inner` elements) with
// a box of box_outer rows x box_inner columns and 128-byte swizzle; reads
// outside the tensor return zeros.
int make_tensor_map_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint32_t box_inner,
                         uint32_t box_outer, const char* what) {
  return make_tensor_map_2d(map, base, BM_BF16, inner, outer, box_inner, box_outer, what);
}

int make_tensor_map_2d(CUtensorMap* map, const void* base, bm_dtype_t dtype, uint64_t inner, uint64_t outer,
                       uint32_t box_inner, uint32_t box_outer, const char* what) {
  EncodeTiled enc = encoder();
  if (enc == nullptr) return fail(BM_ERR_CUDA, "%s: cuTensorMapEncodeTiled is not available", what);
  const uint64_t es = dtype == BM_F32 ? 4 : 2;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {inner * es};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t elem[2] = {1, 1};
  const CUtensorMapDataType type = dtype == BM_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUresult r = enc(map, type, 2, const_cast<void*>(base), dims, strides, box, elem,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(BM_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed (%d)", what, static_cast<int>(r));
  return BM_OK;
}

}  // namespace bm
