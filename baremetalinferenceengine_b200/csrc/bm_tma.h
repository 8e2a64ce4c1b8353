// Host-side TMA descriptor encoding shared by the tensor-core kernels.
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "bm_layer_ops.h"

namespace bm {

// A 2-D bf16 tensor map over [outer][inner] (row pitch `inner` elements) with a
// box of box_outer rows x box_inner columns and 128-byte swizzle; reads outside
// the tensor return zeros. Returns BM_OK or BM_ERR_CUDA (message recorded).
int make_tensor_map_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint32_t box_inner,
                         uint32_t box_outer, const char* what);

// The same for fp32 or bf16 (box_inner * element size at most 128 bytes).
int make_tensor_map_2d(CUtensorMap* map, const void* base, bm_dtype_t dtype, uint64_t inner, uint64_t outer,
                       uint32_t box_inner, uint32_t box_outer, const char* what);

}  // namespace bm
