// Token-embedding gather: out[r, :] = table[ids[r], :], bit-exact.
//
// Reference semantics: ExecutionEngine::run_layers copies one embedding row per
// token with a device-to-device cudaMemcpy (src/execution_engine.cu:98-99),
// after forward() has rejected ids outside the vocabulary on the host
// (src/execution_engine.cu:63-65). Here one launch gathers every row: a row
// group of threads copies one row with 16-byte loads, UNROLL vectors in flight
// per thread. An id outside [0, vocab) leaves its output row unwritten and sets
// BM_DEVERR_BAD_ID in *status. Repeated ids (a Zipf-distributed batch) are
// served from L2, so table reads use the default caching load.
#include <algorithm>

#include "bm_common.cuh"
#include "bm_host.h"

namespace bm {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;

struct GatherArgs {
  void* out;
  const void* table;
  const int32_t* ids;
  int64_t rows;
  int64_t vocab;
  int64_t out_stride;  // elements
  int64_t dim;         // elements
  int64_t nv;          // 16-byte vectors per row (vector path)
  int group;           // threads per row
  int es;              // bytes per element
  int32_t* status;
};

// Vector path: bytes of a row are copied as 16-byte words (the row pitch and
// both base pointers are 16-byte multiples).
__global__ void __launch_bounds__(kThreads) gather_vec_kernel(GatherArgs a) {
  const int G = a.group;
  const int rows_per_block = kThreads / G;
  const int gi = threadIdx.x / G;
  const int t = threadIdx.x - gi * G;
  {  // the first row's id (the table row it names is known only after the wait)
    const int64_t row = static_cast<int64_t>(blockIdx.x) * rows_per_block + gi;
    if (t == 0 && row < a.rows) prefetch_l2(a.ids + row);
  }
  grid_dependency_wait();
  const int64_t row_bytes = a.nv * 16;
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * rows_per_block + gi; row < a.rows;
       row += static_cast<int64_t>(gridDim.x) * rows_per_block) {
    const int32_t id = __ldg(a.ids + row);
    if (id < 0 || id >= a.vocab) {
      if (t == 0) raise_status(a.status, BM_DEVERR_BAD_ID);
      continue;
    }
    const char* src = static_cast<const char*>(a.table) + static_cast<int64_t>(id) * row_bytes;
    char* dst = static_cast<char*>(a.out) + row * a.out_stride * a.es;
    for (int64_t v0 = t; v0 < a.nv; v0 += static_cast<int64_t>(G) * kUnroll) {
      uint4 r[kUnroll];
#pragma unroll
      for (int j = 0; j < kUnroll; ++j) {
        const int64_t v = v0 + static_cast<int64_t>(j) * G;
        if (v < a.nv) r[j] = *reinterpret_cast<const uint4*>(src + v * 16);
      }
#pragma unroll
      for (int j = 0; j < kUnroll; ++j) {
        const int64_t v = v0 + static_cast<int64_t>(j) * G;
        if (v < a.nv) st_plain(dst + v * 16, r[j]);
      }
    }
  }
}

// Scalar path: element-wise copy of the raw storage (no conversion).
template <typename W>
__global__ void __launch_bounds__(kThreads) gather_scalar_kernel(GatherArgs a) {
  grid_dependency_wait();
  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
    const int32_t id = a.ids[row];
    if (id < 0 || id >= a.vocab) {
      if (threadIdx.x == 0) raise_status(a.status, BM_DEVERR_BAD_ID);
      continue;
    }
    const W* src = static_cast<const W*>(a.table) + static_cast<int64_t>(id) * a.dim;
    W* dst = static_cast<W*>(a.out) + row * a.out_stride;
    for (int64_t i = threadIdx.x; i < a.dim; i += kThreads) dst[i] = src[i];
  }
}

}  // namespace
}  // namespace bm

extern "C" int bm_embed_gather(void* out, const void* table, const int32_t* ids, int64_t rows, int64_t dim,
                               int64_t vocab, int64_t out_row_stride, bm_dtype_t dtype, int32_t* d_status,
                               void* stream) {
  using namespace bm;
  if (!valid_dtype(dtype)) return fail(BM_ERR_INVALID_ARGUMENT, "bm_embed_gather: bad dtype %d", static_cast<int>(dtype));
  if (rows < 0 || dim < 0 || vocab < 0) return fail(BM_ERR_INVALID_ARGUMENT, "bm_embed_gather: negative size");
  if (rows == 0 || dim == 0) return BM_OK;
  if (vocab > INT32_MAX) return fail(BM_ERR_INVALID_ARGUMENT, "bm_embed_gather: vocab exceeds int32 ids");
  if (out_row_stride < dim) return fail(BM_ERR_INVALID_ARGUMENT, "bm_embed_gather: out_row_stride < dim");
  if (!out || !table || !ids) return fail(BM_ERR_INVALID_ARGUMENT, "bm_embed_gather: NULL pointer");
  const int es = dtype_size(dtype);
  GatherArgs a{};
  a.out = out;
  a.table = table;
  a.ids = ids;
  a.rows = rows;
  a.vocab = vocab;
  a.out_stride = out_row_stride;
  a.dim = dim;
  a.es = es;
  a.status = d_status;
  cudaStream_t s = as_stream(stream);
  const int64_t cap = static_cast<int64_t>(sm_count()) * (2048 / kThreads) * 64;
  const bool vec_ok = (dim * es) % 16 == 0 && (out_row_stride * es) % 16 == 0 && aligned16(out) && aligned16(table);
  if (vec_ok) {
    a.nv = dim * es / 16;
    // Threads per row: enough for UNROLL vectors each, a power of two up to the block.
    int g = 32;
    while (g < kThreads && static_cast<int64_t>(g) * kUnroll < a.nv) g *= 2;
    a.group = g;
    const int rows_per_block = kThreads / g;
    const int64_t need = (rows + rows_per_block - 1) / rows_per_block;
    const unsigned grid = static_cast<unsigned>(std::max<int64_t>(1, std::min(need, cap)));
    if (const int launch_status = launch_kernel("gather_vec_kernel", gather_vec_kernel, dim3(grid), dim3(kThreads), 0,
                                                s, nullptr, a)) {
      return launch_status;
    }
  } else {
    const unsigned grid = static_cast<unsigned>(std::max<int64_t>(1, std::min(rows, cap)));
    if (es == 4) {
      if (const int launch_status = launch_kernel("gather_scalar_kernel", gather_scalar_kernel<uint32_t>, dim3(grid),
                                                  dim3(kThreads), 0, s, nullptr, a)) {
        return launch_status;
      }
    } else {
      if (const int launch_status = launch_kernel("gather_scalar_kernel", gather_scalar_kernel<uint16_t>, dim3(grid),
                                                  dim3(kThreads), 0, s, nullptr, a)) {
        return launch_status;
      }
    }
  }
  return check_launch("bm_embed_gather");
}
