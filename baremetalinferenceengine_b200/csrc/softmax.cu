// Row softmax in place, the reference's softmax_kernel (src/kernels.cu:150-180):
// x[v][i] = exp(x[v][i] - max_v) / sum_v exp(x[v][j] - max_v) for i < size,
// vectors `stride` elements apart (the gaps left untouched). One CTA per
// vector: one pass keeps a running (max, sum) per thread, merged across the
// block, and a second pass writes; fp32 arithmetic, fp32 or bf16 storage.
#include "bm_common.cuh"
#include "bm_host.h"

namespace bm {
namespace {

constexpr int kSoftmaxThreads = 256;

// (m, s) of two running softmax states merged: max and the rescaled sum.
__device__ __forceinline__ void merge(float& m, float& s, float m2, float s2) {
  const float mn = fmaxf(m, m2);
  if (mn == -INFINITY) return;  // both empty
  s = s * expf(m - mn) + s2 * expf(m2 - mn);
  m = mn;
}

template <typename T>
__global__ void __launch_bounds__(kSoftmaxThreads) softmax_kernel(T* x, int64_t size, int64_t stride) {
  grid_dependency_wait();
  __shared__ float sm[kSoftmaxThreads / 32], ss[kSoftmaxThreads / 32];
  T* v = x + static_cast<int64_t>(blockIdx.x) * stride;
  float m = -INFINITY, s = 0.f;
  for (int64_t i = threadIdx.x; i < size; i += kSoftmaxThreads) {
    const float e = load1<T>(v + i);
    if (e > m) {
      s = s * expf(m - e) + 1.f;
      m = e;
    } else {
      s += expf(e - m);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, off), s2 = __shfl_xor_sync(0xffffffffu, s, off);
    merge(m, s, m2, s2);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sm[warp] = m;
    ss[warp] = s;
  }
  __syncthreads();
  m = sm[0];
  s = ss[0];
#pragma unroll
  for (int w = 1; w < kSoftmaxThreads / 32; ++w) merge(m, s, sm[w], ss[w]);
  const float inv = 1.f / s;
  for (int64_t i = threadIdx.x; i < size; i += kSoftmaxThreads) store1<T>(v + i, expf(load1<T>(v + i) - m) * inv);
}

}  // namespace
}  // namespace bm

extern "C" int bm_softmax(void* x, int64_t size, int64_t num_vectors, int64_t stride, bm_dtype_t dtype,
                          void* stream) {
  using namespace bm;
  if (!valid_dtype(dtype)) return fail(BM_ERR_INVALID_ARGUMENT, "bm_softmax: bad dtype");
  if (size < 0 || num_vectors < 0 || num_vectors > 0x7fffffff) {
    return fail(BM_ERR_INVALID_ARGUMENT, "bm_softmax: negative size or too many vectors");
  }
  if (num_vectors > 1 && stride < size) return fail(BM_ERR_INVALID_ARGUMENT, "bm_softmax: stride < size");
  if (size == 0 || num_vectors == 0) return BM_OK;
  if (!x) return fail(BM_ERR_INVALID_ARGUMENT, "bm_softmax: NULL x");
  const dim3 grid(static_cast<unsigned>(num_vectors));
  if (dtype == BM_F32) {
    if (const int launch_status = launch_kernel("softmax_kernel", softmax_kernel<float>, dim3(grid),
                                                dim3(kSoftmaxThreads), 0, as_stream(stream), nullptr,
                                                static_cast<float*>(x), size, stride)) {
      return launch_status;
    }
  } else {
    if (const int launch_status = launch_kernel("softmax_kernel", softmax_kernel<bf16>, dim3(grid),
                                                dim3(kSoftmaxThreads), 0, as_stream(stream), nullptr,
                                                static_cast<bf16*>(x), size, stride)) {
      return launch_status;
    }
  }
  return check_launch("bm_softmax");
}
