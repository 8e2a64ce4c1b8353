// RMSNorm and fused residual-add + RMSNorm over rows.
//
// Reference semantics: rms_norm_kernel (src/kernels.cu:59-73) computes, for one
// vector, out[i] = in[i] * rsqrtf(sum(in^2)/size + eps) * weight[i], one
// 1024-thread block per vector and one launch per token. Here a launch covers
// all rows:
//   - vector path: a "row group" of G threads (G a multiple of 32) owns one row
//     and holds it in registers as VPT 16-byte vectors per thread, so each row
//     is read from HBM once and written once. The row sum of squares is a warp
//     butterfly plus, when G > 32, a shared-memory pass over the group's warps.
//     A block holds 256/G groups for small rows (one warp per row for dim <=
//     128 vectors) and one group for wide rows (G up to 1024).
//   - scalar path (unaligned pointers, odd pitches, rows wider than 8192
//     vectors): one 256-thread block per row, two passes over the row.
// The fused variant adds `delta` into `residual` first (fp32 add, as
// add_kernel, src/kernels.cu:199-202), stores the sum in the I/O type, and
// normalises the stored values: the same numbers the reference's add then
// rms_norm launches produce (src/execution_engine.cu:118,121).
#include <algorithm>

#include "bm_common.cuh"
#include "bm_host.h"

namespace bm {
namespace {

constexpr int kMaxWarpsPerGroup = 32;

struct RmsArgs {
  void* out;              // [rows][out_stride]
  void* residual;         // in (plain) or residual in/out (fused)
  const void* delta;      // fused only
  const void* weight;     // [dim]
  int64_t rows;
  int64_t in_stride;      // elements
  int64_t out_stride;     // elements
  int dim;
  int nv;                 // 16-byte vectors per row
  int group;              // threads per row
  float eps;
};

template <typename T, int VPT, bool FUSED, int MAXT>
__global__ void __launch_bounds__(MAXT) rmsnorm_vec_kernel(RmsArgs a) {
  constexpr int N = VecWidth<T>::value;
  __shared__ float s_part[2][kMaxWarpsPerGroup];  // [parity][warp of block]

  const int G = a.group;
  const int rows_per_block = blockDim.x / G;
  const int gi = threadIdx.x / G;      // group index in block
  const int t = threadIdx.x - gi * G;  // thread index in group
  const int warp = threadIdx.x >> 5;
  const int warps_per_group = G >> 5;
  const int first_warp = gi * warps_per_group;
  const T* weight = static_cast<const T*>(a.weight);
  {  // the first row's lines, while the previous kernel finishes
    const int64_t row = static_cast<int64_t>(blockIdx.x) * rows_per_block + gi;
    if (row < a.rows) {
      const int64_t bytes = static_cast<int64_t>(a.nv) * 16;
      prefetch_l2_range(static_cast<const T*>(a.residual) + row * a.in_stride, bytes, t, G);
      if constexpr (FUSED) prefetch_l2_range(static_cast<const T*>(a.delta) + row * a.in_stride, bytes, t, G);
      if (gi == 0) prefetch_l2_range(weight, bytes, t, G);
    }
  }
  grid_dependency_wait();

  int parity = 0;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * rows_per_block; base < a.rows;
       base += static_cast<int64_t>(gridDim.x) * rows_per_block) {
    const int64_t row = base + gi;
    const bool valid = row < a.rows;
    T* in_row = static_cast<T*>(a.residual) + row * a.in_stride;

    // The row stays packed in registers between the two halves of the kernel.
    uint4 raw[VPT];
    float ss = 0.f;
    if (valid) {
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const int v = t + j * G;
        if (v < a.nv) raw[j] = ld_stream(in_row + static_cast<int64_t>(v) * N);
      }
      if constexpr (FUSED) {
        const T* d_row = static_cast<const T*>(a.delta) + row * a.in_stride;
        uint4 raw_d[VPT];
#pragma unroll
        for (int j = 0; j < VPT; ++j) {
          const int v = t + j * G;
          if (v < a.nv) raw_d[j] = ld_stream(d_row + static_cast<int64_t>(v) * N);
        }
#pragma unroll
        for (int j = 0; j < VPT; ++j) {
          const int v = t + j * G;
          if (v < a.nv) {
            float x[N], d[N];
            unpack16<T>(raw[j], x);
            unpack16<T>(raw_d[j], d);
#pragma unroll
            for (int e = 0; e < N; ++e) x[e] = x[e] + d[e];
            raw[j] = pack16<T>(x);  // the residual as stored (rounded to T)
            st_plain(in_row + static_cast<int64_t>(v) * N, raw[j]);
          }
        }
      }
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const int v = t + j * G;
        if (v < a.nv) {
          float x[N];
          unpack16<T>(raw[j], x);
#pragma unroll
          for (int e = 0; e < N; ++e) ss += x[e] * x[e];
        }
      }
    }

    ss = warp_sum(ss);
    if (warps_per_group > 1) {
      if ((threadIdx.x & 31) == 0) s_part[parity][warp] = ss;
      __syncthreads();
      ss = 0.f;
      for (int i = 0; i < warps_per_group; ++i) ss += s_part[parity][first_warp + i];
      parity ^= 1;
    }

    if (valid) {
      const float scale = rsqrtf(ss / static_cast<float>(a.dim) + a.eps);
      T* out_row = static_cast<T*>(a.out) + row * a.out_stride;
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const int v = t + j * G;
        if (v < a.nv) {
          float x[N], w[N];
          unpack16<T>(raw[j], x);
          unpack16<T>(ld_keep(weight + static_cast<int64_t>(v) * N), w);
#pragma unroll
          for (int e = 0; e < N; ++e) x[e] = x[e] * scale * w[e];
          st_plain(out_row + static_cast<int64_t>(v) * N, pack16<T>(x));
        }
      }
    }
  }
}

// One 256-thread block per row; two passes over the row (sum, then write).
template <typename T, bool FUSED>
__global__ void __launch_bounds__(256) rmsnorm_scalar_kernel(RmsArgs a) {
  grid_dependency_wait();
  __shared__ float s_warp[8];
  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
    T* in_row = static_cast<T*>(a.residual) + row * a.in_stride;
    float ss = 0.f;
    for (int i = threadIdx.x; i < a.dim; i += blockDim.x) {
      float x = load1<T>(in_row + i);
      if constexpr (FUSED) {
        x = round_to<T>(x + load1<T>(static_cast<const T*>(a.delta) + row * a.in_stride + i));
        store1<T>(in_row + i, x);
      }
      ss += x * x;
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) s_warp[threadIdx.x >> 5] = ss;
    __syncthreads();
    ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += s_warp[i];
    const float scale = rsqrtf(ss / static_cast<float>(a.dim) + a.eps);
    T* out_row = static_cast<T*>(a.out) + row * a.out_stride;
    const T* w = static_cast<const T*>(a.weight);
    for (int i = threadIdx.x; i < a.dim; i += blockDim.x) {
      // Each thread re-reads the elements it stored in the first pass.
      store1<T>(out_row + i, load1<T>(in_row + i) * scale * load1<T>(w + i));
    }
    __syncthreads();  // s_warp is reused by the next row
  }
}

template <typename T, bool FUSED>
int launch_vec(RmsArgs a, int vpt, cudaStream_t stream) {
  const int block = a.group >= 256 ? a.group : 256 / a.group * a.group;
  const int rows_per_block = block / a.group;
  const int64_t need = (a.rows + rows_per_block - 1) / rows_per_block;
  const int64_t cap = static_cast<int64_t>(sm_count()) * (2048 / block) * 64;
  const unsigned grid = static_cast<unsigned>(std::max<int64_t>(1, std::min(need, cap)));
  switch (vpt) {
    case 1:
      if (const int launch_status = launch_kernel("rmsnorm_vec_kernel", rmsnorm_vec_kernel<T, 1, FUSED, 256>,
                                                  dim3(grid), dim3(block), 0, stream, nullptr, a)) {
        return launch_status;
      }
      break;
    case 2:
      if (const int launch_status = launch_kernel("rmsnorm_vec_kernel", rmsnorm_vec_kernel<T, 2, FUSED, 256>,
                                                  dim3(grid), dim3(block), 0, stream, nullptr, a)) {
        return launch_status;
      }
      break;
    case 4:
      if (const int launch_status = launch_kernel("rmsnorm_vec_kernel", rmsnorm_vec_kernel<T, 4, FUSED, 256>,
                                                  dim3(grid), dim3(block), 0, stream, nullptr, a)) {
        return launch_status;
      }
      break;
    default:
      if (block <= 256) {
        if (const int launch_status = launch_kernel("rmsnorm_vec_kernel", rmsnorm_vec_kernel<T, 8, FUSED, 256>,
                                                    dim3(grid), dim3(block), 0, stream, nullptr, a)) {
          return launch_status;
        }
      } else {
        if (const int launch_status = launch_kernel("rmsnorm_vec_kernel", rmsnorm_vec_kernel<T, 8, FUSED, 1024>,
                                                    dim3(grid), dim3(block), 0, stream, nullptr, a)) {
          return launch_status;
        }
      }
      break;
  }
  return check_launch(FUSED ? "bm_add_rmsnorm" : "bm_rmsnorm");
}

template <typename T, bool FUSED>
int launch_scalar(RmsArgs a, cudaStream_t stream) {
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8 * 64;
  const unsigned grid = static_cast<unsigned>(std::max<int64_t>(1, std::min(a.rows, cap)));
  if (const int launch_status = launch_kernel("rmsnorm_scalar_kernel", rmsnorm_scalar_kernel<T, FUSED>, dim3(grid),
                                              dim3(256), 0, stream, nullptr, a)) {
    return launch_status;
  }
  return check_launch(FUSED ? "bm_add_rmsnorm" : "bm_rmsnorm");
}

// Picks the row-group shape: threads per row G and 16-byte vectors per thread.
// Returns false when the row is too wide for the register-resident path.
bool pick_shape(int nv, int* group, int* vpt) {
  if (nv <= 32) {
    *vpt = 1;
    *group = 32;
  } else if (nv <= 64) {
    *vpt = 2;
    *group = 32;
  } else if (nv <= 1024) {
    *vpt = 4;
    *group = ((nv + 3) / 4 + 31) / 32 * 32;
  } else if (nv <= 8 * 1024) {
    *vpt = 8;
    *group = ((nv + 7) / 8 + 31) / 32 * 32;
  } else {
    return false;
  }
  return true;
}

template <bool FUSED>
int run(RmsArgs a, bm_dtype_t dtype, cudaStream_t stream) {
  const int es = dtype_size(dtype);
  const bool vec_ok = (static_cast<int64_t>(a.dim) * es) % 16 == 0 && (a.in_stride * es) % 16 == 0 &&
                      (a.out_stride * es) % 16 == 0 && aligned16(a.out) && aligned16(a.residual) &&
                      aligned16(a.weight) && (!FUSED || aligned16(a.delta));
  int group = 0, vpt = 0;
  a.nv = static_cast<int>(static_cast<int64_t>(a.dim) * es / 16);
  if (vec_ok && pick_shape(a.nv, &group, &vpt)) {
    a.group = group;
    return dtype == BM_F32 ? launch_vec<float, FUSED>(a, vpt, stream) : launch_vec<bf16, FUSED>(a, vpt, stream);
  }
  return dtype == BM_F32 ? launch_scalar<float, FUSED>(a, stream) : launch_scalar<bf16, FUSED>(a, stream);
}

}  // namespace
}  // namespace bm

extern "C" int bm_rmsnorm(void* out, const void* in, const void* weight, int64_t rows, int64_t dim, float eps,
                          int64_t in_stride, int64_t out_stride, bm_dtype_t dtype, void* stream) {
  using namespace bm;
  if (!valid_dtype(dtype)) return fail(BM_ERR_INVALID_ARGUMENT, "bm_rmsnorm: bad dtype %d", static_cast<int>(dtype));
  if (rows < 0 || dim < 0 || dim > INT32_MAX) return fail(BM_ERR_INVALID_ARGUMENT, "bm_rmsnorm: bad rows/dim");
  if (rows == 0 || dim == 0) return BM_OK;
  if (in_stride < dim || out_stride < dim) return fail(BM_ERR_INVALID_ARGUMENT, "bm_rmsnorm: stride < dim");
  if (!out || !in || !weight) return fail(BM_ERR_INVALID_ARGUMENT, "bm_rmsnorm: NULL pointer");
  if (!(eps >= 0.f)) return fail(BM_ERR_INVALID_ARGUMENT, "bm_rmsnorm: eps must be >= 0");
  if (out != in) {
    // Distinct buffers must not overlap (in place means out == in exactly).
    const int es = dtype_size(dtype);
    const char* o0 = static_cast<const char*>(out);
    const char* i0 = static_cast<const char*>(in);
    const char* o1 = o0 + ((rows - 1) * out_stride + dim) * es;
    const char* i1 = i0 + ((rows - 1) * in_stride + dim) * es;
    if (o0 < i1 && i0 < o1) return fail(BM_ERR_INVALID_ARGUMENT, "bm_rmsnorm: out overlaps in without being equal");
  }
  RmsArgs a{};
  a.out = out;
  a.residual = const_cast<void*>(in);
  a.delta = nullptr;
  a.weight = weight;
  a.rows = rows;
  a.in_stride = in_stride;
  a.out_stride = out_stride;
  a.dim = static_cast<int>(dim);
  a.eps = eps;
  return run<false>(a, dtype, as_stream(stream));
}

extern "C" int bm_add_rmsnorm(void* residual, const void* delta, const void* weight, void* out, int64_t rows,
                              int64_t dim, float eps, bm_dtype_t dtype, void* stream) {
  using namespace bm;
  if (!valid_dtype(dtype)) return fail(BM_ERR_INVALID_ARGUMENT, "bm_add_rmsnorm: bad dtype %d", static_cast<int>(dtype));
  if (rows < 0 || dim < 0 || dim > INT32_MAX) return fail(BM_ERR_INVALID_ARGUMENT, "bm_add_rmsnorm: bad rows/dim");
  if (rows == 0 || dim == 0) return BM_OK;
  if (!residual || !delta || !weight || !out) return fail(BM_ERR_INVALID_ARGUMENT, "bm_add_rmsnorm: NULL pointer");
  if (!(eps >= 0.f)) return fail(BM_ERR_INVALID_ARGUMENT, "bm_add_rmsnorm: eps must be >= 0");
  {
    const int64_t bytes = rows * dim * dtype_size(dtype);
    const char* o0 = static_cast<const char*>(out);
    const char* r0 = static_cast<const char*>(residual);
    const char* d0 = static_cast<const char*>(delta);
    if ((o0 < r0 + bytes && r0 < o0 + bytes) || (o0 < d0 + bytes && d0 < o0 + bytes)) {
      return fail(BM_ERR_INVALID_ARGUMENT, "bm_add_rmsnorm: out overlaps residual or delta");
    }
  }
  RmsArgs a{};
  a.out = out;
  a.residual = residual;
  a.delta = delta;
  a.weight = weight;
  a.rows = rows;
  a.in_stride = dim;
  a.out_stride = dim;
  a.dim = static_cast<int>(dim);
  a.eps = eps;
  return run<true>(a, dtype, as_stream(stream));
}
