// fp32 GEMM for few rows: C[M][N] = A[M][K] . B[K][N], all fp32 row-major, on
// CUDA cores. The reference's launch_gemm (src/kernels.cu:83-121) is called by
// its engine with one row per token (src/execution_engine.cu:81,110-125): a
// matrix-vector product that streams B once, so this kernel is built to stream B
// at HBM speed while keeping fp32 arithmetic (the bf16 tensor-core GEMMs of
// gemm_tc.cu serve batched bf16 callers).
//
// A CTA of 256 threads owns 128 columns (lane l: columns 4l..4l+3, one 16-byte
// load of a B row per k) and MT rows of A (its values broadcast to the warp);
// its 8 warps take interleaved k, and a cluster of KS CTAs splits K further. The
// warps' partial sums meet in shared memory; the cluster's CTAs then add theirs
// in a fixed order through distributed shared memory, so results are
// deterministic and no global scratch is needed.
#include <cooperative_groups.h>

#include <algorithm>

#include "bm_common.cuh"
#include "bm_host.h"

namespace cg = cooperative_groups;

namespace bm {
namespace gemm32 {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kCols = 128;     // columns per CTA
constexpr int kMaxCluster = 8;

struct Args {
  float* c;
  const float* a;
  const float* b;
  int m, n, k;
  int k_per_cta;  // K range of one CTA of the cluster
};

// VEC: B rows are 16-byte aligned (N % 4 == 0) and read as float4.
template <int MT, bool VEC>
__global__ void __launch_bounds__(kThreads) gemm_f32_kernel(const Args p) {
  __shared__ __align__(16) float red[kWarps][MT][kCols];
  cg::cluster_group cluster = cg::this_cluster();
  const unsigned ks = cluster.num_blocks(), rank = cluster.block_rank();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int col_block = blockIdx.x / ks;
  const int c0 = col_block * kCols + lane * 4;
  const int m0 = blockIdx.y * MT;
  const int kb = static_cast<int>(rank) * p.k_per_cta;
  const int ke = min(p.k, kb + p.k_per_cta);

  float acc[MT][4];
#pragma unroll
  for (int r = 0; r < MT; ++r)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[r][e] = 0.f;

  const float* arow[MT];
#pragma unroll
  for (int r = 0; r < MT; ++r) arow[r] = p.a + static_cast<int64_t>(min(m0 + r, p.m - 1)) * p.k;

  auto step = [&](int k) {
    float bv[4];
    const float* brow = p.b + static_cast<int64_t>(k) * p.n;
    if (VEC) {
      if (c0 < p.n) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(brow + c0));
        bv[0] = v.x;
        bv[1] = v.y;
        bv[2] = v.z;
        bv[3] = v.w;
      } else {
        bv[0] = bv[1] = bv[2] = bv[3] = 0.f;
      }
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) bv[e] = c0 + e < p.n ? __ldg(brow + c0 + e) : 0.f;
    }
#pragma unroll
    for (int r = 0; r < MT; ++r) {
      const float av = __ldg(arow[r] + k);
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[r][e] = fmaf(av, bv[e], acc[r][e]);
    }
  };
  // warp w takes k = kb + w, kb + w + 8, ...; eight steps' loads in flight together
  int k = kb + warp;
  for (; k + 7 * kWarps < ke; k += 8 * kWarps) {
#pragma unroll
    for (int u = 0; u < 8; ++u) step(k + u * kWarps);
  }
  for (; k < ke; k += kWarps) step(k);

#pragma unroll
  for (int r = 0; r < MT; ++r)
    *reinterpret_cast<float4*>(&red[warp][r][lane * 4]) = make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
  __syncthreads();
  // this CTA's partial, summed over its warps, into red[0]
  for (int i = tid; i < MT * kCols; i += kThreads) {
    const int r = i / kCols, c = i - r * kCols;
    float s = red[0][r][c];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) s += red[w][r][c];
    red[0][r][c] = s;
  }
  cluster.sync();  // every CTA's partial is ready
  if (rank == 0) {
    for (int i = tid; i < MT * kCols; i += kThreads) {
      const int r = i / kCols, c = i - r * kCols;
      float s = red[0][r][c];
      for (unsigned q = 1; q < ks; ++q) s += cluster.map_shared_rank(&red[0][0][0], q)[r * kCols + c];
      const int row = m0 + r, col = col_block * kCols + c;
      if (row < p.m && col < p.n) p.c[static_cast<int64_t>(row) * p.n + col] = s;
    }
  }
  cluster.sync();  // the peers' shared memory stays until the leader has read it
}

template <int MT>
int launch_mt(const Args& p, int col_blocks, int row_tiles, int ks, bool vec, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(col_blocks * ks), static_cast<unsigned>(row_tiles), 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(ks);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t err = vec ? cudaLaunchKernelEx(&cfg, gemm_f32_kernel<MT, true>, p)
                              : cudaLaunchKernelEx(&cfg, gemm_f32_kernel<MT, false>, p);
  if (err != cudaSuccess) return fail(BM_ERR_CUDA, "bm_gemm (fp32): %s", cudaGetErrorString(err));
  return check_launch("bm_gemm (fp32)");
}

}  // namespace gemm32

// c[M][N] = a[M][K] b[K][N] in fp32 (host checks done by the caller).
int gemm_f32(float* c, const float* a, const float* b, int64_t m, int n, int k, cudaStream_t stream) {
  using namespace gemm32;
  if (m == 0 || n == 0) return BM_OK;
  if (k == 0) {  // an empty sum
    const cudaError_t err = cudaMemsetAsync(c, 0, static_cast<size_t>(m) * n * sizeof(float), stream);
    return err == cudaSuccess ? BM_OK : fail(BM_ERR_CUDA, "bm_gemm (fp32): %s", cudaGetErrorString(err));
  }
  const int mt = m >= 8 ? 8 : m >= 4 ? 4 : m >= 2 ? 2 : 1;
  const int64_t row_tiles = (m + mt - 1) / mt;
  if (row_tiles > 65535) return fail(BM_ERR_INVALID_ARGUMENT, "bm_gemm (fp32): more than %d rows", 65535 * 8);
  const int col_blocks = (n + kCols - 1) / kCols;
  // split K over a cluster until the grid covers the GPU twice, keeping >= 64 k per CTA
  const int64_t base = static_cast<int64_t>(col_blocks) * row_tiles;
  int ks = static_cast<int>(std::min<int64_t>(kMaxCluster, (2 * sm_count() + base - 1) / base));
  ks = std::max(1, std::min(ks, (k + 63) / 64));
  Args p{c, a, b, static_cast<int>(m), n, k, (k + ks - 1) / ks};
  const bool vec = n % 4 == 0 && aligned16(b);
  switch (mt) {
    case 8: return launch_mt<8>(p, col_blocks, static_cast<int>(row_tiles), ks, vec, stream);
    case 4: return launch_mt<4>(p, col_blocks, static_cast<int>(row_tiles), ks, vec, stream);
    case 2: return launch_mt<2>(p, col_blocks, static_cast<int>(row_tiles), ks, vec, stream);
    default: return launch_mt<1>(p, col_blocks, static_cast<int>(row_tiles), ks, vec, stream);
  }
}

}  // namespace bm
