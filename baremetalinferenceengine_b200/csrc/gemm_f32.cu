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
// deterministic and no global scratch is needed. Each warp runs its k steps in
// unrolled rounds of eight. When a CTA's K range is short (a few rounds), every
// load of a round is issued before its first multiply-add, the last round's too
// (steps past the range load a valid row and add nothing), so a short K costs a
// memory latency per round, not one per step.
//
// One launch serves several products of the same A (the engine's Q, K and V
// projections: up to three B / C pairs, their column blocks laid end to end), or
// the FFN's two input projections with the SwiGLU applied to the reduced sums
// (out = g / (1 + expf(-g)) * u, the fp32 SwiGLU of src/kernels.cu:185-195 and
// of bm_swiglu, so the result equals the unfused three launches bit for bit).
//
// NORM: A is not read from memory but made in the prologue from the residual
// stream, the RMSNorm that precedes every projection of the engine
// (src/execution_engine.cu:80,109,121 after the adds at :118,126): x = h + d
// (d optional), y = x * rsqrtf(sum(x^2) / K + eps) * w as bm_rmsnorm computes it.
// Every CTA sums the squares of its rows over the whole K and keeps y over its
// own K range in shared memory; the first CTA of each row tile also writes x out
// as the updated residual (to a buffer the other CTAs do not read).
#include <cooperative_groups.h>

#include <algorithm>

#include "bm_common.cuh"
#include "bm_host.h"

namespace cg = cooperative_groups;

namespace bm {
namespace gemm32 {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kCols = 128;  // columns per CTA
constexpr int kMaxCluster = 8;
constexpr int kSteps = 8;   // k steps per warp and round
constexpr int kShortK = 4 * kSteps * kWarps;  // K per CTA up to which the SHORT form runs

struct Args {
  const float* a;
  const float* b[kMaxSharedA];
  float* c[kMaxSharedA];
  int n[kMaxSharedA];
  int block_end[kMaxSharedA];  // column blocks of outputs 0..o together
  int count;                   // products of A (SwiGLU: b[0] gate, b[1] up, one output c[0])
  int m, k;
  int k_per_cta;               // K range of one CTA of the cluster
  // NORM only: A = rmsnorm(norm_h + norm_d) * norm_w, rows [m][k]
  const float* norm_h;
  const float* norm_d;         // may be null: x = h
  const float* norm_w;
  float* norm_out;             // x written here when non-null (never overlapping norm_h / norm_d)
  float eps;
};

// VEC: B rows are 16-byte aligned (N % 4 == 0) and read as float4.
template <bool VEC>
__device__ __forceinline__ void load_b_row(const float* b, int n, int k, int c0, float (&bv)[4]) {
  const float* brow = b + static_cast<int64_t>(k) * n;
  if (VEC) {
    if (c0 < n) {
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
    for (int e = 0; e < 4; ++e) bv[e] = c0 + e < n ? __ldg(brow + c0 + e) : 0.f;
  }
}

// SHORT: each CTA's K range is at most kShortK (the one-token products of small
// models): loads issued a round at a time, at more registers per thread.
template <int MT, bool VEC, bool SWIGLU, bool SHORT, bool NORM>
__global__ void __launch_bounds__(kThreads) gemm_f32_kernel(const Args p) {
  grid_dependency_wait();
  constexpr int kAcc = SWIGLU ? 2 : 1;
  __shared__ __align__(16) float red[kAcc][kWarps][MT][kCols];
  extern __shared__ float a_s[];  // NORM: [MT][k_per_cta] normalised rows, then [k_per_cta] weights: this CTA's K range
  cg::cluster_group cluster = cg::this_cluster();
  const unsigned ks = cluster.num_blocks(), rank = cluster.block_rank();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gblock = static_cast<int>(blockIdx.x / ks);
  // this block's output (selected without indexing the parameter arrays, which would copy them to the stack)
  const int o = SWIGLU ? 0 : (gblock >= p.block_end[0]) + (p.count > 2 && gblock >= p.block_end[1]);
  const int col_block = gblock - (o == 0 ? 0 : o == 1 ? p.block_end[0] : p.block_end[1]);
  const int n = o == 0 ? p.n[0] : o == 1 ? p.n[1] : p.n[2];
  const float* b0 = o == 0 ? p.b[0] : o == 1 ? p.b[1] : p.b[2];
  const float* b1 = SWIGLU ? p.b[1] : nullptr;
  const int c0 = col_block * kCols + lane * 4;
  const int m0 = blockIdx.y * MT;
  const int kb = static_cast<int>(rank) * p.k_per_cta;
  const int ke = min(p.k, kb + p.k_per_cta);

  float acc[kAcc][MT][4];
#pragma unroll
  for (int q = 0; q < kAcc; ++q)
#pragma unroll
    for (int r = 0; r < MT; ++r)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[q][r][e] = 0.f;

  const float* arow[MT];
#pragma unroll
  for (int r = 0; r < MT; ++r) arow[r] = p.a + static_cast<int64_t>(min(m0 + r, p.m - 1)) * p.k;

  // NORM: this CTA's K range of the normalised rows into a_s (every thread calls it)
  auto norm_prologue = [&]() {
    const int kpc = p.k_per_cta;
    float* w_s = a_s + MT * kpc;  // the norm weights of this CTA's K range
    const bool writer = p.norm_out != nullptr && gblock == 0 && rank == 0;
    float* part = &red[0][0][0][0];  // the warps' sums of squares (red is free until the products end)
    for (int r = 0; r < MT; ++r) {
      const int row = m0 + r;  // the same for the whole CTA: the branches below are uniform
      float* ar = a_s + r * kpc;
      if (row >= p.m) {  // a row past the end of the last tile: its products are never stored
        for (int i = tid; i < ke - kb; i += kThreads) ar[i] = 0.f;
        continue;
      }
      const float* hr = p.norm_h + static_cast<int64_t>(row) * p.k;
      const float* dr = p.norm_d != nullptr ? p.norm_d + static_cast<int64_t>(row) * p.k : nullptr;
      float ss = 0.f;
      for (int i = tid; i < p.k; i += kThreads) {  // the weights come in the same round trip as the row
        const bool mine = i >= kb && i < ke;
        const float wv = (r == 0 && mine) ? __ldg(p.norm_w + i) : 0.f;
        float x = hr[i];
        if (dr != nullptr) x += dr[i];
        ss += x * x;
        if (mine) {
          ar[i - kb] = x;
          if (r == 0) w_s[i - kb] = wv;
        }
        if (writer) p.norm_out[static_cast<int64_t>(row) * p.k + i] = x;
      }
      ss = warp_sum(ss);
      if (lane == 0) part[warp] = ss;
      __syncthreads();
      ss = part[0];
#pragma unroll
      for (int w = 1; w < kWarps; ++w) ss += part[w];
      const float scale = rsqrtf(ss / static_cast<float>(p.k) + p.eps);
      for (int i = tid; i < ke - kb; i += kThreads) ar[i] = ar[i] * scale * w_s[i];
      __syncthreads();  // part is reused by the next row; a_s is complete before the products
    }
  };
  // A's value at (row r of the tile, column kk of K)
  auto a_at = [&](int r, int kk) -> float {
    if constexpr (NORM) {
      return a_s[r * p.k_per_cta + (kk - kb)];
    } else {
      return __ldg(arow[r] + kk);
    }
  };

  // warp w takes k = kb + w, kb + w + 8, ... in order, kSteps of them per round
  int k = kb + warp;
  if (SHORT) {
    // a short range (a few rounds): every load of a round is issued before its
    // first multiply-add, steps past the range loading a valid row and adding nothing
    float bv[kAcc][kSteps][4];
    auto load_b_round = [&](int k0) {
#pragma unroll
      for (int u = 0; u < kSteps; ++u) {
        const int kk = min(k0 + u * kWarps, ke - 1);
        load_b_row<VEC>(b0, n, kk, c0, bv[0][u]);
        if (SWIGLU) load_b_row<VEC>(b1, n, kk, c0, bv[kAcc - 1][u]);
      }
    };
    // NORM: the first round's B rows go out before the norm's own loads, so the
    // two memory round trips overlap instead of following one another
    if constexpr (NORM) {
      if (k < ke) load_b_round(k);
      norm_prologue();
    }
    for (bool first = true; k < ke; k += kSteps * kWarps, first = false) {
      float av[kSteps][MT];
      if (!NORM || !first) load_b_round(k);
#pragma unroll
      for (int u = 0; u < kSteps; ++u) {
        const int kk = min(k + u * kWarps, ke - 1);
#pragma unroll
        for (int r = 0; r < MT; ++r) av[u][r] = a_at(r, kk);
      }
#pragma unroll
      for (int u = 0; u < kSteps; ++u) {
        if (k + u * kWarps < ke) {
#pragma unroll
          for (int q = 0; q < kAcc; ++q)
#pragma unroll
            for (int r = 0; r < MT; ++r)
#pragma unroll
              for (int e = 0; e < 4; ++e) acc[q][r][e] = fmaf(av[u][r], bv[q][u][e], acc[q][r][e]);
        }
      }
    }
  } else {
    if constexpr (NORM) norm_prologue();
    // a long range: unrolled rounds (the compiler keeps several steps' loads in
    // flight at the register count of one step), then the remaining steps
    auto step = [&](int kk) {
      float bv[kAcc][4];
      load_b_row<VEC>(b0, n, kk, c0, bv[0]);
      if (SWIGLU) load_b_row<VEC>(b1, n, kk, c0, bv[kAcc - 1]);
#pragma unroll
      for (int r = 0; r < MT; ++r) {
        const float av = a_at(r, kk);
#pragma unroll
        for (int q = 0; q < kAcc; ++q)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[q][r][e] = fmaf(av, bv[q][e], acc[q][r][e]);
      }
    };
    for (; k + (kSteps - 1) * kWarps < ke; k += kSteps * kWarps) {
#pragma unroll
      for (int u = 0; u < kSteps; ++u) step(k + u * kWarps);
    }
    for (; k < ke; k += kWarps) step(k);
  }

#pragma unroll
  for (int q = 0; q < kAcc; ++q)
#pragma unroll
    for (int r = 0; r < MT; ++r)
      *reinterpret_cast<float4*>(&red[q][warp][r][lane * 4]) =
          make_float4(acc[q][r][0], acc[q][r][1], acc[q][r][2], acc[q][r][3]);
  __syncthreads();
  // this CTA's partials, summed over its warps, into red[q][0]
  for (int i = tid; i < kAcc * MT * kCols; i += kThreads) {
    const int q = i / (MT * kCols), rc = i - q * (MT * kCols);
    const int r = rc / kCols, c = rc - r * kCols;
    float s = red[q][0][r][c];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) s += red[q][w][r][c];
    red[q][0][r][c] = s;
  }
  cluster.sync();  // every CTA's partial is ready
  if (rank == 0) {
    float* c_out = o == 0 ? p.c[0] : o == 1 ? p.c[1] : p.c[2];
    for (int i = tid; i < MT * kCols; i += kThreads) {
      const int r = i / kCols, c = i - r * kCols;
      float s = red[0][0][r][c];
      for (unsigned q = 1; q < ks; ++q) s += cluster.map_shared_rank(&red[0][0][0][0], q)[r * kCols + c];
      if (SWIGLU) {
        float u = red[kAcc - 1][0][r][c];
        for (unsigned q = 1; q < ks; ++q) u += cluster.map_shared_rank(&red[kAcc - 1][0][0][0], q)[r * kCols + c];
        s = s / (1.0f + expf(-s)) * u;
      }
      const int row = m0 + r, col = col_block * kCols + c;
      if (row < p.m && col < n) c_out[static_cast<int64_t>(row) * n + col] = s;
    }
  }
  cluster.sync();  // the peers' shared memory stays until the leader has read it
}

template <int MT, bool SWIGLU, bool NORM>
int launch_mt(const Args& p, int col_blocks, int row_tiles, int ks, bool vec, cudaStream_t stream,
              const char* what) {
  const dim3 grid(static_cast<unsigned>(col_blocks * ks), static_cast<unsigned>(row_tiles), 1);
  cudaLaunchAttribute cluster;
  cluster.id = cudaLaunchAttributeClusterDimension;
  cluster.val.clusterDim.x = static_cast<unsigned>(ks);
  cluster.val.clusterDim.y = 1;
  cluster.val.clusterDim.z = 1;
  const int smem = NORM ? (MT + 1) * p.k_per_cta * static_cast<int>(sizeof(float)) : 0;
  auto go = [&](auto kernel) {
    if (smem > 48 * 1024) {
      if (int st = allow_dynamic_smem(reinterpret_cast<const void*>(kernel), smem, what)) return st;
    }
    return launch_kernel(what, kernel, grid, dim3(kThreads), static_cast<size_t>(smem), stream, &cluster, p);
  };
  if (p.k_per_cta <= kShortK) {
    return vec ? go(gemm_f32_kernel<MT, true, SWIGLU, true, NORM>) : go(gemm_f32_kernel<MT, false, SWIGLU, true, NORM>);
  }
  return vec ? go(gemm_f32_kernel<MT, true, SWIGLU, false, NORM>) : go(gemm_f32_kernel<MT, false, SWIGLU, false, NORM>);
}

// Plans and launches: the rows in tiles of MT (at most max_mt), the column blocks
// of every output, and a K split over a cluster until the grid covers the GPU twice.
// NORM: the normalised rows of one CTA's K range must fit its shared memory
// (kMaxNormBytes); run returns kNormDoesNotFit without launching when they do not.
constexpr int kMaxNormBytes = 96 * 1024;
constexpr int kNormDoesNotFit = 1;

template <bool SWIGLU, bool NORM = false>
int run(Args p, int64_t m, bool vec, cudaStream_t stream, const char* what) {
  constexpr int kMaxMt = SWIGLU ? 4 : 8;
  const int mt = m >= kMaxMt ? kMaxMt : m >= 4 ? 4 : m >= 2 ? 2 : 1;
  const int64_t row_tiles = (m + mt - 1) / mt;
  if (row_tiles > 65535) return fail(BM_ERR_INVALID_ARGUMENT, "%s: more than %d rows", what, 65535 * mt);
  const int col_blocks = p.block_end[p.count - 1];
  // the K split is chosen for the plain GEMM's tiling (rows in eights), so the
  // SwiGLU's two products are summed exactly as two bm_gemm calls sum them
  const int plain_mt = m >= 8 ? 8 : m >= 4 ? 4 : m >= 2 ? 2 : 1;
  const int64_t base = static_cast<int64_t>(col_blocks) * ((m + plain_mt - 1) / plain_mt);
  int ks = static_cast<int>(std::min<int64_t>(kMaxCluster, (2 * sm_count() + base - 1) / base));
  ks = std::max(1, std::min(ks, (p.k + 63) / 64));  // keep >= 64 k per CTA
  p.m = static_cast<int>(m);
  p.k_per_cta = (p.k + ks - 1) / ks;
  if (NORM && static_cast<int64_t>(mt + 1) * p.k_per_cta * static_cast<int64_t>(sizeof(float)) > kMaxNormBytes) {
    return kNormDoesNotFit;
  }
  const int rt = static_cast<int>(row_tiles);
  switch (mt) {
    case 8: return launch_mt<(SWIGLU ? 4 : 8), SWIGLU, NORM>(p, col_blocks, rt, ks, vec, stream, what);
    case 4: return launch_mt<4, SWIGLU, NORM>(p, col_blocks, rt, ks, vec, stream, what);
    case 2: return launch_mt<2, SWIGLU, NORM>(p, col_blocks, rt, ks, vec, stream, what);
    default: return launch_mt<1, SWIGLU, NORM>(p, col_blocks, rt, ks, vec, stream, what);
  }
}

}  // namespace gemm32

int gemm_f32_shared_a(float* const* c, const float* a, const float* const* b, const int32_t* n, int count,
                      int64_t m, int k, cudaStream_t stream) {
  using namespace gemm32;
  const char* what = "bm_gemm (fp32)";
  if (m == 0) return BM_OK;
  Args p{};
  p.a = a;
  p.k = k;
  bool vec = true;
  int blocks = 0, live = 0;
  for (int o = 0; o < count; ++o) {
    if (n[o] == 0) continue;  // an empty product: nothing to write
    if (k == 0) {             // an empty sum
      const cudaError_t err = cudaMemsetAsync(c[o], 0, static_cast<size_t>(m) * n[o] * sizeof(float), stream);
      if (err != cudaSuccess) return fail(BM_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
      continue;
    }
    p.b[live] = b[o];
    p.c[live] = c[o];
    p.n[live] = n[o];
    blocks += (n[o] + kCols - 1) / kCols;
    p.block_end[live] = blocks;
    vec = vec && n[o] % 4 == 0 && aligned16(b[o]);
    ++live;
  }
  if (live == 0) return BM_OK;
  p.count = live;
  return run<false>(p, m, vec, stream, what);
}

int gemm_f32(float* c, const float* a, const float* b, int64_t m, int n, int k, cudaStream_t stream) {
  const int32_t n32 = n;
  return gemm_f32_shared_a(&c, a, &b, &n32, 1, m, k, stream);
}

int gemm_f32_swiglu(float* out, const float* x, const float* w_gate, const float* w_up, int64_t rows, int hidden,
                    int dim, cudaStream_t stream) {
  using namespace gemm32;
  const char* what = "bm_gemm_swiglu (fp32)";
  if (rows == 0 || hidden == 0) return BM_OK;
  if (dim == 0) {  // both sums are empty: silu(0) * 0 = 0
    const cudaError_t err = cudaMemsetAsync(out, 0, static_cast<size_t>(rows) * hidden * sizeof(float), stream);
    return err == cudaSuccess ? BM_OK : fail(BM_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
  }
  Args p{};
  p.a = x;
  p.k = dim;
  p.b[0] = w_gate;
  p.b[1] = w_up;
  p.c[0] = out;
  p.n[0] = p.n[1] = hidden;
  p.block_end[0] = (hidden + kCols - 1) / kCols;
  p.count = 1;
  const bool vec = hidden % 4 == 0 && aligned16(w_gate) && aligned16(w_up);
  return run<true>(p, rows, vec, stream, what);
}

int gemm_f32_norm(float* const* c, const float* h, const float* d, const float* norm_w, float eps,
                  float* residual_out, float* normed, const float* const* b, const int32_t* n, int count,
                  bool swiglu, int64_t m, int k, cudaStream_t stream) {
  using namespace gemm32;
  const char* what = "bm_rmsnorm_gemm (fp32)";
  if (m == 0) return BM_OK;
  Args p{};
  p.a = normed;  // read only by the two-launch form
  p.k = k;
  p.norm_h = h;
  p.norm_d = d;
  p.norm_w = norm_w;
  p.norm_out = d != nullptr ? residual_out : nullptr;
  p.eps = eps;
  bool vec = true;
  int blocks = 0, live = 0;
  const int outputs = swiglu ? 1 : count;
  for (int o = 0; o < (swiglu ? 2 : count); ++o) {
    if (!swiglu && n[o] == 0) continue;  // an empty product: nothing to write
    p.b[live] = b[o];
    p.n[live] = n[o];
    if (o < outputs) {
      p.c[live] = c[o];
      blocks += (n[o] + kCols - 1) / kCols;
      p.block_end[live] = blocks;
    }
    vec = vec && n[o] % 4 == 0 && aligned16(b[o]);
    ++live;
  }
  if (live == 0) return BM_OK;
  p.count = swiglu ? 1 : live;
  int st = swiglu ? run<true, true>(p, m, vec, stream, what) : run<false, true>(p, m, vec, stream, what);
  if (st != kNormDoesNotFit) return st;
  // Rows too long for one CTA's shared memory: the norm into `normed`, then the products.
  if (d != nullptr) {
    if (residual_out != nullptr) {
      const cudaError_t err = cudaMemcpyAsync(residual_out, h, static_cast<size_t>(m) * k * sizeof(float),
                                              cudaMemcpyDeviceToDevice, stream);
      if (err != cudaSuccess) return fail(BM_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
      st = bm_add_rmsnorm(residual_out, d, norm_w, normed, m, k, eps, BM_F32, stream);
    } else {
      // the sum is not kept: form it in `normed`, then normalise it in place
      st = bm_add(normed, h, d, m * static_cast<int64_t>(k), BM_F32, stream);
      if (st == BM_OK) st = bm_rmsnorm(normed, normed, norm_w, m, k, eps, k, k, BM_F32, stream);
    }
  } else {
    st = bm_rmsnorm(normed, h, norm_w, m, k, eps, k, k, BM_F32, stream);
  }
  if (st != BM_OK) return st;
  if (swiglu) return gemm_f32_swiglu(c[0], normed, b[0], b[1], m, n[0], k, stream);
  return gemm_f32_shared_a(c, normed, b, n, count, m, k, stream);
}

}  // namespace bm
