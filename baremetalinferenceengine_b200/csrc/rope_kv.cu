// RoPE on Q and K with the K/V write into a static KV cache, for many tokens.
//
// Reference semantics:
//   rope_kernel (src/kernels.cu:126-140): for one token at seq_pos, each pair
//     (x[i], x[i + hd/2]) of every head is rotated by
//     angle = seq_pos / theta^(2i/hd):  x[i] <- x[i] c - x[i+hd/2] s,
//     x[i+hd/2] <- x[i+hd/2] c + x[i] s. launch_rope runs it on q, then on k.
//   kv_store_kernel (src/kernels.cu:211-217):
//     cache[(h * max_seq + pos) * hd + d] = src[h * hd + d].
//   ExecutionEngine::run_layers calls rope, then kv_store for k and for v
//   (src/execution_engine.cu:113-115): four launches per token per layer.
//
// Here one launch covers all tokens and, in the fused mode, does all three
// steps: a block takes one token (grid-stride over tokens), stages that token's
// (cos, sin) row in shared memory — from the position-keyed fp32 table, or
// computed in fp64 when no table is given — and splits the token's work into
// units: a Q pair unit rotates VEC elements from each half of one head in place,
// a K pair unit rotates one K head's VEC pairs straight into k_cache, and a V
// unit copies VEC elements into v_cache. Each thread issues the loads of up to
// UPT units before the table barrier, so HBM latency overlaps the staging.
// The cache layout is [num_seqs][num_kv_heads][max_seq][head_dim]
// (include/kv_cache.h:37-40, with the batch dimension used).
//
// The (cos, sin) table is computed on the device in fp64 with CUDA's pow and
// sincos, following the reference's CPU check loop (tests/kernel_tests.cu:180),
// and rounded once to fp32. Rotation arithmetic is fp32.
#include <algorithm>

#include "bm_common.cuh"
#include "bm_host.h"
#include "rope_kv_device.cuh"

namespace bm {
namespace {

using namespace ropekv;

template <typename T, int VEC, int MODE>
__global__ void __launch_bounds__(256) rope_kv_kernel(RopeArgs a) {
  prefetch_token<T, MODE>(a, blockIdx.x, threadIdx.x, blockDim.x);
  grid_dependency_wait();
  __shared__ float2 cs[kMaxHalf];
  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
    rope_kv_token<T, VEC, MODE>(a, row, threadIdx.x, blockDim.x, cs);
  }
}

// Warp-per-token variant for large batches. Lane l owns pair chunk c = l % upv
// of every head, so the VEC (cos, sin) pairs of that chunk are fetched once per
// token and stay in registers for all of the token's Q and K heads; lanes
// l / upv = 0..hpi-1 take heads h0, h0 + hpi, ... (hpi = 32 / upv heads per
// pass, UNROLL passes' loads in flight together). No shared memory and no block
// barrier: tokens on different warps never wait on one another.
#ifndef BM_ROPE_WARP_UNROLL
#define BM_ROPE_WARP_UNROLL 4  // passes whose loads a lane keeps in flight
#endif
#ifndef BM_ROPE_WARP_MINB
#define BM_ROPE_WARP_MINB 2  // resident 256-thread blocks per SM the register budget must allow
#endif
#ifndef BM_ROPE_WARP_MIN_ROWS
#define BM_ROPE_WARP_MIN_ROWS 512  // smaller batches: one block per token spreads a token wider
#endif
constexpr int kWarpUnroll = BM_ROPE_WARP_UNROLL;
constexpr int64_t kWarpKernelMinRows = BM_ROPE_WARP_MIN_ROWS;

template <typename T, int VEC>
__device__ __forceinline__ void rotate(Chunk<T, VEC>& c1, Chunk<T, VEC>& c2, const float2* cs) {
  float x1[VEC], x2[VEC];
  c1.get(x1);
  c2.get(x2);
#pragma unroll
  for (int e = 0; e < VEC; ++e) {
    rope_rotate(x1[e], x2[e], cs[e], &x1[e], &x2[e]);
  }
  c1.set(x1);
  c2.set(x2);
}

// TABLE: (cos, sin) from the table (a.table != NULL); otherwise computed in fp64,
// whose pow / sincos need far more registers, so each form gets its own build.
template <typename T, int VEC, int MODE, bool TABLE>
__global__ void __launch_bounds__(256, BM_ROPE_WARP_MINB) rope_kv_warp_kernel(RopeArgs a) {
  constexpr int U = kWarpUnroll;
  const int lane = threadIdx.x & 31;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  prefetch_token<T, MODE>(a, warp, lane, 32);
  grid_dependency_wait();
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int upv = MODE == kStore ? 1 : a.upv;  // host guarantees 1 <= upv <= 32 for pair modes
  const int hpi = 32 / upv;
  const int c = lane % upv;
  const int h0 = lane / upv;
  const bool pair_lane = MODE != kStore && h0 < hpi;
  const int64_t cache_head_stride = static_cast<int64_t>(a.max_seq) * a.hd;
  const int nv = a.hkv * a.cpv;

  for (int64_t row = warp; row < a.rows; row += nwarps) {
    const int32_t pos = a.positions ? a.positions[row] : static_cast<int32_t>(a.pos0 + row);
    const int32_t seq = a.seq_ids ? a.seq_ids[row] : 0;
    int32_t bad = 0;
    if (pos < 0) bad |= BM_DEVERR_BAD_POSITION;
    if (MODE != kRope) {
      if (pos >= a.max_seq) bad |= BM_DEVERR_BAD_POSITION;
      if (seq < 0 || seq >= a.num_seqs) bad |= BM_DEVERR_BAD_SEQUENCE;
    }
    if (MODE != kStore && TABLE && pos >= a.table_len) bad |= BM_DEVERR_BAD_POSITION;
    if (bad) {  // uniform across the warp
      if (lane == 0) raise_status(a.status, bad);
      continue;
    }
    const int64_t cache_base =
        MODE == kRope ? 0 : (static_cast<int64_t>(seq) * a.hkv * a.max_seq + pos) * a.hd;

    float2 cs[VEC];
    if (pair_lane) {
      if constexpr (TABLE) {
        const float2* t = a.table + static_cast<int64_t>(pos) * a.half + c * VEC;
        if (VEC % 2 == 0 && a.table_vec4) {
#pragma unroll
          for (int e = 0; e + 1 < VEC; e += 2) {
            const float4 two = __ldg(reinterpret_cast<const float4*>(t + e));
            cs[e] = make_float2(two.x, two.y);
            cs[e + 1] = make_float2(two.z, two.w);
          }
        } else {
#pragma unroll
          for (int e = 0; e < VEC; ++e) cs[e] = __ldg(t + e);
        }
      } else {
#pragma unroll
        for (int e = 0; e < VEC; ++e) cs[e] = angle_cos_sin(pos, c * VEC + e, a.theta, a.hd);
      }
      // Q: rotated in place
      T* qrow = static_cast<T*>(a.q) + row * a.hq * a.hd + c * VEC;
      for (int hb = h0; hb < a.hq; hb += hpi * U) {
        Chunk<T, VEC> x1[U], x2[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int h = hb + u * hpi;
          if (h < a.hq) {
            x1[u].load(qrow + static_cast<int64_t>(h) * a.hd);
            x2[u].load(qrow + static_cast<int64_t>(h) * a.hd + a.half);
          }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int h = hb + u * hpi;
          if (h < a.hq) {
            rotate<T, VEC>(x1[u], x2[u], cs);
            x1[u].store(qrow + static_cast<int64_t>(h) * a.hd);
            x2[u].store(qrow + static_cast<int64_t>(h) * a.hd + a.half);
          }
        }
      }
      // K: rotated into the cache (fused) or in place (rope only)
      T* krow = static_cast<T*>(a.k) + row * a.hkv * a.hd + c * VEC;
      for (int hb = h0; hb < a.hkv; hb += hpi * U) {
        Chunk<T, VEC> x1[U], x2[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int h = hb + u * hpi;
          if (h < a.hkv) {
            x1[u].load(krow + static_cast<int64_t>(h) * a.hd);
            x2[u].load(krow + static_cast<int64_t>(h) * a.hd + a.half);
          }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int h = hb + u * hpi;
          if (h < a.hkv) {
            rotate<T, VEC>(x1[u], x2[u], cs);
            T* dst = MODE == kFused
                         ? static_cast<T*>(a.k_cache) + cache_base + h * cache_head_stride + c * VEC
                         : krow + static_cast<int64_t>(h) * a.hd;
            x1[u].store(dst);
            x2[u].store(dst + a.half);
          }
        }
      }
    }
    // V (fused) or src (store): copied into the cache, VEC elements per lane per pass
    if (MODE != kRope) {
      const T* vrow = static_cast<const T*>(a.v) + row * a.hkv * a.hd;
      T* vdst = static_cast<T*>(a.v_cache) + cache_base;
      for (int i0 = lane; i0 < nv; i0 += 32 * U) {
        Chunk<T, VEC> d[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int i = i0 + u * 32;
          if (i < nv) d[u].load(vrow + static_cast<int64_t>(i) * VEC);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int i = i0 + u * 32;
          if (i < nv) {
            const int h = i / a.cpv;
            d[u].store(vdst + h * cache_head_stride + (i - h * a.cpv) * VEC);
          }
        }
      }
    }
  }
}

__global__ void rope_table_kernel(float2* table, int32_t max_pos, int half, int hd, double theta) {
  grid_dependency_wait();
  const int64_t n = static_cast<int64_t>(max_pos) * half;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < n;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t p = idx / half;
    const int i = static_cast<int>(idx - p * half);
    const double angle = static_cast<double>(p) / pow(theta, 2.0 * i / hd);
    double s, c;
    sincos(angle, &s, &c);
    table[idx] = make_float2(static_cast<float>(c), static_cast<float>(s));
  }
}

template <typename T, int VEC, int MODE>
int launch_typed(const RopeArgs& a, cudaStream_t stream, const char* what) {
  if (a.rows >= kWarpKernelMinRows && (MODE == kStore || (a.upv >= 1 && a.upv <= 32))) {
    const int64_t blocks = (a.rows + 7) / 8;  // 8 warps (tokens in flight) per 256-thread block
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>(blocks, static_cast<int64_t>(sm_count()) * 16));
    auto kernel = a.table != nullptr ? rope_kv_warp_kernel<T, VEC, MODE, true> : rope_kv_warp_kernel<T, VEC, MODE, false>;
    if (const int launch_status = launch_kernel("rope_kv_warp_kernel", kernel, dim3(grid),
                                                dim3(256), 0, stream, nullptr, a)) {
      return launch_status;
    }
    return check_launch(what);
  }
  const int want = (a.total_units + kUPT - 1) / kUPT;
  const int block = std::min(256, std::max(64, (want + 31) / 32 * 32));
  const int64_t cap = static_cast<int64_t>(sm_count()) * (2048 / block);
  const unsigned grid = static_cast<unsigned>(std::max<int64_t>(1, std::min(a.rows, cap)));
  if (const int launch_status = launch_kernel("rope_kv_kernel", rope_kv_kernel<T, VEC, MODE>, dim3(grid), dim3(block),
                                              0, stream, nullptr, a)) {
    return launch_status;
  }
  return check_launch(what);
}

template <int MODE>
int launch(RopeArgs a, bm_dtype_t dtype, cudaStream_t stream, const char* what) {
  const int es = dtype_size(dtype);
  const int vec = 16 / es;
  // Both halves of a pair (or a whole head when only copying) split into VEC-element chunks.
  bool vec_ok = (MODE == kStore ? a.hd : a.half) % vec == 0;
  for (const void* p : {static_cast<const void*>(a.q), static_cast<const void*>(a.k), a.v,
                        static_cast<const void*>(a.k_cache), static_cast<const void*>(a.v_cache)}) {
    if (p != nullptr && !aligned16(p)) vec_ok = false;
  }
  const int v_used = vec_ok ? vec : 1;
  a.table_vec4 = a.table != nullptr && aligned16(a.table);
  set_units(a, v_used, MODE);
  if (a.total_units == 0) return BM_OK;
  if (dtype == BM_F32) {
    return vec_ok ? launch_typed<float, 4, MODE>(a, stream, what) : launch_typed<float, 1, MODE>(a, stream, what);
  }
  return vec_ok ? launch_typed<bf16, 8, MODE>(a, stream, what) : launch_typed<bf16, 1, MODE>(a, stream, what);
}

int check_common(const char* what, int64_t rows, int hd, bm_dtype_t dtype) {
  if (!valid_dtype(dtype)) return fail(BM_ERR_INVALID_ARGUMENT, "%s: bad dtype %d", what, static_cast<int>(dtype));
  if (rows < 0) return fail(BM_ERR_INVALID_ARGUMENT, "%s: negative rows", what);
  if (hd <= 0 || hd > 2 * kMaxHalf) {
    return fail(BM_ERR_INVALID_ARGUMENT, "%s: head_dim %d outside [1, %d]", what, hd, 2 * kMaxHalf);
  }
  return BM_OK;
}

int check_table(const char* what, const void* table, int32_t table_len, double theta) {
  if (table != nullptr) {
    if (table_len <= 0) return fail(BM_ERR_INVALID_ARGUMENT, "%s: table_len must be > 0", what);
    if ((reinterpret_cast<uintptr_t>(table) & 7u) != 0) return fail(BM_ERR_INVALID_ARGUMENT, "%s: table not 8-byte aligned", what);
  } else if (!(theta > 0.0)) {
    return fail(BM_ERR_INVALID_ARGUMENT, "%s: theta must be > 0 without a table", what);
  }
  return BM_OK;
}

}  // namespace
}  // namespace bm

extern "C" int bm_rope_kv_store(void* q, const void* k, const void* v, const int32_t* positions, int32_t pos0,
                                const int32_t* seq_ids, void* k_cache, void* v_cache, const void* rope_table,
                                int32_t table_len, double theta, int64_t rows, int32_t num_q_heads,
                                int32_t num_kv_heads, int32_t head_dim, int32_t max_seq, int32_t num_seqs,
                                bm_dtype_t dtype, int32_t* d_status, void* stream) {
  using namespace bm;
  const char* what = "bm_rope_kv_store";
  if (int st = check_common(what, rows, head_dim, dtype)) return st;
  if (head_dim % 2) return fail(BM_ERR_INVALID_ARGUMENT, "%s: head_dim must be even", what);
  if (num_q_heads < 0 || num_kv_heads < 0 || max_seq <= 0 || num_seqs <= 0) {
    return fail(BM_ERR_INVALID_ARGUMENT, "%s: bad head counts, max_seq or num_seqs", what);
  }
  if (int st = check_table(what, rope_table, table_len, theta)) return st;
  if (rows == 0 || (num_q_heads == 0 && num_kv_heads == 0)) return BM_OK;
  if ((num_q_heads > 0 && !q) || (num_kv_heads > 0 && (!k || !v || !k_cache || !v_cache))) {
    return fail(BM_ERR_INVALID_ARGUMENT, "%s: NULL pointer", what);
  }
  if (!positions && (pos0 < 0 || static_cast<int64_t>(pos0) + rows > max_seq)) {
    return fail(BM_ERR_INVALID_ARGUMENT, "%s: positions pos0..pos0+rows-1 outside [0, max_seq)", what);
  }
  RopeArgs a{};
  a.q = q;
  a.k = const_cast<void*>(k);
  a.v = v;
  a.positions = positions;
  a.pos0 = pos0;
  a.seq_ids = seq_ids;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.table = static_cast<const float2*>(rope_table);
  a.table_len = table_len;
  a.theta = theta;
  a.rows = rows;
  a.hq = num_q_heads;
  a.hkv = num_kv_heads;
  a.hd = head_dim;
  a.half = head_dim / 2;
  a.max_seq = max_seq;
  a.num_seqs = num_seqs;
  a.status = d_status;
  return launch<kFused>(a, dtype, as_stream(stream), what);
}

extern "C" int bm_rope(void* q, void* k, const int32_t* positions, int32_t pos0, const void* rope_table,
                       int32_t table_len, double theta, int64_t rows, int32_t num_q_heads, int32_t num_kv_heads,
                       int32_t head_dim, bm_dtype_t dtype, int32_t* d_status, void* stream) {
  using namespace bm;
  const char* what = "bm_rope";
  if (int st = check_common(what, rows, head_dim, dtype)) return st;
  if (head_dim % 2) return fail(BM_ERR_INVALID_ARGUMENT, "%s: head_dim must be even", what);
  if (num_q_heads < 0 || num_kv_heads < 0) return fail(BM_ERR_INVALID_ARGUMENT, "%s: negative head count", what);
  if (int st = check_table(what, rope_table, table_len, theta)) return st;
  if (rows == 0 || (num_q_heads == 0 && num_kv_heads == 0)) return BM_OK;
  if ((num_q_heads > 0 && !q) || (num_kv_heads > 0 && !k)) return fail(BM_ERR_INVALID_ARGUMENT, "%s: NULL pointer", what);
  if (!positions && pos0 < 0) return fail(BM_ERR_INVALID_ARGUMENT, "%s: negative position", what);
  RopeArgs a{};
  a.q = q;
  a.k = k;
  a.positions = positions;
  a.pos0 = pos0;
  a.table = static_cast<const float2*>(rope_table);
  a.table_len = table_len;
  a.theta = theta;
  a.rows = rows;
  a.hq = num_q_heads;
  a.hkv = num_kv_heads;
  a.hd = head_dim;
  a.half = head_dim / 2;
  a.max_seq = 1;
  a.num_seqs = 1;
  a.status = d_status;
  return launch<kRope>(a, dtype, as_stream(stream), what);
}

extern "C" int bm_kv_store(void* cache, const void* src, const int32_t* positions, int32_t pos0,
                           const int32_t* seq_ids, int64_t rows, int32_t num_heads, int32_t head_dim,
                           int32_t max_seq, int32_t num_seqs, bm_dtype_t dtype, int32_t* d_status, void* stream) {
  using namespace bm;
  const char* what = "bm_kv_store";
  if (int st = check_common(what, rows, head_dim, dtype)) return st;
  if (num_heads < 0 || max_seq <= 0 || num_seqs <= 0) {
    return fail(BM_ERR_INVALID_ARGUMENT, "%s: bad num_heads, max_seq or num_seqs", what);
  }
  if (rows == 0 || num_heads == 0) return BM_OK;
  if (!cache || !src) return fail(BM_ERR_INVALID_ARGUMENT, "%s: NULL pointer", what);
  if (!positions && (pos0 < 0 || static_cast<int64_t>(pos0) + rows > max_seq)) {
    return fail(BM_ERR_INVALID_ARGUMENT, "%s: positions pos0..pos0+rows-1 outside [0, max_seq)", what);
  }
  RopeArgs a{};
  a.v = src;
  a.v_cache = cache;
  a.positions = positions;
  a.pos0 = pos0;
  a.seq_ids = seq_ids;
  a.rows = rows;
  a.hkv = num_heads;
  a.hd = head_dim;
  a.half = head_dim / 2;
  a.max_seq = max_seq;
  a.num_seqs = num_seqs;
  a.status = d_status;
  return launch<kStore>(a, dtype, as_stream(stream), what);
}

extern "C" int bm_rope_table_fill(void* table, int32_t max_pos, int32_t head_dim, double theta, void* stream) {
  using namespace bm;
  const char* what = "bm_rope_table_fill";
  if (max_pos <= 0 || head_dim <= 0 || head_dim % 2 || !(theta > 0.0)) {
    return fail(BM_ERR_INVALID_ARGUMENT, "%s: need max_pos > 0, even head_dim > 0, theta > 0", what);
  }
  if (!table || (reinterpret_cast<uintptr_t>(table) & 7u)) return fail(BM_ERR_INVALID_ARGUMENT, "%s: bad table pointer", what);
  const int half = head_dim / 2;
  const int64_t n = static_cast<int64_t>(max_pos) * half;
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, static_cast<int64_t>(sm_count()) * 8));
  if (const int launch_status = launch_kernel("rope_table_kernel", rope_table_kernel, dim3(grid), dim3(256), 0,
                                              as_stream(stream), nullptr, static_cast<float2*>(table), max_pos, half,
                                              head_dim, theta)) {
    return launch_status;
  }
  return check_launch(what);
}

extern "C" int bm_rope_table_create(int32_t max_pos, int32_t head_dim, double theta, void** table_out) {
  using namespace bm;
  if (!table_out) return fail(BM_ERR_INVALID_ARGUMENT, "bm_rope_table_create: NULL table_out");
  *table_out = nullptr;
  if (max_pos <= 0 || head_dim <= 0 || head_dim % 2 || !(theta > 0.0)) {
    return fail(BM_ERR_INVALID_ARGUMENT, "bm_rope_table_create: need max_pos > 0, even head_dim > 0, theta > 0");
  }
  void* p = nullptr;
  const size_t bytes = static_cast<size_t>(max_pos) * head_dim / 2 * sizeof(float2);
  cudaError_t err = cudaMalloc(&p, bytes);
  if (err != cudaSuccess) return fail(BM_ERR_CUDA, "bm_rope_table_create: cudaMalloc: %s", cudaGetErrorString(err));
  int st = bm_rope_table_fill(p, max_pos, head_dim, theta, nullptr);
  if (st == BM_OK) {
    err = cudaStreamSynchronize(nullptr);
    if (err != cudaSuccess) st = fail(BM_ERR_CUDA, "bm_rope_table_create: %s", cudaGetErrorString(err));
  }
  if (st != BM_OK) {
    cudaFree(p);
    return st;
  }
  *table_out = p;
  return BM_OK;
}

extern "C" int bm_rope_table_destroy(void* table) {
  if (table == nullptr) return BM_OK;
  cudaError_t err = cudaFree(table);
  if (err != cudaSuccess) return bm::fail(BM_ERR_CUDA, "bm_rope_table_destroy: %s", cudaGetErrorString(err));
  return BM_OK;
}
