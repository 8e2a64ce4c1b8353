// One layer step's memory-bound ops, with a single launch for decode-sized batches.
//
// A step is the in-scope half of ExecutionEngine::run_layers for a batch of
// tokens (src/execution_engine.cu:98-126): the embedding row copy (:98-99), the
// residual add before attention with its RMSNorm (:118, :109), RoPE on q and k
// with the K/V cache writes (:113-115), the residual add before the FFN with its
// RMSNorm (:126, :121) and SwiGLU (:124). The GEMM outputs those ops read
// (attn_out, q/k/v, ffn_out, gate/up) are inputs of the step.
//
// Large batches issue the five batched kernels (each streams at the HBM
// roofline on its own). A decode step of 64 Llama-3-8B tokens moves about
// 12 MB, and there five dependent launches cost more than the bytes. But the
// only dependency between the step's ops is the residual, and it is row-local,
// so one launch holds three kinds of independent jobs, one per thread block:
//   row job r:     h1 = embed[ids[r]] + attn_out[r]; y_attn = rmsnorm(h1) * w_attn;
//                  h2 = h1 + ffn_out[r]; y_ffn = rmsnorm(h2) * w_ffn; hidden[r] = h2.
//                  The row stays in registers: hidden is written once, never read
//                  (a bad id keeps hidden's old row as h0, as the gather leaves it);
//   token job t:   RoPE on q[t] and k[t], rotated k and raw v into the cache (the
//                  block-per-token body of rope_kv.cu);
//   SwiGLU job j:  4 16-byte vectors of gate/up per thread.
// No job waits for another. The results equal the five launches': h1 and h2 are
// rounded to the storage type exactly where the separate kernels store them, the
// residual and the copies are bit-identical, and the norms use the same formula
// (in * rsqrt(mean(in^2) + eps) * w) with a different summation order.
#include <algorithm>
#include <initializer_list>

#include "bm_common.cuh"
#include "bm_host.h"
#include "rope_kv_device.cuh"

namespace bm {
namespace {

// Blocks of 128 threads (each thread holding up to 8 of a row's 16-byte vectors)
// for rows of at most 1024 vectors, 256 above: small blocks keep a decode batch's
// jobs in one wave of resident blocks.
constexpr int kMaxWarps = 8;
constexpr int kMaxKV = 8;
constexpr int kSwigluUnroll = 4;  // 16-byte vectors per operand per thread of a SwiGLU job
#ifndef BM_STEP_FUSED_MAX_ROWS
#define BM_STEP_FUSED_MAX_ROWS 512  // batches up to this many tokens take the single launch
#endif
constexpr int64_t kFusedMaxRows = BM_STEP_FUSED_MAX_ROWS;

struct StepArgs {
  int64_t rows, vocab;
  int dim;
  float eps;
  const int32_t* ids;
  const void* embed;
  void* hidden;
  const void* attn_out;
  const void* w_attn;
  void* y_attn;
  const void* ffn_out;
  const void* w_ffn;
  void* y_ffn;
  const void* gate;
  const void* up;
  void* act;
  int64_t swiglu_n;     // rows * ffn elements
  int64_t swiglu_nvec;  // whole 16-byte vectors of them
  int64_t rope_jobs;    // rows, or 0 without heads
  int64_t swiglu_jobs;
  ropekv::RopeArgs rope;
  int32_t* status;
};

// A 16-byte asynchronous copy from global into shared memory (cp.async, cached in
// L2 only), and the wait for this thread's outstanding copies.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(smem))),
               "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Block-wide sum over THREADS threads; every thread gets it. `part` holds one
// slot per warp.
template <int THREADS>
__device__ __forceinline__ float block_sum(float v, float* part) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < THREADS / 32; ++i) s += part[i];
  return s;
}

template <typename T, int KV, int THREADS>
__device__ __forceinline__ void row_job(const StepArgs& a, int64_t row, int tid, float (*part)[kMaxWarps],
                                        uint4* w_s) {
  constexpr int N = VecWidth<T>::value;
  const int nv = a.dim / N;
  const int64_t off = row * a.dim;
  // Both norms' weights go into shared memory asynchronously (w_s: nv vectors of
  // w_attn, then nv of w_ffn): they land while the id and the embedding row come
  // from DRAM, and neither norm waits on a load after its reduction.
  for (int v = tid; v < nv; v += THREADS) {
    cp_async16(w_s + v, static_cast<const T*>(a.w_attn) + static_cast<int64_t>(v) * N);
    cp_async16(w_s + nv + v, static_cast<const T*>(a.w_ffn) + static_cast<int64_t>(v) * N);
  }
  uint4 e[KV], p1[KV], p2[KV];
#pragma unroll
  for (int k = 0; k < KV; ++k) {  // the deltas first: they do not wait for the id
    const int v = tid + k * THREADS;
    if (v < nv) {
      p1[k] = ld_stream(static_cast<const T*>(a.attn_out) + off + static_cast<int64_t>(v) * N);
      p2[k] = ld_stream(static_cast<const T*>(a.ffn_out) + off + static_cast<int64_t>(v) * N);
    }
  }
  const int32_t id = a.ids[row];
  const bool bad = id < 0 || id >= a.vocab;  // uniform across the block
  if (bad) {
    if (tid == 0) raise_status(a.status, BM_DEVERR_BAD_ID);
    const T* src = static_cast<const T*>(a.hidden) + off;  // the gather leaves the row as it was
#pragma unroll
    for (int k = 0; k < KV; ++k) {
      const int v = tid + k * THREADS;
      if (v < nv) e[k] = ld_stream(src + static_cast<int64_t>(v) * N);
    }
  } else {
    const T* src = static_cast<const T*>(a.embed) + static_cast<int64_t>(id) * a.dim;
#pragma unroll
    for (int k = 0; k < KV; ++k) {
      const int v = tid + k * THREADS;
      if (v < nv) e[k] = ld_keep(src + static_cast<int64_t>(v) * N);
    }
  }
  float h[KV][N];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < KV; ++k) {
    const int v = tid + k * THREADS;
    if (v < nv) {
      float x[N], d[N];
      unpack16<T>(e[k], x);
      unpack16<T>(p1[k], d);
#pragma unroll
      for (int i = 0; i < N; ++i) {
        h[k][i] = round_to<T>(x[i] + d[i]);  // the residual as the add stores it
        ss += h[k][i] * h[k][i];
      }
    }
  }
  cp_async_wait_all();  // this thread's weight copies; block_sum's barrier then publishes everyone's
  const float scale1 = rsqrtf(block_sum<THREADS>(ss, part[0]) / static_cast<float>(a.dim) + a.eps);
  ss = 0.f;
#pragma unroll
  for (int k = 0; k < KV; ++k) {
    const int v = tid + k * THREADS;
    if (v < nv) {
      float w[N], y[N], d[N];
      unpack16<T>(w_s[v], w);
#pragma unroll
      for (int i = 0; i < N; ++i) y[i] = h[k][i] * scale1 * w[i];
      st_plain(static_cast<T*>(a.y_attn) + off + static_cast<int64_t>(v) * N, pack16<T>(y));
      unpack16<T>(p2[k], d);
#pragma unroll
      for (int i = 0; i < N; ++i) {
        h[k][i] = round_to<T>(h[k][i] + d[i]);
        ss += h[k][i] * h[k][i];
      }
    }
  }
  const float scale2 = rsqrtf(block_sum<THREADS>(ss, part[1]) / static_cast<float>(a.dim) + a.eps);
#pragma unroll
  for (int k = 0; k < KV; ++k) {
    const int v = tid + k * THREADS;
    if (v < nv) {
      float w[N], y[N];
      unpack16<T>(w_s[nv + v], w);
#pragma unroll
      for (int i = 0; i < N; ++i) y[i] = h[k][i] * scale2 * w[i];
      st_plain(static_cast<T*>(a.y_ffn) + off + static_cast<int64_t>(v) * N, pack16<T>(y));
      st_plain(static_cast<T*>(a.hidden) + off + static_cast<int64_t>(v) * N, pack16<T>(h[k]));
    }
  }
}

template <typename T, int THREADS>
__device__ __forceinline__ void swiglu_job(const StepArgs& a, int64_t job, int tid) {
  constexpr int N = VecWidth<T>::value;
  const int64_t base = job * THREADS * kSwigluUnroll + tid;
  uint4 g[kSwigluUnroll], u[kSwigluUnroll];
#pragma unroll
  for (int k = 0; k < kSwigluUnroll; ++k) {
    const int64_t v = base + static_cast<int64_t>(k) * THREADS;
    if (v < a.swiglu_nvec) {
      g[k] = ld_stream(static_cast<const T*>(a.gate) + v * N);
      u[k] = ld_stream(static_cast<const T*>(a.up) + v * N);
    }
  }
#pragma unroll
  for (int k = 0; k < kSwigluUnroll; ++k) {
    const int64_t v = base + static_cast<int64_t>(k) * THREADS;
    if (v < a.swiglu_nvec) {
      float fg[N], fu[N];
      unpack16<T>(g[k], fg);
      unpack16<T>(u[k], fu);
#pragma unroll
      for (int i = 0; i < N; ++i) fg[i] = swiglu1<T>(fg[i], fu[i]);
      st_plain(static_cast<T*>(a.act) + v * N, pack16<T>(fg));
    }
  }
  if (job == a.swiglu_jobs - 1) {  // elements past the last whole vector
    for (int64_t i = a.swiglu_nvec * N + tid; i < a.swiglu_n; i += THREADS) {
      store1<T>(static_cast<T*>(a.act) + i,
                swiglu1<T>(load1<T>(static_cast<const T*>(a.gate) + i), load1<T>(static_cast<const T*>(a.up) + i)));
    }
  }
}

// Blocks [0, rows): row jobs; [rows, rows + rope_jobs): token jobs; the rest: SwiGLU jobs.
template <typename T, int KV, int THREADS>
__global__ void __launch_bounds__(THREADS) layer_step_small_kernel(StepArgs a) {
  constexpr int N = VecWidth<T>::value;
  __shared__ float2 cs[ropekv::kMaxHalf];
  __shared__ float part[2][kMaxWarps];
  const int tid = threadIdx.x;
  const int64_t job = blockIdx.x;
  const int64_t es = sizeof(T);
  // the job's first lines, while the previous kernel finishes (the norm weights,
  // read by every row job, come into L2 for the later phases)
  if (job < a.rows) {
    if (tid == 0) prefetch_l2(a.ids + job);
    prefetch_l2_range(static_cast<const T*>(a.attn_out) + job * a.dim, a.dim * es, tid, THREADS);
    prefetch_l2_range(static_cast<const T*>(a.ffn_out) + job * a.dim, a.dim * es, tid, THREADS);
    prefetch_l2_range(a.w_attn, a.dim * es, tid, THREADS);
    prefetch_l2_range(a.w_ffn, a.dim * es, tid, THREADS);
  } else if (job < a.rows + a.rope_jobs) {
    ropekv::prefetch_token<T, ropekv::kFused>(a.rope, job - a.rows, tid, THREADS);
  } else {
    const int64_t v = (job - a.rows - a.rope_jobs) * THREADS * kSwigluUnroll + tid;
    if (v < a.swiglu_nvec) {
      prefetch_l2(static_cast<const T*>(a.gate) + v * N);
      prefetch_l2(static_cast<const T*>(a.up) + v * N);
    }
  }
  grid_dependency_wait();
  if (job < a.rows) {
    extern __shared__ uint4 w_s[];  // row jobs: the two norm weight vectors
    row_job<T, KV, THREADS>(a, job, tid, part, w_s);
  } else if (job < a.rows + a.rope_jobs) {
    ropekv::rope_kv_token<T, N, ropekv::kFused>(a.rope, job - a.rows, tid, THREADS, cs);
  } else {
    swiglu_job<T, THREADS>(a, job - a.rows - a.rope_jobs, tid);
  }
}

// Threads per block for rows of nv 16-byte vectors (at most kMaxKV per thread).
int block_threads(int nv) { return nv <= kMaxKV * 128 ? 128 : 256; }

template <typename T>
int launch_small(const StepArgs& a, cudaStream_t stream) {
  constexpr int N = VecWidth<T>::value;
  const int nv = a.dim / N;
  const int threads = block_threads(nv);
  const int64_t blocks = a.rows + a.rope_jobs + a.swiglu_jobs;
  const dim3 grid(static_cast<unsigned>(blocks)), block(threads);
  const char* name = "layer_step_small_kernel";
  const int smem = 2 * nv * 16;  // the row jobs' norm weights
  auto go = [&](auto kernel) {
    if (smem > 48 * 1024) {
      if (int st = allow_dynamic_smem(reinterpret_cast<const void*>(kernel), smem, name)) return st;
    }
    return launch_kernel(name, kernel, grid, block, static_cast<size_t>(smem), stream, nullptr, a);
  };
  if (threads == 256) return go(layer_step_small_kernel<T, 8, 256>);
  if (nv <= 128) return go(layer_step_small_kernel<T, 1, 128>);
  if (nv <= 256) return go(layer_step_small_kernel<T, 2, 128>);
  if (nv <= 512) return go(layer_step_small_kernel<T, 4, 128>);
  return go(layer_step_small_kernel<T, 8, 128>);
}

bool all_aligned16(std::initializer_list<const void*> ptrs) {
  for (const void* p : ptrs) {
    if (!aligned16(p)) return false;
  }
  return true;
}

}  // namespace
}  // namespace bm

extern "C" int bm_layer_step(const bm_layer_step_t* s, bm_dtype_t dtype, int32_t* d_status, void* stream) {
  using namespace bm;
  const char* what = "bm_layer_step";
  if (!s) return fail(BM_ERR_INVALID_ARGUMENT, "%s: NULL step", what);
  if (!valid_dtype(dtype)) return fail(BM_ERR_INVALID_ARGUMENT, "%s: bad dtype %d", what, static_cast<int>(dtype));
  if (s->rows < 0 || s->dim <= 0 || s->ffn <= 0 || s->vocab <= 0 || s->num_q_heads < 0 || s->num_kv_heads < 0 ||
      s->head_dim <= 0 || s->head_dim % 2 || s->max_seq <= 0 || s->num_seqs <= 0) {
    return fail(BM_ERR_INVALID_ARGUMENT, "%s: bad sizes", what);
  }
  if (s->rows == 0) return BM_OK;
  const bool heads = s->num_q_heads > 0 || s->num_kv_heads > 0;
  if (!s->ids || !s->embed || !s->hidden || !s->attn_out || !s->w_attn || !s->y_attn || !s->ffn_out || !s->w_ffn ||
      !s->y_ffn || !s->gate || !s->up || !s->act || !s->positions ||
      (heads && (!s->q || !s->k || !s->v || !s->k_cache || !s->v_cache))) {
    return fail(BM_ERR_INVALID_ARGUMENT, "%s: NULL pointer", what);
  }
  const int es = dtype_size(dtype);
  const int vec = 16 / es;
  const int64_t n_ffn = s->rows * static_cast<int64_t>(s->ffn);
  const bool small = s->rows <= kFusedMaxRows && s->dim % vec == 0 && s->dim / vec <= kMaxKV * 256 &&
                     (s->head_dim / 2) % vec == 0 && s->head_dim / 2 <= ropekv::kMaxHalf &&
                     all_aligned16({s->embed, s->hidden, s->attn_out, s->w_attn, s->y_attn, s->ffn_out, s->w_ffn,
                                    s->y_ffn, s->gate, s->up, s->act}) &&
                     (!heads || all_aligned16({s->q, s->k, s->v, s->k_cache, s->v_cache}));
  if (!small) {
    // The five batched kernels, in the step's order.
    if (int st = bm_embed_gather(s->hidden, s->embed, s->ids, s->rows, s->dim, s->vocab, s->dim, dtype, d_status,
                                 stream)) {
      return st;
    }
    if (int st = bm_add_rmsnorm(s->hidden, s->attn_out, s->w_attn, s->y_attn, s->rows, s->dim, s->eps, dtype,
                                stream)) {
      return st;
    }
    if (int st = bm_rope_kv_store(s->q, s->k, s->v, s->positions, 0, s->seq_ids, s->k_cache, s->v_cache,
                                  s->rope_table, s->rope_table_len, s->theta, s->rows, s->num_q_heads,
                                  s->num_kv_heads, s->head_dim, s->max_seq, s->num_seqs, dtype, d_status, stream)) {
      return st;
    }
    if (int st = bm_add_rmsnorm(s->hidden, s->ffn_out, s->w_ffn, s->y_ffn, s->rows, s->dim, s->eps, dtype,
                                stream)) {
      return st;
    }
    return bm_swiglu(s->act, s->gate, s->up, n_ffn, dtype, stream);
  }
  if (!(s->eps >= 0.f)) return fail(BM_ERR_INVALID_ARGUMENT, "%s: eps must be >= 0", what);
  if (s->rope_table != nullptr) {
    if (s->rope_table_len <= 0 || (reinterpret_cast<uintptr_t>(s->rope_table) & 7u) != 0) {
      return fail(BM_ERR_INVALID_ARGUMENT, "%s: bad rope table", what);
    }
  } else if (!(s->theta > 0.0)) {
    return fail(BM_ERR_INVALID_ARGUMENT, "%s: theta must be > 0 without a table", what);
  }
  StepArgs a{};
  a.rows = s->rows;
  a.vocab = s->vocab;
  a.dim = s->dim;
  a.eps = s->eps;
  a.ids = s->ids;
  a.embed = s->embed;
  a.hidden = s->hidden;
  a.attn_out = s->attn_out;
  a.w_attn = s->w_attn;
  a.y_attn = s->y_attn;
  a.ffn_out = s->ffn_out;
  a.w_ffn = s->w_ffn;
  a.y_ffn = s->y_ffn;
  a.gate = s->gate;
  a.up = s->up;
  a.act = s->act;
  a.swiglu_n = n_ffn;
  a.swiglu_nvec = n_ffn / vec;
  const int64_t per_job = static_cast<int64_t>(block_threads(s->dim / vec)) * kSwigluUnroll;
  a.swiglu_jobs = std::max<int64_t>(1, (a.swiglu_nvec + per_job - 1) / per_job);
  a.status = d_status;
  ropekv::RopeArgs& r = a.rope;
  r.q = s->q;
  r.k = const_cast<void*>(s->k);
  r.v = s->v;
  r.positions = s->positions;
  r.seq_ids = s->seq_ids;
  r.k_cache = s->k_cache;
  r.v_cache = s->v_cache;
  r.table = static_cast<const float2*>(s->rope_table);
  r.table_len = s->rope_table_len;
  r.table_vec4 = s->rope_table != nullptr && aligned16(s->rope_table);
  r.theta = s->theta;
  r.rows = s->rows;
  r.hq = s->num_q_heads;
  r.hkv = s->num_kv_heads;
  r.hd = s->head_dim;
  r.half = s->head_dim / 2;
  r.max_seq = s->max_seq;
  r.num_seqs = s->num_seqs;
  r.status = d_status;
  ropekv::set_units(r, vec, ropekv::kFused);
  a.rope_jobs = heads && r.total_units > 0 ? s->rows : 0;
  cudaStream_t st = as_stream(stream);
  return dtype == BM_F32 ? launch_small<float>(a, st) : launch_small<bf16>(a, st);
}
