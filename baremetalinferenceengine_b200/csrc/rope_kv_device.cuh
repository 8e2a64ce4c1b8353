// Device pieces of the RoPE + K/V-cache kernels (rope_kv.cu), shared with the
// fused small-batch layer step (layer_step.cu): the argument block, the unit
// decomposition of one token, and one token's work done by one thread block.
#pragma once

#include "bm_common.cuh"

namespace bm {
namespace ropekv {

constexpr int kMaxHalf = 512;  // head_dim <= 1024
constexpr int kUPT = 4;        // units whose loads a thread issues up front

enum Mode { kFused = 0, kRope = 1, kStore = 2 };

struct RopeArgs {
  void* q;                    // [rows][hq][hd]
  void* k;                    // [rows][hkv][hd]
  const void* v;              // [rows][hkv][hd] (kFused: v; kStore: src)
  const int32_t* positions;   // NULL: pos0 + row
  const int32_t* seq_ids;     // NULL: 0
  void* k_cache;              // [num_seqs][hkv][max_seq][hd]
  void* v_cache;              // kStore: the destination cache
  const float2* table;        // [table_len][half] or NULL
  double theta;
  int64_t rows;
  int32_t pos0;
  int32_t table_len;
  int hq, hkv, hd, half, max_seq, num_seqs;
  int upv;                    // pair units per head (half / VEC)
  int cpv;                    // copy units per head (hd / VEC)
  int q_units, k_units, total_units;
  bool table_vec4;            // table 16-byte aligned: (cos, sin) pairs read two at a time
  int32_t* status;
};

// VEC consecutive elements of T, held between load and store.
template <typename T, int VEC>
struct Chunk {
  static_assert(VEC * sizeof(T) == 16, "vector chunks are 16 bytes");
  uint4 raw;
  __device__ __forceinline__ void load(const T* p) { raw = ld_stream(p); }
  __device__ __forceinline__ void store(T* p) const { st_plain(p, raw); }
  __device__ __forceinline__ void get(float* f) const { unpack16<T>(raw, f); }
  __device__ __forceinline__ void set(const float* f) { raw = pack16<T>(f); }
};
template <typename T>
struct Chunk<T, 1> {
  float x;
  __device__ __forceinline__ void load(const T* p) { x = load1<T>(p); }
  __device__ __forceinline__ void store(T* p) const { store1<T>(p, x); }
  __device__ __forceinline__ void get(float* f) const { f[0] = x; }
  __device__ __forceinline__ void set(const float* f) { x = f[0]; }
};

// (cos, sin) of pos / theta^(2i/hd) in fp64, rounded once to fp32: the angle of
// the reference's CPU check loop (tests/kernel_tests.cu:180). Kept out of line:
// it is the cold path (no table), and inlined fp64 pow/sincos would swell the
// hot loops' register counts.
static __device__ __noinline__ float2 angle_cos_sin(int pos, int i, double theta, int hd) {
  const double angle = static_cast<double>(pos) / pow(theta, 2.0 * i / hd);
  double s, c;
  sincos(angle, &s, &c);
  return make_float2(static_cast<float>(c), static_cast<float>(s));
}

// Where unit u of a token lives: kind 0 = Q pair, 1 = K pair, 2 = V copy;
// head h and chunk c within the head.
struct Unit {
  int kind, h, c;
};

__device__ __forceinline__ Unit decode(const RopeArgs& a, int u) {
  Unit r;
  if (u < a.q_units) {
    r.kind = 0;
    r.h = u / a.upv;
    r.c = u - r.h * a.upv;
  } else if (u < a.q_units + a.k_units) {
    u -= a.q_units;
    r.kind = 1;
    r.h = u / a.upv;
    r.c = u - r.h * a.upv;
  } else {
    u -= a.q_units + a.k_units;
    r.kind = 2;
    r.h = u / a.cpv;
    r.c = u - r.h * a.cpv;
  }
  return r;
}

template <typename T, int VEC, int MODE>
__device__ __forceinline__ void load_unit(const RopeArgs& a, const Unit& u, int64_t row, Chunk<T, VEC>& c1,
                                          Chunk<T, VEC>& c2) {
  if (u.kind == 0) {
    const T* base = static_cast<const T*>(a.q) + (row * a.hq + u.h) * a.hd + u.c * VEC;
    c1.load(base);
    c2.load(base + a.half);
  } else if (u.kind == 1) {
    const T* base = static_cast<const T*>(a.k) + (row * a.hkv + u.h) * a.hd + u.c * VEC;
    c1.load(base);
    c2.load(base + a.half);
  } else {
    const T* base = static_cast<const T*>(a.v) + (row * a.hkv + u.h) * a.hd + u.c * VEC;
    c1.load(base);
  }
}

template <typename T, int VEC, int MODE>
__device__ __forceinline__ void finish_unit(const RopeArgs& a, const Unit& u, int64_t row, int64_t cache_base,
                                            int64_t cache_head_stride, const float2* cs, Chunk<T, VEC>& c1,
                                            Chunk<T, VEC>& c2) {
  if (u.kind == 2) {
    // V (kFused) or src (kStore): plain copy into the cache.
    T* dst = static_cast<T*>(a.v_cache) + cache_base + u.h * cache_head_stride + u.c * VEC;
    c1.store(dst);
    return;
  }
  float x1[VEC], x2[VEC];
  c1.get(x1);
  c2.get(x2);
#pragma unroll
  for (int e = 0; e < VEC; ++e) {
    const float2 t = cs[u.c * VEC + e];  // (cos, sin)
    rope_rotate(x1[e], x2[e], t, &x1[e], &x2[e]);
  }
  c1.set(x1);
  c2.set(x2);
  T* dst;
  if (u.kind == 0) {
    dst = static_cast<T*>(a.q) + (row * a.hq + u.h) * a.hd + u.c * VEC;
  } else if (MODE == kFused) {
    dst = static_cast<T*>(a.k_cache) + cache_base + u.h * cache_head_stride + u.c * VEC;
  } else {
    dst = static_cast<T*>(a.k) + (row * a.hkv + u.h) * a.hd + u.c * VEC;
  }
  c1.store(dst);
  c2.store(dst + a.half);
}

// prefetch_l2 of one token's position, sequence id and q / k / v rows: the lines
// its first loads will touch (idx of count participants).
template <typename T, int MODE>
__device__ __forceinline__ void prefetch_token(const RopeArgs& a, int64_t row, int idx, int count) {
  if (row >= a.rows) return;
  if (idx == 0) {
    if (a.positions) prefetch_l2(a.positions + row);
    if (a.seq_ids) prefetch_l2(a.seq_ids + row);
  }
  const int64_t es = sizeof(T);
  if (MODE != kStore) {
    prefetch_l2_range(static_cast<const T*>(a.q) + row * a.hq * a.hd, a.hq * a.hd * es, idx, count);
    prefetch_l2_range(static_cast<const T*>(a.k) + row * a.hkv * a.hd, a.hkv * a.hd * es, idx, count);
  }
  if (MODE != kRope) {
    prefetch_l2_range(static_cast<const T*>(a.v) + row * a.hkv * a.hd, a.hkv * a.hd * es, idx, count);
  }
}

// Unit counts of one token for chunks of v_used elements (host side): pair
// units per head, copy units per head, and the token's Q, K and total units.
inline void set_units(RopeArgs& a, int v_used, int mode) {
  a.upv = a.half / v_used;
  a.cpv = a.hd / v_used;
  if (mode == kStore) {
    a.q_units = 0;
    a.k_units = 0;
    a.total_units = a.hkv * a.cpv;
  } else {
    a.q_units = a.hq * a.upv;
    a.k_units = a.hkv * a.upv;
    a.total_units = a.q_units + a.k_units + (mode == kFused ? a.hkv * a.cpv : 0);
  }
}

// One token's RoPE and K/V-cache work by the whole block (tid of nthreads
// threads). cs: kMaxHalf (cos, sin) pairs of shared memory, staged here. Every
// thread of the block must call it for the same row: it holds block barriers.
template <typename T, int VEC, int MODE>
__device__ __forceinline__ void rope_kv_token(const RopeArgs& a, int64_t row, int tid, int nthreads, float2* cs) {
  const int64_t cache_head_stride = static_cast<int64_t>(a.max_seq) * a.hd;
  // This thread's first UPT units' loads go out with the position's, before the
  // table barrier (a row found bad below discards them).
  Chunk<T, VEC> c1[kUPT], c2[kUPT];
#pragma unroll
  for (int j = 0; j < kUPT; ++j) {
    const int u = tid + j * nthreads;
    if (u < a.total_units) load_unit<T, VEC, MODE>(a, decode(a, u), row, c1[j], c2[j]);
  }
  const int32_t pos = a.positions ? a.positions[row] : static_cast<int32_t>(a.pos0 + row);
  const int32_t seq = a.seq_ids ? a.seq_ids[row] : 0;
  int32_t bad = 0;
  if (pos < 0) bad |= BM_DEVERR_BAD_POSITION;
  if (MODE != kRope) {
    if (pos >= a.max_seq) bad |= BM_DEVERR_BAD_POSITION;
    if (seq < 0 || seq >= a.num_seqs) bad |= BM_DEVERR_BAD_SEQUENCE;
  }
  if (MODE != kStore && a.table != nullptr && pos >= a.table_len) bad |= BM_DEVERR_BAD_POSITION;
  if (bad) {  // uniform across the block: every thread read the same row
    if (tid == 0) raise_status(a.status, bad);
    return;
  }
  const int64_t cache_base =
      MODE == kRope ? 0 : (static_cast<int64_t>(seq) * a.hkv * a.max_seq + pos) * a.hd;

  if (MODE != kStore) {
    for (int i = tid; i < a.half; i += nthreads) {
      float2 t;
      if (a.table != nullptr) {
        t = __ldg(a.table + static_cast<int64_t>(pos) * a.half + i);
      } else {
        t = angle_cos_sin(pos, i, a.theta, a.hd);
      }
      cs[i] = t;
    }
    __syncthreads();
  }

#pragma unroll
  for (int j = 0; j < kUPT; ++j) {
    const int u = tid + j * nthreads;
    if (u < a.total_units) {
      finish_unit<T, VEC, MODE>(a, decode(a, u), row, cache_base, cache_head_stride, cs, c1[j], c2[j]);
    }
  }
  // Units beyond the first UPT per thread (very wide tokens).
  for (int u = tid + kUPT * nthreads; u < a.total_units; u += nthreads) {
    Chunk<T, VEC> d1, d2;
    const Unit un = decode(a, u);
    load_unit<T, VEC, MODE>(a, un, row, d1, d2);
    finish_unit<T, VEC, MODE>(a, un, row, cache_base, cache_head_stride, cs, d1, d2);
  }
  if (MODE != kStore) __syncthreads();  // cs is restaged for the next token
}

}  // namespace ropekv
}  // namespace bm
