// Decode-attention kernels and their launchers, shared by attention_f32.cu and
// attention_bf16.cu (one translation unit per storage type, so the two sets of
// template instances compile in parallel) and by attention.cu (the C ABI; it
// instantiates nothing). See attention.cu for the design.
#pragma once

#include <algorithm>
#include <cmath>

#include "bm_common.cuh"
#include "bm_host.h"

namespace bm {
namespace attn {

constexpr int kThreads = 128;  // = positions per tile
constexpr int kWarps = kThreads / 32;
constexpr int kMaxGroup = 16;
constexpr int kMaxHeadDim = 256;

struct AttnArgs {
  void* out;              // [batch][hq][hd]
  const void* q;          // [batch][hq][hd]
  const void* k_cache;    // [num_seqs][hkv][max_seq][hd]
  const void* v_cache;
  const int32_t* seq_ids; // NULL: 0
  const int32_t* lens;    // NULL: len0 for every query
  int32_t len0;
  int64_t batch;
  int hq, hkv, hd, group, max_seq, num_seqs;
  int max_len;            // the caller's bound on every query's length (plans cover it)
  int splits, split_len;  // positions per split (a multiple of kThreads)
  float qscale;           // log2(e) * softmax scale
  float* ws;              // [batch][hkv][splits][group][hd + 2]: o..., m, l
  int32_t* status;
  // ROPE form (bm_rope_kv_decode_attention): each query's new token is rotated and
  // stored in the cache by the CTA that attends to its position, before it attends
  const void* k_new;          // [batch][hkv][hd], not yet rotated
  const void* v_new;          // [batch][hkv][hd]
  const int32_t* positions;   // [batch]: the new token's cache position
  const float2* rope_table;   // [rope_len][hd / 2] (cos, sin)
  int rope_len;
};

__device__ __forceinline__ int query_len(const AttnArgs& a, int64_t b) { return a.lens ? a.lens[b] : a.len0; }

// Returns the query's status bits (0 = valid). A length above the caller's
// max_len is flagged on every path: the split plans only cover max_len
// positions, so such a query would otherwise lose its last positions silently.
__device__ __forceinline__ int32_t check_query(const AttnArgs& a, int64_t b, int* seq, int* len) {
  *seq = a.seq_ids ? a.seq_ids[b] : 0;
  *len = query_len(a, b);
  int32_t bad = 0;
  if (*seq < 0 || *seq >= a.num_seqs) bad |= BM_DEVERR_BAD_SEQUENCE;
  if (*len <= 0 || *len > a.max_seq || *len > a.max_len) bad |= BM_DEVERR_BAD_POSITION;
  return bad;
}

// Block-wide max or sum of G values per thread (vals[g]); every thread gets the results.
// (Loops run to the compile-time GM so the register array is never indexed at run time.)
template <bool MAX, int GM>
__device__ __forceinline__ void block_reduce(float (&vals)[GM], int G, float (*scratch)[kMaxGroup]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int g = 0; g < GM; ++g) {
    if (g < G) {
      float v = vals[g];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const float o = __shfl_xor_sync(0xffffffffu, v, off);
        v = MAX ? fmaxf(v, o) : v + o;
      }
      if (lane == 0) scratch[warp][g] = v;
    }
  }
  __syncthreads();
#pragma unroll
  for (int g = 0; g < GM; ++g) {
    if (g < G) {
      float v = scratch[0][g];
#pragma unroll
      for (int w = 1; w < kWarps; ++w) v = MAX ? fmaxf(v, scratch[w][g]) : v + scratch[w][g];
      vals[g] = v;
    }
  }
  __syncthreads();
}

// A cache load: the read-only path, or (COHERENT) one served by L2, for a cache
// that the same kernel writes (the ROPE form stores the new token's rows first).
template <bool COHERENT, typename V>
__device__ __forceinline__ V ld_cache(const V* p) {
  if constexpr (COHERENT) {
    return __ldcg(p);
  } else {
    return __ldg(p);
  }
}

// Loads N consecutive elements of T (N * sizeof(T) a power of two from 2 to 32
// bytes, aligned to the smaller of that size and 16) as floats.
template <typename T, int N, bool COHERENT = false>
__device__ __forceinline__ void load_n(const T* p, float* f) {
  constexpr int kBytes = N * static_cast<int>(sizeof(T));
  static_assert(kBytes == 2 || kBytes == 4 || kBytes == 8 || kBytes == 16 || kBytes == 32, "unsupported width");
  if constexpr (kBytes == 32) {
    constexpr int kHalf = 16 / static_cast<int>(sizeof(T));
    unpack16<T>(ld_cache<COHERENT>(reinterpret_cast<const uint4*>(p)), f);
    unpack16<T>(ld_cache<COHERENT>(reinterpret_cast<const uint4*>(p + kHalf)), f + kHalf);
  } else if constexpr (kBytes == 16) {
    unpack16<T>(ld_cache<COHERENT>(reinterpret_cast<const uint4*>(p)), f);
  } else if constexpr (kBytes == 8) {
    const uint2 r = ld_cache<COHERENT>(reinterpret_cast<const uint2*>(p));
    if constexpr (sizeof(T) == 4) {
      f[0] = __uint_as_float(r.x);
      f[1] = __uint_as_float(r.y);
    } else {
      f[0] = bf16_lo(r.x);
      f[1] = bf16_hi(r.x);
      f[2] = bf16_lo(r.y);
      f[3] = bf16_hi(r.y);
    }
  } else if constexpr (kBytes == 4) {
    const uint32_t r = ld_cache<COHERENT>(reinterpret_cast<const unsigned int*>(p));
    if constexpr (sizeof(T) == 4) {
      f[0] = __uint_as_float(r);
    } else {
      f[0] = bf16_lo(r);
      f[1] = bf16_hi(r);
    }
  } else {
    f[0] = load1<T>(p);
  }
}

// GM: the group size rounded up to a power of two (register arrays are sized by
// it); DPL = ceil(head_dim / 32) dimensions per lane in the mix. CONTIG (head_dim
// = 32 * DPL, DPL a power of two): lane l owns dimensions [l*DPL, l*DPL + DPL)
// and reads them with one vector load; otherwise it owns l, l + 32, ...
//
// ROPE: the query's new token comes unrotated (q, k_new, v_new at positions[b]).
// Every CTA rotates the group's queries as it stages them; the CTA whose split
// holds the position also rotates k_new into the K cache and copies v_new into the
// V cache there, then reads the caches through L2 (its own stores included). The
// rotation and the stored values are those of bm_rope_kv_store (rope_rotate, the
// rotated q rounded to T as it would be stored), so the output is the two calls'.
template <typename T, int GM, int DPL, bool CONTIG, bool ROPE = false>
__global__ void __launch_bounds__(kThreads) attention_split_kernel(AttnArgs a) {
  grid_dependency_wait();
  constexpr int VEC = VecWidth<T>::value;
  constexpr int KCHUNKS = (32 * DPL + VEC - 1) / VEC;  // 16-byte chunks of the longest K row
  constexpr int KB = KCHUNKS < 8 ? KCHUNKS : 8;           // chunks loaded together
  extern __shared__ float smem[];
  // layout: q_s [G][hd] | p_s [G][kThreads] | red [kWarps][G][hd]
  const int G = a.group, hd = a.hd;
  float* q_s = smem;
  float* p_s = q_s + G * hd;
  float* red = p_s + G * kThreads;
  __shared__ float scratch[kWarps][kMaxGroup];
  __shared__ float m_s[kMaxGroup], l_s[kMaxGroup], alpha_s[kMaxGroup];

  const int64_t b = blockIdx.z;
  const int kvh = blockIdx.y;
  const int split = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int seq, len;
  const int32_t bad = check_query(a, b, &seq, &len);
  if (bad) {  // uniform: every thread of the CTA read the same query
    if (tid == 0 && kvh == 0 && split == 0) raise_status(a.status, bad);
    return;
  }
  const int start = split * a.split_len;
  const int end = min(len, start + a.split_len);
  float* ws = a.ws ? a.ws + (((b * a.hkv + kvh) * a.splits + split) * G) * static_cast<int64_t>(hd + 2) : nullptr;
  if (start >= end) {  // this split lies past the query's length: an empty partial
    if (ws != nullptr && tid < G) {
      ws[tid * (hd + 2) + hd] = -INFINITY;
      ws[tid * (hd + 2) + hd + 1] = 0.f;
    }
    return;
  }

  const int64_t head_base = (static_cast<int64_t>(seq) * a.hkv + kvh) * a.max_seq * hd;
  // queries of the group, pre-scaled, in shared memory
  const T* qb = static_cast<const T*>(a.q) + (b * a.hq + static_cast<int64_t>(kvh) * G) * hd;
  if constexpr (ROPE) {
    const int half = hd / 2;
    int pos = a.positions[b];
    if (pos < 0 || pos >= len || pos >= a.rope_len) {  // nothing rotated or stored, as bm_rope_kv_store skips it
      if (tid == 0 && kvh == 0 && split == 0) raise_status(a.status, BM_DEVERR_BAD_POSITION);
      pos = -1;
    }
    float2* cs = reinterpret_cast<float2*>(red);  // (cos, sin) of pos: red is free until the end
    if (pos >= 0) {
      for (int i = tid; i < half; i += kThreads) cs[i] = __ldg(a.rope_table + static_cast<int64_t>(pos) * half + i);
    }
    __syncthreads();
    for (int i = tid; i < G * hd; i += kThreads) {
      float x = load1<T>(qb + i);
      if (pos >= 0) {
        const int g = i / hd, d = i - g * hd, pr = d < half ? d : d - half;
        float o1, o2;
        rope_rotate(load1<T>(qb + g * hd + pr), load1<T>(qb + g * hd + pr + half), cs[pr], &o1, &o2);
        x = round_to<T>(d < half ? o1 : o2);
      }
      q_s[i] = x * a.qscale;
    }
    if (pos >= start && pos < end) {  // this split attends to the new position: its K and V rows go in first
      const T* kn = static_cast<const T*>(a.k_new) + (b * a.hkv + kvh) * static_cast<int64_t>(hd);
      const T* vn = static_cast<const T*>(a.v_new) + (b * a.hkv + kvh) * static_cast<int64_t>(hd);
      T* kc = const_cast<T*>(static_cast<const T*>(a.k_cache)) + head_base + static_cast<int64_t>(pos) * hd;
      T* vc = const_cast<T*>(static_cast<const T*>(a.v_cache)) + head_base + static_cast<int64_t>(pos) * hd;
      for (int d = tid; d < hd; d += kThreads) {
        const int pr = d < half ? d : d - half;
        float o1, o2;
        rope_rotate(load1<T>(kn + pr), load1<T>(kn + pr + half), cs[pr], &o1, &o2);
        store1<T>(kc + d, d < half ? o1 : o2);
        vc[d] = vn[d];
      }
    }
  } else {
    for (int i = tid; i < G * hd; i += kThreads) q_s[i] = load1<T>(qb + i) * a.qscale;
  }
  if (tid < G) {
    m_s[tid] = -INFINITY;
    l_s[tid] = 0.f;
  }
  const T* kbase = static_cast<const T*>(a.k_cache) + head_base;
  const T* vbase = static_cast<const T*>(a.v_cache) + head_base;
  auto dim_of = [&](int i) { return CONTIG ? lane * DPL + i : lane + 32 * i; };

  float acc[GM][DPL];
#pragma unroll
  for (int g = 0; g < GM; ++g)
#pragma unroll
    for (int i = 0; i < DPL; ++i) acc[g][i] = 0.f;
  __syncthreads();

  for (int tile = start; tile < end; tile += kThreads) {
    const int p = tile + tid;
    float s[GM];
#pragma unroll
    for (int g = 0; g < GM; ++g) s[g] = 0.f;
    if (p < end) {
      // the K row in batches of KB 16-byte chunks (compile-time counts), each
      // batch's loads in flight together
      const T* krow = kbase + static_cast<int64_t>(p) * hd;
#pragma unroll
      for (int cb = 0; cb < KCHUNKS; cb += KB) {
        uint4 kr[KB];
#pragma unroll
        for (int c = 0; c < KB; ++c) {
          if ((cb + c) * VEC < hd) kr[c] = ld_cache<ROPE>(reinterpret_cast<const uint4*>(krow + (cb + c) * VEC));
        }
#pragma unroll
        for (int c = 0; c < KB; ++c) {
          if ((cb + c) * VEC < hd) {
            float k[VEC];
            unpack16<T>(kr[c], k);
#pragma unroll
            for (int g = 0; g < GM; ++g) {
              if (g < G) {
                float dot = s[g];
#pragma unroll
                for (int e = 0; e < VEC; ++e) dot = fmaf(q_s[g * hd + (cb + c) * VEC + e], k[e], dot);
                s[g] = dot;
              }
            }
          }
        }
      }
    } else {
#pragma unroll
      for (int g = 0; g < GM; ++g) s[g] = -INFINITY;
    }
    // online softmax (base 2): tile max, rescale factors, probabilities, tile sum
    float t[GM];
#pragma unroll
    for (int g = 0; g < GM; ++g) t[g] = s[g];
    block_reduce<true, GM>(t, G, scratch);
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      if (g < G) {
        const float m_new = fmaxf(m_s[g], t[g]);
        const float pr = (p < end) ? exp2f(s[g] - m_new) : 0.f;
        p_s[g * kThreads + tid] = pr;
        t[g] = pr;
        s[g] = m_new;  // reuse: the new running max
      }
    }
    block_reduce<false, GM>(t, G, scratch);  // tile sums; its barriers also publish p_s
    float m_mine = 0.f, sum_mine = 0.f;  // thread g < G updates query g's running state
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      if (g == tid) {
        m_mine = s[g];
        sum_mine = t[g];
      }
    }
    if (tid < G) {
      const float alpha = exp2f(m_s[tid] - m_mine);
      alpha_s[tid] = alpha;
      l_s[tid] = l_s[tid] * alpha + sum_mine;
      m_s[tid] = m_mine;
    }
    __syncthreads();
    // mix: rescale, then accumulate p * V over this warp's positions of the tile,
    // two positions' V loads in flight at a time
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      if (g < G) {
        const float al = alpha_s[g];
#pragma unroll
        for (int i = 0; i < DPL; ++i) acc[g][i] *= al;
      }
    }
    const int tile_end = min(end - tile, kThreads);
    for (int j0 = warp; j0 < tile_end; j0 += 2 * kWarps) {
      float v[2][DPL];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int j = j0 + u * kWarps;
        const T* vrow = vbase + static_cast<int64_t>(tile + min(j, tile_end - 1)) * hd;
        if constexpr (CONTIG) {
          load_n<T, DPL, ROPE>(vrow + lane * DPL, v[u]);
        } else {
#pragma unroll
          for (int i = 0; i < DPL; ++i) {
            const int d = lane + 32 * i;
            v[u][i] = d < hd ? load1<T>(vrow + d) : 0.f;
          }
        }
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int j = j0 + u * kWarps;
        if (j < tile_end) {
#pragma unroll
          for (int g = 0; g < GM; ++g) {
            if (g < G) {
              const float pr = p_s[g * kThreads + j];
#pragma unroll
              for (int i = 0; i < DPL; ++i) acc[g][i] = fmaf(pr, v[u][i], acc[g][i]);
            }
          }
        }
      }
    }
    __syncthreads();  // p_s, alpha_s are rewritten by the next tile
  }

  // sum the warps' accumulators
#pragma unroll
  for (int g = 0; g < GM; ++g) {
    if (g < G) {
#pragma unroll
      for (int i = 0; i < DPL; ++i) {
        const int d = dim_of(i);
        if (d < hd) red[(warp * G + g) * hd + d] = acc[g][i];
      }
    }
  }
  __syncthreads();
  for (int i = tid; i < G * hd; i += kThreads) {
    float o = red[i];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) o += red[w * G * hd + i];
    const int g = i / hd, d = i - g * hd;
    if (ws == nullptr) {
      T* out = static_cast<T*>(a.out) + (b * a.hq + static_cast<int64_t>(kvh) * G + g) * hd;
      store1<T>(out + d, o / l_s[g]);
    } else {
      ws[g * (hd + 2) + d] = o;
      if (d == 0) {
        ws[g * (hd + 2) + hd] = m_s[g];
        ws[g * (hd + 2) + hd + 1] = l_s[g];
      }
    }
  }
}

// One CTA of kCombineThreads per (query, q head): merges the splits' (max, sum,
// output) partials. Every load that needs no other result is issued at once:
// thread s reads split s's maximum and sum, thread d the first kCombineChunk
// splits' outputs of dimension d, so the partials cost one L2 round trip and two
// barriers (the maximum, then the weights exp2(max_s - max) and the weighted sum).
// The sums and products run in the same order as a split-by-split merge, so the
// result does not depend on how the loads were grouped.
constexpr int kCombineThreads = 128;
constexpr int kCombineChunk = 16;  // output loads in flight per thread

// Block-wide max or sum of v (NW warps); every thread gets the result.
template <int NW>
__device__ __forceinline__ float combine_block_reduce(float v, bool is_max, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float o = __shfl_xor_sync(0xffffffffu, v, off);
    v = is_max ? fmaxf(v, o) : v + o;
  }
  if (lane == 0) red[warp] = v;
  __syncthreads();
  v = red[0];
#pragma unroll
  for (int w = 1; w < NW; ++w) v = is_max ? fmaxf(v, red[w]) : v + red[w];
  __syncthreads();
  return v;
}

template <typename T>
__global__ void __launch_bounds__(kCombineThreads) attention_combine_kernel(AttnArgs a) {
  grid_dependency_wait();
  extern __shared__ float stats[];  // [splits] maxima, turned into weights; [splits] sums
  __shared__ float red[2][kCombineThreads / 32];
  const int64_t b = blockIdx.y;
  const int h = blockIdx.x;
  int seq, len;
  if (check_query(a, b, &seq, &len)) return;  // reported by the split kernel
  const int kvh = h / a.group, g = h - kvh * a.group;
  const int hd = a.hd, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, S = a.splits;
  const float* base = a.ws + ((b * a.hkv + kvh) * S * a.group + g) * static_cast<int64_t>(hd + 2);
  const int64_t split_stride = static_cast<int64_t>(a.group) * (hd + 2);
  // An empty split writes only its maximum (-inf) and sum: its output slots hold
  // whatever the workspace held before. They are loaded like the others (the
  // addresses are inside the workspace) but never weighted, not even by 0.
  float v[kCombineChunk];
#pragma unroll
  for (int j = 0; j < kCombineChunk; ++j) v[j] = (j < S && tid < hd) ? base[j * split_stride + tid] : 0.f;
  float m = -INFINITY;
  for (int s = tid; s < S; s += kCombineThreads) {
    const float ms = base[s * split_stride + hd], ls = base[s * split_stride + hd + 1];
    stats[s] = ms;
    stats[S + s] = ls;
    m = fmaxf(m, ms);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  if (lane == 0) red[0][warp] = m;
  __syncthreads();
  m = red[0][0];
#pragma unroll
  for (int w = 1; w < kCombineThreads / 32; ++w) m = fmaxf(m, red[0][w]);  // finite: split 0 is never empty
  float l = 0.f;
  for (int s = tid; s < S; s += kCombineThreads) {  // each thread its own splits: no barrier needed
    const float ms = stats[s];
    const float w = ms == -INFINITY ? 0.f : exp2f(ms - m);
    stats[s] = w;
    l += stats[S + s] * w;
  }
  l = warp_sum(l);
  if (lane == 0) red[1][warp] = l;
  __syncthreads();  // also publishes the weights
  l = red[1][0];
#pragma unroll
  for (int w = 1; w < kCombineThreads / 32; ++w) l += red[1][w];
  T* out = static_cast<T*>(a.out) + (b * a.hq + h) * hd;
  for (int d = tid; d < hd; d += kCombineThreads) {
    float o = 0.f;
    for (int s0 = 0; s0 < S; s0 += kCombineChunk) {
      if (s0 > 0 || d != tid) {
#pragma unroll
        for (int j = 0; j < kCombineChunk; ++j) v[j] = s0 + j < S ? base[(s0 + j) * split_stride + d] : 0.f;
      }
#pragma unroll
      for (int j = 0; j < kCombineChunk; ++j) {
        if (s0 + j < S) {
          const float w = stats[s0 + j];
          if (w != 0.f) o = fmaf(v[j], w, o);
        }
      }
    }
    store1<T>(out + d, o / l);
  }
}

// Launches the combine step for a split plan.
template <typename T>
int launch_combine(const AttnArgs& a, cudaStream_t stream) {
  if (const int launch_status = launch_kernel("attention_combine_kernel", attention_combine_kernel<T>,
                                              dim3(dim3(a.hq, static_cast<unsigned>(a.batch))), dim3(kCombineThreads),
                                              2 * static_cast<size_t>(a.splits) * sizeof(float), stream, nullptr, a)) {
    return launch_status;
  }
  return check_launch("bm_decode_attention (combine)");
}

// Splits for `pairs` (query, kv head) pairs over at most max_len positions:
// enough CTAs to fill the GPU several times, each split a whole number of tiles.

template <typename T, int GM, bool ROPE>
int launch_group(const AttnArgs& a, size_t smem, cudaStream_t stream) {
  const dim3 grid(a.splits, a.hkv, static_cast<unsigned>(a.batch));
  auto go = [&](auto kernel) {
    if (smem > 48 * 1024) {
      if (int st = allow_dynamic_smem(reinterpret_cast<const void*>(kernel), static_cast<int>(smem), "bm_decode_attention")) {
        return st;
      }
    }
    if (const int launch_status =
            launch_kernel("bm_decode_attention", kernel, dim3(grid), dim3(kThreads), smem, stream, nullptr, a)) {
      return launch_status;
    }
    return check_launch("bm_decode_attention");
  };
  const int dpl = (a.hd + 31) / 32;
  if (a.hd % 32 == 0 && (dpl & (dpl - 1)) == 0) {  // head_dim 32, 64, 128, 256: contiguous lanes
    switch (dpl) {
      case 1: return go(attention_split_kernel<T, GM, 1, true, ROPE>);
      case 2: return go(attention_split_kernel<T, GM, 2, true, ROPE>);
      case 4: return go(attention_split_kernel<T, GM, 4, true, ROPE>);
      default: return go(attention_split_kernel<T, GM, 8, true, ROPE>);
    }
  }
  // any other head_dim: strided lanes, the smallest power-of-two count covering it
  if (dpl <= 1) return go(attention_split_kernel<T, GM, 1, false, ROPE>);
  if (dpl <= 2) return go(attention_split_kernel<T, GM, 2, false, ROPE>);
  if (dpl <= 4) return go(attention_split_kernel<T, GM, 4, false, ROPE>);
  return go(attention_split_kernel<T, GM, 8, false, ROPE>);
}

template <typename T, bool ROPE = false>
int launch(AttnArgs a, cudaStream_t stream) {
  const size_t smem = sizeof(float) * (static_cast<size_t>(a.group) * a.hd + a.group * kThreads +
                                       static_cast<size_t>(kWarps) * a.group * a.hd);
  int st;
  if (a.group <= 1) {
    st = launch_group<T, 1, ROPE>(a, smem, stream);
  } else if (a.group <= 2) {
    st = launch_group<T, 2, ROPE>(a, smem, stream);
  } else if (a.group <= 4) {
    st = launch_group<T, 4, ROPE>(a, smem, stream);
  } else if (a.group <= 8) {
    st = launch_group<T, 8, ROPE>(a, smem, stream);
  } else {
    st = launch_group<T, 16, ROPE>(a, smem, stream);
  }
  if (st != BM_OK || a.splits == 1) return st;
  return launch_combine<T>(a, stream);
}


// One instance per storage type, each in its own translation unit; the _rope
// forms are the ROPE kernels (the new token rotated and stored in the same launch).
int launch_f32(const AttnArgs& a, cudaStream_t stream);
int launch_bf16(const AttnArgs& a, cudaStream_t stream);
int launch_f32_rope(const AttnArgs& a, cudaStream_t stream);
int launch_bf16_rope(const AttnArgs& a, cudaStream_t stream);

// The tensor-core kernel (attention_tc.cu): bf16 caches with head_dim 128.
bool tc_eligible(const AttnArgs& a, bm_dtype_t dtype);
int launch_tc(const AttnArgs& a, cudaStream_t stream);

// Its balanced persistent form (attention_tc_balanced.cu): one CTA per SM over an
// equal share of all (query, kv head) tiles, for batches of at most
// kBalancedMaxBatch queries and at least kBalancedMinPairs (query, kv head)
// pairs (fewer pairs are split evenly by the per-pair grid already, which starts
// faster); workspace: balanced_workspace_bytes(group, ctas).
constexpr int kBalancedMaxBatch = 2048;
#ifndef BM_ATTN_BALANCED_MIN_PAIRS
#define BM_ATTN_BALANCED_MIN_PAIRS 32
#endif
constexpr int kBalancedMinPairs = BM_ATTN_BALANCED_MIN_PAIRS;
bool balanced_eligible(const AttnArgs& a, bm_dtype_t dtype);
size_t balanced_workspace_bytes(int group, int ctas);
int launch_tc_balanced(AttnArgs a, int ctas, cudaStream_t stream);

// The TMA-fed CUDA-core kernel (attention_f32_tma.cu): fp32 caches with head_dim 128.
bool f32_tma_eligible(const AttnArgs& a, bm_dtype_t dtype);
int launch_f32_tma(const AttnArgs& a, cudaStream_t stream);

}  // namespace attn
}  // namespace bm
