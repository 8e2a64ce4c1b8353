// Decode attention for fp32 caches with head_dim 128: TMA-fed, CUDA-core math.
// Same contract and results as the other attention kernels (reference semantics:
// src/kernels.cu:225-264, batched and GQA as bm_decode_attention documents),
// fp32 throughout so that it meets the fp32 tolerance.
//
// One CTA per (query, kv head, split). Warp 0 streams the split's K and V rows
// with TMA, 64 positions a tile, each row as four 128-byte-swizzled boxes of 32
// floats, through a 3-stage ring (64 KB a stage), so that every SM keeps far more
// bytes in flight than per-thread loads could. Two groups of four warps compute
// from shared memory, group h taking tiles h, h + 2, ... with its own running
// softmax state (one group's barrier waits overlap the other's arithmetic); the
// two states merge at the end like two splits. In each group:
//   scores  two threads per position, 64 dimensions each (16-byte reads that the
//           swizzle spreads over all banks), q from shared memory, one shuffle to
//           join the halves;
//   softmax tile maxima by warp shuffles and one reducing named barrier (which
//           also makes the abort decision uniform), base-2 online update;
//   mix     lane l owns dimensions 4l..4l+3, warp w positions w, w+4, ...;
//           positions past the query's length are never read.
// The warps' accumulators are summed through shared memory at the end.
// Every mbarrier wait is bounded in time (BM_DEVERR_TIMEOUT past the limit).
#include <cuda.h>

#include "attention_kernels.cuh"
#include "bm_tc.cuh"
#include "bm_tma.h"

namespace bm {
namespace attn {

using namespace bm::tc;

namespace {

constexpr int kFTile = 64;                 // positions per tile
constexpr int kFHd = 128;
constexpr int kFStages = 3;
constexpr int kFGroupThreads = 128;        // one compute group: four warps
constexpr int kFCompute = 2 * kFGroupThreads;  // compute threads (warps 1-8)
constexpr int kFThreads = 32 + kFCompute;
constexpr int kFBoxBytes = kFTile * 128;   // 64 rows x 32 floats: 8 KB
constexpr int kFHalfBytes = 4 * kFBoxBytes;  // K or V of a tile: 32 KB
constexpr int kFStageBytes = 2 * kFHalfBytes;
constexpr int kQStride = kFHd + 4;         // q row in shared memory, the upper half 4 floats further on
constexpr int kOffQ = kFStages * kFStageBytes;
constexpr int kOffP = kOffQ + kMaxGroup * kQStride * 4;
constexpr int kOffW = kOffP + 2 * kMaxGroup * kFTile * 4;  // per group: [4][16] tile maxima
constexpr int kOffM = kOffW + 2 * 4 * kMaxGroup * 4;       // per group: [16] final running maxima
constexpr int kOffL = kOffM + 2 * kMaxGroup * 4;           // per group: [4][16] row sums
constexpr int kOffBar = kOffL + 2 * 4 * kMaxGroup * 4;
constexpr int kFSmemBytes = kOffBar + (2 * kFStages + 1) * 8 + 8 + 1024;
constexpr uint64_t kFWaitNs = 2000000000ull;
constexpr uint64_t kFDrainNs = 200000000ull;

// Byte offset of the 16-byte chunk holding dims [4c, 4c+4) of row r in a tile:
// box c / 8, chunk c % 8 of the row's 128 bytes, XOR-swizzled by r % 8.
__device__ __forceinline__ uint32_t chunk_offset(int r, int c) {
  return static_cast<uint32_t>((c >> 3) * kFBoxBytes + r * 128 + ((((c & 7) ^ (r & 7))) << 4));
}

// The four warps of compute group h meet at named barrier 1 + h; the result is
// true when any of them saw `flag` set, the same for all.
__device__ __forceinline__ bool group_sync_any(int h, bool flag) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %2, 0;\n\t"
      "bar.red.or.pred p, %1, 128, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(1 + h), "r"(static_cast<uint32_t>(flag))
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void group_sync(int h) { asm volatile("bar.sync %0, 128;" ::"r"(1 + h) : "memory"); }

template <int GM>
__global__ void __launch_bounds__(kFThreads, 1)
    attention_f32_tma_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                             const AttnArgs a) {
  grid_dependency_wait();
  const int64_t b = blockIdx.z;
  const int kvh = blockIdx.y;
  const int split = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int seq, len;
  const int32_t bad = check_query(a, b, &seq, &len);
  if (bad) {
    if (tid == 0 && kvh == 0 && split == 0) raise_status(a.status, bad);
    return;
  }
  const int G = a.group;
  const int start = split * a.split_len;
  const int end = min(len, start + a.split_len);
  float* ws = a.ws ? a.ws + (((b * a.hkv + kvh) * a.splits + split) * G) * static_cast<int64_t>(kFHd + 2) : nullptr;
  if (start >= end) {
    if (ws != nullptr && tid < G) {
      ws[tid * (kFHd + 2) + kFHd] = -INFINITY;
      ws[tid * (kFHd + 2) + kFHd + 1] = 0.f;
    }
    return;
  }
  const int n_tiles = (end - start + kFTile - 1) / kFTile;
  const int row0 = (seq * a.hkv + kvh) * a.max_seq + start;

  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                         ~static_cast<uintptr_t>(1023));
  float* q_s = reinterpret_cast<float*>(smem + kOffQ);
  float* p_s = reinterpret_cast<float*>(smem + kOffP);
  float* wm_all = reinterpret_cast<float*>(smem + kOffW);
  float* mfin = reinterpret_cast<float*>(smem + kOffM);
  float* lsum = reinterpret_cast<float*>(smem + kOffL);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* empty = full + kFStages;
  uint64_t* spare = empty + kFStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(spare + 1);

  if (tid == 0) {
    for (int s = 0; s < kFStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kFGroupThreads);  // one group consumes a tile
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();  // barriers exist: the first copies start while the queries are staged
  if (warp >= 1) {  // the group's queries, each row's upper half 4 floats further on (no bank clash)
    const float* qb = static_cast<const float*>(a.q) + (b * a.hq + static_cast<int64_t>(kvh) * G) * kFHd;
    for (int i = tid - 32; i < G * kFHd; i += kFCompute) {
      const int g = i / kFHd, d = i - g * kFHd;
      q_s[g * kQStride + d + (d >= 64 ? 4 : 0)] = __ldg(qb + i);
    }
    asm volatile("bar.sync 3, 256;" ::: "memory");  // every compute thread reads all of q_s
  }

  float m_run[GM], l_part[GM], acc[GM][4];  // compute threads: running max, sum share, accumulator
  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      uint32_t last_parity[kFStages];
      bool filled[kFStages];
      for (int s = 0; s < kFStages; ++s) filled[s] = false;
      for (int i = 0; i < n_tiles; ++i) {
        const int s = i % kFStages;
        const uint32_t par = static_cast<uint32_t>((i / kFStages) & 1);
        if (!wait_phase(&empty[s], par ^ 1u, abort_flag, a.status, kFWaitNs, true)) break;
        unsigned char* st = smem + s * kFStageBytes;
        mbar_expect_tx(&full[s], kFStageBytes);
        const int y = row0 + i * kFTile;
#pragma unroll
        for (int bx = 0; bx < 4; ++bx) {
          tma_load_2d(st + bx * kFBoxBytes, &tk, &full[s], bx * 32, y);
          tma_load_2d(st + kFHalfBytes + bx * kFBoxBytes, &tv, &full[s], bx * 32, y);
        }
        filled[s] = true;
        last_parity[s] = par;
      }
      for (int s = 0; s < kFStages; ++s) {  // no copy may still land once the CTA reuses stage 0
        if (filled[s]) wait_phase(&full[s], last_parity[s], abort_flag, a.status, kFDrainNs, false);
      }
    }
  } else {
    // ---------------- compute (warps 1-8: two groups of four) ----------------
    const int grp = (warp - 1) >> 2, cw = (warp - 1) & 3, ct = (tid - 32) & (kFGroupThreads - 1);
    const int pos = ct >> 1, half = ct & 1;  // scores: position pos, dims [64 half, 64 half + 64)
    const float* qh = q_s + half * (64 + 4);
    float* wm = wm_all + grp * 4 * kMaxGroup;
    float* p_g = p_s + grp * kMaxGroup * kFTile;
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      m_run[g] = -INFINITY;
      l_part[g] = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[g][e] = 0.f;
    }
    for (int i = grp; i < n_tiles; i += 2) {
      const int s = i % kFStages;
      int ok = 1;
      if (lane == 0) {
        ok = wait_phase(&full[s], static_cast<uint32_t>((i / kFStages) & 1), abort_flag, a.status, kFWaitNs, true);
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      const unsigned char* kt = smem + s * kFStageBytes;
      const unsigned char* vt = kt + kFHalfBytes;
      const int tile_start = start + i * kFTile;
      const int tile_valid = min(end - tile_start, kFTile);
      // scores
      float sc[GM];
#pragma unroll
      for (int g = 0; g < GM; ++g) sc[g] = 0.f;
      if (ok) {
#pragma unroll 4
        for (int c = 0; c < 16; ++c) {
          const float4 kv = *reinterpret_cast<const float4*>(kt + chunk_offset(pos, half * 16 + c));
#pragma unroll
          for (int g = 0; g < GM; ++g) {
            const float4 qv = *reinterpret_cast<const float4*>(qh + g * kQStride + c * 4);
            float d = sc[g];
            d = fmaf(qv.x, kv.x, d);
            d = fmaf(qv.y, kv.y, d);
            d = fmaf(qv.z, kv.z, d);
            d = fmaf(qv.w, kv.w, d);
            sc[g] = d;
          }
        }
      }
      const bool valid = pos < tile_valid;
#pragma unroll
      for (int g = 0; g < GM; ++g) {
        const float full_dot = sc[g] + __shfl_xor_sync(0xffffffffu, sc[g], 1);
        sc[g] = (valid && g < G) ? full_dot * a.qscale : -INFINITY;
        float v = sc[g];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
        if (lane == 0) wm[cw * kMaxGroup + g] = v;
      }
      if (group_sync_any(grp, *abort_flag != 0)) break;
#pragma unroll
      for (int g = 0; g < GM; ++g) {
        if (g < G) {
          const float tmax =
              fmaxf(fmaxf(wm[g], wm[kMaxGroup + g]), fmaxf(wm[2 * kMaxGroup + g], wm[3 * kMaxGroup + g]));
          const float m_new = fmaxf(m_run[g], tmax);  // finite: every tile holds a valid position
          const float alpha = exp2f(m_run[g] - m_new);
          m_run[g] = m_new;
          const float p = valid ? exp2f(sc[g] - m_new) : 0.f;
          l_part[g] = l_part[g] * alpha + (half == 0 ? p : 0.f);
          if (half == 0) p_g[g * kFTile + pos] = p;
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[g][e] *= alpha;
        }
      }
      group_sync(grp);  // P of this tile is written
      // mix: lane owns dims 4 lane .. 4 lane + 3; rows past the length are not read
      for (int j = cw; j < tile_valid; j += 4) {
        const float4 vv = *reinterpret_cast<const float4*>(vt + chunk_offset(j, lane));
#pragma unroll
        for (int g = 0; g < GM; ++g) {
          if (g < G) {
            const float p = p_g[g * kFTile + j];
            acc[g][0] = fmaf(p, vv.x, acc[g][0]);
            acc[g][1] = fmaf(p, vv.y, acc[g][1]);
            acc[g][2] = fmaf(p, vv.z, acc[g][2]);
            acc[g][3] = fmaf(p, vv.w, acc[g][3]);
          }
        }
      }
      mbar_arrive(&empty[s]);  // this thread is done with the stage
      group_sync(grp);  // P and the maxima may be rewritten by the group's next tile
    }
    // row sums (each half-0 thread holds its positions' share) and the running maxima
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      const float v = warp_sum(l_part[g]);
      if (lane == 0) lsum[(grp * 4 + cw) * kMaxGroup + g] = v;
    }
    if (ct == 0) {
#pragma unroll
      for (int g = 0; g < GM; ++g) mfin[grp * kMaxGroup + g] = m_run[g];  // the same in every thread of the group
    }
  }
  __syncthreads();  // the producer has drained its copies: stage 0 is free for the reduction
  float* red = reinterpret_cast<float*>(smem);  // [2 groups x 4 warps][GM][128]: at most 64 KB, stage 0
  if (warp >= 1) {
    const int cw = warp - 1;  // group * 4 + warp of the group
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      *reinterpret_cast<float4*>(red + (cw * GM + g) * kFHd + lane * 4) =
          make_float4(acc[g][0], acc[g][1], acc[g][2], acc[g][3]);
    }
  }
  __syncthreads();
  if (warp >= 1) {
    for (int i = tid - 32; i < G * kFHd; i += kFCompute) {
      const int g = i / kFHd, d = i - g * kFHd;
      // merge the two groups' (max, sum, output) like two splits
      const float m0 = mfin[g], m1 = mfin[kMaxGroup + g];
      const float m = fmaxf(m0, m1);  // finite: group 0 holds at least one tile
      const float f0 = exp2f(m0 - m), f1 = m1 == -INFINITY ? 0.f : exp2f(m1 - m);
      float o0 = 0.f, o1 = 0.f, l0 = 0.f, l1 = 0.f;
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        o0 += red[(w * GM + g) * kFHd + d];
        o1 += red[((4 + w) * GM + g) * kFHd + d];
        l0 += lsum[w * kMaxGroup + g];
        l1 += lsum[(4 + w) * kMaxGroup + g];
      }
      const float o = o0 * f0 + o1 * f1;
      const float l = l0 * f0 + l1 * f1;
      if (ws == nullptr) {
        float* out = static_cast<float*>(a.out) + (b * a.hq + static_cast<int64_t>(kvh) * G + g) * kFHd;
        out[d] = o / l;
      } else {
        ws[g * (kFHd + 2) + d] = o;
        if (d == 0) {
          ws[g * (kFHd + 2) + kFHd] = m;
          ws[g * (kFHd + 2) + kFHd + 1] = l;
        }
      }
    }
  }
}

}  // namespace

bool f32_tma_eligible(const AttnArgs& a, bm_dtype_t dtype) {
  const int64_t rows = static_cast<int64_t>(a.num_seqs) * a.hkv * a.max_seq;
  return dtype == BM_F32 && a.hd == kFHd && a.group <= kMaxGroup && aligned16(a.q) && aligned16(a.k_cache) &&
         aligned16(a.v_cache) && rows + kFTile < (int64_t{1} << 31);
}

int launch_f32_tma(const AttnArgs& a, cudaStream_t stream) {
  const char* what = "bm_decode_attention";
  const uint64_t rows = static_cast<uint64_t>(a.num_seqs) * a.hkv * a.max_seq;
  CUtensorMap tk, tv;
  if (int st = make_tensor_map_2d(&tk, a.k_cache, BM_F32, kFHd, rows, 32, kFTile, what)) return st;
  if (int st = make_tensor_map_2d(&tv, a.v_cache, BM_F32, kFHd, rows, 32, kFTile, what)) return st;
  const dim3 grid(a.splits, a.hkv, static_cast<unsigned>(a.batch));
  auto go = [&](auto kernel) {
    if (int st = allow_dynamic_smem(reinterpret_cast<const void*>(kernel), kFSmemBytes, what)) return st;
    if (const int launch_status = launch_kernel(what, kernel, dim3(grid), dim3(kFThreads), kFSmemBytes, stream,
                                                nullptr, tk, tv, a)) {
      return launch_status;
    }
    return check_launch(what);
  };
  int st;
  if (a.group <= 1) {
    st = go(attention_f32_tma_kernel<1>);
  } else if (a.group <= 2) {
    st = go(attention_f32_tma_kernel<2>);
  } else if (a.group <= 4) {
    st = go(attention_f32_tma_kernel<4>);
  } else if (a.group <= 8) {
    st = go(attention_f32_tma_kernel<8>);
  } else {
    st = go(attention_f32_tma_kernel<16>);
  }
  if (st != BM_OK || a.splits == 1) return st;
  return launch_combine<float>(a, stream);
}

}  // namespace attn
}  // namespace bm
