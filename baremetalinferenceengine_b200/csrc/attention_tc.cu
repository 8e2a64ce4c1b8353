// Decode attention on the tensor cores (tcgen05 + TMA) for bf16 caches with
// head_dim 128, the Llama-3 8B/70B shape. Same contract and results as the
// CUDA-core kernel in attention_kernels.cuh (reference semantics:
// src/kernels.cu:225-264, batched and GQA as bm_decode_attention documents).
//
// One CTA per (query, kv head, split), as in the CUDA-core kernel, but the two
// contractions of each 128-position tile run as tcgen05.mma with fp32
// accumulators in TMEM:
//   scores  S^T[pos][g] = K[pos][:] . Q[g][:]      M=128 positions, N=16, K=128
//           (A = the K tile, K-major; B = the group's queries, zero-padded to 16)
//   mix     O^T[d][g]   = V^T[d][pos] . P^T[pos][g] M=128 dims, N=16, K=128
//           (A = the V tile read MN-major; B = the bf16 probabilities, K-major)
// Six warps:
//   warp 0     TMA: the K and V tiles of the split, 2 boxes of 128 rows x 64
//              dims each (128-byte swizzle), into a 3-stage ring (64 KB a stage);
//   warp 1     owns TMEM (64 columns: two score and two mix buffers); one thread
//              issues the score MMAs of tile i, then the mix MMAs of tile i-1;
//   warps 2-5  thread t owns TMEM lane t: position t of the tile for the
//              softmax (tile maxima through shared memory, base-2 online
//              softmax, bf16 P written swizzled for the mix MMA) and dimension
//              t for the rescale-and-accumulate of each tile's mix output.
// Positions past the query's length are masked (p = 0), and the V rows behind
// them in the last tile are cleared in shared memory first, so that stale cache
// contents (which may hold NaN) cannot reach the mix. Every mbarrier wait is
// bounded in time: past the limit the CTA raises BM_DEVERR_TIMEOUT, lets its
// copies and MMAs land, frees TMEM and returns.
#include <cuda.h>

#include "attention_kernels.cuh"
#include "bm_tc.cuh"
#include "bm_tma.h"

namespace bm {
namespace attn {

using namespace bm::tc;

namespace {

constexpr int kTcTile = 128;     // positions per tile: M of the score MMA
constexpr int kTcHd = 128;       // head_dim: M of the mix MMA
constexpr int kTcN = 16;         // queries of a group, zero-padded: N of both MMAs
constexpr int kTcStages = 3;
constexpr int kTcThreads = 192;
constexpr int kTcSoftmaxThreads = 128;
constexpr int kBoxBytes = kTcTile * 64 * 2;            // 128 rows x 64 dims of bf16: 16 KB
constexpr int kStageBytes = 4 * kBoxBytes;             // K (2 boxes) + V (2 boxes): 64 KB
constexpr int kQBytes = kTcN * kTcHd * 2;              // 4 KB
constexpr int kPBytes = kTcN * kTcTile * 2;            // 4 KB
constexpr int kOffQ = kTcStages * kStageBytes;
constexpr int kOffP = kOffQ + kQBytes;                 // two P buffers
constexpr int kOffMax = kOffP + 2 * kPBytes;           // [2][4][16] floats
constexpr int kOffL = kOffMax + 2 * 4 * kTcN * 4;      // [4][16] floats
constexpr int kOffBar = kOffL + 4 * kTcN * 4;
constexpr int kNumBars = 2 * kTcStages + 5 * 2 + 2;
constexpr int kTcSmemBytes = kOffBar + kNumBars * 8 + 16 + 1024 /* alignment slack */;
constexpr uint32_t kTmemCols = 64;
constexpr uint64_t kWaitNs = 2000000000ull;
constexpr uint64_t kDrainNs = 200000000ull;

constexpr uint32_t kIdescScore = instr_desc_bf16(false, false, kTcN, kTcTile);
constexpr uint32_t kIdescMix = instr_desc_bf16(true, false, kTcN, kTcHd);

// Byte offset of element (row, col) of a K-major, 128-byte-swizzled operand of
// `rows` rows whose K extent is split into 64-element atoms.
__device__ __forceinline__ uint32_t swz_offset(int row, int col, int rows) {
  const int atom = col >> 6, byte = (col & 63) * 2;
  return static_cast<uint32_t>(atom * rows * 128 + row * 128 + ((((byte >> 4) ^ (row & 7)) << 4) | (byte & 15)));
}

// Lane 0 waits, the warp gets its verdict (and reconverges for warp-wide tcgen05 ops).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int32_t* status) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = wait_phase(bar, parity, abort_flag, status, kWaitNs, true);
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// The four softmax warps meet here once per tile (barrier 1, 128 threads); the
// result is true when any of them saw the abort flag set, the same for all.
__device__ __forceinline__ bool softmax_warps_sync_any(bool flag) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.or.pred p, 1, 128, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(flag))
      : "memory");
  return r != 0;
}

// GM: the group size rounded up to a power of two; the softmax works on GM
// queries (the MMAs always on 16, the rows past GM of P stay zero).
template <int GM>
__global__ void __launch_bounds__(kTcThreads, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
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
  float* ws = a.ws ? a.ws + (((b * a.hkv + kvh) * a.splits + split) * G) * static_cast<int64_t>(kTcHd + 2) : nullptr;
  if (start >= end) {
    if (ws != nullptr && tid < G) {
      ws[tid * (kTcHd + 2) + kTcHd] = -INFINITY;
      ws[tid * (kTcHd + 2) + kTcHd + 1] = 0.f;
    }
    return;
  }
  const int n_tiles = (end - start + kTcTile - 1) / kTcTile;
  const int row0 = (seq * a.hkv + kvh) * a.max_seq + start;  // tensor-map row of the split's first position

  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                         ~static_cast<uintptr_t>(1023));
  unsigned char* q_s = smem + kOffQ;
  unsigned char* p_s = smem + kOffP;
  float* wmax = reinterpret_cast<float*>(smem + kOffMax);
  float* lsum = reinterpret_cast<float*>(smem + kOffL);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* empty = full + kTcStages;
  uint64_t* sfull = empty + kTcStages;  // score MMA done          (1 arrival: commit)
  uint64_t* sfree = sfull + 2;          // scores read from TMEM   (128)
  uint64_t* pfull = sfree + 2;          // P written               (128)
  uint64_t* ofull = pfull + 2;          // mix MMA done            (commit)
  uint64_t* ofree = ofull + 2;          // mix output read         (128)
  uint64_t* mma_done = ofree + 2;
  uint64_t* q_ready = mma_done + 1;     // queries and zeroed P in shared memory (128)
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(q_ready + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_s + 1);

  if (tid == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sfull[i], 1);
      mbar_init(&sfree[i], kTcSoftmaxThreads);
      mbar_init(&pfull[i], kTcSoftmaxThreads);
      mbar_init(&ofull[i], 1);
      mbar_init(&ofree[i], kTcSoftmaxThreads);
    }
    mbar_init(mma_done, 1);
    mbar_init(q_ready, kTcSoftmaxThreads);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_base_s, kTmemCols);
  tc_fence_before();
  __syncthreads();  // barriers and TMEM exist: the first copies start while the queries are staged
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_s;
  if (warp >= 2) {
    // the group's queries, rows >= G zero, as the score MMA's K-major B operand
    const int t = tid - 64;
    const bf16* qb = static_cast<const bf16*>(a.q) + (b * a.hq + static_cast<int64_t>(kvh) * G) * kTcHd;
    for (int c = t; c < kTcN * (kTcHd / 8); c += kTcSoftmaxThreads) {
      const int row = c / (kTcHd / 8), col = (c % (kTcHd / 8)) * 8;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (row < G) v = __ldg(reinterpret_cast<const uint4*>(qb + row * kTcHd + col));
      *reinterpret_cast<uint4*>(q_s + swz_offset(row, col, kTcN)) = v;
    }
    for (int c = t; c < 2 * kPBytes / 16; c += kTcSoftmaxThreads) {  // both P buffers start at zero
      *reinterpret_cast<uint4*>(p_s + c * 16) = make_uint4(0u, 0u, 0u, 0u);
    }
    fence_proxy_async_smem();
    mbar_arrive(q_ready);
  }

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer ----------------
    uint32_t last_parity[kTcStages];
    bool filled[kTcStages];
    for (int s = 0; s < kTcStages; ++s) filled[s] = false;
    for (int i = 0; i < n_tiles; ++i) {
      const int s = i % kTcStages;
      const uint32_t par = static_cast<uint32_t>((i / kTcStages) & 1);
      if (!wait_phase(&empty[s], par ^ 1u, abort_flag, a.status, kWaitNs, true)) break;
      unsigned char* st = smem + s * kStageBytes;
      mbar_expect_tx(&full[s], kStageBytes);
      const int y = row0 + i * kTcTile;
      tma_load_2d(st, &tk, &full[s], 0, y);
      tma_load_2d(st + kBoxBytes, &tk, &full[s], 64, y);
      tma_load_2d(st + 2 * kBoxBytes, &tv, &full[s], 0, y);
      tma_load_2d(st + 3 * kBoxBytes, &tv, &full[s], 64, y);
      filled[s] = true;
      last_parity[s] = par;
    }
    for (int s = 0; s < kTcStages; ++s) {
      if (filled[s]) wait_phase(&full[s], last_parity[s], abort_flag, a.status, kDrainNs, false);
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer ----------------
    bool issued = false;
    const uint32_t q_addr = smem_u32(q_s);
    const bool q_ok = wait_phase(q_ready, 0, abort_flag, a.status, kWaitNs, true);
    for (int i = 0; q_ok && i <= n_tiles; ++i) {
      if (i < n_tiles) {  // scores of tile i
        const int s = i % kTcStages;
        if (!wait_phase(&full[s], static_cast<uint32_t>((i / kTcStages) & 1), abort_flag, a.status, kWaitNs, true)) {
          break;
        }
        if (!wait_phase(&sfree[i & 1], static_cast<uint32_t>(((i >> 1) & 1) ^ 1), abort_flag, a.status, kWaitNs,
                        true)) {
          break;
        }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + s * kStageBytes);
#pragma unroll
        for (int kk = 0; kk < kTcHd / 16; ++kk) {
          const uint64_t ad = smem_desc(k_addr + (kk >> 2) * kBoxBytes + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = smem_desc(q_addr + (kk >> 2) * (kTcN * 128) + (kk & 3) * 32, 16, 1024);
          mma_bf16(tmem_base + (i & 1) * kTcN, ad, bd, kIdescScore, kk > 0 ? 1u : 0u);
        }
        issued = true;
        mma_commit(&sfull[i & 1]);
      }
      if (i >= 1) {  // mix of tile i - 1
        const int j = i - 1;
        if (!wait_phase(&pfull[j & 1], static_cast<uint32_t>((j >> 1) & 1), abort_flag, a.status, kWaitNs, true)) {
          break;
        }
        if (!wait_phase(&ofree[j & 1], static_cast<uint32_t>(((j >> 1) & 1) ^ 1), abort_flag, a.status, kWaitNs,
                        true)) {
          break;
        }
        tc_fence_after();
        const uint32_t v_addr = smem_u32(smem + (j % kTcStages) * kStageBytes + 2 * kBoxBytes);
        const uint32_t p_addr = smem_u32(p_s + (j & 1) * kPBytes);
#pragma unroll
        for (int kk = 0; kk < kTcTile / 16; ++kk) {
          // V^T: dims contiguous (MN-major), 64-dim blocks a box apart, 8-position groups 1024 bytes apart
          const uint64_t ad = smem_desc(v_addr + kk * 2048, kBoxBytes, 1024);
          const uint64_t bd = smem_desc(p_addr + (kk >> 2) * (kTcN * 128) + (kk & 3) * 32, 16, 1024);
          mma_bf16(tmem_base + 2 * kTcN + (j & 1) * kTcN, ad, bd, kIdescMix, kk > 0 ? 1u : 0u);
        }
        mma_commit(&ofull[j & 1]);
        mma_commit(&empty[j % kTcStages]);  // K and V of tile j are no longer read
      }
    }
    if (issued) {
      mma_commit(mma_done);
      wait_phase(mma_done, 0, abort_flag, a.status, kDrainNs, false);
    }
  }

  // ---------------- softmax and accumulation (warps 2-5) ----------------
  // A timed-out wait sets the abort flag and the warp carries on to the next
  // tile barrier, where all four warps see the flag and leave together.
  const int quarter = warp & 3;
  const int t = quarter * 32 + lane;  // TMEM lane: tile position t (scores), dimension t (mix)
  float m_run[GM], l_part[GM], acc[GM], alpha_prev[GM];
  if (warp >= 2) {
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      m_run[g] = -INFINITY;
      l_part[g] = 0.f;
      acc[g] = 0.f;
      alpha_prev[g] = 0.f;
    }
    auto accumulate = [&](int j) {  // tile j's mix output, rescaled by its own factor
      warp_wait(&ofull[j & 1], static_cast<uint32_t>((j >> 1) & 1), abort_flag, a.status);
      tc_fence_after();
      uint32_t o[kTcN];
      tmem_load16(tmem_base + lane_addr + 2 * kTcN + (j & 1) * kTcN, o);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&ofree[j & 1]);
#pragma unroll
      for (int g = 0; g < GM; ++g) acc[g] = fmaf(acc[g], alpha_prev[g], __uint_as_float(o[g]));
    };
    for (int i = 0; i < n_tiles; ++i) {
      warp_wait(&sfull[i & 1], static_cast<uint32_t>((i >> 1) & 1), abort_flag, a.status);
      tc_fence_after();
      uint32_t r[kTcN];
      tmem_load16(tmem_base + lane_addr + (i & 1) * kTcN, r);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&sfree[i & 1]);
      const int tile_start = start + i * kTcTile;
      const bool valid = tile_start + t < end;
      float s[GM];
#pragma unroll
      for (int g = 0; g < GM; ++g) s[g] = valid ? __uint_as_float(r[g]) * a.qscale : -INFINITY;
      // tile maxima: warp shuffles, then the four warps through shared memory
      float* wm = wmax + (i & 1) * 4 * kTcN;
#pragma unroll
      for (int g = 0; g < GM; ++g) {
        float v = s[g];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
        if (lane == 0) wm[quarter * kTcN + g] = v;
      }
      if (softmax_warps_sync_any(*abort_flag != 0)) break;
      float alpha[GM];
      unsigned char* pb = p_s + (i & 1) * kPBytes;
#pragma unroll
      for (int g = 0; g < GM; ++g) {
        // every tile holds a valid position, so the tile maximum is finite
        const float tmax = fmaxf(fmaxf(wm[g], wm[kTcN + g]), fmaxf(wm[2 * kTcN + g], wm[3 * kTcN + g]));
        const float m_new = fmaxf(m_run[g], tmax);
        alpha[g] = exp2f(m_run[g] - m_new);
        m_run[g] = m_new;
        const float p = (valid && g < G) ? exp2f(s[g] - m_new) : 0.f;
        l_part[g] = l_part[g] * alpha[g] + p;
        *reinterpret_cast<bf16*>(pb + swz_offset(g, t, kTcN)) = __float2bfloat16_rn(p);
      }
      if (!valid) {  // clear this stage's V row t, so stale cache contents cannot reach the mix
        const int s_idx = i % kTcStages;
        wait_phase(&full[s_idx], static_cast<uint32_t>((i / kTcStages) & 1), abort_flag, a.status, kWaitNs, true);
        unsigned char* vrow = smem + s_idx * kStageBytes + 2 * kBoxBytes + t * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          *reinterpret_cast<uint4*>(vrow + c * 16) = make_uint4(0u, 0u, 0u, 0u);
          *reinterpret_cast<uint4*>(vrow + kBoxBytes + c * 16) = make_uint4(0u, 0u, 0u, 0u);
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(&pfull[i & 1]);
      if (i >= 1) accumulate(i - 1);
#pragma unroll
      for (int g = 0; g < GM; ++g) alpha_prev[g] = alpha[g];
      if (i == n_tiles - 1) accumulate(i);
    }
    // the row sums: each thread holds its positions' share
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      const float v = warp_sum(l_part[g]);
      if (lane == 0) lsum[quarter * kTcN + g] = v;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp >= 2) {
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      if (g < G) {
        const float l = lsum[g] + lsum[kTcN + g] + lsum[2 * kTcN + g] + lsum[3 * kTcN + g];
        if (ws == nullptr) {
          bf16* out = static_cast<bf16*>(a.out) + (b * a.hq + static_cast<int64_t>(kvh) * G + g) * kTcHd;
          out[t] = __float2bfloat16_rn(acc[g] / l);
        } else {
          ws[g * (kTcHd + 2) + t] = acc[g];
          if (t == 0) {
            ws[g * (kTcHd + 2) + kTcHd] = m_run[g];
            ws[g * (kTcHd + 2) + kTcHd + 1] = l;
          }
        }
      }
    }
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace

bool tc_eligible(const AttnArgs& a, bm_dtype_t dtype) {
  const int64_t rows = static_cast<int64_t>(a.num_seqs) * a.hkv * a.max_seq;
  return dtype == BM_BF16 && a.hd == kTcHd && a.group <= kTcN && aligned16(a.q) && aligned16(a.k_cache) &&
         aligned16(a.v_cache) && rows + kTcTile < (int64_t{1} << 31);
}

int launch_tc(const AttnArgs& a, cudaStream_t stream) {
  const char* what = "bm_decode_attention";
  const uint64_t rows = static_cast<uint64_t>(a.num_seqs) * a.hkv * a.max_seq;
  CUtensorMap tk, tv;
  if (int st = make_tensor_map_bf16(&tk, a.k_cache, kTcHd, rows, 64, kTcTile, what)) return st;
  if (int st = make_tensor_map_bf16(&tv, a.v_cache, kTcHd, rows, 64, kTcTile, what)) return st;
  const dim3 grid(a.splits, a.hkv, static_cast<unsigned>(a.batch));
  auto go = [&](auto kernel) {
    if (int st = allow_dynamic_smem(reinterpret_cast<const void*>(kernel), kTcSmemBytes, what)) return st;
    if (const int launch_status = launch_kernel(what, kernel, dim3(grid), dim3(kTcThreads), kTcSmemBytes, stream,
                                                nullptr, tk, tv, a)) {
      return launch_status;
    }
    return check_launch(what);
  };
  int st;
  if (a.group <= 1) {
    st = go(attention_tc_kernel<1>);
  } else if (a.group <= 2) {
    st = go(attention_tc_kernel<2>);
  } else if (a.group <= 4) {
    st = go(attention_tc_kernel<4>);
  } else if (a.group <= 8) {
    st = go(attention_tc_kernel<8>);
  } else {
    st = go(attention_tc_kernel<16>);
  }
  if (st != BM_OK) return st;
  if (a.splits == 1) return BM_OK;
  return launch_combine<bf16>(a, stream);
}

}  // namespace attn
}  // namespace bm
