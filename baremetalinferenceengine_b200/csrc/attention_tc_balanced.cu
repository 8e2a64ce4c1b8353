// Decode attention on the tensor cores with the work balanced across the SMs:
// the persistent form of attention_tc.cu (same MMAs, TMEM layout, softmax and
// masking; same contract and results: reference semantics src/kernels.cu:225-264,
// batched and GQA as bm_decode_attention documents).
//
// The one-CTA-per-(query, kv head, split) grid of attention_tc.cu plans its
// splits from the longest length alone (the host does not see the lengths), so
// with ragged lengths its CTAs carry anything from nothing to a whole split, and
// each CTA pays its start-up (barriers, TMEM, first copies) and its drain. Here
// one CTA per SM walks an equal share of all the work:
//   - every (query, kv head) pair is cut into tiles of 128 positions, ceil(len /
//     128) of them; laid end to end, pair by pair (query-major), they form one
//     sequence of `total` tiles;
//   - CTA k of nc takes tiles [k*total/nc, (k+1)*total/nc): each CTA computes the
//     per-query tile prefix from the lengths in device memory (a block scan into
//     shared memory, batch <= kBalancedMaxBatch) and walks its range;
//   - a run of the range inside one pair is a segment. The producer loads the
//     pair's queries by TMA into one of two query buffers at each segment start;
//     the softmax warps reset the running maximum, sum and output there, and at
//     the segment end write the normalised output when the segment holds the
//     whole pair, else its (output, max, sum) partial into the workspace;
//   - only a CTA's first and last segments can be partial, so partials take two
//     slots per CTA. A pair that starts in CTA k and ends in CTA k' > k is
//     recorded by CTA k, and balanced_combine_kernel merges its partials.
// Every mbarrier wait is bounded in time as in attention_tc.cu.
#include <cuda.h>

#include "attention_kernels.cuh"
#include "bm_tc.cuh"
#include "bm_tma.h"

namespace bm {
namespace attn {

using namespace bm::tc;

namespace {

constexpr int kTile = 128;  // positions per tile: M of the score MMA
constexpr int kHd = 128;    // head_dim: M of the mix MMA
constexpr int kN = 16;      // queries of a group, padded: N of both MMAs
constexpr int kStages = 3;
constexpr int kThreadsB = 192;
constexpr int kSoftmaxThreads = 128;
constexpr int kBoxBytes = kTile * 64 * 2;        // 128 rows x 64 dims of bf16: 16 KB
constexpr int kStageBytes = 4 * kBoxBytes;       // K (2 boxes) + V (2 boxes): 64 KB
constexpr int kQBytes = kN * kHd * 2;            // 4 KB
constexpr int kPBytes = kN * kTile * 2;          // 4 KB
constexpr int kOffQ = kStages * kStageBytes;     // two query buffers
constexpr int kOffP = kOffQ + 2 * kQBytes;       // two P buffers
constexpr int kOffMax = kOffP + 2 * kPBytes;     // [2][4][16] floats
constexpr int kOffL = kOffMax + 2 * 4 * kN * 4;  // [4][16] floats
constexpr int kOffScan = kOffL + 4 * kN * 4;     // [6] ints (warp totals of the scan)
constexpr int kOffBar = kOffScan + 8 * 4;
constexpr int kNumBars = 2 * kStages + 5 * 2 + 2 * 2 + 1;
constexpr int kOffMisc = kOffBar + kNumBars * 8;   // TMEM base, abort flag
constexpr int kOffPre = kOffMisc + 16;             // tile prefix per query [batch + 1]
constexpr int kSmemBytes = kOffPre + (kBalancedMaxBatch + 1) * 4 + 1024 /* alignment slack */;
static_assert(kSmemBytes <= 232448, "shared memory per CTA");
static_assert(kOffQ % 1024 == 0 && kOffP % 1024 == 0 && kQBytes % 1024 == 0, "swizzled operands 1024-aligned");
static_assert(kOffBar % 8 == 0, "mbarriers 8-aligned");
constexpr uint32_t kTmemCols = 64;
constexpr uint64_t kWaitNs = 2000000000ull;
constexpr uint64_t kDrainNs = 200000000ull;

constexpr uint32_t kIdescScore = instr_desc_bf16(false, false, kN, kTile);
constexpr uint32_t kIdescMix = instr_desc_bf16(true, false, kN, kHd);

// Per-CTA record in the workspace: the pair whose first tile is in this CTA and
// whose last tile is in a later one (pair = -1: none), the CTA holding its last
// tile, the slot of this CTA's partial for it, and the plan's tile count (CTAs
// between the two whose ranges are empty hold no partial).
struct SplitRecord {
  int64_t total;
  int32_t pair, k_last, slot_first, unused;
};
static_assert(sizeof(SplitRecord) == 24, "record layout");

__device__ __forceinline__ float* partial_slots(const AttnArgs& a) {
  return a.ws + static_cast<int64_t>(a.splits) * (sizeof(SplitRecord) / sizeof(float));
}

// Byte offset of element (row, col) of a K-major, 128-byte-swizzled operand of
// `rows` rows whose K extent is split into 64-element atoms.
__device__ __forceinline__ uint32_t swz_offset(int row, int col, int rows) {
  const int atom = col >> 6, byte = (col & 63) * 2;
  return static_cast<uint32_t>(atom * rows * 128 + row * 128 + ((((byte >> 4) ^ (row & 7)) << 4) | (byte & 15)));
}

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int32_t* status) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = wait_phase(bar, parity, abort_flag, status, kWaitNs, true);
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// The softmax warps' per-tile meeting (barrier 1, 128 threads): true when any
// of them saw the abort flag, the same for all.
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

__device__ __forceinline__ void softmax_warps_sync() { asm volatile("bar.sync 2, 128;" ::: "memory"); }

__device__ __forceinline__ int tiles_of(int len) { return (len + kTile - 1) / kTile; }

// Position in the tile sequence: query b, kv head kvh, tile tip of the pair's
// ntiles. pre[b] = tiles of the queries before b (per kv head).
struct Cursor {
  int b, kvh, tip, ntiles, seq, len;

  __device__ void load_query(const AttnArgs& a, const int* pre) {
    ntiles = pre[b + 1] - pre[b];
    check_query(a, b, &seq, &len);
  }
  // g < total: the largest b with hkv * pre[b] <= g holds tile g.
  __device__ void init(const AttnArgs& a, const int* pre, int nb, int64_t g) {
    int lo = 0, hi = nb - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (static_cast<int64_t>(a.hkv) * pre[mid] <= g) {
        lo = mid;
      } else {
        hi = mid - 1;
      }
    }
    b = lo;
    load_query(a, pre);
    const int64_t r = g - static_cast<int64_t>(a.hkv) * pre[b];
    kvh = static_cast<int>(r / ntiles);
    tip = static_cast<int>(r - static_cast<int64_t>(kvh) * ntiles);
  }
  // Only called while a later tile exists, so a query with tiles follows.
  __device__ void advance(const AttnArgs& a, const int* pre) {
    if (++tip < ntiles) return;
    tip = 0;
    if (++kvh < a.hkv) return;
    kvh = 0;
    do {
      ++b;
    } while (pre[b + 1] == pre[b]);
    load_query(a, pre);
  }
};

// The CTA of nc whose range [k*total/nc, (k+1)*total/nc) holds tile t.
__device__ __forceinline__ int cta_of(int64_t t, int64_t total, int nc) {
  int c = static_cast<int>(t * nc / total);
  while (c + 1 < nc && total * (c + 1) / nc <= t) ++c;
  return c;
}

template <int GM>
__global__ void __launch_bounds__(kThreadsB, 1)
    attention_tc_balanced_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                                 const __grid_constant__ CUtensorMap tq, const AttnArgs a) {
  grid_dependency_wait();
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                         ~static_cast<uintptr_t>(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nb = static_cast<int>(a.batch);
  const int nc = static_cast<int>(gridDim.x), k = static_cast<int>(blockIdx.x);
  const int G = a.group;
  SplitRecord* records = reinterpret_cast<SplitRecord*>(a.ws);
  if (tid == 0) records[k] = SplitRecord{0, -1, -1, -1, 0};

  // ---------------- the plan: tiles per query, prefix in shared memory ----------------
  int* pre = reinterpret_cast<int*>(smem + kOffPre);
  int* scan = reinterpret_cast<int*>(smem + kOffScan);
  {
    const int per = (nb + kThreadsB - 1) / kThreadsB;
    const int b_lo = min(nb, tid * per), b_hi = min(nb, b_lo + per);
    int local = 0;
    for (int b = b_lo; b < b_hi; ++b) {
      int seq, len;
      const int32_t bad = check_query(a, b, &seq, &len);
      if (bad && k == 0) raise_status(a.status, bad);
      local += bad ? 0 : tiles_of(len);
    }
    int incl = local;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += v;
    }
    if (lane == 31) scan[warp] = incl;
    __syncthreads();
    int run = incl - local;
    for (int w = 0; w < warp; ++w) run += scan[w];
    for (int b = b_lo; b < b_hi; ++b) {
      pre[b] = run;
      int seq, len;
      run += check_query(a, b, &seq, &len) ? 0 : tiles_of(len);
    }
    if (tid == kThreadsB - 1) pre[nb] = run;
  }
  __syncthreads();
  const int64_t total = static_cast<int64_t>(a.hkv) * pre[nb];
  const int64_t t0 = total * k / nc, t1 = total * (k + 1) / nc;
  if (t0 >= t1) return;  // no tiles here (the same for every thread)
  const int n = static_cast<int>(t1 - t0);
  // the query box: 16 rows, or all of q's rows when it has fewer (two 64-column boxes)
  const uint32_t q_box_bytes = 2u * static_cast<uint32_t>(a.batch * a.hq < kN ? a.batch * a.hq : kN) * 128u;

  unsigned char* q_s = smem + kOffQ;
  unsigned char* p_s = smem + kOffP;
  float* wmax = reinterpret_cast<float*>(smem + kOffMax);
  float* lsum = reinterpret_cast<float*>(smem + kOffL);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* empty = full + kStages;
  uint64_t* sfull = empty + kStages;  // score MMA done          (commit)
  uint64_t* sfree = sfull + 2;        // scores read from TMEM   (128)
  uint64_t* pfull = sfree + 2;        // P written               (128)
  uint64_t* ofull = pfull + 2;        // mix MMA done            (commit)
  uint64_t* ofree = ofull + 2;        // mix output read         (128)
  uint64_t* qfull = ofree + 2;        // queries loaded          (TMA bytes)
  uint64_t* qfree = qfull + 2;        // last score MMA of the segment done (commit)
  uint64_t* mma_done = qfree + 2;
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_s + 1);

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sfull[i], 1);
      mbar_init(&sfree[i], kSoftmaxThreads);
      mbar_init(&pfull[i], kSoftmaxThreads);
      mbar_init(&ofull[i], 1);
      mbar_init(&ofree[i], kSoftmaxThreads);
      mbar_init(&qfull[i], 1);
      mbar_init(&qfree[i], 1);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  // both P buffers start at zero: rows past the group are never written
  for (int c = tid; c < 2 * kPBytes / 16; c += kThreadsB) {
    *reinterpret_cast<uint4*>(p_s + c * 16) = make_uint4(0u, 0u, 0u, 0u);
  }
  fence_proxy_async_smem();
  if (warp == 1) tmem_alloc(tmem_base_s, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_s;

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer: queries at each segment start, K and V per tile ----------------
    uint32_t last_parity[kStages];
    bool filled[kStages] = {false, false, false};
    bool q_filled[2] = {false, false};
    uint32_t q_parity[2] = {0u, 0u};
    Cursor c;
    c.init(a, pre, nb, t0);
    int seg = -1;
    for (int i = 0; i < n; ++i) {
      if (i > 0) c.advance(a, pre);
      if (i == 0 || c.tip == 0) {
        ++seg;
        const int qb = seg & 1;
        const uint32_t qpar = static_cast<uint32_t>((seg >> 1) & 1);
        if (!wait_phase(&qfree[qb], qpar ^ 1u, abort_flag, a.status, kWaitNs, true)) break;
        mbar_expect_tx(&qfull[qb], q_box_bytes);
        const int qrow = c.b * a.hq + c.kvh * G;
        tma_load_2d(q_s + qb * kQBytes, &tq, &qfull[qb], 0, qrow);
        tma_load_2d(q_s + qb * kQBytes + kN * 128, &tq, &qfull[qb], 64, qrow);
        q_filled[qb] = true;
        q_parity[qb] = qpar;
      }
      const int s = i % kStages;
      const uint32_t par = static_cast<uint32_t>((i / kStages) & 1);
      if (!wait_phase(&empty[s], par ^ 1u, abort_flag, a.status, kWaitNs, true)) break;
      unsigned char* st = smem + s * kStageBytes;
      mbar_expect_tx(&full[s], kStageBytes);
      const int y = (c.seq * a.hkv + c.kvh) * a.max_seq + c.tip * kTile;
      tma_load_2d(st, &tk, &full[s], 0, y);
      tma_load_2d(st + kBoxBytes, &tk, &full[s], 64, y);
      tma_load_2d(st + 2 * kBoxBytes, &tv, &full[s], 0, y);
      tma_load_2d(st + 3 * kBoxBytes, &tv, &full[s], 64, y);
      filled[s] = true;
      last_parity[s] = par;
    }
    for (int s = 0; s < kStages; ++s) {
      if (filled[s]) wait_phase(&full[s], last_parity[s], abort_flag, a.status, kDrainNs, false);
    }
    for (int qb = 0; qb < 2; ++qb) {
      if (q_filled[qb]) wait_phase(&qfull[qb], q_parity[qb], abort_flag, a.status, kDrainNs, false);
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer: scores of tile i, then the mix of tile i-1 ----------------
    bool issued = false;
    Cursor c;
    c.init(a, pre, nb, t0);
    int seg = -1;
    for (int i = 0; i <= n; ++i) {
      if (i < n) {
        if (i > 0) c.advance(a, pre);
        const bool first = i == 0 || c.tip == 0;
        const bool last = i == n - 1 || c.tip == c.ntiles - 1;
        if (first) {
          ++seg;
          if (!wait_phase(&qfull[seg & 1], static_cast<uint32_t>((seg >> 1) & 1), abort_flag, a.status, kWaitNs,
                          true)) {
            break;
          }
        }
        const int s = i % kStages;
        if (!wait_phase(&full[s], static_cast<uint32_t>((i / kStages) & 1), abort_flag, a.status, kWaitNs, true)) {
          break;
        }
        if (!wait_phase(&sfree[i & 1], static_cast<uint32_t>(((i >> 1) & 1) ^ 1), abort_flag, a.status, kWaitNs,
                        true)) {
          break;
        }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + s * kStageBytes);
        const uint32_t q_addr = smem_u32(q_s + (seg & 1) * kQBytes);
#pragma unroll
        for (int kk = 0; kk < kHd / 16; ++kk) {
          const uint64_t ad = smem_desc(k_addr + (kk >> 2) * kBoxBytes + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = smem_desc(q_addr + (kk >> 2) * (kN * 128) + (kk & 3) * 32, 16, 1024);
          mma_bf16(tmem_base + (i & 1) * kN, ad, bd, kIdescScore, kk > 0 ? 1u : 0u);
        }
        issued = true;
        mma_commit(&sfull[i & 1]);
        if (last) mma_commit(&qfree[seg & 1]);  // this query buffer may be reloaded
      }
      if (i >= 1) {
        const int j = i - 1;
        if (!wait_phase(&pfull[j & 1], static_cast<uint32_t>((j >> 1) & 1), abort_flag, a.status, kWaitNs, true)) {
          break;
        }
        if (!wait_phase(&ofree[j & 1], static_cast<uint32_t>(((j >> 1) & 1) ^ 1), abort_flag, a.status, kWaitNs,
                        true)) {
          break;
        }
        tc_fence_after();
        const uint32_t v_addr = smem_u32(smem + (j % kStages) * kStageBytes + 2 * kBoxBytes);
        const uint32_t p_addr = smem_u32(p_s + (j & 1) * kPBytes);
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk) {
          // V^T: dims contiguous (MN-major), 64-dim blocks a box apart, 8-position groups 1024 bytes apart
          const uint64_t ad = smem_desc(v_addr + kk * 2048, kBoxBytes, 1024);
          const uint64_t bd = smem_desc(p_addr + (kk >> 2) * (kN * 128) + (kk & 3) * 32, 16, 1024);
          mma_bf16(tmem_base + 2 * kN + (j & 1) * kN, ad, bd, kIdescMix, kk > 0 ? 1u : 0u);
        }
        mma_commit(&ofull[j & 1]);
        mma_commit(&empty[j % kStages]);  // K and V of tile j are no longer read
      }
    }
    if (issued) {
      mma_commit(mma_done);
      wait_phase(mma_done, 0, abort_flag, a.status, kDrainNs, false);
    }
  } else if (warp >= 2) {
    // ---------------- softmax and accumulation, segment by segment ----------------
    // A timed-out wait sets the abort flag and the warps leave together at the
    // next tile barrier.
    const int quarter = warp & 3;
    const int t = quarter * 32 + lane;  // TMEM lane: tile position t (scores), dimension t (mix)
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    float m_run[GM], l_part[GM], acc[GM], alpha_prev[GM];
    auto accumulate = [&](int j) {  // tile j's mix output, rescaled by its own factor
      warp_wait(&ofull[j & 1], static_cast<uint32_t>((j >> 1) & 1), abort_flag, a.status);
      tc_fence_after();
      uint32_t o[kN];
      tmem_load16(tmem_base + lane_addr + 2 * kN + (j & 1) * kN, o);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&ofree[j & 1]);
#pragma unroll
      for (int g = 0; g < GM; ++g) acc[g] = fmaf(acc[g], alpha_prev[g], __uint_as_float(o[g]));
    };
    Cursor c;
    c.init(a, pre, nb, t0);
    int seg = -1, seg_tip0 = 0;
    float* slots = partial_slots(a);
    for (int i = 0; i < n; ++i) {
      if (i > 0) c.advance(a, pre);
      const bool first = i == 0 || c.tip == 0;
      const bool last = i == n - 1 || c.tip == c.ntiles - 1;
      if (first) {
        ++seg;
        seg_tip0 = c.tip;
#pragma unroll
        for (int g = 0; g < GM; ++g) {
          m_run[g] = -INFINITY;
          l_part[g] = 0.f;
          acc[g] = 0.f;
          alpha_prev[g] = 0.f;
        }
      }
      warp_wait(&sfull[i & 1], static_cast<uint32_t>((i >> 1) & 1), abort_flag, a.status);
      tc_fence_after();
      uint32_t r[kN];
      tmem_load16(tmem_base + lane_addr + (i & 1) * kN, r);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&sfree[i & 1]);
      const bool valid = c.tip * kTile + t < c.len;
      float s[GM];
#pragma unroll
      for (int g = 0; g < GM; ++g) s[g] = valid ? __uint_as_float(r[g]) * a.qscale : -INFINITY;
      float* wm = wmax + (i & 1) * 4 * kN;
#pragma unroll
      for (int g = 0; g < GM; ++g) {
        float v = s[g];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
        if (lane == 0) wm[quarter * kN + g] = v;
      }
      if (softmax_warps_sync_any(*abort_flag != 0)) break;
      float alpha[GM];
      unsigned char* pb = p_s + (i & 1) * kPBytes;
#pragma unroll
      for (int g = 0; g < GM; ++g) {
        // every tile holds a valid position, so the tile maximum is finite
        const float tmax = fmaxf(fmaxf(wm[g], wm[kN + g]), fmaxf(wm[2 * kN + g], wm[3 * kN + g]));
        const float m_new = fmaxf(m_run[g], tmax);
        alpha[g] = exp2f(m_run[g] - m_new);
        m_run[g] = m_new;
        const float p = (valid && g < G) ? exp2f(s[g] - m_new) : 0.f;
        l_part[g] = l_part[g] * alpha[g] + p;
        *reinterpret_cast<bf16*>(pb + swz_offset(g, t, kN)) = __float2bfloat16_rn(p);
      }
      if (!valid) {  // clear this stage's V row t, so stale cache contents cannot reach the mix
        const int s_idx = i % kStages;
        wait_phase(&full[s_idx], static_cast<uint32_t>((i / kStages) & 1), abort_flag, a.status, kWaitNs, true);
        unsigned char* vrow = smem + s_idx * kStageBytes + 2 * kBoxBytes + t * 128;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          *reinterpret_cast<uint4*>(vrow + q * 16) = make_uint4(0u, 0u, 0u, 0u);
          *reinterpret_cast<uint4*>(vrow + kBoxBytes + q * 16) = make_uint4(0u, 0u, 0u, 0u);
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(&pfull[i & 1]);
      if (!first) accumulate(i - 1);
#pragma unroll
      for (int g = 0; g < GM; ++g) alpha_prev[g] = alpha[g];
      if (!last) continue;
      // ---- the segment ends: its output or its partial ----
      accumulate(i);
#pragma unroll
      for (int g = 0; g < GM; ++g) {
        const float v = warp_sum(l_part[g]);
        if (lane == 0) lsum[quarter * kN + g] = v;
      }
      softmax_warps_sync();
      const bool whole = seg_tip0 == 0 && c.tip == c.ntiles - 1;
      const int slot = 2 * k + (seg > 0 ? 1 : 0);
#pragma unroll
      for (int g = 0; g < GM; ++g) {
        if (g < G) {
          const float l = lsum[g] + lsum[kN + g] + lsum[2 * kN + g] + lsum[3 * kN + g];
          if (whole) {
            bf16* out = static_cast<bf16*>(a.out) + (static_cast<int64_t>(c.b) * a.hq + c.kvh * G + g) * kHd;
            out[t] = __float2bfloat16_rn(acc[g] / l);
          } else {
            float* w = slots + (static_cast<int64_t>(slot) * G + g) * (kHd + 2);
            w[t] = acc[g];
            if (t == 0) {
              w[kHd] = m_run[g];
              w[kHd + 1] = l;
            }
          }
        }
      }
      if (t == 0 && !whole && seg_tip0 == 0) {  // the pair starts here and ends in a later CTA
        const int64_t last_tile =
            static_cast<int64_t>(a.hkv) * pre[c.b] + static_cast<int64_t>(c.kvh + 1) * c.ntiles - 1;
        records[k] = SplitRecord{total, c.b * a.hkv + c.kvh, cta_of(last_tile, total, nc), slot, 0};
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// One CTA per (query of a group, CTA of the main kernel): when that CTA recorded
// a pair split across CTAs, merges the pair's partials for that query.
__global__ void __launch_bounds__(kCombineThreads) balanced_combine_kernel(const AttnArgs a) {
  grid_dependency_wait();
  extern __shared__ float w_s[];  // [pieces]
  __shared__ float red[kCombineThreads / 32];
  const int g = blockIdx.x, k = blockIdx.y, nc = a.splits;
  const SplitRecord rec = reinterpret_cast<const SplitRecord*>(a.ws)[k];
  const int64_t pairs = a.batch * a.hkv;
  if (rec.total <= 0 || rec.pair < 0 || rec.pair >= pairs || rec.k_last <= k || rec.k_last >= nc ||
      (rec.slot_first >> 1) != k) {
    return;
  }
  // CTA c's range [total*c/nc, total*(c+1)/nc) may be empty when total < nc: no partial there
  auto holds_tiles = [&](int c) { return rec.total * c / nc < rec.total * (c + 1) / nc; };
  const int64_t b = rec.pair / a.hkv;
  const int kvh = static_cast<int>(rec.pair - b * a.hkv);
  const int pieces = rec.k_last - k + 1;
  const float* slots = partial_slots(a);
  const int64_t slot_stride = static_cast<int64_t>(a.group) * (kHd + 2);
  auto piece = [&](int i) {
    const int slot = i == 0 ? rec.slot_first : 2 * (k + i);
    return slots + slot * slot_stride + static_cast<int64_t>(g) * (kHd + 2);
  };
  const int tid = threadIdx.x;
  float m = -INFINITY;
  for (int i = tid; i < pieces; i += kCombineThreads) {
    if (holds_tiles(k + i)) m = fmaxf(m, piece(i)[kHd]);
  }
  m = combine_block_reduce<kCombineThreads / 32>(m, true, red);  // finite: CTA k holds a partial
  float l = 0.f;
  for (int i = tid; i < pieces; i += kCombineThreads) {
    float w = 0.f;
    if (holds_tiles(k + i)) {
      const float* pc = piece(i);
      w = exp2f(pc[kHd] - m);
      l += pc[kHd + 1] * w;
    }
    w_s[i] = w;
  }
  l = combine_block_reduce<kCombineThreads / 32>(l, false, red);  // its barriers also publish w_s
  float o = 0.f;
  for (int i = 0; i < pieces; ++i) {
    const float w = w_s[i];
    if (w != 0.f) o = fmaf(piece(i)[tid], w, o);  // pieces of empty CTAs hold stale values: skipped
  }
  bf16* out = static_cast<bf16*>(a.out) + (b * a.hq + static_cast<int64_t>(kvh) * a.group + g) * kHd;
  out[tid] = __float2bfloat16_rn(o / l);
}

}  // namespace

size_t balanced_workspace_bytes(int group, int ctas) {
  return static_cast<size_t>(ctas) * sizeof(SplitRecord) +
         static_cast<size_t>(2) * ctas * group * (kHd + 2) * sizeof(float);
}

bool balanced_eligible(const AttnArgs& a, bm_dtype_t dtype) {
  return tc_eligible(a, dtype) && a.batch <= kBalancedMaxBatch && a.batch * a.hkv >= kBalancedMinPairs &&
         a.batch * a.hq < (int64_t{1} << 31);
}

int launch_tc_balanced(AttnArgs a, int ctas, cudaStream_t stream) {
  const char* what = "bm_decode_attention";
  const uint64_t rows = static_cast<uint64_t>(a.num_seqs) * a.hkv * a.max_seq;
  CUtensorMap tk, tv, tq;
  if (int st = make_tensor_map_bf16(&tk, a.k_cache, kHd, rows, 64, kTile, what)) return st;
  if (int st = make_tensor_map_bf16(&tv, a.v_cache, kHd, rows, 64, kTile, what)) return st;
  const uint64_t q_rows = static_cast<uint64_t>(a.batch) * a.hq;
  if (int st = make_tensor_map_bf16(&tq, a.q, kHd, q_rows, 64, static_cast<uint32_t>(std::min<uint64_t>(kN, q_rows)),
                                    what)) {
    return st;
  }
  a.splits = ctas;  // the combine step reads the CTA count from here
  auto go = [&](auto kernel) {
    if (int st = allow_dynamic_smem(reinterpret_cast<const void*>(kernel), kSmemBytes, what)) return st;
    if (const int launch_status = launch_kernel(what, kernel, dim3(ctas), dim3(kThreadsB), kSmemBytes, stream,
                                                nullptr, tk, tv, tq, a)) {
      return launch_status;
    }
    return check_launch(what);
  };
  int st;
  if (a.group <= 1) {
    st = go(attention_tc_balanced_kernel<1>);
  } else if (a.group <= 2) {
    st = go(attention_tc_balanced_kernel<2>);
  } else if (a.group <= 4) {
    st = go(attention_tc_balanced_kernel<4>);
  } else if (a.group <= 8) {
    st = go(attention_tc_balanced_kernel<8>);
  } else {
    st = go(attention_tc_balanced_kernel<16>);
  }
  if (st != BM_OK) return st;
  if (const int launch_status = launch_kernel("balanced_combine_kernel", balanced_combine_kernel,
                                              dim3(dim3(a.group, ctas)), dim3(kCombineThreads),
                                              static_cast<size_t>(ctas) * sizeof(float), stream, nullptr, a)) {
    return launch_status;
  }
  return check_launch("bm_decode_attention (combine)");
}

}  // namespace attn
}  // namespace bm
