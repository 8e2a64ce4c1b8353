// Tensor-core GEMMs for sm_100a: tcgen05.mma with operands staged by TMA and
// fp32 accumulators in tensor memory (TMEM); bf16 in, bf16 out.
//
//   bm_gemm_swiglu: out[R][F] = silu(x · w_gate) * (x · w_up)
//     the FFN front half of src/execution_engine.cu:122-124 (two launch_gemm
//     calls, then launch_swiglu) as one kernel: the gate and up products never
//     leave the SM, the SwiGLU runs in the epilogue.
//   bm_gemm: c[M][N] = a · b, the GEMM of src/kernels.cu:83-121 (launch_gemm).
// A operand [rows][K] row-major (K contiguous); weights [K][N] row-major (N
// contiguous), the layout launch_gemm's B has (include/kernels.cuh:20).
//
// One persistent CTA per SM walks output tiles of 128 rows x 256 accumulator
// columns (SwiGLU: 128 gate + 128 up columns of the same 128 outputs; plain:
// 256 outputs). Six warps:
//   warp 0     TMA producer: per 64-wide K step, one 128x64 A box and four 64x64
//              weight boxes (128-byte swizzle) into a 4-stage shared-memory ring;
//   warp 1     owns the TMEM allocation (512 columns: two accumulators); one
//              thread issues tcgen05.mma (M=128, N=256, K=16; A K-major, B
//              MN-major) and commits each stage back to the producer and each
//              finished accumulator to the epilogue;
//   warps 2-5  epilogue: tcgen05.ld of their 32 TMEM lanes (one row each),
//              SwiGLU or conversion, 16-byte stores; the accumulator is handed
//              back so the next tile's MMAs overlap this tile's epilogue.
// Every wait on an mbarrier is bounded in time: past kWaitLimitNs the CTA sets
// BM_DEVERR_TIMEOUT in the status word, lets its copies and MMAs in flight land
// (again bounded), frees its TMEM and returns.
#include <cuda.h>

#include <algorithm>

#include "bm_common.cuh"
#include "bm_host.h"
#include "bm_tc.cuh"
#include "bm_tma.h"

namespace bm {
namespace gemm {

using namespace bm::tc;

constexpr int kBlockM = 128;       // output rows per tile (TMEM lanes)
constexpr int kBlockN = 256;       // accumulator columns per tile (MMA N)
constexpr int kBlockK = 64;        // K per stage: one 128-byte swizzle row of bf16
constexpr int kStages = 4;
constexpr int kBoxN = 64;          // weight box width (128 bytes of bf16)
constexpr int kABytes = kBlockM * kBlockK * 2;                 // 16 KB
constexpr int kBBoxBytes = kBlockK * kBoxN * 2;                // 8 KB
constexpr int kBBytes = kBBoxBytes * (kBlockN / kBoxN);        // 32 KB
constexpr int kStageBytes = kABytes + kBBytes;                 // 48 KB
constexpr int kThreads = 192;
constexpr int kEpilogueThreads = 128;
constexpr int kTmemCols = 2 * kBlockN;
constexpr int kSmemBytes = kStages * kStageBytes + 1024 /* alignment slack */ + 256 /* barriers */;
constexpr uint64_t kWaitLimitNs = 2000000000ull;   // 2 s: far above any legitimate wait
constexpr uint64_t kDrainLimitNs = 200000000ull;   // 0.2 s for copies in flight at exit
constexpr int kGroupM = 16;        // tile order: 16 row blocks advance together (L2 reuse)

struct Args {
  void* out;
  int64_t rows;
  int n;          // output columns
  int k;
  int m_blocks, n_blocks, k_steps;
  int32_t* status;
};


// Instruction descriptor: fp32 accumulator, bf16 A and B, A K-major, B
// MN-major, N = kBlockN, M = kBlockM.
constexpr uint32_t kInstrDesc = instr_desc_bf16(false, true, kBlockN, kBlockM);

__device__ __forceinline__ float silu(float g) { return __fdividef(g, 1.0f + exp2f(g * -1.4426950408889634f)); }

// Tile t -> (row block, column block): kGroupM row blocks advance through the
// column blocks together, so concurrently running CTAs share A and B tiles in L2.
__device__ __forceinline__ void tile_coords(const Args& a, int t, int* mb, int* nb) {
  const int per_group = kGroupM * a.n_blocks;
  const int group = t / per_group;
  const int first_m = group * kGroupM;
  const int group_m = min(a.m_blocks - first_m, kGroupM);
  const int r = t - group * per_group;
  *mb = first_m + r % group_m;
  *nb = r / group_m;
}

// SWIGLU: tb0 = w_gate, tb1 = w_up, 128 output columns per tile.
// Otherwise tb0 = tb1 = b, 256 output columns per tile.
template <bool SWIGLU>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb0,
                   const __grid_constant__ CUtensorMap tb1, const Args a) {
  grid_dependency_wait();
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // stages 1024-byte aligned (the swizzle atom); barriers after them
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                         ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* mma_done = acc_empty + 2;
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_s + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = a.m_blocks * a.n_blocks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], kEpilogueThreads);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_base_s, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_s;

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer ----------------
    int stage = 0;
    uint32_t phase = 0;
    uint32_t last_parity[kStages];
    bool filled[kStages];
    for (int s = 0; s < kStages; ++s) filled[s] = false;
    bool ok = true;
    for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
      int mb, nb;
      tile_coords(a, t, &mb, &nb);
      const int m0 = mb * kBlockM;
      const int n0 = nb * (SWIGLU ? kBlockN / 2 : kBlockN);
      for (int ks = 0; ks < a.k_steps; ++ks) {
        if (!wait_phase(&empty[stage], phase ^ 1u, abort_flag, a.status, kWaitLimitNs, true)) {
          ok = false;
          break;
        }
        unsigned char* sa = smem + stage * kStageBytes;
        unsigned char* sb = sa + kABytes;
        mbar_expect_tx(&full[stage], kStageBytes);
        const int k0 = ks * kBlockK;
        tma_load_2d(sa, &ta, &full[stage], k0, m0);
        if (SWIGLU) {
          tma_load_2d(sb, &tb0, &full[stage], n0, k0);
          tma_load_2d(sb + kBBoxBytes, &tb0, &full[stage], n0 + kBoxN, k0);
          tma_load_2d(sb + 2 * kBBoxBytes, &tb1, &full[stage], n0, k0);
          tma_load_2d(sb + 3 * kBBoxBytes, &tb1, &full[stage], n0 + kBoxN, k0);
        } else {
#pragma unroll
          for (int j = 0; j < kBlockN / kBoxN; ++j) tma_load_2d(sb + j * kBBoxBytes, &tb0, &full[stage], n0 + j * kBoxN, k0);
        }
        filled[stage] = true;
        last_parity[stage] = phase;
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    // let every copy in flight land before the CTA can exit
    for (int s = 0; s < kStages; ++s) {
      if (filled[s]) wait_phase(&full[s], last_parity[s], abort_flag, a.status, kDrainLimitNs, false);
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer ----------------
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool issued = false, ok = true;
    for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
      if (!wait_phase(&acc_empty[acc], acc_phase ^ 1u, abort_flag, a.status, kWaitLimitNs, true)) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kBlockN);
      for (int ks = 0; ks < a.k_steps; ++ks) {
        if (!wait_phase(&full[stage], phase, abort_flag, a.status, kWaitLimitNs, true)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + stage * kStageBytes);
        const uint32_t sb = sa + kABytes;
#pragma unroll
        for (int kk = 0; kk < kBlockK / 16; ++kk) {
          // A: K-major, 16 K-elements = 32 bytes further along each swizzled row
          const uint64_t a_desc = smem_desc(sa + kk * 32, 16, 1024);
          // B: MN-major, 16 K-rows = two 8-row groups of 1024 bytes further on;
          // 64-column blocks kBBoxBytes apart
          const uint64_t b_desc = smem_desc(sb + kk * 2048, kBBoxBytes, 1024);
          mma_bf16(d_tmem, a_desc, b_desc, kInstrDesc, (ks | kk) != 0 ? 1u : 0u);
        }
        issued = true;
        mma_commit(&empty[stage]);  // the stage is free once these MMAs have read it
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
      mma_commit(&acc_full[acc]);  // the accumulator is complete once every MMA so far has finished
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (issued) {  // no MMA may still write TMEM when it is freed
      mma_commit(mma_done);
      wait_phase(mma_done, 0, abort_flag, a.status, kDrainLimitNs, false);
    }
  } else if (warp >= 2) {
    // ---------------- epilogue ----------------
    const int quarter = warp & 3;  // TMEM lanes [32 * quarter, 32 * quarter + 32) belong to this warp
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    int acc = 0;
    uint32_t acc_phase = 0;
    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out);
    for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
      // one lane waits; the shuffle hands its verdict to the warp and reconverges
      // it for the warp-wide tcgen05.ld
      int ok = 1;
      if (lane == 0) ok = wait_phase(&acc_full[acc], acc_phase, abort_flag, a.status, kWaitLimitNs, true);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      int mb, nb;
      tile_coords(a, t, &mb, &nb);
      const int64_t row = static_cast<int64_t>(mb) * kBlockM + quarter * 32 + lane;
      const uint32_t tbase = tmem_base + lane_addr + static_cast<uint32_t>(acc * kBlockN);
      constexpr int kOutCols = SWIGLU ? kBlockN / 2 : kBlockN;
      const int n0 = nb * kOutCols;
#pragma unroll 1
      for (int c = 0; c < kOutCols; c += 32) {
        uint32_t g[32];
        float o[32];
        tmem_load32(tbase + c, g);
        if (SWIGLU) {
          uint32_t u[32];
          tmem_load32(tbase + kOutCols + c, u);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = silu(__uint_as_float(g[i])) * __uint_as_float(u[i]);
        } else {
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __uint_as_float(g[i]);
        }
        if (row < a.rows) {
          __nv_bfloat16* dst = out + row * a.n + n0 + c;
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            if (n0 + c + v * 8 < a.n) st_plain(dst + v * 8, pack16<__nv_bfloat16>(o + v * 8));
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
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


// ---------------------------------------------------------------------------
// CTA-pair variant for row counts above one row block: a cluster of two CTAs on
// two SMs computes a 256-row tile with tcgen05.mma.cta_group::2 (M=256, N=256).
// Each CTA loads its own 128 rows of A and its own half of B (SwiGLU: the leader
// the 128 gate columns, the peer the 128 up columns; plain: 128 columns each), so
// each SM reads 8 KB of operands per 128 cycles of math instead of 12 KB per 64,
// and each CTA's accumulator holds gate and up of its own 128 rows. The leader's
// producer posts the transaction bytes of both CTAs on the leader's full
// barrier; both CTAs' copies count on it; one thread of the leader issues the
// MMAs and commits to the barriers of both CTAs; both epilogues hand the
// accumulator back through the leader's barrier. No load uses multicast.

#ifndef BM_GEMM_PAIR_STAGES
#define BM_GEMM_PAIR_STAGES 6  // 6 x 32 KB (7 fit; measured no faster)
#endif
#ifndef BM_GEMM_PAIR_GROUP_M
// tile order: this many pair row blocks advance together (L2 reuse); 16 measured 2.5%
// faster than 8 on the 70B FFN (16384 x 8192 -> 28672) and no slower on the 8B one
#define BM_GEMM_PAIR_GROUP_M 16
#endif
#ifndef BM_GEMM_WIDE_SWIGLU
#define BM_GEMM_WIDE_SWIGLU 1  // bm_gemm_swiglu over more than one row block: the wide tile below
#endif
constexpr int kPairStages = BM_GEMM_PAIR_STAGES;
constexpr int kPairStageBytes = kABytes + kBBytes / 2;           // 16 KB of A + 16 KB of B: 32 KB
constexpr int kPairSmemBytes = kPairStages * kPairStageBytes + 1024 + 256;
static_assert(kPairSmemBytes <= 232448, "shared memory per CTA");
constexpr int kGroupMPair = BM_GEMM_PAIR_GROUP_M;
constexpr uint32_t kPairInstrDesc = instr_desc_bf16(false, true, kBlockN, 2 * kBlockM);

__device__ __forceinline__ void pair_tile_coords(const Args& a, int t, int* mb, int* nb) {
  const int per_group = kGroupMPair * a.n_blocks;
  const int group = t / per_group;
  const int first_m = group * kGroupMPair;
  const int group_m = min(a.m_blocks - first_m, kGroupMPair);
  const int r = t - group * per_group;
  *mb = first_m + r % group_m;
  *nb = r / group_m;
}

template <bool SWIGLU>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_tc_pair_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb0,
                        const __grid_constant__ CUtensorMap tb1, const Args a) {
  grid_dependency_wait();
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                         ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kPairStages * kPairStageBytes);
  uint64_t* empty = full + kPairStages;
  uint64_t* acc_full = empty + kPairStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* mma_done = acc_empty + 2;
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_s + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0: the leader, which issues the MMAs
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int tiles = a.m_blocks * a.n_blocks;
  constexpr int kOutCols = SWIGLU ? kBlockN / 2 : kBlockN;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 2 * kEpilogueThreads);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc_pair(tmem_base_s, kTmemCols);
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers exist before any copy or arrival reaches them
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_s;

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    int stage = 0;
    uint32_t phase = 0;
    uint32_t last_parity[kPairStages];
    bool filled[kPairStages];
    for (int s = 0; s < kPairStages; ++s) filled[s] = false;
    bool ok = true;
    const CUtensorMap* tb = (SWIGLU && !leader) ? &tb1 : &tb0;
    for (int t = pair; t < tiles && ok; t += npairs) {
      int mb, nb;
      pair_tile_coords(a, t, &mb, &nb);
      const int m0 = mb * 2 * kBlockM + static_cast<int>(rank) * kBlockM;
      const int n0 = SWIGLU ? nb * kOutCols : nb * kOutCols + static_cast<int>(rank) * (kBlockN / 2);
      for (int ks = 0; ks < a.k_steps; ++ks) {
        if (!wait_phase(&empty[stage], phase ^ 1u, abort_flag, a.status, kWaitLimitNs, true)) {
          ok = false;
          break;
        }
        unsigned char* sa = smem + stage * kPairStageBytes;
        unsigned char* sb = sa + kABytes;
        const uint32_t bar = cluster_addr(&full[stage], 0);
        if (leader) mbar_expect_tx(&full[stage], 2 * kPairStageBytes);
        const int k0 = ks * kBlockK;
        tma_load_2d_pair(sa, &ta, bar, k0, m0);
        tma_load_2d_pair(sb, tb, bar, n0, k0);
        tma_load_2d_pair(sb + kBBoxBytes, tb, bar, n0 + kBoxN, k0);
        filled[stage] = true;
        last_parity[stage] = phase;
        if (++stage == kPairStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    if (leader) {  // every copy of the pair counts on the leader's barriers: let them land
      for (int s = 0; s < kPairStages; ++s) {
        if (filled[s]) wait_phase(&full[s], last_parity[s], abort_flag, a.status, kDrainLimitNs, false);
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer (leader) ----------------
    bool issued = false;
    if (leader) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = pair; t < tiles && ok; t += npairs) {
        if (!wait_phase(&acc_empty[acc], acc_phase ^ 1u, abort_flag, a.status, kWaitLimitNs, true)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kBlockN);
        for (int ks = 0; ks < a.k_steps; ++ks) {
          if (!wait_phase(&full[stage], phase, abort_flag, a.status, kWaitLimitNs, true)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * kPairStageBytes);
          const uint32_t sb = sa + kABytes;
#pragma unroll
          for (int kk = 0; kk < kBlockK / 16; ++kk) {
            const uint64_t a_desc = smem_desc(sa + kk * 32, 16, 1024);
            const uint64_t b_desc = smem_desc(sb + kk * 2048, kBBoxBytes, 1024);
            mma_bf16_pair(d_tmem, a_desc, b_desc, kPairInstrDesc, (ks | kk) != 0 ? 1u : 0u);
          }
          issued = true;
          mma_commit_pair(&empty[stage], 0x3);  // both CTAs may refill this stage
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit_pair(&acc_full[acc], 0x3);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // no pair MMA may still write either CTA's TMEM when it is freed: the leader
      // drains them here, and the cluster barrier at the end holds the peer back
      if (issued) {
        mma_commit_pair(mma_done, 0x3);
        wait_phase(mma_done, 0, abort_flag, a.status, kDrainLimitNs, false);
      }
    }
  } else if (warp >= 2) {
    // ---------------- epilogue (both CTAs) ----------------
    const int quarter = warp & 3;
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    int acc = 0;
    uint32_t acc_phase = 0;
    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out);
    for (int t = pair; t < tiles; t += npairs) {
      int ok = 1;
      if (lane == 0) ok = wait_phase(&acc_full[acc], acc_phase, abort_flag, a.status, kWaitLimitNs, true);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      int mb, nb;
      pair_tile_coords(a, t, &mb, &nb);
      const int64_t row = static_cast<int64_t>(mb) * 2 * kBlockM + rank * kBlockM + quarter * 32 + lane;
      const uint32_t tbase = tmem_base + lane_addr + static_cast<uint32_t>(acc * kBlockN);
      const int n0 = nb * kOutCols;
#pragma unroll 1
      for (int c = 0; c < kOutCols; c += 32) {
        uint32_t g[32];
        float o[32];
        tmem_load32(tbase + c, g);
        if (SWIGLU) {
          uint32_t u[32];
          tmem_load32(tbase + kOutCols + c, u);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = silu(__uint_as_float(g[i])) * __uint_as_float(u[i]);
        } else {
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __uint_as_float(g[i]);
        }
        if (row < a.rows) {
          __nv_bfloat16* dst = out + row * a.n + n0 + c;
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            if (n0 + c + v * 8 < a.n) st_plain(dst + v * 8, pack16<__nv_bfloat16>(o + v * 8));
          }
        }
      }
      tc_fence_before();
      mbar_arrive_cluster(cluster_addr(&acc_empty[acc], 0));
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // neither CTA leaves while the other may still reach its shared memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

// Wide SwiGLU tiles for CTA pairs: each pair computes 256 rows x 256 outputs with
// two MMAs per K slice (M=256, N=256: gate, then up) that share the A slice, so
// every SM reads 48 KB of operands per 256 cycles of math where the tile above
// reads 32 KB per 128 (a quarter fewer L2 -> shared-memory bytes per FLOP; the
// tile above waits on arriving operands about 40 % of the time). Each CTA loads
// its 128 rows of A and its half (128 columns) of both weights' 256; the two
// accumulators fill all 512 TMEM columns, so a tile's MMAs wait for the previous
// tile's epilogue, which eight warps (two per TMEM lane quarter, one per column
// half) drain. Four stages of 48 KB.
constexpr int kWideStages = 4;
constexpr int kWideHalfB = kBBoxBytes * 2;                        // 128 weight columns x 64 K: 16 KB
constexpr int kWideStageBytes = kABytes + 2 * kWideHalfB;         // 48 KB
constexpr int kWideSmemBytes = kWideStages * kWideStageBytes + 1024 + 256;
static_assert(kWideSmemBytes <= 232448, "shared memory per CTA");
constexpr int kWideOut = 256;                                     // output columns per tile
constexpr int kWideEpilogueThreads = 256;
constexpr int kWideThreads = 64 + kWideEpilogueThreads;

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kWideThreads, 1)
    gemm_tc_wide_swiglu_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tg,
                               const __grid_constant__ CUtensorMap tu, const Args a) {
  grid_dependency_wait();
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                         ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kWideStages * kWideStageBytes);
  uint64_t* empty = full + kWideStages;
  uint64_t* acc_full = empty + kWideStages;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* mma_done = acc_empty + 1;
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_s + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0: the leader, which issues the MMAs
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int tiles = a.m_blocks * a.n_blocks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kWideStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 2 * kWideEpilogueThreads);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc_pair(tmem_base_s, kTmemCols);
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers exist before any copy or arrival reaches them
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_s;

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    int stage = 0;
    uint32_t phase = 0;
    uint32_t last_parity[kWideStages];
    bool filled[kWideStages];
    for (int s = 0; s < kWideStages; ++s) filled[s] = false;
    bool ok = true;
    for (int t = pair; t < tiles && ok; t += npairs) {
      int mb, nb;
      pair_tile_coords(a, t, &mb, &nb);
      const int m0 = mb * 2 * kBlockM + static_cast<int>(rank) * kBlockM;
      const int nh = nb * kWideOut + static_cast<int>(rank) * (kWideOut / 2);  // this CTA's half of the columns
      for (int ks = 0; ks < a.k_steps; ++ks) {
        if (!wait_phase(&empty[stage], phase ^ 1u, abort_flag, a.status, kWaitLimitNs, true)) {
          ok = false;
          break;
        }
        unsigned char* sa = smem + stage * kWideStageBytes;
        unsigned char* sg = sa + kABytes;
        unsigned char* su = sg + kWideHalfB;
        const uint32_t bar = cluster_addr(&full[stage], 0);
        if (leader) mbar_expect_tx(&full[stage], 2 * kWideStageBytes);
        const int k0 = ks * kBlockK;
        tma_load_2d_pair(sa, &ta, bar, k0, m0);
        tma_load_2d_pair(sg, &tg, bar, nh, k0);
        tma_load_2d_pair(sg + kBBoxBytes, &tg, bar, nh + kBoxN, k0);
        tma_load_2d_pair(su, &tu, bar, nh, k0);
        tma_load_2d_pair(su + kBBoxBytes, &tu, bar, nh + kBoxN, k0);
        filled[stage] = true;
        last_parity[stage] = phase;
        if (++stage == kWideStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    if (leader) {  // every copy of the pair counts on the leader's barriers: let them land
      for (int s = 0; s < kWideStages; ++s) {
        if (filled[s]) wait_phase(&full[s], last_parity[s], abort_flag, a.status, kDrainLimitNs, false);
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer (leader) ----------------
    bool issued = false;
    if (leader) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = pair; t < tiles && ok; t += npairs) {
        if (!wait_phase(acc_empty, acc_phase ^ 1u, abort_flag, a.status, kWaitLimitNs, true)) break;
        tc_fence_after();
        for (int ks = 0; ks < a.k_steps; ++ks) {
          if (!wait_phase(&full[stage], phase, abort_flag, a.status, kWaitLimitNs, true)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * kWideStageBytes);
          const uint32_t sg = sa + kABytes;
          const uint32_t su = sg + kWideHalfB;
#pragma unroll
          for (int kk = 0; kk < kBlockK / 16; ++kk) {
            const uint64_t a_desc = smem_desc(sa + kk * 32, 16, 1024);
            const uint32_t acc = (ks | kk) != 0 ? 1u : 0u;
            mma_bf16_pair(tmem_base, a_desc, smem_desc(sg + kk * 2048, kBBoxBytes, 1024), kPairInstrDesc, acc);
            mma_bf16_pair(tmem_base + kWideOut, a_desc, smem_desc(su + kk * 2048, kBBoxBytes, 1024),
                          kPairInstrDesc, acc);
          }
          issued = true;
          mma_commit_pair(&empty[stage], 0x3);  // both CTAs may refill this stage
          if (++stage == kWideStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit_pair(acc_full, 0x3);
        acc_phase ^= 1u;
      }
      // no pair MMA may still write either CTA's TMEM when it is freed: the leader
      // drains them here, and the cluster barrier at the end holds the peer back
      if (issued) {
        mma_commit_pair(mma_done, 0x3);
        wait_phase(mma_done, 0, abort_flag, a.status, kDrainLimitNs, false);
      }
    }
  } else if (warp >= 2) {
    // ---------------- epilogue (both CTAs, eight warps) ----------------
    const int quarter = warp & 3;             // the TMEM lanes this warp may read
    const int half = (warp - 2) >> 2;         // which 128 of the tile's 256 output columns
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    uint32_t acc_phase = 0;
    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out);
    for (int t = pair; t < tiles; t += npairs) {
      int ok = 1;
      if (lane == 0) ok = wait_phase(acc_full, acc_phase, abort_flag, a.status, kWaitLimitNs, true);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      int mb, nb;
      pair_tile_coords(a, t, &mb, &nb);
      const int64_t row = static_cast<int64_t>(mb) * 2 * kBlockM + rank * kBlockM + quarter * 32 + lane;
      const uint32_t tbase = tmem_base + lane_addr;
      const int n0 = nb * kWideOut;
#pragma unroll 1
      for (int c = half * (kWideOut / 2); c < (half + 1) * (kWideOut / 2); c += 32) {
        uint32_t g[32], u[32];
        float o[32];
        tmem_load32(tbase + c, g);
        tmem_load32(tbase + kWideOut + c, u);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = silu(__uint_as_float(g[i])) * __uint_as_float(u[i]);
        if (row < a.rows) {
          __nv_bfloat16* dst = out + row * a.n + n0 + c;
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            if (n0 + c + v * 8 < a.n) st_plain(dst + v * 8, pack16<__nv_bfloat16>(o + v * 8));
          }
        }
      }
      tc_fence_before();
      mbar_arrive_cluster(cluster_addr(acc_empty, 0));
      acc_phase ^= 1u;
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // neither CTA leaves while the other may still reach its shared memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Host side

int check_shapes(const char* what, int64_t rows, int64_t n, int64_t k, bm_dtype_t dtype) {
  if (dtype != BM_BF16) {
    return fail(BM_ERR_INVALID_ARGUMENT, "%s: bf16 only (the tensor-core path takes bf16 operands)", what);
  }
  if (rows < 0 || rows > (int64_t{1} << 31) - kBlockM) return fail(BM_ERR_INVALID_ARGUMENT, "%s: bad row count", what);
  if (n <= 0 || k <= 0 || n % 8 != 0 || k % 8 != 0 || n > (1 << 30) || k > (1 << 30)) {
    return fail(BM_ERR_INVALID_ARGUMENT, "%s: N and K must be positive multiples of 8 (16-byte rows)", what);
  }
  return BM_OK;
}

template <bool SWIGLU>
int run(const char* what, void* out, const void* x, const void* w0, const void* w1, int64_t rows, int n, int k,
        int32_t* d_status, void* stream) {
  if (!out || !x || !w0 || !w1) return fail(BM_ERR_INVALID_ARGUMENT, "%s: NULL pointer", what);
  if (!aligned16(out) || !aligned16(x) || !aligned16(w0) || !aligned16(w1)) {
    return fail(BM_ERR_INVALID_ARGUMENT, "%s: pointers must be 16-byte aligned", what);
  }
  if (rows == 0) return BM_OK;
  CUtensorMap ta, tb0, tb1;
  if (int st = make_tensor_map_bf16(&ta, x, static_cast<uint64_t>(k), static_cast<uint64_t>(rows), kBlockK, kBlockM, what)) return st;
  if (int st = make_tensor_map_bf16(&tb0, w0, static_cast<uint64_t>(n), static_cast<uint64_t>(k), kBoxN, kBlockK, what)) return st;
  if (int st = make_tensor_map_bf16(&tb1, w1, static_cast<uint64_t>(n), static_cast<uint64_t>(k), kBoxN, kBlockK, what)) return st;
  Args a{};
  a.out = out;
  a.rows = rows;
  a.n = n;
  a.k = k;
  // more than one row block: CTA pairs with 256-row tiles; otherwise single CTAs
  const bool paired = rows > kBlockM && sm_count() >= 2;
  const int block_rows = paired ? 2 * kBlockM : kBlockM;
  a.m_blocks = static_cast<int>((rows + block_rows - 1) / block_rows);
  const bool wide = SWIGLU && paired && BM_GEMM_WIDE_SWIGLU;
  const int out_cols = wide ? kWideOut : SWIGLU ? kBlockN / 2 : kBlockN;
  a.n_blocks = (n + out_cols - 1) / out_cols;
  a.k_steps = (k + kBlockK - 1) / kBlockK;
  a.status = d_status;
  const int64_t tiles = static_cast<int64_t>(a.m_blocks) * a.n_blocks;
  if (tiles > (int64_t{1} << 31) - 1) return fail(BM_ERR_INVALID_ARGUMENT, "%s: too many tiles", what);
  if (wide) {
    const int grid = 2 * static_cast<int>(std::min<int64_t>(tiles, sm_count() / 2));
    auto kernel = gemm_tc_wide_swiglu_kernel;
    if (int st = allow_dynamic_smem(reinterpret_cast<const void*>(kernel), kWideSmemBytes, what)) return st;
    return launch_kernel(what, kernel, dim3(grid), dim3(kWideThreads), kWideSmemBytes, as_stream(stream), nullptr,
                         ta, tb0, tb1, a);
  }
  if (paired) {
    const int grid = 2 * static_cast<int>(std::min<int64_t>(tiles, sm_count() / 2));
    auto kernel = gemm_tc_pair_kernel<SWIGLU>;
    if (int st = allow_dynamic_smem(reinterpret_cast<const void*>(kernel), kPairSmemBytes, what)) return st;
    if (const int launch_status = launch_kernel(what, kernel, dim3(grid), dim3(kThreads), kPairSmemBytes,
                                                as_stream(stream), nullptr, ta, tb0, tb1, a)) {
      return launch_status;
    }
    return check_launch(what);
  }
  const int grid = static_cast<int>(std::min<int64_t>(tiles, sm_count()));
  auto kernel = gemm_tc_kernel<SWIGLU>;
  if (int st = allow_dynamic_smem(reinterpret_cast<const void*>(kernel), kSmemBytes, what)) return st;
  if (const int launch_status = launch_kernel(what, kernel, dim3(grid), dim3(kThreads), kSmemBytes,
                                              as_stream(stream), nullptr, ta, tb0, tb1, a)) {
    return launch_status;
  }
  return check_launch(what);
}

}  // namespace gemm
}  // namespace bm

extern "C" int bm_gemm_swiglu(void* out, const void* x, const void* w_gate, const void* w_up, int64_t rows,
                              int32_t dim, int32_t hidden, bm_dtype_t dtype, int32_t* d_status, void* stream) {
  using namespace bm;
  const char* what = "bm_gemm_swiglu";
  if (dtype == BM_F32) {  // fp32 operands: CUDA cores, any shape (gemm_f32.cu)
    if (rows < 0 || rows > (int64_t{1} << 31) || dim < 0 || hidden < 0) {
      return fail(BM_ERR_INVALID_ARGUMENT, "%s: negative or too large size", what);
    }
    if (rows == 0 || hidden == 0) return BM_OK;
    if (!out || (dim > 0 && (!x || !w_gate || !w_up))) return fail(BM_ERR_INVALID_ARGUMENT, "%s: NULL pointer", what);
    return gemm_f32_swiglu(static_cast<float*>(out), static_cast<const float*>(x), static_cast<const float*>(w_gate),
                           static_cast<const float*>(w_up), rows, hidden, dim, as_stream(stream));
  }
  if (int st = gemm::check_shapes(what, rows, hidden, dim, dtype)) return st;
  return gemm::run<true>(what, out, x, w_gate, w_up, rows, hidden, dim, d_status, stream);
}

extern "C" int bm_gemm(void* c, const void* a, const void* b, int64_t m, int32_t n, int32_t k, bm_dtype_t dtype,
                       int32_t* d_status, void* stream) {
  using namespace bm;
  const char* what = "bm_gemm";
  if (dtype == BM_F32) {  // fp32 operands: CUDA cores, any shape (gemm_f32.cu)
    if (m < 0 || m > (int64_t{1} << 31) || n < 0 || k < 0) {
      return fail(BM_ERR_INVALID_ARGUMENT, "%s: negative or too large size", what);
    }
    if (m == 0 || n == 0) return BM_OK;
    if (!c || (k > 0 && (!a || !b))) return fail(BM_ERR_INVALID_ARGUMENT, "%s: NULL pointer", what);
    return gemm_f32(static_cast<float*>(c), static_cast<const float*>(a), static_cast<const float*>(b), m, n, k,
                    as_stream(stream));
  }
  if (int st = gemm::check_shapes(what, m, n, k, dtype)) return st;
  return gemm::run<false>(what, c, a, b, b, m, n, k, d_status, stream);
}

extern "C" int bm_gemm_shared_a(void* const* c, const void* a, const void* const* b, const int32_t* n,
                                int32_t count, int64_t m, int32_t k, bm_dtype_t dtype, int32_t* d_status,
                                void* stream) {
  using namespace bm;
  const char* what = "bm_gemm_shared_a";
  if (count < 1 || count > kMaxSharedA) return fail(BM_ERR_INVALID_ARGUMENT, "%s: count outside [1, 3]", what);
  if (!c || !b || !n) return fail(BM_ERR_INVALID_ARGUMENT, "%s: NULL array", what);
  if (m < 0 || m > (int64_t{1} << 31) || k < 0) return fail(BM_ERR_INVALID_ARGUMENT, "%s: negative or too large size", what);
  for (int o = 0; o < count; ++o) {
    if (n[o] < 0) return fail(BM_ERR_INVALID_ARGUMENT, "%s: negative width", what);
    if (m > 0 && n[o] > 0 && (!c[o] || (k > 0 && (!a || !b[o])))) {
      return fail(BM_ERR_INVALID_ARGUMENT, "%s: NULL pointer", what);
    }
  }
  if (dtype == BM_F32) {
    return gemm_f32_shared_a(reinterpret_cast<float* const*>(c), static_cast<const float*>(a),
                             reinterpret_cast<const float* const*>(b), n, count, m, k, as_stream(stream));
  }
  if (dtype != BM_BF16) return fail(BM_ERR_INVALID_ARGUMENT, "%s: bad dtype", what);
  for (int o = 0; o < count; ++o) {
    if (m == 0 || n[o] == 0) continue;  // an empty product: nothing to write
    if (int st = bm_gemm(c[o], a, b[o], m, n[o], k, dtype, d_status, stream)) return st;
  }
  return BM_OK;
}

extern "C" int bm_rmsnorm_gemm(void* const* c, const void* h, const void* d, const void* norm_weight, float eps,
                               void* residual_out, void* normed, const void* const* b, const int32_t* n,
                               int32_t count, int32_t swiglu, int64_t m, int32_t k, bm_dtype_t dtype,
                               int32_t* d_status, void* stream) {
  using namespace bm;
  const char* what = "bm_rmsnorm_gemm";
  if (!valid_dtype(dtype)) return fail(BM_ERR_INVALID_ARGUMENT, "%s: bad dtype", what);
  if (!c || !b || !n) return fail(BM_ERR_INVALID_ARGUMENT, "%s: NULL array", what);
  if (swiglu ? count != 2 : (count < 1 || count > kMaxSharedA)) {
    return fail(BM_ERR_INVALID_ARGUMENT, "%s: count must be 2 with swiglu, else 1 to 3", what);
  }
  if (m < 0 || m > (int64_t{1} << 31) || k <= 0) return fail(BM_ERR_INVALID_ARGUMENT, "%s: bad size", what);
  if (swiglu && n[0] != n[1]) return fail(BM_ERR_INVALID_ARGUMENT, "%s: gate and up widths differ", what);
  for (int o = 0; o < count; ++o) {
    if (n[o] < 0) return fail(BM_ERR_INVALID_ARGUMENT, "%s: negative width", what);
    if (m > 0 && n[o] > 0 && (!b[o] || ((o == 0 || !swiglu) && !c[o]))) {
      return fail(BM_ERR_INVALID_ARGUMENT, "%s: NULL pointer", what);
    }
  }
  if (m == 0) return BM_OK;
  if (!h || !norm_weight || !normed) return fail(BM_ERR_INVALID_ARGUMENT, "%s: NULL pointer", what);
  const size_t row_bytes = static_cast<size_t>(k) * dtype_size(dtype), bytes = row_bytes * static_cast<size_t>(m);
  auto overlaps = [bytes](const void* x, const void* y) {
    const char *p = static_cast<const char*>(x), *q = static_cast<const char*>(y);
    return x != nullptr && y != nullptr && p < q + bytes && q < p + bytes;
  };
  if (overlaps(residual_out, h) || overlaps(residual_out, d)) {
    return fail(BM_ERR_INVALID_ARGUMENT, "%s: residual_out overlaps h or d", what);
  }
  if (dtype == BM_F32) {
    return gemm_f32_norm(reinterpret_cast<float* const*>(c), static_cast<const float*>(h),
                         static_cast<const float*>(d), static_cast<const float*>(norm_weight), eps,
                         static_cast<float*>(residual_out), static_cast<float*>(normed),
                         reinterpret_cast<const float* const*>(b), n, count, swiglu != 0, m, k, as_stream(stream));
  }
  // bf16: the norm (with the add) into `normed`, then the tensor-core products
  int st;
  if (d != nullptr && residual_out != nullptr) {
    const cudaError_t err = cudaMemcpyAsync(residual_out, h, bytes, cudaMemcpyDeviceToDevice, as_stream(stream));
    if (err != cudaSuccess) return fail(BM_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
    st = bm_add_rmsnorm(residual_out, d, norm_weight, normed, m, k, eps, dtype, stream);
  } else if (d != nullptr) {
    st = bm_add(normed, h, d, m * static_cast<int64_t>(k), dtype, stream);
    if (st == BM_OK) st = bm_rmsnorm(normed, normed, norm_weight, m, k, eps, k, k, dtype, stream);
  } else {
    st = bm_rmsnorm(normed, h, norm_weight, m, k, eps, k, k, dtype, stream);
  }
  if (st != BM_OK) return st;
  if (swiglu) return bm_gemm_swiglu(c[0], normed, b[0], b[1], m, k, n[0], dtype, d_status, stream);
  return bm_gemm_shared_a(c, normed, b, n, count, m, k, dtype, d_status, stream);
}
