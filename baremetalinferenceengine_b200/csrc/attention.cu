// Decode attention over the static KV cache: one query token per entry, GQA.
//
// Reference semantics (src/kernels.cu:225-264): for one token and each head h,
//   scores[j] = dot(q[h], k_cache[h][j]) * rsqrt(head_dim), j < seq_len;
//   w = softmax(scores);  out[h][d] = sum_j w[j] * v_cache[h][j][d]
// as three launches (scores, softmax, mix), one block per head, fp32, batch 1.
//
// Here a batch of queries (query b reads cache sequence seq_ids[b] over positions
// [0, lens[b])) runs in one launch, q head h reading kv head h / G where
// G = num_q_heads / num_kv_heads (GQA), fp32 or bf16 cache. The sequence is cut
// into splits of S positions; one CTA of 128 threads takes (query, kv head,
// split) and processes it in tiles of 128 positions:
//   scores: thread t dots position t's K row (16-byte loads) with the G queries
//           of the group, held pre-scaled (by log2(e) / sqrt(head_dim)) in
//           shared memory;
//   softmax: running max and sum per query, base-2 exponentials (exp2f), tile
//           maxima and sums by warp shuffles plus a shared-memory pass;
//   mix:    warp w takes positions w, w+4, ...; lane l owns head_dim/32
//           dimensions (contiguous, one vector load, when head_dim is a
//           multiple of 32) and accumulates p * V for the G queries.
// The four warps' accumulators are summed through shared memory at the end.
// With one split the CTA writes the normalised output; with several it writes
// (max, sum, unnormalised output) per query to the workspace and
// attention_combine_kernel merges the splits.
#include "attention_kernels.cuh"

namespace bm {
namespace attn {

#ifndef BM_ATTN_BALANCED
#define BM_ATTN_BALANCED 1  // bf16 head_dim 128: the balanced persistent kernel when it applies
#endif
#ifndef BM_ATTN_STAGED_MIN_TILES
#define BM_ATTN_STAGED_MIN_TILES 4
#endif
// Splits of the TMA-fed kernels hold at least this many 128-position tiles.
constexpr int kStagedMinTiles = BM_ATTN_STAGED_MIN_TILES;
// Splits of the CUDA-core kernel hold at least two: a sequence of one or two tiles
// runs whole in one CTA rather than paying a second launch to merge its halves.
constexpr int kCudaCoreMinTiles = 2;

// min_tiles: the fewest tiles a split may hold (the tensor-core kernel pays a
// fixed start-up per CTA, so its splits keep at least four tiles). The CUDA-core
// kernel fits several CTAs on an SM: its plan aims at four CTAs per SM. The staged
// kernels (tensor-core and TMA-fed, min_tiles kStagedMinTiles) hold one CTA per SM
// and pay their start-up again in every wave, so with fewer pairs than SMs theirs
// aims at one wave (at most one CTA per SM); with more, many short CTAs keep the last
// wave's idle tail small, as on CUDA cores.
void plan_splits(int64_t pairs, int max_len, int sms, int* splits, int* split_len, int min_tiles = 1) {
  const int tiles = (max_len + kThreads - 1) / kThreads;
  const int64_t want = min_tiles >= kStagedMinTiles && pairs < sms
                           ? std::max<int64_t>(1, sms / pairs)
                           : std::max<int64_t>(1, (static_cast<int64_t>(sms) * 4 + pairs - 1) / pairs);
  const int n = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, tiles / std::max(min_tiles, 1))));
  const int tiles_per_split = (tiles + n - 1) / n;
  *split_len = tiles_per_split * kThreads;
  *splits = (tiles + tiles_per_split - 1) / tiles_per_split;
}

size_t workspace_bytes(int64_t batch, int hkv, int group, int hd, int splits) {
  return splits <= 1 ? 0 : static_cast<size_t>(batch) * hkv * splits * group * (hd + 2) * sizeof(float);
}

int check_args(const char* what, int64_t batch, int hq, int hkv, int hd, int max_seq, int num_seqs, int max_len,
               bm_dtype_t dtype) {
  if (!valid_dtype(dtype)) return fail(BM_ERR_INVALID_ARGUMENT, "%s: bad dtype", what);
  if (batch < 0 || batch > 65535) return fail(BM_ERR_INVALID_ARGUMENT, "%s: batch outside [0, 65535]", what);
  if (hq <= 0 || hkv <= 0 || hq % hkv != 0 || hq / hkv > kMaxGroup || hkv > 65535) {
    return fail(BM_ERR_INVALID_ARGUMENT, "%s: need num_q_heads a multiple of num_kv_heads, at most %d per kv head",
                what, kMaxGroup);
  }
  if (hd <= 0 || hd > kMaxHeadDim || (hd * dtype_size(dtype)) % 16 != 0) {
    return fail(BM_ERR_INVALID_ARGUMENT, "%s: head_dim rows must be whole 16-byte vectors, head_dim <= %d", what,
                kMaxHeadDim);
  }
  if (max_seq <= 0 || num_seqs <= 0) return fail(BM_ERR_INVALID_ARGUMENT, "%s: bad max_seq or num_seqs", what);
  if (max_len <= 0 || max_len > max_seq) return fail(BM_ERR_INVALID_ARGUMENT, "%s: max_len outside [1, max_seq]", what);
  return BM_OK;
}


}  // namespace attn

using namespace attn;


namespace {

// The call's sizes and pointers as the kernels take them (no plan yet).
AttnArgs fill_args(void* out, const void* q, const void* k_cache, const void* v_cache, const int32_t* seq_ids,
                   const int32_t* lens, int32_t len0, int32_t max_len, int64_t batch, int32_t hq, int32_t hkv,
                   int32_t hd, int32_t max_seq, int32_t num_seqs, float scale, int32_t* d_status) {
  if (!(scale > 0.f)) scale = 1.0f / sqrtf(static_cast<float>(hd));
  AttnArgs a{};
  a.out = out;
  a.q = q;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.seq_ids = seq_ids;
  a.lens = lens;
  a.len0 = len0;
  a.batch = batch;
  a.hq = hq;
  a.hkv = hkv;
  a.hd = hd;
  a.group = hq / hkv;
  a.max_seq = max_seq;
  a.num_seqs = num_seqs;
  a.max_len = max_len;
  a.qscale = scale * 1.4426950408889634f;  // scores in base 2: exp(x) = exp2(x * log2(e))
  a.status = d_status;
  return a;
}

int check_call(const char* what, void* out, const void* q, const void* k_cache, const void* v_cache, int64_t batch,
               int32_t hq, int32_t hkv, int32_t hd, int32_t max_seq, int32_t num_seqs, int32_t max_len,
               bm_dtype_t dtype) {
  if (int st = check_args(what, batch, hq, hkv, hd, max_seq, num_seqs, max_len, dtype)) return st;
  if (batch == 0) return BM_OK;
  if (!out || !q || !k_cache || !v_cache) return fail(BM_ERR_INVALID_ARGUMENT, "%s: NULL pointer", what);
  const int es = dtype_size(dtype);
  if (!aligned16(k_cache) || !aligned16(v_cache) || (hd * es) % 16 != 0) {
    return fail(BM_ERR_INVALID_ARGUMENT, "%s: caches must be 16-byte aligned", what);
  }
  return BM_OK;
}

// CTAs of the balanced kernel: one per SM, no more than there are tiles.
int balanced_ctas(const AttnArgs& a, int32_t max_len) {
  const int64_t tiles = a.batch * a.hkv * ((max_len + kThreads - 1) / kThreads);
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(sm_count(), tiles)));
}

// Fewest tiles a split of the per-pair grid holds on the path these arguments take.
int grid_min_tiles(const AttnArgs& a, bm_dtype_t dtype) {
  return tc_eligible(a, dtype) || f32_tma_eligible(a, dtype) ? kStagedMinTiles : kCudaCoreMinTiles;
}

// The per-(query, kv head, split) grid's plan: splits sized for the GPU, cut back
// to what the caller's workspace holds (maybe one split per pair).
void plan_grid(AttnArgs& a, void* workspace, size_t workspace_size, bm_dtype_t dtype) {
  const int64_t batch = a.batch;
  const int hkv = a.hkv, hd = a.hd, max_len = a.max_len;
  plan_splits(batch * hkv, max_len, sm_count(), &a.splits, &a.split_len, grid_min_tiles(a, dtype));
  const size_t need = workspace_bytes(batch, hkv, a.group, hd, a.splits);
  if (need > 0 && (workspace == nullptr || workspace_size < need)) {
    // Less scratch than the plan wants: as many splits as it holds (maybe one).
    const size_t per_split = workspace_bytes(batch, hkv, a.group, hd, 2) / 2;
    const int fit = workspace == nullptr ? 1 : static_cast<int>(std::min<size_t>(workspace_size / per_split, a.splits));
    const int tiles = (max_len + kThreads - 1) / kThreads;
    const int tiles_per_split = (tiles + std::max(fit, 1) - 1) / std::max(fit, 1);
    a.split_len = tiles_per_split * kThreads;
    a.splits = (tiles + tiles_per_split - 1) / tiles_per_split;
  }
  a.ws = a.splits > 1 ? static_cast<float*>(workspace) : nullptr;
}

}  // namespace

int decode_attention(void* out, const void* q, const void* k_cache, const void* v_cache, const int32_t* seq_ids,
                     const int32_t* lens, int32_t len0, int32_t max_len, int64_t batch, int32_t hq, int32_t hkv,
                     int32_t hd, int32_t max_seq, int32_t num_seqs, float scale, void* workspace,
                     size_t workspace_size, bm_dtype_t dtype, int32_t* d_status, void* stream) {
  const char* what = "bm_decode_attention";
  if (int st = check_call(what, out, q, k_cache, v_cache, batch, hq, hkv, hd, max_seq, num_seqs, max_len, dtype)) {
    return st;
  }
  if (batch == 0) return BM_OK;
  AttnArgs a = fill_args(out, q, k_cache, v_cache, seq_ids, lens, len0, max_len, batch, hq, hkv, hd, max_seq,
                         num_seqs, scale, d_status);
  const bool tc = tc_eligible(a, dtype);
  cudaStream_t s = as_stream(stream);
  if (BM_ATTN_BALANCED && balanced_eligible(a, dtype) && workspace != nullptr &&
      reinterpret_cast<uintptr_t>(workspace) % 16 == 0) {
    const int ctas = balanced_ctas(a, max_len);
    if (workspace_size >= balanced_workspace_bytes(a.group, ctas)) {
      a.ws = static_cast<float*>(workspace);
      return launch_tc_balanced(a, ctas, s);
    }
  }
  plan_grid(a, workspace, workspace_size, dtype);
  if (tc) return launch_tc(a, s);
  if (f32_tma_eligible(a, dtype)) return launch_f32_tma(a, s);
  return dtype == BM_F32 ? launch_f32(a, s) : launch_bf16(a, s);
}

int rope_kv_decode_attention(void* out, void* q, const void* k, const void* v, const int32_t* positions,
                             const void* rope_table, int32_t table_len, const int32_t* seq_ids, void* k_cache,
                             void* v_cache, const int32_t* lens, int32_t max_len, int64_t batch, int32_t hq,
                             int32_t hkv, int32_t hd, int32_t max_seq, int32_t num_seqs, float scale, void* workspace,
                             size_t workspace_size, bm_dtype_t dtype, int32_t* d_status, void* stream) {
  const char* what = "bm_rope_kv_decode_attention";
  if (int st = check_call(what, out, q, k_cache, v_cache, batch, hq, hkv, hd, max_seq, num_seqs, max_len, dtype)) {
    return st;
  }
  if (batch == 0) return BM_OK;
  if (!k || !v || !positions || !lens || !rope_table) return fail(BM_ERR_INVALID_ARGUMENT, "%s: NULL pointer", what);
  if (hd % 2 != 0 || table_len <= 0 || reinterpret_cast<uintptr_t>(rope_table) % 8 != 0) {
    return fail(BM_ERR_INVALID_ARGUMENT, "%s: need an even head_dim and an 8-byte aligned table", what);
  }
  AttnArgs a = fill_args(out, q, k_cache, v_cache, seq_ids, lens, 0, max_len, batch, hq, hkv, hd, max_seq, num_seqs,
                         scale, d_status);
  if (tc_eligible(a, dtype) || f32_tma_eligible(a, dtype)) {
    // the staged kernels (head_dim 128) read the caches by TMA: the new rows go in first
    if (int st = bm_rope_kv_store(q, k, v, positions, 0, seq_ids, k_cache, v_cache, rope_table, table_len, 0.0,
                                  batch, hq, hkv, hd, max_seq, num_seqs, dtype, d_status, stream)) {
      return st;
    }
    return decode_attention(out, q, k_cache, v_cache, seq_ids, lens, 0, max_len, batch, hq, hkv, hd, max_seq,
                            num_seqs, scale, workspace, workspace_size, dtype, d_status, stream);
  }
  a.k_new = k;
  a.v_new = v;
  a.positions = positions;
  a.rope_table = static_cast<const float2*>(rope_table);
  a.rope_len = table_len;
  plan_grid(a, workspace, workspace_size, dtype);
  cudaStream_t s = as_stream(stream);
  return dtype == BM_F32 ? launch_f32_rope(a, s) : launch_bf16_rope(a, s);
}

int decode_attention_scratch_need(const void* q, const void* k_cache, const void* v_cache, int32_t max_len,
                                  int64_t batch, int32_t hq, int32_t hkv, int32_t hd, int32_t max_seq,
                                  int32_t num_seqs, bm_dtype_t dtype, size_t* grid_bytes, size_t* balanced_bytes) {
  const char* what = "bm_decode_attention_static_scratch";
  *grid_bytes = *balanced_bytes = 0;
  // the output pointer is not known here and not needed for the plan: q stands in
  if (int st = check_call(what, const_cast<void*>(q), q, k_cache, v_cache, batch, hq, hkv, hd, max_seq, num_seqs,
                          max_len, dtype)) {
    return st;
  }
  if (batch == 0) return BM_OK;
  const AttnArgs a = fill_args(nullptr, q, k_cache, v_cache, nullptr, nullptr, 0, max_len, batch, hq, hkv, hd,
                               max_seq, num_seqs, 0.f, nullptr);
  int splits = 1, split_len = 0;
  plan_splits(batch * hkv, max_len, sm_count(), &splits, &split_len, grid_min_tiles(a, dtype));
  *grid_bytes = workspace_bytes(batch, hkv, a.group, hd, splits);
  *balanced_bytes = BM_ATTN_BALANCED && balanced_eligible(a, dtype)
                        ? balanced_workspace_bytes(a.group, balanced_ctas(a, max_len))
                        : SIZE_MAX;
  return BM_OK;
}

size_t decode_attention_workspace(int64_t batch, int32_t hq, int32_t hkv, int32_t hd, int32_t max_len) {
  if (batch <= 0 || hkv <= 0 || hq % hkv != 0 || max_len <= 0) return 0;
  int splits = 1, split_len = 0;
  plan_splits(batch * hkv, max_len, sm_count(), &splits, &split_len);
  size_t bytes = workspace_bytes(batch, hkv, hq / hkv, hd, splits);
  // a bf16 cache may take the balanced path, which needs its records and partials
  // whenever a pair has more than one tile
  if (BM_ATTN_BALANCED && hd == 128 && hq / hkv <= kMaxGroup && batch <= kBalancedMaxBatch &&
      batch * hkv >= kBalancedMinPairs && max_len > kThreads) {
    bytes = std::max(bytes, balanced_workspace_bytes(hq / hkv, sm_count()));
  }
  return bytes;
}

}  // namespace bm

extern "C" int bm_decode_attention_workspace_size(int64_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                                                  int32_t head_dim, int32_t max_len, size_t* bytes_out) {
  if (!bytes_out) return bm::fail(BM_ERR_INVALID_ARGUMENT, "bm_decode_attention_workspace_size: NULL bytes_out");
  *bytes_out = bm::decode_attention_workspace(batch, num_q_heads, num_kv_heads, head_dim, max_len);
  return BM_OK;
}

extern "C" int bm_decode_attention(void* out, const void* q, const void* k_cache, const void* v_cache,
                                   const int32_t* seq_ids, const int32_t* lens, int32_t max_len, int64_t batch,
                                   int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, int32_t max_seq,
                                   int32_t num_seqs, float scale, void* workspace, size_t workspace_bytes,
                                   bm_dtype_t dtype, int32_t* d_status, void* stream) {
  if (!lens) return bm::fail(BM_ERR_INVALID_ARGUMENT, "bm_decode_attention: NULL lens");
  return bm::decode_attention(out, q, k_cache, v_cache, seq_ids, lens, 0, max_len, batch, num_q_heads, num_kv_heads,
                              head_dim, max_seq, num_seqs, scale, workspace, workspace_bytes, dtype, d_status, stream);
}

extern "C" int bm_rope_kv_decode_attention(void* out, void* q, const void* k, const void* v,
                                           const int32_t* positions, const void* rope_table, int32_t rope_table_len,
                                           const int32_t* seq_ids, void* k_cache, void* v_cache, const int32_t* lens,
                                           int32_t max_len, int64_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                                           int32_t head_dim, int32_t max_seq, int32_t num_seqs, float scale,
                                           void* workspace, size_t workspace_bytes, bm_dtype_t dtype,
                                           int32_t* d_status, void* stream) {
  return bm::rope_kv_decode_attention(out, q, k, v, positions, rope_table, rope_table_len, seq_ids, k_cache, v_cache,
                                      lens, max_len, batch, num_q_heads, num_kv_heads, head_dim, max_seq, num_seqs,
                                      scale, workspace, workspace_bytes, dtype, d_status, stream);
}
