// Batch-aware static KV cache: per-layer K/V buffers laid out
// [num_seqs][kv_heads][max_seq][head_dim] (the reference's include/kv_cache.h:37-40
// with its batch dimension used) and one length per sequence, where the
// reference keeps a single current_seq_pos_ (src/kv_cache.cu:38-47).
//
// append() is host bookkeeping: it gives each new token the next position of its
// sequence and uploads the (position, sequence) pairs from a pinned staging
// buffer into two device arrays that bm_rope_kv_store reads. An event guards
// the staging buffer, so an append never overwrites values a previous upload is
// still reading. The device arrays themselves are rewritten by every append, so
// appends and the kernels that read their arrays must share one stream (stream
// order keeps an upload behind the previous step's readers). Not thread-safe: one
// host thread drives one cache.
#include <algorithm>
#include <cstring>
#include <new>
#include <vector>

#include "bm_host.h"

struct bm_kv_cache {
  int32_t num_layers = 0, num_seqs = 0, kv_heads = 0, max_seq = 0, head_dim = 0, max_tokens = 0;
  bm_dtype_t dtype = BM_F32;
  std::vector<void*> keys, values;
  std::vector<int32_t> lens;
  int32_t* d_positions = nullptr;
  int32_t* d_seq_ids = nullptr;
  int32_t* h_staging = nullptr;  // pinned: [max_tokens] positions, then [max_tokens] sequence ids
  cudaEvent_t staging_free = nullptr;
};

namespace {

void release(bm_kv_cache* c) {
  for (void* p : c->keys) cudaFree(p);
  for (void* p : c->values) cudaFree(p);
  if (c->d_positions) cudaFree(c->d_positions);
  if (c->d_seq_ids) cudaFree(c->d_seq_ids);
  if (c->h_staging) cudaFreeHost(c->h_staging);
  if (c->staging_free) cudaEventDestroy(c->staging_free);
  delete c;
}

}  // namespace

extern "C" int bm_kv_cache_create(int32_t num_layers, int32_t num_seqs, int32_t num_kv_heads, int32_t max_seq,
                                  int32_t head_dim, int32_t max_tokens, bm_dtype_t dtype, bm_kv_cache_t** cache_out) {
  using namespace bm;
  if (!cache_out) return fail(BM_ERR_INVALID_ARGUMENT, "bm_kv_cache_create: NULL cache_out");
  *cache_out = nullptr;
  if (!valid_dtype(dtype)) return fail(BM_ERR_INVALID_ARGUMENT, "bm_kv_cache_create: bad dtype");
  if (num_layers <= 0 || num_seqs <= 0 || num_kv_heads <= 0 || max_seq <= 0 || head_dim <= 0 || max_tokens <= 0) {
    return fail(BM_ERR_INVALID_ARGUMENT, "bm_kv_cache_create: every size must be > 0");
  }
  auto* c = new (std::nothrow) bm_kv_cache;
  if (!c) return fail(BM_ERR_INVALID_ARGUMENT, "bm_kv_cache_create: out of host memory");
  c->num_layers = num_layers;
  c->num_seqs = num_seqs;
  c->kv_heads = num_kv_heads;
  c->max_seq = max_seq;
  c->head_dim = head_dim;
  c->max_tokens = max_tokens;
  c->dtype = dtype;
  c->lens.assign(num_seqs, 0);
  const size_t bytes = static_cast<size_t>(num_seqs) * num_kv_heads * max_seq * head_dim * dtype_size(dtype);
  cudaError_t err = cudaSuccess;
  for (int l = 0; l < num_layers && err == cudaSuccess; ++l) {
    void *k = nullptr, *v = nullptr;
    err = cudaMalloc(&k, bytes);
    if (err == cudaSuccess) c->keys.push_back(k);
    if (err == cudaSuccess) err = cudaMalloc(&v, bytes);
    if (err == cudaSuccess) c->values.push_back(v);
    if (err == cudaSuccess) err = cudaMemset(k, 0, bytes);
    if (err == cudaSuccess) err = cudaMemset(v, 0, bytes);
  }
  if (err == cudaSuccess) err = cudaMalloc(&c->d_positions, sizeof(int32_t) * max_tokens);
  if (err == cudaSuccess) err = cudaMalloc(&c->d_seq_ids, sizeof(int32_t) * max_tokens);
  if (err == cudaSuccess) err = cudaMallocHost(&c->h_staging, sizeof(int32_t) * 2 * static_cast<size_t>(max_tokens));
  if (err == cudaSuccess) err = cudaEventCreateWithFlags(&c->staging_free, cudaEventDisableTiming);
  if (err == cudaSuccess) err = cudaDeviceSynchronize();  // the memsets are done before first use
  if (err != cudaSuccess) {
    release(c);
    return fail(BM_ERR_CUDA, "bm_kv_cache_create: %s", cudaGetErrorString(err));
  }
  *cache_out = c;
  return BM_OK;
}

extern "C" int bm_kv_cache_destroy(bm_kv_cache_t* cache) {
  if (!cache) return BM_OK;
  if (cache->staging_free) cudaEventSynchronize(cache->staging_free);
  release(cache);
  return BM_OK;
}

extern "C" int bm_kv_cache_layer(const bm_kv_cache_t* cache, int32_t layer, void** keys, void** values) {
  using namespace bm;
  if (!cache || !keys || !values) return fail(BM_ERR_INVALID_ARGUMENT, "bm_kv_cache_layer: NULL pointer");
  if (layer < 0 || layer >= cache->num_layers) return fail(BM_ERR_INVALID_ARGUMENT, "bm_kv_cache_layer: bad layer");
  *keys = cache->keys[layer];
  *values = cache->values[layer];
  return BM_OK;
}

extern "C" int bm_kv_cache_seq_len(const bm_kv_cache_t* cache, int32_t seq, int32_t* len_out) {
  using namespace bm;
  if (!cache || !len_out) return fail(BM_ERR_INVALID_ARGUMENT, "bm_kv_cache_seq_len: NULL pointer");
  if (seq < 0 || seq >= cache->num_seqs) return fail(BM_ERR_INVALID_ARGUMENT, "bm_kv_cache_seq_len: bad sequence");
  *len_out = cache->lens[seq];
  return BM_OK;
}

extern "C" int bm_kv_cache_reset(bm_kv_cache_t* cache, int32_t seq) {
  using namespace bm;
  if (!cache) return fail(BM_ERR_INVALID_ARGUMENT, "bm_kv_cache_reset: NULL cache");
  if (seq == -1) {
    std::fill(cache->lens.begin(), cache->lens.end(), 0);
    return BM_OK;
  }
  if (seq < 0 || seq >= cache->num_seqs) return fail(BM_ERR_INVALID_ARGUMENT, "bm_kv_cache_reset: bad sequence");
  cache->lens[seq] = 0;
  return BM_OK;
}

extern "C" int bm_kv_cache_append(bm_kv_cache_t* cache, const int32_t* seq_ids, int64_t rows,
                                  const int32_t** positions_dev, const int32_t** seq_ids_dev, void* stream) {
  using namespace bm;
  if (!cache || !positions_dev || !seq_ids_dev) return fail(BM_ERR_INVALID_ARGUMENT, "bm_kv_cache_append: NULL pointer");
  if (rows < 0 || rows > cache->max_tokens) {
    return fail(BM_ERR_INVALID_ARGUMENT, "bm_kv_cache_append: %lld tokens outside [0, %d]", static_cast<long long>(rows),
                cache->max_tokens);
  }
  if (rows > 0 && !seq_ids) return fail(BM_ERR_INVALID_ARGUMENT, "bm_kv_cache_append: NULL seq_ids");
  // Positions on a copy of the lengths: nothing changes unless every token fits.
  std::vector<int32_t> lens = cache->lens;
  std::vector<int32_t> pos(static_cast<size_t>(rows));
  for (int64_t r = 0; r < rows; ++r) {
    const int32_t s = seq_ids[r];
    if (s < 0 || s >= cache->num_seqs) {
      return fail(BM_ERR_INVALID_ARGUMENT, "bm_kv_cache_append: token %lld has sequence %d outside [0, %d)",
                  static_cast<long long>(r), s, cache->num_seqs);
    }
    if (lens[s] >= cache->max_seq) {
      return fail(BM_ERR_INVALID_ARGUMENT, "bm_kv_cache_append: sequence %d would pass max_seq %d", s, cache->max_seq);
    }
    pos[r] = lens[s]++;
  }
  cudaStream_t st = as_stream(stream);
  cudaError_t err = cudaEventSynchronize(cache->staging_free);  // the previous upload has left the staging buffer
  if (err == cudaSuccess && rows > 0) {
    std::memcpy(cache->h_staging, pos.data(), sizeof(int32_t) * rows);
    std::memcpy(cache->h_staging + cache->max_tokens, seq_ids, sizeof(int32_t) * rows);
    err = cudaMemcpyAsync(cache->d_positions, cache->h_staging, sizeof(int32_t) * rows, cudaMemcpyHostToDevice, st);
    if (err == cudaSuccess) {
      err = cudaMemcpyAsync(cache->d_seq_ids, cache->h_staging + cache->max_tokens, sizeof(int32_t) * rows,
                            cudaMemcpyHostToDevice, st);
    }
    if (err == cudaSuccess) err = cudaEventRecord(cache->staging_free, st);
  }
  if (err != cudaSuccess) return fail(BM_ERR_CUDA, "bm_kv_cache_append: %s", cudaGetErrorString(err));
  cache->lens.swap(lens);
  *positions_dev = cache->d_positions;
  *seq_ids_dev = cache->d_seq_ids;
  return BM_OK;
}
