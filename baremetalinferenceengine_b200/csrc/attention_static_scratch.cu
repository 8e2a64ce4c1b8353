// Decode attention for callers that cannot allocate device memory.
//
// bm_decode_attention splits long sequences across CTAs and keeps the partial
// results in a scratch buffer that its caller allocates. Some callers have no way
// to do that: code running inside a host application that owns all device memory
// through its own arena and forbids stray cudaMalloc calls, plugins loaded into a
// process that reserved the GPU's memory up front, or latency-critical paths where
// cudaMalloc's implicit device synchronisation is not acceptable. This variant
// takes the same inputs and outputs and keeps the split partials in a fixed array
// compiled into this library instead.
//
// The array is kStaticScratchBytes (8 MiB) of device memory, file-scope and
// 256-byte aligned; every GPU that loads the library holds its own copy until the
// process exits. Limits and behaviour:
//   - the arguments are checked first, as bm_decode_attention checks them; then a
//     call whose plan needs more than 8 MiB of partials is rejected with
//     BM_ERR_INVALID_ARGUMENT. The plan is the one bm_decode_attention runs when
//     its workspace is this array: the balanced tensor-core kernel where it
//     applies (at most a few MiB), else the per-pair grid's splits, whose need
//     grows with batch * num_q_heads * head_dim;
//   - the first call in a CUDA context looks up that context's copy of the array
//     (cudaGetSymbolAddress, with the device current) and caches the address under
//     the context's unique id, so a device reset or another context on the same
//     device gets its own lookup; make that first call on each device before
//     capturing any stream;
//   - every call shares the array, which keeps the last call's contents. No part
//     of it needs clearing: every partial that the combine step reads is written
//     earlier in the same call. Calls whose work overlaps on the GPU (several
//     streams, or several host threads without ordering) race on the array; the
//     caller must serialise them.
// The function calls no cudaMalloc, cudaFree or allocating library routine.
#include <cuda.h>

#include <mutex>

#include "bm_host.h"

namespace bm {

// Validates the call as bm_decode_attention does and returns the split scratch of
// its two plans: the per-pair grid's and the balanced kernel's (SIZE_MAX where that
// kernel does not apply) (attention.cu).
int decode_attention_scratch_need(const void* q, const void* k_cache, const void* v_cache, int32_t max_len,
                                  int64_t batch, int32_t hq, int32_t hkv, int32_t hd, int32_t max_seq,
                                  int32_t num_seqs, bm_dtype_t dtype, size_t* grid_bytes, size_t* balanced_bytes);

namespace {

constexpr size_t kStaticScratchBytes = 8u << 20;
__device__ __align__(256) unsigned char g_attention_scratch[kStaticScratchBytes];

using CtxGetCurrent = CUresult (*)(CUcontext*);
using CtxGetId = CUresult (*)(CUcontext, unsigned long long*);

// The driver's context queries, looked up once through the runtime.
struct ContextQueries {
  CtxGetCurrent current = nullptr;
  CtxGetId id = nullptr;
};

const ContextQueries& context_queries() {
  static std::once_flag once;
  static ContextQueries q;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult r;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &r) == cudaSuccess &&
        r == cudaDriverEntryPointSuccess) {
      q.current = reinterpret_cast<CtxGetCurrent>(p);
    }
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &r) == cudaSuccess &&
        r == cudaDriverEntryPointSuccess) {
      q.id = reinterpret_cast<CtxGetId>(p);
    }
  });
  return q;
}

constexpr int kMaxCachedContexts = 64;
std::mutex g_scratch_mutex;
unsigned long long g_cached_context[kMaxCachedContexts] = {};
void* g_cached_address[kMaxCachedContexts] = {};
int g_cached = 0;

// The current context's copy of g_attention_scratch. In host code the array's
// name only stands in for the symbol: the device address comes from
// cudaGetSymbolAddress, once per context (keyed by the context's unique id; a
// driver without cuCtxGetId gets a fresh lookup every call).
int scratch_address(void** out) {
  int dev = -1;
  cudaError_t err = cudaGetDevice(&dev);  // also makes the device's primary context current if none is
  if (err != cudaSuccess) return fail(BM_ERR_CUDA, "bm_decode_attention_static_scratch: %s", cudaGetErrorString(err));
  const ContextQueries& cq = context_queries();
  unsigned long long id = 0;
  CUcontext ctx = nullptr;
  const bool keyed = cq.current != nullptr && cq.id != nullptr && cq.current(&ctx) == CUDA_SUCCESS &&
                     ctx != nullptr && cq.id(ctx, &id) == CUDA_SUCCESS;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (keyed) {
    for (int i = 0; i < g_cached; ++i) {
      if (g_cached_context[i] == id) {
        *out = g_cached_address[i];
        return BM_OK;
      }
    }
  }
  void* p = nullptr;
  err = cudaGetSymbolAddress(&p, g_attention_scratch);
  if (err != cudaSuccess || p == nullptr) {
    return fail(BM_ERR_CUDA, "bm_decode_attention_static_scratch: cudaGetSymbolAddress on device %d: %s", dev,
                cudaGetErrorString(err));
  }
  if (keyed) {
    const int slot = g_cached < kMaxCachedContexts ? g_cached++ : static_cast<int>(id % kMaxCachedContexts);
    g_cached_context[slot] = id;
    g_cached_address[slot] = p;
  }
  *out = p;
  return BM_OK;
}

}  // namespace
}  // namespace bm

extern "C" int bm_decode_attention_static_scratch(void* out, const void* q, const void* k_cache,
                                                  const void* v_cache, const int32_t* seq_ids, const int32_t* lens,
                                                  int32_t max_len, int64_t batch, int32_t num_q_heads,
                                                  int32_t num_kv_heads, int32_t head_dim, int32_t max_seq,
                                                  int32_t num_seqs, float scale, bm_dtype_t dtype, int32_t* d_status,
                                                  void* stream) {
  using namespace bm;
  if (!lens) return fail(BM_ERR_INVALID_ARGUMENT, "bm_decode_attention_static_scratch: NULL lens");
  size_t grid = 0, balanced = 0;
  if (int st = decode_attention_scratch_need(q, k_cache, v_cache, max_len, batch, num_q_heads, num_kv_heads,
                                             head_dim, max_seq, num_seqs, dtype, &grid, &balanced)) {
    return st;
  }
  if (batch == 0) return BM_OK;
  // bm_decode_attention given this array runs the balanced kernel when it applies
  // (its partials always fit), else the per-pair grid, which must fit whole.
  const size_t need = std::min(grid, balanced);
  if (need > kStaticScratchBytes) {
    return fail(BM_ERR_INVALID_ARGUMENT,
                "bm_decode_attention_static_scratch: this batch needs %zu bytes of split scratch, more than the %zu "
                "bytes of the static array; call bm_decode_attention with a workspace of that size instead",
                need, kStaticScratchBytes);
  }
  void* scratch = nullptr;
  if (need > 0 || balanced != SIZE_MAX) {
    if (int st = scratch_address(&scratch)) return st;
  }
  return decode_attention(out, q, k_cache, v_cache, seq_ids, lens, 0, max_len, batch, num_q_heads, num_kv_heads,
                          head_dim, max_seq, num_seqs, scale, scratch, scratch ? kStaticScratchBytes : 0, dtype,
                          d_status, stream);
}
