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
//   - a call whose split plan needs more than 8 MiB of partials is rejected with
//     BM_ERR_INVALID_ARGUMENT; bm_decode_attention_workspace_size reports the need,
//     which grows with batch * num_q_heads * head_dim;
//   - the first call on a device looks up that device's copy of the array
//     (cudaGetSymbolAddress, with the device current) and caches the address;
//     make that first call on each device before capturing any stream;
//   - every call shares the array, which keeps the last call's contents. No part
//     of it needs clearing: every partial that the combine step reads is written
//     earlier in the same call. Calls whose work overlaps on the GPU (several
//     streams, or several host threads without ordering) race on the array; the
//     caller must serialise them.
// The function calls no cudaMalloc, cudaFree or allocating library routine.
#include <mutex>

#include "bm_host.h"

namespace bm {

// Bytes of split partials bm_decode_attention plans for these sizes (attention.cu).
size_t decode_attention_workspace(int64_t batch, int32_t hq, int32_t hkv, int32_t hd, int32_t max_len);

namespace {

constexpr size_t kStaticScratchBytes = 8u << 20;
__device__ __align__(256) unsigned char g_attention_scratch[kStaticScratchBytes];

constexpr int kMaxScratchDevices = 64;
std::mutex g_scratch_mutex;
void* g_scratch_address[kMaxScratchDevices] = {};

// The current device's copy of g_attention_scratch, looked up once per device. In
// host code the array's name only stands in for the symbol: the device address
// must come from cudaGetSymbolAddress.
int scratch_address(void** out) {
  int dev = -1;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return fail(BM_ERR_CUDA, "bm_decode_attention_static_scratch: %s", cudaGetErrorString(err));
  if (dev < 0 || dev >= kMaxScratchDevices) {
    return fail(BM_ERR_INVALID_ARGUMENT, "bm_decode_attention_static_scratch: device %d beyond %d", dev,
                kMaxScratchDevices);
  }
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_address[dev] == nullptr) {
    void* p = nullptr;
    err = cudaGetSymbolAddress(&p, g_attention_scratch);
    if (err != cudaSuccess || p == nullptr) {
      return fail(BM_ERR_CUDA, "bm_decode_attention_static_scratch: cudaGetSymbolAddress: %s",
                  cudaGetErrorString(err));
    }
    g_scratch_address[dev] = p;
  }
  *out = g_scratch_address[dev];
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
  const size_t need = decode_attention_workspace(batch, num_q_heads, num_kv_heads, head_dim, max_len);
  if (need > kStaticScratchBytes) {
    return fail(BM_ERR_INVALID_ARGUMENT,
                "bm_decode_attention_static_scratch: this batch needs %zu bytes of split scratch, more than the %zu "
                "bytes of the static array; call bm_decode_attention with a workspace of that size instead",
                need, kStaticScratchBytes);
  }
  void* scratch = nullptr;
  if (need > 0) {
    if (int st = scratch_address(&scratch)) return st;
  }
  return decode_attention(out, q, k_cache, v_cache, seq_ids, lens, 0, max_len, batch, num_q_heads, num_kv_heads,
                          head_dim, max_seq, num_seqs, scale, scratch, need > 0 ? kStaticScratchBytes : 0, dtype,
                          d_status, stream);
}
