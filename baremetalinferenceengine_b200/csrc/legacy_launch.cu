// The reference's single-token launch API (include/kernels.cuh, C++ linkage),
// served by the batched C ABI with rows = 1 and fp32 storage.
//
// Error behaviour mirrors the reference's CUDA_CHECK (include/cuda_utils.h:8-16):
// a failure prints its reason and calls exit(EXIT_FAILURE). Where the reference
// would hand a kernel an argument that makes it write out of bounds (a KV
// position outside the cache, an odd head_dim), this API stops with the same
// message-and-exit instead of writing.
#include <cstdio>
#include <cstdlib>

#include "bm_host.h"
#include "bm_layer_ops.h"
#include "kernels.cuh"

namespace {

void check_or_exit(int status, const char* what, const char* file, int line) {
  if (status != BM_OK) {
    std::fprintf(stderr, "bm error at %s:%d in %s: %s: %s\n", file, line, what, bm_status_string(status),
                 bm_last_error_message());
    std::exit(EXIT_FAILURE);
  }
}

#define BM_LAUNCH_CHECK(call, what) check_or_exit((call), (what), __FILE__, __LINE__)

}  // namespace

// Reference: include/kernels.cuh:9, src/kernels.cu:75-78.
void launch_rms_norm(float* out, float* in, float* weight, int size, float eps, cudaStream_t stream) {
  if (size <= 0) return;  // the reference kernel writes nothing for an empty vector
  BM_LAUNCH_CHECK(bm_rmsnorm(out, in, weight, 1, size, eps, size, size, BM_F32, stream), "launch_rms_norm");
}

// Reference: include/kernels.cuh:15, src/kernels.cu:142-148. cos/sin are
// computed per pair in fp64 from theta (no table), as the reference's CPU
// check loop does (tests/kernel_tests.cu:175-187).
void launch_rope(float* q, float* k, int seq_pos, int head_dim, int num_heads, int num_kv_heads, float theta,
                 cudaStream_t stream) {
  if (head_dim <= 0 || head_dim % 2 != 0) {
    BM_LAUNCH_CHECK(BM_ERR_INVALID_ARGUMENT, "launch_rope (head_dim must be even and positive)");
  }
  if (seq_pos < 0) BM_LAUNCH_CHECK(BM_ERR_INVALID_ARGUMENT, "launch_rope (negative seq_pos)");
  BM_LAUNCH_CHECK(bm_rope(q, k, nullptr, seq_pos, nullptr, 0, static_cast<double>(theta), 1, num_heads,
                          num_kv_heads, head_dim, BM_F32, nullptr, stream),
                  "launch_rope");
}

// Reference: include/kernels.cuh:29, src/kernels.cu:192-195.
void launch_swiglu(float* out, float* gate, float* up, int size, cudaStream_t stream) {
  if (size <= 0) return;
  BM_LAUNCH_CHECK(bm_swiglu(out, gate, up, size, BM_F32, stream), "launch_swiglu");
}

// Reference: include/kernels.cuh:32, src/kernels.cu:204-207.
void launch_add(float* out, float* a, float* b, int size, cudaStream_t stream) {
  if (size <= 0) return;
  BM_LAUNCH_CHECK(bm_add(out, a, b, size, BM_F32, stream), "launch_add");
}

// Reference: include/kernels.cuh:36, src/kernels.cu:219-222. One sequence
// (the reference's cache has batch size 1), position seq_pos.
void launch_kv_store(float* cache, float* src, int seq_pos, int num_heads, int head_dim, int max_seq_len,
                     cudaStream_t stream) {
  if (num_heads <= 0 || head_dim <= 0) return;
  if (seq_pos < 0 || seq_pos >= max_seq_len) {
    BM_LAUNCH_CHECK(BM_ERR_INVALID_ARGUMENT, "launch_kv_store (seq_pos outside [0, max_seq_len))");
  }
  BM_LAUNCH_CHECK(bm_kv_store(cache, src, nullptr, seq_pos, nullptr, 1, num_heads, head_dim, max_seq_len, 1,
                              BM_F32, nullptr, stream),
                  "launch_kv_store");
}

// Reference: include/kernels.cuh:41, src/kernels.cu:258-264. One token, num_heads
// query heads over as many kv heads, positions [0, seq_len) of a cache laid out
// [num_heads][max_seq_len][head_dim]. The reference API hands its kernels
// `scores` (at least num_heads * seq_len floats) as scratch; here it holds the
// per-split partial results when the sequence is split across CTAs (as many
// splits as fit in it), so the call allocates nothing.
void launch_attention(float* out, float* q, float* k_cache, float* v_cache, float* scores, int num_heads,
                      int head_dim, int max_seq_len, int seq_len, cudaStream_t stream) {
  if (seq_len <= 0 || seq_len > max_seq_len) {
    BM_LAUNCH_CHECK(BM_ERR_INVALID_ARGUMENT, "launch_attention (seq_len outside [1, max_seq_len])");
  }
  const size_t scratch = scores ? sizeof(float) * static_cast<size_t>(num_heads) * seq_len : 0;
  BM_LAUNCH_CHECK(bm::decode_attention(out, q, k_cache, v_cache, nullptr, nullptr, seq_len, seq_len, 1, num_heads,
                                       num_heads, head_dim, max_seq_len, 1, 0.f, scores, scratch, BM_F32, nullptr,
                                       stream),
                  "launch_attention");
}

// Reference: include/kernels.cuh:20, src/kernels.cu:83-121. C[M][N] = A[M][K] B[K][N]
// in fp32 (the engine calls it with M = 1 per token): bm_gemm's CUDA-core path.
void launch_gemm(float* C, float* A, float* B, int M, int N, int K, cudaStream_t stream) {
  if (M <= 0 || N <= 0) return;  // the reference's grid is empty
  BM_LAUNCH_CHECK(bm_gemm(C, A, B, M, N, K < 0 ? 0 : K, BM_F32, nullptr, stream), "launch_gemm");
}

// Reference: include/kernels.cuh:23, src/kernels.cu:174-176.
void launch_softmax(float* x, int size, cudaStream_t stream) { launch_softmax_batch(x, size, 1, size, stream); }

// Reference: include/kernels.cuh:26, src/kernels.cu:178-180. num_vectors vectors of
// `size` elements, `stride` apart, in place.
void launch_softmax_batch(float* x, int size, int num_vectors, int stride, cudaStream_t stream) {
  if (size <= 0 || num_vectors <= 0) return;
  BM_LAUNCH_CHECK(bm_softmax(x, size, num_vectors, stride, BM_F32, stream), "launch_softmax_batch");
}
