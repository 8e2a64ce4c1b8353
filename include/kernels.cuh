// kernels.cuh — drop-in launch API for BareMetalInferenceEngine's kernels.
//
// These are C++ (name-mangled) functions with exactly the signatures of the
// reference's include/kernels.cuh — all nine of them — so src/execution_engine.cu
// and its tests compile unchanged against this header and link against
// libbm_layer_ops.so alone. Each one is a single-token, fp32 call into the
// batched C ABI of bm_layer_ops.h (rows = 1, dtype = BM_F32) on `stream`.
//
// Error behaviour follows the reference's CUDA_CHECK (include/cuda_utils.h:8-16):
// an argument the reference would pass to a kernel that then writes out of
// bounds, or a failed launch, prints the reason to stderr and calls
// exit(EXIT_FAILURE). The batched C ABI reports the same conditions as status
// codes instead.
#ifndef KERNELS_CUH
#define KERNELS_CUH

#include <cuda_runtime.h>

// Reference include/kernels.cuh:9. Normalises one vector of `size` floats;
// out may equal in.
void launch_rms_norm(float* out, float* in, float* weight, int size, float eps = 1e-5f, cudaStream_t stream = 0);

// Reference include/kernels.cuh:15. Rotates q [num_heads][head_dim] and
// k [num_kv_heads][head_dim] in place for one token at seq_pos, pairing element
// i with i + head_dim/2. head_dim must be even.
void launch_rope(float* q, float* k, int seq_pos, int head_dim, int num_heads, int num_kv_heads, float theta = 10000.0f, cudaStream_t stream = 0);

// Reference include/kernels.cuh:29. out = silu(gate) * up over `size` floats.
void launch_swiglu(float* out, float* gate, float* up, int size, cudaStream_t stream = 0);

// Reference include/kernels.cuh:32. out = a + b; out may equal a or b.
void launch_add(float* out, float* a, float* b, int size, cudaStream_t stream = 0);

// Reference include/kernels.cuh:36. Writes src [num_heads][head_dim] into
// position seq_pos of a cache laid out [num_heads][max_seq_len][head_dim].
// seq_pos must be in [0, max_seq_len).
void launch_kv_store(float* cache, float* src, int seq_pos, int num_heads, int head_dim, int max_seq_len, cudaStream_t stream = 0);

// Reference include/kernels.cuh:41. Attention of one query per head over the
// first seq_len positions of a [num_heads][max_seq_len][head_dim] cache; scores
// (at least num_heads * seq_len floats) is scratch. Served by the split decode
// attention of bm_layer_ops.h, which keeps its per-split partials in `scores`.
void launch_attention(float* out, float* q, float* k_cache, float* v_cache, float* scores, int num_heads, int head_dim, int max_seq_len, int seq_len, cudaStream_t stream = 0);

// Reference include/kernels.cuh:20. C[M][N] = A[M][K] B[K][N], fp32 row-major,
// any sizes: bm_gemm's fp32 path (CUDA cores, K split over a cluster).
void launch_gemm(float* C, float* A, float* B, int M, int N, int K, cudaStream_t stream = 0);

// Reference include/kernels.cuh:23,26. Softmax in place over one vector, or over
// num_vectors vectors `stride` floats apart (the gaps untouched): bm_softmax.
void launch_softmax(float* x, int size, cudaStream_t stream = 0);
void launch_softmax_batch(float* x, int size, int num_vectors, int stride, cudaStream_t stream = 0);

#endif  // KERNELS_CUH
