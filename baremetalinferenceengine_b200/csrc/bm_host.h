// Host-side helpers shared by the C ABI entry points: error reporting into a
// thread-local message, launch checks and per-device launch sizing.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "bm_layer_ops.h"

namespace bm {

// Records a message for bm_last_error_message() and returns `status`.
int fail(int status, const char* fmt, ...) __attribute__((format(printf, 2, 3)));

// Clears the thread's last error message.
void clear_error();

// Returns BM_OK, or BM_ERR_CUDA with the launch error of `what` recorded.
int check_launch(const char* what);

// Streaming multiprocessors of the current device (cached per device).
int sm_count();

// fp32 GEMMs on CUDA cores (gemm_f32.cu); host checks are the caller's.
// c[M][N] = a[M][K] b[K][N].
int gemm_f32(float* c, const float* a, const float* b, int64_t m, int n, int k, cudaStream_t stream);
// c[o][M][n[o]] = a[M][K] b[o][K][n[o]] for o < count <= kMaxSharedA, one launch.
constexpr int kMaxSharedA = 3;
int gemm_f32_shared_a(float* const* c, const float* a, const float* const* b, const int32_t* n, int count,
                      int64_t m, int k, cudaStream_t stream);
// out[rows][hidden] = silu(x w_gate) * (x w_up), x [rows][dim], w_* [dim][hidden].
int gemm_f32_swiglu(float* out, const float* x, const float* w_gate, const float* w_up, int64_t rows, int hidden,
                    int dim, cudaStream_t stream);

// cudaFuncSetAttribute(kernel, MaxDynamicSharedMemorySize, bytes) on the current
// device, once per (device, kernel): later calls cost a lookup, not a driver call.
int allow_dynamic_smem(const void* kernel, int bytes, const char* what);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int dtype_size(bm_dtype_t dt) { return dt == BM_F32 ? 4 : 2; }

inline bool valid_dtype(int dt) { return dt == BM_F32 || dt == BM_BF16; }

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// bm_decode_attention with a host-side length for every query (lens == NULL:
// len0), as the reference's single-token launch_attention needs.
int decode_attention(void* out, const void* q, const void* k_cache, const void* v_cache, const int32_t* seq_ids,
                     const int32_t* lens, int32_t len0, int32_t max_len, int64_t batch, int32_t hq, int32_t hkv,
                     int32_t hd, int32_t max_seq, int32_t num_seqs, float scale, void* workspace,
                     size_t workspace_size, bm_dtype_t dtype, int32_t* d_status, void* stream);

}  // namespace bm
