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

// Programmatic dependent launch for this library's kernels: on unless the
// environment sets BM_PDL=0 (read once).
bool pdl_enabled();

// Launches `kernel` with programmatic stream serialization when pdl_enabled():
// its blocks may be scheduled while the previous kernel on the stream finishes,
// and it waits for that kernel (grid_dependency_wait) before touching memory, so
// launch latency overlaps the previous kernel's tail, also inside CUDA graphs.
// extra_attr (optional) is one more launch attribute (a cluster shape).
template <typename... KArgs, typename... Args>
int launch_kernel(const char* what, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                  cudaStream_t stream, const cudaLaunchAttribute* extra_attr, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (extra_attr != nullptr) attr[n++] = *extra_attr;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
  if (err != cudaSuccess) return fail(BM_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(err));
  return check_launch(what);
}

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
// The same products of y = rmsnorm(h + d) * norm_w (d may be null), y made in the
// kernel's prologue; residual_out (may be null) receives h + d. swiglu: b[0], b[1]
// are the gate and up weights (n[0] == n[1]) and c[0] the one output. Rows too long
// for shared memory run the norm into `normed` first (two or three launches).
int gemm_f32_norm(float* const* c, const float* h, const float* d, const float* norm_w, float eps,
                  float* residual_out, float* normed, const float* const* b, const int32_t* n, int count,
                  bool swiglu, int64_t m, int k, cudaStream_t stream);

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
