// ref_kernels_shim.cu — TEST INFRASTRUCTURE. C entry points over the
// reference's own CUDA kernels (src/kernels.cu, compiled for sm_100a with its
// five layer-op launchers renamed ref_launch_* by oracle/Makefile), so tests
// can run the reference's kernels on the same device buffers as ours and the
// benchmark can time them the way ExecutionEngine::run_layers calls them
// (one token per launch). Built into oracle/_ref/libref_kernels.so.
//
// The -D renames apply to this file too, so the launch_* names below resolve to
// the reference's kernels. Launch errors exit through the reference's CUDA_CHECK.
#include "kernels.cuh"

extern "C" {

void ref_rms_norm(float* out, float* in, float* weight, int size, float eps, void* stream) {
  launch_rms_norm(out, in, weight, size, eps, static_cast<cudaStream_t>(stream));
}

void ref_rope(float* q, float* k, int seq_pos, int head_dim, int num_heads, int num_kv_heads, float theta,
              void* stream) {
  launch_rope(q, k, seq_pos, head_dim, num_heads, num_kv_heads, theta, static_cast<cudaStream_t>(stream));
}

void ref_swiglu(float* out, float* gate, float* up, int size, void* stream) {
  launch_swiglu(out, gate, up, size, static_cast<cudaStream_t>(stream));
}

void ref_add(float* out, float* a, float* b, int size, void* stream) {
  launch_add(out, a, b, size, static_cast<cudaStream_t>(stream));
}

void ref_kv_store(float* cache, float* src, int seq_pos, int num_heads, int head_dim, int max_seq_len,
                  void* stream) {
  launch_kv_store(cache, src, seq_pos, num_heads, head_dim, max_seq_len, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
