// ref_kernels_shim.cu — TEST INFRASTRUCTURE. C entry points over the
// reference's own CUDA kernels (src/kernels.cu, compiled for sm_100a with its
// five layer-op launchers renamed ref_launch_* by oracle/Makefile), so tests
// can run the reference's kernels on the same device buffers as ours and the
// benchmark can time them the way ExecutionEngine::run_layers calls them
// (one token per launch). Built into oracle/_ref/libref_kernels.so.
//
// The -D renames apply to this file too, so the launch_* names below resolve to
// the reference's kernels. Launch errors exit through the reference's CUDA_CHECK.
#include <cstdint>

#include "cuda_utils.h"
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

// One layer step's memory-bound ops over `rows` tokens with the reference's own
// kernels, issued the way ExecutionEngine::run_layers issues them for one token
// (src/execution_engine.cu:98-126), token after token on the default stream:
//   ops & 1   embedding row: cudaMemcpy device-to-device (:98-99)
//   ops & 2   launch_add(hidden += attn_out) then launch_rms_norm (:118, :109)
//   ops & 4   launch_rope(q, k) then launch_kv_store of k and of v into the
//             token's sequence cache [kv_heads][max_seq][head_dim] (:113-115)
//   ops & 8   launch_add(hidden += ffn_out) then launch_rms_norm (:126, :121)
//   ops & 16  launch_swiglu (:124)
// Token ids, positions and sequence ids are HOST arrays, as the engine holds
// them. Row-major device buffers, fp32 (the reference's kernels are fp32 only).
// Returns the number of kernel launches plus copies issued.
int64_t ref_layer_step_rows(int ops, int64_t rows, const int32_t* ids, const int32_t* positions,
                            const int32_t* seq_ids, const float* embed, float* hidden, float* attn_out,
                            float* w_attn, float* y_attn, float* q, float* k, float* v, float* k_cache,
                            float* v_cache, float* ffn_out, float* w_ffn, float* y_ffn, float* gate, float* up,
                            float* act, int dim, int hq, int hkv, int hd, int ffn, int max_seq, float theta,
                            float eps) {
  int64_t issued = 0;
  const size_t seq_stride = static_cast<size_t>(hkv) * max_seq * hd;
  for (int64_t r = 0; r < rows; ++r) {
    float* h = hidden + r * dim;
    if (ops & 1) {
      CUDA_CHECK(cudaMemcpy(h, embed + static_cast<size_t>(ids[r]) * dim, dim * sizeof(float),
                            cudaMemcpyDeviceToDevice));
      issued += 1;
    }
    if (ops & 2) {
      launch_add(h, h, attn_out + r * dim, dim);
      launch_rms_norm(y_attn + r * dim, h, w_attn, dim, eps);
      issued += 2;
    }
    if (ops & 4) {
      float* kr = k + r * hkv * hd;
      launch_rope(q + r * hq * hd, kr, positions[r], hd, hq, hkv, theta);
      launch_kv_store(k_cache + seq_ids[r] * seq_stride, kr, positions[r], hkv, hd, max_seq);
      launch_kv_store(v_cache + seq_ids[r] * seq_stride, v + r * hkv * hd, positions[r], hkv, hd, max_seq);
      issued += 3;
    }
    if (ops & 8) {
      launch_add(h, h, ffn_out + r * dim, dim);
      launch_rms_norm(y_ffn + r * dim, h, w_ffn, dim, eps);
      issued += 2;
    }
    if (ops & 16) {
      launch_swiglu(act + r * ffn, gate + r * ffn, up + r * ffn, ffn);
      issued += 1;
    }
  }
  return issued;
}

}  // extern "C"
