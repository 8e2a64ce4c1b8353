// execution_engine.h — drop-in ExecutionEngine on the batched, fused layer ops.
//
// The public interface is the reference's (include/execution_engine.h:11-74:
// constructor, forward, reset, set_verbose, and the same exceptions), so the
// reference's src/main.cpp, src/benchmark.cpp, src/server.cpp and
// tests/logits_test.cu compile unchanged against this header. The
// implementation (execution_engine.cu beside it) differs from the reference's
// run_layers (src/execution_engine.cu:89-128) in two ways:
//   - all tokens of one forward() call go through each layer together: one
//     launch per op for the whole batch instead of one per token, attention
//     included (each token attends to its own causal length in the same launch);
//   - the memory-bound ops are the fused B200 kernels of bm_layer_ops.h: the
//     embedding gather, the residual add fused into the RMSNorm that follows it
//     (:118+:121, :126+:109, :126+:80), RoPE fused with both KV-cache writes
//     (:113-115), and the split decode attention (:116).
// The projections are this library's fp32 GEMMs: Q, K and V in one launch
// (bm_gemm_shared_a), the gate and up projections with the SwiGLU in their
// epilogue (bm_gemm_swiglu, :122-124), the others through launch_gemm. Every launch goes to the
// engine's own stream, and a one-token forward (a decode step) replays a CUDA
// graph of the whole layer loop, captured on the second such call: positions and
// attended lengths come from small device arrays refreshed before each replay,
// and attention is planned for the cache's full length so the launches never
// change.
#ifndef EXECUTION_ENGINE_H
#define EXECUTION_ENGINE_H

#include <cuda_runtime.h>

#include <memory>
#include <string>
#include <vector>

#include "kv_cache.h"
#include "memory_allocator.h"
#include "weights.h"

class ExecutionEngine {
 public:
  // Throws std::runtime_error if the allocator is missing a tensor the model needs.
  ExecutionEngine(std::shared_ptr<MemoryAllocator> allocator, std::shared_ptr<KVCache> kv_cache,
                  const ModelConfig& config);
  ~ExecutionEngine();

  // Feeds tokens through the model, extending the sequence held in the KV cache,
  // and returns the logits that follow the last token. Throws
  // std::invalid_argument for bad tokens, or std::runtime_error when the sequence
  // would exceed the KV cache.
  std::vector<float> forward(const std::vector<int>& input_tokens);

  // Starts a new sequence.
  void reset();

  void set_verbose(bool verbose) { verbose_ = verbose; }

 private:
  struct LayerWeights {
    float* attention_norm;
    float* q_proj;
    float* k_proj;
    float* v_proj;
    float* o_proj;
    float* ffn_norm;
    float* gate_proj;
    float* up_proj;
    float* down_proj;
  };

  float* weight(const std::string& name) const;
  void reserve(int tokens);  // grows the per-token activation buffers

  std::shared_ptr<MemoryAllocator> allocator_;
  std::shared_ptr<KVCache> kv_cache_;
  ModelConfig config_;

  float* token_embeddings_ = nullptr;
  float* final_norm_ = nullptr;
  float* lm_head_ = nullptr;
  std::vector<LayerWeights> layers_;

  // [capacity][dim] / [capacity][hidden_dim] activations, fp32
  int capacity_ = 0;
  std::vector<std::shared_ptr<DeviceBuffer<float>>> activations_;
  float* hidden_ = nullptr;    // the residual stream; each add writes the other buffer of the pair
  float* hidden_alt_ = nullptr;
  float* normed_ = nullptr;    // norm output, for rows too long to normalise inside a product
  float* q_ = nullptr;
  float* k_ = nullptr;
  float* v_ = nullptr;
  float* attention_out_ = nullptr;
  float* projected_ = nullptr;
  float* activated_ = nullptr;
  std::shared_ptr<DeviceBuffer<int>> token_args_;  // [3][capacity]: a call's ids, positions, lens
  int* ids_ = nullptr;                             // this call's three arrays in token_args_
  // Every layer and the logits of the last token for T tokens on stream_;
  // attention planned for at most max_len attended positions.
  void run(int T, int max_len);

  cudaStream_t stream_ = nullptr;
  cudaGraphExec_t decode_graph_ = nullptr;  // a one-token forward, replayed
  int graph_capacity_ = -1;                 // capacity_ when the graph was captured
  int eager_decode_steps_ = 0;              // one-token forwards run before the capture
  int* staging_ = nullptr;                  // pinned host: ids, positions, lens of a call
  int* positions_ = nullptr;                // cache position per token
  int* lens_ = nullptr;                     // attended positions per token
  float* logits_host_ = nullptr;            // pinned host: the last token's logits
  std::shared_ptr<DeviceBuffer<char>> attention_workspace_;  // split partials of decode attention

  std::shared_ptr<DeviceBuffer<float>> logits_;  // [vocab]
  std::shared_ptr<DeviceBuffer<float>> rope_table_;  // [max_seq][head_dim/2] (cos, sin)

  bool verbose_ = false;
};

#endif  // EXECUTION_ENGINE_H
