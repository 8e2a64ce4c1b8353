// execution_engine.cu — ExecutionEngine on the fused B200 layer ops (see the header).
#include "execution_engine.h"

#include <iostream>
#include <stdexcept>
#include <utility>

#include "bm_layer_ops.h"
#include "kernels.cuh"

namespace {

void check(int status, const char* what) {
  if (status != BM_OK) {
    throw std::runtime_error(std::string(what) + ": " + bm_status_string(status) + ": " + bm_last_error_message());
  }
}

}  // namespace

ExecutionEngine::ExecutionEngine(std::shared_ptr<MemoryAllocator> allocator, std::shared_ptr<KVCache> kv_cache,
                                 const ModelConfig& config)
    : allocator_(allocator), kv_cache_(kv_cache), config_(config) {
  token_embeddings_ = weight("model.embed_tokens.weight");
  final_norm_ = weight("model.norm.weight");
  lm_head_ = weight("lm_head.weight");
  for (int l = 0; l < config_.num_layers; ++l) {
    const std::string p = "model.layers." + std::to_string(l) + ".";
    layers_.push_back({weight(p + "input_layernorm.weight"), weight(p + "self_attn.q_proj.weight"),
                       weight(p + "self_attn.k_proj.weight"), weight(p + "self_attn.v_proj.weight"),
                       weight(p + "self_attn.o_proj.weight"), weight(p + "post_attention_layernorm.weight"),
                       weight(p + "mlp.gate_proj.weight"), weight(p + "mlp.up_proj.weight"),
                       weight(p + "mlp.down_proj.weight")});
  }
  const int max_seq = kv_cache_->get_max_seq_len();
  logits_ = std::make_shared<DeviceBuffer<float>>(config_.vocab_size);
  CUDA_CHECK(cudaMallocHost(&logits_host_, sizeof(float) * config_.vocab_size));
  // (cos, sin) per position, computed once on the device in fp64 and kept in L2-sized fp32
  rope_table_ = std::make_shared<DeviceBuffer<float>>(static_cast<size_t>(max_seq) * config_.head_dim());
  CUDA_CHECK(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
  check(bm_rope_table_fill(rope_table_->get(), max_seq, config_.head_dim(), config_.rope_theta, stream_),
        "bm_rope_table_fill");
  reserve(1);
}

ExecutionEngine::~ExecutionEngine() {
  if (decode_graph_) cudaGraphExecDestroy(decode_graph_);
  if (staging_) cudaFreeHost(staging_);
  if (logits_host_) cudaFreeHost(logits_host_);
  if (stream_) cudaStreamDestroy(stream_);
}

float* ExecutionEngine::weight(const std::string& name) const {
  float* tensor = static_cast<float*>(allocator_->get_device_tensor(name));
  if (!tensor) throw std::runtime_error("Model is missing tensor " + name);
  return tensor;
}

void ExecutionEngine::reserve(int tokens) {
  if (tokens <= capacity_) return;
  const size_t dim = config_.dim;
  const size_t hidden = config_.hidden_dim;
  const size_t n = static_cast<size_t>(tokens);
  activations_.clear();
  auto buffer = [&](size_t elements) {
    activations_.push_back(std::make_shared<DeviceBuffer<float>>(elements));
    return activations_.back()->get();
  };
  hidden_ = buffer(n * dim);
  hidden_alt_ = buffer(n * dim);
  normed_ = buffer(n * dim);
  q_ = buffer(n * dim);
  k_ = buffer(n * dim);
  v_ = buffer(n * dim);
  attention_out_ = buffer(n * dim);
  projected_ = buffer(n * dim);
  activated_ = buffer(n * hidden);
  token_args_ = std::make_shared<DeviceBuffer<int>>(3 * n);
  if (staging_) CUDA_CHECK(cudaFreeHost(staging_));
  CUDA_CHECK(cudaMallocHost(&staging_, 3 * n * sizeof(int)));
  size_t ws = 0;
  check(bm_decode_attention_workspace_size(tokens, config_.num_heads, config_.num_heads, config_.head_dim(),
                                           kv_cache_->get_max_seq_len(), &ws),
        "bm_decode_attention_workspace_size");
  attention_workspace_ = std::make_shared<DeviceBuffer<char>>(ws);
  capacity_ = tokens;
}

void ExecutionEngine::reset() { kv_cache_->reset(); }

std::vector<float> ExecutionEngine::forward(const std::vector<int>& input_tokens) {
  // Argument checks and messages as the reference's forward (src/execution_engine.cu:62-69).
  if (input_tokens.empty()) throw std::invalid_argument("forward() needs at least one token");
  for (int token : input_tokens) {
    if (token < 0 || token >= config_.vocab_size) {
      throw std::invalid_argument("Token " + std::to_string(token) + " is outside the vocabulary");
    }
  }
  const int max_seq = kv_cache_->get_max_seq_len();
  const size_t end_pos = static_cast<size_t>(kv_cache_->get_current_seq_pos()) + input_tokens.size();
  if (end_pos > static_cast<size_t>(max_seq)) {
    throw std::runtime_error("Sequence would exceed the KV cache's " + std::to_string(max_seq) + " positions");
  }
  if (verbose_) std::cout << "Forward pass for " << input_tokens.size() << " tokens" << std::endl;

  const int T = static_cast<int>(input_tokens.size());
  reserve(T);
  const int pos0 = kv_cache_->get_current_seq_pos();
  // ids, positions and attended lengths (token t: pos0 + t + 1), laid out
  // [ids | positions | lengths] in pinned staging and sent in one copy; for one
  // token the device pointers are always the same, as the decode graph needs
  for (int t = 0; t < T; ++t) {
    staging_[t] = input_tokens[t];
    staging_[T + t] = pos0 + t;
    staging_[2 * T + t] = pos0 + t + 1;
  }
  ids_ = token_args_->get();
  positions_ = ids_ + T;
  lens_ = ids_ + 2 * T;
  CUDA_CHECK(cudaMemcpyAsync(ids_, staging_, sizeof(int) * 3 * T, cudaMemcpyHostToDevice, stream_));

  if (T > 1) {
    run(T, pos0 + T);
  } else if (decode_graph_ && graph_capacity_ == capacity_) {
    CUDA_CHECK(cudaGraphLaunch(decode_graph_, stream_));
  } else if (eager_decode_steps_ < 1 || graph_capacity_ >= 0) {
    // the first decode step runs eagerly (it sets up every kernel outside a
    // capture); so does every step after the buffers moved under a graph
    ++eager_decode_steps_;
    if (decode_graph_ && graph_capacity_ != capacity_) {
      CUDA_CHECK(cudaGraphExecDestroy(decode_graph_));
      decode_graph_ = nullptr;
      graph_capacity_ = -1;
    }
    run(1, max_seq);
  } else {
    cudaGraph_t graph = nullptr;
    CUDA_CHECK(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
    try {
      run(1, max_seq);
    } catch (...) {
      cudaStreamEndCapture(stream_, &graph);
      if (graph) cudaGraphDestroy(graph);
      throw;
    }
    CUDA_CHECK(cudaStreamEndCapture(stream_, &graph));
    CUDA_CHECK(cudaGraphInstantiate(&decode_graph_, graph, 0));
    CUDA_CHECK(cudaGraphDestroy(graph));
    graph_capacity_ = capacity_;
    CUDA_CHECK(cudaGraphLaunch(decode_graph_, stream_));
  }
  kv_cache_->increment_seq_pos(T);

  // the logits come back through pinned memory (a pageable destination would be
  // staged by the driver)
  CUDA_CHECK(cudaMemcpyAsync(logits_host_, logits_->get(), sizeof(float) * config_.vocab_size,
                             cudaMemcpyDeviceToHost, stream_));
  CUDA_CHECK(cudaStreamSynchronize(stream_));
  return std::vector<float>(logits_host_, logits_host_ + config_.vocab_size);
}

void ExecutionEngine::run(int T, int max_len) {
  const int dim = config_.dim;
  const int hidden_dim = config_.hidden_dim;
  const int heads = config_.num_heads;
  const int head_dim = config_.head_dim();
  const int max_seq = kv_cache_->get_max_seq_len();
  const float eps = config_.norm_eps;
  check(bm_embed_gather(hidden_, token_embeddings_, ids_, T, dim, config_.vocab_size, dim, BM_F32, nullptr,
                        stream_),
        "bm_embed_gather");

  // The residual stream alternates between hidden_ and hidden_alt_: every residual
  // add is fused into the norm of the product that follows it (bm_rmsnorm_gemm), whose
  // kernel still reads the old rows while it writes the new ones.
  float* h = hidden_;
  float* h_next = hidden_alt_;
  for (int l = 0; l < config_.num_layers; ++l) {
    const LayerWeights& w = layers_[l];
    float* k_cache = kv_cache_->get_key_cache(l);
    float* v_cache = kv_cache_->get_value_cache(l);

    // The previous layer's residual add (its down projection), this layer's attention
    // norm (:109, :80 for layer 0) and the Q, K and V projections (:110-112): one launch.
    {
      void* outs[3] = {q_, k_, v_};
      const void* weights[3] = {w.q_proj, w.k_proj, w.v_proj};
      const int32_t widths[3] = {dim, dim, dim};
      const float* delta = l == 0 ? nullptr : projected_;
      check(bm_rmsnorm_gemm(outs, h, delta, w.attention_norm, eps, delta ? h_next : nullptr, normed_, weights,
                            widths, 3, 0, T, dim, BM_F32, nullptr, stream_),
            "bm_rmsnorm_gemm");
      if (delta) std::swap(h, h_next);
    }
    if (T == 1) {
      // A decode step (:113-116): the token's RoPE, its K/V store at positions_[0] and
      // its attention over [0, lens_[0]) in one launch.
      check(bm_rope_kv_decode_attention(attention_out_, q_, k_, v_, positions_, rope_table_->get(), max_seq,
                                        nullptr, k_cache, v_cache, lens_, max_len, 1, heads, heads, head_dim,
                                        max_seq, 1, 0.f, attention_workspace_->get(), attention_workspace_->size(),
                                        BM_F32, nullptr, stream_),
            "bm_rope_kv_decode_attention");
    } else {
      // Token t at cache position positions_[t] of the one sequence the reference's cache holds.
      check(bm_rope_kv_store(q_, k_, v_, positions_, 0, nullptr, k_cache, v_cache, rope_table_->get(),
                             max_seq, config_.rope_theta, T, heads, heads, head_dim, max_seq, 1, BM_F32, nullptr,
                             stream_),
            "bm_rope_kv_store");
      // All T tokens' attention in one launch: query t over cache positions [0, lens_[t]).
      check(bm_decode_attention(attention_out_, q_, k_cache, v_cache, nullptr, lens_, max_len, T, heads,
                                heads, head_dim, max_seq, 1, 0.f, attention_workspace_->get(),
                                attention_workspace_->size(), BM_F32, nullptr, stream_),
            "bm_decode_attention");
    }
    launch_gemm(projected_, attention_out_, w.o_proj, T, dim, dim, stream_);
    // The attention residual add (:118), the FFN norm (:121) and the gate and up
    // projections with the SwiGLU in the epilogue (:122-124): one launch.
    {
      void* outs[2] = {activated_, nullptr};
      const void* weights[2] = {w.gate_proj, w.up_proj};
      const int32_t widths[2] = {hidden_dim, hidden_dim};
      check(bm_rmsnorm_gemm(outs, h, projected_, w.ffn_norm, eps, h_next, normed_, weights, widths, 2, 1, T, dim,
                            BM_F32, nullptr, stream_),
            "bm_rmsnorm_gemm");
      std::swap(h, h_next);
    }
    launch_gemm(projected_, activated_, w.down_proj, T, dim, hidden_dim, stream_);
  }

  // Only the last token's logits are returned: its final residual add and norm with
  // the vocabulary product, one launch.
  const size_t last = static_cast<size_t>(T - 1) * dim;
  {
    void* outs[1] = {logits_->get()};
    const void* weights[1] = {lm_head_};
    const int32_t widths[1] = {config_.vocab_size};
    check(bm_rmsnorm_gemm(outs, h + last, projected_ + last, final_norm_, eps, nullptr, normed_ + last, weights,
                          widths, 1, 0, 1, dim, BM_F32, nullptr, stream_),
          "bm_rmsnorm_gemm");
  }
}

