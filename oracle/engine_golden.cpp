// engine_golden.cpp — TEST INFRASTRUCTURE. Runs the reference's unmodified
// ExecutionEngine (src/execution_engine.cu) with the reference's own kernels on
// a model export and writes the logits after every token in the format the
// reference's tests/logits_test.cu reads (tests/logits_test.cu:35-44):
//   int32 vocab_size, int32 count, int32 tokens[count], float logits[count][vocab_size].
// oracle/Makefile links it with the reference's sources into
// oracle/_ref/engine_golden_ref. The same export and these logits then check
// logits_test.cu built against libbm_layer_ops.so (the drop-in).
//
// Usage: engine_golden_ref <model_dir> <token> [<token> ...]
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <memory>
#include <vector>

#include "execution_engine.h"
#include "kv_cache.h"
#include "memory_allocator.h"
#include "weights.h"

int main(int argc, char** argv) {
  if (argc < 3) {
    std::fprintf(stderr, "usage: %s <model_dir> <token>...\n", argv[0]);
    return 2;
  }
  const std::string dir = argv[1];
  std::vector<int> tokens;
  for (int i = 2; i < argc; ++i) tokens.push_back(std::atoi(argv[i]));

  ModelLoader loader;
  if (!loader.load(dir)) return 2;
  const ModelConfig& config = loader.get_config();
  auto allocator = std::make_shared<MemoryAllocator>();
  allocator->allocate_and_copy_weights(loader.get_tensors());
  auto kv_cache = std::make_shared<KVCache>(1, config.max_seq_len, config.num_layers, config.num_heads,
                                            config.head_dim());
  ExecutionEngine engine(allocator, kv_cache, config);

  std::ofstream out(dir + "/reference_logits.bin", std::ios::binary);
  const int32_t header[2] = {config.vocab_size, static_cast<int32_t>(tokens.size())};
  out.write(reinterpret_cast<const char*>(header), sizeof(header));
  for (int t : tokens) {
    const int32_t v = t;
    out.write(reinterpret_cast<const char*>(&v), sizeof(v));
  }
  for (int t : tokens) {  // one token at a time, as logits_test checks every position
    const std::vector<float> logits = engine.forward({t});
    out.write(reinterpret_cast<const char*>(logits.data()), logits.size() * sizeof(float));
  }
  std::printf("wrote %zu positions of %d logits\n", tokens.size(), config.vocab_size);
  return out ? 0 : 1;
}
