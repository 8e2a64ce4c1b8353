// Decode-attention kernels for bf16 caches (see attention_kernels.cuh).
#include "attention_kernels.cuh"

namespace bm {
namespace attn {

int launch_bf16(const AttnArgs& a, cudaStream_t stream) { return launch<bf16>(a, stream); }
int launch_bf16_rope(const AttnArgs& a, cudaStream_t stream) { return launch<bf16, true>(a, stream); }

}  // namespace attn
}  // namespace bm
