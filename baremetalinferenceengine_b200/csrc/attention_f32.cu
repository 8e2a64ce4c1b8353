// Decode-attention kernels for fp32 caches (see attention_kernels.cuh).
#include "attention_kernels.cuh"

namespace bm {
namespace attn {

int launch_f32(const AttnArgs& a, cudaStream_t stream) { return launch<float>(a, stream); }
int launch_f32_rope(const AttnArgs& a, cudaStream_t stream) { return launch<float, true>(a, stream); }

}  // namespace attn
}  // namespace bm
