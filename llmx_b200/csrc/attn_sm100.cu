// Placeholder until the tcgen05 prefill kernel lands.
#include "attn_internal.h"

namespace llmx_b200 {
bool sm100_supports(const AttnArgs &) { return false; }
cudaError_t launch_sm100(const AttnArgs &, cudaStream_t) { return cudaErrorNotSupported; }
}  // namespace llmx_b200
