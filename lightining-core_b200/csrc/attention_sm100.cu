// bf16 attention dispatch.  The tcgen05 flash-attention kernel lives in this file; shapes it
// does not take run the fp32-math SIMT kernel (attention_simt.cu) -- never a CPU path.
#include "common.cuh"
#include "lc_internal.hpp"

namespace lcb {

bool attention_bf16_tc_supported(const AttnArgs&) { return false; }

cudaError_t attention_bf16(const AttnArgs& a, cudaStream_t s) { return attention_bf16_simt(a, s); }

}  // namespace lcb
