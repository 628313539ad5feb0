// tc_stubs.cu — the tensor-core prefill attention is not built yet: every
// problem is reported unsupported, so the CUDA-core kernel serves it.
#include "launch.hpp"

namespace popcorn {
namespace launch {

bool fa_tcgen05_supports(const FlashAttention&) { return false; }
cudaError_t flash_attention_tcgen05(const FlashAttention&, cudaStream_t) { return cudaErrorNotSupported; }

}  // namespace launch
}  // namespace popcorn
