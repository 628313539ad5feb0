// tc_stubs.cu — tensor-core entry points not built yet: every problem is
// reported unsupported, so the CUDA-core kernels serve it.
#include "launch.hpp"

namespace popcorn {
namespace launch {

bool tcgen05_supports(const Matmul&) { return false; }
cudaError_t matmul_tcgen05(const Matmul&, cudaStream_t) { return cudaErrorNotSupported; }
bool fa_tcgen05_supports(const FlashAttention&) { return false; }
cudaError_t flash_attention_tcgen05(const FlashAttention&, cudaStream_t) { return cudaErrorNotSupported; }

}  // namespace launch
}  // namespace popcorn
