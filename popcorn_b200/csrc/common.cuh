// common.cuh — launch helpers shared by the kernel translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace popcorn {
namespace launch {

int current_sm_count();

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int grid_for(int64_t work_items, int threads, int sm_count) {
    int64_t blocks = (work_items + threads - 1) / threads;
    int64_t cap = int64_t(sm_count) * 8;
    if (blocks > cap) blocks = cap;
    return int(blocks < 1 ? 1 : blocks);
}

// Launches with programmatic stream serialisation allowed: the kernel may
// start while its predecessor on the stream drains; every kernel of this
// library calls griddepcontrol.wait before it reads a predecessor's output.
template <class F, class... Args>
cudaError_t launch_k(F kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// Raises a kernel's dynamic shared memory limit once per process.
template <class F>
cudaError_t allow_smem(F kernel, size_t bytes) {
    if (bytes <= 48 * 1024) return cudaSuccess;
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes));
}

}  // namespace launch
}  // namespace popcorn
