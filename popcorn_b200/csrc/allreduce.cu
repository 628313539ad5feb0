// allreduce.cu — one-shot all-reduce of tensor-parallel partial sums over
// peer memory (NVLink / NVSwitch), fused with the residual add and the next
// RMSNorm: for each row,
//   o    = round(sum over ranks r = 0..world-1, in rank order, of P_r)
//   s    = round(residual + o)                      (Add.metal:7-25)
//   norm = RMSNorm(s, weight, eps, add_one)         (RMSNorm.metal:7-42)
// — the sequence all-reduce(sum) -> Add -> RMSNorm that the NCCL path runs
// as three steps, with one rounding per stored value.
//
// Every rank owns two partial buffers (the o_proj and the down_proj partial
// sums alternate between them) and a control block; all are plain
// cudaMalloc allocations opened by the peers through CUDA IPC, so a kernel
// reads a peer's partial with ordinary loads over NVLink (no TMA, no
// multicast, no library kernel on peer memory). Protocol per call, buffer b:
//   * e = this rank's epoch[b] + 1 (every rank runs the same call sequence);
//   * CTA 0 publishes flag[b] = e with a system-scope release: the partial
//     was written by the preceding kernel, complete in stream order;
//   * every CTA waits (bounded) until each peer's flag[b] >= e, then sums
//     the peers' rows with system-scope-acquired, L1-bypassing loads;
//   * the last CTA out sets epoch[b] = e.
// A rank overwrites buffer b only after the next call on the other buffer,
// which waits for every peer to have passed this call (and so to have read
// buffer b): the alternation is the consumed-barrier.
//
// A wait that gives up sets the device error word and skips the sum (its
// outputs are then garbage, never a hang).
#include "common.cuh"
#include "dtype.cuh"
#include "launch.hpp"
#include "peer_reduce.cuh"
#include "popcorn.hpp"

namespace popcorn {

__device__ unsigned int g_allreduce_error_word;

namespace launch {

namespace {

constexpr int kArThreads = 256;

template <class T>
__global__ void __launch_bounds__(kArThreads) allreduce_add_rmsnorm_kernel(const PeerAllReduce p) {
    pdl_wait();
    __shared__ float red[kArThreads / 32];
    __shared__ int s_ok;
    __shared__ unsigned int s_epoch;
    const int tid = threadIdx.x;
    const int b = p.buffer;
    unsigned int* my_ctl = p.ctl[p.rank];
    if (tid == 0) {
        const unsigned int e = my_ctl[kCtlEpoch + b] + 1u;
        s_epoch = e;
        if (blockIdx.x == 0) {
            // this rank's partial was written by the preceding kernel
            __threadfence_system();
            pr_st_release_sys(&my_ctl[kCtlFlag + b], e);
        }
        s_ok = pr_wait_peers(p, e, &g_allreduce_error_word) ? 1 : 0;
    }
    __syncthreads();
    pr_reduce_row<T, kArThreads>(p, blockIdx.x, s_ok != 0, tid, red, [] { __syncthreads(); });
    // the last CTA out advances this rank's epoch for buffer b
    if (tid == 0) {
        __threadfence();
        const unsigned int done = atomicAdd(&my_ctl[kCtlExit], 1u);
        if (done == gridDim.x - 1) {
            my_ctl[kCtlExit] = 0u;
            my_ctl[kCtlEpoch + b] = s_epoch;
            __threadfence();
        }
    }
}

}  // namespace

bool peer_allreduce_supports(const PeerAllReduce& p) {
    return (p.dtype == PC_BF16 || p.dtype == PC_F16) && p.H % kPrVec == 0 && p.H <= 8192 &&
           p.world >= 1 && p.world <= kMaxPeers && p.rank >= 0 && p.rank < p.world && (p.buffer == 0 || p.buffer == 1);
}

cudaError_t peer_allreduce_add_rmsnorm(const PeerAllReduce& p, cudaStream_t s) {
    if (p.rows == 0) return cudaSuccess;
    dim3 g(unsigned(p.rows)), blk(kArThreads);
    if (p.dtype == PC_BF16) return launch_k(allreduce_add_rmsnorm_kernel<TBF16>, g, blk, 0, s, p);
    return launch_k(allreduce_add_rmsnorm_kernel<TF16>, g, blk, 0, s, p);
}

uint32_t read_and_clear_allreduce_errors() {
    unsigned int v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_allreduce_error_word, sizeof(v)) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    if (v) cudaMemcpyToSymbol(g_allreduce_error_word, &zero, sizeof(zero));
    return v;
}

namespace {
RegisterFunctions reg_ar({
    {"allreduce_add_rmsnorm_bf16", reinterpret_cast<const void*>(allreduce_add_rmsnorm_kernel<TBF16>)},
    {"allreduce_add_rmsnorm_f16", reinterpret_cast<const void*>(allreduce_add_rmsnorm_kernel<TF16>)},
});
}  // namespace

}  // namespace launch
}  // namespace popcorn
