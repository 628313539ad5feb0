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
#include "popcorn.hpp"

namespace popcorn {

__device__ unsigned int g_allreduce_error_word;

namespace launch {

namespace {

__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint4 ld_volatile16(const void* p) {
    uint4 v;
    asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}

constexpr int kArThreads = 256;
constexpr int kArVec = 8;        // 16-bit elements per 16-byte chunk
constexpr int kArMaxChunks = 4;  // chunks per thread: rows up to 8192 elements

template <class T>
__global__ void __launch_bounds__(kArThreads) allreduce_add_rmsnorm_kernel(const PeerAllReduce p) {
    pdl_wait();
    __shared__ float red[kArThreads / 32];
    __shared__ float s_scale;
    __shared__ int s_ok;
    __shared__ unsigned int s_epoch;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int b = p.buffer;
    unsigned int* my_ctl = p.ctl[p.rank];  // [0..1] flags, [2..3] epochs, [4] CTA count
    if (tid == 0) {
        const unsigned int e = my_ctl[2 + b] + 1u;
        s_epoch = e;
        if (blockIdx.x == 0) {
            __threadfence_system();
            st_release_sys(&my_ctl[b], e);
        }
        // wait for every rank's partial of this call
        int ok = 1;
        for (int r = 0; r < p.world && ok; ++r) {
            long i = 0;
            while (ld_acquire_sys(&p.ctl[r][b]) < e) {
                if (++i > (1l << 22)) {
                    atomicOr(&g_allreduce_error_word, 8u);
                    ok = 0;
                    break;
                }
                __nanosleep(64);
            }
        }
        s_ok = ok;
    }
    __syncthreads();
    const int64_t row = blockIdx.x;
    const int64_t H = p.H;
    const int nchunks = int(H / kArVec);
    float acc[kArMaxChunks][kArVec];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kArMaxChunks; ++j) {
        const int c = tid + j * kArThreads;
        if (c >= nchunks) continue;
        float o[kArVec];
#pragma unroll
        for (int e = 0; e < kArVec; ++e) o[e] = 0.f;
        if (s_ok) {
            for (int r = 0; r < p.world; ++r) {
                const uint4 w = ld_volatile16(static_cast<const char*>(p.partial[r][b]) + (row * H + int64_t(c) * kArVec) * 2);
                float f[kArVec];
                unpack8<T>(w, f);
#pragma unroll
                for (int e = 0; e < kArVec; ++e) o[e] += f[e];
            }
        }
        const uint4 rw = *reinterpret_cast<const uint4*>(static_cast<const char*>(p.residual) + (row * H + int64_t(c) * kArVec) * 2);
        float res[kArVec];
        unpack8<T>(rw, res);
#pragma unroll
        for (int e = 0; e < kArVec; ++e) {
            const float s = Elem<T>::round(res[e] + Elem<T>::round(o[e]));
            acc[j][e] = s;
            ss += s * s;
        }
        uint4 so;
        so.x = pack2<T>(acc[j][0], acc[j][1]);
        so.y = pack2<T>(acc[j][2], acc[j][3]);
        so.z = pack2<T>(acc[j][4], acc[j][5]);
        so.w = pack2<T>(acc[j][6], acc[j][7]);
        *reinterpret_cast<uint4*>(static_cast<char*>(p.sum_out) + (row * H + int64_t(c) * kArVec) * 2) = so;
    }
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (warp == 0) {
        float v = lane < kArThreads / 32 ? red[lane] : 0.f;
        v = warp_sum(v);
        if (lane == 0) s_scale = rsqrtf(v / float(H) + p.eps);
    }
    __syncthreads();
    const float scale = s_scale;
#pragma unroll
    for (int j = 0; j < kArMaxChunks; ++j) {
        const int c = tid + j * kArThreads;
        if (c >= nchunks) continue;
        float v[kArVec];
#pragma unroll
        for (int e = 0; e < kArVec; ++e) {
            float x = acc[j][e] * scale;
            if (p.weight) {
                float w = p.weight[c * kArVec + e];
                if (p.add_one) w = 1.0f + w;
                x *= w;
            }
            v[e] = x;
        }
        uint4 no;
        no.x = pack2<T>(v[0], v[1]);
        no.y = pack2<T>(v[2], v[3]);
        no.z = pack2<T>(v[4], v[5]);
        no.w = pack2<T>(v[6], v[7]);
        *reinterpret_cast<uint4*>(static_cast<char*>(p.norm_out) + (row * H + int64_t(c) * kArVec) * 2) = no;
    }
    // the last CTA out advances this rank's epoch for buffer b
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const unsigned int done = atomicAdd(&my_ctl[4], 1u);
        if (done == gridDim.x - 1) {
            my_ctl[4] = 0u;
            my_ctl[2 + b] = s_epoch;
            __threadfence();
        }
    }
}

}  // namespace

bool peer_allreduce_supports(const PeerAllReduce& p) {
    return (p.dtype == PC_BF16 || p.dtype == PC_F16) && p.H % kArVec == 0 && p.H <= kArVec * kArMaxChunks * kArThreads &&
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
