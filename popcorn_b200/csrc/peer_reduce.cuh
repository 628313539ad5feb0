// peer_reduce.cuh — the row step of the tensor-parallel all-reduce over peer
// memory, shared by the stand-alone all-reduce kernel (allreduce.cu) and the
// GEMM epilogue that fuses it (gemm_tcgen05.cu):
//   o    = round(sum over ranks r, in rank order, of P_r[row])   (fp32 sum)
//   s    = round(residual[row] + o)                              (Add.metal)
//   norm = RMSNorm(s)                                            (RMSNorm.metal)
// plus the system-scope flag helpers of the protocol.
#pragma once

#include "async.cuh"
#include "dtype.cuh"
#include "launch.hpp"

namespace popcorn {
namespace launch {

__device__ __forceinline__ unsigned int pr_ld_acquire_sys(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void pr_st_release_sys(unsigned int* p, unsigned int v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint4 pr_ld_volatile16(const void* p) {
    uint4 v;
    asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}

// Control block of a rank (uint32 words): flag[2] (published epoch per
// buffer), epoch[2] (last completed call per buffer), exit count of the
// current kernel, tiles-done count per buffer (fused GEMM).
enum { kCtlFlag = 0, kCtlEpoch = 2, kCtlExit = 4, kCtlTiles = 5 };

// Bounded wait until every rank has published epoch >= e for buffer b.
// Returns false (and sets `err` bit 3) on give-up.
__device__ __forceinline__ bool pr_wait_peers(const PeerAllReduce& p, unsigned int e, unsigned int* err) {
    for (int r = 0; r < p.world; ++r) {
        long i = 0;
        while (pr_ld_acquire_sys(&p.ctl[r][kCtlFlag + p.buffer]) < e) {
            if (++i > (1l << 22)) {
                atomicOr(err, 8u);
                return false;
            }
            __nanosleep(64);
        }
    }
    return true;
}

constexpr int kPrVec = 8;        // 16-bit elements per 16-byte chunk
constexpr int kPrMaxChunks = 8;  // per thread: NT * 8 * 8 elements per row at most

// One row by NT threads (thread index tid in [0, NT)); `red` holds NT/32
// floats of shared memory; `sync()` is a barrier over the NT threads. With
// `ok` false the sum is skipped (its outputs are then not meaningful).
template <class T, int NT, class Sync>
__device__ __forceinline__ void pr_reduce_row(const PeerAllReduce& p, int64_t row, bool ok, int tid, float* red,
                                              Sync sync) {
    const int lane = tid & 31, warp = tid >> 5;
    const int64_t H = p.H;
    const int nchunks = int(H / kPrVec);
    float acc[kPrMaxChunks][kPrVec];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kPrMaxChunks; ++j) {
        const int c = tid + j * NT;
        if (c >= nchunks) continue;
        float o[kPrVec];
#pragma unroll
        for (int e = 0; e < kPrVec; ++e) o[e] = 0.f;
        if (ok) {
            for (int r = 0; r < p.world; ++r) {
                const uint4 w = pr_ld_volatile16(static_cast<const char*>(p.partial[r][p.buffer]) +
                                                 (row * H + int64_t(c) * kPrVec) * 2);
                float f[kPrVec];
                unpack8<T>(w, f);
#pragma unroll
                for (int e = 0; e < kPrVec; ++e) o[e] += f[e];
            }
        }
        const uint4 rw =
            *reinterpret_cast<const uint4*>(static_cast<const char*>(p.residual) + (row * H + int64_t(c) * kPrVec) * 2);
        float res[kPrVec];
        unpack8<T>(rw, res);
#pragma unroll
        for (int e = 0; e < kPrVec; ++e) {
            const float s = Elem<T>::round(res[e] + Elem<T>::round(o[e]));
            acc[j][e] = s;
            ss += s * s;
        }
        *reinterpret_cast<uint4*>(static_cast<char*>(p.sum_out) + (row * H + int64_t(c) * kPrVec) * 2) =
            make_uint4(pack2<T>(acc[j][0], acc[j][1]), pack2<T>(acc[j][2], acc[j][3]), pack2<T>(acc[j][4], acc[j][5]),
                       pack2<T>(acc[j][6], acc[j][7]));
    }
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    sync();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < NT / 32; ++w) tot += red[w];
    const float scale = rsqrtf(tot / float(H) + p.eps);
#pragma unroll
    for (int j = 0; j < kPrMaxChunks; ++j) {
        const int c = tid + j * NT;
        if (c >= nchunks) continue;
        float v[kPrVec];
#pragma unroll
        for (int e = 0; e < kPrVec; ++e) {
            float x = acc[j][e] * scale;
            if (p.weight) {
                float w = p.weight[c * kPrVec + e];
                if (p.add_one) w = 1.0f + w;
                x *= w;
            }
            v[e] = x;
        }
        *reinterpret_cast<uint4*>(static_cast<char*>(p.norm_out) + (row * H + int64_t(c) * kPrVec) * 2) =
            make_uint4(pack2<T>(v[0], v[1]), pack2<T>(v[2], v[3]), pack2<T>(v[4], v[5]), pack2<T>(v[6], v[7]));
    }
    sync();  // `red` is reused by the next row
}

}  // namespace launch
}  // namespace popcorn
