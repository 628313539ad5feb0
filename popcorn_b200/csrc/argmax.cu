// argmax.cu — Kernels.Argmax (Argmax.metal:5-76, Argmax.swift): the index
// of the largest element of each row of x [rows, N], int32; ties go to the
// lowest index and NaN never wins (Argmax.metal:7-9). Rows with N < 32 follow
// `argmax` (start from element 0), longer rows `argmax_row` (start from
// (-inf, 0x7fffffff)): the routing of Argmax.swift:21.
//
// B200 design: the "better" relation is a total order on non-NaN (value,
// -index) pairs, so any split of a row gives the reference's answer. Short
// rows: one thread each. Rows up to 64K elements: one CTA per row, 16-byte
// loads, warp then CTA reduction. Longer rows with few of them (an LM head's
// vocabulary at decode: 1-32 rows of ~256K logits): the row is cut into
// chunks spread over every SM (pass 1, partial winners into caller scratch)
// and one warp per row reduces the chunk winners (pass 2).
#include "common.cuh"
#include "dtype.cuh"
#include "launch.hpp"
#include "popcorn.hpp"

namespace popcorn {
namespace launch {

namespace {

constexpr int32_t kNoIndex = 0x7fffffff;
constexpr int kArgThreads = 512;

__device__ __forceinline__ bool better(float cv, int32_t ci, float bv, int32_t bi) {
    return cv > bv || (cv == bv && ci < bi);
}

__device__ __forceinline__ void warp_best(float& v, int32_t& i) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_down_sync(0xffffffffu, v, off);
        const int32_t oi = __shfl_down_sync(0xffffffffu, i, off);
        if (better(ov, oi, v, i)) {
            v = ov;
            i = oi;
        }
    }
}

// Elements [i0, i1) of a row into this thread's running best; 16-byte loads
// when the row pointer and bounds allow.
template <class T>
__device__ __forceinline__ void scan(const void* row, int64_t i0, int64_t i1, int tid, int nthreads, float& bv,
                                     int32_t& bi) {
    constexpr int es = Elem<T>::bytes;
    constexpr int vec = 16 / es;
    const bool vec_ok = (reinterpret_cast<uintptr_t>(row) % 16 == 0) && (i0 % vec == 0);
    int64_t i = i0;
    if (vec_ok) {
        const int64_t nv = (i1 - i0) / vec;
        for (int64_t c = tid; c < nv; c += nthreads) {
            const int64_t base = i0 + c * vec;
            const uint4 w = *reinterpret_cast<const uint4*>(static_cast<const char*>(row) + base * es);
            float f[vec];
            if constexpr (es == 4) {
                f[0] = __uint_as_float(w.x);
                f[1] = __uint_as_float(w.y);
                f[2] = __uint_as_float(w.z);
                f[3] = __uint_as_float(w.w);
            } else {
                float g[8];
                unpack8<T>(w, g);
#pragma unroll
                for (int e = 0; e < vec; ++e) f[e] = g[e];
            }
#pragma unroll
            for (int e = 0; e < vec; ++e)
                if (better(f[e], int32_t(base + e), bv, bi)) {
                    bv = f[e];
                    bi = int32_t(base + e);
                }
        }
        i = i0 + nv * vec;
    }
    for (int64_t j = i + tid; j < i1; j += nthreads) {
        const float v = Elem<T>::load(row, j);
        if (better(v, int32_t(j), bv, bi)) {
            bv = v;
            bi = int32_t(j);
        }
    }
}

// CTA-wide best of (bv, bi); the result is valid in thread 0.
__device__ __forceinline__ void cta_best(float& bv, int32_t& bi) {
    __shared__ float sv[32];
    __shared__ int32_t si[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    warp_best(bv, bi);
    if (lane == 0) {
        sv[warp] = bv;
        si[warp] = bi;
    }
    __syncthreads();
    if (warp == 0) {
        const int nw = (blockDim.x + 31) >> 5;
        bv = lane < nw ? sv[lane] : -INFINITY;
        bi = lane < nw ? si[lane] : kNoIndex;
        warp_best(bv, bi);
    }
}

template <class T>
__global__ void argmax_short_kernel(const void* x, int32_t* out, int64_t rows, int64_t N) {
    pdl_wait();
    const int64_t r = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
    if (r >= rows) return;
    const void* row = static_cast<const char*>(x) + r * N * Elem<T>::bytes;
    float bv = Elem<T>::load(row, 0);  // `argmax`: element 0 first (Argmax.metal:20-21)
    int32_t bi = 0;
    for (int64_t i = 1; i < N; ++i) {
        const float v = Elem<T>::load(row, i);
        if (better(v, int32_t(i), bv, bi)) {
            bv = v;
            bi = int32_t(i);
        }
    }
    out[r] = bi;
}

template <class T>
__global__ void __launch_bounds__(kArgThreads) argmax_row_kernel(const void* x, int32_t* out, int64_t N) {
    pdl_wait();
    const void* row = static_cast<const char*>(x) + int64_t(blockIdx.x) * N * Elem<T>::bytes;
    float bv = -INFINITY;
    int32_t bi = kNoIndex;
    scan<T>(row, 0, N, threadIdx.x, blockDim.x, bv, bi);
    cta_best(bv, bi);
    if (threadIdx.x == 0) out[blockIdx.x] = bi;
}

// Pass 1: chunk blockIdx.x of row blockIdx.y -> (value, index) partial.
template <class T>
__global__ void __launch_bounds__(kArgThreads)
    argmax_chunk_kernel(const void* x, int64_t N, int64_t chunk, float* pv, int32_t* pi) {
    pdl_wait();
    const void* row = static_cast<const char*>(x) + int64_t(blockIdx.y) * N * Elem<T>::bytes;
    const int64_t i0 = int64_t(blockIdx.x) * chunk;
    const int64_t i1 = i0 + chunk < N ? i0 + chunk : N;
    float bv = -INFINITY;
    int32_t bi = kNoIndex;
    scan<T>(row, i0, i1, threadIdx.x, blockDim.x, bv, bi);
    cta_best(bv, bi);
    if (threadIdx.x == 0) {
        const int64_t k = int64_t(blockIdx.y) * gridDim.x + blockIdx.x;
        pv[k] = bv;
        pi[k] = bi;
    }
}

// Pass 2: one warp per row over its chunk winners.
__global__ void argmax_final_kernel(const float* pv, const int32_t* pi, int32_t* out, int64_t rows, int chunks) {
    pdl_wait();
    const int64_t r = blockIdx.x * int64_t(blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (r >= rows) return;
    float bv = -INFINITY;
    int32_t bi = kNoIndex;
    for (int c = lane; c < chunks; c += 32) {
        const float v = pv[r * chunks + c];
        const int32_t i = pi[r * chunks + c];
        if (better(v, i, bv, bi)) {
            bv = v;
            bi = i;
        }
    }
    warp_best(bv, bi);
    if (lane == 0) out[r] = bi;
}

template <class T>
cudaError_t run_argmax(const Argmax& p, cudaStream_t s) {
    if (p.N < 32) {
        const unsigned blocks = unsigned((p.rows + 127) / 128);
        return launch_k(argmax_short_kernel<T>, dim3(blocks), dim3(128), 0, s, p.x, p.out, p.rows, p.N);
    }
    if (p.chunks <= 1) return launch_k(argmax_row_kernel<T>, dim3(unsigned(p.rows)), dim3(kArgThreads), 0, s, p.x, p.out, p.N);
    const int64_t chunk = p.chunk;
    cudaError_t e = launch_k(argmax_chunk_kernel<T>, dim3(unsigned(p.chunks), unsigned(p.rows)), dim3(kArgThreads), 0,
                             s, p.x, p.N, chunk, p.part_v, p.part_i);
    if (e != cudaSuccess) return e;
    return launch_k(argmax_final_kernel, dim3(unsigned((p.rows + 7) / 8)), dim3(256), 0, s, p.part_v, p.part_i, p.out,
                    p.rows, p.chunks);
}

}  // namespace

// Two-pass plan: chunks per row (1: one CTA per row) and the chunk length,
// a multiple of 8 elements so every chunk starts on a 16-byte boundary.
void argmax_plan(Argmax& p, int sm_count) {
    p.chunks = 1;
    p.chunk = p.N;
    if (p.N <= 65536 || p.rows >= sm_count) return;
    int64_t c = (2 * int64_t(sm_count) + p.rows - 1) / p.rows;  // about two CTAs per SM
    const int64_t max_c = (p.N + 4095) / 4096;                 // chunks of >= 4096 elements
    if (c > max_c) c = max_c;
    if (c < 2) return;
    int64_t chunk = (p.N + c - 1) / c;
    chunk = (chunk + 7) / 8 * 8;
    p.chunk = chunk;
    p.chunks = int((p.N + chunk - 1) / chunk);
}

cudaError_t argmax(const Argmax& p, cudaStream_t s) {
    if (p.rows == 0 || p.N == 0) return cudaSuccess;
    switch (p.dtype) {
    case PC_F32: return run_argmax<TF32>(p, s);
    case PC_F16: return run_argmax<TF16>(p, s);
    case PC_BF16: return run_argmax<TBF16>(p, s);
    }
    return cudaErrorInvalidValue;
}

namespace {
RegisterFunctions reg_argmax({
    {"argmax", reinterpret_cast<const void*>(argmax_short_kernel<TF32>)},
    {"argmax_row", reinterpret_cast<const void*>(argmax_row_kernel<TF32>)},
    {"argmax_row_bf16", reinterpret_cast<const void*>(argmax_row_kernel<TBF16>)},
    {"argmax_row_f16", reinterpret_cast<const void*>(argmax_row_kernel<TF16>)},
    {"argmax_chunks", reinterpret_cast<const void*>(argmax_chunk_kernel<TF32>)},
    {"argmax_final", reinterpret_cast<const void*>(argmax_final_kernel)},
});
}  // namespace

}  // namespace launch
}  // namespace popcorn
