// matmul.cu — general Matmul (m > 1, or m == 1 without transposeB).
//
// Semantics: C[m,n] = sum_k A[m,k] * B(k,n) with fp32 accumulation and one
// rounding at the store (Matmul.metal:7-27; MPPMatmul.metal:20-63 computes
// the same product on Apple tensor units). B(k,n) = B[n,k] with transposeB
// (linear-layer layout) else B[k,n].
//
// This file holds the CUDA-core kernel that serves every dtype combination
// and shape. 16-bit transposeB problems large enough for the tensor cores
// go to the tcgen05 kernel (gemm_tcgen05.cu) instead.
#include "common.cuh"
#include "dtype.cuh"
#include "launch.hpp"
#include "popcorn.hpp"

namespace popcorn {
namespace launch {

namespace {

constexpr int kBM = 64, kBN = 64, kBK = 16;

// 256 threads, 64x64 output tile, 4x4 outputs per thread, k-tiles of 16
// staged (as fp32) in shared memory.
template <class AT, class BT, class CT>
__global__ void __launch_bounds__(256) matmul_tiled_kernel(const Matmul p) {
    __shared__ float As[kBK][kBM + 4];
    __shared__ float Bs[kBK][kBN + 4];
    pdl_launch_dependents();
    pdl_wait();
    const int tid = threadIdx.x;
    const int64_t m0 = int64_t(blockIdx.y) * kBM, n0 = int64_t(blockIdx.x) * kBN;
    const int tr = tid / 16, tc = tid % 16;  // 16 x 16 threads, 4x4 each
    float acc[4][4] = {};
    for (int64_t k0 = 0; k0 < p.K; k0 += kBK) {
        for (int i = tid; i < kBM * kBK; i += 256) {
            int mm = i / kBK, kk = i % kBK;
            int64_t gm = m0 + mm, gk = k0 + kk;
            As[kk][mm] = (gm < p.M && gk < p.K) ? Elem<AT>::load(p.a, gm * p.K + gk) : 0.f;
        }
        for (int i = tid; i < kBN * kBK; i += 256) {
            int nn, kk;
            if (p.transpose_b) { nn = i / kBK; kk = i % kBK; }
            else { kk = i / kBN; nn = i % kBN; }
            int64_t gn = n0 + nn, gk = k0 + kk;
            float v = 0.f;
            if (gn < p.N && gk < p.K) v = Elem<BT>::load(p.b, p.transpose_b ? gn * p.K + gk : gk * p.N + gn);
            Bs[kk][nn] = v;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < kBK; ++kk) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[kk][tr * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tc * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        int64_t gm = m0 + tr * 4 + i;
        if (gm >= p.M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            int64_t gn = n0 + tc * 4 + j;
            if (gn < p.N) Elem<CT>::store(p.c, gm * p.N + gn, acc[i][j]);
        }
    }
}

template <class AT, class BT, class CT>
cudaError_t run_tiled(const Matmul& p, cudaStream_t s) {
    dim3 grid(unsigned((p.N + kBN - 1) / kBN), unsigned((p.M + kBM - 1) / kBM));
    return launch_k(matmul_tiled_kernel<AT, BT, CT>, grid, dim3(256), 0, s, p);
}

}  // namespace

cudaError_t matmul_tcgen05(const Matmul& p, cudaStream_t s);
bool tcgen05_supports(const Matmul& p);

bool matmul_uses_tensor_cores(const Matmul& p) { return tcgen05_supports(p); }

cudaError_t matmul(const Matmul& p, cudaStream_t s) {
    if (p.M == 0 || p.N == 0) return cudaSuccess;
    if (tcgen05_supports(p)) return matmul_tcgen05(p, s);
    int a = p.a_dtype, b = p.b_dtype, c = p.c_dtype;
    if (a == PC_F32 && b == PC_F32 && c == PC_F32) return run_tiled<TF32, TF32, TF32>(p, s);
    if (a == PC_F32 && b == PC_BF16 && c == PC_F32) return run_tiled<TF32, TBF16, TF32>(p, s);
    if (a == PC_F32 && b == PC_F16 && c == PC_F32) return run_tiled<TF32, TF16, TF32>(p, s);
    if (a == PC_BF16 && b == PC_BF16 && c == PC_F32) return run_tiled<TBF16, TBF16, TF32>(p, s);
    if (a == PC_BF16 && b == PC_BF16 && c == PC_BF16) return run_tiled<TBF16, TBF16, TBF16>(p, s);
    if (a == PC_F16 && b == PC_F16 && c == PC_F32) return run_tiled<TF16, TF16, TF32>(p, s);
    if (a == PC_F16 && b == PC_F16 && c == PC_F16) return run_tiled<TF16, TF16, TF16>(p, s);
    if (a == PC_F32 && b == PC_BF16 && c == PC_BF16) return run_tiled<TF32, TBF16, TBF16>(p, s);
    if (a == PC_F32 && b == PC_F16 && c == PC_F16) return run_tiled<TF32, TF16, TF16>(p, s);
    return cudaErrorInvalidValue;
}

namespace {
RegisterFunctions reg_matmul({
    {"matmul", reinterpret_cast<const void*>(matmul_tiled_kernel<TF32, TF32, TF32>)},
    {"matmul_bf16", reinterpret_cast<const void*>(matmul_tiled_kernel<TF32, TBF16, TF32>)},
    {"matmul_f16", reinterpret_cast<const void*>(matmul_tiled_kernel<TF32, TF16, TF32>)},
    {"matmul_bf16_bf16_f32", reinterpret_cast<const void*>(matmul_tiled_kernel<TBF16, TBF16, TF32>)},
    {"matmul_bf16_bf16_bf16", reinterpret_cast<const void*>(matmul_tiled_kernel<TBF16, TBF16, TBF16>)},
    {"matmul_f16_f16_f32", reinterpret_cast<const void*>(matmul_tiled_kernel<TF16, TF16, TF32>)},
    {"matmul_f16_f16_f16", reinterpret_cast<const void*>(matmul_tiled_kernel<TF16, TF16, TF16>)},
});
}  // namespace

}  // namespace launch
}  // namespace popcorn
