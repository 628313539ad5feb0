// batched.cu — fused helpers for batched decode (B sequences per step), each
// equal to a reference op sequence with the same rounding points:
//
//  * qkv_scatter: the output of ONE Matmul against the concatenated
//    [W_q; W_k; W_v] ([B, (Nq+2Nkv)*Hd]) is split into q [B,Nq,1,Hd] and the
//    new key/value rows, which go to the caches [B,Nkv,Smax,Hd] at the
//    position exactly as KVCacheWrite stores them (KVCacheWrite.metal:17-26).
//    Replaces three Matmuls + two KVCacheWrites by one Matmul + this copy.
//  * gated_activation: out = round(act(g)) * u from ONE Matmul against the
//    concatenated [W_gate; W_up] ([rows, 2F]: g = columns 0..F-1, u = F..2F-1)
//    — GeluTanh (or SiLU) then Mul (GeluTanh.metal:6-35, Mul.metal:7-25).
//  * add_rmsnorm: s = round(a + b) (Add.metal:7-25), then
//    n = RMSNorm(s) (RMSNorm.metal:7-42); both outputs stored.
//
// All three are bandwidth-trivial at decode sizes; 16-byte accesses where
// the layout allows.
#include "common.cuh"
#include "dtype.cuh"
#include "launch.hpp"
#include "peer_reduce.cuh"
#include "popcorn.hpp"

namespace popcorn {
namespace launch {

namespace {

// One 16-byte chunk per thread (the caller checked Hd * elem % 16 == 0 and
// 16-byte aligned bases, so a chunk never straddles two rows).
__global__ void qkv_scatter_kernel(const QKVScatter p, int es) {
    pdl_wait();
    const int64_t offset = p.pos_dev ? int64_t(*p.pos_dev) : p.offset;
    if (offset < 0 || offset >= p.Smax) return;
    const int vec = 16 / es;
    const int64_t row_chunks = (p.Nq + 2 * p.Nkv) * p.Hd / vec;  // chunks of one qkv row
    const int64_t head_chunks = p.Hd / vec;
    const int64_t total = p.B * row_chunks;
    for (int64_t c = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; c < total; c += int64_t(gridDim.x) * blockDim.x) {
        const int64_t b = c / row_chunks, rc = c % row_chunks;
        const uint4 v = reinterpret_cast<const uint4*>(p.qkv)[c];
        const int64_t h = rc / head_chunks, d = rc % head_chunks;  // head index over q, k, v blocks
        if (h < p.Nq) {
            reinterpret_cast<uint4*>(p.q)[(b * p.Nq + h) * head_chunks + d] = v;
        } else {
            const bool is_v = h >= p.Nq + p.Nkv;
            const int64_t hk = h - p.Nq - (is_v ? p.Nkv : 0);
            uint4* cache = reinterpret_cast<uint4*>(is_v ? p.v_cache : p.k_cache);
            cache[((b * p.Nkv + hk) * p.Smax + offset) * head_chunks + d] = v;
        }
    }
}

template <class T, int ACT>
__global__ void gated_activation_kernel(const void* gu, void* out, int64_t rows, int64_t F) {
    pdl_wait();
    const int64_t total = rows * F;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = i / F, f = i % F;
        const float g = Elem<T>::load(gu, r * 2 * F + f);
        const float u = Elem<T>::load(gu, r * 2 * F + F + f);
        const float a = Elem<T>::round(ACT == 0 ? gelu_tanh(g) : silu(g));
        Elem<T>::store(out, i, a * u);
    }
}

template <class T>
__global__ void add_rmsnorm_kernel(const AddRMSNorm p) {
    pdl_wait();
    __shared__ float red[32];
    __shared__ float s_scale;
    const int64_t base = int64_t(blockIdx.x) * p.H;
    float acc = 0.f;
    for (int64_t i = threadIdx.x; i < p.H; i += blockDim.x) {
        const float s = Elem<T>::round(Elem<T>::load(p.a, base + i) + Elem<T>::load(p.b, base + i));
        Elem<T>::store(p.sum_out, base + i, s);
        acc += s * s;
    }
    acc = warp_sum(acc);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = acc;
    __syncthreads();
    if (warp == 0) {
        float v = lane < int(blockDim.x >> 5) ? red[lane] : 0.f;
        v = warp_sum(v);
        if (lane == 0) s_scale = rsqrtf(v / float(p.H) + p.eps);
    }
    __syncthreads();
    const float scale = s_scale;
    for (int64_t i = threadIdx.x; i < p.H; i += blockDim.x) {
        // the rounded sum, as RMSNorm reads it back from memory
        float v = Elem<T>::round(Elem<T>::load(p.a, base + i) + Elem<T>::load(p.b, base + i)) * scale;
        if (p.weight) {
            float w = p.weight[i];
            if (p.add_one) w = 1.0f + w;
            v *= w;
        }
        Elem<T>::store(p.norm_out, base + i, v);
    }
}

// 16-bit rows with H % 8 == 0: the row step of the peer all-reduce with a
// single "rank" (the partial b), so this kernel and the fused all-reduce
// accumulate the sum of squares in the same order and round identically —
// the NCCL path and the peer path of a tensor-parallel model then agree bit
// for bit wherever the collective's sums agree.
template <class T>
__global__ void __launch_bounds__(256) add_rmsnorm_rows_kernel(const AddRMSNorm a) {
    pdl_wait();
    __shared__ float red[256 / 32];
    PeerAllReduce p{};
    p.partial[0][0] = a.b;
    p.world = 1;
    p.buffer = 0;
    p.residual = a.a;
    p.sum_out = a.sum_out;
    p.norm_out = a.norm_out;
    p.weight = a.weight;
    p.rows = a.rows;
    p.H = a.H;
    p.eps = a.eps;
    p.add_one = a.add_one;
    pr_reduce_row<T, 256>(p, blockIdx.x, true, threadIdx.x, red, [] { __syncthreads(); });
}

}  // namespace

cudaError_t qkv_scatter(const QKVScatter& p, cudaStream_t s) {
    const int es = dtype_stride(p.dtype);
    const int64_t chunks = p.B * (p.Nq + 2 * p.Nkv) * p.Hd * es / 16;
    if (chunks == 0) return cudaSuccess;
    return launch_k(qkv_scatter_kernel, dim3(grid_for(chunks, 256, current_sm_count())), dim3(256), 0, s, p, es);
}

cudaError_t gated_activation(const void* gu, void* out, int dtype, int64_t rows, int64_t F, int act, cudaStream_t s) {
    const int64_t n = rows * F;
    if (n == 0) return cudaSuccess;
    dim3 g(grid_for(n, 256, current_sm_count())), b(256);
    switch (dtype) {
    case PC_F32: return act == 0 ? launch_k(gated_activation_kernel<TF32, 0>, g, b, 0, s, gu, out, rows, F)
                                 : launch_k(gated_activation_kernel<TF32, 1>, g, b, 0, s, gu, out, rows, F);
    case PC_F16: return act == 0 ? launch_k(gated_activation_kernel<TF16, 0>, g, b, 0, s, gu, out, rows, F)
                                 : launch_k(gated_activation_kernel<TF16, 1>, g, b, 0, s, gu, out, rows, F);
    case PC_BF16: return act == 0 ? launch_k(gated_activation_kernel<TBF16, 0>, g, b, 0, s, gu, out, rows, F)
                                  : launch_k(gated_activation_kernel<TBF16, 1>, g, b, 0, s, gu, out, rows, F);
    }
    return cudaErrorInvalidValue;
}

cudaError_t add_rmsnorm(const AddRMSNorm& p, cudaStream_t s) {
    if (p.rows == 0) return cudaSuccess;
    const bool rows16 = (p.dtype == PC_BF16 || p.dtype == PC_F16) && p.H % kPrVec == 0 &&
                        p.H <= int64_t(256) * kPrVec * kPrMaxChunks && aligned16(p.a) && aligned16(p.b) &&
                        aligned16(p.sum_out) && aligned16(p.norm_out);
    if (rows16) {
        dim3 g(unsigned(p.rows)), b(256);
        if (p.dtype == PC_BF16) return launch_k(add_rmsnorm_rows_kernel<TBF16>, g, b, 0, s, p);
        return launch_k(add_rmsnorm_rows_kernel<TF16>, g, b, 0, s, p);
    }
    const int threads = p.H >= 4096 ? 1024 : (p.H >= 1024 ? 256 : 128);
    dim3 g(unsigned(p.rows)), b(threads);
    switch (p.dtype) {
    case PC_F32: return launch_k(add_rmsnorm_kernel<TF32>, g, b, 0, s, p);
    case PC_F16: return launch_k(add_rmsnorm_kernel<TF16>, g, b, 0, s, p);
    case PC_BF16: return launch_k(add_rmsnorm_kernel<TBF16>, g, b, 0, s, p);
    }
    return cudaErrorInvalidValue;
}

namespace {
RegisterFunctions reg_batched({
    {"qkv_scatter", reinterpret_cast<const void*>(qkv_scatter_kernel)},
    {"gated_activation_bf16", reinterpret_cast<const void*>(gated_activation_kernel<TBF16, 0>)},
    {"gated_activation_f16", reinterpret_cast<const void*>(gated_activation_kernel<TF16, 0>)},
    {"gated_activation", reinterpret_cast<const void*>(gated_activation_kernel<TF32, 0>)},
    {"add_rmsnorm_bf16", reinterpret_cast<const void*>(add_rmsnorm_kernel<TBF16>)},
    {"add_rmsnorm_f16", reinterpret_cast<const void*>(add_rmsnorm_kernel<TF16>)},
    {"add_rmsnorm", reinterpret_cast<const void*>(add_rmsnorm_kernel<TF32>)},
});
}  // namespace

}  // namespace launch
}  // namespace popcorn
