// rope.cu — rotary position embedding and the decode step's per-head q / k
// normalisation (the step before FlashDecoding in Gemma4TextInference.swift:
// 352-381):
//
//  * rope_build_cos_sin (RopeBuildCosSin.metal:5-21): angle = position[t] *
//    inv_freq[i] in fp32; cos / sin tables [T, Hd/2] (fp32) times scaling.
//  * rope_apply (RopeApply.metal:6-49): x [B, T, Nh, Hd]; each head's halves
//    x1 = x[:Hd/2], x2 = x[Hd/2:] become (x1 c - x2 s, x1 s + x2 c).
//  * qk_norm_rope (extension, one launch for the reference's RMSNorm(q) ->
//    RopeApply -> Transpose12 and RMSNorm(k) -> RopeApply -> Transpose12 ->
//    KVCacheWrite, RMSNorm(v) -> Transpose12 -> KVCacheWrite at T = 1, where
//    Transpose12 moves nothing): in place on q [B, Nq, 1, Hd] and on the new
//    key / value rows already in the caches at the position (written there
//    by the QKV projection), with the same rounding points: the normalised
//    head is stored (rounded) before RoPE reads it.
#include "common.cuh"
#include "dtype.cuh"
#include "launch.hpp"
#include "popcorn.hpp"

namespace popcorn {
namespace launch {

namespace {

__global__ void rope_build_kernel(const int32_t* positions, const float* inv_freq, float* cos_out, float* sin_out,
                                  int64_t T, int64_t Hd2, float scaling) {
    pdl_wait();
    const int64_t n = T * Hd2;
    for (int64_t k = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; k < n; k += int64_t(gridDim.x) * blockDim.x) {
        const int64_t t = k / Hd2, i = k % Hd2;
        const float angle = float(positions[t]) * inv_freq[i];
        cos_out[k] = cosf(angle) * scaling;
        sin_out[k] = sinf(angle) * scaling;
    }
}

template <class X, class TT, class O>
__global__ void rope_apply_kernel(const void* x, const void* cos_t, const void* sin_t, void* out, int64_t B, int64_t T,
                                  int64_t Nh, int64_t Hd2) {
    pdl_wait();
    const int64_t total = B * T * Nh * Hd2;
    for (int64_t k = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; k < total; k += int64_t(gridDim.x) * blockDim.x) {
        const int64_t i = k % Hd2;
        const int64_t bth = k / Hd2;  // (b * T + t) * Nh + h
        const int64_t t = (bth / Nh) % T;
        const int64_t base = bth * 2 * Hd2;
        const float x1 = Elem<X>::load(x, base + i), x2 = Elem<X>::load(x, base + Hd2 + i);
        const float c = Elem<TT>::load(cos_t, t * Hd2 + i), s = Elem<TT>::load(sin_t, t * Hd2 + i);
        Elem<O>::store(out, base + i, x1 * c - x2 * s);
        Elem<O>::store(out, base + Hd2 + i, x1 * s + x2 * c);
    }
}

// One CTA per (b, head) over the q heads, then the k heads, then the v
// heads; Hd/2 threads, thread i owns elements i and i + Hd/2.
template <class T>
__global__ void qk_norm_rope_kernel(const QKNormRope p) {
    pdl_wait();
    __shared__ float red[32];
    const int64_t pos = p.pos_dev ? int64_t(*p.pos_dev) : p.offset;
    if (pos < 0 || pos >= p.Smax || (p.table_rows != 1 && pos >= p.table_rows)) return;
    const int64_t heads = p.Nq + 2 * p.Nkv;
    const int64_t b = blockIdx.x / heads, h = blockIdx.x % heads;
    const int64_t Hd2 = p.Hd / 2;
    const int i = threadIdx.x;
    void* base;
    const float* w;
    bool rope = true;
    if (h < p.Nq) {
        base = static_cast<char*>(p.q) + ((b * p.Nq + h) * p.Hd) * Elem<T>::bytes;
        w = p.q_norm;
    } else if (h < p.Nq + p.Nkv) {
        base = static_cast<char*>(p.k_cache) + (((b * p.Nkv + (h - p.Nq)) * p.Smax + pos) * p.Hd) * Elem<T>::bytes;
        w = p.k_norm;
    } else {
        if (!p.norm_v) return;
        base = static_cast<char*>(p.v_cache) +
               (((b * p.Nkv + (h - p.Nq - p.Nkv)) * p.Smax + pos) * p.Hd) * Elem<T>::bytes;
        w = nullptr;  // Gemma4TextInference.swift:368: the value norm has no weight
        rope = false;
    }
    float x1 = 0.f, x2 = 0.f;
    if (i < Hd2) {
        x1 = Elem<T>::load(base, i);
        x2 = Elem<T>::load(base, Hd2 + i);
    }
    float ss = warp_sum(x1 * x1 + x2 * x2);
    const int lane = i & 31, warp = i >> 5;
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = 0.f;
    const int nw = (blockDim.x + 31) >> 5;
    for (int k = 0; k < nw; ++k) tot += red[k];
    const float scale = rsqrtf(tot / float(p.Hd) + p.eps);
    if (i >= Hd2) return;
    float w1 = 1.f, w2 = 1.f;
    if (w) {
        w1 = p.add_one ? 1.0f + w[i] : w[i];
        w2 = p.add_one ? 1.0f + w[Hd2 + i] : w[Hd2 + i];
    }
    // the normalised head as RMSNorm stores it
    const float y1 = Elem<T>::round(x1 * scale * w1), y2 = Elem<T>::round(x2 * scale * w2);
    if (!rope) {
        Elem<T>::store(base, i, y1);
        Elem<T>::store(base, Hd2 + i, y2);
        return;
    }
    const int64_t row = p.table_rows == 1 ? 0 : pos;
    const float c = p.cos_t[row * Hd2 + i], s = p.sin_t[row * Hd2 + i];
    Elem<T>::store(base, i, y1 * c - y2 * s);
    Elem<T>::store(base, Hd2 + i, y1 * s + y2 * c);
}

template <class X, class TT>
cudaError_t run_rope_o(const RopeApply& p, cudaStream_t s, dim3 g, dim3 b) {
    switch (p.out_dtype) {
    case PC_F32: return launch_k(rope_apply_kernel<X, TT, TF32>, g, b, 0, s, p.x, p.cos_t, p.sin_t, p.out, p.B, p.T, p.Nh, p.Hd2);
    case PC_F16: return launch_k(rope_apply_kernel<X, TT, TF16>, g, b, 0, s, p.x, p.cos_t, p.sin_t, p.out, p.B, p.T, p.Nh, p.Hd2);
    case PC_BF16: return launch_k(rope_apply_kernel<X, TT, TBF16>, g, b, 0, s, p.x, p.cos_t, p.sin_t, p.out, p.B, p.T, p.Nh, p.Hd2);
    }
    return cudaErrorInvalidValue;
}

}  // namespace

cudaError_t rope_build_cos_sin(const int32_t* positions, const float* inv_freq, float* cos_out, float* sin_out,
                               int64_t T, int64_t Hd2, float scaling, cudaStream_t s) {
    const int64_t n = T * Hd2;
    if (n == 0) return cudaSuccess;
    return launch_k(rope_build_kernel, dim3(grid_for(n, 256, current_sm_count())), dim3(256), 0, s, positions,
                    inv_freq, cos_out, sin_out, T, Hd2, scaling);
}

cudaError_t rope_apply(const RopeApply& p, cudaStream_t s) {
    const int64_t n = p.B * p.T * p.Nh * p.Hd2;
    if (n == 0) return cudaSuccess;
    dim3 g(grid_for(n, 256, current_sm_count())), b(256);
    if (p.x_dtype == PC_F32 && p.t_dtype == PC_F32) return run_rope_o<TF32, TF32>(p, s, g, b);
    if (p.x_dtype == PC_BF16 && p.t_dtype == PC_BF16) return run_rope_o<TBF16, TBF16>(p, s, g, b);
    if (p.x_dtype == PC_BF16 && p.t_dtype == PC_F32) return run_rope_o<TBF16, TF32>(p, s, g, b);
    if (p.x_dtype == PC_F16 && p.t_dtype == PC_F32) return run_rope_o<TF16, TF32>(p, s, g, b);
    if (p.x_dtype == PC_F16 && p.t_dtype == PC_F16) return run_rope_o<TF16, TF16>(p, s, g, b);
    return cudaErrorInvalidValue;
}

cudaError_t qk_norm_rope(const QKNormRope& p, cudaStream_t s) {
    const int64_t ctas = p.B * (p.Nq + 2 * p.Nkv);
    if (ctas == 0) return cudaSuccess;
    const unsigned threads = unsigned((p.Hd / 2 + 31) / 32 * 32);
    switch (p.dtype) {
    case PC_F32: return launch_k(qk_norm_rope_kernel<TF32>, dim3(unsigned(ctas)), dim3(threads), 0, s, p);
    case PC_F16: return launch_k(qk_norm_rope_kernel<TF16>, dim3(unsigned(ctas)), dim3(threads), 0, s, p);
    case PC_BF16: return launch_k(qk_norm_rope_kernel<TBF16>, dim3(unsigned(ctas)), dim3(threads), 0, s, p);
    }
    return cudaErrorInvalidValue;
}

namespace {
RegisterFunctions reg_rope({
    {"rope_build_cos_sin", reinterpret_cast<const void*>(rope_build_kernel)},
    {"rope_apply", reinterpret_cast<const void*>(rope_apply_kernel<TF32, TF32, TF32>)},
    {"rope_apply_bf16", reinterpret_cast<const void*>(rope_apply_kernel<TBF16, TBF16, TBF16>)},
    {"rope_apply_f32_tables_bf16", reinterpret_cast<const void*>(rope_apply_kernel<TBF16, TF32, TBF16>)},
    {"rope_apply_f16", reinterpret_cast<const void*>(rope_apply_kernel<TF16, TF16, TF16>)},
    {"rope_apply_f32_tables_f16", reinterpret_cast<const void*>(rope_apply_kernel<TF16, TF32, TF16>)},
    {"qk_norm_rope_bf16", reinterpret_cast<const void*>(qk_norm_rope_kernel<TBF16>)},
    {"qk_norm_rope_f16", reinterpret_cast<const void*>(qk_norm_rope_kernel<TF16>)},
    {"qk_norm_rope", reinterpret_cast<const void*>(qk_norm_rope_kernel<TF32>)},
});
}  // namespace

}  // namespace launch
}  // namespace popcorn
