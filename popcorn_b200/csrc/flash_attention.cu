// flash_attention.cu — prefill attention (Sq >= 1), CUDA-core path.
//
// Semantics (FlashAttention.metal:31-162): query row q of (b, hq) sits at
// position posQ = Sk - Sq + q (:73-76) and attends to the keys its mask
// allows (:97-99): causal j <= posQ, sliding window additionally
// posQ - j < window, bidirectional all; q is pre-scaled; online softmax in
// fp32 with natural exp (as exp2 of log2e-scaled scores); O / l stored once.
//
// One warp per query row, lanes over head dims, keys streamed from L2.
// Sequences long enough for the tensor cores (16-bit, Sq >= 32) are served
// by the tcgen05 kernel in fa_tcgen05.cu instead.
#include "common.cuh"
#include "dtype.cuh"
#include "launch.hpp"
#include "popcorn.hpp"

namespace popcorn {
namespace launch {

namespace {

constexpr float kLog2e = 1.4426950408889634f;

template <class QT, class KV, class OT>
__global__ void __launch_bounds__(128) fa_plain_kernel(const FlashAttention p) {
    constexpr int MAXE = 16;  // Hd <= 512
    pdl_launch_dependents();
    pdl_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t qi = int64_t(blockIdx.x) * 4 + warp;
    const int64_t hq = blockIdx.y, b = blockIdx.z;
    if (qi >= p.Sq) return;
    const int64_t Hd = p.Hd;
    const int64_t hkv = hq * p.Nkv / p.Nq;
    const int64_t posQ = p.Sk - p.Sq + qi;
    const int64_t qb = ((b * p.Nq + hq) * p.Sq + qi) * Hd;
    const int64_t kv0 = (b * p.Nkv + hkv) * p.Sk;
    float q[MAXE], o[MAXE];
    const float qs = p.scale * kLog2e;
#pragma unroll
    for (int i = 0; i < MAXE; ++i) {
        int64_t d = lane + 32 * i;
        q[i] = d < Hd ? Elem<QT>::load(p.q, qb + d) * qs : 0.f;
        o[i] = 0.f;
    }
    int64_t jlo = 0, jhi = p.Sk;  // allowed keys [jlo, jhi)
    if (p.mask_kind != 2) jhi = posQ + 1 < p.Sk ? posQ + 1 : p.Sk;
    if (p.mask_kind == 1) jlo = posQ - p.window + 1 > 0 ? posQ - p.window + 1 : 0;
    float m = -INFINITY, l = 0.f;
    for (int64_t j = jlo; j < jhi; ++j) {
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < MAXE; ++i) {
            int64_t d = lane + 32 * i;
            if (d < Hd) acc = fmaf(q[i], Elem<KV>::load(p.k, (kv0 + j) * Hd + d), acc);
        }
        float sv = warp_sum(acc);
        float mnew = fmaxf(m, sv);
        float so = exp2f(m - mnew);
        float pv = exp2f(sv - mnew);
        l = l * so + pv;
        m = mnew;
#pragma unroll
        for (int i = 0; i < MAXE; ++i) {
            int64_t d = lane + 32 * i;
            float vv = d < Hd ? Elem<KV>::load(p.v, (kv0 + j) * Hd + d) : 0.f;
            o[i] = fmaf(pv, vv, o[i] * so);
        }
    }
    const float inv_l = l > 0.f ? 1.0f / l : 0.f;
#pragma unroll
    for (int i = 0; i < MAXE; ++i) {
        int64_t d = lane + 32 * i;
        if (d < Hd) Elem<OT>::store(p.out, qb + d, o[i] * inv_l);
    }
}

template <class QT, class KV>
cudaError_t run_plain_o(const FlashAttention& p, cudaStream_t s) {
    dim3 grid(unsigned((p.Sq + 3) / 4), unsigned(p.Nq), unsigned(p.B));
    switch (p.out_dtype) {
    case PC_F32: return launch_k(fa_plain_kernel<QT, KV, TF32>, grid, dim3(128), 0, s, p);
    case PC_F16: return launch_k(fa_plain_kernel<QT, KV, TF16>, grid, dim3(128), 0, s, p);
    case PC_BF16: return launch_k(fa_plain_kernel<QT, KV, TBF16>, grid, dim3(128), 0, s, p);
    }
    return cudaErrorInvalidValue;
}

template <class QT>
cudaError_t run_plain_kv(const FlashAttention& p, cudaStream_t s) {
    switch (p.kv_dtype) {
    case PC_F32: return run_plain_o<QT, TF32>(p, s);
    case PC_F16: return run_plain_o<QT, TF16>(p, s);
    case PC_BF16: return run_plain_o<QT, TBF16>(p, s);
    }
    return cudaErrorInvalidValue;
}

}  // namespace

cudaError_t flash_attention_tcgen05(const FlashAttention& p, cudaStream_t s);
bool fa_tcgen05_supports(const FlashAttention& p);

bool flash_attention_uses_tensor_cores(const FlashAttention& p) { return fa_tcgen05_supports(p); }

cudaError_t flash_attention(const FlashAttention& p, cudaStream_t s) {
    if (fa_tcgen05_supports(p)) return flash_attention_tcgen05(p, s);
    switch (p.q_dtype) {
    case PC_F32: return run_plain_kv<TF32>(p, s);
    case PC_F16: return run_plain_kv<TF16>(p, s);
    case PC_BF16: return run_plain_kv<TBF16>(p, s);
    }
    return cudaErrorInvalidValue;
}

namespace {
RegisterFunctions reg_fa({
    {"flash_attention", reinterpret_cast<const void*>(fa_plain_kernel<TF32, TF32, TF32>)},
    {"flash_attention_bf16", reinterpret_cast<const void*>(fa_plain_kernel<TBF16, TBF16, TBF16>)},
    {"flash_attention_bf16_to_f32", reinterpret_cast<const void*>(fa_plain_kernel<TBF16, TBF16, TF32>)},
    {"flash_attention_f32_bf16_to_bf16", reinterpret_cast<const void*>(fa_plain_kernel<TF32, TBF16, TBF16>)},
    {"flash_attention_f16", reinterpret_cast<const void*>(fa_plain_kernel<TF16, TF16, TF16>)},
});
}  // namespace

}  // namespace launch
}  // namespace popcorn
