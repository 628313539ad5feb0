// gemv.cu — the skinny Matmul (m == 1, linear-layer layout) and its fused
// decode forms: RMSNorm prologue, residual-add epilogue, gated-MLP (GeGLU /
// SwiGLU) epilogue and the QKV epilogue that writes K and V straight into
// the cache.
//
// Semantics: y[n] = sum_k x[k] * W[n,k] in fp32 with one rounding at the
// store (Matvec.metal:56-127); fused forms keep the reference's rounding
// points between ops (each intermediate is what the unfused op would have
// stored in the activation dtype).
//
// B200 design. The op is HBM-bound: every weight byte is read once, 2 bytes
// per 2 FLOPs. Each warp owns ROWS rows; each lane streams 16-byte chunks of
// its rows with ld.global.nc.L1::no_allocate (no L1 pollution), several
// chunks per row in flight, double-buffered in registers so the next batch
// is in flight while the current one is reduced. The activation row is
// converted to fp32 once per CTA into shared memory, split into two float4
// planes (elements 0-3 / 4-7 of every chunk) so a warp's x reads are
// conflict-free. The first weight batch is issued before griddepcontrol.wait,
// so under programmatic dependent launch the weight stream starts while the
// previous kernel is still draining.
#include "common.cuh"
#include "dtype.cuh"
#include "launch.hpp"
#include "popcorn.hpp"

namespace popcorn {
namespace launch {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

template <class WT> struct WVec { static constexpr int n = 8; };
template <> struct WVec<TF32> { static constexpr int n = 4; };

template <class WT>
__device__ __forceinline__ void widen(const uint4& v, float* f) {
    if constexpr (WVec<WT>::n == 8) {
        unpack8<WT>(v, f);
    } else {
        f[0] = __uint_as_float(v.x); f[1] = __uint_as_float(v.y);
        f[2] = __uint_as_float(v.z); f[3] = __uint_as_float(v.w);
    }
}

template <class OT, int EPI>
__device__ __forceinline__ void gemv_store(const Gemv& p, int64_t n, float a, float b, int64_t pos) {
    if constexpr (EPI == int(Epilogue::kStore)) {
        Elem<OT>::store(p.out, n, a);
    } else if constexpr (EPI == int(Epilogue::kResidual)) {
        float y = Elem<OT>::round(a);
        Elem<OT>::store(p.out, n, y + Elem<OT>::load(p.residual, n));
    } else if constexpr (EPI == int(Epilogue::kGated)) {
        float g = Elem<OT>::round(a);
        float u = Elem<OT>::round(b);
        float act = Elem<OT>::round(p.activation == 0 ? gelu_tanh(g) : silu(g));
        Elem<OT>::store(p.out, n, act * u);
    } else {  // kQKV
        if (n < p.q_rows) {
            Elem<OT>::store(p.out, n, a);
        } else {
            int64_t r = n - p.q_rows;
            void* cache = p.k_cache;
            if (r >= p.kv_rows) {
                r -= p.kv_rows;
                cache = p.v_cache;
            }
            int64_t h = r / p.Hd, d = r % p.Hd;
            if (pos >= 0 && pos < p.Smax) Elem<OT>::store(cache, (h * p.Smax + pos) * p.Hd + d, a);
        }
    }
}

// Vectorised kernel: K % VEC == 0, W rows 16-byte aligned, K*4 bytes of x
// fit in shared memory.
template <class XT, class WT, class OT, int ROWS, int U, bool NORM, int EPI>
__global__ void __launch_bounds__(kThreads) gemv_vec_kernel(const Gemv p) {
    constexpr int VEC = WVec<WT>::n;
    constexpr int NR = (EPI == int(Epilogue::kGated) ? 2 : 1) * ROWS;
    extern __shared__ float4 xs[];  // [nchunks] lo plane, then [nchunks] hi plane (VEC == 8)
    __shared__ float red[kWarps];
    __shared__ float s_scale;

    pdl_launch_dependents();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t K = p.K;
    const int nchunks = int(K / VEC);
    const int64_t n0 = (int64_t(blockIdx.x) * kWarps + warp) * ROWS;
    constexpr int es = Elem<WT>::bytes;

    const char* wp[NR];
    bool valid[NR];
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
        int64_t n = n0 + r;
        bool v = n < p.N;
        int64_t nn = v ? n : 0;
        if constexpr (EPI == int(Epilogue::kGated)) {
            wp[2 * r] = static_cast<const char*>(p.w) + nn * K * es;
            wp[2 * r + 1] = static_cast<const char*>(p.w2) + nn * K * es;
            valid[2 * r] = valid[2 * r + 1] = v;
        } else {
            wp[r] = static_cast<const char*>(p.w) + nn * K * es;
            valid[r] = v;
        }
    }

    uint4 cur[NR][U];
    auto load_batch = [&](uint4 (&dst)[NR][U], int c0) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
            int c = c0 + 32 * u;
#pragma unroll
            for (int r = 0; r < NR; ++r)
                if (valid[r] && c < nchunks) dst[r][u] = ldg_stream(wp[r] + int64_t(c) * 16);
        }
    };
    // Weights do not depend on the previous kernel: start streaming them now.
    load_batch(cur, lane);

    pdl_wait();

    // Activation row -> fp32 shared memory (optionally RMS-normalised and
    // rounded to the activation dtype, as RMSNorm would have stored it).
    float ss = 0.f;
    for (int64_t i = tid; i < K; i += kThreads) {
        float v = Elem<XT>::load(p.x, i);
        if constexpr (NORM) ss += v * v;
        int c = int(i / VEC), e = int(i % VEC);
        float* plane = reinterpret_cast<float*>(xs + (e < 4 ? 0 : nchunks) + c);
        plane[e & 3] = v;
    }
    if constexpr (NORM) {
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        if (warp == 0) {
            float v = lane < kWarps ? red[lane] : 0.f;
            v = warp_sum(v);
            if (lane == 0) s_scale = rsqrtf(v / float(K) + p.eps);
        }
        __syncthreads();
        float scale = s_scale;
        for (int64_t i = tid; i < K; i += kThreads) {
            int c = int(i / VEC), e = int(i % VEC);
            float* plane = reinterpret_cast<float*>(xs + (e < 4 ? 0 : nchunks) + c);
            float v = plane[e & 3] * scale;
            if (p.norm_weight) {
                float w = p.norm_weight[i];
                if (p.add_one) w = 1.0f + w;
                v *= w;
            }
            plane[e & 3] = Elem<XT>::round(v);
        }
    }
    __syncthreads();

    float acc[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) acc[r] = 0.f;

    for (int c0 = lane; c0 < nchunks; c0 += 32 * U) {
        uint4 nxt[NR][U];
        if (c0 + 32 * U < nchunks) load_batch(nxt, c0 + 32 * U);
#pragma unroll
        for (int u = 0; u < U; ++u) {
            int c = c0 + 32 * u;
            if (c < nchunks) {
                float xf[8];
                float4 lo = xs[c];
                xf[0] = lo.x; xf[1] = lo.y; xf[2] = lo.z; xf[3] = lo.w;
                if constexpr (VEC == 8) {
                    float4 hi = xs[nchunks + c];
                    xf[4] = hi.x; xf[5] = hi.y; xf[6] = hi.z; xf[7] = hi.w;
                }
#pragma unroll
                for (int r = 0; r < NR; ++r) {
                    float wf[8];
                    widen<WT>(cur[r][u], wf);
                    float a = acc[r];
#pragma unroll
                    for (int e = 0; e < VEC; ++e) a = fmaf(xf[e], wf[e], a);
                    acc[r] = a;
                }
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
            for (int r = 0; r < NR; ++r) cur[r][u] = nxt[r][u];
    }

#pragma unroll
    for (int r = 0; r < NR; ++r) acc[r] = warp_sum(acc[r]);

    int64_t pos = -1;
    if constexpr (EPI == int(Epilogue::kQKV)) pos = p.pos_dev ? int64_t(*p.pos_dev) : p.offset;
    if (lane == 0) {
#pragma unroll
        for (int r = 0; r < ROWS; ++r) {
            int64_t n = n0 + r;
            if (n >= p.N) break;
            if constexpr (EPI == int(Epilogue::kGated))
                gemv_store<OT, EPI>(p, n, acc[2 * r], acc[2 * r + 1], pos);
            else
                gemv_store<OT, EPI>(p, n, acc[r], 0.f, pos);
        }
    }
}

// Generic kernel for any K / alignment: one warp per output row, scalar
// loads; x (optionally normalised) staged in shared memory as fp32.
template <class XT, class WT, class OT, bool NORM, int EPI>
__global__ void __launch_bounds__(kThreads) gemv_scalar_kernel(const Gemv p) {
    extern __shared__ float xsf[];
    __shared__ float red[kWarps];
    __shared__ float s_scale;
    pdl_launch_dependents();
    pdl_wait();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t K = p.K;
    float ss = 0.f;
    for (int64_t i = tid; i < K; i += kThreads) {
        float v = Elem<XT>::load(p.x, i);
        ss += v * v;
        xsf[i] = v;
    }
    if constexpr (NORM) {
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        if (warp == 0) {
            float v = lane < kWarps ? red[lane] : 0.f;
            v = warp_sum(v);
            if (lane == 0) s_scale = rsqrtf(v / float(K) + p.eps);
        }
        __syncthreads();
        float scale = s_scale;
        for (int64_t i = tid; i < K; i += kThreads) {
            float v = xsf[i] * scale;
            if (p.norm_weight) {
                float w = p.norm_weight[i];
                if (p.add_one) w = 1.0f + w;
                v *= w;
            }
            xsf[i] = Elem<XT>::round(v);
        }
    }
    __syncthreads();
    int64_t n = int64_t(blockIdx.x) * kWarps + warp;
    if (n >= p.N) return;
    float a = 0.f, b = 0.f;
    for (int64_t k = lane; k < K; k += 32) {
        a = fmaf(xsf[k], Elem<WT>::load(p.w, n * K + k), a);
        if constexpr (EPI == int(Epilogue::kGated)) b = fmaf(xsf[k], Elem<WT>::load(p.w2, n * K + k), b);
    }
    a = warp_sum(a);
    if constexpr (EPI == int(Epilogue::kGated)) b = warp_sum(b);
    int64_t pos = -1;
    if constexpr (EPI == int(Epilogue::kQKV)) pos = p.pos_dev ? int64_t(*p.pos_dev) : p.offset;
    if (lane == 0) gemv_store<OT, EPI>(p, n, a, b, pos);
}

constexpr size_t kMaxSmem = 200 * 1024;

template <class XT, class WT, class OT, int ROWS, int U, bool NORM, int EPI>
cudaError_t run_vec(const Gemv& p, cudaStream_t s) {
    auto kern = gemv_vec_kernel<XT, WT, OT, ROWS, U, NORM, EPI>;
    size_t smem = size_t(p.K) * 4;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = allow_smem(kern, kMaxSmem);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    int64_t rows_per_cta = int64_t(kWarps) * ROWS;
    int64_t grid = (p.N + rows_per_cta - 1) / rows_per_cta;
    return launch_k(kern, dim3(unsigned(grid)), dim3(kThreads), smem, s, p);
}

template <class XT, class WT, class OT, bool NORM, int EPI>
cudaError_t run_scalar(const Gemv& p, cudaStream_t s) {
    auto kern = gemv_scalar_kernel<XT, WT, OT, NORM, EPI>;
    size_t smem = size_t(p.K) * 4;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = allow_smem(kern, kMaxSmem);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    int64_t grid = (p.N + kWarps - 1) / kWarps;
    return launch_k(kern, dim3(unsigned(grid)), dim3(kThreads), smem, s, p);
}

// Rows per warp: enough CTAs to cover every SM at least ~3 times over.
template <class XT, class WT, class OT, bool NORM, int EPI>
cudaError_t dispatch_rows(const Gemv& p, cudaStream_t s) {
    constexpr int VEC = WVec<WT>::n;
    bool vec_ok = (p.K % VEC == 0) && aligned16(p.w) && (EPI != int(Epilogue::kGated) || aligned16(p.w2));
    if (!vec_ok) return run_scalar<XT, WT, OT, NORM, EPI>(p, s);
    int sms = current_sm_count();
    int64_t ctas_rows2 = (p.N + 2 * kWarps - 1) / (2 * kWarps);
    if (EPI != int(Epilogue::kGated) && ctas_rows2 >= int64_t(sms) * 4)
        return run_vec<XT, WT, OT, 2, 4, NORM, EPI>(p, s);
    return run_vec<XT, WT, OT, 1, 4, NORM, EPI>(p, s);
}

template <class XT, class WT, class OT>
cudaError_t dispatch_epi(const Gemv& p, cudaStream_t s) {
    switch (p.epilogue) {
    case Epilogue::kStore:
        return p.has_norm ? dispatch_rows<XT, WT, OT, true, 0>(p, s) : dispatch_rows<XT, WT, OT, false, 0>(p, s);
    case Epilogue::kResidual:
        return dispatch_rows<XT, WT, OT, false, 1>(p, s);
    case Epilogue::kGated:
        return p.has_norm ? dispatch_rows<XT, WT, OT, true, 2>(p, s) : dispatch_rows<XT, WT, OT, false, 2>(p, s);
    case Epilogue::kQKV:
        return dispatch_rows<XT, WT, OT, true, 3>(p, s);
    }
    return cudaErrorInvalidValue;
}

// Plain matvec forms (any dtype combination the op accepts).
template <class XT, class WT, class OT>
cudaError_t dispatch_plain(const Gemv& p, cudaStream_t s) {
    return dispatch_rows<XT, WT, OT, false, 0>(p, s);
}

}  // namespace

cudaError_t gemv(const Gemv& p, cudaStream_t s) {
    if (p.N == 0) return cudaSuccess;
    if (size_t(p.K) * 4 > kMaxSmem) {
        if (p.epilogue != Epilogue::kStore || p.has_norm) return cudaErrorInvalidValue;
        Matmul m{p.x, p.x_dtype, p.w, p.w_dtype, p.out, p.out_dtype, 1, p.K, p.N, 1};
        return matmul(m, s);
    }
    int x = p.x_dtype, w = p.w_dtype, o = p.out_dtype;
    bool fused = p.has_norm || p.epilogue != Epilogue::kStore;
    if (fused) {
        if (x == PC_BF16 && w == PC_BF16 && o == PC_BF16) return dispatch_epi<TBF16, TBF16, TBF16>(p, s);
        if (x == PC_F16 && w == PC_F16 && o == PC_F16) return dispatch_epi<TF16, TF16, TF16>(p, s);
        return cudaErrorInvalidValue;
    }
    if (x == PC_F32 && w == PC_F32 && o == PC_F32) return dispatch_plain<TF32, TF32, TF32>(p, s);
    if (w == PC_BF16) {
        if (x == PC_F32 && o == PC_F32) return dispatch_plain<TF32, TBF16, TF32>(p, s);
        if (x == PC_BF16 && o == PC_F32) return dispatch_plain<TBF16, TBF16, TF32>(p, s);
        if (x == PC_BF16 && o == PC_BF16) return dispatch_plain<TBF16, TBF16, TBF16>(p, s);
        if (x == PC_F32 && o == PC_BF16) return dispatch_plain<TF32, TBF16, TBF16>(p, s);
    }
    if (w == PC_F16) {
        if (x == PC_F32 && o == PC_F32) return dispatch_plain<TF32, TF16, TF32>(p, s);
        if (x == PC_F16 && o == PC_F32) return dispatch_plain<TF16, TF16, TF32>(p, s);
        if (x == PC_F16 && o == PC_F16) return dispatch_plain<TF16, TF16, TF16>(p, s);
        if (x == PC_F32 && o == PC_F16) return dispatch_plain<TF32, TF16, TF16>(p, s);
    }
    return cudaErrorInvalidValue;
}

namespace {
RegisterFunctions reg_gemv({
    {"matvec_nk_f32_f32_f32", reinterpret_cast<const void*>(gemv_vec_kernel<TF32, TF32, TF32, 1, 4, false, 0>)},
    {"matvec_nk_f32_bf16_f32", reinterpret_cast<const void*>(gemv_vec_kernel<TF32, TBF16, TF32, 1, 4, false, 0>)},
    {"matvec_nk_bf16_bf16_f32", reinterpret_cast<const void*>(gemv_vec_kernel<TBF16, TBF16, TF32, 1, 4, false, 0>)},
    {"matvec_nk_bf16_bf16_bf16", reinterpret_cast<const void*>(gemv_vec_kernel<TBF16, TBF16, TBF16, 1, 4, false, 0>)},
    {"matvec_nk_f32_bf16_bf16", reinterpret_cast<const void*>(gemv_vec_kernel<TF32, TBF16, TBF16, 1, 4, false, 0>)},
    {"matvec_nk_f32_f16_f32", reinterpret_cast<const void*>(gemv_vec_kernel<TF32, TF16, TF32, 1, 4, false, 0>)},
    {"matvec_nk_f16_f16_f32", reinterpret_cast<const void*>(gemv_vec_kernel<TF16, TF16, TF32, 1, 4, false, 0>)},
    {"matvec_nk_f16_f16_f16", reinterpret_cast<const void*>(gemv_vec_kernel<TF16, TF16, TF16, 1, 4, false, 0>)},
    {"matvec_nk_f32_f16_f16", reinterpret_cast<const void*>(gemv_vec_kernel<TF32, TF16, TF16, 1, 4, false, 0>)},
    {"rmsnorm_matvec_bf16", reinterpret_cast<const void*>(gemv_vec_kernel<TBF16, TBF16, TBF16, 1, 4, true, 0>)},
    {"rmsnorm_matvec_f16", reinterpret_cast<const void*>(gemv_vec_kernel<TF16, TF16, TF16, 1, 4, true, 0>)},
    {"matvec_residual_bf16", reinterpret_cast<const void*>(gemv_vec_kernel<TBF16, TBF16, TBF16, 1, 4, false, 1>)},
    {"matvec_residual_f16", reinterpret_cast<const void*>(gemv_vec_kernel<TF16, TF16, TF16, 1, 4, false, 1>)},
    {"geglu_matvec_bf16", reinterpret_cast<const void*>(gemv_vec_kernel<TBF16, TBF16, TBF16, 1, 4, true, 2>)},
    {"geglu_matvec_f16", reinterpret_cast<const void*>(gemv_vec_kernel<TF16, TF16, TF16, 1, 4, true, 2>)},
    {"swiglu_matvec_bf16", reinterpret_cast<const void*>(gemv_vec_kernel<TBF16, TBF16, TBF16, 1, 4, false, 2>)},
    {"swiglu_matvec_f16", reinterpret_cast<const void*>(gemv_vec_kernel<TF16, TF16, TF16, 1, 4, false, 2>)},
    {"qkv_matvec_bf16", reinterpret_cast<const void*>(gemv_vec_kernel<TBF16, TBF16, TBF16, 1, 4, true, 3>)},
    {"qkv_matvec_f16", reinterpret_cast<const void*>(gemv_vec_kernel<TF16, TF16, TF16, 1, 4, true, 3>)},
});
}  // namespace

}  // namespace launch
}  // namespace popcorn
