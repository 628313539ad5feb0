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
// per 2 FLOPs. One persistent CTA per SM: a producer warp streams 8-row x
// kc-column weight tiles HBM -> shared memory with 1-D bulk copies
// (cp.async.bulk, no multicast) into a 2-8 stage mbarrier ring of up to
// ~150 KB (short matvecs) or ~190 KB (long ones), starting before griddepcontrol.wait (weights never depend on the
// previous kernel, so under programmatic dependent launch the stream starts
// while that kernel drains). Eight consumer warps own one weight row each
// per stage; the activation row is converted to fp32 once per CTA into
// shared memory, split into two float4 planes (elements 0-3 / 4-7 of every
// 16-byte chunk) so a warp's x reads are conflict-free. Rows whose length
// is not a multiple of 16 bytes use a plain one-warp-per-row kernel.
#include <cstdlib>

#include "async.cuh"
#include "common.cuh"
#include "dtype.cuh"
#include "launch.hpp"
#include "popcorn.hpp"

namespace popcorn {

__device__ unsigned int g_gemv_error_word;

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

// Bulk-copy kernel: K % VEC == 0 and 16-byte aligned weight rows.
//
// One CTA per SM (persistent): warp 8 is the producer, warps 0-7 consume.
// A tile is 8 outputs; a stage holds their 8 rows of one weight matrix
// (gated: W_gate and W_up in alternate stages) over kc columns. When kc is
// the whole row the 8 rows are contiguous and the stage is ONE bulk copy:
// the copy engine streams at full rate only with stages of about 16 KB or
// more in few copies (8 copies of 2.3 KB reach ~4.5 TB/s, one of 18-37 KB
// ~7.3 TB/s on B200). The producer fills the ring before the CTA waits for
// its predecessor (griddepcontrol.wait): weights never depend on it. Each
// consumer warp owns one output (its gate and up rows when gated), lanes
// stride 16-byte chunks (conflict-free shared loads), and the k-chunks of a
// row accumulate in registers until the warp reduction and the epilogue.
struct GemvPlan {
    int kc;           // columns per stage (multiple of 8)
    int nkc;          // stages per tile
    int ntiles;       // tiles of 8 outputs
    int stages;       // ring depth
    int stage_bytes;  // 8 rows * kc * elem
};

constexpr int kConsumers = 8;
constexpr int kTmaThreads = (kConsumers + 1) * 32;

template <class XT, class WT, class OT, bool NORM, int EPI>
__global__ void __launch_bounds__(kTmaThreads, 1) gemv_tma_kernel(const Gemv p, const GemvPlan g) {
    constexpr int VEC = WVec<WT>::n;
    constexpr int es = Elem<WT>::bytes;
    constexpr bool GATED = EPI == int(Epilogue::kGated);
    constexpr int R = GATED ? 2 : 1;  // weight rows per output
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t full[8], empty[8];
    __shared__ float red[kConsumers];
    __shared__ float s_scale;
    __shared__ volatile int s_abort;
    __shared__ volatile int s_issued;
    __shared__ volatile int s_consumed;

    pdl_launch_dependents();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t K = p.K;
    const int nx = int(K / VEC);  // 16-byte chunks of a full row
    unsigned char* ring = smem;
    float4* xs = reinterpret_cast<float4*>(smem + size_t(g.stages) * g.stage_bytes);

    // The norm weights depend on nothing: the consumers request them before
    // the producer issues the ring's bulk copies, so they do not queue
    // behind the ring's weight traffic on this SM.
    constexpr bool kX16 = Elem<XT>::bytes == 2 && VEC == 8;
    constexpr int kXC = 8;  // chunks per thread: rows up to 8 * 8 * 256 elements
    const bool chunked = kX16 && K <= int64_t(kXC) * 8 * kConsumers * 32 &&
                         (reinterpret_cast<uintptr_t>(p.x) & 15) == 0;
    float4 nwv[NORM ? kXC : 1][2];
    const bool nw_chunked = NORM && chunked && p.norm_weight && (reinterpret_cast<uintptr_t>(p.norm_weight) & 15) == 0;
    if constexpr (NORM) {
        if (nw_chunked && warp < kConsumers) {
#pragma unroll
            for (int j = 0; j < kXC; ++j) {
                const int c = tid + j * kConsumers * 32;
                if (c < nx) {
                    nwv[j][0] = __ldg(reinterpret_cast<const float4*>(p.norm_weight) + 2 * c);
                    nwv[j][1] = __ldg(reinterpret_cast<const float4*>(p.norm_weight) + 2 * c + 1);
                }
            }
        }
    }

    if (tid == 0) {
        for (int s = 0; s < g.stages; ++s) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), kConsumers);
        }
        s_abort = 0;
        s_issued = 0;
        s_consumed = 0;
        mbar_fence_init();
    }
    __syncthreads();

    if (warp == kConsumers) {
        // ---- producer ----
        if (lane == 0) {
            int it = 0;
            for (int tile = blockIdx.x; tile < g.ntiles; tile += gridDim.x) {
                for (int kci = 0; kci < g.nkc && !s_abort; ++kci) {
                    const int64_t k0 = int64_t(kci) * g.kc;
                    const int kcols = int(K - k0 < g.kc ? K - k0 : g.kc);
                    const uint32_t row_bytes = uint32_t(kcols) * es;
                    const int64_t n0 = int64_t(tile) * 8;
                    const int nvalid = int(p.N - n0 < 8 ? p.N - n0 : 8);
                    for (int m = 0; m < R; ++m, ++it) {
                        const int s = it % g.stages;
                        const uint32_t ph = uint32_t(it / g.stages) & 1u;
                        if (s_abort || !mbar_wait(smem_u32(&empty[s]), ph ^ 1u, &g_gemv_error_word)) {
                            s_abort = 1;
                            break;
                        }
                        const uint32_t bar = smem_u32(&full[s]);
                        mbar_expect_tx(bar, row_bytes * nvalid);
                        unsigned char* st = ring + size_t(s) * g.stage_bytes;
                        const char* base = static_cast<const char*>(m == 0 ? p.w : p.w2);
                        if (kcols == K) {
                            bulk_g2s(smem_u32(st), base + n0 * K * es, row_bytes * nvalid, bar);
                        } else {
                            for (int r = 0; r < nvalid; ++r)
                                bulk_g2s(smem_u32(st + size_t(r) * g.kc * es), base + ((n0 + r) * K + k0) * es,
                                         row_bytes, bar);
                        }
                        s_issued = it + 1;
                    }
                }
                if (s_abort) break;
            }
            // Own loads issued: warm L2 for the next kernel of the chain.
            for (int r = 0; r < 2; ++r) prefetch_share_l2(p.pf.ptr[r], p.pf.bytes[r], blockIdx.x, gridDim.x);
        }
    } else {
        // ---- consumers ----
        // 16-bit x in 16-byte chunks (one load per 8 elements, all in flight
        // at once); the norm weights depend on nothing and load before the
        // wait for the previous kernel.
        pdl_wait();
        float ss = 0.f;
        auto stage_scalar = [&]() {
            for (int64_t i = tid; i < K; i += kConsumers * 32) {
                float v = Elem<XT>::load(p.x, i);
                if constexpr (NORM) ss += v * v;
                int c = int(i / VEC), e = int(i % VEC);
                float* plane = reinterpret_cast<float*>(xs + (e < 4 ? 0 : nx) + c);
                plane[e & 3] = v;
            }
        };
        if constexpr (!kX16) {
            stage_scalar();
        } else if (chunked) {
            uint4 xr[kXC];
#pragma unroll
            for (int j = 0; j < kXC; ++j) {
                const int c = tid + j * kConsumers * 32;
                if (c < nx) xr[j] = __ldcg(reinterpret_cast<const uint4*>(p.x) + c);
            }
#pragma unroll
            for (int j = 0; j < kXC; ++j) {
                const int c = tid + j * kConsumers * 32;
                if (c < nx) {
                    float f[8];
                    unpack8<XT>(xr[j], f);
                    if constexpr (NORM)
#pragma unroll
                        for (int e = 0; e < 8; ++e) ss += f[e] * f[e];
                    xs[c] = make_float4(f[0], f[1], f[2], f[3]);
                    xs[nx + c] = make_float4(f[4], f[5], f[6], f[7]);
                }
            }
        } else {
            stage_scalar();
        }
        if constexpr (NORM) {
            ss = warp_sum(ss);
            if (lane == 0) red[warp] = ss;
            named_sync(1, kConsumers * 32);
            if (warp == 0) {
                float v = lane < kConsumers ? red[lane] : 0.f;
                v = warp_sum(v);
                if (lane == 0) s_scale = rsqrtf(v / float(K) + p.eps);
            }
            named_sync(1, kConsumers * 32);
            const float scale = s_scale;
            if (chunked) {
                // each thread rewrites the chunks it staged (no barrier needed)
#pragma unroll
                for (int j = 0; j < kXC; ++j) {
                    const int c = tid + j * kConsumers * 32;
                    if (c < nx) {
                        const float4 lo = xs[c], hi = xs[nx + c];
                        float f[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
                        float w[8] = {1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f};
                        if (nw_chunked) {
                            const float4 a = nwv[j][0], b = nwv[j][1];
                            const float ww[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
                            for (int e = 0; e < 8; ++e) w[e] = p.add_one ? 1.0f + ww[e] : ww[e];
                        } else if (p.norm_weight) {
#pragma unroll
                            for (int e = 0; e < 8; ++e) {
                                const float ww = p.norm_weight[int64_t(c) * 8 + e];
                                w[e] = p.add_one ? 1.0f + ww : ww;
                            }
                        }
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            float v = f[e] * scale;
                            if (p.norm_weight) v *= w[e];
                            f[e] = Elem<XT>::round(v);
                        }
                        xs[c] = make_float4(f[0], f[1], f[2], f[3]);
                        xs[nx + c] = make_float4(f[4], f[5], f[6], f[7]);
                    }
                }
            } else {
                for (int64_t i = tid; i < K; i += kConsumers * 32) {
                    int c = int(i / VEC), e = int(i % VEC);
                    float* plane = reinterpret_cast<float*>(xs + (e < 4 ? 0 : nx) + c);
                    float v = plane[e & 3] * scale;
                    if (p.norm_weight) {
                        float w = p.norm_weight[i];
                        if (p.add_one) w = 1.0f + w;
                        v *= w;
                    }
                    plane[e & 3] = Elem<XT>::round(v);
                }
            }
        }
        named_sync(1, kConsumers * 32);

        int64_t pos = -1;
        if constexpr (EPI == int(Epilogue::kQKV)) pos = p.pos_dev ? int64_t(*p.pos_dev) : p.offset;

        int it = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < g.ntiles && ok; tile += gridDim.x) {
            const int64_t n = int64_t(tile) * 8 + warp;
            const bool valid = n < p.N;
            float acc[R];
#pragma unroll
            for (int m = 0; m < R; ++m) acc[m] = 0.f;
            for (int kci = 0; kci < g.nkc && ok; ++kci) {
                const int64_t k0 = int64_t(kci) * g.kc;
                const int kcols = int(K - k0 < g.kc ? K - k0 : g.kc);
                const int c0 = int(k0 / VEC);
                const int nc = kcols / VEC;
                // whole rows: the stage's row pitch is kcols (== K)
                const int pitch = kcols == K ? kcols : g.kc;
#pragma unroll
                for (int m = 0; m < R; ++m, ++it) {
                    const int s = it % g.stages;
                    const uint32_t ph = uint32_t(it / g.stages) & 1u;
                    if (s_abort || !mbar_wait(smem_u32(&full[s]), ph, &g_gemv_error_word)) {
                        s_abort = 1;
                        ok = false;
                        break;
                    }
                    if (valid) {
                        const unsigned char* row = ring + size_t(s) * g.stage_bytes + size_t(warp) * pitch * es;
                        float a = acc[m];
#pragma unroll 4
                        for (int c = lane; c < nc; c += 32) {
                            uint4 wv = *reinterpret_cast<const uint4*>(row + size_t(c) * 16);
                            float wf[8];
                            widen<WT>(wv, wf);
                            float4 lo = xs[c0 + c];
                            a = fmaf(lo.x, wf[0], a);
                            a = fmaf(lo.y, wf[1], a);
                            a = fmaf(lo.z, wf[2], a);
                            a = fmaf(lo.w, wf[3], a);
                            if constexpr (VEC == 8) {
                                float4 hi = xs[nx + c0 + c];
                                a = fmaf(hi.x, wf[4], a);
                                a = fmaf(hi.y, wf[5], a);
                                a = fmaf(hi.z, wf[6], a);
                                a = fmaf(hi.w, wf[7], a);
                            }
                        }
                        acc[m] = a;
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(smem_u32(&empty[s]));
                    if (warp == 0 && lane == 0) s_consumed = it + 1;
                }
            }
            if (!ok) break;
#pragma unroll
            for (int m = 0; m < R; ++m) acc[m] = warp_sum(acc[m]);
            if (lane == 0 && valid) gemv_store<OT, EPI>(p, n, acc[0], R > 1 ? acc[R - 1] : 0.f, pos);
        }
    }
    __syncthreads();
    if (s_abort && tid == 0) {
        // A wait gave up: drain (bounded) the copies that were issued but not
        // consumed, so none lands after the CTA has left.
        for (int j = s_consumed; j < s_issued; ++j)
            mbar_wait(smem_u32(&full[j % g.stages]), uint32_t(j / g.stages) & 1u, &g_gemv_error_word);
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

constexpr size_t kTmaSmemBudget = 200 * 1024;  // upper bound (the attribute set once per kernel)

// Shared memory a CTA may use for its ring and activation planes:
// POPCORN_GEMV_SMEM_KB (tuning) when set, else 0 (the default rule in
// make_plan).
size_t gemv_smem_override() {
    static size_t b = [] {
        size_t v = 0;
        if (const char* e = getenv("POPCORN_GEMV_SMEM_KB")) {
            const long kb = atol(e);
            if (kb >= 32 && size_t(kb) * 1024 <= kTmaSmemBudget) v = size_t(kb) * 1024;
        }
        return v;
    }();
    return b;
}

// Short GEMVs (at most this many 8-row tiles per CTA, every decode-layer
// matvec) get a ring of about 150 KB instead of 200 KB: with every SM
// issuing its whole ring at once, fewer bytes outstanding bring the first
// stages in sooner (config-2 step 1.286 -> 1.276 ms), while the long LM head
// GEMV keeps the deeper ring (203 vs 206 us).
constexpr int kShortTilesPerCta = 32;
constexpr size_t kShortBudget = 150 * 1024;
// POPCORN_GEMV_SHORT_TILES overrides kShortTilesPerCta (tuning).
int short_tiles_per_cta() {
    static const int v = [] {
        const char* e = getenv("POPCORN_GEMV_SHORT_TILES");
        return e ? atoi(e) : kShortTilesPerCta;
    }();
    return v;
}

bool make_plan(const Gemv& p, GemvPlan& g) {
    const int es = dtype_stride(p.w_dtype);
    const int64_t K = p.K;
    const int64_t max_stage = 40 * 1024;
    int nkc = int((K * es * 8 + max_stage - 1) / max_stage);
    if (nkc < 1) nkc = 1;
    int64_t kc = (K + nkc - 1) / nkc;
    kc = (kc + 7) / 8 * 8;
    nkc = int((K + kc - 1) / kc);
    g.kc = int(kc);
    g.nkc = nkc;
    g.ntiles = int((p.N + 7) / 8);
    g.stage_bytes = int(8 * kc * es);
    size_t xbytes = size_t(K) * 4;
    const int sms = current_sm_count();
    size_t budget = gemv_smem_override();
    if (budget == 0) budget = (g.ntiles + sms - 1) / sms <= short_tiles_per_cta() ? kShortBudget : kTmaSmemBudget;
    if (xbytes + 2 * size_t(g.stage_bytes) > budget) return false;
    g.stages = int((budget - xbytes) / g.stage_bytes);
    if (g.stages > 8) g.stages = 8;
    return g.stages >= 2;
}

template <class XT, class WT, class OT, bool NORM, int EPI>
cudaError_t run_tma(const Gemv& p, const GemvPlan& g, cudaStream_t s) {
    auto kern = gemv_tma_kernel<XT, WT, OT, NORM, EPI>;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = allow_smem(kern, kTmaSmemBudget + 1024);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    size_t smem = size_t(g.stages) * g.stage_bytes + size_t(p.K) * 4;
    int grid = g.ntiles < current_sm_count() ? g.ntiles : current_sm_count();
    return launch_k(kern, dim3(unsigned(grid)), dim3(kTmaThreads), smem, s, p, g);
}

template <class XT, class WT, class OT, bool NORM, int EPI>
cudaError_t dispatch_rows(const Gemv& p, cudaStream_t s) {
    constexpr int VEC = WVec<WT>::n;
    bool vec_ok = (p.K % VEC == 0) && (p.K * Elem<WT>::bytes) % 16 == 0 && aligned16(p.w) &&
                  (EPI != int(Epilogue::kGated) || aligned16(p.w2));
    GemvPlan g{};
    if (vec_ok && make_plan(p, g)) return run_tma<XT, WT, OT, NORM, EPI>(p, g, s);
    return run_scalar<XT, WT, OT, NORM, EPI>(p, s);
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

uint32_t read_and_clear_gemv_errors() {
    unsigned int v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_gemv_error_word, sizeof(v)) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    if (v) cudaMemcpyToSymbol(g_gemv_error_word, &zero, sizeof(zero));
    return v;
}

namespace {
RegisterFunctions reg_gemv({
    {"matvec_nk_f32_f32_f32", reinterpret_cast<const void*>(gemv_tma_kernel<TF32, TF32, TF32, false, 0>)},
    {"matvec_nk_f32_bf16_f32", reinterpret_cast<const void*>(gemv_tma_kernel<TF32, TBF16, TF32, false, 0>)},
    {"matvec_nk_bf16_bf16_f32", reinterpret_cast<const void*>(gemv_tma_kernel<TBF16, TBF16, TF32, false, 0>)},
    {"matvec_nk_bf16_bf16_bf16", reinterpret_cast<const void*>(gemv_tma_kernel<TBF16, TBF16, TBF16, false, 0>)},
    {"matvec_nk_f32_bf16_bf16", reinterpret_cast<const void*>(gemv_tma_kernel<TF32, TBF16, TBF16, false, 0>)},
    {"matvec_nk_f32_f16_f32", reinterpret_cast<const void*>(gemv_tma_kernel<TF32, TF16, TF32, false, 0>)},
    {"matvec_nk_f16_f16_f32", reinterpret_cast<const void*>(gemv_tma_kernel<TF16, TF16, TF32, false, 0>)},
    {"matvec_nk_f16_f16_f16", reinterpret_cast<const void*>(gemv_tma_kernel<TF16, TF16, TF16, false, 0>)},
    {"matvec_nk_f32_f16_f16", reinterpret_cast<const void*>(gemv_tma_kernel<TF32, TF16, TF16, false, 0>)},
    {"rmsnorm_matvec_bf16", reinterpret_cast<const void*>(gemv_tma_kernel<TBF16, TBF16, TBF16, true, 0>)},
    {"rmsnorm_matvec_f16", reinterpret_cast<const void*>(gemv_tma_kernel<TF16, TF16, TF16, true, 0>)},
    {"matvec_residual_bf16", reinterpret_cast<const void*>(gemv_tma_kernel<TBF16, TBF16, TBF16, false, 1>)},
    {"matvec_residual_f16", reinterpret_cast<const void*>(gemv_tma_kernel<TF16, TF16, TF16, false, 1>)},
    {"geglu_matvec_bf16", reinterpret_cast<const void*>(gemv_tma_kernel<TBF16, TBF16, TBF16, true, 2>)},
    {"geglu_matvec_f16", reinterpret_cast<const void*>(gemv_tma_kernel<TF16, TF16, TF16, true, 2>)},
    {"swiglu_matvec_bf16", reinterpret_cast<const void*>(gemv_tma_kernel<TBF16, TBF16, TBF16, false, 2>)},
    {"swiglu_matvec_f16", reinterpret_cast<const void*>(gemv_tma_kernel<TF16, TF16, TF16, false, 2>)},
    {"qkv_matvec_bf16", reinterpret_cast<const void*>(gemv_tma_kernel<TBF16, TBF16, TBF16, true, 3>)},
    {"qkv_matvec_f16", reinterpret_cast<const void*>(gemv_tma_kernel<TF16, TF16, TF16, true, 3>)},
});
}  // namespace

}  // namespace launch
}  // namespace popcorn
