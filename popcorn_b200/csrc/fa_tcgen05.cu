// fa_tcgen05.cu — prefill FlashAttention on the 5th-generation tensor cores
// (sm_100a): S = Q.K^T and O += P.V as tcgen05.mma with fp32 accumulators in
// tensor memory, Q/K/V tiles by TMA (128-byte swizzle, no multicast).
//
// Semantics (FlashAttention.metal:31-162; MPPFlashAttention.metal:39-244):
// query row q of (b, hq) sits at posQ = Sk - Sq + q and attends to the keys
// its mask allows (causal j <= posQ; sliding window also posQ - j < window;
// bidirectional all); KV head hkv = hq * Nkv / Nq; online softmax in fp32
// (natural exp, evaluated as exp2 of log2e-scaled scores); O / l stored once.
// The scale multiplies the fp32 scores (the reference scales q first: the
// same product up to fp32 rounding). P enters the second product in the
// input type: f16 directly (11 significant bits), bf16 as a hi + lo pair
// (P = hi + lo, two MMAs, ~16 significant bits), so the output keeps the
// fp32-accumulation tolerance of the reference semantics.
//
// One CTA per (128-query tile, query head, batch), heaviest causal tiles
// first. Warp 0 lane 0 loads Q once and then the K and V tiles of every
// 64-key step into two-stage rings, each tile as soon as its stage frees;
// warp 1 lane 0 issues the MMAs, whichever group is ready first: S(j+1) =
// Q.K(j+1)^T into the other of two S accumulators while the softmax warps
// work on S(j), and O += P(j).V(j). Warps 2-5 own one query row per thread (TMEM lane): they
// read S, mask, keep the running max and sum, write P to shared memory in
// the MMA's swizzled K-major layout, and rescale O in tensor memory only
// when the running max grows by more than 2^8 (P stays <= 256; the final
// O / l is exact for any max used consistently). TMEM: S0, S1 (64 columns
// each) and O (Hd columns) in one 512-column allocation.
//
// Softmax per step: ex2.approx, one select per key only on tiles that cross
// a row's mask edge, P packed with cvt.rn.{bf16,f16}x2. Measured (config 4:
// B 4, 8 Q / 4 KV heads, S 2048, Hd 256, causal, bf16): 121 us = 568
// TFLOP/s. The remaining limit is the K/V load latency (~2.5 us) against a
// two-stage ring: at Hd 256 shared memory holds no third stage.
//
// Every mbarrier wait is bounded; on give-up the CTA sets the error word,
// skips its remaining work, frees its tensor memory and leaves.
#include "async.cuh"
#include "common.cuh"
#include "dtype.cuh"
#include "launch.hpp"
#include "popcorn.hpp"
#include "tcgen05.cuh"

namespace popcorn {

__device__ unsigned int g_fa_error_word;

#ifdef PC_FA_TRACE
// Development-only: per CTA globaltimer at start / end and its step count.
__device__ unsigned long long g_fa_trace[4096 * 3];
__device__ unsigned long long g_fa_steps[8][64];  // one CTA: per step event times
#define FA_STEP(ev, j) do { if (lin == 0 && (j) < 64) g_fa_steps[ev][j] = fa_now(); } while (0)
__device__ __forceinline__ unsigned long long fa_now() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
#endif

namespace launch {

namespace {

using namespace tc;

constexpr int kBMq = 128;               // query rows per CTA (MMA M)
constexpr int kBNk = 64;                // keys per step (one 128-byte swizzle atom of P)
constexpr int kFaThreads = 6 * 32;      // warp 0 TMA, warp 1 MMA, warps 2-5 softmax
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleLog2 = 8.0f;    // rescale O when the max grows by more than this (log2 units)
constexpr uint32_t kTmemCols = 512;

struct FaArgs {
    void* out;
    int64_t Sq, Sk;
    int B, Nq, Nkv;
    float c;          // scale * log2(e)
    int mask_kind;    // 0 causal, 1 sliding window, 2 bidirectional
    int window;
    int n_qtiles;
};

// 2^x with the hardware's approximate exponential (PTX ex2.approx: relative
// error ~2^-22, far below P's representation error).
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Two floats -> one 32-bit word of two 16-bit values (lo, hi), round to
// nearest even (P is finite and >= 0: the same result as the bit-level rule).
template <class T> __device__ __forceinline__ uint32_t cvt_pair(float lo, float hi);
template <> __device__ __forceinline__ uint32_t cvt_pair<TBF16>(float lo, float hi) {
    uint32_t d;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
}
template <> __device__ __forceinline__ uint32_t cvt_pair<TF16>(float lo, float hi) {
    uint32_t d;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
}

// Warp-uniform bounded wait: lane 0 waits, the warp learns the outcome.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, int lane) {
    int ok = 1;
    if (lane == 0) ok = mbar_wait_spin(bar, parity, &g_fa_error_word) ? 1 : 0;
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

template <int HD, class IT, class OT>
__global__ void __launch_bounds__(kFaThreads, 1)
    fa_tcgen05_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                      const __grid_constant__ CUtensorMap map_v, const FaArgs a) {
    constexpr int ATOMS = HD / 64;                    // 128-byte swizzle atoms along the head dim
    constexpr int Q_BYTES = kBMq * HD * 2;            // ATOMS blocks of 128 rows x 128 B
    constexpr int KV_BYTES = kBNk * HD * 2;
    constexpr int Q_BLOCK = kBMq * 128, KV_BLOCK = kBNk * 128, P_BLOCK = kBMq * 128;
    constexpr uint32_t S_COLS = kBNk;
    constexpr uint32_t O_COL = 2 * S_COLS;
    constexpr bool BF = IT::code == TBF16::code;
    constexpr int NP = BF ? 2 : 1;  // P parts: bf16 hi + lo, or one f16
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t q_full, k_full[2], k_empty[2], v_full[2], v_empty[2], s_full[2], s_free[2], p_full,
        o_done;
    __shared__ uint32_t s_tmem;
    __shared__ volatile int s_abort;

    pdl_launch_dependents();
    unsigned char* sq =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* sk = sq + Q_BYTES;      // two K stages
    unsigned char* sv = sk + 2 * KV_BYTES; // two V stages
    unsigned char* sp = sv + 2 * KV_BYTES;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    // This CTA's query tile, head and batch. The grid is one-dimensional and
    // CTAs start in index order, so the index runs over (head, batch) fastest
    // and over query tiles from the last (the heaviest under a causal mask)
    // to the first: every head's heavy tiles start before any light one, and
    // the light tiles fill the last wave.
    const int hb = int(blockIdx.x % unsigned(a.Nq * a.B));
    const int qt = a.n_qtiles - 1 - int(blockIdx.x / unsigned(a.Nq * a.B));
    const int hq = hb % a.Nq, b = hb / a.Nq;
    const int hkv = int(int64_t(hq) * a.Nkv / a.Nq);
    const int64_t q0 = int64_t(qt) * kBMq;
    const int64_t qlast = (q0 + kBMq < a.Sq ? q0 + kBMq : a.Sq) - 1;
    // Key tiles [t_lo, t_lo + nt) that hold an allowed key for some row.
    const int64_t nkt_all = (a.Sk + kBNk - 1) / kBNk;
    int64_t t_lo = 0, t_hi = nkt_all;
    if (a.mask_kind != 2) {
        const int64_t kmax = a.Sk - a.Sq + qlast;
        t_hi = kmax < 0 ? 0 : (kmax / kBNk + 1 < nkt_all ? kmax / kBNk + 1 : nkt_all);
    }
    if (a.mask_kind == 1) {
        const int64_t kmin = a.Sk - a.Sq + q0 - a.window + 1;
        if (kmin > 0) t_lo = kmin / kBNk;
    }
    const int nt = t_hi > t_lo ? int(t_hi - t_lo) : 0;
#ifndef PC_FA_TRACE
#define FA_STEP(ev, j) ((void)0)
#else
    const unsigned lin = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
    if (threadIdx.x == 0 && lin < 4096) {
        g_fa_trace[lin * 3] = fa_now();
        g_fa_trace[lin * 3 + 2] = unsigned(nt);
    }
#endif

    if (tid == 0) {
        mbar_init(smem_u32(&q_full), 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(smem_u32(&k_full[i]), 1);
            mbar_init(smem_u32(&k_empty[i]), 1);
            mbar_init(smem_u32(&v_full[i]), 1);
            mbar_init(smem_u32(&v_empty[i]), 1);
            mbar_init(smem_u32(&s_full[i]), 1);
            mbar_init(smem_u32(&s_free[i]), 4);
        }
        mbar_init(smem_u32(&p_full), 4);
        mbar_init(smem_u32(&o_done), 1);
        s_abort = 0;
        mbar_fence_init();
    }
    if (warp == 0) tmem_alloc(smem_u32(&s_tmem), kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    pdl_wait();

    if (warp == 0) {
        if (lane == 0 && nt > 0) {
            // ---- TMA loads ----
            const int zq = b * a.Nq + hq, zkv = b * a.Nkv + hkv;
            mbar_expect_tx(smem_u32(&q_full), Q_BYTES);
#pragma unroll
            for (int at = 0; at < ATOMS; ++at)
                tma_load_3d(smem_u32(sq + at * Q_BLOCK), &map_q, at * 64, int(q0), zq, smem_u32(&q_full));
            int kf = 0, vf = 0;  // K and V tiles issued
            uint32_t idle = 0;
            // K and V tiles are issued independently, each as soon as its stage frees.
            while ((kf < nt || vf < nt) && !s_abort) {
                bool progressed = false;
                if (kf < nt && (kf == 0 || kf - vf < 2) &&
                    mbar_test_wait(smem_u32(&k_empty[kf & 1]), (uint32_t(kf >> 1) & 1u) ^ 1u)) {
                    const int st = kf & 1;
                    mbar_expect_tx(smem_u32(&k_full[st]), KV_BYTES);
#pragma unroll
                    for (int at = 0; at < ATOMS; ++at)
                        tma_load_3d(smem_u32(sk + st * KV_BYTES + at * KV_BLOCK), &map_k, at * 64,
                                    int((t_lo + kf) * kBNk), zkv, smem_u32(&k_full[st]));
                    FA_STEP(0, kf);
                    ++kf;
                    progressed = true;
                }
                if (vf < kf && mbar_test_wait(smem_u32(&v_empty[vf & 1]), (uint32_t(vf >> 1) & 1u) ^ 1u)) {
                    const int st = vf & 1;
                    mbar_expect_tx(smem_u32(&v_full[st]), KV_BYTES);
#pragma unroll
                    for (int at = 0; at < ATOMS; ++at)
                        tma_load_3d(smem_u32(sv + st * KV_BYTES + at * KV_BLOCK), &map_v, at * 64,
                                    int((t_lo + vf) * kBNk), zkv, smem_u32(&v_full[st]));
                    FA_STEP(1, vf);
                    ++vf;
                    progressed = true;
                }
                if (progressed) {
                    idle = 0;
                } else if (++idle > (1u << 26)) {  // bounded: about seconds of polling
                    atomicOr(&g_fa_error_word, 1u);
                    s_abort = 1;
                }
            }
            if (s_abort) {
                // leave no copy in flight: wait (bounded) for the last ones issued
                mbar_wait_spin(smem_u32(&q_full), 0u, &g_fa_error_word);
                for (int i = kf - 2 < 0 ? 0 : kf - 2; i < kf; ++i)
                    mbar_wait_spin(smem_u32(&k_full[i & 1]), uint32_t(i >> 1) & 1u, &g_fa_error_word);
                for (int i = vf - 2 < 0 ? 0 : vf - 2; i < vf; ++i)
                    mbar_wait_spin(smem_u32(&v_full[i & 1]), uint32_t(i >> 1) & 1u, &g_fa_error_word);
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && nt > 0) {
            // ---- MMA issue ----
            const uint32_t idesc_s = make_idesc(BF, kBMq, kBNk, false);
            const uint32_t idesc_o = make_idesc(BF, kBMq, HD, true);
            const uint32_t q_base = smem_u32(sq), k_base = smem_u32(sk), v_base = smem_u32(sv), p_base = smem_u32(sp);
            bool ok = mbar_wait_spin(smem_u32(&q_full), 0u, &g_fa_error_word);
            // Issue whichever MMA group is ready: S(ns) once its K tile has
            // landed and its accumulator is free, O += P(np).V(np) once P and V
            // are there, so neither waits behind the other's operands.
            int ns = 0, np = 0;
            uint32_t idle = 0;
            while (ok && np < nt && !s_abort) {
                bool progressed = false;
                if (ns < nt && ns <= np + 1) {
                    const int buf = ns & 1;
                    if (mbar_test_wait(smem_u32(&s_free[buf]), (uint32_t(ns >> 1) & 1u) ^ 1u) &&
                        mbar_test_wait(smem_u32(&k_full[buf]), uint32_t(ns >> 1) & 1u)) {
                        tc_fence_after();
                        const uint32_t kb = k_base + buf * KV_BYTES;
#pragma unroll
                        for (int kk = 0; kk < HD / 16; ++kk)
                            tc_mma(tmem + uint32_t(buf) * S_COLS,
                                   smem_desc_sw128(q_base + (kk >> 2) * Q_BLOCK + (kk & 3) * 32),
                                   smem_desc_sw128(kb + (kk >> 2) * KV_BLOCK + (kk & 3) * 32), idesc_s,
                                   kk > 0 ? 1u : 0u);
                        tc_commit(smem_u32(&k_empty[buf]));
                        FA_STEP(2, ns);
                        tc_commit(smem_u32(&s_full[buf]));
                        ++ns;
                        progressed = true;
                    }
                }
                if (np < ns) {
                    const int vs = np & 1;
                    if (mbar_test_wait(smem_u32(&p_full), uint32_t(np) & 1u) &&
                        mbar_test_wait(smem_u32(&v_full[vs]), uint32_t(np >> 1) & 1u)) {
                        tc_fence_after();
                        const uint32_t vb = v_base + vs * KV_BYTES;
#pragma unroll
                        for (int part = 0; part < NP; ++part)
#pragma unroll
                            for (int kk = 0; kk < kBNk / 16; ++kk)
                                tc_mma(tmem + O_COL, smem_desc_sw128(p_base + part * P_BLOCK + kk * 32),
                                       smem_desc_sw128_mn(vb + kk * 2048, KV_BLOCK), idesc_o,
                                       (np > 0 || part > 0 || kk > 0) ? 1u : 0u);
                        tc_commit(smem_u32(&v_empty[vs]));
                        FA_STEP(3, np);
                        tc_commit(smem_u32(&o_done));
                        ++np;
                        progressed = true;
                    }
                }
                if (progressed) {
                    idle = 0;
                } else if (++idle > (1u << 26)) {  // bounded: about seconds of polling
                    atomicOr(&g_fa_error_word, 1u);
                    ok = false;
                }
            }
            if (!ok) s_abort = 1;
        }
    } else {
        // ---- softmax: one query row per thread ----
        const int quarter = warp & 3;               // TMEM lanes this warp may access
        const int row = quarter * 32 + lane;
        const uint32_t lane_off = uint32_t(quarter * 32) << 16;
        const int64_t qi = q0 + row;
        const int64_t posQ = a.Sk - a.Sq + qi;
        float m_used = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < nt && ok; ++j) {
            const int buf = j & 1;
            ok = warp_wait(smem_u32(&s_full[buf]), uint32_t(j >> 1) & 1u, lane) && !s_abort;
            if (!ok) break;
            if (warp == 2 && lane == 0) FA_STEP(4, j);
            tc_fence_after();
            float s[kBNk];
#pragma unroll
            for (int c = 0; c < kBNk / 32; ++c) tmem_ld32(tmem + uint32_t(buf) * S_COLS + uint32_t(c * 32) + lane_off, s + c * 32);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&s_free[buf]));
            // allowed keys of this row: [key_lo, key_hi), as offsets into this tile
            const int64_t key0 = (t_lo + j) * kBNk;
            int64_t hi = a.mask_kind == 2 ? a.Sk : (posQ + 1 < a.Sk ? posQ + 1 : a.Sk);
            int64_t lo = a.mask_kind == 1 ? posQ - a.window + 1 : 0;
            hi -= key0;
            lo -= key0;
            const int chi = hi < 0 ? 0 : (hi > kBNk ? kBNk : int(hi));
            const int clo = lo < 0 ? 0 : (lo > kBNk ? kBNk : int(lo));
            float mx = -INFINITY;
            if (__all_sync(0xffffffffu, clo == 0 && chi == kBNk)) {
                // no key of this tile is masked for any row of the warp
#pragma unroll
                for (int c = 0; c < kBNk; ++c) {
                    s[c] *= a.c;
                    mx = fmaxf(mx, s[c]);
                }
            } else {
#pragma unroll
                for (int c = 0; c < kBNk; ++c) {
                    s[c] = (c >= clo && c < chi) ? s[c] * a.c : -INFINITY;
                    mx = fmaxf(mx, s[c]);
                }
            }
            // lazy rescale: keep the old max unless the new one exceeds it by 2^8
            const float m_new = fmaxf(m_used, mx);
            float factor = 1.f;
            if (m_new > m_used + kRescaleLog2) {  // also when m_used is -inf and the tile has a key
                factor = m_used == -INFINITY ? 0.f : ex2(m_used - m_new);
                m_used = m_new;
                l *= factor;
            }
            float lsum = 0.f;
            const float mu = m_used == -INFINITY ? 0.f : m_used;  // all s are -inf then: ex2 gives 0
#pragma unroll
            for (int c = 0; c < kBNk; ++c) {
                s[c] = ex2(s[c] - mu);
                lsum += s[c];
            }
            l += lsum;
            // P's buffer is free and O is settled once PV(j-1) has completed.
            if (j > 0) {
                ok = warp_wait(smem_u32(&o_done), uint32_t(j - 1) & 1u, lane) && !s_abort;
                if (!ok) break;
                if (warp == 2 && lane == 0) FA_STEP(5, j);
                tc_fence_after();
                // O rows that were accumulated under the old max (factor 0: O
                // is zero there, nothing to do)
                if (__any_sync(0xffffffffu, factor != 1.f && factor != 0.f)) {
#pragma unroll 1
                    for (int c = 0; c < HD / 32; ++c) {
                        float o[32];
                        tmem_ld32(tmem + O_COL + uint32_t(c * 32) + lane_off, o);
#pragma unroll
                        for (int e = 0; e < 32; ++e) o[e] *= (factor == 0.f ? 1.f : factor);
                        tmem_st32(tmem + O_COL + uint32_t(c * 32) + lane_off, o);
                    }
                    tmem_wait_st();
                }
            }
            // P row -> shared memory, K-major with 128-byte swizzle (A operand);
            // bf16: the hi part, then lo = p - hi in the second block
#pragma unroll
            for (int c8 = 0; c8 < kBNk / 8; ++c8) {
                uint32_t h[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) h[i] = cvt_pair<IT>(s[c8 * 8 + 2 * i], s[c8 * 8 + 2 * i + 1]);
                const uint32_t off = row * 128 + ((c8 ^ (row & 7)) << 4);
                *reinterpret_cast<uint4*>(sp + off) = make_uint4(h[0], h[1], h[2], h[3]);
                if constexpr (NP == 2) {
                    // lo = p - hi (exact in fp32), rounded again
                    uint32_t w[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float h0 = __uint_as_float(h[i] << 16), h1 = __uint_as_float(h[i] & 0xffff0000u);
                        w[i] = cvt_pair<IT>(s[c8 * 8 + 2 * i] - h0, s[c8 * 8 + 2 * i + 1] - h1);
                    }
                    *reinterpret_cast<uint4*>(sp + P_BLOCK + off) = make_uint4(w[0], w[1], w[2], w[3]);
                }
            }
            fence_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&p_full));
            if (warp == 2 && lane == 0) FA_STEP(6, j);
        }
        if (nt > 0 && ok) {
            ok = warp_wait(smem_u32(&o_done), uint32_t(nt - 1) & 1u, lane) && !s_abort;
            tc_fence_after();
        }
        if (!ok) s_abort = 1;
        // ---- O / l -> out ----
        const float inv = l > 0.f ? 1.0f / l : 0.f;
        const bool valid = qi < a.Sq;
        const int64_t obase = ((int64_t(b) * a.Nq + hq) * a.Sq + qi) * HD;
#pragma unroll 1
        for (int c = 0; c < HD / 32; ++c) {
            float o[32];
            if (nt > 0 && ok) {
                tmem_ld32(tmem + O_COL + uint32_t(c * 32) + lane_off, o);
            } else {
#pragma unroll
                for (int e = 0; e < 32; ++e) o[e] = 0.f;
            }
            if (valid) {
                if constexpr (Elem<OT>::bytes == 4) {
                    float4* d4 = reinterpret_cast<float4*>(static_cast<float*>(a.out) + obase + c * 32);
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        d4[e] = make_float4(o[4 * e] * inv, o[4 * e + 1] * inv, o[4 * e + 2] * inv, o[4 * e + 3] * inv);
                } else {
                    uint4* d4 = reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.out) + obase + c * 32);
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        d4[e] = make_uint4(pack2<OT>(o[8 * e] * inv, o[8 * e + 1] * inv),
                                           pack2<OT>(o[8 * e + 2] * inv, o[8 * e + 3] * inv),
                                           pack2<OT>(o[8 * e + 4] * inv, o[8 * e + 5] * inv),
                                           pack2<OT>(o[8 * e + 6] * inv, o[8 * e + 7] * inv));
                }
            }
        }
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, kTmemCols);
#ifdef PC_FA_TRACE
    if (threadIdx.x == 0 && lin < 4096) g_fa_trace[lin * 3 + 1] = fa_now();
#endif
}

// 3-D map [heads*batch, S, HD] (16-bit), box = 64 x rows x 1, 128-byte swizzle.
bool make_map_3d(CUtensorMap* map, const void* base, int dtype, int64_t S, int64_t HD, int64_t planes, int rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {cuuint64_t(HD), cuuint64_t(S), cuuint64_t(planes)};
    cuuint64_t strides[2] = {cuuint64_t(HD) * 2, cuuint64_t(S) * HD * 2};
    cuuint32_t box[3] = {64, cuuint32_t(rows), 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, dtype == PC_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                    const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <int HD>
constexpr size_t fa_smem() {
    return size_t(kBMq) * HD * 2 + 4 * size_t(kBNk) * HD * 2 + 2 * size_t(kBMq) * kBNk * 2 + 1024;
}

template <int HD, class IT, class OT>
cudaError_t run_fa(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const FaArgs& fa, cudaStream_t s) {
    auto kern = fa_tcgen05_kernel<HD, IT, OT>;
    constexpr size_t smem = fa_smem<HD>();
    static bool configured = false;
    if (!configured) {
        cudaError_t e = allow_smem(kern, smem);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    dim3 grid(unsigned(int64_t(fa.n_qtiles) * fa.Nq * fa.B));
    return launch_k(kern, grid, dim3(kFaThreads), smem, s, mq, mk, mv, fa);
}

template <int HD, class IT>
cudaError_t run_fa_o(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const FaArgs& fa,
                     int out_dtype, cudaStream_t s) {
    if (out_dtype == PC_F32) return run_fa<HD, IT, TF32>(mq, mk, mv, fa, s);
    return run_fa<HD, IT, IT>(mq, mk, mv, fa, s);
}

}  // namespace

// Served: q, k, v all bf16 or all f16; out f32 or the input type; head dim
// 128 or 256; 16-byte aligned bases; grid dimensions in range; Sq >= 32
// (shorter queries stay on the plain kernel, as FlashAttention.route does).
bool fa_tcgen05_supports(const FlashAttention& p) {
    const bool types = (p.q_dtype == PC_BF16 || p.q_dtype == PC_F16) && p.kv_dtype == p.q_dtype &&
                       (p.out_dtype == PC_F32 || p.out_dtype == p.q_dtype);
    return types && (p.Hd == 128 || p.Hd == 256) && p.Sq >= 32 && p.Sk >= 1 && aligned16(p.q) && aligned16(p.k) &&
           aligned16(p.v) && aligned16(p.out) && p.Nq <= 65535 && p.B <= 65535 &&
           (p.Sq + kBMq - 1) / kBMq * p.Nq * p.B < (int64_t(1) << 31) && p.Sk < (int64_t(1) << 31) && p.Sq < (int64_t(1) << 31) &&
           encode_fn() != nullptr;
}

cudaError_t flash_attention_tcgen05(const FlashAttention& p, cudaStream_t s) {
    CUtensorMap mq, mk, mv;
    if (!make_map_3d(&mq, p.q, p.q_dtype, p.Sq, p.Hd, p.B * p.Nq, kBMq) ||
        !make_map_3d(&mk, p.k, p.kv_dtype, p.Sk, p.Hd, p.B * p.Nkv, kBNk) ||
        !make_map_3d(&mv, p.v, p.kv_dtype, p.Sk, p.Hd, p.B * p.Nkv, kBNk))
        return cudaErrorInvalidValue;
    FaArgs fa{};
    fa.out = p.out;
    fa.Sq = p.Sq;
    fa.Sk = p.Sk;
    fa.B = int(p.B);
    fa.Nq = int(p.Nq);
    fa.Nkv = int(p.Nkv);
    fa.c = p.scale * kLog2e;
    fa.mask_kind = p.mask_kind;
    fa.window = p.window;
    fa.n_qtiles = int((p.Sq + kBMq - 1) / kBMq);

    if (p.q_dtype == PC_BF16)
        return p.Hd == 128 ? run_fa_o<128, TBF16>(mq, mk, mv, fa, p.out_dtype, s)
                           : run_fa_o<256, TBF16>(mq, mk, mv, fa, p.out_dtype, s);
    return p.Hd == 128 ? run_fa_o<128, TF16>(mq, mk, mv, fa, p.out_dtype, s)
                       : run_fa_o<256, TF16>(mq, mk, mv, fa, p.out_dtype, s);
}

uint32_t read_and_clear_fa_errors() {
    unsigned int v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_fa_error_word, sizeof(v)) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    if (v) cudaMemcpyToSymbol(g_fa_error_word, &zero, sizeof(zero));
    return v;
}

namespace {
RegisterFunctions reg_fa_tc({
    {"flash_attention_tc_bf16", reinterpret_cast<const void*>(fa_tcgen05_kernel<256, TBF16, TBF16>)},
    {"flash_attention_tc_f16", reinterpret_cast<const void*>(fa_tcgen05_kernel<256, TF16, TF16>)},
});
}  // namespace

}  // namespace launch
}  // namespace popcorn

#ifdef PC_FA_TRACE
extern "C" __attribute__((visibility("default"))) int pc_debug_fa_trace(unsigned long long* host) {
    return int(cudaMemcpyFromSymbol(host, popcorn::g_fa_trace, sizeof(popcorn::g_fa_trace)));
}
extern "C" __attribute__((visibility("default"))) int pc_debug_fa_steps(unsigned long long* host) {
    return int(cudaMemcpyFromSymbol(host, popcorn::g_fa_steps, sizeof(popcorn::g_fa_steps)));
}
#endif
