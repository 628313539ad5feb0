// flash_decoding.cu — split-KV GQA decode attention (Sq = 1) for sm_100a.
//
// Semantics (FlashDecoding.metal:29-231): per (b, hq) the query at position
// len-1 attends to keys [0, len) of KV head hkv = hq*Nkv/Nq (:56); q is
// pre-scaled (:66); softmax uses natural exp (computed here as exp2 of
// log2e-scaled scores, the same function); the key range is split into
// partitions whose unnormalised (m, l, O) are merged by a log-sum-exp combine
// (:182-231). Sliding-window masks keep keys with posQ - j < window (:97-99).
//
// B200 design.
//  * One CTA per (b, KV head, head group, split), sized to one wave (one
//    CTA per SM): the G query heads that share a KV head are served from ONE
//    read of their K/V rows (the reference re-reads K/V once per query head).
//  * A producer warp streams 32-key K and V tiles HBM -> shared memory with
//    the bulk-copy engine (cp.async.bulk, 1-D, no multicast) into a ring of
//    up to 8 stages (<= 128 KB in flight per SM), tracked by full/empty
//    mbarriers.
//  * Four groups of four consumer warps take tiles round-robin; each warp
//    scores 8 keys per tile: lanes hold Hd/32 contiguous head dims (one
//    16-byte shared load per key row at Hd 256, conflict-free), then a
//    transpose-reduction folds the 8 x G partial dots across the warp in 9G
//    shuffles instead of 40G. Online softmax per warp; the eight warp states
//    merge at the end.
//  * The split count is chosen for whole waves over the SMs; a small
//    parallel kernel merges the splits (skipped with one split).
//  * Before griddepcontrol.wait the producer warms L2 with the first ring's
//    worth of the split's K/V rows (cp.async.bulk.prefetch.L2), overlapping
//    the read with the previous kernel's tail.
//  * Every mbarrier wait is bounded; a wait that gives up sets a device
//    error word (pc_device_error_check) and the CTA drains its copies and
//    leaves.
#include <algorithm>

#include "async.cuh"
#include "common.cuh"
#include "dtype.cuh"
#include "launch.hpp"
#include "popcorn.hpp"
#include "trace.cuh"

namespace popcorn {

__device__ unsigned int g_fd_error_word;
namespace launch {
PC_DT_BUFFER
}

namespace launch {

namespace {

constexpr int kTileKeys = 32;  // 8 keys per warp per tile
constexpr int kThreads = 128;  // generic and combine kernels
constexpr int kWarps = 4;
constexpr float kLog2e = 1.4426950408889634f;

// E consecutive elements of a row (in shared memory) -> floats.
template <class KV, int E>
__device__ __forceinline__ void load_slice(const char* p, float* f) {
    if constexpr (Elem<KV>::bytes == 2) {
        if constexpr (E == 2) {
            float2 a = unpack2<KV>(*reinterpret_cast<const uint32_t*>(p));
            f[0] = a.x; f[1] = a.y;
        } else if constexpr (E == 4) {
            uint2 v = *reinterpret_cast<const uint2*>(p);
            float2 a = unpack2<KV>(v.x), b = unpack2<KV>(v.y);
            f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
        } else {
#pragma unroll
            for (int c = 0; c < E / 8; ++c) unpack8<KV>(reinterpret_cast<const uint4*>(p)[c], f + 8 * c);
        }
    } else {
        if constexpr (E == 2) {
            float2 a = *reinterpret_cast<const float2*>(p);
            f[0] = a.x; f[1] = a.y;
        } else {
#pragma unroll
            for (int c = 0; c < E / 4; ++c) {
                float4 a = reinterpret_cast<const float4*>(p)[c];
                f[4 * c] = a.x; f[4 * c + 1] = a.y; f[4 * c + 2] = a.z; f[4 * c + 3] = a.w;
            }
        }
    }
}

template <class KV, int HD>
struct FDShape {
    static constexpr int E = HD / 32;
    static constexpr int kRowBytes = HD * Elem<KV>::bytes;
    static constexpr int kTileBytes = kTileKeys * kRowBytes;  // one of K or V
    static constexpr int kStageBytes = 2 * kTileBytes;
    // Four consumer groups of four warps take tiles round-robin (two when
    // the ring has fewer than four stages). The ring depth is a multiple of
    // the group count, so tiles t and t + kStages belong to the same group
    // and no group ever waits on a stage's phase two steps ahead of the one
    // in flight (the parity would alias).
    static constexpr int kRing = std::max(2, std::min(8, 131072 / kStageBytes));
    static constexpr int kGroups = kRing >= 4 ? 4 : 2;
    static constexpr int kStages = kRing / kGroups * kGroups;
    static constexpr int kCWarps = 4 * kGroups;
    static constexpr int kThreads = (kCWarps + 1) * 32;
};

template <class KV, int HD, int G>
constexpr size_t fd_smem_bytes() {
    using S = FDShape<KV, HD>;
    size_t ring = size_t(S::kStages) * S::kStageBytes;
    size_t merge = (size_t(S::kCWarps) * G * (HD + 3) + 2 * G) * 4;
    return ring > merge ? ring : merge;
}

struct FDArgs {
    FlashDecode p;
    int splits;
    int64_t chunk;
    int G;        // query heads per CTA
    int hgroups;  // head groups per KV head
    float* po;
    float* pm;
    float* pl;
};

// Keys of sequence b: seq_lens[b] clamped to [0, S] (a larger value would
// read past the cache's rows), or S without seq_lens.
__device__ __forceinline__ int64_t seq_len(const FlashDecode& p, int64_t b) {
    if (!p.seq_lens) return p.S;
    const int64_t n = int64_t(p.seq_lens[b]);
    return n < 0 ? 0 : (n > p.S ? p.S : n);
}

// Key range [jb, je) of this CTA's split for sequence length len.
__device__ __forceinline__ void split_range(const FDArgs& a, int64_t len, int split, int64_t& jb, int64_t& je) {
    jb = int64_t(split) * a.chunk;
    je = jb + a.chunk;
    if (je > len) je = len;
    if (a.p.mask_kind == 1 && a.p.window > 0) {
        int64_t lo = len - a.p.window;  // keys with posQ - j < window
        if (jb < lo) jb = lo;
    }
}

// Merges the NW warp states (mm/ll [NW][G], oo [NW][G][HD]) and writes this
// CTA's (m, l, O) for heads hq0..hq0+G-1 — or the normalised output when the
// plan has a single split. The per-warp weights exp2(m_w - M) and the merged
// (M, L) of each head are computed once into `fw` (NW*G + 2*G floats of
// shared memory) before the per-element sums. Every thread of the CTA calls it.
template <int G, int HD, int NW>
__device__ __forceinline__ void write_result(const FDArgs& a, int64_t b, int64_t hq0, int split, const float* mm,
                                             const float* ll, const float* oo, float* fw, int tid, int nthreads) {
    const FlashDecode& p = a.p;
    float* Mg = fw + NW * G;
    float* Lg = Mg + G;
    if (tid < G) {
        const int g = tid;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < NW; ++w) M = fmaxf(M, mm[w * G + g]);
        float L = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            const float mw = mm[w * G + g];
            const float f = (M == -INFINITY || mw == -INFINITY) ? 0.f : exp2f(mw - M);
            fw[w * G + g] = f;
            L += f * ll[w * G + g];
        }
        Mg[g] = M;
        Lg[g] = L;
    }
    __syncthreads();
    for (int idx = tid; idx < G * HD; idx += nthreads) {
        const int g = idx / HD, d = idx % HD;
        const float M = Mg[g], L = Lg[g];
        float O = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) O += fw[w * G + g] * oo[(w * G + g) * HD + d];
        int64_t hq = hq0 + g;
        if (a.splits == 1) {
            float r = L > 0.f ? O * (1.0f / L) : 0.f;
            int64_t o = (b * p.Nq + hq) * HD + d;
            if (p.out_dtype == PC_F32) Elem<TF32>::store(p.out, o, r);
            else if (p.out_dtype == PC_BF16) Elem<TBF16>::store(p.out, o, r);
            else Elem<TF16>::store(p.out, o, r);
        } else {
            int64_t slot = (b * p.Nq + hq) * a.splits + split;
            a.po[slot * HD + d] = O;
            if (d == 0) {
                a.pm[slot] = M;
                a.pl[slot] = L;
            }
        }
    }
}

template <class KV, int HD, int G>
__global__ void __launch_bounds__(FDShape<KV, HD>::kThreads, 1) fd_partial_kernel(const FDArgs a) {
    using S = FDShape<KV, HD>;
    constexpr int E = S::E;
    constexpr int NST = S::kStages;
    constexpr int kGroups = S::kGroups;
    constexpr int kCWarps = S::kCWarps;
    constexpr int kFastThreads = S::kThreads;
    extern __shared__ __align__(128) char smem[];
    __shared__ __align__(8) uint64_t full[NST], empty[NST];
    __shared__ volatile int s_abort;
    __shared__ volatile int s_issued;
    __shared__ volatile int s_consumed[kGroups];
    DT_SHARED

    pdl_launch_dependents();
    const FlashDecode& p = a.p;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int split = blockIdx.x;
    const int64_t hkv = blockIdx.y / a.hgroups;
    const int hg = blockIdx.y % a.hgroups;
    const int64_t b = blockIdx.z;
    const int64_t gtot = p.Nq / p.Nkv;
    const int64_t hq0 = hkv * gtot + int64_t(hg) * G;

    if (tid == 0) {
        DT_INIT();
        DT_MARK(0);
        for (int s = 0; s < NST; ++s) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), 4);  // the four warps of the group that read it
        }
        s_abort = 0;
        s_issued = 0;
        for (int g = 0; g < kGroups; ++g) s_consumed[g] = 0;
        mbar_fence_init();
    }
    __syncthreads();

    const int64_t head_off = (b * p.Nkv + hkv) * p.S * HD;  // elements
    const char* kbase = static_cast<const char*>(p.k) + head_off * Elem<KV>::bytes;
    const char* vbase = static_cast<const char*>(p.v) + head_off * Elem<KV>::bytes;
    int n_early = 0;  // tiles the producer copied before the wait
    if (warp == kCWarps && lane == 0 && p.kv_early) {
        // The caller promised that the previous kernel writes neither
        // seq_lens nor any K/V row but the newest of each sequence: copy
        // every tile of this split that holds no newest row now, while the
        // previous kernel drains (the first NST tiles take stages whose
        // empty barriers have not been armed yet).
        const int64_t len0 = seq_len(p, b);
        int64_t jb0, je0;
        split_range(a, len0, split, jb0, je0);
        for (int t = 0; t < NST && jb0 + int64_t(t) * kTileKeys < je0; ++t) {
            const int64_t j0 = jb0 + int64_t(t) * kTileKeys;
            const int64_t nk = je0 - j0 < kTileKeys ? je0 - j0 : kTileKeys;
            if (j0 + nk >= len0) break;  // holds key len0 - 1, the newest
            const uint32_t bytes = uint32_t(nk) * S::kRowBytes;
            const uint32_t bar = smem_u32(&full[t]);
            mbar_expect_tx(bar, 2 * bytes);
            char* st = smem + size_t(t) * S::kStageBytes;
            bulk_g2s(smem_u32(st), kbase + j0 * S::kRowBytes, bytes, bar);
            bulk_g2s(smem_u32(st + S::kTileBytes), vbase + j0 * S::kRowBytes, bytes, bar);
            n_early = t + 1;
            s_issued = n_early;
            if (t == 0) DT_MARK(4);
        }
    } else if (warp == kCWarps && lane == 0) {
        // Before waiting for the previous kernel: warm L2 with this split's
        // keys. A prefetch only fills L2 (which always holds the latest data),
        // so rows the previous kernel is still writing are read correctly
        // after the wait; seq_lens read here only bounds the hint.
        int64_t hint_len = p.seq_lens ? int64_t(p.seq_lens[b]) : p.S;
        if (hint_len < 0 || hint_len > p.S) hint_len = p.S;
        int64_t pb, pe;
        split_range(a, hint_len, split, pb, pe);
        // Only the first ring's worth: L2 must still hold the lines when the
        // bulk copies read them, or the prefetch would double the traffic.
        if (pe > pb + int64_t(NST) * kTileKeys) pe = pb + int64_t(NST) * kTileKeys;
        for (int64_t j0 = pb; j0 < pe; j0 += kTileKeys) {
            const uint32_t bytes = uint32_t((pe - j0 < kTileKeys ? pe - j0 : kTileKeys) * S::kRowBytes);
            bulk_prefetch_l2(kbase + j0 * S::kRowBytes, bytes);
            bulk_prefetch_l2(vbase + j0 * S::kRowBytes, bytes);
        }
    }

    pdl_wait();  // q, the cache and seq_lens may come from the previous kernel
    if (tid == 0) DT_MARK(1);

    const int64_t len = seq_len(p, b);
    int64_t jb, je;
    split_range(a, len, split, jb, je);

    float* mm = reinterpret_cast<float*>(smem);
    float* ll = mm + kCWarps * G;
    float* oo = ll + kCWarps * G;

    if (jb >= je) {  // no keys for this split (FlashDecoding.metal:78-87)
        if (p.kv_early) {
            // Copies issued before the wait (only if the caller broke the
            // early-copy promise) land before the ring is reused.
            __syncthreads();
            if (tid == 0)
                for (int t = 0; t < s_issued; ++t) mbar_wait(smem_u32(&full[t]), 0u, &g_fd_error_word);
            __syncthreads();
        }
        if (tid < kCWarps * G) {
            mm[tid] = -INFINITY;
            ll[tid] = 0.f;
        }
        for (int i = tid; i < kCWarps * G * HD; i += kFastThreads) oo[i] = 0.f;
        __syncthreads();
        write_result<G, HD, kCWarps>(a, b, hq0, split, mm, ll, oo, oo + kCWarps * G * HD, tid, kFastThreads);
        return;
    }

    const int ntiles = int((je - jb + kTileKeys - 1) / kTileKeys);

    float m[G], l[G], o[G][E];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int e = 0; e < E; ++e) o[g][e] = 0.f;
    }

    if (warp == kCWarps) {
        // ---- producer ----
        if (lane == 0) {
            for (int t = n_early; t < ntiles; ++t) {
                const int s = t % NST;
                const uint32_t ph = uint32_t(t / NST) & 1u;
                if (s_abort || !mbar_wait(smem_u32(&empty[s]), ph ^ 1u, &g_fd_error_word)) {
                    s_abort = 1;
                    break;
                }
                const int64_t j0 = jb + int64_t(t) * kTileKeys;
                const int64_t nk = je - j0 < kTileKeys ? je - j0 : kTileKeys;
                const uint32_t bytes = uint32_t(nk) * S::kRowBytes;
                const uint32_t bar = smem_u32(&full[s]);
                mbar_expect_tx(bar, 2 * bytes);
                char* st = smem + size_t(s) * S::kStageBytes;
                bulk_g2s(smem_u32(st), kbase + j0 * S::kRowBytes, bytes, bar);
                bulk_g2s(smem_u32(st + S::kTileBytes), vbase + j0 * S::kRowBytes, bytes, bar);
                s_issued = t + 1;
                if (t == 0 && n_early == 0) DT_MARK(4);
                DT_MARK(7);
            }
            // Own loads issued: warm L2 for the next kernel of the chain.
            const int part = int(blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z));
            const int nparts = int(gridDim.x * gridDim.y * gridDim.z);
            for (int r = 0; r < 2; ++r) prefetch_share_l2(p.pf.ptr[r], p.pf.bytes[r], part, nparts);
        }
    } else {
        // ---- consumers: group `grp` takes tiles grp, grp + 2, ... ----
        const int grp = warp >> 2, gw = warp & 3;
        float q[G][E];
        const float qs = p.scale * kLog2e;
#pragma unroll
        for (int g = 0; g < G; ++g) {
            int64_t qb = ((b * p.Nq) + hq0 + g) * HD + lane * E;
#pragma unroll
            for (int e = 0; e < E; ++e) q[g][e] = Elem<KV>::load(p.q, qb + e) * qs;
        }
        for (int t = grp; t < ntiles; t += kGroups) {
            const int s = t % NST;
            const uint32_t parity = uint32_t(t / NST) & 1u;
            if (s_abort || !mbar_wait(smem_u32(&full[s]), parity, &g_fd_error_word)) {
                s_abort = 1;
                break;
            }
            if (tid == 0) {
                if (t == 0) DT_MARK(3);
                DT_MARK(6);
            }
            const int64_t j0 = jb + int64_t(t) * kTileKeys;
            const int nk = int(je - j0 < kTileKeys ? je - j0 : kTileKeys);
            const int kw0 = gw * 8;  // this warp's first key in the tile
            const char* ktile = smem + size_t(s) * S::kStageBytes;
            const char* vtile = ktile + S::kTileBytes;

            if (kw0 < nk) {
                // Partial dots: vals[i*G + g] for the warp's 8 keys.
                float vals[8 * G];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    float kf[E];
                    if (kw0 + i < nk) {
                        load_slice<KV, E>(ktile + (kw0 + i) * S::kRowBytes + lane * E * Elem<KV>::bytes, kf);
                    } else {
#pragma unroll
                        for (int e = 0; e < E; ++e) kf[e] = 0.f;
                    }
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        float acc = 0.f;
#pragma unroll
                        for (int e = 0; e < E; ++e) acc = fmaf(q[g][e], kf[e], acc);
                        vals[i * G + g] = acc;
                    }
                }
                // Transpose-reduction: after the xor-16/8/4 steps lane L holds
                // the partial sums of key (L >> 2) & 7; xor-2/1 finish them.
                {
                    const bool hi = lane & 16;
#pragma unroll
                    for (int i = 0; i < 4 * G; ++i) {
                        float lo_v = vals[i], hi_v = vals[i + 4 * G];
                        float send = hi ? lo_v : hi_v, keep = hi ? hi_v : lo_v;
                        vals[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
                    }
                }
                {
                    const bool hi = lane & 8;
#pragma unroll
                    for (int i = 0; i < 2 * G; ++i) {
                        float lo_v = vals[i], hi_v = vals[i + 2 * G];
                        float send = hi ? lo_v : hi_v, keep = hi ? hi_v : lo_v;
                        vals[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
                    }
                }
                {
                    const bool hi = lane & 4;
#pragma unroll
                    for (int i = 0; i < G; ++i) {
                        float lo_v = vals[i], hi_v = vals[i + G];
                        float send = hi ? lo_v : hi_v, keep = hi ? hi_v : lo_v;
                        vals[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
                    }
                }
                const int my_key = (lane >> 2) & 7;
                const bool valid = kw0 + my_key < nk;
                float pr[G];
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    float sv = vals[g];
                    sv += __shfl_xor_sync(0xffffffffu, sv, 2);
                    sv += __shfl_xor_sync(0xffffffffu, sv, 1);
                    float mx = valid ? sv : -INFINITY;
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
                    float mnew = fmaxf(m[g], mx);
                    float so = exp2f(m[g] - mnew);  // 0 while m is -inf
                    float pv = valid ? exp2f(sv - mnew) : 0.f;
                    float ps = pv;
                    ps += __shfl_xor_sync(0xffffffffu, ps, 4);
                    ps += __shfl_xor_sync(0xffffffffu, ps, 8);
                    ps += __shfl_xor_sync(0xffffffffu, ps, 16);
                    l[g] = l[g] * so + ps;
                    m[g] = mnew;
#pragma unroll
                    for (int e = 0; e < E; ++e) o[g][e] *= so;
                    pr[g] = pv;
                }
                // O += p_i * V_i over the warp's keys.
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    float pi[G];
#pragma unroll
                    for (int g = 0; g < G; ++g) pi[g] = __shfl_sync(0xffffffffu, pr[g], i * 4);
                    if (kw0 + i < nk) {
                        float vf[E];
                        load_slice<KV, E>(vtile + (kw0 + i) * S::kRowBytes + lane * E * Elem<KV>::bytes, vf);
#pragma unroll
                        for (int g = 0; g < G; ++g)
#pragma unroll
                            for (int e = 0; e < E; ++e) o[g][e] = fmaf(pi[g], vf[e], o[g][e]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&empty[s]));
            if (gw == 0 && lane == 0) s_consumed[grp] = t + 1;
        }
    }

    __syncthreads();  // every tile consumed (or abandoned); the ring is free
    if (p.kv_early) {
        // Early copies past the tile count seen after the wait (a broken
        // early-copy promise) are drained before the merge reuses the ring.
        if (tid == 0 && !s_abort)
            for (int t = ntiles; t < s_issued && t < NST; ++t)
                mbar_wait(smem_u32(&full[t]), 0u, &g_fd_error_word);
        __syncthreads();
    }
    if (s_abort) {
        if (tid == 0) {
            // Drain (bounded) the copies issued for tiles nobody consumed.
            int done = s_consumed[0];
            for (int g = 1; g < kGroups; ++g) done = s_consumed[g] < done ? s_consumed[g] : done;
            for (int t = done; t < s_issued; ++t)
                mbar_wait(smem_u32(&full[t % NST]), uint32_t(t / NST) & 1u, &g_fd_error_word);
        }
        __syncthreads();
        return;
    }

    // Merge the eight consumer warps' softmax states.
    if (warp < kCWarps) {
        if (lane == 0) {
#pragma unroll
            for (int g = 0; g < G; ++g) {
                mm[warp * G + g] = m[g];
                ll[warp * G + g] = l[g];
            }
        }
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int e = 0; e < E; ++e) oo[(warp * G + g) * HD + lane * E + e] = o[g][e];
    }
    __syncthreads();
    if (tid == 0) DT_MARK(2);
    write_result<G, HD, kCWarps>(a, b, hq0, split, mm, ll, oo, oo + kCWarps * G * HD, tid, kFastThreads);
    DT_COMMIT(200);
}

// Generic kernel (any Hd <= 512, any alignment, q dtype may differ from
// K/V): one query head per CTA, plain loads, one key per warp step.
template <class QT, class KV>
__global__ void __launch_bounds__(kThreads) fd_generic_kernel(const FDArgs a) {
    constexpr int MAXE = 16;
    __shared__ float mm[kWarps], ll[kWarps];
    extern __shared__ float oo[];  // [kWarps][Hd]
    pdl_launch_dependents();
    pdl_wait();
    const FlashDecode& p = a.p;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int split = blockIdx.x;
    const int64_t hq = blockIdx.y;
    const int64_t b = blockIdx.z;
    const int64_t Hd = p.Hd;
    const int64_t hkv = hq * p.Nkv / p.Nq;
    const int64_t len = seq_len(p, b);
    int64_t jb, je;
    split_range(a, len, split, jb, je);
    float q[MAXE], o[MAXE];
    const float qs = p.scale * kLog2e;
    for (int i = 0; i < MAXE; ++i) {
        int64_t d = lane + 32 * i;
        q[i] = d < Hd ? Elem<QT>::load(p.q, (b * p.Nq + hq) * Hd + d) * qs : 0.f;
        o[i] = 0.f;
    }
    float m = -INFINITY, l = 0.f;
    const int64_t kv0 = (b * p.Nkv + hkv) * p.S;
    for (int64_t j = jb + warp; j < je; j += kWarps) {
        float acc = 0.f;
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
        for (int i = 0; i < MAXE; ++i) {
            int64_t d = lane + 32 * i;
            float vv = d < Hd ? Elem<KV>::load(p.v, (kv0 + j) * Hd + d) : 0.f;
            o[i] = fmaf(pv, vv, o[i] * so);
        }
    }
    if (lane == 0) {
        mm[warp] = m;
        ll[warp] = l;
    }
    for (int i = 0; i < MAXE; ++i) {
        int64_t d = lane + 32 * i;
        if (d < Hd) oo[warp * Hd + d] = o[i];
    }
    __syncthreads();
    for (int64_t d = tid; d < Hd; d += kThreads) {
        float M = -INFINITY;
        for (int w = 0; w < kWarps; ++w) M = fmaxf(M, mm[w]);
        float L = 0.f, O = 0.f;
        if (M != -INFINITY) {
            for (int w = 0; w < kWarps; ++w) {
                float f = mm[w] == -INFINITY ? 0.f : exp2f(mm[w] - M);
                L += f * ll[w];
                O += f * oo[w * Hd + d];
            }
        }
        if (a.splits == 1) {
            float r = L > 0.f ? O * (1.0f / L) : 0.f;
            int64_t oi = (b * p.Nq + hq) * Hd + d;
            if (p.out_dtype == PC_F32) Elem<TF32>::store(p.out, oi, r);
            else if (p.out_dtype == PC_BF16) Elem<TBF16>::store(p.out, oi, r);
            else Elem<TF16>::store(p.out, oi, r);
        } else {
            int64_t slot = (b * p.Nq + hq) * a.splits + split;
            a.po[slot * Hd + d] = O;
            if (d == 0) {
                a.pm[slot] = M;
                a.pl[slot] = L;
            }
        }
    }
}

// Log-sum-exp combine of the splits (FlashDecoding.metal:182-231).
// One CTA of 256 threads per (b, hq). The split weights exp2(m_s - M) go to
// shared memory once; then the threads form groups x columns (a column is 4
// head dims, loaded as float4): each thread sums its column over every
// groups-th split with several independent loads in flight, and the group
// partial sums are added in shared memory.
constexpr int kCombThreads = 256;
constexpr int kCombK = 8;  // splits per thread on the one-round-trip path

// blockIdx.z takes head dims [z * dchunk, (z + 1) * dchunk): more CTAs for
// the few (b, hq) rows of a decode step.
template <class OT>
__global__ void __launch_bounds__(kCombThreads) fd_combine_kernel(const float* po, const float* pm, const float* pl,
                                                                  void* out, int64_t Nq, int64_t Hd, int splits,
                                                                  int64_t dchunk) {
    extern __shared__ float sh[];  // wts[splits (padded to 4)], part[groups][dchunk]
    float* wts = sh;
    float* part = sh + ((splits + 3) & ~3);
    __shared__ float red[kCombThreads / 32];
    __shared__ float s_M, s_L;
    DT_SHARED
    if (threadIdx.x == 0) {
        DT_INIT();
        DT_MARK(0);
    }
    pdl_launch_dependents();
    pdl_wait();
    if (threadIdx.x == 0) DT_MARK(1);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t bh = int64_t(blockIdx.y) * Nq + blockIdx.x;
    const float* m = pm + bh * splits;
    const float* l = pl + bh * splits;
    {
        // Few splits (every decode step): each thread owns one float4
        // column of the chunk and up to kCombK splits, and issues all of its
        // loads (m, l and O of those splits) at once, so the whole combine
        // costs one round trip to L2 and two CTA barriers.
        const int64_t d0 = int64_t(blockIdx.z) * dchunk;
        const int64_t dn = Hd - d0 < dchunk ? Hd - d0 : dchunk;
        const int cols = int(dn / 4);
        const int groups = cols > 0 ? kCombThreads / cols : 0;
        if ((Hd & 3) == 0 && (dn & 3) == 0 && cols > 0 && cols <= kCombThreads && splits <= groups * kCombK) {
            float* red_m = sh;                    // [groups]
            float* red_l = sh + groups;           // [groups]
            float4* part = reinterpret_cast<float4*>(sh + 2 * ((groups + 1) & ~1));  // [groups][cols]
            const int col = tid % cols, grp = tid / cols;
            const bool act = grp < groups;
            const float* o = po + bh * splits * Hd + d0;
            float ms[kCombK], ls[kCombK];
            float4 ov[kCombK];
#pragma unroll
            for (int k = 0; k < kCombK; ++k) {
                const int s = grp + k * groups;
                if (act && s < splits) {
                    ms[k] = m[s];
                    ls[k] = l[s];
                    ov[k] = reinterpret_cast<const float4*>(o + int64_t(s) * Hd)[col];
                } else {
                    ms[k] = -INFINITY;
                    ls[k] = 0.f;
                    ov[k] = make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
            float mloc = -INFINITY;
#pragma unroll
            for (int k = 0; k < kCombK; ++k) mloc = fmaxf(mloc, ms[k]);
            if (act && col == 0) red_m[grp] = mloc;
            __syncthreads();
            float M = -INFINITY;
            for (int g = 0; g < groups; ++g) M = fmaxf(M, red_m[g]);
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            float lsum = 0.f;
#pragma unroll
            for (int k = 0; k < kCombK; ++k) {
                const float f = (M == -INFINITY || ms[k] == -INFINITY) ? 0.f : exp2f(ms[k] - M);
                lsum = fmaf(f, ls[k], lsum);
                acc.x = fmaf(f, ov[k].x, acc.x); acc.y = fmaf(f, ov[k].y, acc.y);
                acc.z = fmaf(f, ov[k].z, acc.z); acc.w = fmaf(f, ov[k].w, acc.w);
            }
            if (act) {
                part[grp * cols + col] = acc;
                if (col == 0) red_l[grp] = lsum;
            }
            __syncthreads();
            float L = 0.f;
            for (int g = 0; g < groups; ++g) L += red_l[g];
            const float inv_l = L > 0.f ? 1.0f / L : 0.f;
            for (int d = tid; d < dn; d += kCombThreads) {
                const int c = d >> 2, e = d & 3;
                float v = 0.f;
                for (int g = 0; g < groups; ++g) v += reinterpret_cast<const float*>(part + g * cols + c)[e];
                Elem<OT>::store(out, bh * Hd + d0 + d, v * inv_l);
            }
            DT_COMMIT(201);
            return;
        }
    }
    float mx = -INFINITY;
    for (int s = tid; s < splits; s += kCombThreads) mx = fmaxf(mx, m[s]);
    mx = warp_max(mx);
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    if (tid == 0) {
        float v = red[0];
        for (int w = 1; w < kCombThreads / 32; ++w) v = fmaxf(v, red[w]);
        s_M = v;
    }
    __syncthreads();
    const float M = s_M;
    float lsum = 0.f;
    for (int s = tid; s < splits; s += kCombThreads) {
        float f = (M == -INFINITY || m[s] == -INFINITY) ? 0.f : exp2f(m[s] - M);
        wts[s] = f;
        lsum += f * l[s];
    }
    lsum = warp_sum(lsum);
    __syncthreads();
    if (lane == 0) red[warp] = lsum;
    __syncthreads();
    if (tid == 0) {
        float v = 0.f;
        for (int w = 0; w < kCombThreads / 32; ++w) v += red[w];
        s_L = v;
    }
    __syncthreads();
    const int64_t d0 = int64_t(blockIdx.z) * dchunk;
    const int64_t dn = Hd - d0 < dchunk ? Hd - d0 : dchunk;
    const float* o = po + bh * splits * Hd + d0;
    const float L = s_L;
    const float inv_l = L > 0.f ? 1.0f / L : 0.f;
    if ((Hd & 3) == 0 && (dn & 3) == 0 && dn / 4 <= kCombThreads) {
        const int cols = int(dn / 4);
        const int groups = kCombThreads / cols;
        const int col = tid % cols, grp = tid / cols;
        if (grp < groups) {
            float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0;
            int s = grp;
            for (; s + groups < splits; s += 2 * groups) {
                float4 v0 = reinterpret_cast<const float4*>(o + int64_t(s) * Hd)[col];
                float4 v1 = reinterpret_cast<const float4*>(o + int64_t(s + groups) * Hd)[col];
                float w0 = wts[s], w1 = wts[s + groups];
                a0.x = fmaf(w0, v0.x, a0.x); a0.y = fmaf(w0, v0.y, a0.y);
                a0.z = fmaf(w0, v0.z, a0.z); a0.w = fmaf(w0, v0.w, a0.w);
                a1.x = fmaf(w1, v1.x, a1.x); a1.y = fmaf(w1, v1.y, a1.y);
                a1.z = fmaf(w1, v1.z, a1.z); a1.w = fmaf(w1, v1.w, a1.w);
            }
            if (s < splits) {
                float4 v0 = reinterpret_cast<const float4*>(o + int64_t(s) * Hd)[col];
                float w0 = wts[s];
                a0.x = fmaf(w0, v0.x, a0.x); a0.y = fmaf(w0, v0.y, a0.y);
                a0.z = fmaf(w0, v0.z, a0.z); a0.w = fmaf(w0, v0.w, a0.w);
            }
            float4 r = make_float4(a0.x + a1.x, a0.y + a1.y, a0.z + a1.z, a0.w + a1.w);
            reinterpret_cast<float4*>(part + int64_t(grp) * dn)[col] = r;
        }
        __syncthreads();
        for (int64_t d = tid; d < dn; d += kCombThreads) {
            float acc = 0.f;
            for (int g = 0; g < groups; ++g) acc += part[g * dn + d];
            Elem<OT>::store(out, bh * Hd + d0 + d, acc * inv_l);
        }
    } else {
        for (int64_t d = tid; d < dn; d += kCombThreads) {
            float acc = 0.f;
            for (int s = 0; s < splits; ++s) acc = fmaf(wts[s], o[int64_t(s) * Hd + d], acc);
            Elem<OT>::store(out, bh * Hd + d0 + d, acc * inv_l);
        }
    }
    DT_COMMIT(201);
}

bool fast_path(const FlashDecode& p) {
    bool hd_ok = p.Hd == 64 || p.Hd == 128 || p.Hd == 256 || p.Hd == 512;
    bool ring_fits = !(p.kv_dtype == PC_F32 && p.Hd == 512);  // two stages must fit
    return hd_ok && ring_fits && p.q_dtype == p.kv_dtype && aligned16(p.k) && aligned16(p.v);
}

int heads_per_cta(const FlashDecode& p) {
    int64_t g = p.Nq / p.Nkv;
    int64_t cap = 32 / (p.Hd / 32);  // G * Hd/32 <= 32
    for (int c : {8, 4, 2})
        if (c <= cap && g % c == 0) return c;
    return 1;
}

template <class KV, int HD, int G>
cudaError_t run_fast(const FDArgs& a, dim3 grid, cudaStream_t s) {
    auto kern = fd_partial_kernel<KV, HD, G>;
    constexpr size_t smem = fd_smem_bytes<KV, HD, G>();
    static bool configured = false;
    if (!configured) {
        cudaError_t e = allow_smem(kern, smem);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    return launch_k(kern, grid, dim3(FDShape<KV, HD>::kThreads), smem, s, a);
}

// Register budget: q and O slices take 2*G*Hd/32 floats per lane; keep
// G*Hd/32 <= 32 (the plan never asks for more).
template <class KV, int HD>
cudaError_t run_fast_g(const FDArgs& a, dim3 grid, cudaStream_t s) {
    switch (a.G) {
    case 1: return run_fast<KV, HD, 1>(a, grid, s);
    case 2: return run_fast<KV, HD, 2>(a, grid, s);
    case 4:
        if constexpr (HD <= 256) return run_fast<KV, HD, 4>(a, grid, s);
        break;
    case 8:
        if constexpr (HD <= 128) return run_fast<KV, HD, 8>(a, grid, s);
        break;
    }
    return cudaErrorInvalidValue;
}

template <class KV>
cudaError_t run_fast_hd(const FDArgs& a, dim3 grid, cudaStream_t s) {
    switch (a.p.Hd) {
    case 64: return run_fast_g<KV, 64>(a, grid, s);
    case 128: return run_fast_g<KV, 128>(a, grid, s);
    case 256: return run_fast_g<KV, 256>(a, grid, s);
    case 512: return run_fast_g<KV, 512>(a, grid, s);
    }
    return cudaErrorInvalidValue;
}

template <class QT>
cudaError_t run_generic_q(const FDArgs& a, dim3 grid, cudaStream_t s) {
    size_t smem = size_t(kWarps) * a.p.Hd * 4;
    switch (a.p.kv_dtype) {
    case PC_F32: return launch_k(fd_generic_kernel<QT, TF32>, grid, dim3(kThreads), smem, s, a);
    case PC_F16: return launch_k(fd_generic_kernel<QT, TF16>, grid, dim3(kThreads), smem, s, a);
    case PC_BF16: return launch_k(fd_generic_kernel<QT, TBF16>, grid, dim3(kThreads), smem, s, a);
    }
    return cudaErrorInvalidValue;
}

}  // namespace

// Split plan. The fast kernel runs one CTA per SM, so the grid should be
// whole waves of sm_count CTAs: among split counts from the smallest that
// fills one wave up to four times that, pick the one whose waves x
// keys-per-split is least (ties: fewer splits, i.e. less combine work).
FlashDecodePlan flash_decode_plan(const FlashDecode& p, int sm_count) {
    FlashDecodePlan plan{};
    plan.fast = fast_path(p);
    plan.heads_per_cta = plan.fast ? heads_per_cta(p) : 1;
    const int64_t hgroups = (p.Nq / p.Nkv) / plan.heads_per_cta;
    const int64_t base = p.B * p.Nkv * hgroups;
    const int64_t wave = plan.fast ? int64_t(sm_count) : int64_t(sm_count) * 4;
    int64_t max_tiles = (p.S + kTileKeys - 1) / kTileKeys;
    if (max_tiles < 1) max_tiles = 1;
    int64_t s_lo = (wave + base - 1) / base;
    if (s_lo < 1) s_lo = 1;
    // Cap the keys per split so that uneven work (ragged lengths leave some
    // splits short or empty; later waves start when earlier CTAs finish)
    // averages out over many CTAs.
    const int64_t tile_cap = p.seq_lens ? 64 : 256;
    const int64_t s_min = (max_tiles + tile_cap - 1) / tile_cap;
    const int64_t s_hi = std::max(s_lo * 4, s_min);
    int64_t best_tiles = 0;
    double best_cost = 1e30;
    for (int64_t s = std::max<int64_t>(1, s_min); s <= s_hi && s <= max_tiles && s <= 1024; ++s) {
        int64_t tiles = (max_tiles + s - 1) / s;   // tiles per split
        int64_t splits = (max_tiles + tiles - 1) / tiles;
        int64_t ctas = base * splits;
        int64_t waves = (ctas + wave - 1) / wave;
        double cost = double(waves) * double(tiles) + 0.02 * double(splits);
        if (cost < best_cost - 1e-9) {
            best_cost = cost;
            best_tiles = tiles;
        }
    }
    if (best_tiles == 0) best_tiles = max_tiles;
    plan.chunk = best_tiles * kTileKeys;
    plan.splits = int((p.S + plan.chunk - 1) / plan.chunk);
    if (plan.splits < 1) plan.splits = 1;
    plan.scratch_o = size_t(p.B * p.Nq) * plan.splits * p.Hd * 4;
    plan.scratch_ml = size_t(p.B * p.Nq) * plan.splits * 4;
    return plan;
}

cudaError_t flash_decode(const FlashDecode& p, const FlashDecodePlan& plan, float* po, float* pm, float* pl,
                         cudaStream_t s) {
    FDArgs a{p, plan.splits, plan.chunk, plan.heads_per_cta, int((p.Nq / p.Nkv) / plan.heads_per_cta), po, pm, pl};
    if (plan.fast) {
        dim3 grid(unsigned(plan.splits), unsigned(p.Nkv * a.hgroups), unsigned(p.B));
        switch (p.kv_dtype) {
        case PC_BF16: return run_fast_hd<TBF16>(a, grid, s);
        case PC_F16: return run_fast_hd<TF16>(a, grid, s);
        case PC_F32: return run_fast_hd<TF32>(a, grid, s);
        default: return cudaErrorInvalidValue;
        }
    }
    dim3 grid(unsigned(plan.splits), unsigned(p.Nq), unsigned(p.B));
    switch (p.q_dtype) {
    case PC_F32: return run_generic_q<TF32>(a, grid, s);
    case PC_F16: return run_generic_q<TF16>(a, grid, s);
    case PC_BF16: return run_generic_q<TBF16>(a, grid, s);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t flash_decode_combine(const FlashDecode& p, const FlashDecodePlan& plan, const float* po, const float* pm,
                                 const float* pl, cudaStream_t s) {
    if (plan.splits <= 1) return cudaSuccess;
    // 64 head dims per CTA when that gives more CTAs for few rows
    const int64_t dchunk = (p.Hd % 64 == 0 && p.Hd > 64 && p.B * p.Nq < 4 * current_sm_count()) ? 64 : p.Hd;
    dim3 grid(unsigned(p.Nq), unsigned(p.B), unsigned(p.Hd / dchunk));
    const int64_t groups = (dchunk % 4 == 0 && dchunk / 4 <= kCombThreads) ? kCombThreads / (dchunk / 4) : 0;
    size_t smem = (size_t((plan.splits + 3) & ~3) + size_t(groups) * dchunk + 2 * size_t(groups + 2)) * 4;
    switch (p.out_dtype) {
    case PC_F32:
        return launch_k(fd_combine_kernel<TF32>, grid, dim3(kCombThreads), smem, s, po, pm, pl, p.out, p.Nq, p.Hd,
                        plan.splits, dchunk);
    case PC_F16:
        return launch_k(fd_combine_kernel<TF16>, grid, dim3(kCombThreads), smem, s, po, pm, pl, p.out, p.Nq, p.Hd,
                        plan.splits, dchunk);
    case PC_BF16:
        return launch_k(fd_combine_kernel<TBF16>, grid, dim3(kCombThreads), smem, s, po, pm, pl, p.out, p.Nq, p.Hd,
                        plan.splits, dchunk);
    }
    return cudaErrorInvalidValue;
}

uint32_t read_and_clear_fd_errors() {
    unsigned int v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_fd_error_word, sizeof(v)) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    if (v) cudaMemcpyToSymbol(g_fd_error_word, &zero, sizeof(zero));
    return v;
}

namespace {
RegisterFunctions reg_fd({
    {"flash_decoding_partial_bf16", reinterpret_cast<const void*>(fd_partial_kernel<TBF16, 256, 2>)},
    {"flash_decoding_partial_f16", reinterpret_cast<const void*>(fd_partial_kernel<TF16, 256, 2>)},
    {"flash_decoding_partial_f32", reinterpret_cast<const void*>(fd_partial_kernel<TF32, 256, 2>)},
    {"flash_decoding_partial_generic", reinterpret_cast<const void*>(fd_generic_kernel<TF32, TF32>)},
    {"flash_decoding_reduce_bf16", reinterpret_cast<const void*>(fd_combine_kernel<TBF16>)},
    {"flash_decoding_reduce_f16", reinterpret_cast<const void*>(fd_combine_kernel<TF16>)},
    {"flash_decoding_reduce_f32", reinterpret_cast<const void*>(fd_combine_kernel<TF32>)},
});
}  // namespace

uint32_t read_and_clear_gemv_errors();
uint32_t read_and_clear_gemm_errors();
uint32_t read_and_clear_fa_errors();
uint32_t read_and_clear_allreduce_errors();
uint32_t read_and_clear_step_errors();
uint32_t read_and_clear_aq_errors();

}  // namespace launch
}  // namespace popcorn

#ifdef PC_DECODE_TRACE
extern "C" __attribute__((visibility("default"))) int pc_debug_fd_trace(unsigned long long* host, int max,
                                                                        int reset) {
    unsigned int n = 0;
    cudaDeviceSynchronize();
    cudaMemcpyFromSymbol(&n, popcorn::launch::g_dt_n, sizeof(n));
    if (n > PC_DT_MAX) n = PC_DT_MAX;
    if (host && max > 0)
        cudaMemcpyFromSymbol(host, popcorn::launch::g_dt_buf, size_t(n < unsigned(max) ? n : max) * 9 * 8);
    if (reset) {
        unsigned int z = 0;
        cudaMemcpyToSymbol(popcorn::launch::g_dt_n, &z, sizeof(z));
    }
    return int(n);
}
#endif

extern "C" int pc_device_error_check(int device, uint32_t* flags) {
    int prev = 0;
    cudaGetDevice(&prev);
    if (cudaSetDevice(device) != cudaSuccess) {
        cudaGetLastError();
        return PC_ERR_GPU_DEVICE_REMOVED;
    }
    cudaDeviceSynchronize();
    *flags = popcorn::launch::read_and_clear_fd_errors() | popcorn::launch::read_and_clear_gemv_errors() |
             popcorn::launch::read_and_clear_gemm_errors() | popcorn::launch::read_and_clear_step_errors() |
             popcorn::launch::read_and_clear_fa_errors() | popcorn::launch::read_and_clear_allreduce_errors() |
             popcorn::launch::read_and_clear_aq_errors();
    cudaSetDevice(prev);
    return PC_OK;
}
