// decode_step.cu — one persistent kernel for a whole batch-1 decode step
// through a stack of layers (the config-2 Gemma-2-2B-shape layer).
//
// Each layer is the same op sequence as the five-kernel path (decode.py),
// with the same rounding points (every intermediate rounded to the
// activation dtype where the unfused reference op stores it):
//   op0  qkv  = W_qkv . round(RMSNorm(x))        q -> q, k/v -> caches[pos]
//   op1  split-KV attention partials over caches[0 .. pos]
//   op2  log-sum-exp combine -> attn
//   op3  h    = x + round(W_o . attn)
//   op4  act  = round(act(round(W_g . hn))) * round(W_u . hn), hn = round(RMSNorm(h))
//   op5  x'   = h + round(W_d . act)
// (Gemma4TextInference.swift:312-436; FlashDecoding.metal:29-231;
// Matvec.metal:56-127; RMSNorm.metal:7-42; GeluTanh / Mul / Add .metal.)
//
// Why one kernel. At batch 1 every op streams a few to 85 MB once; as
// separate launches each pays a ramp-up and a drain of the HBM pipe. Here
// one CTA per SM (co-resident, cooperative launch) walks every op of every
// layer. Sixteen consumer warps form four groups of four; each group has its
// own two-slot shared-memory ring and its own producer warp, which walks the
// CTA's stages in consumption order (StageCursor) and fills the group's
// slots with ONE 1-D bulk copy per stage (no multicast): four whole weight
// rows (a warp per row), one 16-18 KB column chunk of a long row (the four
// warps split it), or one 32-key K or V tile. Gate and up rows travel in
// separate stages. A second cursor runs up to l2_ahead bytes ahead issuing
// L2 prefetches. The weights of the next op therefore stream while the
// consumers still finish the current one.
//
// Ops are ordered by per-op arrival counters in global memory (release: a
// CTA barrier, then one thread's threadfence + atomicAdd; acquire:
// ld.acquire). No copy ever waits: the attention tile holding the new K/V row
// is copied early too, and its consumers patch that one row from global
// memory after op0's counter is complete. The split-KV combine (op2) runs
// inside op1: the splits of a KV head (never more attention items than
// CTAs, so all run at once) count in on a per-head counter, wait for each
// other, and each combines a 1/splits slice of the head's outputs.
//
// Measured on B200 (config 2, 26 layers, ctx 4096): 1.402 ms per token;
// the five-kernel graph, whose GEMV prologues were since shortened, takes
// 1.311 ms. Streaming phases reach 5.4-6.9 TB/s; what remains is latency at
// each op boundary (the activation row's loads queue behind the SM's
// in-flight weight copies) and in the attention phase.
//
// Every wait (mbarrier or counter) is bounded: on give-up the CTA sets the
// device error word and skips its remaining work but keeps taking part in
// every CTA barrier, so nothing hangs; the caller must then re-zero the
// workspace counters.
#include <cstdlib>

#include "async.cuh"
#include "common.cuh"
#include "dtype.cuh"
#include "launch.hpp"
#include "popcorn.hpp"

namespace popcorn {

__device__ unsigned int g_step_error_word;

#ifdef PC_STEP_TRACE
// Development-only timeline: per CTA and op, globaltimer at consumer start,
// consumer end and the producer's first issue.
constexpr int kTraceMax = 160 * 64 * 6 * 3;
__device__ unsigned long long g_step_trace[kTraceMax];
__device__ __forceinline__ void trace_mark(int slot) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    if (slot < kTraceMax) g_step_trace[slot] = t;
}
#define TRACE(l, k, w) trace_mark(((blockIdx.x * 64 + (l)) * 6 + (k)) * 3 + (w))
#else
#define TRACE(l, k, w) ((void)0)
#endif

namespace launch {

namespace {

constexpr int kHD = 256;                  // head dim served
constexpr int kE = kHD / 32;              // head dims per lane
constexpr int kCW = 16;                   // consumer warps
constexpr int kStepThreads = (kCW + 4) * 32;   // 16 consumer warps + one producer warp per group
constexpr int kGroups = 4;                // consumer groups of 4 warps, each with its own ring
constexpr int kGW = kCW / kGroups;        // warps per group = weight rows per GEMV tile
constexpr int kSlots = 2;                 // ring slots per group
constexpr int kRing = kGroups * kSlots;
constexpr int kStageMax = 20 * 1024;
constexpr int kTileKeys = 32;
constexpr int kChunkRegs = 3;             // 8-element chunks per consumer thread: rows up to 12288
constexpr int kNormChunks = 2;            // normalised rows (hidden size) up to 8192
constexpr int kOps = 6;
constexpr float kLog2e = 1.4426950408889634f;

struct GemvOp {
    const void* w;
    const void* w2;
    int K, N, R, rows, kc, nkc;
};

__device__ __forceinline__ unsigned int ld_acquire(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Bounded spin until *c >= target; false on give-up.
__device__ __forceinline__ bool wait_counter(const unsigned int* c, unsigned int target) {
    for (long i = 0; i < 4000000; ++i) {
        if (ld_acquire(c) >= target) return true;
        __nanosleep(32);
    }
    atomicOr(&g_step_error_word, 1u);
    return false;
}

__device__ __forceinline__ uint4 ldcg16(const void* p) {
    return __ldcg(reinterpret_cast<const uint4*>(p));
}

template <class T>
__device__ __forceinline__ float widen16(uint32_t bits) {
    uint16_t b = static_cast<uint16_t>(bits);
    return Elem<T>::load(&b, 0);
}

// One head of 256 elements held by a warp, 8 per lane (lane l: elements
// 8l..8l+7): RMSNorm with weight w (NULL = none) when `norm`, the result
// rounded to T as RMSNorm stores it; then, when cs is set, RoPE with table
// row (cs, sn): element i pairs with i + 128, which lane l ^ 16 holds, and
// the rotated value is rounded as RopeApply stores it (RMSNorm.metal:7-42,
// RopeApply.metal:6-49). Every lane of the warp must call it.
template <class T>
__device__ __forceinline__ void head_norm_rope(float* f, int lane, bool norm, const float* w, float eps,
                                               bool add_one, const float* cs, const float* sn) {
    if (norm) {
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) ss += f[e] * f[e];
        ss = warp_sum(ss);
        const float scale = rsqrtf(ss / float(kHD) + eps);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            float v = f[e] * scale;
            if (w) v *= add_one ? 1.0f + w[lane * 8 + e] : w[lane * 8 + e];
            f[e] = Elem<T>::round(v);
        }
    }
    if (cs) {
        const int i0 = (lane & 15) * 8;
        const bool second = lane & 16;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const float other = __shfl_xor_sync(0xffffffffu, f[e], 16);
            const float c = __ldg(cs + i0 + e), sv = __ldg(sn + i0 + e);
            f[e] = Elem<T>::round(second ? other * sv + f[e] * c : f[e] * c - other * sv);
        }
    }
}

template <class T>
__device__ __forceinline__ uint4 pack8(const float* f) {
    return make_uint4(pack2<T>(f[0], f[1]), pack2<T>(f[2], f[3]), pack2<T>(f[4], f[5]), pack2<T>(f[6], f[7]));
}

}  // namespace

// The producer's walk over every stage this CTA loads in one step, in
// consumption order. One cursor issues the ring copies; a second one runs
// ahead of it issuing L2 prefetches, so HBM keeps streaming while the
// consumers wait at an op boundary with a full ring.
struct StageCursor {
    const DecodeStep* p;
    int bid, grid, len, ktiles;
    int l, k;            // op
    int unit;            // GEMV: tile; attention: item
    int t, t1;           // attention: key tile within the item, end
    int kci, m;          // GEMV: column chunk, matrix; attention: m = K / V
    int rot;             // tile counter (group = rot % kGroups)
    bool valid;
    // the current op, loaded once when the cursor enters it
    const char* w0;      // GEMV: weights (gate); attention: K cache
    const char* w1;      // up weights; attention: V cache
    int K, N, tr, kc, nkc, R, ntiles, nitems;

    __device__ void init(const DecodeStep* p_, int bid_, int grid_, int len_) {
        p = p_;
        bid = bid_;
        grid = grid_;
        len = len_;
        ktiles = (len + kTileKeys - 1) / kTileKeys;
        nitems = p->Nkv * p->splits;
        l = 0;
        k = -1;
        rot = 0;
        valid = true;
        next_op();
    }
    // attention item -> first / end key tile (end clipped to the context)
    __device__ bool item_tiles(int item) {
        const int split = item % p->splits;
        t = split * p->chunk_tiles;
        t1 = t + p->chunk_tiles;
        if (t1 > ktiles) t1 = ktiles;
        return t < t1;
    }
    __device__ void load_op() {
        const DecodeLayer& L = p->layers[l];
        if (k == 1) {
            w0 = static_cast<const char*>(L.k_cache);
            w1 = static_cast<const char*>(L.v_cache);
            return;
        }
        const int i = k == 0 ? 0 : k - 2;  // ops 0, 3, 4, 5 -> plan slots 0..3
        K = k == 0 ? p->H : k == 3 ? p->Nq * kHD : k == 4 ? p->H : p->F;
        N = k == 0 ? (p->Nq + 2 * p->Nkv) * kHD : k == 4 ? p->F : p->H;
        R = k == 4 ? 2 : 1;
        w0 = static_cast<const char*>(k == 0 ? L.w_qkv : k == 3 ? L.w_o : k == 4 ? L.w_gate : L.w_down);
        w1 = static_cast<const char*>(L.w_up);
        tr = p->rows[i];
        kc = p->kc[i];
        nkc = p->nkc[i];
        ntiles = (N + tr - 1) / tr;
    }
    __device__ void next_op() {
        for (;;) {
            ++k;
            if (k == kOps) {
                k = 0;
                ++l;
            }
            if (l >= p->L) {
                valid = false;
                return;
            }
            if (k == 2) continue;
            kci = m = 0;
            load_op();
            if (k == 1) {
                for (unit = bid; unit < nitems; unit += grid)
                    if (item_tiles(unit)) return;
            } else {
                unit = bid;
                if (unit < ntiles) return;
            }
        }
    }
    __device__ void advance() {
        if (k == 1) {
            if (++m < 2) return;
            m = 0;
            ++rot;
            if (++t < t1) return;
            for (unit += grid; unit < nitems; unit += grid)
                if (item_tiles(unit)) return;
            next_op();
            return;
        }
        if (++m < R) return;
        m = 0;
        if (++kci < nkc) return;
        kci = 0;
        ++rot;
        unit += grid;
        if (unit < ntiles) return;
        next_op();
    }
    // Source, size and group of the current stage; `needs_op0` when it holds
    // the K/V row that op0 of this layer writes (the copy is then stale in
    // that row and the consumers patch it).
    __device__ const char* src(uint32_t& bytes, int& group, bool& needs_op0) const {
        group = rot % kGroups;
        if (k == 1) {
            const int hkv = unit / p->splits;
            const int64_t j0 = int64_t(t) * kTileKeys;
            const int nk = int(len - j0 < kTileKeys ? len - j0 : kTileKeys);
            bytes = uint32_t(nk) * kHD * 2;
            needs_op0 = t == ktiles - 1;
            return (m ? w1 : w0) + (int64_t(hkv) * p->Smax + j0) * kHD * 2;
        }
        needs_op0 = false;
        const int n0 = unit * tr;
        const int nvalid = N - n0 < tr ? N - n0 : tr;
        const int k0 = kci * kc;
        const int kcols = K - k0 < kc ? K - k0 : kc;
        bytes = uint32_t(kcols) * 2 * nvalid;
        return (m ? w1 : w0) + (int64_t(n0) * K + k0) * 2;
    }
};

// QK: the layers carry the per-head q / k / v norms and RoPE (a separate
// instance, so the plain layer's attention items carry none of that code).
template <class T, int GQ, bool QK>
__global__ void __launch_bounds__(kStepThreads, 1) decode_step_kernel(const __grid_constant__ DecodeStep p) {
    extern __shared__ __align__(128) unsigned char smem[];
    // full/empty barrier of slot s of group g at index g * kSlots + s
    __shared__ __align__(8) uint64_t full[kRing], empty[kRing];
    __shared__ float red[kCW];
    __shared__ float gpart[2][kGroups][kGW * 2];  // per-warp row segment sums
    __shared__ volatile int s_abort;
    unsigned char* ring = smem;
    // The activation planes (GEMV ops) and the attention warp states share
    // one area: ops are separated by a barrier of all consumer warps.
    float* xsf = reinterpret_cast<float*>(smem + kRing * kStageMax);
    float* merge = xsf;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    constexpr int G = GQ;  // query heads per KV head
    const int grid = gridDim.x;

    if (tid == 0) {
        for (int s = 0; s < kRing; ++s) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), kGW);  // every warp of the group arrives
        }
        s_abort = 0;
        mbar_fence_init();
    }
    __syncthreads();
    pdl_launch_dependents();
    pdl_wait();

    const int pos = p.pos[0];
    const int len = pos + 1;
    if (tid == 0 && (pos < 0 || pos >= p.Smax || (p.rope_rows > 1 && pos >= p.rope_rows))) {
        atomicOr(&g_step_error_word, 2u);  // position outside the cache: do nothing
        s_abort = 1;
    }
    __syncthreads();
    const int ktiles_total = (len + kTileKeys - 1) / kTileKeys;
    unsigned int* head_cnt = p.counters + p.L * kOps + 1;

    auto gemv_op = [&](int l, int k) -> GemvOp {
        const DecodeLayer& L = p.layers[l];
        switch (k) {
        case 0: return {L.w_qkv, nullptr, p.H, (p.Nq + 2 * p.Nkv) * kHD, 1, p.rows[0], p.kc[0], p.nkc[0]};
        case 3: return {L.w_o, nullptr, p.Nq * kHD, p.H, 1, p.rows[1], p.kc[1], p.nkc[1]};
        case 4: return {L.w_gate, L.w_up, p.H, p.F, 2, p.rows[2], p.kc[2], p.nkc[2]};
        default: return {L.w_down, nullptr, p.F, p.H, 1, p.rows[3], p.kc[3], p.nkc[3]};
        }
    };
    // Attention item i -> (kv head, split); key tiles [t0, t1) of the split.
    auto fd_item = [&](int i, int& hkv, int& t0, int& t1) {
        hkv = i / p.splits;
        const int split = i % p.splits;
        t0 = split * p.chunk_tiles;
        t1 = t0 + p.chunk_tiles;
        if (t1 > ktiles_total) t1 = ktiles_total;
    };
    // Tiles (GEMV row tiles and attention key tiles) go to the groups in
    // turn; `rot` counts this CTA's tiles across all ops, identically in the
    // producer and in every consumer warp.

    if (warp >= kCW) {
        // ================= producers: warp kCW + g fills group g's ring =================
        if (lane == 0) {
            const int g = warp - kCW;
            int fill = 0;
            StageCursor ic, pc;
            ic.init(&p, blockIdx.x, grid, len);
            pc = ic;
            int64_t issued = 0, prefetched = 0;
            const int64_t ahead = p.l2_ahead / kGroups;
            while (ic.valid && !s_abort) {
                if (ic.rot % kGroups != g) {
                    ic.advance();
                    continue;
                }
                // keep the L2 prefetch cursor up to `ahead` bytes ahead
                while (pc.valid && prefetched - issued < ahead) {
                    if (pc.rot % kGroups == g) {
                        uint32_t nb;
                        int gg;
                        bool dep;
                        const char* a = pc.src(nb, gg, dep);
                        bulk_prefetch_l2(a, nb);
                        prefetched += nb;
                    }
                    pc.advance();
                }
                uint32_t bytes;
                int gg;
                bool holds_new_row;  // patched by the consumers (see op1)
                const char* a = ic.src(bytes, gg, holds_new_row);
                const int b = g * kSlots + fill % kSlots;
                if (!mbar_wait(smem_u32(&empty[b]), (uint32_t(fill / kSlots) & 1u) ^ 1u, &g_step_error_word)) {
                    s_abort = 1;
                    break;
                }
                ++fill;
                const uint32_t bar = smem_u32(&full[b]);
                mbar_expect_tx(bar, bytes);
                bulk_g2s(smem_u32(ring + b * kStageMax), a, bytes, bar);
                issued += bytes;
                ic.advance();
            }
        }
    } else {
        // ================= consumers (4 groups x 4 warps) =================
        const int ctid = tid;  // 0..511
        const int grp = warp / kGW, gw = warp % kGW;
        int cf = 0;   // fills of this group's ring consumed
        int rot = 0;
        // Wait for the next fill of this group's ring; returns its barrier index.
        auto next_fill = [&]() -> int {
            const int b = grp * kSlots + cf % kSlots;
            if (!s_abort && !mbar_wait(smem_u32(&full[b]), uint32_t(cf / kSlots) & 1u, &g_step_error_word)) s_abort = 1;
            ++cf;
            return b;
        };
        void* cur = p.x;
        void* nxt = p.x2;
        for (int l = 0; l < p.L; ++l) {
            const DecodeLayer& L = p.layers[l];
            for (int k = 0; k < kOps; ++k) {
                if (k == 2) continue;  // the split combine runs inside op1
                // Norm weights depend on nothing: load them before waiting.
                const bool norm = (k == 0 || k == 4);
                const float* nw = k == 0 ? L.attn_norm : L.mlp_norm;
                float4 nwv[kNormChunks][2];
                if (norm && nw) {
#pragma unroll
                    for (int j = 0; j < kNormChunks; ++j) {
                        const int c = ctid + j * kCW * 32;
                        if (c < p.H / 8) {
                            nwv[j][0] = __ldg(reinterpret_cast<const float4*>(nw) + 2 * c);
                            nwv[j][1] = __ldg(reinterpret_cast<const float4*>(nw) + 2 * c + 1);
                        }
                    }
                }
                // ---- dependency: the op that produced this op's input ----
                named_sync(1, kCW * 32);
                if (ctid == 0 && !s_abort) {
                    int dep = -1;
                    if (k == 0 && l > 0) dep = (l - 1) * kOps + 5;
                    if (k == 1) dep = l * kOps + 0;  // q; the K/V tiles already stream meanwhile
                    if (k == 3) dep = l * kOps + 1;
                    if (k == 4 || k == 5) dep = l * kOps + k - 1;
                    if (dep >= 0 && !wait_counter(&p.counters[dep], unsigned(grid))) s_abort = 1;
                }
                named_sync(1, kCW * 32);
                if (ctid == 0) TRACE(l, k, 0);

                if (k == 1) {
                    // ---- split-KV attention: warp gw of a group takes keys 8gw..8gw+7 of a tile ----
                    const int nitems = p.Nkv * p.splits;
                    for (int i = blockIdx.x; i < nitems; i += grid) {
                        int hkv, t0, t1;
                        fd_item(i, hkv, t0, t1);
                        const int split = i % p.splits;
                        const int hq0 = hkv * G;
                        float q[G][kE], o[G][kE], m[G], lsum[G];
                        const float qs = p.scale * kLog2e;
#pragma unroll
                        for (int g = 0; g < G; ++g) {
                            m[g] = -INFINITY;
                            lsum[g] = 0.f;
#pragma unroll
                            for (int e = 0; e < kE; ++e) o[g][e] = 0.f;
                        }
                        // the step's RoPE table row (Gemma4TextInference.swift:346-351)
                        const int64_t trow = (p.rope_rows == 1 ? 0 : int64_t(pos)) * (kHD / 2);
                        const float* rcos = p.has_rope && L.rope_cos ? L.rope_cos + trow : nullptr;
                        const float* rsin = p.has_rope && L.rope_sin ? L.rope_sin + trow : nullptr;
                        const bool qk_xform = QK && (p.qk_norm || rcos);
#pragma unroll
                        for (int g = 0; g < G; ++g) {
                            uint4 qv = ldcg16(static_cast<const char*>(p.q) + (int64_t(hq0 + g) * kHD + lane * kE) * 2);
                            float f[8];
                            unpack8<T>(qv, f);
                            // q is stored as the QKV projection wrote it; each item
                            // normalises and rotates its own copy
                            if (qk_xform) head_norm_rope<T>(f, lane, p.qk_norm, L.q_norm, p.eps, p.add_one, rcos, rsin);
#pragma unroll
                            for (int e = 0; e < kE; ++e) q[g][e] = f[e] * qs;
                        }
                        const int ntl = t1 > t0 ? t1 - t0 : 0;
                        for (int tt = 0; tt < ntl; ++tt, ++rot) {
                            if (rot % kGroups != grp) continue;
                            const int sk = next_fill();
                            const int sv = next_fill();
                            const int64_t j0 = int64_t(t0 + tt) * kTileKeys;
                            const int nk = int(len - j0 < kTileKeys ? len - j0 : kTileKeys);
                            const int kw0 = gw * 8;
                            char* ktile = reinterpret_cast<char*>(ring + sk * kStageMax);
                            char* vtile = reinterpret_cast<char*>(ring + sv * kStageMax);
                            if (t0 + tt == ktiles_total - 1) {
                                // The tile was copied before op0 wrote the new key/value
                                // row (copies never wait); patch that row from global
                                // memory now that op0 is complete.
                                if (gw == 0 && !s_abort) {
                                    const int64_t row = (int64_t(hkv) * p.Smax + pos) * kHD * 2 + lane * 16;
                                    uint4 kv = ldcg16(static_cast<const char*>(L.k_cache) + row);
                                    uint4 vv = ldcg16(static_cast<const char*>(L.v_cache) + row);
                                    if (qk_xform) {
                                        // the new key / value heads get their norms and RoPE
                                        // here, the one item that holds them, which also
                                        // writes them back to the caches for later steps
                                        float f[8];
                                        unpack8<T>(kv, f);
                                        head_norm_rope<T>(f, lane, p.qk_norm, L.k_norm, p.eps, p.add_one, rcos, rsin);
                                        kv = pack8<T>(f);
                                        *reinterpret_cast<uint4*>(static_cast<char*>(L.k_cache) + row) = kv;
                                        if (p.qk_norm && p.norm_v) {
                                            unpack8<T>(vv, f);
                                            head_norm_rope<T>(f, lane, true, nullptr, p.eps, false, nullptr, nullptr);
                                            vv = pack8<T>(f);
                                            *reinterpret_cast<uint4*>(static_cast<char*>(L.v_cache) + row) = vv;
                                        }
                                    }
                                    *reinterpret_cast<uint4*>(ktile + (pos - j0) * kHD * 2 + lane * 16) = kv;
                                    *reinterpret_cast<uint4*>(vtile + (pos - j0) * kHD * 2 + lane * 16) = vv;
                                    // generic writes before the slot's next bulk copy
                                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                                }
                                named_sync(2 + grp, kGW * 32);
                            }
                            if (!s_abort && kw0 < nk) {
                                float vals[8 * G];
#pragma unroll
                                for (int i8 = 0; i8 < 8; ++i8) {
                                    float kf[kE];
                                    if (kw0 + i8 < nk) {
                                        unpack8<T>(*reinterpret_cast<const uint4*>(ktile + (kw0 + i8) * kHD * 2 + lane * 16), kf);
                                    } else {
#pragma unroll
                                        for (int e = 0; e < kE; ++e) kf[e] = 0.f;
                                    }
#pragma unroll
                                    for (int g = 0; g < G; ++g) {
                                        float acc = 0.f;
#pragma unroll
                                        for (int e = 0; e < kE; ++e) acc = fmaf(q[g][e], kf[e], acc);
                                        vals[i8 * G + g] = acc;
                                    }
                                }
                                // Transposed reduction: after three exchange rounds lane
                                // quad (lane >> 2) holds partial scores of key (lane >> 2) & 7.
                                {
                                    const bool hi = lane & 16;
#pragma unroll
                                    for (int i2 = 0; i2 < 4 * G; ++i2) {
                                        float lo_v = vals[i2], hi_v = vals[i2 + 4 * G];
                                        float send = hi ? lo_v : hi_v, keep = hi ? hi_v : lo_v;
                                        vals[i2] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
                                    }
                                }
                                {
                                    const bool hi = lane & 8;
#pragma unroll
                                    for (int i2 = 0; i2 < 2 * G; ++i2) {
                                        float lo_v = vals[i2], hi_v = vals[i2 + 2 * G];
                                        float send = hi ? lo_v : hi_v, keep = hi ? hi_v : lo_v;
                                        vals[i2] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
                                    }
                                }
                                {
                                    const bool hi = lane & 4;
#pragma unroll
                                    for (int i2 = 0; i2 < G; ++i2) {
                                        float lo_v = vals[i2], hi_v = vals[i2 + G];
                                        float send = hi ? lo_v : hi_v, keep = hi ? hi_v : lo_v;
                                        vals[i2] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
                                    }
                                }
                                const int my_key = (lane >> 2) & 7;
                                const bool valid = kw0 + my_key < nk;
                                float pr[G];
#pragma unroll
                                for (int g = 0; g < G; ++g) {
                                    float sv2 = vals[g];
                                    sv2 += __shfl_xor_sync(0xffffffffu, sv2, 2);
                                    sv2 += __shfl_xor_sync(0xffffffffu, sv2, 1);
                                    float mx = valid ? sv2 : -INFINITY;
                                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
                                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
                                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
                                    const float mnew = fmaxf(m[g], mx);
                                    const float so = exp2f(m[g] - mnew);
                                    const float pv = valid ? exp2f(sv2 - mnew) : 0.f;
                                    float ps = pv;
                                    ps += __shfl_xor_sync(0xffffffffu, ps, 4);
                                    ps += __shfl_xor_sync(0xffffffffu, ps, 8);
                                    ps += __shfl_xor_sync(0xffffffffu, ps, 16);
                                    lsum[g] = lsum[g] * so + ps;
                                    m[g] = mnew;
#pragma unroll
                                    for (int e = 0; e < kE; ++e) o[g][e] *= so;
                                    pr[g] = pv;
                                }
#pragma unroll
                                for (int i8 = 0; i8 < 8; ++i8) {
                                    float pi[G];
#pragma unroll
                                    for (int g = 0; g < G; ++g) pi[g] = __shfl_sync(0xffffffffu, pr[g], i8 * 4);
                                    if (kw0 + i8 < nk) {
                                        float vf[kE];
                                        unpack8<T>(*reinterpret_cast<const uint4*>(vtile + (kw0 + i8) * kHD * 2 + lane * 16), vf);
#pragma unroll
                                        for (int g = 0; g < G; ++g)
#pragma unroll
                                            for (int e = 0; e < kE; ++e) o[g][e] = fmaf(pi[g], vf[e], o[g][e]);
                                    }
                                }
                            }
                            __syncwarp();
                            if (lane == 0) {
                                mbar_arrive(smem_u32(&empty[sk]));
                                mbar_arrive(smem_u32(&empty[sv]));
                            }
                        }
                        // merge the 16 warp states of the G heads
                        if (ctid == 0) TRACE(l, 2, 2);
                        float* mm = merge;
                        float* ll = mm + kCW * G;
                        float* oo = ll + kCW * G;
                        if (lane == 0)
#pragma unroll
                            for (int g = 0; g < G; ++g) {
                                mm[warp * G + g] = m[g];
                                ll[warp * G + g] = lsum[g];
                            }
#pragma unroll
                        for (int g = 0; g < G; ++g)
#pragma unroll
                            for (int e = 0; e < kE; ++e) oo[(warp * G + g) * kHD + lane * kE + e] = o[g][e];
                        named_sync(1, kCW * 32);
                        for (int idx = ctid; idx < G * kHD; idx += kCW * 32) {
                            const int g = idx / kHD, d = idx % kHD;
                            float M = -INFINITY;
                            for (int w = 0; w < kCW; ++w) M = fmaxf(M, mm[w * G + g]);
                            float Ls = 0.f, O = 0.f;
                            if (M != -INFINITY)
                                for (int w = 0; w < kCW; ++w) {
                                    const float mw = mm[w * G + g];
                                    const float f = mw == -INFINITY ? 0.f : exp2f(mw - M);
                                    Ls += f * ll[w * G + g];
                                    O += f * oo[(w * G + g) * kHD + d];
                                }
                            const int64_t slot = int64_t(hq0 + g) * p.splits + split;
                            p.po[slot * kHD + d] = O;
                            if (d == 0) {
                                p.pm[slot] = M;
                                p.pl[slot] = Ls;
                            }
                        }
                        // Every split of this KV head arrives, waits for the others,
                        // then combines its own slice of the G heads' outputs (one
                        // load per thread). Items never exceed the grid, so all
                        // splits of a head run concurrently.
                        named_sync(1, kCW * 32);
                        if (ctid == 0 && !s_abort) {
                            __threadfence();
                            atomicAdd(&head_cnt[l * p.Nkv + hkv], 1u);
                            if (!wait_counter(&head_cnt[l * p.Nkv + hkv], unsigned(p.splits))) s_abort = 1;
                        }
                        named_sync(1, kCW * 32);
                        {
                            if (ctid == 0) TRACE(l, 2, 0);
                            const int ns = p.splits;
                            const int nout = G * kHD;
                            const int slice = (nout + ns - 1) / ns;
                            const int o0 = split * slice;
                            const int o1 = o0 + slice < nout ? o0 + slice : nout;
                            float* sm_m = merge;              // [G][ns]
                            float* sm_l = sm_m + G * ns;      // [G][ns]
                            float* sm_v = sm_l + G * ns;      // [slice][ns]
                            for (int i2 = ctid; i2 < G * ns; i2 += kCW * 32) {
                                sm_m[i2] = __ldcg(p.pm + int64_t(hq0) * ns + i2);
                                sm_l[i2] = __ldcg(p.pl + int64_t(hq0) * ns + i2);
                            }
                            for (int i2 = ctid; i2 < (o1 - o0) * ns; i2 += kCW * 32) {
                                const int o = o0 + i2 / ns, s2 = i2 % ns;
                                const int g = o / kHD, d = o % kHD;
                                sm_v[i2] = __ldcg(p.po + (int64_t(hq0 + g) * ns + s2) * kHD + d);
                            }
                            named_sync(1, kCW * 32);
                            if (ctid < o1 - o0 && !s_abort) {
                                const int o = o0 + ctid;
                                const int g = o / kHD, d = o % kHD;
                                const float* mg = sm_m + g * ns;
                                const float* lg = sm_l + g * ns;
                                const float* vg = sm_v + ctid * ns;
                                float M = -INFINITY;
                                for (int s2 = 0; s2 < ns; ++s2) M = fmaxf(M, mg[s2]);
                                float Ls = 0.f, acc = 0.f;
                                for (int s2 = 0; s2 < ns; ++s2) {
                                    const float ms = mg[s2];
                                    const float f = (M == -INFINITY || ms == -INFINITY) ? 0.f : exp2f(ms - M);
                                    Ls += f * lg[s2];
                                    acc = fmaf(f, vg[s2], acc);
                                }
                                const float inv = Ls > 0.f ? 1.0f / Ls : 0.f;
                                Elem<T>::store(p.attn, int64_t(hq0 + g) * kHD + d, acc * inv);
                            }
                            if (ctid == 0) TRACE(l, 2, 1);
                        }
                        named_sync(1, kCW * 32);
                    }
                } else {
                    // ---- GEMV op: stage the activation row, then stream row tiles ----
                    const GemvOp g = gemv_op(l, k);
                    const void* xin = k == 0 ? cur : k == 3 ? p.attn : k == 4 ? p.h : p.act;
                    const int nxc = g.K / 8;  // 8-element chunks of the row
                    // fp32 planes: elements 0-3 of each chunk, then elements 4-7
                    // The row is read with one 16-byte load per 8 elements, all
                    // issued before any is used (one memory round trip).
                    uint4 xr[kChunkRegs];
#pragma unroll
                    for (int j = 0; j < kChunkRegs; ++j) {
                        const int c = ctid + j * kCW * 32;
                        if (c < nxc) xr[j] = ldcg16(static_cast<const char*>(xin) + size_t(c) * 16);
                    }
                    float scale = 1.f;
                    if (norm) {
                        float ss = 0.f;
#pragma unroll
                        for (int j = 0; j < kChunkRegs; ++j) {
                            const int c = ctid + j * kCW * 32;
                            if (c < nxc) {
                                float f[8];
                                unpack8<T>(xr[j], f);
#pragma unroll
                                for (int e = 0; e < 8; ++e) ss += f[e] * f[e];
                            }
                        }
                        ss = warp_sum(ss);
                        if (lane == 0) red[warp] = ss;
                        named_sync(1, kCW * 32);
                        float v = lane < kCW ? red[lane] : 0.f;
                        v = warp_sum(v);
                        scale = rsqrtf(v / float(g.K) + p.eps);
                    }
                    float4* xw = reinterpret_cast<float4*>(xsf);
#pragma unroll
                    for (int j = 0; j < kChunkRegs; ++j) {
                        const int c = ctid + j * kCW * 32;
                        if (c < nxc) {
                            float f[8];
                            unpack8<T>(xr[j], f);
                            if (norm) {
                                const int jn = j < kNormChunks ? j : 0;
                                const float w[8] = {nwv[jn][0].x, nwv[jn][0].y, nwv[jn][0].z, nwv[jn][0].w,
                                                    nwv[jn][1].x, nwv[jn][1].y, nwv[jn][1].z, nwv[jn][1].w};
#pragma unroll
                                for (int e = 0; e < 8; ++e) {
                                    float v = f[e] * scale;
                                    if (nw) v *= p.add_one ? 1.0f + w[e] : w[e];
                                    f[e] = Elem<T>::round(v);
                                }
                            }
                            xw[c] = make_float4(f[0], f[1], f[2], f[3]);
                            xw[nxc + c] = make_float4(f[4], f[5], f[6], f[7]);
                        }
                    }
                    named_sync(1, kCW * 32);
                    const float4* x4 = reinterpret_cast<const float4*>(xsf);
                    const int tr = g.rows, segs = kGW / tr;  // warps per row
                    const int r = gw % tr, seg = gw / tr;
                    const int ntiles = (g.N + tr - 1) / tr;
                    int tcount = 0;
                    for (int tile = blockIdx.x; tile < ntiles; tile += grid, ++rot) {
                        if (rot % kGroups != grp) continue;
                        const int n = tile * tr + r;
                        const bool valid = n < g.N;
                        float acc[2] = {0.f, 0.f};
                        for (int kci = 0; kci < g.nkc; ++kci) {
                            const int k0 = kci * g.kc;
                            const int kcols = g.K - k0 < g.kc ? g.K - k0 : g.kc;
                            const int nc = kcols / 8, c0 = k0 / 8;
                            const int cb = seg * nc / segs, ce = (seg + 1) * nc / segs;
                            for (int m = 0; m < g.R; ++m) {
                                const int b = next_fill();
                                if (valid && !s_abort) {
                                    const unsigned char* row = ring + b * kStageMax + size_t(r) * kcols * 2;
                                    float a = acc[m];
#pragma unroll 4
                                    for (int c = cb + lane; c < ce; c += 32) {
                                        const float4 lo = x4[c0 + c], hi = x4[nxc + c0 + c];
                                        float wf[8];
                                        unpack8<T>(*reinterpret_cast<const uint4*>(row + size_t(c - 0) * 16), wf);
                                        a = fmaf(lo.x, wf[0], a);
                                        a = fmaf(lo.y, wf[1], a);
                                        a = fmaf(lo.z, wf[2], a);
                                        a = fmaf(lo.w, wf[3], a);
                                        a = fmaf(hi.x, wf[4], a);
                                        a = fmaf(hi.y, wf[5], a);
                                        a = fmaf(hi.z, wf[6], a);
                                        a = fmaf(hi.w, wf[7], a);
                                    }
                                    acc[m] = a;
                                }
                                __syncwarp();
                                if (lane == 0) mbar_arrive(smem_u32(&empty[b]));
                            }
                        }
                        float y0 = warp_sum(acc[0]);
                        float y1 = warp_sum(acc[1]);
                        if (segs > 1) {
                            // the row's segments meet in shared memory (double-buffered by tile)
                            float* gp = gpart[tcount & 1][grp];
                            if (lane == 0) {
                                gp[gw * 2] = y0;
                                gp[gw * 2 + 1] = y1;
                            }
                            named_sync(2 + grp, kGW * 32);
                            y0 = y1 = 0.f;
                            for (int sg = 0; sg < segs; ++sg) {
                                y0 += gp[(sg * tr + r) * 2];
                                y1 += gp[(sg * tr + r) * 2 + 1];
                            }
                        }
                        ++tcount;
                        if (lane == 0 && seg == 0 && valid && !s_abort) {
                            if (k == 0) {
                                const int QN = p.Nq * kHD, KN = p.Nkv * kHD;
                                if (n < QN) {
                                    Elem<T>::store(p.q, n, y0);
                                } else {
                                    int rr = n - QN;
                                    void* cache = L.k_cache;
                                    if (rr >= KN) {
                                        rr -= KN;
                                        cache = L.v_cache;
                                    }
                                    Elem<T>::store(cache, (int64_t(rr / kHD) * p.Smax + pos) * kHD + rr % kHD, y0);
                                }
                            } else if (k == 3) {
                                const float y = Elem<T>::round(y0);
                                Elem<T>::store(p.h, n, y + widen16<T>(__ldcg(static_cast<const unsigned short*>(cur) + n)));
                            } else if (k == 4) {
                                const float gt = Elem<T>::round(y0), ut = Elem<T>::round(y1);
                                const float av = Elem<T>::round(p.activation == 0 ? gelu_tanh(gt) : silu(gt));
                                Elem<T>::store(p.act, n, av * ut);
                            } else {
                                const float y = Elem<T>::round(y0);
                                Elem<T>::store(nxt, n, y + widen16<T>(__ldcg(static_cast<const unsigned short*>(p.h) + n)));
                            }
                        }
                    }
                }
                // ---- publish: this CTA is done with op (l, k) ----
                named_sync(1, kCW * 32);
                if (ctid == 0) {
                    __threadfence();  // cumulative over the CTA's writes ordered by the barrier
                    atomicAdd(&p.counters[l * kOps + k], 1u);
                    TRACE(l, k, 1);
                }
            }
            void* t = cur;
            cur = nxt;
            nxt = t;
        }
    }
    __syncthreads();
    // The last CTA out resets the op and head counters for the next launch.
    if (tid == 0 && !s_abort) {
        __threadfence();
        const unsigned int done = atomicAdd(&p.counters[p.L * kOps], 1u);
        if (done == unsigned(grid) - 1) {
            for (int i = 0; i <= p.L * kOps + p.L * p.Nkv; ++i) atomicExch(&p.counters[i], 0u);
            __threadfence();
        }
    }
}

size_t decode_step_smem(const DecodeStep& p) {
    const size_t xs = size_t(p.xs_bytes);
    const int G = p.Nq / p.Nkv;
    size_t mg = size_t(kCW) * G * (kHD + 2) * 4;  // warp states of the merge
    const size_t cmb = (size_t(2) * G * p.splits + size_t((G * kHD + p.splits - 1) / p.splits + 1) * p.splits) * 4;
    if (cmb > mg) mg = cmb;
    return size_t(kRing) * kStageMax + (xs > mg ? xs : mg);
}

bool decode_step_plan(DecodeStep& p, int sm_count) {
    if (p.Hd != kHD || p.Nq % p.Nkv != 0) return false;
    const int gq = p.Nq / p.Nkv;
    if (gq != 1 && gq != 2 && gq != 4) return false;
    if (p.H % 8 || p.F % 8 || (p.Nq * kHD) % 8) return false;
    const int Ks[4] = {p.H, p.Nq * kHD, p.H, p.F};
    for (int i = 0; i < 4; ++i) {
        // A stage is one contiguous block of one matrix: tr whole rows
        // (tr = 4, 2 or 1, as many as fit), else one column chunk of a row.
        // The bulk-copy engine streams at full rate only with stages of
        // about 16 KB or more in one copy.
        int tr = kGW;
        while (tr > 1 && int64_t(tr) * Ks[i] * 2 > kStageMax) tr /= 2;
        int kc = Ks[i], nkc = 1;
        if (int64_t(Ks[i]) * 2 > kStageMax) {
            nkc = (Ks[i] * 2 + kStageMax - 1) / kStageMax;
            kc = (Ks[i] + nkc - 1) / nkc;
            kc = (kc + 7) / 8 * 8;
            nkc = (Ks[i] + kc - 1) / kc;
        }
                p.rows[i] = tr;
        p.kc[i] = kc;
        p.nkc[i] = nkc;
    }
    int kmax = p.H > p.F ? p.H : p.F;
    if (p.Nq * kHD > kmax) kmax = p.Nq * kHD;
    if (kmax > kChunkRegs * 8 * kCW * 32 || p.H > kNormChunks * 8 * kCW * 32) return false;
    // L2 prefetch distance beyond the ring, per CTA (148 x 128 KB = 19 MB of
    // the 126 MB L2; measured at config 2: 0 -> 1.424 ms, 128 KB -> 1.402,
    // 256 KB -> 1.418, 512 KB -> 1.78). POPCORN_STEP_L2_AHEAD overrides it
    // (bytes; 0 = off).
    p.l2_ahead = 128 * 1024;
    if (const char* e = getenv("POPCORN_STEP_L2_AHEAD")) p.l2_ahead = atoll(e);
    p.xs_bytes = (kmax * 4 + 127) / 128 * 128;
    // attention split: about one item per SM and never more items than CTAs
    // (the splits of a head wait for each other)
    if (p.Nkv > sm_count) return false;
    const int max_tiles = (p.Smax + kTileKeys - 1) / kTileKeys;
    int splits = sm_count / p.Nkv;
    if (splits > max_tiles) splits = max_tiles;
    if (splits < 1) splits = 1;
    p.chunk_tiles = (max_tiles + splits - 1) / splits;
    p.splits = (max_tiles + p.chunk_tiles - 1) / p.chunk_tiles;
    return decode_step_smem(p) + 2048 <= 227 * 1024;
}

size_t decode_step_workspace_bytes(const DecodeStep& p) {
    size_t o = size_t(p.Nq) * p.splits * kHD * 4;
    size_t ml = size_t(p.Nq) * p.splits * 4;
    return o + 2 * ml + size_t(p.L * kOps + 1 + p.L * p.Nkv) * 4 + 1024;
}

template <class T, bool QK>
static void (*pick_step(int gq))(DecodeStep) {
    return gq == 1 ? decode_step_kernel<T, 1, QK> : gq == 2 ? decode_step_kernel<T, 2, QK> : decode_step_kernel<T, 4, QK>;
}

cudaError_t decode_step(const DecodeStep& p, cudaStream_t s) {
    const size_t smem = decode_step_smem(p);
    void (*kern)(DecodeStep) = nullptr;
    const int gq = p.Nq / p.Nkv;
    const bool qk = p.qk_norm || p.has_rope;
    if (p.dtype == PC_BF16)
        kern = qk ? pick_step<TBF16, true>(gq) : pick_step<TBF16, false>(gq);
    else
        kern = qk ? pick_step<TF16, true>(gq) : pick_step<TF16, false>(gq);
    cudaError_t e = allow_smem(kern, smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(p.grid));
    cfg.blockDim = dim3(kStepThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs co-resident: they wait on each other
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

uint32_t read_and_clear_step_errors() {
    unsigned int v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_step_error_word, sizeof(v)) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    if (v) cudaMemcpyToSymbol(g_step_error_word, &zero, sizeof(zero));
    return v;
}

namespace {
RegisterFunctions reg_step({
    {"decode_step_f16", reinterpret_cast<const void*>(decode_step_kernel<TF16, 2, false>)},
    {"decode_step_bf16", reinterpret_cast<const void*>(decode_step_kernel<TBF16, 2, false>)},
    {"decode_step_qk_f16", reinterpret_cast<const void*>(decode_step_kernel<TF16, 2, true>)},
    {"decode_step_qk_bf16", reinterpret_cast<const void*>(decode_step_kernel<TBF16, 2, true>)},
});
}  // namespace

}  // namespace launch
}  // namespace popcorn

#ifdef PC_STEP_TRACE
extern "C" __attribute__((visibility("default"))) int pc_debug_step_trace(unsigned long long* host, size_t n) {
    return int(cudaMemcpyFromSymbol(host, popcorn::g_step_trace, n * 8));
}
#endif
