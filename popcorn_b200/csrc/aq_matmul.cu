// aq_matmul.cu — Matmul against a block-affine 4-bit quantized RHS
// (Matmul.swift:99-131, 279-351; AffineQuantizedMatmul.metal) and the
// embedding gathers (EmbeddingGather.metal, AffineQuantizedEmbeddingGather
// .metal).
//
// Format (AffineQuantizationFormat.swift:22-29, AffineQuantizedTensor.swift):
// W [N, K] as u32 words [N, K/8], value k of a row in bits 4(k%8)..4(k%8)+3
// of word k/8; one scale and (optional) bias per 64 consecutive k of a row,
// [N, K/64]; w = q * scale + bias. c[m, n] = sum_k x[m, k] w[n, k], fp32
// accumulation, one rounding at the store.
//
// B200 design. At decode (m <= 8) the op streams 0.5625 bytes per weight:
// 7.3 TB/s means ~52 weights per SM clock, about 2.5 instructions per weight
// of budget — too few for nibble extraction + int->float + FMA per weight.
// So the dot products run on the tensor cores (mma.sync m16n8k16, fp32
// accumulate): a warp computes 16 output rows x 8 tokens. The order of k
// inside one MMA is free, so a thread takes two whole words of a row per
// 64-value group and each word turns into four bf16x2 A-operands with one
// shift + one lop3 + one packed subtract per PAIR ((w >> 4j) & 0x000F000F |
// 0x43004300 is the bf16 pair (128 + q_j, 128 + q_j+4), exact); the matching
// x values are paired the same way with byte permutes (x is shared by all 16
// rows). Per group the fresh accumulator D = sum(x q) becomes
// acc += scale * D + bias * sum(x), the algebraic form of aq_qmv_fast_typed
// (AffineQuantizedMatmul.metal:71-160). Products of bf16 (or f16) values are
// exact in the tensor core; f32 activations are split into bf16 hi + lo
// parts (two MMAs, ~16 significant bits, error ~1e-5 relative).
//
// Work split: a CTA (8 warps) owns 16 rows x up to 8 tokens; its warps take
// contiguous runs of the K groups; weights come straight from global memory
// into registers (8-byte loads, four groups per batch in flight), partials
// meet in shared memory in warp order. When rows are few (down / o_proj at
// decode), the K groups are also split over CTAs: each writes an fp32
// partial to caller scratch and the last CTA of a tile sums them in order
// (deterministic).
#include <type_traits>

#include "async.cuh"
#include "common.cuh"
#include "dtype.cuh"
#include "tcgen05.cuh"
#include "launch.hpp"
#include "popcorn.hpp"

namespace popcorn {
namespace launch {

__device__ unsigned int g_aq_error_word;

namespace {

constexpr int kAqWarps = 8;
constexpr int kAqThreads = kAqWarps * 32;
constexpr int kAqBatch = 8;  // groups whose weight loads are in flight together
constexpr int kAqSmemMax = 64 * 1024;  // staged x per chunk

__device__ __forceinline__ uint2 ldg_nc_u2(const void* p) {
    uint2 r;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}

// Four 16-bit A pairs (q_j, q_j+4), j = 0..3, of one packed word, in the
// MMA's element type, offset by a constant: bf16 0x4300 | q = 128 + q, f16
// 0x6400 | q = 1024 + q (both exact). The offset times sum(x) is removed in
// fp32 after the group's MMAs.
template <bool F16>
__device__ __forceinline__ void word_pairs(uint32_t w, uint32_t* a) {
    constexpr uint32_t magic = F16 ? 0x64006400u : 0x43004300u;
#pragma unroll
    for (int j = 0; j < 4; ++j)
        asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(a[j]) : "r"(w >> (4 * j)), "r"(0x000F000Fu), "r"(magic));
}

template <bool F16>
__device__ __forceinline__ void mma16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
    if constexpr (F16)
        asm(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    else
        asm(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t s) { return __byte_perm(a, b, s); }

// x values 16t .. 16t+15 of one group for the thread's token, as the eight
// B pairs of the group's four k-steps: step s uses (b[2s], b[2s+1]) with
// k-pairs (0,4)(1,5) | (2,6)(3,7) | (8,12)(9,13) | (10,14)(11,15) —
// the positions the A pairs of word_pairs take. q[i] holds the 16-bit pair
// (x_2i, x_2i+1).
__device__ __forceinline__ void x_pairs(const uint32_t* q, uint32_t* b) {
    b[0] = prmt(q[0], q[2], 0x5410);
    b[1] = prmt(q[0], q[2], 0x7632);
    b[2] = prmt(q[1], q[3], 0x5410);
    b[3] = prmt(q[1], q[3], 0x7632);
    b[4] = prmt(q[4], q[6], 0x5410);
    b[5] = prmt(q[4], q[6], 0x7632);
    b[6] = prmt(q[5], q[7], 0x5410);
    b[7] = prmt(q[5], q[7], 0x7632);
}

__device__ __forceinline__ uint32_t bf16_bits(float v) { return float_to_bf16_bits(v) & 0xFFFFu; }

// x of tokens [m0, m0 + mt) and groups [c0, c0 + cg) into shared memory, as
// the B pairs of x_pairs: per (group j, token n, part, plane, thread t) one
// 16-byte vector (plane 0: b0-b3, plane 1: b4-b7; part 1: the lo half of an
// f32 x), and the groups' sums sum(x) (fp32) per (j, n). One unit is a
// quarter group (16 values, thread slot t) so that four threads share a
// group and all its loads are in flight at once; the quarters' sums meet by
// shuffles within the four lanes (the same order on each lane). All
// `nthreads` threads (a multiple of 4) from `tid` take part; the caller
// synchronises.
//
// nscale (optional, fused RMSNorm): token n's value k is staged as
// round((x * nscale[n]) * nw[k]) in x's type, nw[k] the norm weight (plus
// one when the form asks for it, no weight: 1) as RMSNorm applies it — what
// RMSNorm would have stored (RMSNorm.metal:7-42) — and the group sums are of
// those values.
template <class XT>
__device__ __forceinline__ float norm_value(float v, float scale, const float* nw, int64_t k) {
    v *= scale;
    if (nw) v *= nw[k];
    return Elem<XT>::round(v);
}

template <class XT>
__device__ __forceinline__ void stage_x(const AqMatmul& p, int64_t m0, int mt, int64_t c0, int cg, uint4* xs,
                                        float* sxs, int tid, int nthreads, const float* nscale = nullptr,
                                        const float* nw = nullptr) {
    constexpr bool XF32 = std::is_same<XT, TF32>::value;
    constexpr int NP = XF32 ? 2 : 1;
    auto at = [&](int j, int n, int part, int plane, int tt) -> uint4& {
        return xs[((((size_t(j) * mt + n) * NP + part) * 2 + plane) * 4) + tt];
    };
    // the unit count is a multiple of 4 and so is nthreads: a quad of lanes
    // runs the same iterations
    const unsigned quad = 0xFu << (threadIdx.x & 28);
    for (int u = tid; u < 4 * cg * mt; u += nthreads) {
        const int tt = u & 3, jn = u >> 2;
        const int j = jn / mt, n = jn % mt;
        const int64_t k0 = (c0 + j) * 64 + tt * 16;
        const char* src = static_cast<const char*>(p.x) + ((m0 + n) * p.K + k0) * Elem<XT>::bytes;
        float sx = 0.f;
        uint32_t b[8];
        if constexpr (!XF32) {
            const uint4 l0 = __ldg(reinterpret_cast<const uint4*>(src));
            const uint4 l1 = __ldg(reinterpret_cast<const uint4*>(src) + 1);
            uint32_t q[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                float2 f = unpack2<XT>(q[i]);
                if (nscale) {
                    f.x = norm_value<XT>(f.x, nscale[n], nw, k0 + 2 * i);
                    f.y = norm_value<XT>(f.y, nscale[n], nw, k0 + 2 * i + 1);
                    q[i] = pack2<XT>(f.x, f.y);
                }
                sx += f.x;
                sx += f.y;
            }
            x_pairs(q, b);
            at(j, n, 0, 0, tt) = make_uint4(b[0], b[1], b[2], b[3]);
            at(j, n, 0, 1, tt) = make_uint4(b[4], b[5], b[6], b[7]);
        } else {
            uint32_t qh[8], ql[8];
            float4 f4[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) f4[i] = __ldg(reinterpret_cast<const float4*>(src) + i);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float e[4] = {f4[i].x, f4[i].y, f4[i].z, f4[i].w};
                if (nscale)
#pragma unroll
                    for (int h = 0; h < 4; ++h) e[h] = norm_value<XT>(e[h], nscale[n], nw, k0 + 4 * i + h);
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const float e0 = e[2 * h], e1 = e[2 * h + 1];
                    const uint32_t h0 = bf16_bits(e0), h1 = bf16_bits(e1);
                    const uint32_t l0 = bf16_bits(e0 - __uint_as_float(h0 << 16));
                    const uint32_t l1 = bf16_bits(e1 - __uint_as_float(h1 << 16));
                    qh[2 * i + h] = h0 | (h1 << 16);
                    ql[2 * i + h] = l0 | (l1 << 16);
                    // the sum of what the MMAs multiply (hi + lo), so the
                    // offset term cancels exactly
                    sx += __uint_as_float(h0 << 16) + __uint_as_float(l0 << 16);
                    sx += __uint_as_float(h1 << 16) + __uint_as_float(l1 << 16);
                }
            }
            x_pairs(qh, b);
            at(j, n, 0, 0, tt) = make_uint4(b[0], b[1], b[2], b[3]);
            at(j, n, 0, 1, tt) = make_uint4(b[4], b[5], b[6], b[7]);
            x_pairs(ql, b);
            at(j, n, NP - 1, 0, tt) = make_uint4(b[0], b[1], b[2], b[3]);
            at(j, n, NP - 1, 1, tt) = make_uint4(b[4], b[5], b[6], b[7]);
        }
        sx += __shfl_xor_sync(quad, sx, 1);
        sx += __shfl_xor_sync(quad, sx, 2);
        if (tt == 0) sxs[j * mt + n] = sx;
    }
}

// One group of 16 rows x 8 tokens: A from the two packed words of rows g and
// g + 8, B from the staged x; returns D = sum over the group of x (kOff + q).
template <bool F16, int NP>
__device__ __forceinline__ void group_mma(uint32_t wa0, uint32_t wa1, uint32_t wb0, uint32_t wb1, const uint4* xlo,
                                          const uint4* xhi, bool tok, float* d) {
    uint32_t a0[4], a1[4], a2[4], a3[4];
    word_pairs<F16>(wa0, a0);
    word_pairs<F16>(wa1, a2);
    word_pairs<F16>(wb0, a1);
    word_pairs<F16>(wb1, a3);
    // step s: A regs {row g pos 2t.., row g+8 pos 2t.., row g pos 2t+8.., row g+8 pos 2t+8..}
    const uint32_t s0[4] = {a0[0], a1[0], a0[1], a1[1]};
    const uint32_t s1[4] = {a0[2], a1[2], a0[3], a1[3]};
    const uint32_t s2[4] = {a2[0], a3[0], a2[1], a3[1]};
    const uint32_t s3[4] = {a2[2], a3[2], a2[3], a3[3]};
#pragma unroll
    for (int part = 0; part < NP; ++part) {
        uint4 lo = make_uint4(0u, 0u, 0u, 0u), hi = lo;
        if (tok) {
            lo = xlo[part * 8];
            hi = xhi[part * 8];
        }
        mma16816<F16>(d, s0, lo.x, lo.y);
        mma16816<F16>(d, s1, lo.z, lo.w);
        mma16816<F16>(d, s2, hi.x, hi.y);
        mma16816<F16>(d, s3, hi.z, hi.w);
    }
}

template <class XT, class ST, class OT>
__global__ void __launch_bounds__(kAqThreads, 2) aq_matmul_kernel(const AqMatmul p) {
    constexpr bool F16 = std::is_same<XT, TF16>::value;
    constexpr bool XF32 = std::is_same<XT, TF32>::value;
    constexpr int NP = XF32 ? 2 : 1;  // x parts: bf16 hi (+ lo) for f32 x
    constexpr float kOff = F16 ? 1024.f : 128.f;
    extern __shared__ __align__(16) unsigned char aq_smem[];
    __shared__ float red[kAqWarps][32][4];
    __shared__ int s_last;
    pdl_wait();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int64_t G = p.K / 64, wpr = p.K / 8;
    const int64_t row0 = int64_t(blockIdx.x) * 16 + g, row1 = row0 + 8;
    const bool v0 = row0 < p.N, v1 = row1 < p.N;
    const int64_t m0 = int64_t(blockIdx.z) * 8;
    const int mt = int(p.M - m0 < 8 ? p.M - m0 : 8);
    const bool tok = g < mt;  // this thread's B column (token) exists
    // K groups of this CTA slice
    const int ks = gridDim.y, kslice = blockIdx.y;
    const int64_t gs0 = G * kslice / ks, gs1 = G * (kslice + 1) / ks;
    const int chunk = p.chunk_groups;
    // shared x: per chunk group j, token n, part, plane (b0-3 | b4-7), thread t: 16 B
    uint4* xs = reinterpret_cast<uint4*>(aq_smem);
    float* sxs = reinterpret_cast<float*>(aq_smem + size_t(chunk) * mt * NP * 2 * 4 * 16);
    auto xs_at = [&](int j, int n, int part, int plane, int tt) -> uint4& {
        return xs[((((size_t(j) * mt + n) * NP + part) * 2 + plane) * 4) + tt];
    };

    const uint32_t* w0p = p.w + row0 * wpr + 2 * t;
    const uint32_t* w1p = p.w + row1 * wpr + 2 * t;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};

    for (int64_t c0 = gs0; c0 < gs1; c0 += chunk) {
        const int cg = int(gs1 - c0 < chunk ? gs1 - c0 : chunk);
        // ---- stage x of the chunk (permuted into B pairs) and its group sums ----
        if (c0 != gs0) __syncthreads();
        stage_x<XT>(p, m0, mt, c0, cg, xs, sxs, tid, kAqThreads);
        __syncthreads();
        // ---- this warp's run of the chunk's groups ----
        const int ja = cg * warp / kAqWarps, jb = cg * (warp + 1) / kAqWarps;
        for (int jb0 = ja; jb0 < jb; jb0 += kAqBatch) {
            uint2 wa[kAqBatch], wb[kAqBatch];
            float sc[kAqBatch][2], co[kAqBatch][2];
#pragma unroll
            for (int u = 0; u < kAqBatch; ++u) {
                const int64_t gr = c0 + jb0 + u;
                const bool in = jb0 + u < jb;
                wa[u] = in && v0 ? ldg_nc_u2(w0p + gr * 8) : make_uint2(0u, 0u);
                wb[u] = in && v1 ? ldg_nc_u2(w1p + gr * 8) : make_uint2(0u, 0u);
                sc[u][0] = in && v0 ? Elem<ST>::load(p.scales, row0 * G + gr) : 0.f;
                sc[u][1] = in && v1 ? Elem<ST>::load(p.scales, row1 * G + gr) : 0.f;
                co[u][0] = in && v0 && p.biases ? Elem<ST>::load(p.biases, row0 * G + gr) : 0.f;
                co[u][1] = in && v1 && p.biases ? Elem<ST>::load(p.biases, row1 * G + gr) : 0.f;
            }
#pragma unroll
            for (int u = 0; u < kAqBatch; ++u) {
                const int j = jb0 + u;
                if (j >= jb) break;  // warp-uniform
                float d[4] = {0.f, 0.f, 0.f, 0.f};
                group_mma<F16, NP>(wa[u].x, wa[u].y, wb[u].x, wb[u].y, &xs_at(j, g, 0, 0, t), &xs_at(j, g, 0, 1, t),
                                   tok, d);
                // D = sum x (kOff + q): acc += scale * D + (bias - kOff * scale) * sum(x)
                const float sxa = 2 * t < mt ? sxs[j * mt + 2 * t] : 0.f;
                const float sxb = 2 * t + 1 < mt ? sxs[j * mt + 2 * t + 1] : 0.f;
                const float k0 = fmaf(-kOff, sc[u][0], co[u][0]), k1 = fmaf(-kOff, sc[u][1], co[u][1]);
                acc[0] += fmaf(sc[u][0], d[0], k0 * sxa);
                acc[1] += fmaf(sc[u][0], d[1], k0 * sxb);
                acc[2] += fmaf(sc[u][1], d[2], k1 * sxa);
                acc[3] += fmaf(sc[u][1], d[3], k1 * sxb);
            }
        }
    }
    // the warps' partials, summed in warp order
#pragma unroll
    for (int i = 0; i < 4; ++i) red[warp][lane][i] = acc[i];
    __syncthreads();
    if (warp != 0) return;
    float tot[4] = {0.f, 0.f, 0.f, 0.f};
    for (int w = 0; w < kAqWarps; ++w)
#pragma unroll
        for (int i = 0; i < 4; ++i) tot[i] += red[w][lane][i];
    // element i: row (i < 2 ? row0 : row1), token m0 + 2t + (i & 1)
    if (ks == 1) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int64_t row = i < 2 ? row0 : row1;
            const int tk = 2 * t + (i & 1);
            if (row < p.N && tk < mt) Elem<OT>::store(p.out, (m0 + tk) * p.N + row, tot[i]);
        }
        return;
    }
    // split over CTAs: partial [kslice][M][N] in fp32; the last CTA of the
    // tile sums the slices in order
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t row = i < 2 ? row0 : row1;
        const int tk = 2 * t + (i & 1);
        if (row < p.N && tk < mt) p.ws[(int64_t(kslice) * p.M + m0 + tk) * p.N + row] = tot[i];
    }
    __threadfence();
    __syncwarp();
    const int64_t tile = int64_t(blockIdx.z) * gridDim.x + blockIdx.x;
    if (lane == 0) s_last = atomicAdd(&p.cnt[tile], 1u) == unsigned(ks) - 1;
    __syncwarp();
    if (!s_last) return;
    __threadfence();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t row = i < 2 ? row0 : row1;
        const int tk = 2 * t + (i & 1);
        if (row < p.N && tk < mt) {
            float sum = 0.f;
            for (int k = 0; k < ks; ++k) sum += __ldcg(p.ws + (int64_t(k) * p.M + m0 + tk) * p.N + row);
            Elem<OT>::store(p.out, (m0 + tk) * p.N + row, sum);
        }
    }
    if (lane == 0) p.cnt[tile] = 0u;  // every slice has arrived
}

// Final values of a warp's 16-row tile: tot[i] is row tile*16 + g + (i < 2 ?
// 0 : 8), token m0 + 2t + (i & 1). The epilogue keeps the reference's
// rounding points: Matmul stores round(y); Add (Add.metal) then stores
// round(round(y) + r); the gated form takes interleaved [gate; up] tiles
// (rows 16u..16u+7 are gate rows 8u.., rows 16u+8.. the up rows) and stores
// round(round(act(round(g))) * round(u)) (GeluTanh / Mul .metal); the QKV
// form stores q and the new K/V rows into the caches at the position
// (KVCacheWrite.metal:17-26).
template <class OT>
__device__ __forceinline__ void aq_epilogue(const AqMatmul& p, int tile, int g, int t, int mt, int64_t m0,
                                            const float* tot) {
    if (p.epilogue == kAqGated) {
        const int64_t F = p.N / 2, n = int64_t(tile) * 8 + g;
#pragma unroll
        for (int ii = 0; ii < 2; ++ii) {
            const int tk = 2 * t + ii;
            if (n >= F || tk >= mt) continue;
            const float gt = Elem<OT>::round(tot[ii]), up = Elem<OT>::round(tot[2 + ii]);
            const float a = Elem<OT>::round(p.activation == 0 ? gelu_tanh(gt) : silu(gt));
            Elem<OT>::store(p.out, (m0 + tk) * F + n, a * up);
        }
        return;
    }
    int64_t pos = 0;
    if (p.epilogue == kAqQKV) {
        pos = p.pos_dev ? int64_t(*p.pos_dev) : p.offset;
        if (pos < 0 || pos >= p.Smax) return;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t row = int64_t(tile) * 16 + g + (i < 2 ? 0 : 8);
        const int tk = 2 * t + (i & 1);
        if (row >= p.N || tk >= mt) continue;
        const int64_t m = m0 + tk;
        if (p.epilogue == kAqResidual) {
            Elem<OT>::store(p.out, m * p.N + row, Elem<OT>::round(tot[i]) + Elem<OT>::load(p.residual, m * p.N + row));
        } else if (p.epilogue == kAqQKV) {
            if (row < p.q_rows) {
                Elem<OT>::store(p.q_out, m * p.q_rows + row, tot[i]);
            } else {
                int64_t r = row - p.q_rows;
                void* cache = p.k_cache;
                if (r >= p.kv_rows) {
                    r -= p.kv_rows;
                    cache = p.v_cache;
                }
                const int64_t nkv = p.kv_rows / p.Hd;
                Elem<OT>::store(cache, ((m * nkv + r / p.Hd) * p.Smax + pos) * p.Hd + r % p.Hd, tot[i]);
            }
        } else {
            Elem<OT>::store(p.out, m * p.N + row, tot[i]);
        }
    }
}

// ---- TMA-fed persistent form (K % 256 == 0) --------------------------------
//
// One CTA per SM, sixteen warps, each an independent stream: a warp takes
// units (16-row tile, K slice) in turn and feeds itself with 3-D TMA copies
// (no multicast) of one 256-value segment of its 16 rows (2 KB) into a
// private two-slot ring, one segment ahead of the one it multiplies. The
// packed matrix is viewed as [32 words][N rows][K/256 segments]; the 128-byte
// swizzle makes the 8-byte loads of eight different rows conflict-free. The
// four scales (and biases) of a row's segment are 8 contiguous bytes: the
// warp's lanes copy them with cp.async into the slot, tracked by the same
// barrier as the segment's TMA copy. No CTA-wide barrier sits in the stream: when a
// tile's K is split over ks warps (few rows), the last warp to finish sums
// the partials from shared memory in slice order (deterministic). x is staged
// once per CTA (its token tile).
constexpr int kQWarps = 16;
constexpr int kQThreads = kQWarps * 32;
// Two slots: 16 warps x 2 copies of 2 KB in flight per SM. More copies in
// flight stream SLOWER on B200 (a per-warp TMA ring with no arithmetic:
// 2 x 2 KB and 3 x 2 KB per warp 6.35-6.5 TB/s, 4 x 2 KB 4.7 TB/s, 6 x 2 KB
// 3.4 TB/s), and this kernel's warps are busy issuing their arithmetic.
constexpr int kQSlots = 2;       // ring slots per warp
constexpr int kQAhead = kQSlots - 1;
constexpr int kQSegBytes = 2048;  // 16 rows x 128 B

// Stage cursor of one warp: unit v = warp, warp + 16, ... of its CTA's unit
// list (v = i * ks + k: tile blockIdx.x + i * gridDim.x, slice k), then the
// segments of the unit's slice.
struct AqCursor {
    int v, seg, seg1, tile, k;
    bool valid;
    __device__ void set_unit(const AqTmaPlan& q, int ntiles, int nseg) {
        const int i = v / q.ks;
        k = v % q.ks;
        tile = int(blockIdx.x) + i * int(gridDim.x);
        valid = tile < ntiles;
        seg = nseg * k / q.ks;
        seg1 = nseg * (k + 1) / q.ks;
    }
    __device__ void advance(const AqTmaPlan& q, int ntiles, int nseg) {
        if (++seg < seg1) return;
        v += kQWarps;
        set_unit(q, ntiles, nseg);
    }
};

// ONE: the token tile is a single token (batch-1 decode), known at compile
// time: only B column 0 and accumulator columns of token 0 carry data.
template <class XT, class ST, class OT, bool ONE>
__global__ void __launch_bounds__(kQThreads, 1)
    aq_qmv_tma_kernel(const __grid_constant__ CUtensorMap wmap, const AqMatmul p, const AqTmaPlan q) {
    constexpr bool F16 = std::is_same<XT, TF16>::value;
    constexpr bool XF32 = std::is_same<XT, TF32>::value;
    constexpr int NP = XF32 ? 2 : 1;
    constexpr float kOff = F16 ? 1024.f : 128.f;
    extern __shared__ __align__(1024) unsigned char q_smem[];
    __shared__ __align__(8) uint64_t full[kQWarps][kQSlots];
    __shared__ unsigned int tile_cnt[2 * kQWarps];
    __shared__ int slot_tile[2 * kQWarps];
    __shared__ float nscale[8];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int64_t G = p.K / 64;
    const int nseg = int(p.K / 256);
    const int ntiles = int((p.N + 15) / 16);
    const int ts_count = 2 * (kQWarps / q.ks);  // partial slots: two rounds of tiles
    // per-warp rings (1024-aligned), tile partials, staged x, x sums
    unsigned char* ring = q_smem + size_t(warp) * kQSlots * kQSegBytes;
    unsigned char* meta = q_smem + size_t(kQWarps) * kQSlots * kQSegBytes + size_t(warp) * kQSlots * 256;
    float* parts = reinterpret_cast<float*>(q_smem + size_t(kQWarps) * kQSlots * (kQSegBytes + 256));
    uint4* xs = reinterpret_cast<uint4*>(reinterpret_cast<unsigned char*>(parts) + size_t(ts_count) * q.ks * 512);
    float* sxs = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(xs) + size_t(G) * q.mt * NP * 128);
    // fused RMSNorm: the norm weights [K] and the quarter-group sums of
    // squares [mt][G][4]
    float* nws = sxs + size_t(G) * q.mt;
    float* nsq = nws + (p.norm_weight ? p.K : 0);
    const int64_t m0 = int64_t(blockIdx.z) * q.mt;
    const int mt = ONE ? 1 : int(p.M - m0 < q.mt ? p.M - m0 : q.mt);

    if (lane == 0)
        for (int i = 0; i < kQSlots; ++i) mbar_init(smem_u32(&full[warp][i]), 1);
    if (tid < ts_count) {
        tile_cnt[tid] = 0u;
        slot_tile[tid] = tid;  // partial slot i first serves the CTA's i-th tile
    }
    mbar_fence_init();
    pdl_launch_dependents();

    AqCursor ic;  // issue cursor (lane 0)
    ic.v = warp;
    ic.set_unit(q, ntiles, nseg);
    int issued = 0;
    // Copies of the weights (never produced by the previous kernel) start
    // before the wait on it.
    // Segment `issued` into its slot: lanes 0-15 copy the four scales of row
    // lane, lanes 16-31 the four biases of row lane - 16 (8-byte cp.async,
    // tracked by the slot's barrier), then lane 0 adds the TMA copy of the
    // weights and the barrier's one arrival.
    auto issue = [&]() {
        if (!ic.valid) return;
        const int slot = issued % kQSlots;
        const uint32_t bar = smem_u32(&full[warp][slot]);
        const int64_t row = int64_t(ic.tile) * 16 + (lane & 15);
        const void* src = lane < 16 ? p.scales : p.biases;
        // rows beyond N and absent biases are zero-filled (source size 0), so
        // the consumers read the slot without conditions
        const bool real = row < p.N && src;
        const char* a = real ? static_cast<const char*>(src) + (row * G + int64_t(ic.seg) * 4) * 2
                             : static_cast<const char*>(p.scales);
        asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(smem_u32(meta + (slot * 32 + lane) * 8)),
                     "l"(a), "r"(real ? 8 : 0)
                     : "memory");
        asm volatile("cp.async.mbarrier.arrive.shared.b64 [%0];" ::"r"(bar) : "memory");
        __syncwarp();
        if (lane == 0) {
            mbar_expect_tx(bar, uint32_t(kQSegBytes));
            tc::tma_load_3d(smem_u32(ring + size_t(slot) * kQSegBytes), &wmap, 0, ic.tile * 16, ic.seg, bar);
        }
        ++issued;
        ic.advance(q, ntiles, nseg);
    };
    if (lane == 0) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&wmap)) : "memory");
    __syncwarp();
    for (int i = 0; i < kQAhead; ++i) issue();
    // the norm weights are parameters, never written by the previous kernel:
    // loaded before the wait on it (made visible by the barrier after the
    // sums of squares)
    if (p.norm && p.norm_weight)
        for (int k = tid; k < int(p.K); k += kQThreads) nws[k] = p.add_one ? 1.0f + p.norm_weight[k] : p.norm_weight[k];

    pdl_wait();
    if (p.norm) {
        // fused RMSNorm: token n's scale rsqrt(mean(x^2) + eps). The sums of
        // squares of quarter groups (16 values, two 16-byte loads, all in
        // flight) go to the sums area, then one warp per token adds its
        // quarters (lane-strided, then a butterfly: every lane the same
        // value); the staging pass below re-reads x from L1.
        float* sq = nsq;
        for (int u = tid; u < 4 * int(G) * mt; u += kQThreads) {
            const int tt = u & 3, jn = u >> 2;
            const int j = jn / mt, n = jn % mt;
            const char* src =
                static_cast<const char*>(p.x) + ((m0 + n) * p.K + int64_t(j) * 64 + tt * 16) * Elem<XT>::bytes;
            float ss = 0.f;
            if constexpr (!XF32) {
                const uint4 c0 = __ldg(reinterpret_cast<const uint4*>(src));
                const uint4 c1 = __ldg(reinterpret_cast<const uint4*>(src) + 1);
                float f[8];
                unpack8<XT>(c0, f);
#pragma unroll
                for (int e = 0; e < 8; ++e) ss += f[e] * f[e];
                unpack8<XT>(c1, f);
#pragma unroll
                for (int e = 0; e < 8; ++e) ss += f[e] * f[e];
            } else {
                float4 c[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) c[i] = __ldg(reinterpret_cast<const float4*>(src) + i);
#pragma unroll
                for (int i = 0; i < 4; ++i) ss += c[i].x * c[i].x + c[i].y * c[i].y + c[i].z * c[i].z + c[i].w * c[i].w;
            }
            sq[(n * int(G) + j) * 4 + tt] = ss;
        }
        __syncthreads();
        if (warp < mt) {
            float ss = 0.f;
            for (int i = lane; i < 4 * int(G); i += 32) ss += sq[warp * 4 * int(G) + i];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            if (lane == 0) nscale[warp] = rsqrtf(ss / float(p.K) + p.eps);
        }
        __syncthreads();
    }
    stage_x<XT>(p, m0, mt, 0, int(G), xs, sxs, tid, kQThreads, p.norm ? nscale : nullptr,
                p.norm && p.norm_weight ? nws : nullptr);
    __syncthreads();  // x staged, barriers and partial slots initialised
    // per-thread shared offsets: the weights' swizzled 8-byte word pair of
    // group jl of a segment (row g; row g + 8 is 1 KB further), and x
    uint32_t woff[4];
#pragma unroll
    for (int jl = 0; jl < 4; ++jl) woff[jl] = g * 128 + (t & 1) * 8 + ((((jl << 1) | (t >> 1)) ^ g) << 4);
    const size_t xstep = size_t(mt) * NP * 8;  // uint4s per group
    // B column g reads token min(g, mt - 1): columns past the last token
    // repeat it and their outputs are never stored
    const uint4* xthr = xs + size_t(g < mt ? g : mt - 1) * NP * 8 + t;

    AqCursor cc;  // consume cursor
    cc.v = warp;
    cc.set_unit(q, ntiles, nseg);
    int consumed = 0;
    bool ok = true;
    while (cc.valid && ok) {
        const int tile = cc.tile, k = cc.k, v = cc.v;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        while (cc.valid && cc.v == v) {
            issue();  // keep kQAhead segments in flight
            const int slot = consumed % kQSlots;
            if (!mbar_wait(smem_u32(&full[warp][slot]), uint32_t(consumed / kQSlots) & 1u, &g_aq_error_word)) {
                ok = false;
                break;
            }
            const unsigned char* stg = ring + size_t(slot) * kQSegBytes;
            // the segment's four scales / biases of rows g and g + 8
            const uint2* ms = reinterpret_cast<const uint2*>(meta + slot * 32 * 8);
            const uint2 sa = ms[g], sb = ms[g + 8], ba = ms[16 + g], bb = ms[24 + g];
            const float sc0[4] = {unpack2<ST>(sa.x).x, unpack2<ST>(sa.x).y, unpack2<ST>(sa.y).x, unpack2<ST>(sa.y).y};
            const float sc1[4] = {unpack2<ST>(sb.x).x, unpack2<ST>(sb.x).y, unpack2<ST>(sb.y).x, unpack2<ST>(sb.y).y};
            const float bi0[4] = {unpack2<ST>(ba.x).x, unpack2<ST>(ba.x).y, unpack2<ST>(ba.y).x, unpack2<ST>(ba.y).y};
            const float bi1[4] = {unpack2<ST>(bb.x).x, unpack2<ST>(bb.x).y, unpack2<ST>(bb.y).x, unpack2<ST>(bb.y).y};
            const uint4* xseg = xthr + size_t(cc.seg) * 4 * xstep;
            // sum(x) of the segment's four groups (token 0 only when ONE)
            float4 sx4 = make_float4(0.f, 0.f, 0.f, 0.f);
            if constexpr (ONE) sx4 = *reinterpret_cast<const float4*>(sxs + cc.seg * 4);
#pragma unroll
            for (int jl = 0; jl < 4; ++jl) {
                const int j = cc.seg * 4 + jl;
                // 128-byte swizzle: 16-byte chunk c of row line g sits at c ^ (g & 7)
                const uint2 wa = *reinterpret_cast<const uint2*>(stg + woff[jl]);
                const uint2 wb = *reinterpret_cast<const uint2*>(stg + woff[jl] + 8 * 128);
                const uint4* xl = xseg + jl * xstep;
                float d[4] = {0.f, 0.f, 0.f, 0.f};
                group_mma<F16, NP>(wa.x, wa.y, wb.x, wb.y, xl, xl + 4, true, d);
                // D = sum x (kOff + q): acc += scale * D + (bias - kOff * scale) * sum(x)
                if constexpr (ONE) {
                    // accumulator columns 2t, 2t + 1: only t == 0, column 0 is
                    // a token. The offset leaves D inside one fma (D - kOff *
                    // sum(x) = sum x q, the only rounding that of the small
                    // result), then acc += scale * that + bias * sum(x).
                    const float sxa = jl == 0 ? sx4.x : jl == 1 ? sx4.y : jl == 2 ? sx4.z : sx4.w;
                    const float e0 = fmaf(-kOff, sxa, d[0]), e2 = fmaf(-kOff, sxa, d[2]);
                    acc[0] = fmaf(sc0[jl], e0, fmaf(bi0[jl], sxa, acc[0]));
                    acc[2] = fmaf(sc1[jl], e2, fmaf(bi1[jl], sxa, acc[2]));
                } else {
                    const float k0 = fmaf(-kOff, sc0[jl], bi0[jl]), k1 = fmaf(-kOff, sc1[jl], bi1[jl]);
                    const float sxa = 2 * t < mt ? sxs[j * mt + 2 * t] : 0.f;
                    const float sxb = 2 * t + 1 < mt ? sxs[j * mt + 2 * t + 1] : 0.f;
                    acc[0] += fmaf(sc0[jl], d[0], k0 * sxa);
                    acc[1] += fmaf(sc0[jl], d[1], k0 * sxb);
                    acc[2] += fmaf(sc1[jl], d[2], k1 * sxa);
                    acc[3] += fmaf(sc1[jl], d[3], k1 * sxb);
                }
            }
            __syncwarp();  // the slot is refilled by a later issue()
            ++consumed;
            cc.advance(q, ntiles, nseg);
        }
        if (!ok) break;
        // element i: row (i < 2 ? r0 : r1), token m0 + 2t + (i & 1)
        if (q.ks == 1) {
            aq_epilogue<OT>(p, tile, g, t, mt, m0, acc);
            continue;
        }
        // K split over ks warps of this CTA: partial into the tile's slot; the
        // last to arrive sums the slices in order
        const int ti = v / q.ks;  // the tile's index in this CTA's list
        const int ts = ti % ts_count;
        if (lane == 0) {
            int spins = 0;
            while (*reinterpret_cast<volatile int*>(&slot_tile[ts]) != ti && ++spins < (1 << 22)) __nanosleep(64);
            if (spins >= (1 << 22)) atomicOr(&g_aq_error_word, 1u);
        }
        __syncwarp();
        float* slot_parts = parts + size_t(ts) * q.ks * 128;
#pragma unroll
        for (int i = 0; i < 4; ++i) slot_parts[size_t(k) * 128 + i * 32 + lane] = acc[i];
        __threadfence_block();
        __syncwarp();
        unsigned int prev = 0;
        if (lane == 0) prev = atomicAdd(&tile_cnt[ts], 1u);
        prev = __shfl_sync(0xffffffffu, prev, 0);
        if (prev != unsigned(q.ks) - 1) continue;
        __threadfence_block();
        float tot[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float sum = 0.f;
            for (int kk = 0; kk < q.ks; ++kk)
                sum += *reinterpret_cast<volatile float*>(&slot_parts[size_t(kk) * 128 + i * 32 + lane]);
            tot[i] = sum;
        }
        aq_epilogue<OT>(p, tile, g, t, mt, m0, tot);
        __syncwarp();
        if (lane == 0) {
            tile_cnt[ts] = 0u;
            __threadfence_block();
            *reinterpret_cast<volatile int*>(&slot_tile[ts]) = ti + ts_count;  // the slot's next tile
        }
    }
    // a wait gave up: drain (bounded) this warp's copies still in flight
    if (!ok && lane == 0)
        for (int j = consumed; j < issued; ++j)
            mbar_wait(smem_u32(&full[warp][j % kQSlots]), uint32_t(j / kQSlots) & 1u, &g_aq_error_word);
}

// ---- embedding gathers ------------------------------------------------------

template <class TT, class OT>
__global__ void embedding_gather_kernel(const int32_t* ids, const void* table, void* out, int64_t T, int64_t H,
                                        int64_t vocab, unsigned int* err) {
    pdl_wait();
    const int64_t n = blockIdx.y;
    const int64_t id = ids[n];
    if (id < 0 || id >= vocab) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(err, 16u);
        return;
    }
    for (int64_t h = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; h < H; h += int64_t(gridDim.x) * blockDim.x)
        Elem<OT>::store(out, n * H + h, Elem<TT>::load(table, id * H + h));
}

template <class ST, class OT>
__global__ void aq_embedding_gather_kernel(const int32_t* ids, const uint32_t* w, const void* scales,
                                           const void* biases, void* out, int64_t T, int64_t H, int64_t vocab,
                                           unsigned int* err) {
    pdl_wait();
    const int64_t n = blockIdx.y;
    const int64_t id = ids[n];
    if (id < 0 || id >= vocab) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(err, 16u);
        return;
    }
    const int64_t G = H / 64;
    for (int64_t h = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; h < H; h += int64_t(gridDim.x) * blockDim.x) {
        const float s = Elem<ST>::load(scales, id * G + h / 64);
        const float b = biases ? Elem<ST>::load(biases, id * G + h / 64) : 0.f;
        const uint32_t q = (__ldg(w + id * (H / 8) + h / 8) >> ((h % 8) * 4)) & 15u;
        Elem<OT>::store(out, n * H + h, float(q) * s + b);
    }
}

// staged bytes per chunk group: mt tokens x parts x 128 B, plus its sums
inline size_t aq_group_bytes(const AqMatmul& p) {
    const int64_t mt = p.M < 8 ? p.M : 8;
    return size_t(mt) * (p.x_dtype == PC_F32 ? 2 : 1) * 128 + size_t(mt) * 4;
}

cudaError_t launch_aq(void (*kern)(AqMatmul), const AqMatmul& p, dim3 grid, cudaStream_t s) {
    const size_t smem = size_t(p.chunk_groups) * aq_group_bytes(p);
    cudaError_t e = allow_smem(kern, smem);
    if (e != cudaSuccess) return e;
    return launch_k(kern, grid, dim3(kAqThreads), smem, s, p);
}

template <class XT, class ST>
cudaError_t run_aq_o(const AqMatmul& p, dim3 grid, cudaStream_t s) {
    switch (p.out_dtype) {
    case PC_F32: return launch_aq(aq_matmul_kernel<XT, ST, TF32>, p, grid, s);
    case PC_F16: return launch_aq(aq_matmul_kernel<XT, ST, TF16>, p, grid, s);
    case PC_BF16: return launch_aq(aq_matmul_kernel<XT, ST, TBF16>, p, grid, s);
    }
    return cudaErrorInvalidValue;
}

}  // namespace

bool aq_tma_plan(const AqMatmul& p, AqTmaPlan& q);

int aq_matmul_plan(const AqMatmul& p, int sm_count) {
    AqTmaPlan q{};
    if (!p.no_tma && aq_tma_plan(p, q)) return 1;  // the TMA form needs no split
    const int64_t tiles = ((p.N + 15) / 16) * ((p.M + 7) / 8);
    const int64_t G = p.K / 64;
    int64_t ks = 1;
    if (tiles < 2 * sm_count) ks = (2 * sm_count + tiles - 1) / tiles;
    const int64_t max_ks = G / (2 * kAqWarps);  // >= two groups per warp
    if (ks > max_ks) ks = max_ks;
    if (ks < 1) ks = 1;
    if (ks > 64) ks = 64;
    return int(ks);
}

size_t aq_matmul_workspace(const AqMatmul& p, int kslices) {
    if (kslices <= 1) return 0;
    const int64_t tiles = ((p.N + 15) / 16) * ((p.M + 7) / 8);
    return size_t(kslices) * p.M * p.N * 4 + size_t(tiles) * 4 + 256;
}

// TMA form plan: K split over ks (1, 2, 4, 8 or 16) warps when the 16-row
// tiles are fewer than the GPU's warps; x of mt tokens staged per CTA.
bool aq_tma_plan(const AqMatmul& p, AqTmaPlan& q) {
    if (p.K % 256 != 0 || (reinterpret_cast<uintptr_t>(p.w) & 15) || (reinterpret_cast<uintptr_t>(p.scales) & 7) ||
        (p.biases && (reinterpret_cast<uintptr_t>(p.biases) & 7)) || p.N >= (int64_t(1) << 31) ||
        p.K / 256 > 65535 || tc::encode_fn() == nullptr)
        return false;
    const int64_t nseg = p.K / 256, G = p.K / 64;
    const int64_t tiles = (p.N + 15) / 16;
    const int sms = current_sm_count();
    q.ks = 1;
    while (q.ks < kQWarps && tiles * q.ks < int64_t(sms) * kQWarps && 2 * q.ks <= nseg) q.ks *= 2;
    const size_t fixed =
        size_t(kQWarps) * kQSlots * (kQSegBytes + 256) + size_t(2 * (kQWarps / q.ks)) * q.ks * 512;
    const size_t norm_fixed = p.norm && p.norm_weight ? size_t(p.K) * 4 : 0;  // norm weights
    if (fixed + norm_fixed >= 220 * 1024) return false;
    const size_t budget = 220 * 1024 - fixed - norm_fixed;
    const size_t per_token = size_t(G) * ((p.x_dtype == PC_F32 ? 2 : 1) * 128 + 4 + (p.norm ? 16 : 0));
    int64_t mt = int64_t(budget / per_token);
    if (mt > 8) mt = 8;
    if (mt > p.M) mt = p.M;
    if (mt < 1) return false;
    q.mt = int(mt);
    q.mtiles = int((p.M + mt - 1) / mt);
    q.smem = fixed + norm_fixed + size_t(q.mt) * per_token;
    return true;
}

bool make_aq_map(CUtensorMap* map, const AqMatmul& p, const AqTmaPlan& q) {
    tc::EncodeTiledFn fn = tc::encode_fn();
    cuuint64_t dims[3] = {32, cuuint64_t(p.N), cuuint64_t(p.K / 256)};
    cuuint64_t strides[2] = {cuuint64_t(p.K / 2), 128};
    cuuint32_t box[3] = {32, 16, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<uint32_t*>(p.w), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <class XT, class ST>
cudaError_t run_tma_o(const CUtensorMap& map, const AqMatmul& p, const AqTmaPlan& q, cudaStream_t s) {
    auto go = [&](void (*kern)(CUtensorMap, AqMatmul, AqTmaPlan)) {
        cudaError_t e = allow_smem(kern, q.smem);
        if (e != cudaSuccess) return e;
        const int64_t tiles = (p.N + 15) / 16;
        // CTAs: every SM, each with at least one tile per warp-slice round
        int64_t ctas = current_sm_count();
        if (ctas > tiles) ctas = tiles;
        dim3 grid(unsigned(ctas), 1, unsigned(q.mtiles));
        return launch_k(kern, grid, dim3(kQThreads), q.smem, s, map, p, q);
    };
    const bool one = q.mt == 1;
    switch (p.out_dtype) {
    case PC_F32: return go(one ? aq_qmv_tma_kernel<XT, ST, TF32, true> : aq_qmv_tma_kernel<XT, ST, TF32, false>);
    case PC_F16: return go(one ? aq_qmv_tma_kernel<XT, ST, TF16, true> : aq_qmv_tma_kernel<XT, ST, TF16, false>);
    case PC_BF16: return go(one ? aq_qmv_tma_kernel<XT, ST, TBF16, true> : aq_qmv_tma_kernel<XT, ST, TBF16, false>);
    }
    return cudaErrorInvalidValue;
}

cudaError_t aq_matmul(const AqMatmul& p0, cudaStream_t s) {
    if (p0.M == 0 || p0.N == 0) return cudaSuccess;
    AqMatmul p = p0;
    AqTmaPlan q{};
    if (p.kslices <= 1 && !p.no_tma && aq_tma_plan(p, q)) {
        CUtensorMap map;
        if (make_aq_map(&map, p, q)) {
            const bool s16 = p.s_dtype == PC_F16;
            if (p.x_dtype == PC_BF16) return s16 ? run_tma_o<TBF16, TF16>(map, p, q, s) : run_tma_o<TBF16, TBF16>(map, p, q, s);
            if (p.x_dtype == PC_F16) return s16 ? run_tma_o<TF16, TF16>(map, p, q, s) : run_tma_o<TF16, TBF16>(map, p, q, s);
            if (p.x_dtype == PC_F32) return s16 ? run_tma_o<TF32, TF16>(map, p, q, s) : run_tma_o<TF32, TBF16>(map, p, q, s);
            return cudaErrorInvalidValue;
        }
    }
    // the fused forms exist in the TMA form only
    if (p.norm || p.epilogue != kAqStore) return cudaErrorInvalidValue;
    if (p.kslices < 1) p.kslices = 1;
    if (p.kslices > 1) {
        // partials, then the per-tile arrival counters (zeroed per launch)
        const int64_t tiles = ((p.N + 15) / 16) * ((p.M + 7) / 8);
        char* ws = static_cast<char*>(p.workspace);
        p.ws = reinterpret_cast<float*>(ws);
        p.cnt = reinterpret_cast<unsigned int*>(ws + (size_t(p.kslices) * p.M * p.N * 4 + 255) / 256 * 256);
        cudaError_t e = cudaMemsetAsync(p.cnt, 0, size_t(tiles) * 4, s);
        if (e != cudaSuccess) return e;
    }
    dim3 grid(unsigned((p.N + 15) / 16), unsigned(p.kslices), unsigned((p.M + 7) / 8));
    // groups staged per chunk: the slice, or as many as fit
    const int64_t slice = (p.K / 64 + p.kslices - 1) / p.kslices;
    const int64_t fit = int64_t(kAqSmemMax / aq_group_bytes(p));
    p.chunk_groups = int(slice < fit ? slice : fit);
    const bool s16 = p.s_dtype == PC_F16;
    if (p.x_dtype == PC_BF16) return s16 ? run_aq_o<TBF16, TF16>(p, grid, s) : run_aq_o<TBF16, TBF16>(p, grid, s);
    if (p.x_dtype == PC_F16) return s16 ? run_aq_o<TF16, TF16>(p, grid, s) : run_aq_o<TF16, TBF16>(p, grid, s);
    if (p.x_dtype == PC_F32) return s16 ? run_aq_o<TF32, TF16>(p, grid, s) : run_aq_o<TF32, TBF16>(p, grid, s);
    return cudaErrorInvalidValue;
}

cudaError_t embedding_gather(const EmbeddingGather& p, cudaStream_t s) {
    if (p.T == 0 || p.H == 0) return cudaSuccess;
    unsigned int* err = nullptr;
    cudaGetSymbolAddress(reinterpret_cast<void**>(&err), g_aq_error_word);
    const unsigned bx = unsigned((p.H + 255) / 256 < 64 ? (p.H + 255) / 256 : 64);
    dim3 grid(bx, unsigned(p.T)), blk(256);
    if (p.packed) {
        auto go = [&](auto st, auto ot) {
            using S = decltype(st);
            using O = decltype(ot);
            return launch_k(aq_embedding_gather_kernel<S, O>, grid, blk, 0, s, p.ids, p.packed, p.scales, p.biases,
                            p.out, p.T, p.H, p.vocab, err);
        };
        const bool s16 = p.table_dtype == PC_F16;
        switch (p.out_dtype) {
        case PC_F32: return s16 ? go(TF16{}, TF32{}) : go(TBF16{}, TF32{});
        case PC_F16: return s16 ? go(TF16{}, TF16{}) : go(TBF16{}, TF16{});
        case PC_BF16: return s16 ? go(TF16{}, TBF16{}) : go(TBF16{}, TBF16{});
        }
        return cudaErrorInvalidValue;
    }
    auto go = [&](auto tt, auto ot) {
        using TT = decltype(tt);
        using O = decltype(ot);
        return launch_k(embedding_gather_kernel<TT, O>, grid, blk, 0, s, p.ids, p.table, p.out, p.T, p.H, p.vocab,
                        err);
    };
    if (p.table_dtype == PC_F32 && p.out_dtype == PC_F32) return go(TF32{}, TF32{});
    if (p.table_dtype == PC_F16 && p.out_dtype == PC_F16) return go(TF16{}, TF16{});
    if (p.table_dtype == PC_BF16 && p.out_dtype == PC_BF16) return go(TBF16{}, TBF16{});
    if (p.table_dtype == PC_BF16 && p.out_dtype == PC_F32) return go(TBF16{}, TF32{});
    return cudaErrorInvalidValue;
}

uint32_t read_and_clear_aq_errors() {
    unsigned int v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_aq_error_word, sizeof(v)) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    if (v) cudaMemcpyToSymbol(g_aq_error_word, &zero, sizeof(zero));
    return v;
}

namespace {
RegisterFunctions reg_aq({
    {"aq_qmv_fast_bf16_bf16_bf16_b4_g64", reinterpret_cast<const void*>(aq_matmul_kernel<TBF16, TBF16, TBF16>)},
    {"aq_qmv_fast_bf16_bf16_f32_b4_g64", reinterpret_cast<const void*>(aq_matmul_kernel<TBF16, TBF16, TF32>)},
    {"aq_qmv_fast_f32_bf16_f32_b4_g64", reinterpret_cast<const void*>(aq_matmul_kernel<TF32, TBF16, TF32>)},
    {"aq_qmv_fast_f16_f16_f16_b4_g64", reinterpret_cast<const void*>(aq_matmul_kernel<TF16, TF16, TF16>)},
    {"aq_fused_bf16_b4_g64", reinterpret_cast<const void*>(aq_qmv_tma_kernel<TBF16, TBF16, TBF16, true>)},
    {"aq_fused_f16_b4_g64", reinterpret_cast<const void*>(aq_qmv_tma_kernel<TF16, TF16, TF16, true>)},
    {"aq_matvec_simd4_bf16_bf16_bf16_b4_g64", reinterpret_cast<const void*>(aq_matmul_kernel<TBF16, TBF16, TBF16>)},
    {"aq_matvec_simd4_bf16_bf16_f32_b4_g64", reinterpret_cast<const void*>(aq_matmul_kernel<TBF16, TBF16, TF32>)},
    {"aq_matvec_simd4_f32_bf16_f32_b4_g64", reinterpret_cast<const void*>(aq_matmul_kernel<TF32, TBF16, TF32>)},
    {"aq_matvec_simd4_f16_f16_f16_b4_g64", reinterpret_cast<const void*>(aq_matmul_kernel<TF16, TF16, TF16>)},
    {"embedding_gather", reinterpret_cast<const void*>(embedding_gather_kernel<TF32, TF32>)},
    {"embedding_gather_f16", reinterpret_cast<const void*>(embedding_gather_kernel<TF16, TF16>)},
    {"embedding_gather_bf16", reinterpret_cast<const void*>(embedding_gather_kernel<TBF16, TBF16>)},
    {"embedding_gather_bf16_to_f32", reinterpret_cast<const void*>(embedding_gather_kernel<TBF16, TF32>)},
    {"aq_embedding_gather_bf16_bf16_b4_g64", reinterpret_cast<const void*>(aq_embedding_gather_kernel<TBF16, TBF16>)},
    {"aq_embedding_gather_bf16_f32_b4_g64", reinterpret_cast<const void*>(aq_embedding_gather_kernel<TBF16, TF32>)},
    {"aq_embedding_gather_f16_f16_b4_g64", reinterpret_cast<const void*>(aq_embedding_gather_kernel<TF16, TF16>)},
});
}  // namespace

}  // namespace launch
}  // namespace popcorn
