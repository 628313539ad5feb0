// popcorn_oracle.cpp — CPU restatement of the reference decode-step kernels.
//
// TEST INFRASTRUCTURE ONLY. This library is the parity checker for the CUDA
// path and the timed CPU baseline in bench.py. Nothing in the product
// (popcorn_b200/, include/) links, loads or calls it.
//
// Every function restates one Metal kernel of finnvoor/Popcorn, keeping its
// arithmetic (fp32 accumulators, the same partition / tile / reduction
// structure, the same rounding points) so that results agree with the
// reference to the last few fp32 ulps before the final store:
//
//   or_kv_cache_write      Sources/Popcorn/Kernels/KVCacheWrite.metal:7-59
//   or_rmsnorm             Sources/Popcorn/Kernels/RMSNorm.metal:7-42 with the
//                          threadgroup width of Kernels/DispatchSize.swift:6-27,67-105
//   or_matvec_nk           Sources/Popcorn/Kernels/Matvec.metal:56-127
//   or_matmul              Sources/Popcorn/Kernels/Matmul.metal:7-27
//   or_gelu_tanh           Sources/Popcorn/Kernels/GeluTanh.metal:6-35
//   or_mul / or_add        Sources/Popcorn/Kernels/Mul.metal:7-25, Add.metal:7-25
//   or_rope_build          Sources/Popcorn/Kernels/RopeBuildCosSin.metal:5-21
//   or_rope_apply          Sources/Popcorn/Kernels/RopeApply.metal:6-49
//   or_aq_matmul           Sources/Popcorn/Kernels/Quantized/AffineQuantizedMatmul.metal:9-160,
//                          routing Kernels/Matmul.swift:279-333
//   or_embedding_gather    Sources/Popcorn/Kernels/EmbeddingGather.metal:6-30
//   or_aq_embedding_gather Sources/Popcorn/Kernels/Quantized/AffineQuantizedEmbeddingGather.metal:6-27
//   or_argmax              Sources/Popcorn/Kernels/Argmax.metal:5-76, routing
//                          Argmax.swift:21 (n >= 32 -> argmax_row)
//   or_flash_decoding      Sources/Popcorn/Kernels/FlashDecoding.metal:29-231
//                          with P = 8 from Kernels/FlashDecoding.swift:77
//   or_flash_attention     Sources/Popcorn/Kernels/FlashAttention.metal:31-162
//   or_attention_exact     Tests/PopcornTests/Kernels/BidirectionalFATests.swift:9-53
//                          (generalised to GQA, masks and Sq != Sk; float64)
//
// Element conversions follow Sources/Popcorn/PopcornDTypes.h:9-53: bf16 loads
// are a 16-bit shift, bf16 stores are round-to-nearest-even with no NaN
// special case (:29-34); f16 uses IEEE round-to-nearest-even (_Float16).
//
// Pinning: every function above with a reference test is checked against it
// (tests/golden/reference_kats.json, tests/test_oracle.py). The affine-
// quantized Matmul and the quantized embedding gather have none in the
// reference: their restatements are parity unpinned (checked only against a
// float64 dequantised product and their own format definition).
//
// Extensions that the reference does not have (f16 FlashDecoding / matvec /
// KV write, ragged per-sequence lengths, SiLU) reuse the same templates with
// the f16 load/store of PopcornDTypes.h:10,37, as the reference's own
// template instantiations would.

#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>
#include <algorithm>
#include <limits>
#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

// Tensor.DataType raw order, Sources/Popcorn/Tensor.swift:135-148.
enum DType : int { U8 = 0, U16, U32, U64, I8, I16, I32, I64, F32, F16, BF16 };

inline float bits_to_float(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }
inline uint32_t float_to_bits(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }

// PopcornDTypes.h:29-34 — RNE with no NaN special case.
inline uint16_t f32_to_bf16(float x) {
    uint32_t bits = float_to_bits(x);
    uint32_t lsb = (bits >> 16) & 1u;
    return uint16_t((bits + 0x7fffu + lsb) >> 16);
}

inline float load(const void* p, int dt, int64_t i) {
    switch (dt) {
    case F32: return static_cast<const float*>(p)[i];
    case F16: return float(static_cast<const _Float16*>(p)[i]);
    case BF16: return bits_to_float(uint32_t(static_cast<const uint16_t*>(p)[i]) << 16);
    case I8: return float(static_cast<const int8_t*>(p)[i]);
    case U8: return float(static_cast<const uint8_t*>(p)[i]);
    default: return 0.0f;
    }
}

inline void store(void* p, int dt, int64_t i, float x) {
    switch (dt) {
    case F32: static_cast<float*>(p)[i] = x; break;
    case F16: static_cast<_Float16*>(p)[i] = (_Float16)x; break;
    case BF16: static_cast<uint16_t*>(p)[i] = f32_to_bf16(x); break;
    default: break;
    }
}

// The value a store to `dt` followed by a load gives back (a rounding point).
inline float round_to(int dt, float x) {
    switch (dt) {
    case F16: return float((_Float16)x);
    case BF16: return bits_to_float(uint32_t(f32_to_bf16(x)) << 16);
    default: return x;
    }
}

// simd_sum over 32 lanes as a butterfly (xor 16, 8, 4, 2, 1).
inline float simd_sum32(float* v) {
    for (int off = 16; off >= 1; off >>= 1) {
        float t[32];
        for (int l = 0; l < 32; ++l) t[l] = v[l] + v[l ^ off];
        std::memcpy(v, t, sizeof(t));
    }
    return v[0];
}

inline float gelu_tanh_scalar(float v) {
    // GeluTanh.metal:6-11 (inner argument clamped to +-20).
    const float k0 = 0.7978845608028654f;
    const float k1 = 0.044715f;
    float inner = std::min(std::max(k0 * (v + k1 * v * v * v), -20.0f), 20.0f);
    return 0.5f * v * (1.0f + std::tanh(inner));
}

inline float silu_scalar(float v) { return v / (1.0f + std::exp(-v)); }

// DispatchSize.swift:6-27, 67-105 with simdWidth 32 and a 1024-thread cap.
int reduction_width(int64_t rows, int64_t n) {
    int sg;
    if (rows <= 4) sg = n <= 256 ? 8 : (n <= 1536 ? 16 : 32);
    else if (rows <= 16) sg = n <= 256 ? 4 : (n <= 3072 ? 16 : 32);
    else if (rows <= 64) sg = n <= 768 ? 4 : (n <= 3072 ? 8 : (n <= 8192 ? 16 : 32));
    else if (rows <= 256) sg = n <= 256 ? 1 : (n <= 3072 ? 2 : (n <= 8192 ? 4 : 32));
    else if (rows <= 512) sg = n <= 768 ? 1 : (n <= 1536 ? 2 : (n <= 3072 ? 16 : (n <= 8192 ? 8 : 32)));
    else sg = n <= 768 ? 2 : (n <= 1536 ? 8 : (n <= 3072 ? 32 : 16));
    int preferred = std::min(1024, sg * 32);
    int64_t np2 = 1;
    while (np2 < n) np2 <<= 1;
    int64_t cap = ((np2 + 31) / 32) * 32;
    return int(std::max<int64_t>(32, std::min<int64_t>(preferred, cap)));
}

}  // namespace

extern "C" {

int or_version(void) { return 1; }

int or_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void or_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

void or_convert(const void* src, int sdt, void* dst, int ddt, int64_t n) {
    for (int64_t i = 0; i < n; ++i) store(dst, ddt, i, load(src, sdt, i));
}

// KVCacheWrite.metal:7-59. Element (b,h,s,d) of src goes to
// ((b*Nkv + h)*Smax + offset + s)*Hd + d of the cache; the value is a load
// followed by a store (bit-exact copy when the dtypes agree, RNE otherwise).
void or_kv_cache_write(const void* src, int sdt, void* cache, int cdt, int64_t B, int64_t Nkv,
                       int64_t Snew, int64_t Smax, int64_t Hd, int64_t offset) {
    int64_t total = B * Nkv * Snew * Hd;
    for (int64_t i = 0; i < total; ++i) {
        int64_t d = i % Hd, r = i / Hd;
        int64_t s = r % Snew; r /= Snew;
        int64_t h = r % Nkv, b = r / Nkv;
        int64_t dst = ((b * Nkv + h) * Smax + offset + s) * Hd + d;
        store(cache, cdt, dst, load(src, sdt, i));
    }
}

// RMSNorm.metal:7-42. One threadgroup of `width` threads per row: each thread
// sums x^2 over i = tid, tid+width, ...; a power-of-two tree folds the
// partials; scale = 1/sqrt(ss/H + eps); out = (x*scale)*(w or 1+w), stored
// once. `w` may be null (no weight). width <= 0 picks DispatchSize's width.
void or_rmsnorm(const void* x, int xdt, const float* w, void* out, int odt, int64_t rows, int64_t H,
                float eps, int add_one, int width) {
    int tg = width > 0 ? width : reduction_width(rows, H);
#pragma omp parallel for schedule(static)
    for (int64_t row = 0; row < rows; ++row) {
        std::vector<float> partial(tg, 0.0f);
        int64_t base = row * H;
        for (int t = 0; t < tg; ++t) {
            float acc = 0.0f;
            for (int64_t i = t; i < H; i += tg) {
                float v = load(x, xdt, base + i);
                acc += v * v;
            }
            partial[t] = acc;
        }
        for (int stride = tg >> 1; stride > 0; stride >>= 1)
            for (int t = 0; t < stride; ++t) partial[t] += partial[t + stride];
        float scale = 1.0f / std::sqrt(partial[0] / float(H) + eps);
        for (int64_t i = 0; i < H; ++i) {
            float v = load(x, xdt, base + i) * scale;
            if (w) {
                float ww = w[i];
                if (add_one) ww = 1.0f + ww;
                v *= ww;
            }
            store(out, odt, base + i, v);
        }
    }
}

// Matvec.metal:56-127 (matvec_nk_simd4): y[n] = sum_k x[k] * W[n,k], W is
// [N,K] row-major. Lane l accumulates float4 products over k4 = l, l+32, ...
// when K % 4 == 0 (else scalar over k = l, l+32, ...); the four components
// are added x+y+z+w; the 32 lanes are folded by simd_sum; one store.
void or_matvec_nk(const void* x, int xdt, const void* w, int wdt, void* out, int odt, int64_t K,
                  int64_t N) {
    std::vector<float> xf(K);
    for (int64_t k = 0; k < K; ++k) xf[k] = load(x, xdt, k);
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
        float lanes[32];
        int64_t base = n * K;
        for (int l = 0; l < 32; ++l) {
            if ((K & 3) == 0) {
                float v0 = 0, v1 = 0, v2 = 0, v3 = 0;
                for (int64_t k4 = l; k4 < K / 4; k4 += 32) {
                    int64_t k = k4 * 4;
                    v0 += xf[k + 0] * load(w, wdt, base + k + 0);
                    v1 += xf[k + 1] * load(w, wdt, base + k + 1);
                    v2 += xf[k + 2] * load(w, wdt, base + k + 2);
                    v3 += xf[k + 3] * load(w, wdt, base + k + 3);
                }
                lanes[l] = v0 + v1 + v2 + v3;
            } else {
                float acc = 0;
                for (int64_t k = l; k < K; k += 32) acc += xf[k] * load(w, wdt, base + k);
                lanes[l] = acc;
            }
        }
        store(out, odt, n, simd_sum32(lanes));
    }
}

// Matmul.metal:7-27: one fp32 accumulator per output, k ascending.
// transB: B is [N,K] (linear-layer layout), else [K,N].
void or_matmul(const void* a, int adt, const void* b, int bdt, void* c, int cdt, int64_t M,
               int64_t K, int64_t N, int transB) {
#pragma omp parallel for schedule(static)
    for (int64_t m = 0; m < M; ++m) {
        std::vector<float> arow(K);
        for (int64_t k = 0; k < K; ++k) arow[k] = load(a, adt, m * K + k);
        for (int64_t n = 0; n < N; ++n) {
            float acc = 0.0f;
            if (transB)
                for (int64_t k = 0; k < K; ++k) acc += arow[k] * load(b, bdt, n * K + k);
            else
                for (int64_t k = 0; k < K; ++k) acc += arow[k] * load(b, bdt, k * N + n);
            store(c, cdt, m * N + n, acc);
        }
    }
}

void or_gelu_tanh(const void* x, int xdt, void* out, int odt, int64_t n) {
    for (int64_t i = 0; i < n; ++i) store(out, odt, i, gelu_tanh_scalar(load(x, xdt, i)));
}

// SiLU has no reference kernel; restated as silu(g) = g / (1 + exp(-g)).
void or_silu(const void* x, int xdt, void* out, int odt, int64_t n) {
    for (int64_t i = 0; i < n; ++i) store(out, odt, i, silu_scalar(load(x, xdt, i)));
}

void or_mul(const void* a, const void* b, void* out, int dt, int64_t n) {
    for (int64_t i = 0; i < n; ++i) store(out, dt, i, load(a, dt, i) * load(b, dt, i));
}

void or_add(const void* a, const void* b, void* out, int dt, int64_t n) {
    for (int64_t i = 0; i < n; ++i) store(out, dt, i, load(a, dt, i) + load(b, dt, i));
}

// RopeBuildCosSin.metal:13-20: angle = position[t] * inv_freq[i] in fp32;
// cos / sin tables [T, Hd2] (fp32) times `scaling`.
void or_rope_build(const int32_t* positions, const float* inv_freq, float* cos_out, float* sin_out, int64_t T,
                   int64_t Hd2, float scaling) {
    for (int64_t t = 0; t < T; ++t)
        for (int64_t i = 0; i < Hd2; ++i) {
            const float angle = float(positions[t]) * inv_freq[i];
            cos_out[t * Hd2 + i] = std::cos(angle) * scaling;
            sin_out[t * Hd2 + i] = std::sin(angle) * scaling;
        }
}

// RopeApply.metal:15-48: x [B, T, Nh, 2*Hd2]; per head the halves
// x1 = x[:Hd2], x2 = x[Hd2:] become (x1 c - x2 s, x1 s + x2 c) with the
// tables' row t; fp32 arithmetic, one rounding at each store.
void or_rope_apply(const void* x, int xdt, const void* cos_t, const void* sin_t, int tdt, void* out, int odt,
                   int64_t B, int64_t T, int64_t Nh, int64_t Hd2) {
    const int64_t Hd = 2 * Hd2;
    for (int64_t b = 0; b < B; ++b)
        for (int64_t t = 0; t < T; ++t)
            for (int64_t h = 0; h < Nh; ++h) {
                const int64_t base = ((b * T + t) * Nh + h) * Hd;
                for (int64_t i = 0; i < Hd2; ++i) {
                    const float x1 = load(x, xdt, base + i), x2 = load(x, xdt, base + Hd2 + i);
                    const float c = load(cos_t, tdt, t * Hd2 + i), sn = load(sin_t, tdt, t * Hd2 + i);
                    store(out, odt, base + i, x1 * c - x2 * sn);
                    store(out, odt, base + Hd2 + i, x1 * sn + x2 * c);
                }
            }
}

// Argmax.metal:7-9: a candidate wins on a larger value, or an equal value at
// a lower index (NaN never wins: both comparisons are false).
static bool argmax_better(float cv, int32_t ci, float bv, int32_t bi) { return cv > bv || (cv == bv && ci < bi); }

// Per row of x [rows, N]: n < 32 follows `argmax` (:11-27, starts from
// element 0), n >= 32 follows `argmax_row` (:29-76, starts from (-inf,
// 0x7fffffff)); the reduction order of argmax_row does not change the result
// because the order relation above is total on non-NaN values.
void or_argmax(const void* x, int dt, int64_t rows, int64_t N, int32_t* out) {
    for (int64_t r = 0; r < rows; ++r) {
        float bv;
        int32_t bi;
        int64_t i0;
        if (N < 32) {
            bv = load(x, dt, r * N);
            bi = 0;
            i0 = 1;
        } else {
            bv = -INFINITY;
            bi = 0x7fffffff;
            i0 = 0;
        }
        for (int64_t i = i0; i < N; ++i) {
            const float v = load(x, dt, r * N + i);
            if (argmax_better(v, int32_t(i), bv, bi)) {
                bv = v;
                bi = int32_t(i);
            }
        }
        out[r] = bi;
    }
}

// FlashDecoding.metal:29-174 (partial) + :182-231 (reduce), Sq = 1.
//
// Keys of (b, hkv) live at ((b*Nkv + hkv)*kv_stride + j)*Hd: the reference
// passes kv_stride == Sk (:58). The ragged extension passes the cache length
// Smax as kv_stride and a per-sequence key count `lens[b]` (null = Sk for
// every sequence); the query sits at posQ = len - 1 (:73).
//
// For each (b, hq, part): keys [part*per, min(+per, len)), per = ceil(len/P)
// (:61-63); q is pre-scaled (:66); a partition starting past posQ writes
// m = -inf, l = 0, O = 0 (:78-87); tiles of Bc = 128 keys (:89); a key's
// score is the lane-strided partial dot folded by simd_sum (:104-109);
// online softmax with natural exp (:114-152); O = scale_old*O + sum p*V
// (:154-161); the partial O is left unnormalised (:165-173). The reduce
// takes m_g = max m_k, l_g = sum exp(m_k - m_g) l_k and
// O = sum exp(m_k - m_g) O_k / l_g, stored once (:203-227).
//
// A tile whose keys are all masked has max -inf; exp(-inf - -inf) is NaN in
// IEEE arithmetic. The reference never meets it with a causal mask; with a
// sliding window it can (a partition wholly before the window). Such tiles
// are skipped here (m, l, O unchanged), as the CUDA kernel does.
void or_flash_decoding(const void* q, int qdt, const void* k, const void* v, int kvdt, void* out,
                       int odt, int64_t B, int64_t Nq, int64_t Nkv, int64_t Sk, int64_t kv_stride,
                       const int32_t* lens, int64_t Hd, int64_t P, float scale, int mask_kind,
                       int32_t window, float* pO, float* pM, float* pL) {
    const int64_t Bc = 128, SG = 4;
    std::vector<float> Ob(B * Nq * P * Hd), Mb(B * Nq * P), Lb(B * Nq * P);
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int64_t b = 0; b < B; ++b) {
        for (int64_t hq = 0; hq < Nq; ++hq) {
            int64_t len = lens ? int64_t(lens[b]) : Sk;
            int64_t hkv = hq * Nkv / Nq;
            int64_t qbase = (b * Nq + hq) * Hd;
            int64_t kvh = (b * Nkv + hkv) * kv_stride;
            std::vector<float> Qs(Hd), Os(Hd), S(Bc);
            int64_t posQ = len - 1;
            int64_t per = (len + P - 1) / P;
            for (int64_t part = 0; part < P; ++part) {
                int64_t jLo = part * per, jHi = std::min(jLo + per, len);
                for (int64_t d = 0; d < Hd; ++d) { Qs[d] = load(q, qdt, qbase + d) * scale; Os[d] = 0; }
                float m = -INFINITY, l = 0.0f;
                int64_t slot = (b * Nq + hq) * P + part;
                if (jLo > posQ) {
                    Mb[slot] = -INFINITY; Lb[slot] = 0;
                    for (int64_t d = 0; d < Hd; ++d) Ob[slot * Hd + d] = 0;
                    continue;
                }
                for (int64_t js = jLo; js < jHi; js += Bc) {
                    int64_t bc = std::min(Bc, jHi - js);
                    for (int64_t i = 0; i < bc; ++i) {
                        int64_t kk = js + i;
                        bool allowed = (mask_kind == 2) || (kk <= posQ);
                        if (mask_kind == 1) allowed = allowed && ((posQ - kk) < window);
                        float acc = -INFINITY;
                        if (allowed) {
                            float lanes[32];
                            int64_t kb = (kvh + kk) * Hd;
                            for (int ln = 0; ln < 32; ++ln) {
                                float part_ = 0.0f;
                                for (int64_t d = ln; d < Hd; d += 32) part_ += Qs[d] * load(k, kvdt, kb + d);
                                lanes[ln] = part_;
                            }
                            acc = simd_sum32(lanes);
                        }
                        S[i] = acc;
                    }
                    float tmax = -INFINITY;
                    for (int64_t i = 0; i < bc; ++i) tmax = std::max(tmax, S[i]);
                    if (tmax == -INFINITY) continue;  // fully masked tile (see header)
                    float m_new = std::max(m, tmax);
                    float scale_old = std::exp(m - m_new);
                    float psum = 0.0f;
                    for (int64_t i = 0; i < bc; ++i) { S[i] = std::exp(S[i] - m_new); psum += S[i]; }
                    l = scale_old * l + psum;
                    m = m_new;
                    for (int64_t d = 0; d < Hd; ++d) {
                        float acc = 0.0f;
                        for (int64_t i = 0; i < bc; ++i) acc += S[i] * load(v, kvdt, (kvh + js + i) * Hd + d);
                        Os[d] = scale_old * Os[d] + acc;
                    }
                }
                (void)SG;
                Mb[slot] = m; Lb[slot] = l;
                for (int64_t d = 0; d < Hd; ++d) Ob[slot * Hd + d] = Os[d];
            }
            // Reduce.
            int64_t pm = (b * Nq + hq) * P;
            float mg = -INFINITY;
            for (int64_t kx = 0; kx < P; ++kx) mg = std::max(mg, Mb[pm + kx]);
            float lg = 0.0f;
            for (int64_t kx = 0; kx < P; ++kx) lg += std::exp(Mb[pm + kx] - mg) * Lb[pm + kx];
            float inv_l = 1.0f / lg;
            for (int64_t d = 0; d < Hd; ++d) {
                float acc = 0.0f;
                for (int64_t kx = 0; kx < P; ++kx) acc += std::exp(Mb[pm + kx] - mg) * Ob[(pm + kx) * Hd + d];
                store(out, odt, qbase + d, acc * inv_l);
            }
        }
    }
    if (pO) std::memcpy(pO, Ob.data(), Ob.size() * 4);
    if (pM) std::memcpy(pM, Mb.data(), Mb.size() * 4);
    if (pL) std::memcpy(pL, Lb.data(), Lb.size() * 4);
}

// FlashAttention.metal:31-162: one pass per (b, hq, query row), Bc = 128,
// posQ = Sk - Sq + q, q pre-scaled, online softmax, final O / l.
void or_flash_attention(const void* q, int qdt, const void* k, const void* v, int kvdt, void* out,
                        int odt, int64_t B, int64_t Nq, int64_t Nkv, int64_t Sq, int64_t Sk,
                        int64_t Hd, float scale, int mask_kind, int32_t window) {
    const int64_t Bc = 128;
#pragma omp parallel for collapse(3) schedule(dynamic)
    for (int64_t b = 0; b < B; ++b)
        for (int64_t hq = 0; hq < Nq; ++hq)
            for (int64_t qi = 0; qi < Sq; ++qi) {
                int64_t hkv = hq * Nkv / Nq;
                int64_t qbase = ((b * Nq + hq) * Sq + qi) * Hd;
                int64_t kvh = (b * Nkv + hkv) * Sk;
                std::vector<float> Qs(Hd), Os(Hd, 0.0f), S(Bc);
                for (int64_t d = 0; d < Hd; ++d) Qs[d] = load(q, qdt, qbase + d) * scale;
                float m = -INFINITY, l = 0.0f;
                int64_t posQ = Sk - Sq + qi;
                for (int64_t js = 0; js < Sk; js += Bc) {
                    int64_t bc = std::min(Bc, Sk - js);
                    for (int64_t i = 0; i < bc; ++i) {
                        int64_t kk = js + i;
                        bool allowed = (mask_kind == 2) || (kk <= posQ);
                        if (mask_kind == 1) allowed = allowed && ((posQ - kk) < window);
                        float acc = -INFINITY;
                        if (allowed) {
                            float lanes[32];
                            int64_t kb = (kvh + kk) * Hd;
                            for (int ln = 0; ln < 32; ++ln) {
                                float p_ = 0.0f;
                                for (int64_t d = ln; d < Hd; d += 32) p_ += Qs[d] * load(k, kvdt, kb + d);
                                lanes[ln] = p_;
                            }
                            acc = simd_sum32(lanes);
                        }
                        S[i] = acc;
                    }
                    float tmax = -INFINITY;
                    for (int64_t i = 0; i < bc; ++i) tmax = std::max(tmax, S[i]);
                    if (tmax == -INFINITY) continue;
                    float m_new = std::max(m, tmax);
                    float so = std::exp(m - m_new);
                    float ps = 0.0f;
                    for (int64_t i = 0; i < bc; ++i) { S[i] = std::exp(S[i] - m_new); ps += S[i]; }
                    l = so * l + ps;
                    m = m_new;
                    for (int64_t d = 0; d < Hd; ++d) {
                        float acc = 0.0f;
                        for (int64_t i = 0; i < bc; ++i) acc += S[i] * load(v, kvdt, (kvh + js + i) * Hd + d);
                        Os[d] = so * Os[d] + acc;
                    }
                }
                float inv_l = 1.0f / l;
                for (int64_t d = 0; d < Hd; ++d) store(out, odt, qbase + d, Os[d] * inv_l);
            }
}

// Full-softmax attention in float64, the CPU reference of
// BidirectionalFATests.swift:9-53 generalised to GQA (hkv = hq*Nkv/Nq),
// Sq != Sk (posQ = Sk - Sq + q), the three mask kinds, a KV head stride
// `kv_stride` and optional per-sequence key counts `lens` (Sq must be 1 then).
// Output is float64 [B, Nq, Sq, Hd].
void or_attention_exact(const void* q, int qdt, const void* k, const void* v, int kvdt, double* out,
                        int64_t B, int64_t Nq, int64_t Nkv, int64_t Sq, int64_t Sk, int64_t kv_stride,
                        const int32_t* lens, int64_t Hd, float scale, int mask_kind, int32_t window) {
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int64_t b = 0; b < B; ++b)
        for (int64_t hq = 0; hq < Nq; ++hq) {
            int64_t len = lens ? int64_t(lens[b]) : Sk;
            int64_t hkv = hq * Nkv / Nq;
            int64_t kvh = (b * Nkv + hkv) * kv_stride;
            std::vector<double> s(len);
            for (int64_t qi = 0; qi < Sq; ++qi) {
                int64_t qbase = ((b * Nq + hq) * Sq + qi) * Hd;
                int64_t posQ = len - Sq + qi;
                double mx = -INFINITY;
                for (int64_t j = 0; j < len; ++j) {
                    bool allowed = (mask_kind == 2) || (j <= posQ);
                    if (mask_kind == 1) allowed = allowed && ((posQ - j) < window);
                    if (!allowed) { s[j] = -INFINITY; continue; }
                    double acc = 0.0;
                    for (int64_t d = 0; d < Hd; ++d)
                        acc += double(load(q, qdt, qbase + d)) * double(scale) * double(load(k, kvdt, (kvh + j) * Hd + d));
                    s[j] = acc;
                    mx = std::max(mx, acc);
                }
                double sum = 0.0;
                for (int64_t j = 0; j < len; ++j) { s[j] = (s[j] == -INFINITY) ? 0.0 : std::exp(s[j] - mx); sum += s[j]; }
                for (int64_t d = 0; d < Hd; ++d) {
                    double acc = 0.0;
                    for (int64_t j = 0; j < len; ++j) acc += s[j] * double(load(v, kvdt, (kvh + j) * Hd + d));
                    out[qbase + d] = acc / sum;
                }
            }
        }
}

// One decode layer at batch 1, composed from the ops above with the
// workspace-dtype rounding points of Examples/GemmaCLI/Sources/GemmaCLI/
// Gemma4TextInference.swift:312-436 (each op stores to the workspace dtype):
//
//   xn   = RMSNorm(x, w_attn_norm, 1+w)            -> dt
//   qkv  = W_qkv . xn  ([Nq+2Nkv]*Hd rows)          -> dt
//   KVCacheWrite(k, v -> caches at `pos`)
//   attn = FlashDecoding(q, caches, Sk = pos+1)    -> dt
//   o    = W_o . attn                              -> dt
//   h    = x + o                                   -> dt
//   hn   = RMSNorm(h, w_mlp_norm, 1+w)             -> dt
//   g    = W_gate . hn, u = W_up . hn              -> dt
//   a    = act(g) (GeluTanh, or SiLU when act==1)  -> dt
//   gu   = a * u                                   -> dt
//   d    = W_down . gu                             -> dt
//   out  = h + d                                   -> dt
//
// Weights are [out, in] (transposeB). Caches are [Nkv, Smax, Hd].
// Affine-quantized Matmul c = a . dequant(b)^T, b [N, K] 4-bit values packed
// little-endian in u32 words (value i in bits 4(i%8).. of word i/8, 
// AffineQuantizationFormat.swift:22-29), one scale / bias per 64 values of a
// row (AffineQuantizedTensor.swift:5-18). Routing and arithmetic of
// Matmul.swift:279-333: m == 1 follows aq_qmv_fast_typed
// (AffineQuantizedMatmul.metal:74-160: per lane 16 consecutive k, acc +=
// scale * sum(x q) + bias * sum(x), then the 32 lanes summed pairwise),
// m > 1 follows aq_matvec_simd4_typed (:9-69: per lane k = lane, lane+32 ..
// of each group, acc += x * (q * scale + bias)). biases NULL = no bias.
static float simd_sum32(const float* v) {
    float t[32];
    for (int i = 0; i < 32; ++i) t[i] = v[i];
    for (int s = 16; s > 0; s >>= 1)
        for (int i = 0; i < s; ++i) t[i] += t[i + s];
    return t[0];
}

void or_aq_matmul(const void* x, int xdt, const uint32_t* w, const void* scales, const void* biases, int sdt,
                  void* out, int odt, int64_t M, int64_t N, int64_t K) {
    const int64_t G = 64, kg = K / G, wpr = K / 8;
    auto q_at = [&](int64_t row, int64_t k) { return (w[row * wpr + k / 8] >> ((k % 8) * 4)) & 15u; };
#pragma omp parallel for schedule(static)
    for (int64_t mn = 0; mn < M * N; ++mn) {
        const int64_t m = mn / N, row = mn % N;
        float lanes[32] = {0};
        if (M == 1) {
            for (int64_t kb = 0; kb < K; kb += 512)
                for (int lane = 0; lane < 32; ++lane) {
                    const int64_t k0 = kb + lane * 16;
                    if (k0 >= K) continue;
                    float xv[16], sx = 0.f;
                    for (int j = 0; j < 16; ++j) {
                        xv[j] = k0 + j < K ? load(x, xdt, m * K + k0 + j) : 0.f;
                        sx += xv[j];
                    }
                    const int64_t g = k0 / G;
                    const float sc = load(scales, sdt, row * kg + g);
                    const float bi = biases ? load(biases, sdt, row * kg + g) : 0.f;
                    float qd = 0.f;
                    for (int j = 0; j < 16; ++j) qd += xv[j] * float(q_at(row, k0 + j));
                    lanes[lane] += sc * qd + bi * sx;
                }
        } else {
            for (int64_t g = 0; g < kg; ++g) {
                const float sc = load(scales, sdt, row * kg + g);
                const float bi = biases ? load(biases, sdt, row * kg + g) : 0.f;
                for (int lane = 0; lane < 32; ++lane)
                    for (int64_t i = lane; i < G; i += 32) {
                        const int64_t k = g * G + i;
                        lanes[lane] += load(x, xdt, m * K + k) * (float(q_at(row, k)) * sc + bi);
                    }
            }
        }
        store(out, odt, m * N + row, simd_sum32(lanes));
    }
}

// Exact (float64) dequantised product, for error budgeting.
void or_aq_matmul_exact(const void* x, int xdt, const uint32_t* w, const void* scales, const void* biases, int sdt,
                        double* out, int64_t M, int64_t N, int64_t K) {
    const int64_t kg = K / 64, wpr = K / 8;
    for (int64_t m = 0; m < M; ++m)
        for (int64_t row = 0; row < N; ++row) {
            double acc = 0.0;
            for (int64_t k = 0; k < K; ++k) {
                const double q = double((w[row * wpr + k / 8] >> ((k % 8) * 4)) & 15u);
                const double sc = load(scales, sdt, row * kg + k / 64);
                const double bi = biases ? load(biases, sdt, row * kg + k / 64) : 0.0;
                acc += double(load(x, xdt, m * K + k)) * (q * sc + bi);
            }
            out[m * N + row] = acc;
        }
}

// EmbeddingGather.metal:6-30: out[n, :] = table[ids[n], :] (converted).
void or_embedding_gather(const int32_t* ids, const void* table, int tdt, void* out, int odt, int64_t T, int64_t H) {
    for (int64_t n = 0; n < T; ++n)
        for (int64_t h = 0; h < H; ++h) store(out, odt, n * H + h, load(table, tdt, int64_t(ids[n]) * H + h));
}

// AffineQuantizedEmbeddingGather.metal:6-27: out[n, h] = q * scale + bias of
// row ids[n] (one rounding at the store).
void or_aq_embedding_gather(const int32_t* ids, const uint32_t* w, const void* scales, const void* biases, int sdt,
                            void* out, int odt, int64_t T, int64_t H) {
    const int64_t kg = H / 64, wpr = H / 8;
    for (int64_t n = 0; n < T; ++n) {
        const int64_t row = ids[n];
        for (int64_t h = 0; h < H; ++h) {
            const float sc = load(scales, sdt, row * kg + h / 64);
            const float bi = biases ? load(biases, sdt, row * kg + h / 64) : 0.f;
            const uint32_t q = (w[row * wpr + h / 8] >> ((h % 8) * 4)) & 15u;
            store(out, odt, n * H + h, float(q) * sc + bi);
        }
    }
}

void or_decode_layer(const void* x, int dt, const float* w_attn_norm, const float* w_mlp_norm,
                     const void* w_qkv, const void* w_o, const void* w_gate, const void* w_up,
                     const void* w_down, void* k_cache, void* v_cache, int64_t H, int64_t Nq,
                     int64_t Nkv, int64_t Hd, int64_t F, int64_t Smax, int64_t pos, float eps,
                     float attn_scale, int act, void* out, const float* q_norm, const float* k_norm,
                     int qk_norm, int norm_v, const float* rope_cos, const float* rope_sin) {
    auto el = [&](int64_t n) { return std::vector<uint8_t>(n * (dt == F32 ? 4 : 2)); };
    int64_t QKV = (Nq + 2 * Nkv) * Hd;
    auto xn = el(H), qkv = el(QKV), attn = el(Nq * Hd), o = el(H), h = el(H), hn = el(H);
    auto g = el(F), u = el(F), a = el(F), gu = el(F), dn = el(H);
    or_rmsnorm(x, dt, w_attn_norm, xn.data(), dt, 1, H, eps, 1, 0);
    or_matvec_nk(xn.data(), dt, w_qkv, dt, qkv.data(), dt, H, QKV);
    size_t es = dt == F32 ? 4 : 2;
    uint8_t* kp = qkv.data() + Nq * Hd * es;
    uint8_t* vp = qkv.data() + (Nq + Nkv) * Hd * es;
    // Gemma4TextInference.swift:352-381: per-head RMSNorm of q (q_norm) and k
    // (k_norm), of v without weight, then RoPE of q and k with the step's
    // table row; each result stored in dt (in place here: each op reads its
    // whole head before writing it).
    if (qk_norm) {
        or_rmsnorm(qkv.data(), dt, q_norm, qkv.data(), dt, Nq, Hd, eps, 1, 0);
        or_rmsnorm(kp, dt, k_norm, kp, dt, Nkv, Hd, eps, 1, 0);
        if (norm_v) or_rmsnorm(vp, dt, nullptr, vp, dt, Nkv, Hd, eps, 1, 0);
    }
    if (rope_cos) {
        or_rope_apply(qkv.data(), dt, rope_cos, rope_sin, F32, qkv.data(), dt, 1, 1, Nq, Hd / 2);
        or_rope_apply(kp, dt, rope_cos, rope_sin, F32, kp, dt, 1, 1, Nkv, Hd / 2);
    }
    or_kv_cache_write(kp, dt, k_cache, dt, 1, Nkv, 1, Smax, Hd, pos);
    or_kv_cache_write(vp, dt, v_cache, dt, 1, Nkv, 1, Smax, Hd, pos);
    int32_t len = int32_t(pos + 1);
    or_flash_decoding(qkv.data(), dt, k_cache, v_cache, dt, attn.data(), dt, 1, Nq, Nkv, len, Smax,
                      &len, Hd, 8, attn_scale, 0, -1, nullptr, nullptr, nullptr);
    or_matvec_nk(attn.data(), dt, w_o, dt, o.data(), dt, Nq * Hd, H);
    or_add(x, o.data(), h.data(), dt, H);
    or_rmsnorm(h.data(), dt, w_mlp_norm, hn.data(), dt, 1, H, eps, 1, 0);
    or_matvec_nk(hn.data(), dt, w_gate, dt, g.data(), dt, H, F);
    or_matvec_nk(hn.data(), dt, w_up, dt, u.data(), dt, H, F);
    if (act == 1) or_silu(g.data(), dt, a.data(), dt, F);
    else or_gelu_tanh(g.data(), dt, a.data(), dt, F);
    or_mul(a.data(), u.data(), gu.data(), dt, F);
    or_matvec_nk(gu.data(), dt, w_down, dt, dn.data(), dt, F, H);
    or_add(h.data(), dn.data(), out, dt, H);
}

}  // extern "C"
