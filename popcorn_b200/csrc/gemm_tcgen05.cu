// gemm_tcgen05.cu — tensor-core Matmul for sm_100a (5th-generation tensor
// cores: tcgen05.mma with TMEM accumulators, TMA-fed shared memory).
//
// Semantics: C[m,n] = sum_k A[m,k] * B[n,k] (transposeB, the linear-layer
// layout) or sum_k A[m,k] * B[k,n] (B not transposed: MN-major tiles), with
// fp32 accumulation and one rounding at the store — the
// product Matmul.metal:7-27 / MPPMatmul.metal:20-63 compute. A and B are
// both bf16 or both f16; C is f32 or the input type.
//
// Design (persistent, one CTA per SM, 128 x BN output tiles, BN = 256 for
// large N):
//  * warp 0 lane 0 issues TMA tiled loads (cp.async.bulk.tensor.2d, 128-B
//    swizzle, no multicast) of a 128 x 64 A tile and a BN x 64 B tile per
//    stage into a 4-stage ring (full/empty mbarriers);
//  * warp 1 lane 0 issues tcgen05.mma.cta_group::1.kind::f16 (M = 128,
//    N = BN, K = 16, four per stage) into one of two 128 x BN fp32
//    accumulators in tensor memory; tcgen05.commit releases each stage back
//    to the producer when its MMAs are done and then hands the accumulator
//    to the epilogue;
//  * warps 2-5 read the accumulator with tcgen05.ld, convert, stage 32 x 32
//    boxes in shared memory and store them with TMA (cp.async.bulk.tensor
//    store), while the MMAs of the next tile run into the other accumulator.
// Skinny problems (M <= 64, e.g. batched decode) run swapped: the weight
// matrix takes the 128-row MMA side and the activations the N side, and the
// epilogue writes the transpose.
//
// Every mbarrier wait is bounded; on give-up the CTA sets the error word,
// skips the rest of its work, frees its tensor memory and leaves.
#include <cuda.h>

#include <mutex>

#include <atomic>

#include "async.cuh"
#include "common.cuh"
#include "tcgen05.cuh"
#include "dtype.cuh"
#include "launch.hpp"
#include "peer_reduce.cuh"
#include "popcorn.hpp"

namespace popcorn {

__device__ unsigned int g_gemm_error_word;

namespace launch {

namespace {

using namespace tc;

constexpr int kBM = 128;
constexpr int kBK = 64;  // one 128-byte swizzle atom of 16-bit elements
// Operand ring depth: 4 stages; the skinny (decode-batch) tiles, whose
// stages are mostly weight bytes, stream with a deeper ring (6 stages of
// 16 + 4 KB: config-5 TP1 step 21.095 -> 21.04 ms; 8 stages 21.03).
constexpr int kSkinnyStages = 6;
template <int BN>
constexpr int gemm_stages() {
    return BN <= 64 ? kSkinnyStages : 4;
}

struct GemmArgs {
    void* c;
    int in_f16;           // 1: A/B are f16, 0: bf16
    int64_t M, N, K;      // of the MMA problem (swapped when `swap`)
    int64_t ldc;          // row stride of C in elements
    int swap;             // 1: MMA rows are C columns (C^T = B A^T)
    int tma_store;        // 1: C tiles leave through map_c
    int b_mn;             // 1: B is [K, N] (not transposed): MN-major tiles
    int ksplit;           // K partitions per output tile (1: none)
    float* ws;            // ksplit > 1: fp32 partial tiles [tiles][ksplit][BN][128]
    unsigned int* cnt;    // ksplit > 1: arrivals per tile (zero before the launch; left zero)
    int fuse_ar;          // 1: C is this rank's peer partial buffer; all-reduce + Add + RMSNorm follow
    PeerAllReduce ar;
};

// Persistent form: one CTA per SM walks output tiles t = blockIdx.x,
// blockIdx.x + gridDim.x, ... Warp 0 lane 0 loads (TMA), warp 1 lane 0
// multiplies (tcgen05.mma), warps 2-5 drain accumulators (tcgen05.ld, warp w
// owns TMEM lanes 32*(w%4)..+31). Two accumulators in tensor memory (2 x BN
// columns) let the epilogue of tile i overlap the MMAs of tile i+1.
constexpr int kEpiWarps = 4;
constexpr int kPersistThreads = (2 + kEpiWarps) * 32;

template <int BN, class CT>
__global__ void __launch_bounds__(kPersistThreads, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                        const __grid_constant__ CUtensorMap map_c, const GemmArgs g) {
    constexpr int A_BYTES = kBM * kBK * 2;
    constexpr int B_BYTES = BN * kBK * 2;
    constexpr int STAGE = A_BYTES + B_BYTES;
    constexpr uint32_t ACC_COLS = BN < 32 ? 32 : BN;
    constexpr uint32_t TMEM_COLS = 2 * ACC_COLS;
    constexpr int ES = int(sizeof(typename CT::storage));
    constexpr int BOX = 32 * 32 * ES;
    constexpr int kStages = gemm_stages<BN>();
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t full[kStages], empty[kStages], tfull[2], tempty[2];
    __shared__ uint32_t s_tmem;
    __shared__ volatile int s_abort;
    __shared__ int s_last;
    __shared__ unsigned int s_ar_epoch;
    __shared__ int s_ar_ok;
    __shared__ float s_red[kEpiWarps];

    pdl_launch_dependents();
    unsigned char* smem =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* staging = smem + size_t(kStages) * STAGE;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ktiles = int((g.K + kBK - 1) / kBK);
    const int ntm = int((g.M + kBM - 1) / kBM), ntn = int((g.N + BN - 1) / BN);
    const int ntiles = ntm * ntn;
    // Work units: (output tile, K partition). With split-K the partitions of
    // a tile run on different CTAs; the last to finish sums them in order.
    const int ks = g.ksplit;
    const int kps = (ktiles + ks - 1) / ks;  // K tiles per partition
    const int nunits = ntiles * ks;

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(smem_u32(&tfull[a]), 1);
            mbar_init(smem_u32(&tempty[a]), kEpiWarps);
        }
        s_abort = 0;
        mbar_fence_init();
    }
    if (warp == 0) tmem_alloc(smem_u32(&s_tmem), TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;

    pdl_wait();

    if (warp == 0) {
        if (lane == 0) {
            // ---- TMA producer ----
            int it = 0;
            for (int u = blockIdx.x; u < nunits && !s_abort; u += gridDim.x) {
                const int t = u / ks, kt0 = (u % ks) * kps;
                const int kt1 = kt0 + kps < ktiles ? kt0 + kps : ktiles;
                const int m0 = (t / ntn) * kBM, n0 = (t % ntn) * BN;
                for (int kt = kt0; kt < kt1; ++kt, ++it) {
                    const int s = it % kStages;
                    const uint32_t ph = uint32_t(it / kStages) & 1u;
                    if (s_abort || !mbar_wait(smem_u32(&empty[s]), ph ^ 1u, &g_gemm_error_word)) {
                        s_abort = 1;
                        break;
                    }
                    const uint32_t bar = smem_u32(&full[s]);
                    mbar_expect_tx(bar, STAGE);
                    unsigned char* st = smem + size_t(s) * STAGE;
                    tma_load_2d(smem_u32(st), &map_a, kt * kBK, m0, bar);
                    if (g.b_mn) {
                        // BN / 64 boxes of 64 N-columns x 64 K-rows
#pragma unroll
                        for (int j = 0; j < BN / 64; ++j)
                            tma_load_2d(smem_u32(st + A_BYTES + j * (kBK * 128)), &map_b, n0 + j * 64, kt * kBK, bar);
                    } else {
                        tma_load_2d(smem_u32(st + A_BYTES), &map_b, kt * kBK, n0, bar);
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- MMA issuer ----
            const uint32_t idesc = make_idesc(!g.in_f16, kBM, BN, g.b_mn != 0);
            int it = 0, lt = 0;
            for (int u = blockIdx.x; u < nunits && !s_abort; u += gridDim.x, ++lt) {
                const int kt0 = (u % ks) * kps;
                const int kt1 = kt0 + kps < ktiles ? kt0 + kps : ktiles;
                const int acc = lt & 1;
                if (!mbar_wait(smem_u32(&tempty[acc]), (uint32_t(lt >> 1) & 1u) ^ 1u, &g_gemm_error_word)) {
                    s_abort = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + uint32_t(acc) * ACC_COLS;
                for (int kt = kt0; kt < kt1; ++kt, ++it) {
                    const int s = it % kStages;
                    const uint32_t ph = uint32_t(it / kStages) & 1u;
                    if (s_abort || !mbar_wait(smem_u32(&full[s]), ph, &g_gemm_error_word)) {
                        s_abort = 1;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_base = smem_u32(smem + size_t(s) * STAGE);
                    const uint32_t b_base = a_base + A_BYTES;
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk) {
                        // K-major: the next 16 K-elements are 32 B further along the
                        // swizzled row; MN-major: 16 K-rows (2048 B) further
                        const uint64_t bd = g.b_mn ? smem_desc_sw128_mn(b_base + kk * 2048, kBK * 128)
                                                   : smem_desc_sw128(b_base + kk * 32);
                        tc_mma(d, smem_desc_sw128(a_base + kk * 32), bd, idesc, (kt > kt0 || kk > 0) ? 1u : 0u);
                    }
                    tc_commit(smem_u32(&empty[s]));
                }
                tc_commit(smem_u32(&tfull[acc]));
            }
        }
    } else {
        // ---- epilogue warps ----
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        unsigned int* own_ctl = g.fuse_ar ? g.ar.ctl[g.ar.rank] : nullptr;
        // A finished output tile of this rank's partial; the last one publishes
        // the partial to the peers (system-scope release of this call's epoch).
        auto tile_done = [&]() {
            __threadfence();
            const unsigned int old = atomicAdd(&own_ctl[kCtlTiles + g.ar.buffer], 1u);
            if (old == unsigned(ntiles) - 1) {
                own_ctl[kCtlTiles + g.ar.buffer] = 0u;
                __threadfence_system();
                pr_st_release_sys(&own_ctl[kCtlFlag + g.ar.buffer], s_ar_epoch);
            }
        };
        if (g.fuse_ar) {
            if (warp == 2 && lane == 0) s_ar_epoch = own_ctl[kCtlEpoch + g.ar.buffer] + 1u;
            named_sync(1, kEpiWarps * 32);
        }
        unsigned char* wbuf = staging + size_t(warp - 2) * BOX;
        int lt = 0;
        for (int u = blockIdx.x; u < nunits; u += gridDim.x, ++lt) {
            const int t = u / ks;
            const int m0 = (t / ntn) * kBM, n0 = (t % ntn) * BN;
            const int acc = lt & 1;
            if (s_abort || !mbar_wait(smem_u32(&tfull[acc]), uint32_t(lt >> 1) & 1u, &g_gemm_error_word)) {
                s_abort = 1;
                break;
            }
            tc_fence_after();
            const uint32_t src = tmem + uint32_t(acc) * ACC_COLS + (uint32_t(q * 32) << 16);
            const int64_t gr = int64_t(m0) + q * 32 + lane;
            if (ks > 1) {
                // fp32 partial tile -> workspace, column-major (lanes = rows: coalesced)
                float* wt = g.ws + (size_t(t) * ks + (u % ks)) * size_t(BN) * kBM;
#pragma unroll 1
                for (int c0 = 0; c0 < BN; c0 += 32) {
                    float v[32];
                    tmem_ld32(src + uint32_t(c0), v);
#pragma unroll
                    for (int j = 0; j < 32; ++j) wt[size_t(c0 + j) * kBM + q * 32 + lane] = v[j];
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&tempty[acc]));
                // the last partition of this tile to arrive sums all of them in order
                named_sync(1, kEpiWarps * 32);
                if (warp == 2 && lane == 0) {
                    __threadfence();
                    s_last = atomicAdd(&g.cnt[t], 1u) == unsigned(ks) - 1;
                }
                named_sync(1, kEpiWarps * 32);
                if (s_last) {
                    __threadfence();
                    const float* w0 = g.ws + size_t(t) * ks * size_t(BN) * kBM;
#pragma unroll 1
                    for (int c0 = 0; c0 < BN; c0 += 32) {
                        float v[32];
#pragma unroll
                        for (int j = 0; j < 32; ++j) v[j] = 0.f;
                        for (int sp = 0; sp < ks; ++sp) {
                            const float* wp = w0 + size_t(sp) * BN * kBM;
#pragma unroll
                            for (int j = 0; j < 32; ++j) v[j] += __ldcg(wp + size_t(c0 + j) * kBM + q * 32 + lane);
                        }
                        if (gr < g.M) {
                            // swapped problem: MMA row = output column gr
#pragma unroll
                            for (int j = 0; j < 32; ++j)
                                if (n0 + c0 + j < g.N) Elem<CT>::store(g.c, int64_t(n0 + c0 + j) * g.ldc + gr, v[j]);
                        }
                    }
                    named_sync(1, kEpiWarps * 32);
                    if (warp == 2 && lane == 0) {
                        g.cnt[t] = 0u;  // every partition has arrived
                        if (g.fuse_ar) tile_done();
                    }
                }
                continue;
            }
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 32) {
                float v[32];
                tmem_ld32(src + uint32_t(c0), v);
                if (g.tma_store) {
                    if (lane == 0) bulk_wait_read<0>();  // the buffer's previous store has read it
                    __syncwarp();
                    unsigned char* dst = wbuf + lane * 32 * ES;
                    if constexpr (ES == 4) {
#pragma unroll
                        for (int j = 0; j < 32; j += 4)
                            *reinterpret_cast<float4*>(dst + j * 4) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; j += 8)
                            *reinterpret_cast<uint4*>(dst + j * 2) =
                                make_uint4(pack2<CT>(v[j], v[j + 1]), pack2<CT>(v[j + 2], v[j + 3]),
                                           pack2<CT>(v[j + 4], v[j + 5]), pack2<CT>(v[j + 6], v[j + 7]));
                    }
                    fence_async_smem();
                    __syncwarp();
                    if (lane == 0 && n0 + c0 < g.N && m0 + q * 32 < g.M) {
                        tma_store_2d(&map_c, n0 + c0, m0 + q * 32, smem_u32(wbuf));
                        bulk_commit();
                    }
                } else if (gr < g.M) {
                    if (!g.swap) {
                        const int64_t base = gr * g.ldc + n0 + c0;
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (n0 + c0 + j < g.N) Elem<CT>::store(g.c, base + j, v[j]);
                    } else {
                        // MMA row = output column gr; MMA column = output row
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (n0 + c0 + j < g.N) Elem<CT>::store(g.c, int64_t(n0 + c0 + j) * g.ldc + gr, v[j]);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&tempty[acc]));
            if (g.fuse_ar) {
                named_sync(1, kEpiWarps * 32);  // all rows of the tile stored
                if (warp == 2 && lane == 0) tile_done();
            }
        }
        if (g.tma_store && lane == 0) bulk_wait_read<0>();
        if (g.fuse_ar) {
            // all-reduce of the rows, then Add + RMSNorm (rows spread over the CTAs)
            if (warp == 2 && lane == 0) s_ar_ok = pr_wait_peers(g.ar, s_ar_epoch, &g_gemm_error_word) ? 1 : 0;
            named_sync(1, kEpiWarps * 32);
            const bool ok = s_ar_ok != 0 && !s_abort;
            if constexpr (sizeof(typename CT::storage) == 2) {  // 16-bit partials only
                for (int64_t r = blockIdx.x; r < g.ar.rows; r += gridDim.x)
                    pr_reduce_row<CT, kEpiWarps * 32>(g.ar, r, ok, tid - 64, s_red,
                                                       [] { named_sync(1, kEpiWarps * 32); });
            }
        }
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, TMEM_COLS);
    if (g.fuse_ar && tid == 0) {
        // the last CTA out records this call's epoch for the buffer
        unsigned int* own_ctl = g.ar.ctl[g.ar.rank];
        __threadfence();
        if (atomicAdd(&own_ctl[kCtlExit], 1u) == gridDim.x - 1) {
            own_ctl[kCtlExit] = 0u;
            own_ctl[kCtlEpoch + g.ar.buffer] = s_ar_epoch;
            __threadfence();
        }
    }
}

// ---- host: tensor maps ----------------------------------------------------------

// Row-major [rows, cols] output map with a 32 x 32 box, no swizzle.
bool make_out_map(CUtensorMap* map, void* base, int dtype, int64_t rows, int64_t cols) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const int es = dtype == PC_F32 ? 4 : 2;
    cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
    cuuint64_t strides[1] = {cuuint64_t(cols) * es};
    cuuint32_t box[2] = {32, 32};
    cuuint32_t estr[2] = {1, 1};
    CUtensorMapDataType t = dtype == PC_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                            : dtype == PC_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                               : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    CUresult r = fn(map, t, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// 2-D K-major tensor map over rows x K (16-bit), box = box_rows x 64.
bool make_map(CUtensorMap* map, const void* base, int dtype, int64_t rows, int64_t K, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {cuuint64_t(K), cuuint64_t(rows)};
    cuuint64_t strides[1] = {cuuint64_t(K) * 2};
    cuuint32_t box[2] = {cuuint32_t(kBK), cuuint32_t(box_rows)};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, dtype == PC_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                    const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// 2-D MN-major tensor map over a [K, N] matrix (16-bit), box = 64 N x 64 K.
bool make_map_mn(CUtensorMap* map, const void* base, int dtype, int64_t K, int64_t N) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {cuuint64_t(N), cuuint64_t(K)};
    cuuint64_t strides[1] = {cuuint64_t(N) * 2};
    cuuint32_t box[2] = {64, cuuint32_t(kBK)};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, dtype == PC_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                    const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <int BN, class CT>
cudaError_t launch_bn(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const GemmArgs& g,
                      cudaStream_t s) {
    auto kern = gemm_tcgen05_kernel<BN, CT>;
    constexpr int kStages = gemm_stages<BN>();
    constexpr size_t smem = size_t(kStages) * (kBM * kBK * 2 + BN * kBK * 2) +
                            size_t(kEpiWarps) * 32 * 32 * sizeof(typename CT::storage) + 1024;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = allow_smem(kern, smem);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    const int64_t units = ((g.N + BN - 1) / BN) * ((g.M + kBM - 1) / kBM) * g.ksplit;
    const int sms = current_sm_count();
    dim3 grid(unsigned(units < sms ? units : sms));
    return launch_k(kern, grid, dim3(kPersistThreads), smem, s, ma, mb, mc, g);
}

template <class CT>
cudaError_t launch_ct(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, int bn, const GemmArgs& g,
                      cudaStream_t s) {
    switch (bn) {
    case 256: return launch_bn<256, CT>(ma, mb, mc, g, s);
    case 128: return launch_bn<128, CT>(ma, mb, mc, g, s);
    case 64: return launch_bn<64, CT>(ma, mb, mc, g, s);
    case 32: return launch_bn<32, CT>(ma, mb, mc, g, s);
    }
    return cudaErrorInvalidValue;
}

}  // namespace

// Served: A and B both bf16 or both f16, C f32 or the same type, K a
// multiple of 8 (16-byte row pitch for TMA), 16-byte aligned bases, and a
// problem big enough to use the tensor cores (M >= 16). transposeB (B
// [N, K]) at any such M; B [K, N] when M > 64 (unswapped) and N % 8 == 0.
bool tcgen05_supports(const Matmul& p) {
    bool types = (p.a_dtype == PC_BF16 || p.a_dtype == PC_F16) && p.b_dtype == p.a_dtype &&
                 (p.c_dtype == PC_F32 || p.c_dtype == p.a_dtype);
    bool layout = p.transpose_b || (p.M > 64 && p.N % 8 == 0 && p.N >= 64);
    return types && layout && p.M >= 16 && p.N >= 16 && p.K >= 16 && p.K % 8 == 0 && aligned16(p.a) &&
           aligned16(p.b) && p.M < (int64_t(1) << 31) && p.N < (int64_t(1) << 31) && encode_fn() != nullptr;
}

// Split-K for skinny (swapped) problems: a batched-decode GEMM has few
// 128-row weight tiles (e.g. 8 for N = 1024), so whole-K tiles would stream
// the weights from a handful of SMs. The partition count (each >= 4 K tiles)
// is chosen by the cost of its unit rounds (below). Returns the partition
// count (1: no split) and the output-tile count and width.
static int ksplit_plan(const Matmul& p, int64_t* tiles_out, int* bn_out) {
    if (p.M > 64) return 1;
    const int bn = p.M <= 32 ? 32 : 64;
    const int64_t tiles = ((p.N + kBM - 1) / kBM) * ((p.M + bn - 1) / bn);
    const int64_t ktiles = (p.K + kBK - 1) / kBK;
    const int sms = current_sm_count();
    if (tiles_out) *tiles_out = tiles;
    if (bn_out) *bn_out = bn;
    // Tiles that already cover half the SMs stream whole K (measured: a
    // split of the 224-tile gate/up GEMM at TP1 was slower).
    if (tiles * 2 > sms || ktiles < 8) return 1;
    // The partition count whose units finish soonest, in units of one K tile
    // of streaming: rounds of SM-sized unit batches times (the unit's K
    // tiles + its fp32 partial, about one K tile of bytes), plus the last
    // partition's read of all the partials. A count that leaves a partial
    // extra round costs a whole unit on the busiest SMs. Ties: fewer
    // partitions.
    int64_t best_ks = 1;
    double best = 1e30;
    for (int64_t ks = 1; ks <= ktiles / 4 && ks <= 64; ++ks) {
        const int64_t kps = (ktiles + ks - 1) / ks;
        const int64_t parts = (ktiles + kps - 1) / kps;  // no empty partition
        const int64_t rounds = (tiles * parts + sms - 1) / sms;
        const double t = parts == 1 ? double(rounds) * double(kps)
                                    : double(rounds) * double(kps + 1) + double(parts);
        if (t < best - 1e-9) {
            best = t;
            best_ks = parts;
        }
    }
    return int(best_ks);
}

size_t matmul_tcgen05_workspace(const Matmul& p) {
    int64_t tiles = 0;
    int bn = 0;
    const int ks = ksplit_plan(p, &tiles, &bn);
    if (ks <= 1) return 0;
    return size_t(tiles) * ks * bn * kBM * 4 + size_t(tiles) * 4;
}

static cudaError_t matmul_tcgen05_impl(const Matmul& p, const PeerAllReduce* ar, cudaStream_t s);

cudaError_t matmul_tcgen05(const Matmul& p, cudaStream_t s) { return matmul_tcgen05_impl(p, nullptr, s); }

// The skinny (swapped) form serves any 1 <= M <= 64: rows past M are the
// TMA's zero fill and are never stored.
bool tcgen05_supports_skinny(const Matmul& p) {
    Matmul q = p;
    q.M = 16;
    return p.M >= 1 && p.M <= 64 && p.transpose_b && tcgen05_supports(q);
}

// The skinny GEMM writing this rank's partial (p.c = its peer buffer), then
// the all-reduce + Add + RMSNorm of `ar` in the same kernel.
cudaError_t matmul_tcgen05_allreduce(const Matmul& p, const PeerAllReduce& ar, cudaStream_t s) {
    if (p.M > 64 || p.c_dtype != p.a_dtype || !peer_allreduce_supports(ar) || ar.rows != p.M || ar.H != p.N)
        return cudaErrorInvalidValue;
    return matmul_tcgen05_impl(p, &ar, s);
}

// Split-K arrival counters of Matmul objects: each object owns a range
// (gemm_reserve_counters). The last partition of a tile sets its counter
// back to zero, and the array starts zeroed, so launches need no memset in
// front of them (which would also end the programmatic overlap with the
// previous kernel). Launches of ONE object that overlap on the GPU (two
// streams, no ordering) would race on its range; a launch whose bounded
// wait gave up (device error word set) may leave its counters non-zero.
constexpr int kGemmCounters = 1 << 16;
__device__ unsigned int g_gemm_counters[kGemmCounters];

int gemm_reserve_counters(int64_t n) {
    static std::atomic<int64_t> next{0};
    if (n < 1 || n > kGemmCounters / 8) return -1;
    int64_t start = next.fetch_add(n) % kGemmCounters;
    if (start + n > kGemmCounters) start = 0;  // no range straddles the end
    return int(start);
}

// Device address of g_gemm_counters on the current device (looked up once).
static unsigned int* gemm_counters_here() {
    static std::mutex lock;
    static unsigned int* addr[64] = {nullptr};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        return nullptr;
    }
    std::lock_guard<std::mutex> guard(lock);
    if (!addr[dev]) {
        void* ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_gemm_counters) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        addr[dev] = static_cast<unsigned int*>(ptr);
    }
    return addr[dev];
}

static cudaError_t matmul_tcgen05_impl(const Matmul& p, const PeerAllReduce* ar, cudaStream_t s) {
    // Skinny M: swap so the weight rows fill the 128-row MMA side.
    const bool swap = p.M <= 64;
    GemmArgs g{};
    g.c = p.c;
    g.in_f16 = p.a_dtype == PC_F16 ? 1 : 0;
    g.K = p.K;
    g.ldc = p.N;
    g.swap = swap ? 1 : 0;
    const void* a = swap ? p.b : p.a;
    const void* b = swap ? p.a : p.b;
    g.M = swap ? p.N : p.M;
    g.N = swap ? p.M : p.N;
    int bn = swap ? (g.N <= 32 ? 32 : 64) : (g.N >= 256 ? 256 : 128);
    g.b_mn = p.transpose_b ? 0 : 1;  // supports() keeps B [K, N] unswapped
    CUtensorMap ma, mb, mc;
    const bool mb_ok = g.b_mn ? make_map_mn(&mb, b, p.a_dtype, p.K, g.N) : make_map(&mb, b, p.a_dtype, g.N, p.K, bn);
    if (!make_map(&ma, a, p.a_dtype, g.M, p.K, kBM) || !mb_ok) return cudaErrorInvalidValue;
    const int ces = p.c_dtype == PC_F32 ? 4 : 2;
    g.tma_store = (!swap && (p.N * ces) % 16 == 0 && aligned16(p.c) && make_out_map(&mc, p.c, p.c_dtype, p.M, p.N))
                      ? 1 : 0;
    if (!g.tma_store) mc = ma;  // unused
    g.ksplit = 1;
    if (ar) {
        g.fuse_ar = 1;
        g.ar = *ar;
    }
    if (p.workspace) {
        int64_t tiles = 0;
        const int ks = ksplit_plan(p, &tiles, nullptr);
        if (ks > 1) {
            g.ksplit = ks;
            g.ws = static_cast<float*>(p.workspace);
            unsigned int* own = p.ctr_base >= 0 && p.ctr_base + tiles <= kGemmCounters ? gemm_counters_here() : nullptr;
            if (own) {
                g.cnt = own + p.ctr_base;  // zero between launches
            } else {
                g.cnt = reinterpret_cast<unsigned int*>(static_cast<char*>(p.workspace) +
                                                        size_t(tiles) * ks * bn * kBM * 4);
                cudaError_t e = cudaMemsetAsync(g.cnt, 0, size_t(tiles) * 4, s);
                if (e != cudaSuccess) return e;
            }
        }
    }
    switch (p.c_dtype) {
    case PC_F32: return launch_ct<TF32>(ma, mb, mc, bn, g, s);
    case PC_BF16: return launch_ct<TBF16>(ma, mb, mc, bn, g, s);
    case PC_F16: return launch_ct<TF16>(ma, mb, mc, bn, g, s);
    }
    return cudaErrorInvalidValue;
}

uint32_t read_and_clear_gemm_errors() {
    unsigned int v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_gemm_error_word, sizeof(v)) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    if (v) cudaMemcpyToSymbol(g_gemm_error_word, &zero, sizeof(zero));
    return v;
}

namespace {
RegisterFunctions reg_gemm({
    {"matmul_tc_bf16_tb", reinterpret_cast<const void*>(gemm_tcgen05_kernel<256, TBF16>)},
    {"matmul_tc_f32out_tb", reinterpret_cast<const void*>(gemm_tcgen05_kernel<256, TF32>)},
    {"matmul_tc_f16_tb", reinterpret_cast<const void*>(gemm_tcgen05_kernel<256, TF16>)},
    {"matmul_tc_bf16_nn", reinterpret_cast<const void*>(gemm_tcgen05_kernel<256, TBF16>)},
});
}  // namespace

}  // namespace launch
}  // namespace popcorn
