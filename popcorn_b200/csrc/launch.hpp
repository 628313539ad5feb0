// launch.hpp — parameter blocks and launchers of the sm_100a kernels.
//
// Each launcher enqueues on `stream`, never synchronises and returns the
// CUDA launch status. Shapes have been validated by the kernel objects
// (ops.cu) before any launcher runs.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace popcorn {
namespace launch {

struct DeviceInfo {
    int device;
    int sm_count;
};
DeviceInfo device_info(int device);

// Up to two address ranges whose lines a kernel pulls into L2 once its own
// loads are issued (cp.async.bulk.prefetch.L2), so the next kernel of a
// chain finds its operands in L2. A hint only: it never changes results.
struct L2Prefetch {
    const void* ptr[2];
    uint64_t bytes[2];
};

// KVCacheWrite.metal:7-59 semantics. When pos_dev != nullptr the offset is
// read from device memory (*pos_dev) at run time.
struct KVWrite {
    const void* src;
    int src_dtype;
    void* cache;
    int cache_dtype;
    int64_t B, Nkv, Snew, Smax, Hd, offset;
    const int32_t* pos_dev;
};
cudaError_t kv_cache_write(const KVWrite& p, cudaStream_t stream);

// RMSNorm.metal:7-42 semantics; weight is f32 [H] or null.
struct RMSNorm {
    const void* x;
    int x_dtype;
    const float* weight;
    void* out;
    int out_dtype;
    int64_t rows, H;
    float eps;
    int add_one;
};
cudaError_t rmsnorm(const RMSNorm& p, cudaStream_t stream);

// Row-vector times weight matrix with optional fused prologue/epilogue.
//   y[n] = sum_k xin[k] * W[n,k]     (W [N,K] row-major, linear-layer layout)
// Prologue: xin = round(RMSNorm(x)) when norm_weight != null or has_norm.
// Epilogue kind:
//   kStore     out[n] = y[n]
//   kResidual  out[n] = round(round(y[n]) + residual[n])
//   kGated     out[n] = round(round(act(round(y_gate[n]))) * round(y_up[n]))
//   kQKV       rows [0, q_rows) -> q_out; the next kv_rows -> k_cache at
//              pos; the last kv_rows -> v_cache at pos
enum class Epilogue : int { kStore = 0, kResidual = 1, kGated = 2, kQKV = 3 };
struct Gemv {
    const void* x;
    int x_dtype;
    const void* w;   // gate for kGated
    const void* w2;  // up for kGated
    int w_dtype;
    void* out;
    int out_dtype;
    int64_t K, N;
    bool has_norm;
    const float* norm_weight;  // may be null with has_norm (no weight)
    float eps;
    int add_one;
    Epilogue epilogue;
    const void* residual;  // kResidual, out dtype
    int activation;        // kGated: 0 gelu_tanh, 1 silu
    // kQKV
    void* k_cache;
    void* v_cache;
    int64_t q_rows, kv_rows, Hd, Smax, offset;
    const int32_t* pos_dev;
    L2Prefetch pf;
    int pre_stages = 0;  // stages issued before the activation row is staged (0: the whole ring)
};
cudaError_t gemv(const Gemv& p, cudaStream_t stream);

// General C = A * B (or A * B^T), fp32 accumulation (Matmul.metal:7-27).
struct Matmul {
    const void* a;
    int a_dtype;
    const void* b;
    int b_dtype;
    void* c;
    int c_dtype;
    int64_t M, K, N;
    int transpose_b;
    void* workspace = nullptr;  // tcgen05 split-K partials (matmul_tcgen05_workspace bytes) or null
    int ctr_base = -1;          // split-K arrival counters reserved by gemm_reserve_counters (-1: zeroed per launch)
};
// Reserves `n` split-K arrival counters for one Matmul object; -1 when none.
int gemm_reserve_counters(int64_t n);
cudaError_t matmul(const Matmul& p, cudaStream_t stream);
// True when the tcgen05 tensor-core GEMM serves this problem.
bool matmul_uses_tensor_cores(const Matmul& p);
size_t matmul_tcgen05_workspace(const Matmul& p);

// Elementwise: GeluTanh / SiLU (unary) and Mul / Add (binary).
enum class Unary : int { kGeluTanh = 0, kSilu = 1, kScalarMul = 2 };
enum class Binary : int { kMul = 0, kAdd = 1 };
cudaError_t unary(Unary op, const void* x, int x_dtype, void* out, int out_dtype, int64_t count,
                  cudaStream_t stream, float scalar = 1.0f);
cudaError_t attention_mask_build(float* mask, int64_t Sq, int64_t Sk, int32_t window, cudaStream_t stream);
cudaError_t binary(Binary op, const void* a, const void* b, void* out, int dtype, int64_t count,
                   cudaStream_t stream);

// Split-KV decode attention (FlashDecoding.metal:29-231 semantics).
struct FlashDecode {
    const void* q;  // [B, Nq, 1, Hd]
    int q_dtype;
    const void* k;  // [B, Nkv, S, Hd]
    const void* v;
    int kv_dtype;
    void* out;  // [B, Nq, 1, Hd]
    int out_dtype;
    int64_t B, Nq, Nkv, S, Hd;
    const int32_t* seq_lens;  // [B] on device, or null: every sequence has S keys
    float scale;
    int mask_kind;
    int32_t window;
    L2Prefetch pf;
    int kv_early = 0;  // copy K/V tiles without the newest row before the dependency wait
};
struct FlashDecodePlan {
    int splits;
    int64_t chunk;        // keys per split
    int heads_per_cta;    // query heads sharing one K/V read
    bool fast;            // bulk-copy pipelined kernel (else generic)
    size_t scratch_o;     // bytes of partial O
    size_t scratch_ml;    // bytes of partial m (and of l)
};
FlashDecodePlan flash_decode_plan(const FlashDecode& p, int sm_count);
// Partial pass. partial_o [B,Nq,splits,Hd] f32, partial_m / partial_l
// [B,Nq,splits] f32 (log2 units). With one split it writes the output.
cudaError_t flash_decode(const FlashDecode& p, const FlashDecodePlan& plan, float* partial_o, float* partial_m,
                         float* partial_l, cudaStream_t stream);
// Log-sum-exp combine of the splits into the output (no-op for one split).
cudaError_t flash_decode_combine(const FlashDecode& p, const FlashDecodePlan& plan, const float* partial_o,
                                 const float* partial_m, const float* partial_l, cudaStream_t stream);

// Prefill attention (FlashAttention.metal:31-162 semantics), Sq >= 1.
struct FlashAttention {
    const void* q;  // [B, Nq, Sq, Hd]
    int q_dtype;
    const void* k;  // [B, Nkv, Sk, Hd]
    const void* v;
    int kv_dtype;
    void* out;
    int out_dtype;
    int64_t B, Nq, Nkv, Sq, Sk, Hd;
    float scale;
    int mask_kind;
    int32_t window;
};
cudaError_t flash_attention(const FlashAttention& p, cudaStream_t stream);
bool flash_attention_uses_tensor_cores(const FlashAttention& p);

// Batched-decode helpers (batched.cu).
struct QKVScatter {
    const void* qkv;  // [B, (Nq + 2 Nkv) * Hd]
    void* q;          // [B, Nq, 1, Hd]
    void* k_cache;    // [B, Nkv, Smax, Hd]
    void* v_cache;
    int dtype;
    int64_t B, Nq, Nkv, Hd, Smax, offset;
    const int32_t* pos_dev;  // when set, the position is read on the device
};
cudaError_t qkv_scatter(const QKVScatter& p, cudaStream_t stream);
cudaError_t gated_activation(const void* gate_up, void* out, int dtype, int64_t rows, int64_t F, int act,
                             cudaStream_t stream);
struct AddRMSNorm {
    const void* a;
    const void* b;
    void* sum_out;
    void* norm_out;
    const float* weight;
    int dtype;
    int64_t rows, H;
    float eps;
    int add_one;
};
cudaError_t add_rmsnorm(const AddRMSNorm& p, cudaStream_t stream);

// Rotary embedding and the decode step's per-head norms (rope.cu).
cudaError_t rope_build_cos_sin(const int32_t* positions, const float* inv_freq, float* cos_out, float* sin_out,
                               int64_t T, int64_t Hd2, float scaling, cudaStream_t stream);
struct RopeApply {
    const void* x;  // [B, T, Nh, 2 Hd2]
    const void* cos_t;  // [T, Hd2]
    const void* sin_t;
    void* out;
    int x_dtype, t_dtype, out_dtype;
    int64_t B, T, Nh, Hd2;
};
cudaError_t rope_apply(const RopeApply& p, cudaStream_t stream);
struct QKNormRope {
    void* q;        // [B, Nq, 1, Hd], in place
    void* k_cache;  // [B, Nkv, Smax, Hd]: the row at the position, in place
    void* v_cache;
    const float* q_norm;  // [Hd]
    const float* k_norm;  // [Hd]
    const float* cos_t;   // [table_rows, Hd/2] f32; row 0 when table_rows == 1, else the position's row
    const float* sin_t;
    int dtype;
    int64_t B, Nq, Nkv, Hd, Smax, offset, table_rows;
    const int32_t* pos_dev;  // when set, the position is read on the device
    float eps;
    int add_one, norm_v;
};
cudaError_t qk_norm_rope(const QKNormRope& p, cudaStream_t stream);

// Affine-quantized Matmul and the embedding gathers (aq_matmul.cu).
struct AqMatmul {
    const void* x;  // [M, K]
    int x_dtype;
    const uint32_t* w;   // [N, K/8] 4-bit values, little-endian in u32 words
    const void* scales;  // [N, K/64]
    const void* biases;  // [N, K/64] or NULL
    int s_dtype;
    void* out;  // [M, N]
    int out_dtype;
    int64_t M, N, K;
    int kslices;      // K groups split over CTAs when > 1 (aq_matmul_plan)
    int chunk_groups;  // K groups whose x is staged in shared memory at once (set at launch)
    int no_tma;        // force the register-fed form (tests)
    void* workspace;  // kslices > 1: aq_matmul_workspace bytes
    float* ws;
    unsigned int* cnt;
    // fused forms (TMA form only): RMSNorm of each x row first (norm_weight
    // f32 [K], NULL with norm = 1: no weight), and the epilogue
    int norm, add_one;
    const float* norm_weight;
    float eps;
    int epilogue;         // AqEpilogue
    const void* residual;  // kResidual: [M, N]
    int activation;        // kGated: 0 GeluTanh, 1 SiLU
    void* q_out;           // kQKV: q [M, Nq*Hd]; caches [M, Nkv, Smax, Hd]
    void* k_cache;
    void* v_cache;
    int64_t q_rows, kv_rows, Hd, Smax, offset;
    const int32_t* pos_dev;
};
enum AqEpilogue : int { kAqStore = 0, kAqResidual = 1, kAqGated = 2, kAqQKV = 3 };
struct AqTmaPlan {
    int ks;           // warps sharing a tile's K (1, 2, 4, 8, 16)
    int mt, mtiles;   // tokens staged per CTA, token tiles (grid z)
    size_t smem;
};
int aq_matmul_plan(const AqMatmul& p, int sm_count);
bool aq_tma_plan(const AqMatmul& p, AqTmaPlan& q);
size_t aq_matmul_workspace(const AqMatmul& p, int kslices);
cudaError_t aq_matmul(const AqMatmul& p, cudaStream_t stream);
struct EmbeddingGather {
    const int32_t* ids;  // [T]
    const void* table;   // dense [vocab, H]
    int table_dtype;     // dense: table dtype; quantized: scale dtype
    const uint32_t* packed;  // quantized table [vocab, H/8] (NULL: dense)
    const void* scales;
    const void* biases;
    void* out;  // [T, H]
    int out_dtype;
    int64_t T, H, vocab;
};
cudaError_t embedding_gather(const EmbeddingGather& p, cudaStream_t stream);

// Kernels.Argmax (argmax.cu).
struct Argmax {
    const void* x;  // [rows, N]
    int dtype;
    int32_t* out;   // [rows]
    int64_t rows, N;
    int chunks;     // two-pass form when > 1 (argmax_plan)
    int64_t chunk;
    float* part_v;  // [rows * chunks] scratch of the two-pass form
    int32_t* part_i;
};
void argmax_plan(Argmax& p, int sm_count);
cudaError_t argmax(const Argmax& p, cudaStream_t stream);

// One-shot all-reduce of tensor-parallel partial sums over peer memory,
// fused with the residual add and RMSNorm (allreduce.cu).
constexpr int kMaxPeers = 8;
struct PeerAllReduce {
    const void* partial[kMaxPeers][2];  // each rank's two partial buffers, as mapped here
    unsigned int* ctl[kMaxPeers];       // each rank's control block: flag[2], epoch[2], CTA count
    int rank, world, buffer;
    const void* residual;
    void* sum_out;
    void* norm_out;
    const float* weight;
    int dtype;
    int64_t rows, H;
    float eps;
    int add_one;
};
bool peer_allreduce_supports(const PeerAllReduce& p);
// tcgen05 skinny GEMM (M <= 64, transposeB) whose output is this rank's
// partial buffer, followed in the same kernel by the all-reduce + Add +
// RMSNorm of `ar` (rows = M, H = N).
cudaError_t matmul_tcgen05_allreduce(const Matmul& p, const PeerAllReduce& ar, cudaStream_t stream);
bool tcgen05_supports_skinny(const Matmul& p);
cudaError_t peer_allreduce_add_rmsnorm(const PeerAllReduce& p, cudaStream_t stream);

// One persistent kernel for a batch-1 decode step through a layer stack
// (decode_step.cu). `layers` points to device memory.
struct DecodeLayer {
    const void* w_qkv;
    const void* w_o;
    const void* w_gate;
    const void* w_up;
    const void* w_down;
    const float* attn_norm;
    const float* mlp_norm;
    void* k_cache;  // [Nkv, Smax, Hd]
    void* v_cache;
    const float* q_norm;  // [Hd] per-head norm weights (qk_norm), NULL = none
    const float* k_norm;
    const float* rope_cos;  // [rope_rows, Hd/2]; NULL = no RoPE
    const float* rope_sin;
};
struct DecodeStep {
    const DecodeLayer* layers;
    int L, H, Nq, Nkv, Hd, F, Smax;
    float eps, scale;
    int activation, add_one, dtype;
    void* x;   // [H] input; the output lands in x when L is even, else x2
    void* x2;
    void* h;
    void* q;
    void* attn;
    void* act;
    float* po;
    float* pm;
    float* pl;
    unsigned int* counters;  // L*6 + 1 op counters, then L*Nkv head counters; zero before the first launch; left zero
    const int32_t* pos;      // [1] on the device: position of the new token
    int splits, chunk_tiles;
    int rows[4], kc[4], nkc[4];  // per GEMV op: rows per tile, columns per stage, stages per tile
    int xs_bytes;
    int grid;
    int64_t l2_ahead;  // bytes of L2 prefetch the producer keeps ahead of its ring
    int qk_norm, norm_v;
    int has_rope;  // some layer has RoPE tables
    int64_t rope_rows;
};
bool decode_step_plan(DecodeStep& p, int sm_count);
size_t decode_step_workspace_bytes(const DecodeStep& p);
cudaError_t decode_step(const DecodeStep& p, cudaStream_t stream);

}  // namespace launch
}  // namespace popcorn
