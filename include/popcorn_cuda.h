/*
 * popcorn_cuda.h — C ABI of the B200 (sm_100a) decode-step kernel library.
 *
 * This is the drop-in boundary for finnvoor/Popcorn's decode path. A Swift
 * module (module.modulemap over this header) re-backs Popcorn's public types
 * with these calls; every entry point below names the reference interface
 * it replaces (paths are inside the finnvoor/Popcorn source tree).
 *
 * Conventions
 *  - Every function that can fail returns an int status: 0 (PC_OK) or one
 *    of the negative PopcornError.Code values (Sources/Popcorn/
 *    PopcornError.swift:23-42). The message of the last failure on the
 *    calling thread is pc_last_error_message().
 *  - Validation happens when a kernel object is created, before anything is
 *    launched, as the reference's throwing initialisers do.
 *  - The library never frees or retains caller memory. Tensors are plain
 *    descriptors over caller-owned device pointers, bound at offset 0 with
 *    contiguous row-major layout (Sources/Popcorn/Tensor.swift:5-22).
 *  - Scratch memory always comes from the caller's allocator callbacks.
 *  - Streams are cudaStream_t passed as void*; the library enqueues on the
 *    caller's stream and never synchronises it (the caller owns submission,
 *    as the Metal caller owns the command buffer).
 */
#ifndef POPCORN_CUDA_H
#define POPCORN_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PC_API __attribute__((visibility("default")))
#define PC_MAX_RANK 8

/* PopcornError.Code, Sources/Popcorn/PopcornError.swift:23-42. */
typedef enum pc_status {
    PC_OK = 0,
    PC_ERR_CONSTANT_ALLOCATION_FAILED = -1001,
    PC_ERR_TENSOR_ALLOCATION_FAILED = -1003,
    PC_ERR_KERNEL_FUNCTION_NOT_FOUND = -1006,
    PC_ERR_TENSOR_SHAPE_MISMATCH = -1007,
    PC_ERR_TENSOR_INVALID_RANK = -1008,
    PC_ERR_TENSOR_INVALID_AXIS = -1009,
    PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION = -1010,
    PC_ERR_WORKSPACE_EXHAUSTED = -1012,
    PC_ERR_GPU_OUT_OF_MEMORY = -1013,
    PC_ERR_GPU_TIMEOUT = -1014,
    PC_ERR_GPU_PAGE_FAULT = -1015,
    PC_ERR_GPU_INVALID_RESOURCE = -1016,
    PC_ERR_GPU_DEVICE_REMOVED = -1017,
    PC_ERR_GPU_ACCESS_REVOKED = -1018,
    PC_ERR_GPU_INTERNAL = -1019
} pc_status;

/* Tensor.DataType, Sources/Popcorn/Tensor.swift:135-148 (same order). */
typedef enum pc_dtype {
    PC_U8 = 0, PC_U16 = 1, PC_U32 = 2, PC_U64 = 3,
    PC_I8 = 4, PC_I16 = 5, PC_I32 = 6, PC_I64 = 7,
    PC_F32 = 8, PC_F16 = 9, PC_BF16 = 10
} pc_dtype;

/* Tensor {buffer, shape, dataType}, Sources/Popcorn/Tensor.swift:5-22. */
typedef struct pc_tensor {
    void* data;      /* device pointer, bound at offset 0 */
    int32_t dtype;   /* pc_dtype */
    int32_t rank;    /* 0..PC_MAX_RANK */
    int64_t shape[PC_MAX_RANK];
} pc_tensor;

/* Tensor.Access, Sources/Popcorn/Tensor.swift:182-199. */
typedef enum pc_access { PC_ACCESS_READ = 1, PC_ACCESS_WRITE = 2, PC_ACCESS_READ_WRITE = 3 } pc_access;

/* AttentionMask, Sources/Popcorn/Kernels/AttentionMask.swift:17-41. */
typedef enum pc_mask_kind {
    PC_MASK_CAUSAL = 0,
    PC_MASK_CAUSAL_SLIDING_WINDOW = 1,
    PC_MASK_BIDIRECTIONAL = 2
} pc_mask_kind;
typedef struct pc_attention_mask {
    int32_t kind;    /* pc_mask_kind */
    int32_t window;  /* sliding-window length; -1 when unused */
} pc_attention_mask;

/* ---- errors, sizes ------------------------------------------------------ */

/* Message of the last failing call on this thread (PopcornError
 * .errorDescription, PopcornError.swift:44-58). Never NULL. */
PC_API const char* pc_last_error_message(void);
/* Tensor.DataType.stride, Tensor.swift:152-159; 0 for an unknown dtype. */
PC_API int pc_dtype_stride(int32_t dtype);
/* ScratchSpec.byteCount = max(1, prod(shape) * stride), ScratchSpec.swift:23-25. */
PC_API int64_t pc_scratch_spec_byte_count(const int64_t* shape, int32_t rank, int32_t dtype);
/* Library version (major*10000 + minor*100 + patch). */
PC_API int pc_version(void);

/* ---- device memory (MTLDevice.makeBuffer counterpart for C callers) ----- */

PC_API int pc_device_count(int* count);
PC_API int pc_buffer_alloc(int device, size_t bytes, void** ptr);
PC_API int pc_buffer_free(void* ptr);
PC_API int pc_memcpy_htod_async(void* dst, const void* src, size_t bytes, void* stream);
PC_API int pc_memcpy_dtoh_async(void* dst, const void* src, size_t bytes, void* stream);
PC_API int pc_stream_synchronize(void* stream);
/* Reads and clears the device-side error word of `device` (bit 0: a bounded
 * wait inside a kernel gave up; bit 1: a decode position outside the cache;
 * bit 4: an embedding id outside the table). 0 when clean. Synchronises the
 * device. */
PC_API int pc_device_error_check(int device, uint32_t* flags);

/* ---- KernelLibrary (Sources/Popcorn/KernelLibrary.swift:4-41) ----------- */

typedef struct pc_library pc_library;
/* KernelLibrary(device:), KernelLibrary.swift:7-14. */
PC_API int pc_library_create(int device, pc_library** out);
PC_API void pc_library_destroy(pc_library* library);
/* KernelLibrary.device, KernelLibrary.swift:18. */
PC_API int pc_library_device(const pc_library* library, int* device);
/* KernelLibrary.pipelineState(for:), KernelLibrary.swift:20-41: the same
 * name always yields the same handle (cache identity); unknown names fail
 * with PC_ERR_KERNEL_FUNCTION_NOT_FOUND (-1006). Thread-safe. */
PC_API int pc_library_lookup(pc_library* library, const char* function_name, const void** handle);
PC_API int pc_library_function_count(const pc_library* library);
PC_API const char* pc_library_function_name(const pc_library* library, int index);

/* ---- scratch protocol (Sources/Popcorn/KernelResources.swift:5-36) ------ */

/* KernelScratchAllocator.borrowTemporaryBuffer(length:) / release. borrow
 * returns 0 and a device pointer of at least `length` bytes, and sets
 * *was_reused when the buffer may hold earlier writes in the same encoder
 * (KernelTemporaryBuffer.wasReused, KernelResources.swift:14-20). A
 * non-zero return aborts the encode with that status. release may be NULL;
 * it runs when the composite kernel finishes encoding, before the GPU has
 * run it — stream order protects reuse by later work on the same stream. */
typedef struct pc_scratch_allocator {
    void* ctx;
    int (*borrow)(void* ctx, size_t length, void** ptr, int* was_reused);
    void (*release)(void* ctx, void* ptr);
} pc_scratch_allocator;

/* ---- KernelCommandEncoder (Sources/Popcorn/KernelCommandEncoder.swift) --- */

typedef struct pc_encoder pc_encoder;
typedef struct pc_kernel pc_kernel;

/* Phase of a dispatch hook call: Metal4DispatchPhase, KernelCommandEncoder.swift:243-246. */
typedef enum pc_dispatch_phase { PC_WILL_DISPATCH = 0, PC_DID_DISPATCH = 1 } pc_dispatch_phase;
typedef void (*pc_dispatch_hook)(void* ctx, const char* function_name, int phase, void* stream);

/* KernelCommandEncoder(compute:library:scratch:), KernelCommandEncoder.swift:8-16.
 * `stream` is a cudaStream_t (NULL = legacy default stream). `scratch` is
 * copied; it may be NULL when only non-composite kernels are encoded. */
PC_API int pc_encoder_create(pc_library* library, void* stream, const pc_scratch_allocator* scratch,
                             pc_encoder** out);
PC_API void pc_encoder_destroy(pc_encoder* encoder);
/* encode(_:), KernelCommandEncoder.swift:39-47. */
PC_API int pc_encoder_encode(pc_encoder* encoder, const pc_kernel* kernel);
/* barrier(), KernelCommandEncoder.swift:71-85: clears the access map. On one
 * CUDA stream launches are already ordered, so no GPU work is enqueued. */
PC_API int pc_encoder_barrier(pc_encoder* encoder);
/* Barriers inserted so far (explicit + hazard-driven, :155-168). */
PC_API int64_t pc_encoder_barrier_count(const pc_encoder* encoder);
/* Kernel launches enqueued so far. */
PC_API int64_t pc_encoder_dispatch_count(const pc_encoder* encoder);
/* metal4DispatchHook, KernelCommandEncoder.swift:29-37,237-239. */
PC_API int pc_encoder_set_dispatch_hook(pc_encoder* encoder, pc_dispatch_hook hook, void* ctx);
PC_API int pc_encoder_stream(const pc_encoder* encoder, void** stream);

/* ---- kernel objects (Sources/Popcorn/Kernel.swift:15-70) ----------------- */

PC_API void pc_kernel_destroy(pc_kernel* kernel);
/* Operation name ("FlashAttention", "KVCacheWrite", ...). */
PC_API const char* pc_kernel_name(const pc_kernel* kernel);
/* Kernel.tensors, Kernel.swift:17-19: the user-visible bindings. */
PC_API int pc_kernel_binding_count(const pc_kernel* kernel);
PC_API int pc_kernel_binding(const pc_kernel* kernel, int index, pc_tensor* tensor, int* access);
/* Function names this kernel will launch, ';'-separated (route visible). */
PC_API const char* pc_kernel_function_names(const pc_kernel* kernel);

/* Extension (no reference counterpart): an L2 prefetch hint for the kernels
 * that stream their operands from HBM (decode FlashAttention, the m == 1
 * Matmul and the fused decode ops). Once the kernel has issued its own
 * loads, its CTAs pull [ptr, ptr + bytes) into L2 — typically the next
 * kernel's weights or KV cache — so that a chain of dependent kernels keeps
 * HBM busy across kernel boundaries. Two slots (0, 1); bytes 0 clears a
 * slot. Results never change. Other kernels return
 * PC_ERR_KERNEL_FUNCTION_NOT_FOUND. */
PC_API int pc_kernel_set_l2_prefetch(pc_kernel* kernel, int32_t slot, const void* ptr, uint64_t bytes);

/* Extension (no reference counterpart): scheduling hints. Results never
 * change.
 *  - PC_HINT_KV_EARLY (decode FlashAttention, value 0 or 1): the caller
 *    promises that the kernel enqueued just before this one writes neither
 *    seq_lens nor any K/V row except the newest of each sequence (the decode
 *    step's KV write). The attention then copies every K/V tile that holds
 *    no newest row while the previous kernel drains (before its dependency
 *    wait); the tile with the newest row is copied after the wait.
 * Other kernels / hints return PC_ERR_KERNEL_FUNCTION_NOT_FOUND. */
typedef enum pc_kernel_hint { PC_HINT_KV_EARLY = 2 } pc_kernel_hint;
PC_API int pc_kernel_set_hint(pc_kernel* kernel, int32_t hint, int64_t value);

/* FlashAttention.Path, FlashAttention.swift:94-98 + route(sq:hd:supportsMPP:)
 * :109-113. On B200 the tensor-core prefill kernel plays the MPP role. */
typedef enum pc_attention_path { PC_PATH_PLAIN = 0, PC_PATH_TENSOR = 1, PC_PATH_DECODING = 2 } pc_attention_path;
PC_API int pc_flash_attention_route(int64_t query_len, int64_t head_dim, int32_t dtype);

/* Kernels.FlashAttention(q:k:v:into:scale:mask:), FlashAttention.swift:51-90.
 * q [B,Nq,Sq,Hd], k/v [B,Nkv,Sk,Hd], out [B,Nq,Sq,Hd]. Sq == 1 routes to
 * split-KV FlashDecoding (FlashDecoding.swift:6-90), which borrows its
 * partial (m, l, O) scratch from the encoder's allocator. */
PC_API int pc_kernel_flash_attention(const pc_tensor* q, const pc_tensor* k, const pc_tensor* v,
                                     const pc_tensor* out, float scale, pc_attention_mask mask,
                                     pc_kernel** kernel);
/* Explicit-dimension form, FlashAttention.swift:13-49. */
PC_API int pc_kernel_flash_attention_dims(const pc_tensor* q, const pc_tensor* k, const pc_tensor* v,
                                          const pc_tensor* out, int64_t batch, int64_t query_heads,
                                          int64_t kv_heads, int64_t query_len, int64_t key_len,
                                          int64_t head_dim, float scale, pc_attention_mask mask,
                                          pc_kernel** kernel);
/* Extension (no reference counterpart; the reference shares Sk across the
 * batch, FlashDecoding.metal:55-58): decode attention over a KV cache
 * [B,Nkv,Smax,Hd] with per-sequence key counts seq_lens (int32 [B] on the
 * device, 0 <= len <= Smax). Equals FlashDecoding run per sequence on the
 * compact slice [1,Nkv,len,Hd] with the query at position len-1. A
 * sequence with len 0 yields zeros. The kernels clamp each len to
 * [0, Smax] on the device, so a value outside the contract never reads
 * past the cache. */
PC_API int pc_kernel_flash_decoding_ragged(const pc_tensor* q, const pc_tensor* k_cache,
                                           const pc_tensor* v_cache, const pc_tensor* seq_lens,
                                           const pc_tensor* out, float scale, pc_attention_mask mask,
                                           pc_kernel** kernel);

/* Kernels.KVCacheWrite(source:cache:offset:), KVCacheWrite.swift:38-49.
 * source [B,Nkv,Snew,Hd] into cache [B,Nkv,Smax,Hd] at `offset`.
 * Dtypes (source, cache): f32/f32, bf16/bf16, f32/bf16 (reference), f16/f16
 * (extension). Bit-exact copy, or RNE for f32 -> bf16. */
PC_API int pc_kernel_kv_cache_write(const pc_tensor* source, const pc_tensor* cache, int64_t offset,
                                    pc_kernel** kernel);
/* Explicit-dimension form, KVCacheWrite.swift:8-36. */
PC_API int pc_kernel_kv_cache_write_dims(const pc_tensor* source, const pc_tensor* cache, int64_t batch,
                                         int64_t kv_heads, int64_t new_len, int64_t max_len,
                                         int64_t head_dim, int64_t offset, pc_kernel** kernel);

/* Kernels.RMSNorm(_:weight:into:axis:eps:addOneToWeight:), RMSNorm.swift:39-70.
 * weight may be NULL; when present it is f32 [H] (RMSNorm.metal:44-46). */
PC_API int pc_kernel_rmsnorm(const pc_tensor* x, const pc_tensor* weight, const pc_tensor* out, int32_t axis,
                             float eps, int32_t add_one_to_weight, pc_kernel** kernel);
/* Explicit-dimension form, RMSNorm.swift:10-37. */
PC_API int pc_kernel_rmsnorm_dims(const pc_tensor* x, const pc_tensor* weight, const pc_tensor* out,
                                  int64_t row_count, int64_t hidden_size, float eps,
                                  int32_t add_one_to_weight, pc_kernel** kernel);

/* Kernels.Matmul(_:_:into:transposeB:), Matmul.swift:68-93. a [M,K],
 * b [N,K] (transposeB) or [K,N], c [M,N]. M == 1 routes to the matvec
 * (Matmul.swift:22-32). */
PC_API int pc_kernel_matmul(const pc_tensor* a, const pc_tensor* b, const pc_tensor* c, int32_t transpose_b,
                            pc_kernel** kernel);
/* Explicit-dimension form, Matmul.swift:9-66. */
PC_API int pc_kernel_matmul_dims(const pc_tensor* a, const pc_tensor* b, const pc_tensor* c, int64_t m,
                                 int64_t k, int64_t n, int32_t transpose_b, pc_kernel** kernel);

/* Kernels.GeluTanh(_:into:), GeluTanh.swift:8-26. */
PC_API int pc_kernel_gelu_tanh(const pc_tensor* x, const pc_tensor* out, pc_kernel** kernel);
/* Kernels.Mul(_:_:into:), Mul.swift. */
PC_API int pc_kernel_mul(const pc_tensor* a, const pc_tensor* b, const pc_tensor* out, pc_kernel** kernel);
/* Kernels.Add(_:_:into:), Add.swift. */
PC_API int pc_kernel_add(const pc_tensor* a, const pc_tensor* b, const pc_tensor* out, pc_kernel** kernel);
/* Kernels.Argmax(_:indices:axis:), Argmax.swift:24-37 (axis -1 only): int32
 * index of the largest element of each row, ties to the lowest index, NaN
 * never wins (Argmax.metal:7-76). x f32 (reference); f16 / bf16 are an
 * extension (compared as their exact f32 values). Long rows use caller
 * scratch for their partial winners. */
PC_API int pc_kernel_argmax(const pc_tensor* x, const pc_tensor* indices, int32_t axis, pc_kernel** kernel);
/* Kernels.AttentionMaskBuild(mask:slidingWindow:) (AttentionMaskBuild.swift,
 * AttentionMaskBuild.metal:5-21): f32 mask [Sq, Sk], 0 where query i (at key
 * position Sk - Sq + i) may attend key j (causal, and within the window
 * when sliding_window >= 0), -inf elsewhere. sliding_window < 0: none. */
PC_API int pc_kernel_attention_mask_build(const pc_tensor* mask, int32_t sliding_window, pc_kernel** kernel);
/* Kernels.ScalarMul(_:by:into:) (ScalarMul.swift, ScalarMul.metal:6-25):
 * out = x * scalar, f32 / f16 / bf16, out of x's shape and dtype. */
PC_API int pc_kernel_scalar_mul(const pc_tensor* x, float scalar, const pc_tensor* out, pc_kernel** kernel);
/* Extension: SiLU, silu(g) = g / (1 + exp(-g)) (no reference kernel). */
PC_API int pc_kernel_silu(const pc_tensor* x, const pc_tensor* out, pc_kernel** kernel);

/* ---- fused decode ops (extensions; each equals a reference op sequence) -- */

/* out = Matmul(RMSNorm(x, norm_weight, eps, add_one), w, transposeB) for
 * x [1,K]: the RMSNorm output is rounded to x's dtype before the product,
 * as the unfused pair stores it (RMSNorm.metal:36, Matvec.metal:92). */
PC_API int pc_kernel_rmsnorm_matmul(const pc_tensor* x, const pc_tensor* norm_weight, float eps,
                                    int32_t add_one_to_weight, const pc_tensor* w, const pc_tensor* out,
                                    pc_kernel** kernel);
/* Gated MLP up half: out = act(W_gate xn) * (W_up xn), xn = RMSNorm(x) when
 * norm_weight is given (else xn = x), with each intermediate rounded to the
 * activation dtype as GeluTanh/Mul store them (Gemma4TextInference.swift:
 * 424-429). act: 0 = GeluTanh (GeGLU), 1 = SiLU (SwiGLU). x [1,K],
 * w_gate/w_up [F,K], out [1,F]. */
typedef enum pc_activation { PC_ACT_GELU_TANH = 0, PC_ACT_SILU = 1 } pc_activation;
PC_API int pc_kernel_gated_mlp(const pc_tensor* x, const pc_tensor* norm_weight, float eps,
                               int32_t add_one_to_weight, const pc_tensor* w_gate, const pc_tensor* w_up,
                               int32_t activation, const pc_tensor* out, pc_kernel** kernel);
/* out = residual + Matmul(a, w, transposeB) for a [1,K]: the product is
 * rounded to the output dtype before the add, as Matmul then Add store it
 * (Gemma4TextInference.swift:401-404, 431-434). */
PC_API int pc_kernel_matmul_residual(const pc_tensor* a, const pc_tensor* w, const pc_tensor* residual,
                                     const pc_tensor* out, pc_kernel** kernel);
/* QKV projection of one decode token with the KV-cache write fused:
 * qkv = Matmul(RMSNorm(x), w_qkv) for w_qkv [(Nq+2Nkv)*Hd, K]; the q part
 * goes to q_out [1,Nq,1,Hd]; the k and v parts are written to the caches
 * [1,Nkv,Smax,Hd] at position `offset`, exactly as KVCacheWrite would
 * store them (KVCacheWrite.metal:17-26). The position is `offset`, or, when
 * `position` (int32 [1] on the device) is given, the value it holds when the
 * kernel runs — so one captured CUDA graph can serve every decode step. */
PC_API int pc_kernel_qkv_projection(const pc_tensor* x, const pc_tensor* norm_weight, float eps,
                                    int32_t add_one_to_weight, const pc_tensor* w_qkv, const pc_tensor* q_out,
                                    const pc_tensor* k_cache, const pc_tensor* v_cache, int64_t offset,
                                    const pc_tensor* position, pc_kernel** kernel);

/* ---- batched-decode helpers (extensions; each equals a reference op
 * sequence) ------------------------------------------------------------ */

/* Splits qkv [B, (Nq+2*Nkv)*Hd] (ONE Matmul against the concatenated
 * [W_q; W_k; W_v]) into q_out [B,Nq,1,Hd] and the new key / value rows,
 * written to k_cache / v_cache [B,Nkv,Smax,Hd] at `offset` (or at the int32
 * held by `position` on the device when given) exactly as KVCacheWrite
 * stores them (KVCacheWrite.metal:17-26). Same dtype everywhere; a bit-exact
 * copy. Hd * element size must be a multiple of 16 bytes. */
PC_API int pc_kernel_qkv_scatter(const pc_tensor* qkv, const pc_tensor* q_out, const pc_tensor* k_cache,
                                 const pc_tensor* v_cache, int64_t offset, const pc_tensor* position,
                                 pc_kernel** kernel);
/* out [rows,F] = round(act(g)) * u for gate_up [rows,2F] (g = columns 0..F-1,
 * u = F..2F-1: ONE Matmul against [W_gate; W_up]) — GeluTanh (or SiLU) then
 * Mul (GeluTanh.metal:6-35, Mul.metal:7-25). */
PC_API int pc_kernel_gated_activation(const pc_tensor* gate_up, int32_t activation, const pc_tensor* out,
                                      pc_kernel** kernel);
/* sum_out = a + b (Add.metal), then norm_out = RMSNorm(sum_out, norm_weight,
 * eps, add_one) (RMSNorm.metal:7-42) over the last axis; both stored. */
PC_API int pc_kernel_add_rmsnorm(const pc_tensor* a, const pc_tensor* b, const pc_tensor* norm_weight, float eps,
                                 int32_t add_one_to_weight, const pc_tensor* sum_out, const pc_tensor* norm_out,
                                 pc_kernel** kernel);

/* ---- rotary position embedding ------------------------------------------ */

/* Kernels.RopeBuildCosSin (RopeBuildCosSin.swift:31-50, RopeBuildCosSin.metal:
 * 5-21): cos_out / sin_out [T, Hd/2] f32 = cos / sin(positions[t] *
 * inv_freq[i]) * attention_scaling; positions int32 [T], inv_freq f32 [Hd/2]. */
PC_API int pc_kernel_rope_build_cos_sin(const pc_tensor* positions, const pc_tensor* inv_freq,
                                        const pc_tensor* cos_out, const pc_tensor* sin_out, float attention_scaling,
                                        pc_kernel** kernel);
/* Kernels.RopeApply (RopeApply.swift:48-64, RopeApply.metal:6-49): rotate-half
 * RoPE of x [B, T, Nh, Hd] with tables [T, Hd/2]; (x, tables) dtypes f32/f32,
 * bf16/bf16, bf16/f32 (reference) and f16/f16, f16/f32 (extension); out has
 * x's shape and dtype. */
PC_API int pc_kernel_rope_apply(const pc_tensor* x, const pc_tensor* cos_t, const pc_tensor* sin_t,
                                const pc_tensor* out, pc_kernel** kernel);
/* Extension: the decode step's per-head norms and RoPE in place, one launch
 * for RMSNorm(q, q_norm) -> RopeApply, RMSNorm(k, k_norm) -> RopeApply and
 * (norm_v != 0) RMSNorm(v) without weight (Gemma4TextInference.swift:352-381),
 * with the reference's rounding points. q [B, Nq, 1, Hd]; the new key / value
 * rows are the caches' rows [B, Nkv, Smax, Hd] at the position (offset, or
 * position int32 [1] on the device when given); tables f32 [R, Hd/2], row 0
 * when R == 1 else the position's row. */
PC_API int pc_kernel_qk_norm_rope(const pc_tensor* q, const pc_tensor* k_cache, const pc_tensor* v_cache,
                                  const pc_tensor* q_norm, const pc_tensor* k_norm, const pc_tensor* cos_t,
                                  const pc_tensor* sin_t, float eps, int32_t add_one_to_weight, int32_t norm_v,
                                  int64_t offset, const pc_tensor* position, pc_kernel** kernel);

/* ---- affine-quantized weights and embedding gathers ----------------------- */

/* Kernels.Matmul(_:_:into:) with an AffineQuantizedTensor RHS (Matmul.swift:
 * 99-131, 279-351): c [M, N] = a [M, K] . dequant(b)^T, b the logical
 * [out_features = N, in_features = K] weight stored MLX-style: packed u32
 * [N, K/8] (bits = 4, value k in bits 4(k%8).. of word k/8), scales and
 * biases [N, K/group_size] (biases NULL: none; AffineQuantizedTensor.swift).
 * bits 4 and group_size 64 only; K % 64 == 0. (a, scales, c) dtypes:
 * bf16/bf16/bf16, bf16/bf16/f32, f32/bf16/f32 (reference) and f16/f16/f16
 * (extension). fp32 accumulation, one rounding at the store. An encoder with
 * a scratch allocator splits K over CTAs when the rows are few. */
PC_API int pc_kernel_matmul_affine_quantized(const pc_tensor* a, const pc_tensor* packed, const pc_tensor* scales,
                                             const pc_tensor* biases, int64_t out_features, int64_t in_features,
                                             int32_t bits, int32_t group_size, const pc_tensor* c,
                                             pc_kernel** kernel);
/* An AffineQuantizedTensor argument of the fused 4-bit forms. */
typedef struct pc_affine_quantized {
    const pc_tensor* packed; /* u32 [out_features, in_features / 8] */
    const pc_tensor* scales; /* [out_features, in_features / group_size] */
    const pc_tensor* biases; /* same shape, or NULL */
    int64_t out_features, in_features;
    int32_t bits, group_size;
} pc_affine_quantized;

/* Extensions: the decode forms of the 4-bit Matmul, each equal to a
 * reference op sequence with its rounding points (bf16 x with bf16 scales,
 * or f16 / f16; outputs in x's dtype; in_features % 256 == 0, packed values
 * 16-byte and scales / biases 8-byte aligned):
 *   aq_rmsnorm_matmul: out = Matmul(RMSNorm(x, norm_weight), w);
 *   aq_matmul_residual: out = Add(Matmul(x, w), residual);
 *   aq_gated_mlp: out [rows, F] = act(g) * u, [g, u] = Matmul(RMSNorm(x), w)
 *     with w's rows interleaved in blocks of 8: rows 16i..16i+7 are gate rows
 *     8i..8i+7 and rows 16i+8..16i+15 the up rows 8i..8i+7 (F % 8 == 0);
 *   aq_qkv_projection: Matmul(RMSNorm(x), w_qkv) split into q [B,Nq,1,Hd]
 *     and the new K/V rows written into the caches [B,Nkv,Smax,Hd] at the
 *     position (offset, or position int32 [1] on the device). */
PC_API int pc_kernel_aq_rmsnorm_matmul(const pc_tensor* x, const pc_tensor* norm_weight, float eps,
                                       int32_t add_one_to_weight, const pc_affine_quantized* w,
                                       const pc_tensor* out, pc_kernel** kernel);
PC_API int pc_kernel_aq_matmul_residual(const pc_tensor* x, const pc_affine_quantized* w, const pc_tensor* residual,
                                        const pc_tensor* out, pc_kernel** kernel);
PC_API int pc_kernel_aq_gated_mlp(const pc_tensor* x, const pc_tensor* norm_weight, float eps,
                                  int32_t add_one_to_weight, const pc_affine_quantized* w_gate_up,
                                  int32_t activation, const pc_tensor* out, pc_kernel** kernel);
PC_API int pc_kernel_aq_qkv_projection(const pc_tensor* x, const pc_tensor* norm_weight, float eps,
                                       int32_t add_one_to_weight, const pc_affine_quantized* w_qkv,
                                       const pc_tensor* q_out, const pc_tensor* k_cache, const pc_tensor* v_cache,
                                       int64_t offset, const pc_tensor* position, pc_kernel** kernel);
/* Kernels.EmbeddingGather(ids:table:into:) (EmbeddingGather.swift): out
 * [T, H] = table[ids]; ids int32, (table, out) f32/f32, f16/f16, bf16/bf16,
 * bf16/f32. An id outside the table sets bit 4 of the device error word
 * and leaves its output row unwritten. */
PC_API int pc_kernel_embedding_gather(const pc_tensor* ids, const pc_tensor* table, const pc_tensor* out,
                                      pc_kernel** kernel);
/* Kernels.EmbeddingGather with an AffineQuantizedTensor table [vocab, H]
 * (EmbeddingGather.swift, AffineQuantizedEmbeddingGather.metal): rows
 * dequantised on the fly; ids rank 1 int32; (scales, out) bf16/bf16,
 * bf16/f32 (reference), f16/f16 (extension); bits 4, group_size 64. */
PC_API int pc_kernel_embedding_gather_affine_quantized(const pc_tensor* ids, const pc_tensor* packed,
                                                       const pc_tensor* scales, const pc_tensor* biases,
                                                       int64_t vocab, int64_t hidden, int32_t bits,
                                                       int32_t group_size, const pc_tensor* out,
                                                       pc_kernel** kernel);

/* ---- tensor parallelism over peer memory (extension) ---------------------- */

/* CUDA IPC of a pc_buffer_alloc allocation (64-byte opaque handle), for one
 * process per GPU on one node. pc_ipc_open_handle maps a peer's allocation
 * into this process (peer access enabled lazily); pc_ipc_close_handle
 * unmaps it. */
PC_API int pc_ipc_get_handle(const void* ptr, uint8_t* handle64);
PC_API int pc_ipc_open_handle(const uint8_t* handle64, void** ptr);
PC_API int pc_ipc_close_handle(void* ptr);

/* The ranks of one tensor-parallel group as seen by this process: for every
 * rank, its two partial-sum buffers ([rows, H] of the activation dtype, at
 * least rows * H elements) and its control block (5 x uint32, zero-filled
 * once before first use); this rank's own pointers at index `rank`, the
 * peers' opened with pc_ipc_open_handle. */
#define PC_MAX_PEERS 8
typedef struct pc_peer_group {
    int32_t world, rank;
    void* partial[PC_MAX_PEERS][2];
    uint32_t* control[PC_MAX_PEERS];
} pc_peer_group;
/* All-reduce (sum) of partial buffer `buffer` (0 or 1) across the group,
 * then sum_out = residual + that sum, then norm_out = RMSNorm(sum_out,
 * norm_weight, eps, add_one) — the NCCL all-reduce -> Add (Add.metal) ->
 * RMSNorm (RMSNorm.metal) sequence in one kernel. The ranks' partials are
 * read over peer memory (NVLink) once each rank has published its own;
 * every wait is bounded (device error word bit 3 on give-up). Every rank
 * must issue the same sequence of calls; a rank's buffer b is rewritten
 * only after its next call on the other buffer. residual / sum_out /
 * norm_out [rows, H], bf16 or f16, H a multiple of 8 and at most 8192. */
PC_API int pc_kernel_allreduce_add_rmsnorm(const pc_peer_group* group, int32_t buffer, const pc_tensor* residual,
                                           const pc_tensor* norm_weight, float eps, int32_t add_one_to_weight,
                                           const pc_tensor* sum_out, const pc_tensor* norm_out, pc_kernel** kernel);

/* Matmul + all-reduce + Add + RMSNorm in ONE kernel: the tensor-core GEMM of
 * a [M,K] by w [N,K] (transposeB; M <= 64, bf16 or f16) writes its output
 * tiles into this rank's partial buffer `buffer`; when the rank's last tile
 * is stored it publishes the partial, and the same kernel then sums every
 * rank's rows over peer memory and applies Add(residual) and RMSNorm as
 * pc_kernel_allreduce_add_rmsnorm does (residual / outputs [M, N]). */
PC_API int pc_kernel_matmul_allreduce_add_rmsnorm(const pc_tensor* a, const pc_tensor* w, const pc_peer_group* group,
                                                  int32_t buffer, const pc_tensor* residual,
                                                  const pc_tensor* norm_weight, float eps, int32_t add_one_to_weight,
                                                  const pc_tensor* sum_out, const pc_tensor* norm_out,
                                                  pc_kernel** kernel);

/* ---- fused decode step (extension) ---------------------------------------- */

/* One decode layer's weights and KV caches (device pointers). Weights are
 * [out, in]: w_qkv [(Nq+2*Nkv)*Hd, H], w_o [H, Nq*Hd], w_gate / w_up [F, H],
 * w_down [H, F]; norms f32 [H] (NULL = no weight); caches [Nkv, Smax, Hd]. */
typedef struct pc_decode_layer {
    const void* w_qkv;
    const void* w_o;
    const void* w_gate;
    const void* w_up;
    const void* w_down;
    const float* attn_norm;
    const float* mlp_norm;
    void* k_cache;
    void* v_cache;
    /* Per-head q / k RMSNorm weights f32 [Hd] (used when the descriptor's
     * qk_norm is set; NULL = no weight) and RoPE tables f32 [rope_rows, Hd/2]
     * (NULL = no RoPE), Gemma4TextInference.swift:352-381. */
    const float* q_norm;
    const float* k_norm;
    const float* rope_cos;
    const float* rope_sin;
} pc_decode_layer;

/* A batch-1 decode step through a stack of layers. Each layer is the op
 * sequence of Gemma4TextInference.swift:312-436 restricted to RMSNorm ->
 * QKV -> KVCacheWrite -> FlashAttention (Sq = 1) -> o_proj -> Add ->
 * RMSNorm -> gated MLP -> Add (optionally with the per-head q / k / v norms
 * and RoPE after the QKV projection), with every intermediate rounded to `dtype`
 * where the reference ops store it. `layers` points to `num_layers`
 * pc_decode_layer entries in DEVICE memory. Activation buffers (device,
 * `dtype`): x [H] holds the input and, for an even layer count, the output
 * (odd: x2); h [H], q [Nq*Hd], attn [Nq*Hd], act [F]. position: int32 [1]
 * on the device (the new token's index; it attends to keys 0..position).
 * workspace: pc_decode_stack_workspace_bytes() bytes, zero-filled once
 * before the first use; every launch leaves it zeroed (except after a
 * device error, see pc_device_error_check). Head dim 256, f16 or bf16,
 * Nq / Nkv in {1, 2, 4}, hidden and ffn multiples of 8, hidden <= 8192,
 * max(hidden, ffn, Nq*Hd) <= 12288; every buffer and weight 16-byte
 * aligned. */
typedef struct pc_decode_stack_desc {
    int32_t dtype;
    int32_t num_layers;
    int32_t hidden, q_heads, kv_heads, head_dim, ffn, max_ctx;
    float eps, attn_scale;
    int32_t activation;        /* pc_activation */
    int32_t add_one_to_weight; /* RMSNorm weight is (1 + w) */
    const pc_decode_layer* layers;
    void* x;
    void* x2;
    void* h;
    void* q;
    void* attn;
    void* act;
    const int32_t* position;
    void* workspace;
    uint64_t workspace_bytes;
    /* qk_norm: RMSNorm of each q and new k head after the QKV projection
     * (and of each new v head without weight when norm_v); rope_rows: rows of
     * the layers' RoPE tables (0: no RoPE; 1: the step's row; else indexed
     * by position). */
    int32_t qk_norm, norm_v;
    int64_t rope_rows;
} pc_decode_stack_desc;

/* Extension (no reference counterpart): workspace size for a descriptor. */
PC_API int pc_decode_stack_workspace_bytes(const pc_decode_stack_desc* desc, uint64_t* bytes);
/* Extension: the whole step as ONE persistent kernel (one CTA per SM, all
 * co-resident, ordered by arrival counters in the workspace): per-group
 * producer warps stream the next ops' weights into shared memory while the
 * current op finishes. Results equal the per-op kernels' within the chain
 * tolerance of a whole layer (dot products sum in another order). */
PC_API int pc_kernel_decode_stack(const pc_decode_stack_desc* desc, pc_kernel** kernel);

/* ---- decode attention without allocation ------------------------------- */

/* No counterpart in the reference. For callers that cannot allocate device
 * memory — real-time decode loops that must never allocate (an allocation
 * can synchronise the device and stall the loop), hosts whose device memory
 * belongs to another framework's pool and may not be touched by a library —
 * this runs the same decode attention as
 * pc_kernel_flash_attention (Sq == 1) / pc_kernel_flash_decoding_ragged
 * (seq_lens != NULL) with the same split plan, so the results are
 * identical, but keeps the partial (m, l, O) buffers in a fixed device array
 * inside this library instead of borrowing them from a scratch allocator.
 * The caller passes q [B,Nq,1,Hd], k/v [B,Nkv,S,Hd], out [B,Nq,1,Hd] and
 * an optional seq_lens (i32 [B] on the device, each 0 <= len <= S and
 * clamped to that range on the device; with seq_lens, S may be 0); the work
 * is enqueued on `stream` (cudaStream_t) of the current device.
 *  - The array holds pc_flash_decoding_noalloc_capacity() bytes (1 MiB) on
 *    every GPU that loads the library, until the process exits. A problem
 *    whose partials need more is rejected with PC_ERR_WORKSPACE_EXHAUSTED
 *    before anything is launched.
 *  - Every call shares the array and leaves its contents behind; nothing in
 *    it has to start at zero. Calls whose GPU work overlaps (e.g. on two
 *    streams with no ordering) race on it.
 *  - The first call on a device looks up the array's device address; make
 *    that first call before any stream capture begins.
 * It calls no cudaMalloc / cudaFree and no allocating library routine. */
PC_API int pc_flash_decoding_noalloc(const pc_tensor* q, const pc_tensor* k, const pc_tensor* v, const pc_tensor* out,
                                     const pc_tensor* seq_lens, float scale, pc_attention_mask mask, void* stream);
PC_API size_t pc_flash_decoding_noalloc_capacity(void);

#ifdef __cplusplus
}
#endif

#endif /* POPCORN_CUDA_H */
