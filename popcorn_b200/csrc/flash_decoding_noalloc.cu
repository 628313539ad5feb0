// flash_decoding_noalloc.cu — split-KV decode attention for callers that
// cannot allocate device memory.
//
// The encoder path borrows the decode attention's partial (m, l, O) buffers
// from the caller's scratch allocator. Some callers have none to offer:
// real-time decode loops that must never hit an allocation and its implicit
// device synchronisation, and hosts whose device memory is owned by another
// framework's pool that a library may not draw from. For them this file
// holds the partials in a fixed, file-scope device array instead; the caller
// still passes q, K, V and the output.
//
// Limits and sharing:
//  * The array holds kNoAllocScratchBytes (1 MiB) on every GPU that loads
//    this library, for the life of the process. A problem whose split plan
//    needs more (roughly batch * query_heads * splits * head_dim * 4 bytes)
//    is rejected with PC_ERR_WORKSPACE_EXHAUSTED before anything launches.
//  * Every call uses the same array and leaves its contents behind. Nothing
//    in it has to start at zero: the partial pass writes every (m, l, O)
//    slot it owns, including those of splits with no keys, before the
//    combine pass reads them. Calls whose GPU work overlaps (different
//    streams, no ordering between them) race on the array; order them on
//    one stream or with events.
//  * The device address of the array is looked up once per device, with
//    that device current, on the first call made for it. Make that first
//    call before any stream capture begins.
#include <mutex>
#include <string>

#include "launch.hpp"
#include "popcorn.hpp"

namespace popcorn {
void set_last_error(const std::string& m);
}

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(1) << 20;
constexpr int kMaxDevices = 64;

// In host code this name is a host-side stand-in, not a device address: the
// device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_fd_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_setup_lock;
void* g_scratch_addr[kMaxDevices] = {nullptr};

// Resolves the array's device address for `device` (which must be current).
int scratch_address(int device, void** out) {
    if (device < 0 || device >= kMaxDevices) return PC_ERR_GPU_DEVICE_REMOVED;
    std::lock_guard<std::mutex> guard(g_setup_lock);
    if (!g_scratch_addr[device]) {
        void* ptr = nullptr;
        cudaError_t err = cudaGetSymbolAddress(&ptr, g_fd_noalloc_scratch);
        if (err != cudaSuccess || !ptr) {
            cudaGetLastError();
            popcorn::set_last_error(std::string("cudaGetSymbolAddress of the no-alloc scratch failed: ") +
                                    cudaGetErrorString(err));
            return PC_ERR_GPU_INTERNAL;
        }
        g_scratch_addr[device] = ptr;
    }
    *out = g_scratch_addr[device];
    return PC_OK;
}

bool is_float(int dt) { return dt == PC_F32 || dt == PC_F16 || dt == PC_BF16; }

int reject(int code, const char* msg) {
    popcorn::set_last_error(msg);
    return code;
}

}  // namespace

extern "C" {

size_t pc_flash_decoding_noalloc_capacity(void) { return kNoAllocScratchBytes; }

int pc_flash_decoding_noalloc(const pc_tensor* q, const pc_tensor* k, const pc_tensor* v, const pc_tensor* out,
                              const pc_tensor* seq_lens, float scale, pc_attention_mask mask, void* stream) {
    using namespace popcorn;
    if (!q || !k || !v || !out) return reject(PC_ERR_TENSOR_SHAPE_MISMATCH, "q, k, v and out are required.");
    if (q->rank != 4 || k->rank != 4 || v->rank != 4 || out->rank != 4)
        return reject(PC_ERR_TENSOR_INVALID_RANK, "q, k, v and out must have rank 4.");
    const int64_t B = q->shape[0], Nq = q->shape[1], Sq = q->shape[2], Hd = q->shape[3];
    const int64_t Nkv = k->shape[1], S = k->shape[2];
    if (Sq != 1) return reject(PC_ERR_TENSOR_SHAPE_MISMATCH, "decode attention takes one query token (q [B,Nq,1,Hd]).");
    if (k->shape[0] != B || k->shape[3] != Hd)
        return reject(PC_ERR_TENSOR_SHAPE_MISMATCH, "K must be [B,Nkv,S,Hd] matching q's batch and head dim.");
    for (int i = 0; i < 4; ++i) {
        if (v->shape[i] != k->shape[i]) return reject(PC_ERR_TENSOR_SHAPE_MISMATCH, "V shape must match K.");
        if (out->shape[i] != q->shape[i]) return reject(PC_ERR_TENSOR_SHAPE_MISMATCH, "out shape must match q.");
    }
    if (B < 1 || Nq < 1 || Nkv < 1 || Nq % Nkv != 0)
        return reject(PC_ERR_TENSOR_SHAPE_MISMATCH, "query heads must be a positive multiple of KV heads.");
    if (Hd < 1 || Hd > 512) return reject(PC_ERR_TENSOR_SHAPE_MISMATCH, "head dim must be in 1..512.");
    // As the encoder path: S == 0 is only meaningful with per-sequence lengths.
    if (S < 0 || (!seq_lens && S < 1)) return reject(PC_ERR_TENSOR_SHAPE_MISMATCH, "K/V need at least one key.");
    if (!is_float(q->dtype) || q->dtype != k->dtype || k->dtype != v->dtype || !is_float(out->dtype))
        return reject(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION,
                      "q, k, v must share one of f32/f16/bf16 and out must be f32/f16/bf16.");
    if (mask.kind < 0 || mask.kind > 2 || (mask.kind == PC_MASK_CAUSAL_SLIDING_WINDOW && mask.window < 1))
        return reject(PC_ERR_TENSOR_SHAPE_MISMATCH, "invalid attention mask.");
    if (seq_lens && (seq_lens->dtype != PC_I32 || seq_lens->rank < 1 || seq_lens->shape[0] < B || !seq_lens->data))
        return reject(PC_ERR_UNSUPPORTED_DATA_TYPE_COMBINATION, "seq_lens must be i32 [B] on the device.");
    if (!q->data || !k->data || !v->data || !out->data)
        return reject(PC_ERR_TENSOR_SHAPE_MISMATCH, "a tensor has no device buffer.");

    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) {
        cudaGetLastError();
        return reject(PC_ERR_GPU_DEVICE_REMOVED, "no current CUDA device.");
    }
    launch::FlashDecode p{q->data, q->dtype, k->data, v->data, k->dtype, out->data, out->dtype, B, Nq, Nkv, S, Hd,
                          seq_lens ? static_cast<const int32_t*>(seq_lens->data) : nullptr, scale, mask.kind,
                          mask.window};
    launch::FlashDecodePlan plan = launch::flash_decode_plan(p, launch::device_info(device).sm_count);
    // Same split plan as the encoder path, so both give identical results.
    const size_t o_bytes = (plan.scratch_o + 255) / 256 * 256;
    const size_t ml_bytes = (plan.scratch_ml + 255) / 256 * 256;
    const size_t need = plan.splits > 1 ? o_bytes + 2 * ml_bytes : 0;
    if (need > kNoAllocScratchBytes) {
        std::string m = "decode attention needs " + std::to_string(need) + " bytes of partials (" +
                        std::to_string(plan.splits) + " splits); the no-alloc scratch holds " +
                        std::to_string(kNoAllocScratchBytes) + " bytes.";
        return reject(PC_ERR_WORKSPACE_EXHAUSTED, m.c_str());
    }
    void* base = nullptr;
    int st = scratch_address(device, &base);
    if (st != PC_OK) return st;
    float* po = static_cast<float*>(base);
    float* pm = reinterpret_cast<float*>(static_cast<char*>(base) + o_bytes);
    float* pl = reinterpret_cast<float*>(static_cast<char*>(base) + o_bytes + ml_bytes);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t err = launch::flash_decode(p, plan, po, pm, pl, s);
    if (err == cudaSuccess && plan.splits > 1) err = launch::flash_decode_combine(p, plan, po, pm, pl, s);
    if (err != cudaSuccess) {
        cudaGetLastError();
        return reject(PC_ERR_GPU_INTERNAL, cudaGetErrorString(err));
    }
    return PC_OK;
}

}  // extern "C"
