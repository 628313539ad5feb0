// simple.cu — KV-cache write, RMSNorm and the elementwise ops.
//
// These are bandwidth-trivial at decode sizes (a few KB); they are written
// for coalesced 16-byte accesses and grid sizes in multiples of the SM
// count, and their semantics follow the reference kernels cited per kernel.
#include "common.cuh"
#include "dtype.cuh"
#include "launch.hpp"
#include "popcorn.hpp"

namespace popcorn {
namespace launch {

namespace {

// ---- KV-cache write (KVCacheWrite.metal:7-59) ---------------------------------

// Same-dtype copy in 16-byte chunks; requires (Hd * elem) % 16 == 0 and
// 16-byte aligned bases, so a chunk never straddles two (b,h,s) rows.
__global__ void kv_write_vec_kernel(KVWrite p, int elem_bytes) {
    pdl_wait();
    int64_t offset = p.pos_dev ? int64_t(*p.pos_dev) : p.offset;
    if (offset < 0 || offset + p.Snew > p.Smax) return;
    const int vec = 16 / elem_bytes;
    int64_t chunks_per_row = p.Hd / vec;
    int64_t total = p.B * p.Nkv * p.Snew * chunks_per_row;
    for (int64_t c = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; c < total; c += int64_t(gridDim.x) * blockDim.x) {
        int64_t dc = c % chunks_per_row;
        int64_t r = c / chunks_per_row;
        int64_t s = r % p.Snew;
        int64_t bh = r / p.Snew;
        int64_t dst_row = bh * p.Smax + offset + s;
        const uint4* src = reinterpret_cast<const uint4*>(p.src) + c;
        uint4* dst = reinterpret_cast<uint4*>(static_cast<char*>(p.cache) + (dst_row * p.Hd) * elem_bytes) + dc;
        *dst = *src;
    }
}

template <class S, class C>
__global__ void kv_write_scalar_kernel(KVWrite p) {
    pdl_wait();
    int64_t offset = p.pos_dev ? int64_t(*p.pos_dev) : p.offset;
    if (offset < 0 || offset + p.Snew > p.Smax) return;
    int64_t total = p.B * p.Nkv * p.Snew * p.Hd;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        int64_t d = i % p.Hd;
        int64_t r = i / p.Hd;
        int64_t s = r % p.Snew;
        int64_t bh = r / p.Snew;
        int64_t dst = (bh * p.Smax + offset + s) * p.Hd + d;
        Elem<C>::store(p.cache, dst, Elem<S>::load(p.src, i));
    }
}

// ---- RMSNorm (RMSNorm.metal:7-42) --------------------------------------------

template <class T>
__global__ void rmsnorm_kernel(RMSNorm p) {
    pdl_wait();
    __shared__ float red[32];
    __shared__ float s_scale;
    int64_t row = blockIdx.x;
    int64_t base = row * p.H;
    float acc = 0.f;
    for (int64_t i = threadIdx.x; i < p.H; i += blockDim.x) {
        float v = Elem<T>::load(p.x, base + i);
        acc += v * v;
    }
    acc = warp_sum(acc);
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = acc;
    __syncthreads();
    if (warp == 0) {
        float v = lane < int(blockDim.x >> 5) ? red[lane] : 0.f;
        v = warp_sum(v);
        if (lane == 0) s_scale = rsqrtf(v / float(p.H) + p.eps);
    }
    __syncthreads();
    float scale = s_scale;
    for (int64_t i = threadIdx.x; i < p.H; i += blockDim.x) {
        float v = Elem<T>::load(p.x, base + i) * scale;
        if (p.weight) {
            float w = p.weight[i];
            if (p.add_one) w = 1.0f + w;
            v *= w;
        }
        Elem<T>::store(p.out, base + i, v);
    }
}

// ---- elementwise (GeluTanh.metal, Mul.metal, Add.metal) -----------------------

// OP 0: GeluTanh, 1: SiLU, 2: ScalarMul (ScalarMul.metal:6-25, x * scalar)
template <class T, int OP>
__global__ void unary_kernel(const void* x, void* out, int64_t n, float scalar) {
    pdl_wait();
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        float v = Elem<T>::load(x, i);
        Elem<T>::store(out, i, OP == 0 ? gelu_tanh(v) : OP == 1 ? silu(v) : v * scalar);
    }
}

template <class T, int OP>
__global__ void binary_kernel(const void* a, const void* b, void* out, int64_t n) {
    pdl_wait();
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        float x = Elem<T>::load(a, i), y = Elem<T>::load(b, i);
        Elem<T>::store(out, i, OP == 0 ? x * y : x + y);
    }
}

// AttentionMaskBuild.metal:5-21: additive mask [Sq, Sk]; query i sits at
// key position Sk - Sq + i, key j is allowed when j <= that position and,
// with a window w >= 0, when position - j < w.
__global__ void attention_mask_build_kernel(float* mask, int64_t Sq, int64_t Sk, int32_t window) {
    pdl_wait();
    const int64_t n = Sq * Sk;
    for (int64_t k = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; k < n; k += int64_t(gridDim.x) * blockDim.x) {
        const int64_t i = k / Sk, j = k % Sk;
        const int64_t pos_q = Sk - Sq + i;
        bool allowed = j <= pos_q;
        if (window >= 0) allowed = allowed && (pos_q - j) < window;
        mask[k] = allowed ? 0.0f : -INFINITY;
    }
}

}  // namespace

DeviceInfo device_info(int device) {
    static int cached_sms[64] = {0};
    DeviceInfo d{device, 148};
    if (device >= 0 && device < 64) {
        if (cached_sms[device] == 0) {
            int sms = 0;
            if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) == cudaSuccess && sms > 0)
                cached_sms[device] = sms;
            else
                cached_sms[device] = 148;
        }
        d.sm_count = cached_sms[device];
    }
    return d;
}

int current_sm_count() {
    int dev = 0;
    cudaGetDevice(&dev);
    return device_info(dev).sm_count;
}

cudaError_t attention_mask_build(float* mask, int64_t Sq, int64_t Sk, int32_t window, cudaStream_t stream) {
    const int64_t n = Sq * Sk;
    if (n == 0) return cudaSuccess;
    return launch_k(attention_mask_build_kernel, dim3(grid_for(n, 256, current_sm_count())), dim3(256), 0, stream,
                    mask, Sq, Sk, window);
}

cudaError_t kv_cache_write(const KVWrite& p, cudaStream_t stream) {
    int64_t total = p.B * p.Nkv * p.Snew * p.Hd;
    if (total == 0) return cudaSuccess;
    int sms = current_sm_count();
    int es = dtype_stride(p.src_dtype);
    if (p.src_dtype == p.cache_dtype && (p.Hd * es) % 16 == 0 && aligned16(p.src) && aligned16(p.cache)) {
        int64_t chunks = total * es / 16;
        return launch_k(kv_write_vec_kernel, dim3(grid_for(chunks, 256, sms)), dim3(256), 0, stream, p, es);
    }
    dim3 g(grid_for(total, 256, sms)), b(256);
    if (p.src_dtype == PC_F32 && p.cache_dtype == PC_F32) return launch_k(kv_write_scalar_kernel<TF32, TF32>, g, b, 0, stream, p);
    if (p.src_dtype == PC_BF16 && p.cache_dtype == PC_BF16) return launch_k(kv_write_scalar_kernel<TBF16, TBF16>, g, b, 0, stream, p);
    if (p.src_dtype == PC_F32 && p.cache_dtype == PC_BF16) return launch_k(kv_write_scalar_kernel<TF32, TBF16>, g, b, 0, stream, p);
    if (p.src_dtype == PC_F16 && p.cache_dtype == PC_F16) return launch_k(kv_write_scalar_kernel<TF16, TF16>, g, b, 0, stream, p);
    return cudaErrorInvalidValue;
}

cudaError_t rmsnorm(const RMSNorm& p, cudaStream_t stream) {
    if (p.rows == 0) return cudaSuccess;
    int threads = p.H >= 4096 ? 1024 : (p.H >= 1024 ? 256 : 128);
    dim3 g(unsigned(p.rows)), b(threads);
    switch (p.x_dtype) {
    case PC_F32: return launch_k(rmsnorm_kernel<TF32>, g, b, 0, stream, p);
    case PC_F16: return launch_k(rmsnorm_kernel<TF16>, g, b, 0, stream, p);
    case PC_BF16: return launch_k(rmsnorm_kernel<TBF16>, g, b, 0, stream, p);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t unary(Unary op, const void* x, int x_dtype, void* out, int, int64_t count, cudaStream_t stream,
                  float scalar) {
    dim3 g(grid_for(count, 256, current_sm_count())), b(256);
    auto go = [&](auto t) {
        using T = decltype(t);
        switch (op) {
        case Unary::kGeluTanh: return launch_k(unary_kernel<T, 0>, g, b, 0, stream, x, out, count, scalar);
        case Unary::kSilu: return launch_k(unary_kernel<T, 1>, g, b, 0, stream, x, out, count, scalar);
        case Unary::kScalarMul: return launch_k(unary_kernel<T, 2>, g, b, 0, stream, x, out, count, scalar);
        }
        return cudaErrorInvalidValue;
    };
    switch (x_dtype) {
    case PC_F32: return go(TF32{});
    case PC_F16: return go(TF16{});
    case PC_BF16: return go(TBF16{});
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t binary(Binary op, const void* a, const void* bb, void* out, int dtype, int64_t count, cudaStream_t stream) {
    dim3 g(grid_for(count, 256, current_sm_count())), b(256);
    bool mul = op == Binary::kMul;
    switch (dtype) {
    case PC_F32: return mul ? launch_k(binary_kernel<TF32, 0>, g, b, 0, stream, a, bb, out, count)
                            : launch_k(binary_kernel<TF32, 1>, g, b, 0, stream, a, bb, out, count);
    case PC_F16: return mul ? launch_k(binary_kernel<TF16, 0>, g, b, 0, stream, a, bb, out, count)
                            : launch_k(binary_kernel<TF16, 1>, g, b, 0, stream, a, bb, out, count);
    case PC_BF16: return mul ? launch_k(binary_kernel<TBF16, 0>, g, b, 0, stream, a, bb, out, count)
                             : launch_k(binary_kernel<TBF16, 1>, g, b, 0, stream, a, bb, out, count);
    default: return cudaErrorInvalidValue;
    }
}

namespace {
RegisterFunctions reg_simple({
    {"kv_cache_write", reinterpret_cast<const void*>(kv_write_scalar_kernel<TF32, TF32>)},
    {"kv_cache_write_bf16", reinterpret_cast<const void*>(kv_write_scalar_kernel<TBF16, TBF16>)},
    {"kv_cache_write_f32_to_bf16", reinterpret_cast<const void*>(kv_write_scalar_kernel<TF32, TBF16>)},
    {"kv_cache_write_f16", reinterpret_cast<const void*>(kv_write_scalar_kernel<TF16, TF16>)},
    {"kv_cache_write_vec16", reinterpret_cast<const void*>(kv_write_vec_kernel)},
    {"rmsnorm", reinterpret_cast<const void*>(rmsnorm_kernel<TF32>)},
    {"rmsnorm_f16", reinterpret_cast<const void*>(rmsnorm_kernel<TF16>)},
    {"rmsnorm_bf16", reinterpret_cast<const void*>(rmsnorm_kernel<TBF16>)},
    {"gelu_tanh", reinterpret_cast<const void*>(unary_kernel<TF32, 0>)},
    {"gelu_tanh_f16", reinterpret_cast<const void*>(unary_kernel<TF16, 0>)},
    {"gelu_tanh_bf16", reinterpret_cast<const void*>(unary_kernel<TBF16, 0>)},
    {"silu", reinterpret_cast<const void*>(unary_kernel<TF32, 1>)},
    {"silu_f16", reinterpret_cast<const void*>(unary_kernel<TF16, 1>)},
    {"silu_bf16", reinterpret_cast<const void*>(unary_kernel<TBF16, 1>)},
    {"attention_mask_build", reinterpret_cast<const void*>(attention_mask_build_kernel)},
    {"scalar_mul", reinterpret_cast<const void*>(unary_kernel<TF32, 2>)},
    {"scalar_mul_f16", reinterpret_cast<const void*>(unary_kernel<TF16, 2>)},
    {"scalar_mul_bf16", reinterpret_cast<const void*>(unary_kernel<TBF16, 2>)},
    {"mul", reinterpret_cast<const void*>(binary_kernel<TF32, 0>)},
    {"mul_f16", reinterpret_cast<const void*>(binary_kernel<TF16, 0>)},
    {"mul_bf16", reinterpret_cast<const void*>(binary_kernel<TBF16, 0>)},
    {"add", reinterpret_cast<const void*>(binary_kernel<TF32, 1>)},
    {"add_f16", reinterpret_cast<const void*>(binary_kernel<TF16, 1>)},
    {"add_bf16", reinterpret_cast<const void*>(binary_kernel<TBF16, 1>)},
});
}  // namespace

}  // namespace launch
}  // namespace popcorn
