// dtype.cuh — element loads/stores with the reference's conversion rules.
//
// Sources/Popcorn/PopcornDTypes.h:9-53: a bf16 load is a 16-bit left shift
// into an fp32 word; a bf16 store rounds to nearest even with no NaN special
// case; f16 uses IEEE round-to-nearest-even. These are the only rounding
// points the kernels introduce; all arithmetic runs in fp32.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace popcorn {


// Element tags used as template parameters.
struct TF32 { using storage = float; static constexpr int code = 8; };
struct TF16 { using storage = uint16_t; static constexpr int code = 9; };
struct TBF16 { using storage = uint16_t; static constexpr int code = 10; };

__device__ __forceinline__ float bf16_bits_to_float(uint32_t b) { return __uint_as_float(b << 16); }
__device__ __forceinline__ float f16_bits_to_float(uint32_t b) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(b)));
}

// PopcornDTypes.h:29-34.
__device__ __forceinline__ uint32_t float_to_bf16_bits(float x) {
    uint32_t bits = __float_as_uint(x);
    uint32_t lsb = (bits >> 16) & 1u;
    return (bits + 0x7fffu + lsb) >> 16;
}
__device__ __forceinline__ uint32_t float_to_f16_bits(float x) {
    return static_cast<uint32_t>(__half_as_ushort(__float2half_rn(x)));
}

template <class T> struct Elem;

template <> struct Elem<TF32> {
    static __device__ __forceinline__ float load(const void* p, int64_t i) { return static_cast<const float*>(p)[i]; }
    static __device__ __forceinline__ void store(void* p, int64_t i, float x) { static_cast<float*>(p)[i] = x; }
    static __device__ __forceinline__ float round(float x) { return x; }
    static constexpr int bytes = 4;
};
template <> struct Elem<TF16> {
    static __device__ __forceinline__ float load(const void* p, int64_t i) {
        return f16_bits_to_float(static_cast<const uint16_t*>(p)[i]);
    }
    static __device__ __forceinline__ void store(void* p, int64_t i, float x) {
        static_cast<uint16_t*>(p)[i] = static_cast<uint16_t>(float_to_f16_bits(x));
    }
    static __device__ __forceinline__ float round(float x) { return __half2float(__float2half_rn(x)); }
    static __device__ __forceinline__ uint32_t pack(float x) { return float_to_f16_bits(x); }
    static constexpr int bytes = 2;
};
template <> struct Elem<TBF16> {
    static __device__ __forceinline__ float load(const void* p, int64_t i) {
        return bf16_bits_to_float(static_cast<const uint16_t*>(p)[i]);
    }
    static __device__ __forceinline__ void store(void* p, int64_t i, float x) {
        static_cast<uint16_t*>(p)[i] = static_cast<uint16_t>(float_to_bf16_bits(x));
    }
    static __device__ __forceinline__ float round(float x) { return bf16_bits_to_float(float_to_bf16_bits(x)); }
    static __device__ __forceinline__ uint32_t pack(float x) { return float_to_bf16_bits(x); }
    static constexpr int bytes = 2;
};

// Two packed 16-bit elements (one 32-bit word) -> two floats.
template <class T> __device__ __forceinline__ float2 unpack2(uint32_t w);
template <> __device__ __forceinline__ float2 unpack2<TBF16>(uint32_t w) {
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
template <> __device__ __forceinline__ float2 unpack2<TF16>(uint32_t w) {
    __half2 h = *reinterpret_cast<__half2*>(&w);
    return __half22float2(h);
}

// Eight 16-bit elements held in a uint4 -> eight floats.
template <class T> __device__ __forceinline__ void unpack8(const uint4& v, float* f) {
    float2 a = unpack2<T>(v.x), b = unpack2<T>(v.y), c = unpack2<T>(v.z), d = unpack2<T>(v.w);
    f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y; f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
}

template <class T> __device__ __forceinline__ uint32_t pack2(float a, float b) {
    return Elem<T>::pack(a) | (Elem<T>::pack(b) << 16);
}

// Read-only 16-byte global load that does not allocate in L1.
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// Programmatic dependent launch: wait for the preceding grid's results /
// let the next grid begin its independent prologue. Both are no-ops when
// the launch did not opt in.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// GeluTanh.metal:6-11.
__device__ __forceinline__ float gelu_tanh(float v) {
    const float k0 = 0.7978845608028654f;
    const float k1 = 0.044715f;
    float inner = fminf(fmaxf(k0 * (v + k1 * v * v * v), -20.0f), 20.0f);
    return 0.5f * v * (1.0f + tanhf(inner));
}
__device__ __forceinline__ float silu(float v) { return v / (1.0f + expf(-v)); }

}  // namespace popcorn
