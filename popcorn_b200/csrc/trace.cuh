// trace.cuh — development-only per-CTA timelines of the decode kernels.
//
// Compiled in only with -DPC_DECODE_TRACE (never in the shipped library).
// A traced kernel stamps %globaltimer at up to six points of a CTA's life
// into shared memory and, at exit, appends one record (kind << 32 | CTA
// index, then the eight stamps) to its translation unit's device buffer; the
// host reads the buffer with pc_debug_decode_trace (exported only by a
// traced build). Without the define every macro is empty.
#pragma once

#ifdef PC_DECODE_TRACE
#define PC_DT_MAX (1 << 16)
#define PC_DT_BUFFER                                                      \
    __device__ unsigned long long g_dt_buf[PC_DT_MAX * 9];                \
    __device__ unsigned int g_dt_n;                                       \
    __device__ int dt_nomath_flag;                                        \
    __device__ __forceinline__ unsigned long long dt_now() {              \
        unsigned long long t;                                             \
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));             \
        return t;                                                         \
    }
#define DT_SHARED __shared__ unsigned long long s_dt[8];
#define DT_INIT()                                        \
    do {                                                 \
        if (threadIdx.x == 0)                            \
            for (int i_ = 0; i_ < 8; ++i_) s_dt[i_] = 0; \
    } while (0)
#define DT_MARK(i) (s_dt[i] = dt_now())
#define DT_COMMIT(kind)                                                                     \
    do {                                                                                    \
        if (threadIdx.x == 0) {                                                             \
            s_dt[5] = dt_now();                                                             \
            const unsigned int slot_ = atomicAdd(&g_dt_n, 1u);                              \
            if (slot_ < PC_DT_MAX) {                                                        \
                g_dt_buf[slot_ * 9] = (static_cast<unsigned long long>(kind) << 32) |       \
                                      (blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z)); \
                for (int i_ = 0; i_ < 8; ++i_) g_dt_buf[slot_ * 9 + 1 + i_] = s_dt[i_];     \
            }                                                                               \
        }                                                                                   \
    } while (0)
// Development-only switch of traced builds: consumers skip the arithmetic
// (results are garbage), so a timeline shows the data movement alone.
#define DT_NOMATH (dt_nomath_flag)
#else
#define DT_NOMATH false
#define PC_DT_BUFFER
#define DT_SHARED
#define DT_INIT() ((void)0)
#define DT_MARK(i) ((void)0)
#define DT_COMMIT(kind) ((void)0)
#endif
