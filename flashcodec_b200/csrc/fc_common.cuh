// Shared helpers for the flashcodec_b200 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "../../include/flashcodec_b200.h"

namespace fc {

// ------------------------------------------------------------ error handling
// Thread-local message for fc_last_error_string (defined in fc_capi.cu).
void set_error(const char *fmt, ...);
void clear_error();
int check_launch(const char *what);

inline int dtype_size(int dt) {
    switch (dt) {
        case FC_F32: return 4;
        case FC_BF16: return 2;
        case FC_F16: return 2;
        case FC_I8: return 1;
        default: return 0;
    }
}

inline bool is_float_dtype(int dt) { return dt == FC_F32 || dt == FC_BF16 || dt == FC_F16; }

inline bool aligned(const void *p, int bytes) {
    return (reinterpret_cast<uintptr_t>(p) % (uintptr_t)bytes) == 0;
}

int num_sms();  // SM count of the current device (cached per device)

// --------------------------------------------------------- element converters
// Scalar load of element i of a buffer of runtime dtype `dt`, as fp32.
__device__ __forceinline__ float load_as_f32(const void *p, int64_t i, int dt) {
    switch (dt) {
        case FC_F32: return static_cast<const float *>(p)[i];
        case FC_BF16: return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
        case FC_F16: return __half2float(static_cast<const __half *>(p)[i]);
        default: return (float)static_cast<const int8_t *>(p)[i];
    }
}

// Round-to-nearest-even store of an fp32 value into a buffer of dtype `dt`.
__device__ __forceinline__ void store_from_f32(void *p, int64_t i, int dt, float v) {
    switch (dt) {
        case FC_F32: static_cast<float *>(p)[i] = v; break;
        case FC_BF16: static_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(v); break;
        case FC_F16: static_cast<__half *>(p)[i] = __float2half_rn(v); break;
        default: break;
    }
}

// The value an fp32 number takes once stored as dtype `dt` (RNE), as fp32.
__device__ __forceinline__ float round_to_dtype(float v, int dt) {
    switch (dt) {
        case FC_BF16: return __bfloat162float(__float2bfloat16_rn(v));
        case FC_F16: return __half2float(__float2half_rn(v));
        default: return v;
    }
}

// Typed element traits for the vectorised paths.
template <typename T> struct Elem;
template <> struct Elem<float> {
    static constexpr int code = FC_F32;
    __device__ __forceinline__ static float to_f32(float v) { return v; }
};
template <> struct Elem<__nv_bfloat16> {
    static constexpr int code = FC_BF16;
    __device__ __forceinline__ static float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
};
template <> struct Elem<__half> {
    static constexpr int code = FC_F16;
    __device__ __forceinline__ static float to_f32(__half v) { return __half2float(v); }
};
template <> struct Elem<int8_t> {
    static constexpr int code = FC_I8;
    __device__ __forceinline__ static float to_f32(int8_t v) { return (float)v; }
};

// Four signed bytes of a 32-bit word to fp32 without the integer-to-float
// conversion unit: each byte, biased to unsigned by flipping its sign bit, is
// placed in the low mantissa bits of 2^23 (0x4B0000uu == 2^23 + u), and one
// fp32 subtraction of 2^23 + 128 yields the signed value exactly.  (The
// exponent-bias construction for small integers.)
__device__ __forceinline__ void s8x4_to_f32(uint32_t w, float out[4]) {
    const uint32_t u = w ^ 0x80808080u;
    out[0] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7650)) - 8388736.0f;
    out[1] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7651)) - 8388736.0f;
    out[2] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7652)) - 8388736.0f;
    out[3] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7653)) - 8388736.0f;
}

// Load VEC consecutive elements of type T starting at p (16-, 8- or 4-byte
// aligned when VEC * sizeof(T) is that size) and widen them to fp32.  A plain
// (generic) load, so p may point into global or shared memory.
template <typename T, int VEC>
__device__ __forceinline__ void load_vec_f32(const T *p, float out[VEC]) {
    constexpr int BYTES = VEC * (int)sizeof(T);
    if constexpr (BYTES == 16 || BYTES == 8 || BYTES == 4) {
        using W = typename std::conditional<BYTES == 16, uint4,
                  typename std::conditional<BYTES == 8, uint2, uint32_t>::type>::type;
        const W w = *reinterpret_cast<const W *>(p);
        const uint32_t *u = reinterpret_cast<const uint32_t *>(&w);
        constexpr int WORDS = BYTES / 4;
#pragma unroll
        for (int i = 0; i < WORDS; i++) {
            if constexpr (std::is_same<T, int8_t>::value) {
                s8x4_to_f32(u[i], out + 4 * i);
            } else if constexpr (std::is_same<T, float>::value) {
                out[i] = __uint_as_float(u[i]);
            } else if constexpr (std::is_same<T, __nv_bfloat16>::value) {
                out[2 * i] = __uint_as_float(u[i] << 16);
                out[2 * i + 1] = __uint_as_float(u[i] & 0xFFFF0000u);
            } else {  // __half
                __half2 h = *reinterpret_cast<const __half2 *>(&u[i]);
                float2 f = __half22float2(h);
                out[2 * i] = f.x;
                out[2 * i + 1] = f.y;
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < VEC; i++) out[i] = Elem<T>::to_f32(p[i]);
    }
}

// Round VEC fp32 values to T (round-to-nearest-even, like store_from_f32) and
// store them as one vector at p (aligned to VEC * sizeof(T) when that is 16,
// 8 or 4 bytes; element stores otherwise).
template <typename T, int VEC>
__device__ __forceinline__ void store_vec_from_f32(T *p, const float v[VEC]) {
    constexpr int BYTES = VEC * (int)sizeof(T);
    if constexpr (VEC == 4 && std::is_same<T, float>::value) {
        *reinterpret_cast<float4 *>(p) = make_float4(v[0], v[1], v[2], v[3]);
    } else if constexpr (VEC == 4 && BYTES == 8 && std::is_same<T, __nv_bfloat16>::value) {
        const __nv_bfloat162 lo = __floats2bfloat162_rn(v[0], v[1]);
        const __nv_bfloat162 hi = __floats2bfloat162_rn(v[2], v[3]);
        uint2 w;
        w.x = *reinterpret_cast<const uint32_t *>(&lo);
        w.y = *reinterpret_cast<const uint32_t *>(&hi);
        *reinterpret_cast<uint2 *>(p) = w;
    } else if constexpr (VEC == 4 && BYTES == 8 && std::is_same<T, __half>::value) {
        const __half2 lo = __floats2half2_rn(v[0], v[1]);
        const __half2 hi = __floats2half2_rn(v[2], v[3]);
        uint2 w;
        w.x = *reinterpret_cast<const uint32_t *>(&lo);
        w.y = *reinterpret_cast<const uint32_t *>(&hi);
        *reinterpret_cast<uint2 *>(p) = w;
    } else {
#pragma unroll
        for (int i = 0; i < VEC; i++) store_from_f32(p, i, Elem<T>::code, v[i]);
    }
}

}  // namespace fc
