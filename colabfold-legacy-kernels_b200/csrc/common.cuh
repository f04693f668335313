// common.cuh -- element types, conversions and small vector helpers shared by the kernels.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace cfk {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// Value that a masked logit is replaced by (cuda/volta_mma_attn.cu:25,186-188).
constexpr float kMaskedLogit = -1.0e4f;

template <typename T>
struct Elem;

template <>
struct Elem<__nv_bfloat16> {
    static constexpr bool kBf16 = true;
    __device__ static __forceinline__ float2 to_float2(uint32_t w) {
        // bf16 -> f32 is a 16-bit shift; the low half is element 0.
        return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
    }
    __device__ static __forceinline__ float to_float(uint16_t h) {
        return __uint_as_float(static_cast<uint32_t>(h) << 16);
    }
    __device__ static __forceinline__ uint32_t pack(float lo, float hi) {
        __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&v);
    }
    __device__ static __forceinline__ uint16_t from_float(float f) {
        __nv_bfloat16 v = __float2bfloat16_rn(f);
        return *reinterpret_cast<uint16_t*>(&v);
    }
};

template <>
struct Elem<__half> {
    static constexpr bool kBf16 = false;
    __device__ static __forceinline__ float2 to_float2(uint32_t w) {
        __half2 h = *reinterpret_cast<__half2*>(&w);
        return __half22float2(h);
    }
    __device__ static __forceinline__ float to_float(uint16_t h) {
        return __half2float(*reinterpret_cast<__half*>(&h));
    }
    __device__ static __forceinline__ uint32_t pack(float lo, float hi) {
        __half2 v = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&v);
    }
    __device__ static __forceinline__ uint16_t from_float(float f) {
        __half v = __float2half_rn(f);
        return *reinterpret_cast<uint16_t*>(&v);
    }
};

__device__ __forceinline__ uint4 ld_global_nc_v4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// Streaming load: the data is read once, so do not keep it in L1.
__device__ __forceinline__ uint4 ld_global_stream_v4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ void st_global_v4(void* p, uint4 v) {
    asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
                 "r"(v.w)
                 : "memory");
}

} // namespace cfk
