// act16.cuh - the 16-bit activation element of a context: bf16 (RG_MODE_BF16,
// RG_MODE_INT8_FULL) or fp16 (RG_MODE_F16, RG_MODE_INT8_W).  Buffers hold raw
// 16-bit words; kernels are templated on F16 and convert through these.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace rg {

template <bool F16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    if constexpr (F16) {
        __half2 p = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&p);
    } else {
        __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&p);
    }
}

template <bool F16>
__device__ __forceinline__ float2 unpack2(uint32_t u) {
    if constexpr (F16) {
        return __half22float2(*reinterpret_cast<const __half2*>(&u));
    } else {
        return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u));
    }
}

template <bool F16>
__device__ __forceinline__ float to_f32(uint16_t h) {
    if constexpr (F16) {
        return __half2float(__ushort_as_half(h));
    } else {
        return __bfloat162float(__ushort_as_bfloat16(h));
    }
}

template <bool F16>
__device__ __forceinline__ uint16_t from_f32(float x) {
    if constexpr (F16) {
        return __half_as_ushort(__float2half_rn(x));
    } else {
        return __bfloat16_as_ushort(__float2bfloat16_rn(x));
    }
}

}  // namespace rg
