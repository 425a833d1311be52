// Element decoding shared by the FP32-accumulating GEMV kernels: the storage
// type of each input encoding (In) and its exact conversion to FP32.
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace dnnopt_b200 {

template <In I> struct Elem;
template <> struct Elem<In::F32> { using T = float; };
template <> struct Elem<In::BF16> { using T = uint16_t; };
template <> struct Elem<In::F32R> { using T = float; };
template <> struct Elem<In::RE4> { using T = uint8_t; };
template <> struct Elem<In::RE5> { using T = uint8_t; };

// Reference fp8_e4m3_t decode (include/dnnopt/gemm/gemm_types.h:88-115):
// bias 8, subnormal step 2^-9, field 0x7F/0xFF decodes to +-448.
__device__ __forceinline__ float decode_re4(uint32_t b) {
    uint32_t s = (b >> 7) & 1u, e = (b >> 3) & 0xFu, m = b & 7u;
    float v;
    if (e == 0) v = static_cast<float>(m) * 0.001953125f;           // m * 2^-9
    else if (e == 0xF && m == 7) v = 448.0f;
    else v = __uint_as_float(((e + 119u) << 23) | (m << 20));      // 2^(e-8) * (1+m/8)
    return s ? -v : v;
}

// Reference fp8_e5m2_t decode (gemm_types.h:160-191): bias 16,
// subnormal step 2^-16, exponent field 31 is inf/nan.
__device__ __forceinline__ float decode_re5(uint32_t b) {
    uint32_t s = (b >> 7) & 1u, e = (b >> 2) & 0x1Fu, m = b & 3u;
    if (e == 0) {
        float v = static_cast<float>(m) * 1.52587890625e-05f;       // m * 2^-16
        return s ? -v : v;
    }
    if (e == 0x1F) return __uint_as_float((s << 31) | (0xFFu << 23) | (m << 21));
    return __uint_as_float((s << 31) | ((e + 111u) << 23) | (m << 21));
}

template <In I>
__device__ __forceinline__ float dec(typename Elem<I>::T v) {
    if constexpr (I == In::F32) return v;
    else if constexpr (I == In::BF16) return bf16_bits_to_f32(v);
    else if constexpr (I == In::F32R) return round_to_bf16(v);
    else if constexpr (I == In::RE4) return decode_re4(v);
    else return decode_re5(v);
}

// Four consecutive elements of one B row -> four floats (aligned vector load).
template <In I>
__device__ __forceinline__ void load4(const typename Elem<I>::T* p, float (&o)[4]) {
    if constexpr (sizeof(typename Elem<I>::T) == 4) {
        float4 v = __ldg(reinterpret_cast<const float4*>(p));
        o[0] = dec<I>(v.x); o[1] = dec<I>(v.y); o[2] = dec<I>(v.z); o[3] = dec<I>(v.w);
    } else if constexpr (sizeof(typename Elem<I>::T) == 2) {
        uint2 v = __ldg(reinterpret_cast<const uint2*>(p));
        o[0] = dec<I>(static_cast<uint16_t>(v.x & 0xFFFFu));
        o[1] = dec<I>(static_cast<uint16_t>(v.x >> 16));
        o[2] = dec<I>(static_cast<uint16_t>(v.y & 0xFFFFu));
        o[3] = dec<I>(static_cast<uint16_t>(v.y >> 16));
    } else {
        uint32_t v = __ldg(reinterpret_cast<const unsigned int*>(p));
        o[0] = dec<I>(static_cast<uint8_t>(v & 0xFFu));
        o[1] = dec<I>(static_cast<uint8_t>((v >> 8) & 0xFFu));
        o[2] = dec<I>(static_cast<uint8_t>((v >> 16) & 0xFFu));
        o[3] = dec<I>(static_cast<uint8_t>(v >> 24));
    }
}

}  // namespace dnnopt_b200
