// dnnopt/gemm/gemm_types.h -- storage types of the drop-in C++ API.
//
// Binary-compatible with the reference's types (include/dnnopt/gemm/gemm_types.h
// of xuefenghao5121/DNN-Opt): same names, sizes and member layout, so objects
// compiled against the reference link against libdnnopt_b200.so unchanged.
#pragma once

#include <cstdint>
#include <cstring>

namespace dnnopt {

// 16-bit brain float, stored as raw bits.  Conversion from float rounds to
// nearest-even by adding 0x7FFF plus the lowest kept bit (the reference's
// rounding, gemm_types.h:18-24); conversion to float is a 16-bit shift.
struct bfloat16_t {
    uint16_t raw_bits;

    bfloat16_t() = default;
    constexpr explicit bfloat16_t(uint16_t raw, bool) : raw_bits(raw) {}
    explicit bfloat16_t(float f) {
        uint32_t u;
        std::memcpy(&u, &f, 4);
        raw_bits = static_cast<uint16_t>((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
    }
    operator float() const {
        uint32_t u = static_cast<uint32_t>(raw_bits) << 16;
        float f;
        std::memcpy(&f, &u, 4);
        return f;
    }
    bfloat16_t& operator=(float f) { return *this = bfloat16_t(f); }
};
static_assert(sizeof(bfloat16_t) == 2, "bfloat16_t is 2 bytes");

// The reference's 8-bit float storage types with their float conversions
// (gemm_types.h:51-200 of the reference).  The codecs are the reference's
// own, not OCP, and are restated here value for value so that source using
// them computes what it computed against the reference:
//   e4m3: exponent bias 8, the float mantissa truncated to 3 bits, exponents
//         above 7 saturate to field 7 / mantissa 7 (0.9375), exponents below
//         -6 encode as the byte 0x08 (2^-7), fields 1..15 decode as normal
//         numbers except 0x7F / 0xFF, which decode as +-448, and field 0 as
//         subnormals m * 2^-9;
//   e5m2: exponent bias 16, mantissa truncated to 2 bits, exponents above 30
//         encode as infinity, below -14 (or subnormals shifted out) as a
//         signed zero, field 31 decodes as infinity / NaN with the mantissa in
//         the top NaN payload bits, field 0 as subnormals m * 2^-16.
// The GPU kernels decode the same bytes bit-exactly.
namespace detail {
inline uint32_t f32_bits(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    return u;
}
inline float bits_f32(uint32_t u) {
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}
// Index of the highest set bit of a nonzero value below 8.
inline int top_bit3(uint32_t m) { return m >= 4u ? 2 : (m >= 2u ? 1 : 0); }

inline uint8_t ref_e4m3_encode(float f) {
    const uint32_t u = f32_bits(f);
    const uint32_t s = (u >> 24) & 0x80u;
    const int e = static_cast<int>((u >> 23) & 0xFFu) - 119;   // rebias 127 -> 8
    const uint32_t m = (u >> 20) & 7u;                          // truncated
    if (e > 7) return static_cast<uint8_t>(s | 0x3Fu);
    if (e < -6) return static_cast<uint8_t>(s | 0x08u);
    if (e > 0) return static_cast<uint8_t>(s | (static_cast<uint32_t>(e) << 3) | m);
    return static_cast<uint8_t>(s | ((m | 8u) >> -e));         // leading bit shifted in
}
inline float ref_e4m3_decode(uint8_t b) {
    const uint32_t s = static_cast<uint32_t>(b & 0x80u) << 24;
    const uint32_t e = (b >> 3) & 0xFu, m = b & 7u;
    if (e == 0xFu && m == 7u) return bits_f32(s | 0x43E00000u);                // +-448
    if (e != 0) return bits_f32(s | ((e + 119u) << 23) | (m << 20));
    if (m == 0) return bits_f32(s);
    const int t = top_bit3(m);                                                   // m * 2^-9
    return bits_f32(s | (static_cast<uint32_t>(118 + t) << 23) | ((m << (23 - t)) & 0x7FFFFFu));
}
inline uint8_t ref_e5m2_encode(float f) {
    const uint32_t u = f32_bits(f);
    const uint32_t s = (u >> 24) & 0x80u;
    const int e = static_cast<int>((u >> 23) & 0xFFu) - 111;   // rebias 127 -> 16
    const uint32_t m = (u >> 21) & 3u;
    if (e > 30) return static_cast<uint8_t>(s | 0x7Cu);
    if (e <= -4) return static_cast<uint8_t>(s);                 // below the subnormals
    if (e > 0) return static_cast<uint8_t>(s | (static_cast<uint32_t>(e) << 2) | m);
    return static_cast<uint8_t>(s | ((m | 4u) >> -e));
}
inline float ref_e5m2_decode(uint8_t b) {
    const uint32_t s = static_cast<uint32_t>(b & 0x80u) << 24;
    const uint32_t e = (b >> 2) & 0x1Fu, m = b & 3u;
    if (e == 0x1Fu) return bits_f32(s | 0x7F800000u | (m << 21));
    if (e != 0) return bits_f32(s | ((e + 111u) << 23) | (m << 21));
    if (m == 0) return bits_f32(s);
    const int t = top_bit3(m);                                                   // m * 2^-16
    return bits_f32(s | (static_cast<uint32_t>(111 + t) << 23) | ((m << (23 - t)) & 0x7FFFFFu));
}
}  // namespace detail

struct fp8_e4m3_t {
    uint8_t raw_bits;
    fp8_e4m3_t() = default;
    constexpr explicit fp8_e4m3_t(uint8_t raw, bool) : raw_bits(raw) {}
    explicit fp8_e4m3_t(float f) : raw_bits(detail::ref_e4m3_encode(f)) {}
    operator float() const { return detail::ref_e4m3_decode(raw_bits); }
    fp8_e4m3_t& operator=(float f) { return *this = fp8_e4m3_t(f); }
};
static_assert(sizeof(fp8_e4m3_t) == 1, "fp8_e4m3_t is 1 byte");

struct fp8_e5m2_t {
    uint8_t raw_bits;
    fp8_e5m2_t() = default;
    constexpr explicit fp8_e5m2_t(uint8_t raw, bool) : raw_bits(raw) {}
    explicit fp8_e5m2_t(float f) : raw_bits(detail::ref_e5m2_encode(f)) {}
    operator float() const { return detail::ref_e5m2_decode(raw_bits); }
    fp8_e5m2_t& operator=(float f) { return *this = fp8_e5m2_t(f); }
};
static_assert(sizeof(fp8_e5m2_t) == 1, "fp8_e5m2_t is 1 byte");

// Algorithm selector of the explicit-algorithm gemm_fp32 overload.  The
// enumerators keep the reference's order (ABI).  On B200 every value runs the
// GPU plan selector; kNaive is accepted for source compatibility.
enum class GemmAlgo {
    kAuto,
    kNaive,
    kNeonFp32,
    kBf16Bfmmla,
    kInt8Smmla,
    kInt8Sdot,
    kSveFp32,
    kSveBf16,
    kSveInt8,
    kSmeFp32,
    kFp8E4m3Fdot,
    kFp8E5m2Fdot,
    kSveFp8E4m3,
    kSveFp8E5m2,
};

struct GemmBlockingParams {
    int Mr, Nr, Mc, Nc, Kc;
};

}  // namespace dnnopt
