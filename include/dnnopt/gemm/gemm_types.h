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

// The reference's 8-bit float storage types.  Their codecs (bias 8 for e4m3,
// bias 16 for e5m2) are the reference's own, not OCP; the GPU kernels decode
// them bit-exactly.  Only the raw byte is part of the ABI.
struct fp8_e4m3_t {
    uint8_t raw_bits;
    fp8_e4m3_t() = default;
    constexpr explicit fp8_e4m3_t(uint8_t raw, bool) : raw_bits(raw) {}
};
static_assert(sizeof(fp8_e4m3_t) == 1, "fp8_e4m3_t is 1 byte");

struct fp8_e5m2_t {
    uint8_t raw_bits;
    fp8_e5m2_t() = default;
    constexpr explicit fp8_e5m2_t(uint8_t raw, bool) : raw_bits(raw) {}
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
