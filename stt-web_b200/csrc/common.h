// Internal helpers shared by the host-side translation units of libsttb200.
#pragma once

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/stt_b200.h"

namespace stt {

// Records the message as the calling thread's last error and returns `code`.
int set_error(int code, const char* fmt, ...);
void clear_error();

// IEEE-754 binary16 -> binary32 (subnormals, inf and NaN exact): the conversion the Q4
// matmul shader performs with unpack2x16float (crates/stt-wasm/src/wgsl/shader_naive.wgsl:20-23).
static inline float f16_bits_to_f32(uint16_t bits) {
    uint32_t sign = (uint32_t)(bits >> 15) & 1u;
    uint32_t exp = (uint32_t)(bits >> 10) & 0x1Fu;
    uint32_t man = (uint32_t)bits & 0x3FFu;
    uint32_t out;
    if (exp == 0) {
        if (man == 0) {
            out = sign << 31;
        } else {  // man * 2^-24, renormalised
            uint32_t e = 0, m = man;
            while ((m & 0x400u) == 0) { m <<= 1; ++e; }
            out = (sign << 31) | ((113u - e) << 23) | ((m & 0x3FFu) << 13);
        }
    } else if (exp == 31) {
        out = (sign << 31) | (0xFFu << 23) | (man << 13);
    } else {
        out = (sign << 31) | ((exp - 15u + 127u) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &out, 4);
    return f;
}

// The CPU conversion of crates/stt-wasm/src/gguf.rs:45-73, used there for Q4_0 embedding rows
// (gguf.rs:625, 724) and F16 norm weights (gguf.rs:911-914).  It equals the IEEE conversion
// except for subnormal inputs, which it maps to half their value: its exponent
// 127 - (15 + e - 1) (gguf.rs:62) is one below the IEEE one.  Kept bit-for-bit so those call
// sites give the reference's values.
static inline float f16_bits_to_f32_gguf(uint16_t bits) {
    uint32_t exp = (uint32_t)(bits >> 10) & 0x1Fu;
    uint32_t man = (uint32_t)bits & 0x3FFu;
    if (exp == 0 && man != 0) {
        uint32_t sign = (uint32_t)(bits >> 15) & 1u;
        uint32_t e = 1, m = man;
        while ((m & 0x400u) == 0) { m <<= 1; ++e; }
        uint32_t out = (sign << 31) | ((127u - (15u + e - 1u)) << 23) | ((m & 0x3FFu) << 13);
        float f;
        std::memcpy(&f, &out, 4);
        return f;
    }
    return f16_bits_to_f32(bits);
}

// binary32 -> binary16, round to nearest even (numpy.float16 semantics), with subnormals,
// overflow to inf and NaN kept quiet.
static inline uint16_t f32_to_f16_bits_rne(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) {  // inf / nan
        return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u | ((ax >> 13) & 0x3FFu) : 0u));
    }
    if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);  // rounds to >= 65520 -> inf
    if (ax < 0x38800000u) {                                     // below 2^-14: subnormal half
        if (ax < 0x33000000u) return (uint16_t)sign;            // below 2^-25: rounds to 0
        // value = m * 2^(e-150) and the half subnormal unit is 2^-24, so q = m >> (126 - e)
        uint32_t e = ax >> 23;
        uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
        uint32_t rshift = 126u - e;                             // 14 .. 24
        uint32_t q = m >> rshift;
        uint32_t rem = m & ((1u << rshift) - 1u);
        uint32_t half = 1u << (rshift - 1u);
        if (rem > half || (rem == half && (q & 1u))) ++q;
        return (uint16_t)(sign | q);
    }
    // normal half
    uint32_t e = (ax >> 23) - 127u + 15u;
    uint32_t m = ax & 0x7FFFFFu;
    uint32_t q = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) ++q;  // carry may bump the exponent
    return (uint16_t)(sign | q);
}

// binary32 -> bfloat16 bits, round to nearest even (NaN kept quiet).
static inline uint16_t f32_to_bf16_bits_rne(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    if ((x & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((x >> 16) | 0x40u);
    uint32_t lsb = (x >> 16) & 1u;
    x += 0x7FFFu + lsb;
    return (uint16_t)(x >> 16);
}

static inline float bf16_bits_to_f32(uint16_t b) {
    uint32_t x = (uint32_t)b << 16;
    float f;
    std::memcpy(&f, &x, 4);
    return f;
}

// GGML dtype codes accepted by the loader.  The reference knows 0, 1, 2 (gguf.rs:136-144);
// 30 (BF16) is the extension used for bf16 embedding tables.
enum GgmlType : uint32_t { GGML_F32 = 0, GGML_F16 = 1, GGML_Q4_0 = 2, GGML_BF16 = 30 };

}  // namespace stt
