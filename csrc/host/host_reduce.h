// Reduction math of the host-memory path.
//
// Parity: the reference's Utils::ReduceData / PerformReduce / ApplyAverage
// (OriginCCL src/utils.cpp:312-410): SUM/MAX/MIN element-wise, AVG = SUM then divide the
// final value by the rank count (integer division for integer types). bf16 and fp16 are
// widened to fp32, reduced and rounded once (round to nearest even), as on the GPU.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cstring>

#include "bccl/types.h"

namespace bccl {
namespace hostmath {

inline float Bf16ToFloat(uint16_t b) {
    uint32_t u = static_cast<uint32_t>(b) << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

inline uint16_t FloatToBf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return static_cast<uint16_t>((u >> 16) | 0x40);  // quiet NaN
    u += 0x7fffu + ((u >> 16) & 1u);
    return static_cast<uint16_t>(u >> 16);
}

// IEEE binary16 <-> binary32 from the format definition (1 sign, 5 exponent, 10 fraction bits).
inline float HalfToFloat(uint16_t h) {
    const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1fu;
    const uint32_t frac = h & 0x3ffu;
    uint32_t u;
    if (exp == 0) {
        if (frac == 0) {
            u = sign;
        } else {  // subnormal: frac * 2^-24, renormalise
            int e = -1;
            uint32_t m = frac;
            do {
                ++e;
                m <<= 1;
            } while ((m & 0x400u) == 0);
            u = sign | static_cast<uint32_t>(127 - 15 - e) << 23 | ((m & 0x3ffu) << 13);
        }
    } else if (exp == 31) {
        u = sign | 0x7f800000u | (frac << 13);
    } else {
        u = sign | ((exp + 112u) << 23) | (frac << 13);
    }
    float f;
    memcpy(&f, &u, 4);
    return f;
}

inline uint16_t FloatToHalf(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    const uint16_t sign = static_cast<uint16_t>((u >> 16) & 0x8000u);
    const uint32_t exp = (u >> 23) & 0xffu;
    uint32_t mant = u & 0x7fffffu;
    if (exp == 0xff) return static_cast<uint16_t>(sign | 0x7c00u | (mant ? 0x200u : 0));
    int e = static_cast<int>(exp) - 127 + 15;
    if (e >= 31) return static_cast<uint16_t>(sign | 0x7c00u);  // overflow -> inf
    if (e <= 0) {
        if (e < -10) return sign;  // underflow -> signed zero
        mant |= 0x800000u;         // implicit bit
        const int shift = 14 - e;  // to a 10-bit subnormal fraction
        uint32_t q = mant >> shift;
        const uint32_t rem = mant & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1u))) ++q;
        return static_cast<uint16_t>(sign | q);
    }
    uint32_t q = mant >> 13;
    const uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) ++q;
    uint32_t out = (static_cast<uint32_t>(e) << 10) + q;  // a carry out of q bumps the exponent
    if (out >= 0x7c00u) out = 0x7c00u;
    return static_cast<uint16_t>(sign | out);
}

// dst[i] = epilogue(reduce_p srcs[p][i]) for p in [0, n), in order. dst may alias srcs[0].
// When `final` is false the AVG division and the scale are not applied (partial sums).
void Reduce(DataType dtype, ReduceOp op, void* dst, const void* const* srcs, int n, size_t count, int nranks,
            float scale, bool final);
// dst[i] = epilogue(src[i]) (AVG division / scale only).
void Finish(DataType dtype, ReduceOp op, void* dst, const void* src, size_t count, int nranks, float scale);

}  // namespace hostmath
}  // namespace bccl
