// sdq_dequant.cuh -- register-level unpack + affine reconstruction shared by
// the dequantise kernel and both matmul kernels, so every path produces the
// same bf16 bits for a dequantised weight.
//
// Exactness: q <= 255 and the scale is bf16 (8 significant bits), so s*q is
// exact in bf16x2 FMA's internal product and in binary32; one fma then rounds
// the exact s*q + b once to bf16.  The binary32 path (fmaf, then
// round-to-nearest-even to bf16) gives the same bits because a sum of two
// binary32 values rounded to 24 bits and then to 8 bits is rounded correctly
// (24 >= 2*8 + 2).  This is the rule the CPU oracle states.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>

namespace sdq {

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}
__device__ __forceinline__ uint32_t bf16x2_fma(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ uint32_t bf16x2_sub(uint32_t a, uint32_t b) {
    uint32_t d;
    // a - b as a*1 + (-b): exact here because both operands and the result are
    // small integers.
    asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(0x3F803F80u), "r"(b ^ 0x80008000u));
    return d;
}
// Two binary32 values -> bf16x2 (lo = a, hi = b), round to nearest even.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    uint32_t d;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
}
__device__ __forceinline__ float bf16_bits_to_f32(uint32_t h16) {
    return __uint_as_float(h16 << 16);
}

constexpr uint32_t kBf16x2_128 = 0x43004300u;  // (128.0, 128.0)

// ---- W4: one packed word (nibbles n0..n7, n0 least significant) -----------
// out[j] = (lo: k=2j, hi: k=2j+1) as bf16x2 of s*q + b.
__device__ __forceinline__ void dq4_word_natural(uint32_t w, uint32_t s2, uint32_t b2,
                                                 uint32_t (&out)[4]) {
    const uint32_t lo = w & 0x0F0F0F0Fu;          // bytes n0 n2 n4 n6
    const uint32_t hi = (w >> 4) & 0x0F0F0F0Fu;   // bytes n1 n3 n5 n7
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        // byte0 <- lo.byte j, byte2 <- hi.byte j; bytes 1 and 3 are masked off.
        const uint32_t sel = (uint32_t)j | ((uint32_t)j << 4) | ((uint32_t)(4 + j) << 8) |
                             ((uint32_t)(4 + j) << 12);
        const uint32_t t = (prmt(lo, hi, sel) & 0x00FF00FFu) | kBf16x2_128;  // 128 + q
        out[j] = bf16x2_fma(bf16x2_sub(t, kBf16x2_128), s2, b2);
    }
}

// ---- W8: one packed word (bytes q0..q3, q0 least significant) --------------
// Natural order: out[0] = (q0, q1), out[1] = (q2, q3).  q does not fit a bf16
// magic-number mantissa, so it is widened through binary32, two lanes at a
// time with the packed f32x2 instructions: (2^23 + q) - 2^23 is exact, then
// one fma per value rounds the exact s*q + b to binary32, and the final
// conversion rounds it once more to bf16 (innocuous: 24 >= 2*8 + 2 bits).
__device__ __forceinline__ uint64_t f32x2_sub(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f32x2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t f32x2_dup(float v) {
    const uint64_t u = __float_as_uint(v);
    return u | (u << 32);
}
__device__ __forceinline__ void dq8_word_natural(uint32_t w, float s, float b,
                                                 uint32_t (&out)[2]) {
    constexpr uint64_t kMagic2 = 0x4B0000004B000000ull;   // (2^23, 2^23)
    const uint64_t s2 = f32x2_dup(s), b2 = f32x2_dup(b);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        // byte0 <- w.byte(2h / 2h+1), bytes 1,2 <- 0x00, byte3 <- 0x4B  => 2^23 + q
        const uint32_t lo = prmt(w, 0x4B000000u, (uint32_t)(2 * h) | 0x7440u);
        const uint32_t hi = prmt(w, 0x4B000000u, (uint32_t)(2 * h + 1) | 0x7440u);
        const uint64_t q2 = f32x2_sub((uint64_t)lo | ((uint64_t)hi << 32), kMagic2);
        const uint64_t r = f32x2_fma(s2, q2, b2);
        out[h] = pack_bf16x2(__uint_as_float((uint32_t)r), __uint_as_float((uint32_t)(r >> 32)));
    }
}

}  // namespace sdq
