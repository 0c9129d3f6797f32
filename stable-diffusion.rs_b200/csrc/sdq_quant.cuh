// sdq_quant.cuh -- the affine group quantiser shared by the quantise kernels: one warp
// per group of 64 values, lane l holding values 2l and 2l + 1 (crates/sd-tensor/src/mlx.rs:
// 1861-1911 is the call it replaces; the rounding rules are the oracle's).
#pragma once

#include <cstdint>
#include <cuda_bf16.h>

#include "sdq_dequant.cuh"

namespace sdq {

__device__ __forceinline__ bool is_nan_f(float a) { return a != a; }

// Same total order as the oracle's qmin / qmax.
__device__ __forceinline__ float tmin(float a, float b) {
    if (is_nan_f(a)) return b;
    if (is_nan_f(b)) return a;
    if (a < b) return a;
    if (b < a) return b;
    return (__float_as_uint(a) >> 31) ? a : b;
}
__device__ __forceinline__ float tmax(float a, float b) {
    if (is_nan_f(a)) return b;
    if (is_nan_f(b)) return a;
    if (a > b) return a;
    if (b > a) return b;
    return (__float_as_uint(a) >> 31) ? b : a;
}

// Round-half-to-even binary32 -> bf16 bits, NaN -> 0x7fff (the oracle's rule).
__device__ __forceinline__ uint32_t f32_to_bf16_rne(float f) {
    uint32_t u = __float_as_uint(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fffu;
    u += 0x7fffu + ((u >> 16) & 1u);
    return u >> 16;
}

__device__ __forceinline__ uint32_t quant_one(float v, float s, float b, uint32_t qmax) {
    if (s == 0.0f) return 0u;
    const float t = __fdiv_rn(__fsub_rn(v, b), s);
    const float r = rintf(t);
    if (!(r > 0.0f)) return 0u;
    if (r > (float)qmax) return qmax;
    return (uint32_t)r;
}

// Quantise and pack group gi (row `row`, group g of the row, K values per row) from the
// warp's values: extrema by a warp-shuffle reduction under a total order, scale and bias
// rounded to bf16, codes packed little-end into the row's words.  SB_F32 stores the scale
// and bias as f32 (the same rounded values, widened exactly) for callers that hold f32.
template <int BITS, bool SB_F32 = false>
__device__ __forceinline__ void quantize_group_warp(float v0, float v1, int lane, int64_t gi,
                                                    int64_t row, int64_t g, int64_t k,
                                                    uint32_t* __restrict__ wq,
                                                    void* __restrict__ scales,
                                                    void* __restrict__ biases) {
    constexpr uint32_t qmax = (1u << BITS) - 1u;
    float mn = tmin(v0, v1), mx = tmax(v0, v1);
    // An all-NaN pair leaves NaN here; the oracle starts from +inf / -inf,
    // which tmin / tmax reproduce when every value is NaN:
    if (is_nan_f(mn)) { mn = __int_as_float(0x7f800000); mx = __int_as_float(0xff800000); }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        mn = tmin(mn, __shfl_xor_sync(0xffffffffu, mn, off));
        mx = tmax(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    }
    const float scale = __fdiv_rn(__fsub_rn(mx, mn), (float)qmax);
    const uint32_t sb = f32_to_bf16_rne(scale);
    const uint32_t bb = f32_to_bf16_rne(mn);
    const float s = bf16_bits_to_f32(sb);
    const float b = bf16_bits_to_f32(bb);
    const uint32_t q0 = quant_one(v0, s, b, qmax);
    const uint32_t q1 = quant_one(v1, s, b, qmax);
    const int64_t wbase = row * (k * BITS / 32) + g * (64 * BITS / 32);
    if (BITS == 4) {
        // lane l holds elements 2l, 2l+1: byte (l % 4) of word l / 4.
        uint32_t v = (q0 | (q1 << 4)) << (8 * (lane & 3));
        v |= __shfl_xor_sync(0xffffffffu, v, 1);
        v |= __shfl_xor_sync(0xffffffffu, v, 2);
        if ((lane & 3) == 0) wq[wbase + (lane >> 2)] = v;
    } else {
        // lane l holds elements 2l, 2l+1: half (l % 2) of word l / 2.
        uint32_t v = (q0 | (q1 << 8)) << (16 * (lane & 1));
        v |= __shfl_xor_sync(0xffffffffu, v, 1);
        if ((lane & 1) == 0) wq[wbase + (lane >> 1)] = v;
    }
    if (lane == 0) {
        if (SB_F32) {
            static_cast<float*>(scales)[gi] = s;
            static_cast<float*>(biases)[gi] = b;
        } else {
            static_cast<uint16_t*>(scales)[gi] = (uint16_t)sb;
            static_cast<uint16_t*>(biases)[gi] = (uint16_t)bb;
        }
    }
}

}  // namespace sdq
