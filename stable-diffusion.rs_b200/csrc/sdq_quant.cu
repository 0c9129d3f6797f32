// sdq_quant.cu -- affine group-wise quantise/pack and dequantise kernels.
//
// Quantise (replaces mlx_quantize behind QuantizedArray::quantize,
// crates/sd-tensor/src/mlx.rs:1861-1911): one warp per group of 64 weights
// along K; each lane owns two consecutive weights.  Group extrema come from a
// 5-step warp-shuffle reduction under a total order (-0 < +0, NaN ignored), so
// the result does not depend on the reduction tree.  The packed words are
// assembled with two more shuffle steps and written coalesced.
//
// Dequantise (replaces mlx_dequantize behind QuantizedArray::dequantize,
// mlx.rs:1918-1945): one thread per packed word, vector stores.
//
// Scales and biases may be stored bf16 or f32 (the reference's callers hold f32).  The
// quantiser's values are bf16 either way (the rule rounds them), widened exactly when stored
// as f32; f32 scales read by the dequantiser and the matmul are rounded to bf16 (nearest
// even), which leaves the quantiser's own values unchanged.
//
// f32 -> bf16 conversion (the matmul's pre-pass for f32 activations or scales): 8 values
// per thread, round to nearest even, NaN -> 0x7fff.
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "sdq_dequant.cuh"
#include "sdq_quant.cuh"
#include "sdq_internal.h"

namespace sdq {

template <int BITS, bool IN_BF16, bool SB_F32>
__global__ void __launch_bounds__(256) quantize_kernel(const void* __restrict__ w, int64_t n,
                                                       int64_t k, uint32_t* __restrict__ wq,
                                                       void* __restrict__ scales,
                                                       void* __restrict__ biases) {
    const int lane = threadIdx.x & 31;
    const int64_t groups_per_row = k / 64;
    const int64_t total = n * groups_per_row;
    const int64_t warp0 = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x / 32);
    const int64_t wstride = (int64_t)gridDim.x * (blockDim.x / 32);

    for (int64_t gi = warp0; gi < total; gi += wstride) {
        const int64_t row = gi / groups_per_row;
        const int64_t g = gi - row * groups_per_row;
        const int64_t e0 = row * k + g * 64 + 2 * lane;
        float v0, v1;
        if (IN_BF16) {
            const uint32_t pair = __ldg(reinterpret_cast<const uint32_t*>(
                static_cast<const __nv_bfloat16*>(w) + e0));
            v0 = bf16_bits_to_f32(pair & 0xFFFFu);
            v1 = bf16_bits_to_f32(pair >> 16);
        } else {
            const float2 p = __ldg(reinterpret_cast<const float2*>(static_cast<const float*>(w) + e0));
            v0 = p.x;
            v1 = p.y;
        }
        quantize_group_warp<BITS, SB_F32>(v0, v1, lane, gi, row, g, k, wq, scales, biases);
    }
}

// Scale / bias element i as bf16 bits.
template <bool SB_F32>
__device__ __forceinline__ uint32_t sb_bits(const void* p, int64_t i) {
    if (SB_F32) return f32_to_bf16_rne(static_cast<const float*>(p)[i]);
    return static_cast<const uint16_t*>(p)[i];
}

template <int BITS, bool OUT_F32, bool SB_F32>
__global__ void __launch_bounds__(256) dequantize_kernel(const uint32_t* __restrict__ wq,
                                                         const void* __restrict__ scales,
                                                         const void* __restrict__ biases,
                                                         int64_t n, int64_t k, void* __restrict__ out) {
    constexpr int PER = 32 / BITS;  // elements per word
    const int64_t words_per_row = k / PER;
    const int64_t total = n * words_per_row;
    const int64_t groups_per_row = k / 64;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = i / words_per_row;
        const int64_t wi = i - row * words_per_row;
        const int64_t g = row * groups_per_row + (wi * PER) / 64;
        const uint32_t sbits = sb_bits<SB_F32>(scales, g);
        const uint32_t bbits = sb_bits<SB_F32>(biases, g);
        const uint32_t w = __ldg(wq + i);
        const int64_t e0 = row * k + wi * PER;
        if (BITS == 4) {
            uint32_t o[4];
            dq4_word_natural(w, sbits | (sbits << 16), bbits | (bbits << 16), o);
            if (OUT_F32) {
                float4* dst = reinterpret_cast<float4*>(static_cast<float*>(out) + e0);
                dst[0] = make_float4(__uint_as_float(o[0] << 16), __uint_as_float(o[0] & 0xFFFF0000u),
                                     __uint_as_float(o[1] << 16), __uint_as_float(o[1] & 0xFFFF0000u));
                dst[1] = make_float4(__uint_as_float(o[2] << 16), __uint_as_float(o[2] & 0xFFFF0000u),
                                     __uint_as_float(o[3] << 16), __uint_as_float(o[3] & 0xFFFF0000u));
            } else {
                *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(out) + e0) =
                    make_uint4(o[0], o[1], o[2], o[3]);
            }
        } else {
            uint32_t o[2];
            dq8_word_natural(w, bf16_bits_to_f32(sbits), bf16_bits_to_f32(bbits), o);
            if (OUT_F32) {
                *reinterpret_cast<float4*>(static_cast<float*>(out) + e0) =
                    make_float4(__uint_as_float(o[0] << 16), __uint_as_float(o[0] & 0xFFFF0000u),
                                __uint_as_float(o[1] << 16), __uint_as_float(o[1] & 0xFFFF0000u));
            } else {
                *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(out) + e0) = make_uint2(o[0], o[1]);
            }
        }
    }
}

static int grid_for(int64_t work, int threads, int per_sm_blocks) {
    const int64_t want = (work + threads - 1) / threads;
    const int64_t cap = (int64_t)num_sms() * per_sm_blocks;
    return (int)(want < cap ? (want > 0 ? want : 1) : cap);
}

cudaError_t launch_quantize(const void* w, bool w_bf16, int64_t n, int64_t k, int bits,
                            uint32_t* wq, void* scales, void* biases, bool sb_f32, cudaStream_t st) {
    const int64_t groups = n * (k / 64);
    const int grid = grid_for(groups * 32, 256, 8);
    auto go = [&](auto kern) { kern<<<grid, 256, 0, st>>>(w, n, k, wq, scales, biases); };
    if (bits == 4) {
        if (w_bf16) sb_f32 ? go(quantize_kernel<4, true, true>) : go(quantize_kernel<4, true, false>);
        else sb_f32 ? go(quantize_kernel<4, false, true>) : go(quantize_kernel<4, false, false>);
    } else {
        if (w_bf16) sb_f32 ? go(quantize_kernel<8, true, true>) : go(quantize_kernel<8, true, false>);
        else sb_f32 ? go(quantize_kernel<8, false, true>) : go(quantize_kernel<8, false, false>);
    }
    return cudaGetLastError();
}

cudaError_t launch_dequantize(const uint32_t* wq, const void* scales, const void* biases, bool sb_f32,
                              int64_t n, int64_t k, int bits, void* out, bool out_f32, cudaStream_t st) {
    const int64_t words = n * k * bits / 32;
    const int grid = grid_for(words, 256, 8);
    auto go = [&](auto kern) { kern<<<grid, 256, 0, st>>>(wq, scales, biases, n, k, out); };
    if (bits == 4) {
        if (out_f32) sb_f32 ? go(dequantize_kernel<4, true, true>) : go(dequantize_kernel<4, true, false>);
        else sb_f32 ? go(dequantize_kernel<4, false, true>) : go(dequantize_kernel<4, false, false>);
    } else {
        if (out_f32) sb_f32 ? go(dequantize_kernel<8, true, true>) : go(dequantize_kernel<8, true, false>);
        else sb_f32 ? go(dequantize_kernel<8, false, true>) : go(dequantize_kernel<8, false, false>);
    }
    return cudaGetLastError();
}

__global__ void __launch_bounds__(256) f32_to_bf16_kernel(const float* __restrict__ in,
                                                          uint16_t* __restrict__ out, int64_t count) {
    const int64_t n8 = count / 8;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8;
         i += (int64_t)gridDim.x * blockDim.x) {
        const float4 a = reinterpret_cast<const float4*>(in)[2 * i];
        const float4 b = reinterpret_cast<const float4*>(in)[2 * i + 1];
        uint4 o;
        o.x = f32_to_bf16_rne(a.x) | (f32_to_bf16_rne(a.y) << 16);
        o.y = f32_to_bf16_rne(a.z) | (f32_to_bf16_rne(a.w) << 16);
        o.z = f32_to_bf16_rne(b.x) | (f32_to_bf16_rne(b.y) << 16);
        o.w = f32_to_bf16_rne(b.z) | (f32_to_bf16_rne(b.w) << 16);
        reinterpret_cast<uint4*>(out)[i] = o;
    }
    // The tail of a count that is not a multiple of 8, one value per thread.
    for (int64_t i = n8 * 8 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count;
         i += (int64_t)gridDim.x * blockDim.x)
        out[i] = (uint16_t)f32_to_bf16_rne(in[i]);
}

cudaError_t launch_f32_to_bf16(const float* in, void* out, int64_t count, cudaStream_t st) {
    const int grid = grid_for(count / 8 + 1, 256, 8);
    f32_to_bf16_kernel<<<grid, 256, 0, st>>>(in, static_cast<uint16_t*>(out), count);
    return cudaGetLastError();
}

}  // namespace sdq
