// sdq_gguf.cu -- GGUF tensors straight into the affine quantised format, on the GPU.
//
// The reference loads a GGUF checkpoint by dequantising every tensor to f32 on the host
// (crates/sd-tensor/src/mlx_gguf.rs:235-435) and then quantising the large ones with
// QuantizedArray::quantize (crates/sd-models/src/mlx/quantized.rs:180-211).  Here the raw
// block bytes of one tensor are copied to the device and one kernel does both steps: each
// warp decodes one 64-value group with the reference's f32 arithmetic (no fused
// multiply-adds: every product and difference is rounded as the reference's Rust code
// rounds it) and quantises it with the same group quantiser as sdq_quantize.  The result is
// bit-identical to dequantise-then-quantise, without the f32 copy of the tensor.  The dense
// dequantisation itself (for tensors that stay dense) is the second kernel.
//
// Block layouts (values per block, bytes), as the reference reads them (mlx_gguf.rs:25-40):
//   Q4_0  32,  18: f16 d, 16 bytes of nibbles (low nibbles values 0-15, high 16-31)
//   Q8_0  32,  34: f16 d, 32 signed bytes
//   Q4_K 256, 144: f16 d, f16 dmin, 12 bytes of 6-bit scale/min pairs, 128 nibble bytes
//   Q5_K 256, 176: Q4_K's header, 32 bytes of fifth bits, 128 nibble bytes
//   Q6_K 256, 210: 128 low-nibble bytes, 64 bytes of high bit pairs, 16 signed scales, f16 d
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "sdq_internal.h"
#include "sdq_quant.cuh"

namespace sdq {
namespace {

__device__ __forceinline__ float f16_at(const uint8_t* p) {
    const uint16_t h = (uint16_t)p[0] | (uint16_t)((uint16_t)p[1] << 8);
    return __half2float(__ushort_as_half(h));      // exact, subnormals included
}

// llama.cpp's get_scale_min_k4 as the reference states it (mlx_gguf.rs:346-360): eight
// 6-bit (scale, min) pairs in twelve bytes, the last four split across bytes.
__device__ __forceinline__ void scale_min_k4(int j, const uint8_t* q, int& sc, int& m) {
    if (j < 4) {
        sc = q[j] & 63;
        m = q[j + 4] & 63;
    } else {
        sc = (q[j + 4] & 0x0f) | ((q[j - 4] >> 6) << 4);
        m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

// Value e (flat row-major index) of a tensor of block type T.
template <int T>
__device__ __forceinline__ float decode(const uint8_t* __restrict__ raw, int64_t e) {
    if constexpr (T == SDQ_GGML_F32) {
        return __ldg(reinterpret_cast<const float*>(raw) + e);
    } else if constexpr (T == SDQ_GGML_F16) {
        return __half2float(__ushort_as_half(__ldg(reinterpret_cast<const unsigned short*>(raw) + e)));
    } else if constexpr (T == SDQ_GGML_BF16) {
        return __uint_as_float((uint32_t)__ldg(reinterpret_cast<const unsigned short*>(raw) + e) << 16);
    } else if constexpr (T == SDQ_GGML_Q4_0) {           // mlx_gguf.rs:325-335
        const uint8_t* blk = raw + (e / 32) * 18;
        const int i = (int)(e % 32);
        const int byte = __ldg(blk + 2 + (i & 15));
        const int q = (i < 16 ? (byte & 0x0f) : (byte >> 4)) - 8;
        return __fmul_rn(f16_at(blk), (float)q);
    } else if constexpr (T == SDQ_GGML_Q8_0) {           // mlx_gguf.rs:337-344
        const uint8_t* blk = raw + (e / 32) * 34;
        const int i = (int)(e % 32);
        return __fmul_rn(f16_at(blk), (float)(int8_t)__ldg(blk + 2 + i));
    } else if constexpr (T == SDQ_GGML_Q4_K || T == SDQ_GGML_Q5_K) {   // mlx_gguf.rs:362-410
        constexpr int BYTES = T == SDQ_GGML_Q4_K ? 144 : 176;
        const uint8_t* blk = raw + (e / 256) * BYTES;
        const int i = (int)(e % 256), j = i / 32, l = i % 32;
        int sc, m;
        scale_min_k4(j, blk + 4, sc, m);
        const float d1 = __fmul_rn(f16_at(blk), (float)sc);
        const float m1 = __fmul_rn(f16_at(blk + 2), (float)m);
        const uint8_t* qs = blk + (T == SDQ_GGML_Q4_K ? 16 : 48);
        int q = (__ldg(qs + (j / 2) * 32 + l) >> (4 * (j & 1))) & 0x0f;
        if constexpr (T == SDQ_GGML_Q5_K) q |= ((__ldg(blk + 16 + l) >> j) & 1) << 4;
        return __fsub_rn(__fmul_rn(d1, (float)q), m1);
    } else {                                              // Q6_K, mlx_gguf.rs:412-435
        const uint8_t* blk = raw + (e / 256) * 210;
        const int i = (int)(e % 256), h = i / 128, r = i % 128, quad = r / 32, l = r % 32, is = l / 16;
        const uint8_t* ql = blk + h * 64;
        const uint8_t* qh = blk + 128 + h * 32;
        const int8_t* sc = reinterpret_cast<const int8_t*>(blk + 192) + h * 8;
        const int lo = quad & 1 ? __ldg(ql + l + 32) : __ldg(ql + l);
        const int q = (((quad & 2) ? (lo >> 4) : (lo & 0x0f)) | (((__ldg(qh + l) >> (2 * quad)) & 3) << 4)) - 32;
        return __fmul_rn(__fmul_rn(f16_at(blk + 208), (float)sc[is + 2 * quad]), (float)q);
    }
}

template <int T, int BITS>
__global__ void __launch_bounds__(256) gguf_quantize_kernel(const uint8_t* __restrict__ raw, int64_t n,
                                                            int64_t k, uint32_t* __restrict__ wq,
                                                            __nv_bfloat16* __restrict__ scales,
                                                            __nv_bfloat16* __restrict__ biases) {
    const int lane = threadIdx.x & 31;
    const int64_t groups_per_row = k / 64;
    const int64_t total = n * groups_per_row;
    const int64_t wstride = (int64_t)gridDim.x * (blockDim.x / 32);
    for (int64_t gi = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x / 32); gi < total; gi += wstride) {
        const int64_t row = gi / groups_per_row;
        const int64_t g = gi - row * groups_per_row;
        const int64_t e0 = row * k + g * 64 + 2 * lane;
        quantize_group_warp<BITS>(decode<T>(raw, e0), decode<T>(raw, e0 + 1), lane, gi, row, g, k, wq,
                                  scales, biases);
    }
}

template <int T, bool OUT_F32>
__global__ void __launch_bounds__(256) gguf_dequantize_kernel(const uint8_t* __restrict__ raw,
                                                              int64_t count, void* __restrict__ out) {
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < count;
         e += (int64_t)gridDim.x * blockDim.x) {
        const float v = decode<T>(raw, e);
        if (OUT_F32)
            static_cast<float*>(out)[e] = v;
        else
            static_cast<uint16_t*>(out)[e] = (uint16_t)f32_to_bf16_rne(v);
    }
}

int grid_for(int64_t items, int per_block) {
    const int64_t want = (items + per_block - 1) / per_block;
    const int64_t cap = (int64_t)num_sms() * 16;
    return (int)(want < cap ? (want > 0 ? want : 1) : cap);
}

template <int T>
cudaError_t launch_type(const uint8_t* raw, int64_t n, int64_t k, int bits, uint32_t* wq, void* s,
                        void* b, cudaStream_t st) {
    const int grid = grid_for(n * (k / 64), 8);
    if (bits == 4)
        gguf_quantize_kernel<T, 4><<<grid, 256, 0, st>>>(raw, n, k, wq, static_cast<__nv_bfloat16*>(s),
                                                         static_cast<__nv_bfloat16*>(b));
    else
        gguf_quantize_kernel<T, 8><<<grid, 256, 0, st>>>(raw, n, k, wq, static_cast<__nv_bfloat16*>(s),
                                                         static_cast<__nv_bfloat16*>(b));
    return cudaGetLastError();
}

template <int T>
cudaError_t launch_deq_type(const uint8_t* raw, int64_t count, void* out, bool f32, cudaStream_t st) {
    const int grid = grid_for(count, 256);
    if (f32)
        gguf_dequantize_kernel<T, true><<<grid, 256, 0, st>>>(raw, count, out);
    else
        gguf_dequantize_kernel<T, false><<<grid, 256, 0, st>>>(raw, count, out);
    return cudaGetLastError();
}

}  // namespace

int gguf_block(int type, int& values, int& bytes) {
    switch (type) {
        case SDQ_GGML_F32: values = 1; bytes = 4; return 1;
        case SDQ_GGML_F16: values = 1; bytes = 2; return 1;
        case SDQ_GGML_BF16: values = 1; bytes = 2; return 1;
        case SDQ_GGML_Q4_0: values = 32; bytes = 18; return 1;
        case SDQ_GGML_Q8_0: values = 32; bytes = 34; return 1;
        case SDQ_GGML_Q4_K: values = 256; bytes = 144; return 1;
        case SDQ_GGML_Q5_K: values = 256; bytes = 176; return 1;
        case SDQ_GGML_Q6_K: values = 256; bytes = 210; return 1;
        default: return 0;
    }
}

cudaError_t launch_gguf_quantize(const void* raw, int type, int64_t n, int64_t k, int bits, uint32_t* wq,
                                 void* scales, void* biases, cudaStream_t st) {
    const uint8_t* r = static_cast<const uint8_t*>(raw);
    switch (type) {
        case SDQ_GGML_F32: return launch_type<SDQ_GGML_F32>(r, n, k, bits, wq, scales, biases, st);
        case SDQ_GGML_F16: return launch_type<SDQ_GGML_F16>(r, n, k, bits, wq, scales, biases, st);
        case SDQ_GGML_BF16: return launch_type<SDQ_GGML_BF16>(r, n, k, bits, wq, scales, biases, st);
        case SDQ_GGML_Q4_0: return launch_type<SDQ_GGML_Q4_0>(r, n, k, bits, wq, scales, biases, st);
        case SDQ_GGML_Q8_0: return launch_type<SDQ_GGML_Q8_0>(r, n, k, bits, wq, scales, biases, st);
        case SDQ_GGML_Q4_K: return launch_type<SDQ_GGML_Q4_K>(r, n, k, bits, wq, scales, biases, st);
        case SDQ_GGML_Q5_K: return launch_type<SDQ_GGML_Q5_K>(r, n, k, bits, wq, scales, biases, st);
        default: return launch_type<SDQ_GGML_Q6_K>(r, n, k, bits, wq, scales, biases, st);
    }
}

cudaError_t launch_gguf_dequantize(const void* raw, int type, int64_t count, void* out, bool out_f32,
                                   cudaStream_t st) {
    const uint8_t* r = static_cast<const uint8_t*>(raw);
    switch (type) {
        case SDQ_GGML_F32: return launch_deq_type<SDQ_GGML_F32>(r, count, out, out_f32, st);
        case SDQ_GGML_F16: return launch_deq_type<SDQ_GGML_F16>(r, count, out, out_f32, st);
        case SDQ_GGML_BF16: return launch_deq_type<SDQ_GGML_BF16>(r, count, out, out_f32, st);
        case SDQ_GGML_Q4_0: return launch_deq_type<SDQ_GGML_Q4_0>(r, count, out, out_f32, st);
        case SDQ_GGML_Q8_0: return launch_deq_type<SDQ_GGML_Q8_0>(r, count, out, out_f32, st);
        case SDQ_GGML_Q4_K: return launch_deq_type<SDQ_GGML_Q4_K>(r, count, out, out_f32, st);
        case SDQ_GGML_Q5_K: return launch_deq_type<SDQ_GGML_Q5_K>(r, count, out, out_f32, st);
        default: return launch_deq_type<SDQ_GGML_Q6_K>(r, count, out, out_f32, st);
    }
}

}  // namespace sdq
