// sdq_qmv.cu -- small-M quantised matmul (1 <= M <= 8): Y = X . dequant(W)^T.
//
// The adaLN modulation linears of the Flux transformer run at M = batch = 1
// (crates/sd-models/src/mlx/flux.rs:279-299); there the layer is bound by
// reading the packed weight once from HBM, so the kernel is a weight stream:
//
//   * every lane issues 128-bit non-allocating loads (16 B = 4 packed words)
//     of two weight rows, kept P items ahead in a register ring so that about
//     64 KB per SM are in flight;
//   * the words are dequantised in registers (the same exact s*q + b rule as
//     the dequantise kernel) straight into m16n8k16 tensor-core fragments, so
//     the reduction over K happens inside the tensor core instead of a chain
//     of per-lane FMAs (at M = 8 a CUDA-core dot product would need 8 FMAs
//     per weight and could not keep up with HBM);
//   * X (M <= 8 rows, zero-padded to 8) is staged once per CTA in shared
//     memory, pre-permuted into the fragment order that matches the packed
//     nibble order, so the unpack needs no byte shuffles;
//   * two warps split K for each 16-row block and combine their partial sums
//     through shared memory (named barriers), which doubles the warps per SM
//     available to hide HBM latency.
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "sdq_dequant.cuh"
#include "sdq_internal.h"

namespace sdq {
namespace {

constexpr int kSlots = 8;            // 16-row blocks in flight per CTA
constexpr int kKSplit = 2;           // warps per row block (K halves)
constexpr int kThreads = 32 * kSlots * kKSplit;
constexpr int kRing = 4;             // items (128-bit load pairs) in flight per lane

template <int BITS>
struct QmvCfg {
    static constexpr int KB = BITS == 4 ? 128 : 64;   // k per block (16 words per row)
    static constexpr int RPL = BITS == 4 ? 16 : 8;    // bf16x2 regs per row per lane per block
    static constexpr int NMMA = RPL / 2;              // m16n8k16 per block
    static constexpr int CH = RPL / 4;                // uint4 chunks of X fragments per lane
};

// Fragment register r of quad lane t holds two k of the block (lo, hi half):
//   W4: word w = r / 4 of the lane's 16 bytes, nibbles (j, j+4), j = r % 4:
//       k = 32 t + 8 w + j and k + 4;
//   W8: word w = r / 2, bytes (2j, 2j+1), j = r % 2: k = 16 t + 4 w + 2 j and k + 1.
// The activation fragments are staged in shared memory in the same order.

__device__ __forceinline__ uint4 ld_stream_v4(const uint32_t* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                               uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

struct Item {
    uint4 wg, wh;      // 16 bytes of row g and of row g + 8
    uint32_t sbg, sbh; // scale | bias << 16 (bf16 bits) for those rows
};

template <int BITS>
__global__ void __launch_bounds__(kThreads, 1)
    qmv_kernel(const uint16_t* __restrict__ x, int m, int k, const uint32_t* __restrict__ wq,
               const uint16_t* __restrict__ scales, const uint16_t* __restrict__ biases, int n,
               const uint16_t* __restrict__ bias, uint16_t* __restrict__ y) {
    using C = QmvCfg<BITS>;
    extern __shared__ __align__(16) uint4 xs[];   // [nblk][CH][32 lanes]
    __shared__ float red[kSlots][32][4];

    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int slot = warp % kSlots;
    const int half = warp / kSlots;
    const int g = lane >> 2, t = lane & 3;

    const int nblk = k / C::KB;
    // Split K between the two warps of a slot only when both get a block;
    // otherwise warp half 0 takes everything and no barrier is used.
    const bool split = nblk >= 2;
    const int blk_lo = half == 0 ? 0 : (split ? nblk / 2 : nblk);
    const int blk_hi = half == 0 ? (split ? nblk / 2 : nblk) : nblk;
    const int my_blks = blk_hi - blk_lo;
    const int nrb = (n + 15) / 16;
    const int rb_first = blockIdx.x * kSlots + slot;
    const int rb_stride = gridDim.x * kSlots;
    const int my_rbs = rb_first < nrb ? (nrb - rb_first + rb_stride - 1) / rb_stride : 0;
    const int total = my_rbs * my_blks;
    const int64_t wpr = (int64_t)k * BITS / 32;   // words per row
    const int groups = k / 64;

    auto load_item = [&](int it, Item& d) {
        if (it >= total) return;
        const int q = it / my_blks;
        const int blk = blk_lo + (it - q * my_blks);
        const int rb = rb_first + q * rb_stride;
        const int rg = rb * 16 + g, rh = rg + 8;
        const int grp = BITS == 4 ? 2 * blk + (t >> 1) : blk;
        const int64_t off = (int64_t)blk * 16 + 4 * t;
        if (rg < n) {
            d.wg = ld_stream_v4(wq + (int64_t)rg * wpr + off);
            d.sbg = (uint32_t)__ldg(scales + (int64_t)rg * groups + grp) |
                    ((uint32_t)__ldg(biases + (int64_t)rg * groups + grp) << 16);
        } else {
            d.wg = make_uint4(0, 0, 0, 0);
            d.sbg = 0;
        }
        if (rh < n) {
            d.wh = ld_stream_v4(wq + (int64_t)rh * wpr + off);
            d.sbh = (uint32_t)__ldg(scales + (int64_t)rh * groups + grp) |
                    ((uint32_t)__ldg(biases + (int64_t)rh * groups + grp) << 16);
        } else {
            d.wh = make_uint4(0, 0, 0, 0);
            d.sbh = 0;
        }
    };

    // Start the weight stream before staging X so the first HBM round trips
    // overlap the staging.
    Item ring[kRing];
#pragma unroll
    for (int p = 0; p < kRing; ++p) load_item(p, ring[p]);

    // Stage X (zero-padded to 8 rows) in fragment order: one 16-byte load of 8
    // consecutive k and one 16-byte shared store per thread and step.  An aligned
    // run of 8 k lands in the four components of one lane's uint4 chunk
    // (W4: halves (j, j+4); W8: natural pairs).
    {
        const int chunks_per_row = k / 8;
        const int total_chunks = 8 * chunks_per_row;
        for (int i = threadIdx.x; i < total_chunks; i += kThreads) {
            const int tok = i / chunks_per_row;
            const int kc = (i - tok * chunks_per_row) * 8;       // first k of the run
            const int blk = kc / C::KB;
            const int kk = kc - blk * C::KB;                     // offset inside the block
            int t, c;
            if (BITS == 4) { t = kk >> 5; c = (kk & 31) >> 3; }
            else { t = kk >> 4; c = (kk & 15) >> 3; }
            uint4 v = make_uint4(0, 0, 0, 0);
            if (tok < m) {
                const uint4 raw = *reinterpret_cast<const uint4*>(x + (int64_t)tok * k + kc);
                if (BITS == 4) {
                    // raw = e0e1 e2e3 e4e5 e6e7 -> (e0,e4) (e1,e5) (e2,e6) (e3,e7)
                    v.x = prmt(raw.x, raw.z, 0x5410u);
                    v.y = prmt(raw.x, raw.z, 0x7632u);
                    v.z = prmt(raw.y, raw.w, 0x5410u);
                    v.w = prmt(raw.y, raw.w, 0x7632u);
                } else {
                    v = raw;
                }
            }
            xs[((int64_t)blk * C::CH + c) * 32 + tok * 4 + t] = v;
        }
    }
    __syncthreads();

    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int base = 0; base < total; base += kRing) {
#pragma unroll
        for (int p = 0; p < kRing; ++p) {
            const int it = base + p;
            if (it < total) {
                const Item cur = ring[p];
                load_item(it + kRing, ring[p]);
                const int q = it / my_blks;
                const int bi = it - q * my_blks;
                const int blk = blk_lo + bi;

                uint32_t ag[C::RPL], ah[C::RPL];
                const uint32_t wg[4] = {cur.wg.x, cur.wg.y, cur.wg.z, cur.wg.w};
                const uint32_t wh[4] = {cur.wh.x, cur.wh.y, cur.wh.z, cur.wh.w};
                if (BITS == 4) {
                    const uint32_t sg2 = (cur.sbg & 0xFFFFu) * 0x10001u, bg2 = (cur.sbg >> 16) * 0x10001u;
                    const uint32_t sh2 = (cur.sbh & 0xFFFFu) * 0x10001u, bh2 = (cur.sbh >> 16) * 0x10001u;
#pragma unroll
                    for (int w = 0; w < 4; ++w) {
                        uint32_t o[4];
                        dq4_word_interleaved(wg[w], sg2, bg2, o);
#pragma unroll
                        for (int j = 0; j < 4; ++j) ag[4 * w + j] = o[j];
                        dq4_word_interleaved(wh[w], sh2, bh2, o);
#pragma unroll
                        for (int j = 0; j < 4; ++j) ah[4 * w + j] = o[j];
                    }
                } else {
                    const float sg = bf16_bits_to_f32(cur.sbg & 0xFFFFu), bg = bf16_bits_to_f32(cur.sbg >> 16);
                    const float sh = bf16_bits_to_f32(cur.sbh & 0xFFFFu), bh = bf16_bits_to_f32(cur.sbh >> 16);
#pragma unroll
                    for (int w = 0; w < 4; ++w) {
                        uint32_t o[2];
                        dq8_word_natural(wg[w], sg, bg, o);
                        ag[2 * w] = o[0];
                        ag[2 * w + 1] = o[1];
                        dq8_word_natural(wh[w], sh, bh, o);
                        ah[2 * w] = o[0];
                        ah[2 * w + 1] = o[1];
                    }
                }
                const uint4* xb = xs + (int64_t)blk * C::CH * 32 + lane;
#pragma unroll
                for (int c = 0; c < C::CH; ++c) {
                    const uint4 xv = xb[c * 32];
                    const uint32_t xr[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int i = 2 * c + h;  // mma index: regs 2i, 2i+1
                        const uint32_t a[4] = {ag[2 * i], ah[2 * i], ag[2 * i + 1], ah[2 * i + 1]};
                        mma_bf16_16816(acc, a, xr[2 * h], xr[2 * h + 1]);
                    }
                }

                if (bi == my_blks - 1) {
                    // Row block done: combine the two K halves, add bias, store.
                    const int rb = rb_first + q * rb_stride;
                    if (split && half == 1) {
#pragma unroll
                        for (int e = 0; e < 4; ++e) red[slot][lane][e] = acc[e];
                    }
                    if (split) asm volatile("bar.sync %0, %1;" ::"r"(slot + 1), "r"(64) : "memory");
                    if (half == 0) {
                        if (split) {
#pragma unroll
                            for (int e = 0; e < 4; ++e) acc[e] += red[slot][lane][e];
                        }
                        const int rows[2] = {rb * 16 + g, rb * 16 + g + 8};
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const int row = rows[e >> 1];
                            const int tok = 2 * t + (e & 1);
                            if (row < n && tok < m) {
                                float v = acc[e];
                                if (bias) v += bf16_bits_to_f32(bias[row]);
                                y[(int64_t)tok * n + row] =
                                    (uint16_t)(pack_bf16x2(v, 0.f) & 0xFFFFu);
                            }
                        }
                    }
                    if (split) asm volatile("bar.sync %0, %1;" ::"r"(slot + 1), "r"(64) : "memory");
#pragma unroll
                    for (int e = 0; e < 4; ++e) acc[e] = 0.f;
                }
            }
        }
    }
}

template <int BITS>
cudaError_t launch_qmv_t(const void* x, int m, int64_t k, const uint32_t* wq, const void* scales,
                         const void* biases, int64_t n, const void* bias, void* y,
                         cudaStream_t st) {
    using C = QmvCfg<BITS>;
    const int nblk = (int)(k / C::KB);
    const size_t smem = (size_t)nblk * C::CH * 32 * sizeof(uint4);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static bool configured[64] = {};
    if (dev < 64 && !configured[dev]) {
        e = cudaFuncSetAttribute(qmv_kernel<BITS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 200 * 1024);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    const int64_t nrb = (n + 15) / 16;
    int64_t grid = (nrb + kSlots - 1) / kSlots;
    if (grid > num_sms()) grid = num_sms();
    qmv_kernel<BITS><<<(int)grid, kThreads, smem, st>>>(
        static_cast<const uint16_t*>(x), m, (int)k, wq, static_cast<const uint16_t*>(scales),
        static_cast<const uint16_t*>(biases), (int)n, static_cast<const uint16_t*>(bias),
        static_cast<uint16_t*>(y));
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_qmv(const void* x, int m, int64_t k, const uint32_t* wq, const void* scales,
                       const void* biases, int64_t n, int bits, const void* bias, void* y,
                       cudaStream_t st) {
    return bits == 4 ? launch_qmv_t<4>(x, m, k, wq, scales, biases, n, bias, y, st)
                     : launch_qmv_t<8>(x, m, k, wq, scales, biases, n, bias, y, st);
}

}  // namespace sdq
