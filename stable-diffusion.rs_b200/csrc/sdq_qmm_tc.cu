// sdq_qmm_tc.cu -- large-M quantised matmul on the 5th-generation tensor cores.
//
// Y[m, n] = X[m, k] . dequant(Wq, S, B)[n, k]^T, the op behind
// QuantizedArray::matmul (crates/sd-tensor/src/mlx.rs:1947-1975) that every
// Flux linear goes through (crates/sd-models/src/mlx/quantized.rs:298-318).
//
// The kernel computes the transposed tile D[f, t] = W_dq[f, :] . X[t, :]^T with
//   * A = the dequantised weight tile, 128 features x 64 k, written straight
//     into TENSOR MEMORY by a dequant warpgroup (tcgen05.st) -- it never
//     passes through shared memory;
//   * B = the activation tile, BT tokens x 64 k bf16, loaded by TMA with
//     128-byte swizzle into shared memory;
//   * D = 128 x BT f32 accumulator in TMEM (tcgen05.mma kind::f16, issued by
//     one thread).
// With tokens on the MMA N side (up to 256), every dequantised weight element
// feeds BT = 256 multiply-adds, which keeps the CUDA-core unpack work at about
// a third of the tensor-core time.  One quantisation group (64 k) is exactly
// one pipeline stage, so each stage needs one scale and one bias per row.
//
// Warp roles (512 threads, one CTA per SM, persistent over tiles):
//   warp 0      TMA producer: X tile + packed W tile per stage (no multicast)
//   warp 1      TMEM allocator and MMA issuer
//   warps 4-11  dequant, two warpgroups taking alternate stages (so that one
//               group's TMEM-store and barrier latency hides behind the
//               other's unpacking); thread r of a group owns feature row r
//   warps 12-15 epilogue: TMEM -> registers -> (+bias) -> bf16 -> global
// Every mbarrier wait is bounded (2 s); on expiry the kernel records a status
// bit, drains its own copies and MMAs, frees TMEM and returns.
#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include "sdq_dequant.cuh"
#include "sdq_internal.h"
#include "sdq_ptx.cuh"

namespace sdq {

// Status word for this file's kernels (see sdq_ptx.cuh).
__device__ unsigned int g_tc_status = 0;

namespace {

template <int BITS, int BT, int STAGES>
struct TcCfg {
    static constexpr int BF = 128;                         // features per tile = MMA M
    static constexpr int BK = 64;                          // k per stage = one group
    static constexpr int X_STAGE = BT * BK * 2;            // bytes, 128 B per token row
    static constexpr int W_ROW = BK * BITS / 8;            // packed bytes per feature row
    static constexpr int W_STAGE = BF * W_ROW;
    static constexpr int TX_BYTES = X_STAGE + W_STAGE;
    static constexpr int W_WORDS = BK * BITS / 32;         // packed words per row per stage
    static constexpr uint32_t D_COL = 0;                   // accumulator columns [0, BT)
    static constexpr uint32_t A_COL = 256;                 // A slots: 32 columns each
    static constexpr uint32_t TMEM_COLS = 512;
    static constexpr int SMEM_BYTES = 1024 + STAGES * (X_STAGE + W_STAGE) + 256;
    static_assert(BT % 16 == 0 && BT >= 16 && BT <= 256, "MMA N must be 16..256, step 16");
    static_assert(STAGES * 32 <= 256, "A slots must fit beside the accumulator");
    static_assert(STAGES % 2 == 0, "the two dequant warpgroups alternate stages");
};

template <int BITS, int BT, int STAGES>
__global__ void __launch_bounds__(512, 1)
    qmm_tc_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                  const uint16_t* __restrict__ scales, const uint16_t* __restrict__ biases,
                  const uint16_t* __restrict__ bias, uint16_t* __restrict__ y, int M, int N, int K) {
    using C = TcCfg<BITS, BT, STAGES>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t* sX = smem;                                  // STAGES x X_STAGE (1024-aligned)
    uint8_t* sW = smem + STAGES * C::X_STAGE;            // STAGES x W_STAGE
    uint64_t* bars = reinterpret_cast<uint64_t*>(sW + STAGES * C::W_STAGE);
    uint64_t* full = bars;                // TMA landed (X + W)            count 1 + tx
    uint64_t* afull = bars + STAGES;      // A slot written               count 128
    uint64_t* done = bars + 2 * STAGES;   // MMAs of the stage finished    count 1 (commit)
    uint64_t* dfull = bars + 3 * STAGES;  // accumulator complete          count 1 (commit)
    uint64_t* dempty = dfull + 1;         // accumulator drained           count 128
    uint64_t* drain = dfull + 2;          // abort drain of the MMA pipe   count 1 (commit)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    unsigned int* status = &g_tc_status;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(full + s, 1);
            mbar_init(afull + s, 128);
            mbar_init(done + s, 1);
        }
        mbar_init(dfull, 1);
        mbar_init(dempty, 128);
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmX);
        tma_prefetch_desc(&tmW);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const int nft = (N + C::BF - 1) / C::BF;
    const int ntt = (M + BT - 1) / BT;
    const int ntiles = nft * ntt;
    const int KT = K / C::BK;

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            int it = 0;
            int last_phase[STAGES];
            bool issued[STAGES];
            for (int s = 0; s < STAGES; ++s) { issued[s] = false; last_phase[s] = 0; }
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
                const int tt = tile / nft, ft = tile - tt * nft;
                for (int kt = 0; kt < KT; ++kt, ++it) {
                    const int s = it % STAGES;
                    const uint32_t ph = (it / STAGES) & 1;
                    if (!mbar_wait(done + s, ph ^ 1, abort_flag, status, 1u)) { ok = false; break; }
                    mbar_arrive_expect_tx(full + s, C::TX_BYTES);
                    tma_load_2d(sX + s * C::X_STAGE, &tmX, full + s, kt * C::BK, tt * BT);
                    tma_load_2d(sW + s * C::W_STAGE, &tmW, full + s, kt * C::W_WORDS, ft * C::BF);
                    issued[s] = true;
                    last_phase[s] = (int)ph;
                }
            }
            if (!ok) {
                // Let every copy this CTA started land before shared memory goes away.
                for (int s = 0; s < STAGES; ++s)
                    if (issued[s]) mbar_wait_drain(full + s, (uint32_t)last_phase[s]);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t idesc = idesc_bf16_f32(C::BF, BT);
            int it = 0, tc = 0;
            bool ok = true, any = false;
            for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x, ++tc) {
                if (!mbar_wait(dempty, (tc & 1) ^ 1, abort_flag, status, 2u)) { ok = false; break; }
                tc_fence_after();
                for (int kt = 0; kt < KT; ++kt, ++it) {
                    const int s = it % STAGES;
                    const uint32_t ph = (it / STAGES) & 1;
                    if (!mbar_wait(full + s, ph, abort_flag, status, 2u)) { ok = false; break; }
                    if (!mbar_wait(afull + s, ph, abort_flag, status, 2u)) { ok = false; break; }
                    tc_fence_after();
                    const uint64_t bdesc = smem_desc_sw128(smem_u32(sX + s * C::X_STAGE));
#pragma unroll
                    for (int j = 0; j < C::BK / 16; ++j) {
                        // K step of 16 bf16 = 32 bytes inside the swizzled row (+2 in
                        // 16-byte descriptor units); A advances 8 TMEM columns.
                        tc_mma_ts(tmem + C::D_COL, tmem + C::A_COL + 32u * s + 8u * j,
                                  bdesc + 2ull * j, idesc, (kt | j) != 0);
                    }
                    any = true;
                    tc_commit(done + s);
                }
                if (!ok) break;
                tc_commit(dfull);
            }
            if (!ok && any) {
                tc_commit(drain);
                mbar_wait_drain(drain, 0);
            }
        }
    } else if (warp >= 4 && warp < 12) {
        // ------------------------------------------------------------ dequant
        const int grp_id = (warp - 4) >> 2;                   // takes stages with it % 2 == grp_id
        const int r = (threadIdx.x - 128) & 127;              // feature row in the tile
        const uint32_t lane_base = static_cast<uint32_t>(32 * (warp & 3)) << 16;
        const int G = K / 64;
        int it = 0;
        bool ok = true;
        for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
            const int tt = tile / nft, ft = tile - tt * nft;
            (void)tt;
            const int row = ft * C::BF + r;
            const bool valid = row < N;
            const uint16_t* srow = scales + (int64_t)(valid ? row : 0) * G;
            const uint16_t* brow = biases + (int64_t)(valid ? row : 0) * G;
            for (int kt = 0; kt < KT; ++kt, ++it) {
                if ((it & 1) != grp_id) continue;
                const int s = it % STAGES;
                const uint32_t ph = (it / STAGES) & 1;
                const uint32_t sb = valid ? (uint32_t)__ldg(srow + kt) : 0u;
                const uint32_t bb = valid ? (uint32_t)__ldg(brow + kt) : 0u;
                if (!mbar_wait(full + s, ph, abort_flag, status, 4u)) { ok = false; break; }
                if (!mbar_wait(done + s, ph ^ 1, abort_flag, status, 4u)) { ok = false; break; }
                tc_fence_after();
                uint32_t a[32];
                const uint4* wrow = reinterpret_cast<const uint4*>(sW + s * C::W_STAGE + r * C::W_ROW);
                if (BITS == 4) {
                    const uint32_t s2 = sb * 0x10001u, b2 = bb * 0x10001u;
#pragma unroll
                    for (int v = 0; v < 2; ++v) {
                        const uint4 q = wrow[v];
                        const uint32_t wv[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                        for (int w = 0; w < 4; ++w) {
                            uint32_t o[4];
                            dq4_word_natural(wv[w], s2, b2, o);
#pragma unroll
                            for (int j = 0; j < 4; ++j) a[4 * (4 * v + w) + j] = o[j];
                        }
                    }
                } else {
                    const float sf = bf16_bits_to_f32(sb), bf = bf16_bits_to_f32(bb);
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        const uint4 q = wrow[v];
                        const uint32_t wv[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                        for (int w = 0; w < 4; ++w) {
                            uint32_t o[2];
                            dq8_word_natural(wv[w], sf, bf, o);
                            a[2 * (4 * v + w)] = o[0];
                            a[2 * (4 * v + w) + 1] = o[1];
                        }
                    }
                }
                tmem_st32(tmem + lane_base + C::A_COL + 32u * s, a);
                tc_wait_st();
                tc_fence_before();
                mbar_arrive(afull + s);
            }
        }
    } else if (warp >= 12) {
        // ------------------------------------------------------------ epilogue
        const uint32_t lane_base = static_cast<uint32_t>(32 * (warp & 3)) << 16;
        int tc = 0;
        for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++tc) {
            const int tt = tile / nft, ft = tile - tt * nft;
            if (!mbar_wait(dfull, tc & 1, abort_flag, status, 8u)) break;
            tc_fence_after();
            const int f = ft * C::BF + 32 * (warp & 3) + lane;
            const bool fvalid = f < N;
            const float badd = (bias != nullptr && fvalid) ? bf16_bits_to_f32(bias[f]) : 0.f;
#pragma unroll 1
            for (int c = 0; c < BT / 32; ++c) {
                uint32_t v[32];
                tmem_ld32(tmem + lane_base + C::D_COL + 32u * c, v);
                tc_wait_ld();
                const int t0 = tt * BT + 32 * c;
                if (fvalid) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const int t = t0 + i;
                        if (t < M) {
                            const float val = __uint_as_float(v[i]) + badd;
                            y[(int64_t)t * N + f] = (uint16_t)(pack_bf16x2(val, 0.f) & 0xFFFFu);
                        }
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(dempty);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

// ---------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 get_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

template <int BITS, int BT, int STAGES>
cudaError_t launch_tc_t(const void* x, int64_t m, int64_t k, const uint32_t* wq, const void* scales,
                        const void* biases, int64_t n, const void* bias, void* y, cudaStream_t st,
                        const char** msg) {
    using C = TcCfg<BITS, BT, STAGES>;
    auto enc = get_encoder();
    if (!enc) {
        *msg = "cuTensorMapEncodeTiled is unavailable from the driver";
        return cudaErrorNotSupported;
    }
    CUtensorMap tmX, tmW;
    {
        cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)m};
        cuuint64_t strides[1] = {(cuuint64_t)k * 2};
        cuuint32_t box[2] = {(cuuint32_t)C::BK, (cuuint32_t)BT};
        cuuint32_t estr[2] = {1, 1};
        CUresult r = enc(&tmX, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) {
            *msg = "cuTensorMapEncodeTiled rejected the activation tensor map";
            return cudaErrorInvalidValue;
        }
    }
    {
        cuuint64_t dims[2] = {(cuuint64_t)(k * BITS / 32), (cuuint64_t)n};
        cuuint64_t strides[1] = {(cuuint64_t)(k * BITS / 8)};
        cuuint32_t box[2] = {(cuuint32_t)C::W_WORDS, (cuuint32_t)C::BF};
        cuuint32_t estr[2] = {1, 1};
        CUresult r = enc(&tmW, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint32_t*>(wq), dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) {
            *msg = "cuTensorMapEncodeTiled rejected the packed-weight tensor map";
            return cudaErrorInvalidValue;
        }
    }
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static bool configured[64] = {};
    if (dev < 64 && !configured[dev]) {
        e = cudaFuncSetAttribute(qmm_tc_kernel<BITS, BT, STAGES>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    const int64_t tiles = ((n + 127) / 128) * ((m + BT - 1) / BT);
    const int grid = (int)(tiles < num_sms() ? tiles : num_sms());
    qmm_tc_kernel<BITS, BT, STAGES><<<grid, 512, C::SMEM_BYTES, st>>>(
        tmX, tmW, static_cast<const uint16_t*>(scales), static_cast<const uint16_t*>(biases),
        static_cast<const uint16_t*>(bias), static_cast<uint16_t*>(y), (int)m, (int)n, (int)k);
    return cudaGetLastError();
}

template <int BITS>
cudaError_t launch_tc_bits(const void* x, int64_t m, int64_t k, const uint32_t* wq,
                           const void* scales, const void* biases, int64_t n, const void* bias,
                           void* y, cudaStream_t st, const char** msg) {
    // Tokens per tile: the smallest of 64 / 128 / 256 that covers M, so short
    // activations do not pay for empty MMA columns.
    if (m <= 64) return launch_tc_t<BITS, 64, 4>(x, m, k, wq, scales, biases, n, bias, y, st, msg);
    if (m <= 128) return launch_tc_t<BITS, 128, 4>(x, m, k, wq, scales, biases, n, bias, y, st, msg);
    return launch_tc_t<BITS, 256, 4>(x, m, k, wq, scales, biases, n, bias, y, st, msg);
}

}  // namespace

cudaError_t launch_qmm_tc(const void* x, int64_t m, int64_t k, const uint32_t* wq,
                          const void* scales, const void* biases, int64_t n, int bits,
                          const void* bias, void* y, cudaStream_t st, const char** msg) {
    return bits == 4 ? launch_tc_bits<4>(x, m, k, wq, scales, biases, n, bias, y, st, msg)
                     : launch_tc_bits<8>(x, m, k, wq, scales, biases, n, bias, y, st, msg);
}

cudaError_t read_and_clear_status(unsigned int* out, cudaStream_t st) {
    cudaError_t e = cudaMemcpyFromSymbolAsync(out, g_tc_status, sizeof(unsigned int), 0,
                                              cudaMemcpyDeviceToHost, st);
    if (e != cudaSuccess) return e;
    e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return e;
    if (*out != 0) {
        const unsigned int zero = 0;
        e = cudaMemcpyToSymbolAsync(g_tc_status, &zero, sizeof(unsigned int), 0,
                                    cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    }
    return e;
}

}  // namespace sdq
