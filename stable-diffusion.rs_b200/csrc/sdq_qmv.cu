// sdq_qmv.cu -- small-M quantised matmul (1 <= M <= 8): Y = X . dequant(Wq, S, B)^T.
//
// The adaLN modulation linears of the Flux transformer run at M = batch
// (crates/sd-models/src/mlx/flux.rs:279-299, through quantized::linear,
// crates/sd-models/src/mlx/quantized.rs:298-318).  At M <= 8 the layer is a
// stream of the packed weight from HBM, so this kernel is built around
// keeping that stream saturated with as few instructions per packed word as
// possible:
//
//   * one producer thread streams the packed weights with TMA into a deep
//     shared-memory ring (128 KB in flight per SM); a stage is one box of TR
//     rows x 128 bytes (256 k for W4, 128 k for W8) with 128-byte swizzle --
//     128-byte rows keep the copy engine's per-row request rate well above
//     what HBM delivers, which 32-byte rows (one group of W4) did not;
//   * X is loaded whole at kernel start, one bulk copy per token row, into rows
//     padded to 2K + 16 bytes (a pitch that keeps the B-fragment reads of the
//     8 tokens on distinct banks), and stays resident; rows past M are zeroed;
//   * 16 consumer warps feed the tensor core the raw codes: a nibble n becomes
//     the bf16 value 128 + n with one lop3 (exact), and each group's
//     m16n8k16 MMAs give T = sum_k x_k (128 + q_k) per (row, token); the
//     group's affine map is then applied once in f32,
//         y += s * T + (b - 128 s) * sum_k x_k,
//     with the per-group sums of X precomputed at kernel start.  W8 splits a
//     byte into two nibbles and runs two MMAs (T = 16 T_hi + T_lo, offset
//     2176).  This is the exact affine value s*q + b of every weight, without
//     the bf16 rounding that the dequantise op applies, so the result is within
//     bf16 rounding of the dense product of the dequantised weights -- the
//     matmul is held to a tolerance, not to bits;
//   * warp w owns 16 rows of the TR-row tile (slice w % RS, RS = TR/16) and
//     every KP-th group of K (KP = 16/RS); at the end of a tile the KP partial
//     sums of a slice are added through shared memory in a fixed order, which
//     is the cross-warp reduction step, and the first warp writes Y.
//
// Fragment mapping (lane = 4 g + t): in step kt, lane t of a quad takes
// k0 = 64 kt + 16 t and the 16 k from there, of rows g and g + 8 of its slice.
// W4: the nibble pairs (j, j + 4) of a word are fragment column pairs, so X is
// permuted in place once, inside every 8-run, to (0,4,1,5,2,6,3,7); W8: the
// pairs are (k, k + 2) and X's 4-runs become (0,2,1,3).  Each lane's B
// fragments are then 32 contiguous bytes of its token's (permuted) X row.
//
// The scales and biases of a stage (TR rows x its groups) travel with it: the
// producer warp's lanes copy them with cp.async into a slot beside the weight
// stage and the same full barrier counts their arrival, so they are prefetched
// as deep as the weights.
//
// Every mbarrier wait is bounded (see sdq_ptx.cuh); a timed-out wait sets a
// status bit, the consumers leave together at the next tile boundary and the
// producer drains its copies before the CTA exits.
#include <cstdint>
#include <cstring>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include "sdq_dequant.cuh"
#include "sdq_epilogue.cuh"
#include "sdq_internal.h"
#include "sdq_ptx.cuh"

namespace sdq {

__device__ unsigned int g_qmv_status = 0;

namespace {

constexpr int kConsumerWarps = 16;
constexpr int kThreads = 32 * (kConsumerWarps + 1);   // + the producer warp

template <int BITS, int TR>
struct QmvCfg {
    static constexpr int RS = TR / 16;                 // row slices per tile
    static constexpr int KP = kConsumerWarps / RS;     // k phases (warps per slice)
    static constexpr int W_ROW = 64 * BITS / 8;        // packed bytes per row per step
    static constexpr int SPB = 128 / W_ROW;            // steps per stage (128-byte rows)
    static constexpr int STAGE = TR * 128;             // one box: TR rows x 128 B
    static constexpr int SW = (128 << 10) / STAGE;     // ring stages: 128 KB
    static constexpr int SB_ROW = SPB * 2;             // bytes of one row's scales in a stage
    static constexpr int SB_STAGE = 2 * TR * SB_ROW;   // scales then biases
    static constexpr float QOFF = BITS == 4 ? 128.f : 2176.f;   // code offset folded into T
    static constexpr int RED = (KP - 1) * RS * 32 * 16;   // partial sums of one tile
    // Warps reading one stage: the RS slices times the k phases among its SPB steps.
    static constexpr int READERS = RS * (KP < SPB ? KP : SPB);
    // Consecutive steps a warp takes per visit of a stage (one wait, one release).
    static constexpr int U = SPB > KP ? SPB / KP : 1;
    static_assert(RS * KP == kConsumerWarps, "warps must tile the slices");
    static_assert(KP % SPB == 0 || SPB % KP == 0, "phases and stage steps must nest");
};

__device__ __forceinline__ uint2 lds64(const uint8_t* p) {
    return *reinterpret_cast<const uint2*>(p);
}
__device__ __forceinline__ uint4 lds128(const uint8_t* p) {
    return *reinterpret_cast<const uint4*>(p);
}

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_16816_z(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                            uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%10, %10, %10, %10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
}

// Nibble j and j + 4 of a word as bf16x2 (128 + n_j, 128 + n_{j+4}): exact.
template <int J>
__device__ __forceinline__ uint32_t code_pair(uint32_t w) {
    return ((w >> (4 * J)) & 0x000F000Fu) | 0x43004300u;
}

// Row pitch of the resident X in shared memory: 2K + 16 bytes, which is 16 mod 32,
// so the 8 lanes of a quarter-warp (2 tokens x 4 quads) read 8 distinct 16-byte
// bank groups.
__host__ __device__ constexpr size_t x_pitch(int64_t k) { return (size_t)k * 2 + 16; }
__host__ __device__ constexpr size_t x_bytes(int64_t k) { return (8 * x_pitch(k) + 1023) & ~(size_t)1023; }

// Smem bytes for a configuration: alignment slack, resident X, ring, two
// partial-sum buffers, per-group X sums, barriers.
template <class C>
size_t qmv_smem_bytes(int64_t k) {
    return 1024 + x_bytes(k) + (size_t)C::SW * (C::STAGE + C::SB_STAGE) + 2 * (size_t)C::RED +
           (size_t)(k / 64) * 32 + (size_t)C::SW * 16 + 64;
}

template <int BITS, int TR>
__global__ void __launch_bounds__(kThreads, 1)
    qmv_kernel(const __grid_constant__ CUtensorMap tmW, const uint16_t* __restrict__ x,
               const uint16_t* __restrict__ scales, const uint16_t* __restrict__ biases,
               const EpiArgs epi, void* y, int M, int N, int K) {
    using C = QmvCfg<BITS, TR>;
    constexpr int SW = C::SW;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const int KT = K / 64;
    const int XP = (int)x_pitch(K);
    uint8_t* sX = smem;                                           // [8 tokens][XP]
    uint8_t* sW = sX + x_bytes(K);                                // [SW][TR][128 B], swizzled
    uint8_t* sSB = sW + (size_t)SW * C::STAGE;                    // [SW][2][TR][SPB] bf16
    float4* red = reinterpret_cast<float4*>(sSB + (size_t)SW * C::SB_STAGE);   // [2][KP-1][RS][32]
    float* xsum = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(red) + 2 * C::RED);  // [4][KT][2]
    uint64_t* wfull = reinterpret_cast<uint64_t*>(xsum + (size_t)KT * 8);
    uint64_t* wempty = wfull + SW;
    uint64_t* xfull = wempty + SW;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(xfull + 1);
    unsigned int* status = &g_qmv_status;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int ntiles = (N + TR - 1) / TR;
    const int stages_per_tile = KT / C::SPB;
    const int G = KT;                                             // groups per row

    if (threadIdx.x == 0) {
        for (int i = 0; i < SW; ++i) {
            mbar_init(wfull + i, 1 + 32);                         // expect-tx + 32 cp.async lanes
            mbar_init(wempty + i, C::READERS);                    // one lane per reading warp
        }
        mbar_init(xfull, 1);
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmW);
    }
    __syncthreads();
    // Programmatic dependent launch: the next kernel of the stream may launch now (it waits
    // in its own griddep_wait()); nothing an earlier kernel writes is read before ours.
    griddep_launch_dependents();
    griddep_wait();

    if (warp == kConsumerWarps) {
        // ------------------------------------------------------------ producer
        // Lane 0 issues the copies of X and of each weight stage; all 32 lanes copy
        // the stage's scales and biases and arrive on its full barrier through
        // cp.async, so the barrier completes when all of the stage has landed.
        if (lane == 0) {
            mbar_arrive_expect_tx(xfull, (uint32_t)(M * 2 * K));
            for (int tok = 0; tok < M; ++tok)
                bulk_load(sX + (size_t)tok * XP, x + (int64_t)tok * K, (uint32_t)(2 * K), xfull);
        }
        int it = 0, last_it = -1;
        bool ok = true;
        const bool withhold = g_withhold_first_copy != 0;       // testing hook, normally false
        for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
            for (int sg = 0; sg < stages_per_tile; ++sg, ++it) {
                const int s = it % SW;
                if (!__all_sync(0xffffffffu, mbar_wait_sleep(wempty + s, ((it / SW) & 1) ^ 1,
                                                             abort_flag, status, 1u, 32))) { ok = false; break; }
                if (lane == 0 && !(withhold && it == 0)) {
                    mbar_arrive_expect_tx(wfull + s, C::STAGE);
                    tma_load_2d(sW + (size_t)s * C::STAGE, &tmW, wfull + s, sg * 32, tile * TR);
                }
                uint8_t* sb = sSB + (size_t)s * C::SB_STAGE;
                for (int r = lane; r < TR; r += 32) {
                    const int row = tile * TR + r;
                    const bool in = row < N;
                    const int64_t off = (int64_t)(in ? row : 0) * G + sg * C::SPB;
                    cp_async<C::SB_ROW>(sb + r * C::SB_ROW, scales + off, in ? C::SB_ROW : 0);
                    cp_async<C::SB_ROW>(sb + (TR + r) * C::SB_ROW, biases + off, in ? C::SB_ROW : 0);
                }
                cp_async_arrive(wfull + s);
                last_it = it;
            }
        }
        cp_async_wait_all();
        // Every copy this warp started must land before shared memory goes away.
        if (lane == 0) {
            mbar_wait_drain(xfull, 0);
            if (!ok) {
                for (int j = last_it; j >= 0 && j > last_it - SW; --j)
                    mbar_wait_drain(wfull + j % SW, (uint32_t)((j / SW) & 1));
            }
        }
    } else {
        // ------------------------------------------------------------ consumers
        const int c = warp % C::RS;          // row slice
        const int h = warp / C::RS;          // k phase: steps kt = h, h + KP, ...
        const int g = lane >> 2, t = lane & 3;
        bool ok = mbar_wait_warp(xfull, 0, abort_flag, status, 2u);
        if (ok) {
            // One (group, token) run of 64 values per thread: sum it, then permute each
            // 16-byte chunk in place into the fragment order of the unpack.  Tokens past
            // M were not copied: their runs are zeroed.
            for (int rr = threadIdx.x; rr < KT * 8; rr += 32 * kConsumerWarps) {
                const int tok = rr & 7;
                uint8_t* run = sX + (size_t)tok * XP + (size_t)(rr >> 3) * 128;
                float sum = 0.f;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    uint4 v = make_uint4(0, 0, 0, 0);
                    if (tok < M) v = *reinterpret_cast<uint4*>(run + 16 * j);
                    const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        sum += bf16_bits_to_f32(vv[q] & 0xFFFFu) + bf16_bits_to_f32(vv[q] >> 16);
                    if (BITS == 4)
                        v = make_uint4(prmt(vv[0], vv[2], 0x5410u), prmt(vv[0], vv[2], 0x7632u),
                                       prmt(vv[1], vv[3], 0x5410u), prmt(vv[1], vv[3], 0x7632u));
                    else
                        v = make_uint4(prmt(vv[0], vv[1], 0x5410u), prmt(vv[0], vv[1], 0x7632u),
                                       prmt(vv[2], vv[3], 0x5410u), prmt(vv[2], vv[3], 0x7632u));
                    *reinterpret_cast<uint4*>(run + 16 * j) = v;
                }
                xsum[((tok >> 1) * KT + (rr >> 3)) * 2 + (tok & 1)] = sum;
            }
        }
        ok = named_barrier_and(9, 32 * kConsumerWarps, ok);
        int tile_stage0 = 0;                 // ring index of the current tile's first stage
        int tcount = 0;
        for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++tcount) {
            const int r0 = tile * TR + 16 * c + g, r1 = r0 + 8;
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            // Unit v covers steps [U v, U v + U); this warp takes v = h, h + KP, ...
            for (int v = h; ok && v * C::U < KT; v += C::KP) {
                const int kt0 = v * C::U;
                const int sg = kt0 / C::SPB, sp0 = kt0 - sg * C::SPB;   // stage of the tile, step in it
                const int it = tile_stage0 + sg;
                const int s = it % SW;
                // The warp's last unit in the stage releases it.
                const bool last = (v + C::KP) * C::U >= (sg + 1) * C::SPB || (v + C::KP) * C::U >= KT;
                if (!mbar_wait_warp_parked(wfull + s, (it / SW) & 1, abort_flag, status, 4u, 20000u)) { ok = false; break; }
                const uint16_t* sb = reinterpret_cast<const uint16_t*>(sSB + (size_t)s * C::SB_STAGE);
                const uint8_t* row0 = sW + (size_t)s * C::STAGE + (16 * c + g) * 128;
                const uint8_t* row1 = row0 + 8 * 128;
                // Scales / biases of rows g and g + 8 for the U steps (zero past N).
                uint32_t sr[4];
                if (C::U == 2) {
                    sr[0] = *reinterpret_cast<const uint32_t*>(sb + (16 * c + g) * C::SPB + sp0);
                    sr[1] = *reinterpret_cast<const uint32_t*>(sb + (16 * c + g + 8) * C::SPB + sp0);
                    sr[2] = *reinterpret_cast<const uint32_t*>(sb + (TR + 16 * c + g) * C::SPB + sp0);
                    sr[3] = *reinterpret_cast<const uint32_t*>(sb + (TR + 16 * c + g + 8) * C::SPB + sp0);
                } else {
                    sr[0] = sb[(16 * c + g) * C::SPB + sp0];
                    sr[1] = sb[(16 * c + g + 8) * C::SPB + sp0];
                    sr[2] = sb[(TR + 16 * c + g) * C::SPB + sp0];
                    sr[3] = sb[(TR + 16 * c + g + 8) * C::SPB + sp0];
                }
                // Packed weights of the U steps, read before the stage is released.
                constexpr int WV = BITS == 4 ? 2 : 4;        // words per row per step
                uint32_t wa[C::U][WV], wb[C::U][WV];
#pragma unroll
                for (int u = 0; u < C::U; ++u) {
                    const int sp = sp0 + u;
                    if (BITS == 4) {
                        const int off = (((2 * sp + (t >> 1)) ^ g) << 4) + 8 * (t & 1);
                        const uint2 p0 = lds64(row0 + off), p1 = lds64(row1 + off);
                        wa[u][0] = p0.x; wa[u][1] = p0.y; wb[u][0] = p1.x; wb[u][1] = p1.y;
                    } else {
                        const int off = ((4 * sp + t) ^ g) << 4;
                        const uint4 p0 = lds128(row0 + off), p1 = lds128(row1 + off);
                        wa[u][0] = p0.x; wa[u][1] = p0.y; wa[u][2] = p0.z; wa[u][3] = p0.w;
                        wb[u][0] = p1.x; wb[u][1] = p1.y; wb[u][2] = p1.z; wb[u][3] = p1.w;
                    }
                }
                // Per-group X sums of tokens 2t and 2t + 1 for the U steps.
                float xg[2 * C::U];
                if (C::U == 2) {
                    const float4 q = *reinterpret_cast<const float4*>(xsum + (t * KT + kt0) * 2);
                    xg[0] = q.x; xg[1] = q.y; xg[2] = q.z; xg[3] = q.w;
                } else {
                    const float2 q = *reinterpret_cast<const float2*>(xsum + (t * KT + kt0) * 2);
                    xg[0] = q.x; xg[1] = q.y;
                }
#pragma unroll
                for (int u = 0; u < C::U; ++u) {
                    const int kt = kt0 + u;
                    const uint8_t* xs = sX + (size_t)g * XP + (size_t)kt * 128 + 32 * t;
                    const uint4 x0 = lds128(xs);
                    const uint4 x1 = lds128(xs + 16);
                    float T[4];
                    if (BITS == 4) {
                        mma_16816_z(T, code_pair<0>(wa[u][0]), code_pair<0>(wb[u][0]), code_pair<1>(wa[u][0]),
                                    code_pair<1>(wb[u][0]), x0.x, x0.y);
                        mma_16816(T, code_pair<2>(wa[u][0]), code_pair<2>(wb[u][0]), code_pair<3>(wa[u][0]),
                                  code_pair<3>(wb[u][0]), x0.z, x0.w);
                        mma_16816(T, code_pair<0>(wa[u][1]), code_pair<0>(wb[u][1]), code_pair<1>(wa[u][1]),
                                  code_pair<1>(wb[u][1]), x1.x, x1.y);
                        mma_16816(T, code_pair<2>(wa[u][1]), code_pair<2>(wb[u][1]), code_pair<3>(wa[u][1]),
                                  code_pair<3>(wb[u][1]), x1.z, x1.w);
                    } else {
                        float L[4], H[4];
                        // Low nibbles -> L, high nibbles -> H; word w pairs with X pairs of x[w].
                        const uint32_t xb[4][2] = {{x0.x, x0.y}, {x0.z, x0.w}, {x1.x, x1.y}, {x1.z, x1.w}};
                        mma_16816_z(L, code_pair<0>(wa[u][0]), code_pair<0>(wb[u][0]), code_pair<2>(wa[u][0]),
                                    code_pair<2>(wb[u][0]), xb[0][0], xb[0][1]);
                        mma_16816_z(H, code_pair<1>(wa[u][0]), code_pair<1>(wb[u][0]), code_pair<3>(wa[u][0]),
                                    code_pair<3>(wb[u][0]), xb[0][0], xb[0][1]);
#pragma unroll
                        for (int w = 1; w < 4; ++w) {
                            mma_16816(L, code_pair<0>(wa[u][w]), code_pair<0>(wb[u][w]), code_pair<2>(wa[u][w]),
                                      code_pair<2>(wb[u][w]), xb[w][0], xb[w][1]);
                            mma_16816(H, code_pair<1>(wa[u][w]), code_pair<1>(wb[u][w]), code_pair<3>(wa[u][w]),
                                      code_pair<3>(wb[u][w]), xb[w][0], xb[w][1]);
                        }
#pragma unroll
                        for (int i = 0; i < 4; ++i) T[i] = fmaf(16.f, H[i], L[i]);
                    }
                    // This step's scale / bias of rows g and g + 8 (halves of sr for U = 2).
                    const float sf0 = __uint_as_float(u == 0 ? sr[0] << 16 : sr[0] & 0xFFFF0000u);
                    const float sf1 = __uint_as_float(u == 0 ? sr[1] << 16 : sr[1] & 0xFFFF0000u);
                    const float bo0 = fmaf(-C::QOFF, sf0, __uint_as_float(u == 0 ? sr[2] << 16 : sr[2] & 0xFFFF0000u));
                    const float bo1 = fmaf(-C::QOFF, sf1, __uint_as_float(u == 0 ? sr[3] << 16 : sr[3] & 0xFFFF0000u));
                    // T: (row g, token 2t), (row g, 2t+1), (row g+8, 2t), (row g+8, 2t+1)
                    acc[0] = fmaf(sf0, T[0], fmaf(bo0, xg[2 * u], acc[0]));
                    acc[1] = fmaf(sf0, T[1], fmaf(bo0, xg[2 * u + 1], acc[1]));
                    acc[2] = fmaf(sf1, T[2], fmaf(bo1, xg[2 * u], acc[2]));
                    acc[3] = fmaf(sf1, T[3], fmaf(bo1, xg[2 * u + 1], acc[3]));
                }
                // Release the stage only once its words (read by the MMAs above) and its
                // scales (tied in through zero_after) have been read back.
                const uint32_t dep = zero_after(sr[0], sr[1], sr[2], sr[3]);
                __syncwarp();
                if (last && lane == 0) mbar_arrive(wempty + s + dep);
            }
            // A warp that gave up still reaches the barrier; the vote makes the
            // whole slice leave together.
            float4* rb = red + (size_t)(tcount & 1) * (C::RED / 16);
            if (h > 0) rb[((h - 1) * C::RS + c) * 32 + lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
            if (!named_barrier_and(1 + c, 32 * C::KP, ok)) { ok = false; break; }
            if (h == 0) {
                for (int p = 1; p < C::KP; ++p) {      // fixed order: deterministic sums
                    const float4 v = rb[((p - 1) * C::RS + c) * 32 + lane];
                    acc[0] += v.x; acc[1] += v.y; acc[2] += v.z; acc[3] += v.w;
                }
                // y = resid + gate * act(acc + bias), rounded once (null terms drop out).
                const int m0i = 2 * t, m1i = 2 * t + 1;
                auto put = [&](float a, int tok, int row) {
                    if (row >= N || tok >= M) return;
                    const int64_t o = (int64_t)tok * N + row;
                    if (epi.f32) {          // f32 output, f32 bias (plain output stage only)
                        if (epi.bias != nullptr) a += reinterpret_cast<const float*>(epi.bias)[row];
                        static_cast<float*>(y)[o] = a;
                        return;
                    }
                    a += epi.bias != nullptr ? bf16_bits_to_f32(epi.bias[row]) : 0.f;
                    a = epi_activation(a, epi.act);
                    if (epi.gate != nullptr) a *= bf16_bits_to_f32(epi.gate[row]);
                    if (epi.resid != nullptr) a += bf16_bits_to_f32(epi.resid[o]);
                    static_cast<uint16_t*>(y)[o] = (uint16_t)(pack_bf16x2(a, 0.f) & 0xFFFFu);
                };
                put(acc[0], m0i, r0);
                put(acc[1], m1i, r0);
                put(acc[2], m0i, r1);
                put(acc[3], m1i, r1);
            }
            tile_stage0 += stages_per_tile;
        }
    }
    __syncthreads();
}

template <int BITS, int TR>
cudaError_t launch_t(const void* x, int64_t m, int64_t k, const uint32_t* wq, const void* scales,
                     const void* biases, int64_t n, const EpiArgs& epi, void* y,
                     cudaStream_t st, const char** msg) {
    using C = QmvCfg<BITS, TR>;
    auto enc = tensor_map_encoder();
    if (!enc) {
        *msg = "cuTensorMapEncodeTiled is unavailable from the driver";
        return cudaErrorNotSupported;
    }
    CUtensorMap tmW;
    {
        cuuint64_t dims[2] = {(cuuint64_t)(k * BITS / 32), (cuuint64_t)n};
        cuuint64_t strides[1] = {(cuuint64_t)(k * BITS / 8)};
        cuuint32_t box[2] = {32, (cuuint32_t)TR};
        cuuint32_t estr[2] = {1, 1};
        CUresult r = enc(&tmW, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint32_t*>(wq), dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) {
            *msg = "cuTensorMapEncodeTiled rejected the packed-weight tensor map";
            return cudaErrorInvalidValue;
        }
    }
    const size_t smem = qmv_smem_bytes<C>(k);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static bool configured[64] = {};
    if (dev < 64 && !configured[dev]) {
        e = cudaFuncSetAttribute(qmv_kernel<BITS, TR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kQmvMaxSmem);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    const int64_t tiles = (n + TR - 1) / TR;
    const int grid = (int)(tiles < num_sms() ? tiles : num_sms());
    // Launched with programmatic stream serialisation, so that back-to-back layers overlap
    // this kernel's set-up with the previous kernel's tail.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, qmv_kernel<BITS, TR>, tmW, static_cast<const uint16_t*>(x),
                              static_cast<const uint16_t*>(scales), static_cast<const uint16_t*>(biases), epi,
                              y, (int)m, (int)n, (int)k);
}

template <int BITS, int TR>
bool fits(int64_t k) {
    return qmv_smem_bytes<QmvCfg<BITS, TR>>(k) <= kQmvMaxSmem;
}

// Tile rows: the largest of 128 / 64 / 32 / 16 whose tile count fills the SMs
// as evenly as the smaller ones would (whole waves of equal tiles).
int pick_rows(int64_t n) {
    const int sms = num_sms();
    int best = 0;
    double best_eff = -1.0;
    for (int tr : {128, 64, 32, 16}) {
        const int64_t tiles = (n + tr - 1) / tr;
        const int64_t waves = (tiles + sms - 1) / sms;
        const double eff = (double)tiles / (double)(waves * sms);
        if (eff > best_eff + 1e-9) {
            best_eff = eff;
            best = tr;
        }
    }
    return best;
}

template <int BITS>
cudaError_t launch_bits(const void* x, int64_t m, int64_t k, const uint32_t* wq, const void* scales,
                        const void* biases, int64_t n, const EpiArgs& epi, void* y, cudaStream_t st,
                        const char** msg, bool* taken) {
    // A stage is 128 bytes of every row: K must be a whole number of stages; a
    // stage's scales of one row are copied as one 8-byte (W4) / 4-byte (W8) piece.
    const size_t sb_align = BITS == 4 ? 8 : 4;
    if ((k * BITS / 8) % 128 != 0 || reinterpret_cast<uintptr_t>(scales) % sb_align != 0 ||
        reinterpret_cast<uintptr_t>(biases) % sb_align != 0) {
        *taken = false;
        return cudaSuccess;
    }
    const int tr = pick_rows(n);
    const bool ok = tr == 128 ? fits<BITS, 128>(k) : tr == 64 ? fits<BITS, 64>(k)
                  : tr == 32 ? fits<BITS, 32>(k) : fits<BITS, 16>(k);
    if (!ok) {
        *taken = false;        // X does not fit beside the 128 KB ring: not this kernel's shape
        return cudaSuccess;
    }
    *taken = true;
    switch (tr) {
        case 128: return launch_t<BITS, 128>(x, m, k, wq, scales, biases, n, epi, y, st, msg);
        case 64: return launch_t<BITS, 64>(x, m, k, wq, scales, biases, n, epi, y, st, msg);
        case 32: return launch_t<BITS, 32>(x, m, k, wq, scales, biases, n, epi, y, st, msg);
        default: return launch_t<BITS, 16>(x, m, k, wq, scales, biases, n, epi, y, st, msg);
    }
}

}  // namespace

cudaError_t launch_qmv(const void* x, bool x_f32, int64_t m, int64_t k, const uint32_t* wq,
                       const void* scales, const void* biases, bool sb_f32, int64_t n, int bits,
                       const EpiArgs& epi, void* y, bool y_f32, cudaStream_t st, const char** msg,
                       bool* taken) {
    *taken = false;
    // bf16 activations, scales and biases (the C ABI converts f32 ones first); bf16 or f32 output.
    if (m < 1 || m > 8 || x_f32 || sb_f32 || y_f32 != epi.f32) return cudaSuccess;
    return bits == 4 ? launch_bits<4>(x, m, k, wq, scales, biases, n, epi, y, st, msg, taken)
                     : launch_bits<8>(x, m, k, wq, scales, biases, n, epi, y, st, msg, taken);
}

cudaError_t set_wait_hook_qmv(unsigned long long limit_ns, int withhold, cudaStream_t st) {
    cudaError_t e = cudaMemcpyToSymbolAsync(g_wait_limit_ns, &limit_ns, sizeof(limit_ns), 0,
                                            cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess)
        e = cudaMemcpyToSymbolAsync(g_withhold_first_copy, &withhold, sizeof(withhold), 0,
                                    cudaMemcpyHostToDevice, st);
    return e == cudaSuccess ? cudaStreamSynchronize(st) : e;
}

cudaError_t read_and_clear_qmv_status(unsigned int* out, cudaStream_t st) {
    cudaError_t e = cudaMemcpyFromSymbolAsync(out, g_qmv_status, sizeof(unsigned int), 0,
                                              cudaMemcpyDeviceToHost, st);
    if (e != cudaSuccess) return e;
    e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return e;
    if (*out != 0) {
        const unsigned int zero = 0;
        e = cudaMemcpyToSymbolAsync(g_qmv_status, &zero, sizeof(unsigned int), 0,
                                    cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    }
    return e;
}

}  // namespace sdq
