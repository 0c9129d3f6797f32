// sdq_qmm_tc.cu -- quantised matmul on the 5th-generation tensor cores.
//
// Y[m, n] = X[m, k] . dequant(Wq, S, B)[n, k]^T, the op behind
// QuantizedArray::matmul (crates/sd-tensor/src/mlx.rs:1947-1975) that every
// Flux linear goes through (crates/sd-models/src/mlx/quantized.rs:298-318).
//
// The kernel computes the transposed tile D[f, t] = W_dq[f, :] . X[t, :]^T with
//   * A = the dequantised weight tile, 128 features x 64 k, written straight
//     into TENSOR MEMORY by the dequant warpgroups (tcgen05.st) -- it never
//     passes through shared memory (an A ring in shared memory was tried: the
//     extra 32 KB of shared traffic per step made it slower);
//   * B = the activation tile, BT tokens x 64 k bf16 in shared memory with
//     128-byte swizzle (loaded per step by TMA, or -- for BT = 16 when X fits
//     -- loaded whole by TMA at kernel start and kept resident; rows >= M
//     arrive as zeros from the copy's out-of-range fill);
//   * D = 128 x BT f32 accumulator in TMEM (tcgen05.mma kind::f16, issued by
//     one thread).
// With tokens on the MMA N side, every dequantised weight element feeds BT
// multiply-adds; one quantisation group (64 k) is one pipeline step, so each
// step needs one scale and one bias per row.
//
// Three rings decouple the producers from the consumer:
//   X ring  (SX slots in smem)  TMA producer -> MMA
//   W ring  (SW slots in smem)  TMA producer -> dequant (packed words only: deep)
//   A ring  (SA slots in TMEM)  dequant      -> MMA
// so the weight stream and its unpacking run many steps ahead of the MMAs.
//
// Warp roles (640 threads for W4, 512 for W8; one CTA per SM, persistent over tiles):
//   warp 0      TMA producer of the X ring (or of the resident X)
//   warp 1      TMEM allocator and MMA issuer
//   warp 2      TMA producer of the W ring
//   warps 4-..  dequant warpgroups (three for W4, two for W8) taking the steps
//               of each tile in turn; thread r of a group owns feature row r
//               (TMEM lane r), so the groups store, into different A slots, the
//               same TMEM lanes
//   last 4      epilogue: 32-token chunks of the accumulator -> registers
//               (+bias, or the fused stage resid + gate * act(acc + bias) with
//               the residual tile copied in by TMA ahead of the accumulator;
//               packed to bf16) -> shared staging -> TMA tensor store, with the
//               accumulator released as soon as it has been read
// A packed-weight slot is released only after the words read from it have been
// consumed (stored to TMEM): releasing it right after the shared-memory reads let
// the slot's next TMA fill land before those reads returned, which showed up as
// intermittently corrupt rows whenever the unpacking ran slower than the copies.
// Every mbarrier wait is bounded (2 s); on expiry the kernel records a status
// bit, drains its own copies and MMAs, frees TMEM and returns.
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

// Status word for this file's kernels (see sdq_ptx.cuh).
__device__ unsigned int g_tc_status = 0;

namespace {

// Dequant warpgroups (group g takes the groups of K with kt % DQ == g) and one
// epilogue warpgroup.  W4 runs three dequant groups (20 warps: its unpacking is the
// longer half of a step and its registers allow 640 threads); W8 runs two (16
// warps), its unpacking needing more registers than 640 threads leave.
constexpr int kEpiGroups = 1;
__host__ __device__ constexpr int dq_groups(int bits) { return bits == 4 ? 3 : 2; }
__host__ __device__ constexpr int first_epi_warp(int bits) { return 4 + 4 * dq_groups(bits); }
__host__ __device__ constexpr int tc_threads(int bits) { return 32 * (first_epi_warp(bits) + 4 * kEpiGroups); }

template <int BITS, int BT, int SX, int SW, int SA, bool XRES>
struct TcCfg;

// The exchange of a column-sharded output, fused into the epilogue (npeers > 0): besides
// this rank's copy, each finished output tile is stored at the same place of every peer's
// copy of the [M, world * N] output (peers[i] points at this rank's column block there,
// rows ldy elements apart), by TMA tensor stores over NVLink through one tensor map per
// peer.  When a CTA has finished its tiles and its stores have completed, it adds 1 to
// landed[i], a word in peer i's memory, after a system-scope fence, so a peer that has
// counted every CTA of every sender sees the whole output.  A CTA that gave up counts
// too (the status word carries the error), so no peer waits for it.  grid_out receives
// the number of CTAs launched.  (Host side; the kernel gets PeerArg.)
struct TcSignal {
    int npeers = 0;
    uint16_t* const* peers = nullptr;
    uint32_t* const* landed = nullptr;
    int* grid_out = nullptr;
};
// The kernel's view of it.  Only the pushing instantiation carries the tensor maps: the
// others' parameters stay small (a launch's parameter block is copied for every launch,
// and 900 more bytes of it cost about a microsecond per launch of the short kernels).
template <bool PUSH>
struct PeerArg {
    CUtensorMap map[kTcMaxPeers];
    uint32_t* landed[kTcMaxPeers];
    int npeers;
};
// The other instantiations carry an optional per-chunk completion count instead: token tile
// tt belongs to chunk tt / chunk_tts, and once a tile's Y is in global memory the epilogue
// adds 1 to done[chunk] (done == nullptr, as every current call passes, turns it off).  It
// stays because of what it does to the compiled kernel: with it, ptxas gives config 2's
// kernel 106 registers and the launch takes 256-258 us on a B200; without it, 104
// registers and 262-264 us (the two builds timed alternately on one box).
template <>
struct PeerArg<false> {
    int npeers;
    uint32_t* done;
    int chunk_tts;
    int nchunks;
};

template <int BITS, int BT, int SX, int SW, int SA, bool XRES>
struct TcCfg {
    static constexpr int BF = 128;                         // features per tile = MMA M
    static constexpr int BK = 64;                          // k per step = one group
    static constexpr int X_STAGE = BT * BK * 2;            // bytes, 128 B per token row
    static constexpr int W_ROW = BK * BITS / 8;            // packed bytes per feature row
    static constexpr int W_STAGE = BF * W_ROW;
    static constexpr int W_WORDS = BK * BITS / 32;         // packed words per row per step
    static constexpr uint32_t D_COL = 0;                   // accumulator columns [0, BT)
    static constexpr uint32_t A_COL = (BT + 31) / 32 * 32; // A slots: 32 columns each
    static constexpr int CW = BT % 32 == 0 ? 32 : 16;      // tokens per epilogue chunk
    static constexpr uint32_t TMEM_COLS = 512;
    static constexpr int Y_STAGE = BT * BF * 2;            // bf16 staging of one output tile
    static constexpr int RING_BYTES = (XRES ? 0 : SX * X_STAGE) + SW * W_STAGE + Y_STAGE;
    static_assert(BT % 16 == 0 && BT >= 16 && BT <= 256, "MMA N must be 16..256, step 16");
    static_assert(A_COL + 32 * SA <= TMEM_COLS, "A slots must fit beside the accumulator");
    static_assert(!XRES || BT == 16, "resident activations only for the 16-token tile");
    static_assert(XRES || SX <= SA, "an X slot is released through the done barrier of its step");
};

// Bytes of dynamic shared memory a configuration needs for a given K.
template <class C, bool XRES, int BT>
size_t smem_bytes(int64_t k) {
    size_t b = 1024 + C::RING_BYTES + 1024;   // alignment slack, rings, barriers
    if (XRES) b += (size_t)(k / 64) * (BT * 128);
    return b;
}

// FUSED: the output stage applies gate / residual / activation (EpiArgs::fused); the plain
// instantiation adds the bias only and carries none of that code.  YF32 (plain only): the
// output is f32, written from the accumulator straight to global memory (bias in f32).
// PUSH (plain bf16 only): the epilogue also stores every tile into the peers' outputs
// (TcSignal); the other instantiations carry none of that code.
template <int BITS, int BT, int SX, int SW, int SA, bool XRES, bool FUSED, bool YF32, bool PUSH>
__global__ void __launch_bounds__(tc_threads(BITS), 1)
    qmm_tc_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                  const __grid_constant__ CUtensorMap tmY, const __grid_constant__ CUtensorMap tmR,
                  const uint16_t* __restrict__ xg, const uint16_t* __restrict__ scales,
                  const uint16_t* __restrict__ biases, const EpiArgs epi,
                  uint16_t* y, int M, int N, int K, int64_t ldy, int y_tma, int r_tma,
                  const __grid_constant__ PeerArg<PUSH> pa) {
    using C = TcCfg<BITS, BT, SX, SW, SA, XRES>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const int KT = K / C::BK;
    // Layout: [X ring or resident X (1024-aligned tiles)] [W ring] [barriers].
    uint8_t* sX = smem;
    const size_t x_bytes = XRES ? (size_t)KT * C::X_STAGE : (size_t)SX * C::X_STAGE;
    uint8_t* sW = smem + x_bytes;
    uint8_t* sY = sW + SW * C::W_STAGE;                   // [BT tokens][128 features] bf16
    uint64_t* bars = reinterpret_cast<uint64_t*>(sY + C::Y_STAGE);
    // Step s uses X slot s % SX, W slot s % SW and A slot / barrier pair s % SA.
    //   wfull[w]   packed W landed                       count 1 + tx
    //   wempty[w]  the dequant group of the step read W slot w   count 128
    //   ready[a]   A slot written and X landed: 128 dequant arrivals, plus (with an
    //              X ring) the X producer's arrive + expect-tx, completed by the
    //              bulk copy itself -- so the MMA warp observes the copy directly
    //   done[a]    the MMAs of the step finished          count 1 (one commit per
    //              step); releases A slot a and the step's X slot
    uint64_t* wfull = bars;
    uint64_t* wempty = wfull + SW;
    uint64_t* ready = wempty + SW;
    uint64_t* done = ready + SA;
    uint64_t* dfull = done + SA;             // accumulator complete       count 1 (commit)
    uint64_t* dempty = dfull + 1;            // accumulator drained        count 128 per epilogue group
    uint64_t* drain = dfull + 2;             // abort drain of the MMA pipe
    uint64_t* xfull = dfull + 3;             // resident X landed          count 1 + tx
    uint64_t* rfull = dfull + 4;             // residual tile landed in the staging  count 1 + tx
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rfull + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    unsigned int* status = &g_tc_status;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int i = 0; i < SW; ++i) { mbar_init(wfull + i, 1); mbar_init(wempty + i, 128); }
        for (int i = 0; i < SA; ++i) { mbar_init(ready + i, XRES ? 128 : 129); mbar_init(done + i, 1); }
        mbar_init(dfull, 1);
        mbar_init(dempty, 128 * kEpiGroups);
        mbar_init(drain, 1);
        mbar_init(xfull, 1);
        mbar_init(rfull, 1);
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmX);
        tma_prefetch_desc(&tmW);
        if (y_tma) tma_prefetch_desc(&tmY);
        if (r_tma) tma_prefetch_desc(&tmR);
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


    if (warp == 0) {
        // ------------------------------------------------------------ X producer
        // Step s's X completes ready[s % SA]; the slot is reused by step s + SX once
        // the MMAs of step s are done.
        if (lane == 0 && XRES) {
            // All KT tiles of X (16 rows; rows >= M zero-filled) on one barrier.
            mbar_arrive_expect_tx(xfull, (uint32_t)KT * C::X_STAGE);
            for (int kt = 0; kt < KT; ++kt)
                tma_load_2d(sX + (size_t)kt * C::X_STAGE, &tmX, xfull, kt * C::BK, 0);
            // The copies must land before shared memory is released, whatever the
            // other roles do.
            mbar_wait_drain(xfull, 0);
        } else if (lane == 0) {
            int it = 0, last_it = -1;
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
                const int tt = tile / nft;
                for (int kt = 0; kt < KT; ++kt, ++it) {
                    if (it >= SX) {
                        const int prev = it - SX;       // the step that last used this slot
                        if (!mbar_wait_sleep(done + prev % SA, (prev / SA) & 1, abort_flag, status, 1u, 32)) { ok = false; break; }
                    }
                    uint64_t* bar = ready + it % SA;
                    mbar_arrive_expect_tx(bar, C::X_STAGE);
                    tma_load_2d(sX + (it % SX) * C::X_STAGE, &tmX, bar, kt * C::BK, tt * BT);
                    last_it = it;
                }
            }
            if (!ok) {
                // Let every copy this thread started land before shared memory goes away.
                for (int j = last_it; j >= 0 && j > last_it - SX; --j)
                    mbar_wait_drain(ready + j % SA, (uint32_t)((j / SA) & 1));
            }
        }
    } else if (warp == 2) {
        // ------------------------------------------------------------ W producer
        if (lane == 0) {
            int it = 0, last_it = -1;
            bool ok = true;
            const bool withhold = g_withhold_first_copy != 0;   // testing hook, normally false
            for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
                const int ft = tile % nft;
                for (int kt = 0; kt < KT; ++kt, ++it) {
                    const int s = it % SW;
                    if (!mbar_wait_sleep(wempty + s, ((it / SW) & 1) ^ 1, abort_flag, status, 1u, 32)) { ok = false; break; }
                    if (!(withhold && it == 0)) {
                        mbar_arrive_expect_tx(wfull + s, C::W_STAGE);
                        tma_load_2d(sW + s * C::W_STAGE, &tmW, wfull + s, kt * C::W_WORDS, ft * C::BF);
                    }
                    last_it = it;
                }
            }
            if (!ok) {
                for (int j = last_it; j >= 0 && j > last_it - SW; --j)
                    mbar_wait_drain(wfull + j % SW, (uint32_t)((j / SW) & 1));
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        // The whole warp runs the loop converged, so descriptors and TMEM addresses
        // are warp-uniform; one elected lane issues the MMAs and the commits.  Per
        // step: one wait (A written, X landed), four MMAs, one commit.
        const uint32_t idesc = idesc_bf16_f32(C::BF, BT);
        int a = 0, xs = 0;              // A slot / X slot of the current step
        uint32_t aph = 0;               // phase parity of ready[a] / done[a]
        int tc = 0;
        bool ok = !XRES || mbar_wait_warp(xfull, 0, abort_flag, status, 2u), any = false;
        for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x, ++tc) {
            if (!mbar_wait_warp(dempty, (tc & 1) ^ 1, abort_flag, status, 2u)) { ok = false; break; }
            tc_fence_after();
            for (int kt = 0; kt < KT; ++kt) {
                if (!mbar_wait_warp(ready + a, aph, abort_flag, status, 2u)) { ok = false; break; }
                tc_fence_after();
                const uint8_t* xt = XRES ? sX + (size_t)kt * C::X_STAGE : sX + xs * C::X_STAGE;
                const uint64_t bdesc = smem_desc_sw128(smem_u32(xt));
                const uint32_t abase = tmem + C::A_COL + 32u * a;
#pragma unroll
                for (int j = 0; j < C::BK / 16; ++j) {
                    // K step of 16 bf16 = 32 bytes inside the swizzled row (+2 in
                    // 16-byte descriptor units); A advances 8 TMEM columns.
                    tc_mma_ts_elect(tmem + C::D_COL, abase + 8u * j, bdesc + 2ull * j, idesc,
                                    (kt | j) != 0);
                }
                tc_commit_elect(done + a);
                any = true;
                if (++a == SA) { a = 0; aph ^= 1; }
                if (++xs == SX) xs = 0;
            }
            if (!ok) break;
            tc_commit_elect(dfull);
        }
        if (!ok && any) {
            tc_commit_elect(drain);
            mbar_wait_drain(drain, 0);
        }
    } else if (warp >= 4 && warp < first_epi_warp(BITS)) {
        // ------------------------------------------------------------ dequant
        // Group g unpacks the steps kt = g, g + DQ, ... of every tile; the groups
        // store different A slots of the same TMEM lanes.
        constexpr int kDqGroups = dq_groups(BITS);
        const int g = (warp - 4) >> 2;
        const int r = (threadIdx.x - 128) & 127;              // feature row in the tile
        const uint32_t lane_base = static_cast<uint32_t>(32 * (warp & 3)) << 16;
        const int G = K / 64;
        // The packed tile was written by TMA with a 32-byte (W4) / 64-byte (W8)
        // swizzle: 16-byte chunk v of row r sits at chunk v ^ sw, which spreads a
        // quarter-warp's 128-bit reads over all 32 banks.
        const uint32_t sw = BITS == 4 ? ((r >> 2) & 1) : ((r >> 1) & 3);
        int it = 0;
        bool ok = true;
        for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
            const int ft = tile % nft;
            const int row = ft * C::BF + r;
            const bool valid = row < N;
            const uint16_t* srow = scales + (int64_t)(valid ? row : 0) * G;
            const uint16_t* brow = biases + (int64_t)(valid ? row : 0) * G;
            // Loads are unconditional (row 0 stands in for rows past N) and masked
            // afterwards, so the warp never diverges ahead of its .aligned TMEM ops.
            // The next step's scale and bias are loaded while this one is unpacked.
            const uint32_t vmask = valid ? 0xFFFFu : 0u;
            const int kfirst = g < KT ? g : KT - 1;
            uint32_t sb_next = (uint32_t)__ldg(srow + kfirst) & vmask;
            uint32_t bb_next = (uint32_t)__ldg(brow + kfirst) & vmask;
            const int it0 = it;                                // the tile's first step
            for (int kt = g; kt < KT; kt += kDqGroups) {
                it = it0 + kt;
                const int ws = it % SW, as = it % SA;
                const uint32_t sb = sb_next, bb = bb_next;
                const int kn = kt + kDqGroups < KT ? kt + kDqGroups : kt;
                sb_next = (uint32_t)__ldg(srow + kn) & vmask;
                bb_next = (uint32_t)__ldg(brow + kn) & vmask;
                if (!mbar_wait_warp(wfull + ws, (it / SW) & 1, abort_flag, status, 4u)) { ok = false; break; }
                constexpr int NV = BITS == 4 ? 2 : 4;         // 16-byte chunks per row
                uint4 q[NV];
                const uint8_t* wrow = sW + ws * C::W_STAGE + r * C::W_ROW;
#pragma unroll
                for (int v = 0; v < NV; ++v) q[v] = *reinterpret_cast<const uint4*>(wrow + 16 * (v ^ sw));
                if (!mbar_wait_warp(done + as, ((it / SA) & 1) ^ 1, abort_flag, status, 4u)) { ok = false; break; }
                tc_fence_after();
                uint32_t a[32];
                if (BITS == 4) {
                    const uint32_t s2 = sb * 0x10001u, b2 = bb * 0x10001u;
#pragma unroll
                    for (int v = 0; v < NV; ++v) {
                        const uint32_t wv[4] = {q[v].x, q[v].y, q[v].z, q[v].w};
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
                    for (int v = 0; v < NV; ++v) {
                        const uint32_t wv[4] = {q[v].x, q[v].y, q[v].z, q[v].w};
#pragma unroll
                        for (int w = 0; w < 4; ++w) {
                            uint32_t o[2];
                            dq8_word_natural(wv[w], sf, bf, o);
                            a[2 * (4 * v + w)] = o[0];
                            a[2 * (4 * v + w) + 1] = o[1];
                        }
                    }
                }
                tmem_st32(tmem + lane_base + C::A_COL + 32u * as, a);
                tc_wait_st();
                tc_fence_before();
                mbar_arrive(ready + as);
                // The packed slot is released only now: the tensor-memory store above
                // consumed the words read from it, so those reads have returned.  An
                // arrive right after the reads let the slot's next TMA fill overwrite it
                // before they returned (seen as corrupt rows when the unpacking is slow).
                mbar_arrive(wempty + ws);
            }
            it = it0 + KT;
        }
    } else if (warp >= first_epi_warp(BITS)) {
        // ------------------------------------------------------------ epilogue
        // Group e takes chunks e, e + kEpiGroups, ... (32 tokens; one 16-token chunk
        // when BT = 16): TMEM -> registers (+bias) -> bf16 into the shared staging
        // tile [token][feature].  The accumulator is released as soon as every
        // group has read it.  Then one thread per group writes each chunk with a TMA
        // tensor store, which clips tokens >= M and features >= N; when Y's row
        // pitch or base is not 16-byte aligned the group copies the chunk with
        // plain stores instead.  A timed-out wait is made group-uniform by the
        // reducing barrier, so no warp of the group is left at a named barrier.
        constexpr int CW = C::CW;                         // tokens per chunk
        constexpr int NCH = BT / CW;                      // chunks per tile
        const int e = (warp - first_epi_warp(BITS)) >> 2;
        const int fl = 32 * (warp & 3) + lane;            // feature row within the tile
        const uint32_t lane_base = static_cast<uint32_t>(32 * (warp & 3)) << 16;
        const bool leader = (warp & 3) == 0 && lane == 0;
        // Beyond the bias, the fused stage y = resid + gate * act(acc + bias).  With a
        // TMA-able residual, its tile is copied into the staging chunks before the
        // accumulator is waited on (the copy overlaps the tile's main loop) and the output
        // is formed in place there; otherwise each thread loads its residual elements.
        static_assert(kEpiGroups == 1, "one residual barrier serves one epilogue group");
        int tc = 0;
        for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++tc) {
            const int tt = tile / nft, ft = tile - tt * nft;
            const int f = ft * C::BF + fl;
            float badd = 0.f;
            if (epi.bias != nullptr && f < N)
                badd = YF32 ? reinterpret_cast<const float*>(epi.bias)[f] : bf16_bits_to_f32(epi.bias[f]);
            const float gmul = (FUSED && epi.gate != nullptr && f < N) ? bf16_bits_to_f32(epi.gate[f]) : 1.f;
            // The staging chunks of this group must have been read by the previous
            // tile's stores before they are overwritten.
            if (leader && y_tma) bulk_wait_group_read0();
            named_barrier_sync(1 + e, 128);
            bool ok = true;
            if (FUSED && r_tma) {
                if (leader) {
                    uint32_t bytes = 0;
                    for (int c = e; c < NCH; c += kEpiGroups)
                        if (tt * BT + c * CW < M) bytes += CW * C::BF * 2;
                    mbar_arrive_expect_tx(rfull, bytes);
                    for (int c = e; c < NCH; c += kEpiGroups)
                        if (tt * BT + c * CW < M)
                            tma_load_2d(sY + (size_t)c * CW * C::BF * 2, &tmR, rfull, ft * C::BF,
                                        tt * BT + c * CW);
                }
                ok = __all_sync(0xffffffffu, mbar_wait_sleep(rfull, tc & 1, abort_flag, status, 8u, 64));
                // A copy still in flight must land before shared memory is given up.
                if (!ok && leader) mbar_wait_drain(rfull, tc & 1);
            }
            ok = ok && __all_sync(0xffffffffu,
                                  mbar_wait_sleep(dfull, tc & 1, abort_flag, status, 8u, 64));
            if (ok) {
                tc_fence_after();
                for (int c = e; c < NCH; c += kEpiGroups) {
                    uint16_t* yrow = reinterpret_cast<uint16_t*>(sY + (size_t)c * CW * C::BF * 2) + fl;
#pragma unroll
                    for (int h = 0; h < CW / 16; ++h) {
                        uint32_t v[16];
                        __syncwarp();
                        tmem_ld16(tmem + lane_base + C::D_COL + (uint32_t)(CW * c + 16 * h), v);
                        tc_wait_ld();
                        if constexpr (YF32) {
                            // f32 output: each thread writes its feature of 16 tokens; a warp's
                            // 32 features are 128 contiguous bytes of a token's row.
                            const int t0 = tt * BT + c * CW + 16 * h;
                            if (f < N) {
#pragma unroll
                                for (int j = 0; j < 16; ++j)
                                    if (t0 + j < M)
                                        reinterpret_cast<float*>(y)[(size_t)(t0 + j) * ldy + f] =
                                            __uint_as_float(v[j]) + badd;
                            }
                        } else if constexpr (!FUSED) {
#pragma unroll
                            for (int j = 0; j < 16; ++j)
                                yrow[(16 * h + j) * C::BF] =
                                    (uint16_t)(pack_bf16x2(__uint_as_float(v[j]) + badd, 0.f) & 0xFFFFu);
                        } else {
#pragma unroll
                            for (int j = 0; j < 16; ++j) {
                                const int r = 16 * h + j;
                                float a = epi_activation(__uint_as_float(v[j]) + badd, epi.act) * gmul;
                                if (r_tma) {
                                    a += bf16_bits_to_f32(yrow[r * C::BF]);
                                } else if (epi.resid != nullptr) {
                                    const int t = tt * BT + c * CW + r;
                                    if (t < M && f < N) a += bf16_bits_to_f32(epi.resid[(size_t)t * N + f]);
                                }
                                yrow[r * C::BF] = (uint16_t)(pack_bf16x2(a, 0.f) & 0xFFFFu);
                            }
                        }
                    }
                }
                __syncwarp();
                tc_fence_before();
                mbar_arrive(dempty);
                if (y_tma) fence_proxy_async_smem();
            }
            if (!named_barrier_and(1 + e, 128, ok)) break;
            if (y_tma) {
                if (leader) {
                    for (int c = e; c < NCH; c += kEpiGroups)
                        if (tt * BT + c * CW < M) {
                            tma_store_2d(&tmY, sY + (size_t)c * CW * C::BF * 2, ft * C::BF,
                                         tt * BT + c * CW);
                            if constexpr (PUSH) {
#pragma unroll
                                for (int i = 0; i < kTcMaxPeers; ++i)
                                    if (i < pa.npeers)
                                        tma_store_2d(&pa.map[i], sY + (size_t)c * CW * C::BF * 2, ft * C::BF,
                                                     tt * BT + c * CW);
                            }
                        }
                    bulk_commit_group();
                }
            } else if (!YF32 && f < N) {
                for (int c = e; c < NCH; c += kEpiGroups) {
                    const uint16_t* yrow =
                        reinterpret_cast<const uint16_t*>(sY + (size_t)c * CW * C::BF * 2) + fl;
                    const int t0 = tt * BT + c * CW;
                    const int nr = M - t0 < CW ? M - t0 : CW;
                    for (int r = 0; r < nr; ++r) y[(size_t)(t0 + r) * ldy + f] = yrow[r * C::BF];
                }
            }
            if constexpr (!PUSH) {
                if (pa.done != nullptr) {
                    // This tile's Y must be in global memory before its chunk counts it.
                    if (y_tma) {
                        if (leader) {
                            bulk_wait_group0();
                            __threadfence();
                            atomicAdd(pa.done + tt / pa.chunk_tts, 1u);
                        }
                    } else {
                        __threadfence();
                        named_barrier_sync(1 + e, 128);
                        if (leader) atomicAdd(pa.done + tt / pa.chunk_tts, 1u);
                    }
                }
            }
        }
        if (leader && y_tma) bulk_wait_group0();
        if constexpr (PUSH) {
            if (leader) {
                // The leader issued every store of this CTA into the peers' copies and has
                // seen them complete; it releases at system scope after a proxy and a system
                // fence, so a peer that acquires its landed word sees them.
                asm volatile("fence.proxy.async.global;" ::: "memory");
                __threadfence_system();
#pragma unroll
                for (int i = 0; i < kTcMaxPeers; ++i)
                    if (i < pa.npeers)
                        asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(pa.landed[i]) : "memory");
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
    if constexpr (!PUSH) {
        // A CTA that gave up raises every chunk to its maximum, so that nothing waiting on a
        // count is left waiting (the status word carries the error).
        if (threadIdx.x == 0 && pa.done != nullptr && *abort_flag) {
            for (int i = 0; i < pa.nchunks; ++i) atomicMax(pa.done + i, 0x7FFFFFFFu);
        }
    }
}

// ---------------------------------------------------------------- host side
// Largest dynamic shared memory a CTA may use on sm_100 (227 KB).
constexpr size_t kMaxSmem = kQmvMaxSmem;


template <int BITS, int BT, int SX, int SW, int SA, bool XRES, bool FUSED, bool YF32, bool PUSH>
cudaError_t launch_tc_t(const void* x, int64_t m, int64_t k, const uint32_t* wq, const void* scales,
                        const void* biases, int64_t n, const EpiArgs& epi, void* y, int64_t ldy,
                        cudaStream_t st, const char** msg, const TcSignal& sig, int grid_cap) {
    using C = TcCfg<BITS, BT, SX, SW, SA, XRES>;
    auto enc = tensor_map_encoder();
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
                         BITS == 4 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) {
            *msg = "cuTensorMapEncodeTiled rejected the packed-weight tensor map";
            return cudaErrorInvalidValue;
        }
    }
    // Y (rows ldy elements apart) is written by TMA tensor stores when its row pitch and
    // base are 16-byte aligned; otherwise the tensor map stays unused and the epilogue stores.
    CUtensorMap tmY;
    std::memset(&tmY, 0, sizeof(tmY));
    const bool y_tma = !YF32 && (ldy % 8) == 0 && (reinterpret_cast<uintptr_t>(y) % 16) == 0;
    if (y_tma) {
        cuuint64_t dims[2] = {(cuuint64_t)n, (cuuint64_t)m};
        cuuint64_t strides[1] = {(cuuint64_t)ldy * 2};
        cuuint32_t box[2] = {(cuuint32_t)C::BF, (cuuint32_t)C::CW};
        cuuint32_t estr[2] = {1, 1};
        CUresult r = enc(&tmY, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, y, dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                         CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) {
            *msg = "cuTensorMapEncodeTiled rejected the output tensor map";
            return cudaErrorInvalidValue;
        }
    }
    // One tensor map per peer copy of the output, the same shape and pitch as Y's.
    PeerArg<PUSH> pa;
    std::memset(&pa, 0, sizeof(pa));
    if constexpr (PUSH) {
        if (!y_tma || sig.npeers < 1 || sig.npeers > kTcMaxPeers) {
            *msg = "the fused exchange needs a TMA-stored output and 1 to 7 peers";
            return cudaErrorInvalidValue;
        }
        pa.npeers = sig.npeers;
        for (int i = 0; i < sig.npeers; ++i) {
            pa.landed[i] = sig.landed[i];
            cuuint64_t dims[2] = {(cuuint64_t)n, (cuuint64_t)m};
            cuuint64_t strides[1] = {(cuuint64_t)ldy * 2};
            cuuint32_t box[2] = {(cuuint32_t)C::BF, (cuuint32_t)C::CW};
            cuuint32_t estr[2] = {1, 1};
            CUresult r = enc(&pa.map[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, sig.peers[i], dims, strides, box,
                             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                             CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
            if (r != CUDA_SUCCESS) {
                *msg = "cuTensorMapEncodeTiled rejected a peer's output tensor map";
                return cudaErrorInvalidValue;
            }
        }
    }
    // The residual ([m, n], contiguous) is copied in by TMA under the same conditions.
    CUtensorMap tmR;
    std::memset(&tmR, 0, sizeof(tmR));
    const bool r_tma = FUSED && y_tma && n % 8 == 0 && epi.resid != nullptr &&
                       (reinterpret_cast<uintptr_t>(epi.resid) % 16) == 0;
    if (r_tma) {
        cuuint64_t dims[2] = {(cuuint64_t)n, (cuuint64_t)m};
        cuuint64_t strides[1] = {(cuuint64_t)n * 2};
        cuuint32_t box[2] = {(cuuint32_t)C::BF, (cuuint32_t)C::CW};
        cuuint32_t estr[2] = {1, 1};
        CUresult r = enc(&tmR, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(epi.resid),
                         dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) {
            *msg = "cuTensorMapEncodeTiled rejected the residual tensor map";
            return cudaErrorInvalidValue;
        }
    }
    const size_t smem = smem_bytes<C, XRES, BT>(k);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static bool configured[64] = {};
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        e = cudaFuncSetAttribute(qmm_tc_kernel<BITS, BT, SX, SW, SA, XRES, FUSED, YF32, PUSH>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxSmem);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    const int64_t tiles = ((n + 127) / 128) * ((m + BT - 1) / BT);
    const int64_t cap = grid_cap > 0 && grid_cap < num_sms() ? grid_cap : num_sms();
    const int grid = (int)(tiles < cap ? tiles : cap);
    if (sig.grid_out) *sig.grid_out = grid;
    qmm_tc_kernel<BITS, BT, SX, SW, SA, XRES, FUSED, YF32, PUSH><<<grid, tc_threads(BITS), smem, st>>>(
        tmX, tmW, tmY, tmR, static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(scales),
        static_cast<const uint16_t*>(biases), epi, static_cast<uint16_t*>(y), (int)m, (int)n, (int)k,
        ldy, y_tma ? 1 : 0, r_tma ? 1 : 0, pa);
    return cudaGetLastError();
}

// Tokens per tile for an M x N problem; 0 stands for the 16-token tile with X resident.
// Up to 128 tokens: the smallest of 16 / 64 / 128 that covers M, so short activations do
// not pay for empty MMA columns.  Beyond that the tile height is chosen so the tiles fill
// whole waves of the SMs: cost = waves x (per-step time + a fixed per-tile share), the
// step time being the MMA's (BT tokens) or the unpacking's (about 128 tokens' worth for
// W4, 288 for W8), whichever is longer.  1024 x 3072 output at W4 thus runs as 144 tiles
// of 176 tokens in one wave instead of 96 tiles of 256.
template <int BITS>
int choose_tile(int64_t m, int64_t k, int64_t n, int grid_cap) {
    constexpr int SWs = BITS == 4 ? 16 : 12;
    using CR = TcCfg<BITS, 16, 1, SWs, 14, true>;
    if (m <= 16) return smem_bytes<CR, true, 16>(k) <= kMaxSmem ? 0 : 16;
    if (m <= 64) return 64;
    if (m <= 128) return 128;
    const int64_t sms = grid_cap > 0 && grid_cap < num_sms() ? grid_cap : num_sms();
    const int64_t nft = (n + 127) / 128;
    const int64_t dq = BITS == 4 ? 128 : 288, fixed = 32;
    int64_t best = -1;
    int bt = 128;
    for (int cand : {128, 176, 240, 256}) {
        const int64_t tiles = (m + cand - 1) / cand * nft;
        const int64_t cost = (tiles + sms - 1) / sms * ((cand > dq ? cand : dq) + fixed);
        if (best < 0 || cost <= best) {                // ties go to the taller tile
            best = cost;
            bt = cand;
        }
    }
    return bt;
}

// The plain or the fused instantiation of a configuration, as the output stage asks.
template <int BITS, int BT, int SX, int SW, int SA, bool XRES>
cudaError_t launch_tc_f(const void* x, int64_t m, int64_t k, const uint32_t* wq, const void* scales,
                        const void* biases, int64_t n, const EpiArgs& epi, void* y, int64_t ldy,
                        cudaStream_t st, const char** msg, const TcSignal& sig, int grid_cap) {
    if (sig.npeers > 0) {  // the sharded linear: plain bf16 output stage, tiles pushed to peers
        if (epi.fused() || epi.f32) return cudaErrorInvalidValue;
        return launch_tc_t<BITS, BT, SX, SW, SA, XRES, false, false, true>(x, m, k, wq, scales, biases, n, epi, y,
                                                                           ldy, st, msg, sig, grid_cap);
    }
    if (epi.fused())
        return launch_tc_t<BITS, BT, SX, SW, SA, XRES, true, false, false>(x, m, k, wq, scales, biases, n, epi, y,
                                                                           ldy, st, msg, sig, grid_cap);
    if (epi.f32)           // f32 output (the bias, if any, f32 too)
        return launch_tc_t<BITS, BT, SX, SW, SA, XRES, false, true, false>(x, m, k, wq, scales, biases, n, epi, y,
                                                                           ldy, st, msg, sig, grid_cap);
    return launch_tc_t<BITS, BT, SX, SW, SA, XRES, false, false, false>(x, m, k, wq, scales, biases, n, epi, y,
                                                                        ldy, st, msg, sig, grid_cap);
}

template <int BITS>
cudaError_t launch_tc_bits(const void* x, int64_t m, int64_t k, const uint32_t* wq,
                           const void* scales, const void* biases, int64_t n, const EpiArgs& epi,
                           void* y, int64_t ldy, cudaStream_t st, const char** msg, const TcSignal& sig,
                           int grid_cap) {
    // Ring depths fill the shared memory budget; the packed-weight ring is the deep one.
    constexpr int SWs = BITS == 4 ? 16 : 12;
    constexpr int SWL = BITS == 4 ? 8 : 4;
    switch (choose_tile<BITS>(m, k, n, grid_cap)) {
        case 0: return launch_tc_f<BITS, 16, 1, SWs, 14, true>(x, m, k, wq, scales, biases, n, epi, y, ldy, st, msg, sig, grid_cap);
        case 16: return launch_tc_f<BITS, 16, 8, 12, 14, false>(x, m, k, wq, scales, biases, n, epi, y, ldy, st, msg, sig, grid_cap);
        case 64: return launch_tc_f<BITS, 64, 8, 12, 12, false>(x, m, k, wq, scales, biases, n, epi, y, ldy, st, msg, sig, grid_cap);
        case 128: return launch_tc_f<BITS, 128, 6, 8, 8, false>(x, m, k, wq, scales, biases, n, epi, y, ldy, st, msg, sig, grid_cap);
        case 176: return launch_tc_f<BITS, 176, 5, SWL, 8, false>(x, m, k, wq, scales, biases, n, epi, y, ldy, st, msg, sig, grid_cap);
        case 240: return launch_tc_f<BITS, 240, 4, SWL, 8, false>(x, m, k, wq, scales, biases, n, epi, y, ldy, st, msg, sig, grid_cap);
        default: return launch_tc_f<BITS, 256, 4, SWL, 8, false>(x, m, k, wq, scales, biases, n, epi, y, ldy, st, msg, sig, grid_cap);
    }
}

}  // namespace

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
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

cudaError_t launch_qmm_tc(const void* x, int64_t m, int64_t k, const uint32_t* wq,
                          const void* scales, const void* biases, int64_t n, int bits,
                          const EpiArgs& epi, void* y, cudaStream_t st, const char** msg) {
    const TcSignal off{};
    return bits == 4 ? launch_tc_bits<4>(x, m, k, wq, scales, biases, n, epi, y, n, st, msg, off, 0)
                     : launch_tc_bits<8>(x, m, k, wq, scales, biases, n, epi, y, n, st, msg, off, 0);
}

int qmm_tc_tile_tokens(int64_t m, int64_t k, int64_t n, int bits, int grid_cap) {
    const int t = bits == 4 ? choose_tile<4>(m, k, n, grid_cap) : choose_tile<8>(m, k, n, grid_cap);
    return t == 0 ? 16 : t;
}

cudaError_t launch_qmm_tc_push(const void* x, int64_t m, int64_t k, const uint32_t* wq,
                               const void* scales, const void* biases, int64_t n, int bits,
                               const EpiArgs& epi, void* y, int64_t ldy, cudaStream_t st,
                               const char** msg, uint16_t* const* peers, uint32_t* const* landed,
                               int npeers, int grid_cap, int* grid_out) {
    if (npeers < 1 || npeers > kTcMaxPeers) return cudaErrorInvalidValue;
    TcSignal sig{};
    sig.npeers = npeers;
    sig.peers = peers;
    sig.landed = landed;
    sig.grid_out = grid_out;
    return bits == 4 ? launch_tc_bits<4>(x, m, k, wq, scales, biases, n, epi, y, ldy, st, msg, sig, grid_cap)
                     : launch_tc_bits<8>(x, m, k, wq, scales, biases, n, epi, y, ldy, st, msg, sig, grid_cap);
}

cudaError_t set_wait_hook_tc(unsigned long long limit_ns, int withhold, cudaStream_t st) {
    cudaError_t e = cudaMemcpyToSymbolAsync(g_wait_limit_ns, &limit_ns, sizeof(limit_ns), 0,
                                            cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess)
        e = cudaMemcpyToSymbolAsync(g_withhold_first_copy, &withhold, sizeof(withhold), 0,
                                    cudaMemcpyHostToDevice, st);
    return e == cudaSuccess ? cudaStreamSynchronize(st) : e;
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
