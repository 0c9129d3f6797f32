// sdq_ptx.cuh -- thin inline-PTX wrappers for sm_100a: mbarriers with bounded
// waits, TMA tensor loads, and the tcgen05 (TMEM + 5th-gen tensor core) ops.
// Everything here is written from the public PTX ISA; no library kernels.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace sdq {

// Kernels OR a code into a device-side status word when a bounded wait gives
// up (instead of spinning forever); the host reads it with
// sdq_device_status().  Bits: 1 = TMA producer, 2 = MMA issuer, 4 = dequant,
// 8 = epilogue.

// Wall-clock limit for one bounded wait (nanoseconds of %globaltimer).
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

// Testing hooks (set through sdq_debug_wait_hook; every file that includes this header has
// its own copy, and the hook sets each): the limit the waits use (kWaitLimitNs unless a test
// shortened it), and a switch that makes the weight producer of every CTA skip its first copy
// together with the arrival that goes with it, so that the consumers' wait on that stage runs
// out and the abort path (status bit, drain, TMEM release, early return) is taken.
static __device__ unsigned long long g_wait_limit_ns = kWaitLimitNs;
static __device__ int g_withhold_first_copy = 0;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\t"
        "mbarrier.arrive.release.cta.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\t"
        "mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
            smem_u32(bar)),
        "r"(bytes)
        : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait with a suspend-time hint: a thread whose phase is not complete may be
// suspended (issuing nothing) until the phase completes or `hint_ns` passes.
__device__ __forceinline__ bool mbar_try_wait_hint(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Wait for the phase with `parity` to complete, giving up after the wait limit or
// as soon as another role of this CTA has raised `*abort`.  Returns false when
// it gave up (and then sets the abort flag and the global status bit).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          unsigned int* status, unsigned int status_bit) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = globaltimer(), lim = g_wait_limit_ns;
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63u) == 0u) {
            if (*abort) return false;
            if (globaltimer() - t0 > lim) {
                *abort = 1;
                atomicOr(status, status_bit);
                return false;
            }
        }
    }
}

// mbar_wait for roles off the critical path (producers running ahead, the
// epilogue waiting out a whole tile): after the first failed test the thread
// sleeps `sleep_ns` between tests, so its spinning does not take issue slots
// from the dequant warps that share its SM sub-partition.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, volatile int* abort,
                                                unsigned int* status, unsigned int status_bit,
                                                unsigned int sleep_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = globaltimer(), lim = g_wait_limit_ns;
    for (uint32_t it = 1;; ++it) {
        __nanosleep(sleep_ns);
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 15u) == 0u) {
            if (*abort) return false;
            if (globaltimer() - t0 > lim) {
                *abort = 1;
                atomicOr(status, status_bit);
                return false;
            }
        }
    }
}

// Warp-collective form of mbar_wait for warps that go on to issue
// .sync.aligned tcgen05 instructions (tcgen05.st / ld / wait::*): each lane
// waits (and so acquires) on its own, then the warp votes, which also
// reconverges it.  Lanes leave a spin loop at different iterations; an
// .aligned instruction issued by a diverged warp is undefined (in practice
// parts of a TMEM store were not there when the MMA read them).  The vote
// also keeps the give-up decision uniform across the warp.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort,
                                               unsigned int* status, unsigned int status_bit) {
    const bool ok = mbar_wait(bar, parity, abort, status, status_bit);
    return __all_sync(0xffffffffu, ok);
}

// mbar_wait_warp whose tests suspend the waiting warp for up to `hint_ns` instead of
// spinning, for consumers that share their sub-partition with other busy warps.
__device__ __forceinline__ bool mbar_wait_warp_parked(uint64_t* bar, uint32_t parity,
                                                      volatile int* abort, unsigned int* status,
                                                      unsigned int status_bit, uint32_t hint_ns) {
    bool ok = mbar_try_wait_hint(bar, parity, hint_ns);
    if (!ok) {
        const unsigned long long t0 = globaltimer(), lim = g_wait_limit_ns;
        for (uint32_t it = 1;; ++it) {
            if (mbar_try_wait_hint(bar, parity, hint_ns)) { ok = true; break; }
            if ((it & 7u) == 0u) {
                if (*abort) break;
                if (globaltimer() - t0 > lim) {
                    *abort = 1;
                    atomicOr(status, status_bit);
                    break;
                }
            }
        }
    }
    return __all_sync(0xffffffffu, ok);
}

// Bounded wait used only while draining after an abort: ignores the abort flag.
__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity) {
    const unsigned long long t0 = globaltimer(), lim = g_wait_limit_ns;
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer() - t0 > lim) return false;
    }
    return true;
}

// ---------------------------------------------------------------- programmatic dependent launch
// A kernel launched with the programmatic-stream-serialisation attribute may start while
// the previous kernel in its stream is still running.  griddep_wait() returns once that
// kernel has completed and its memory operations are visible; nothing the earlier kernels
// write may be read (or overwritten) before it.  griddep_launch_dependents() lets the next
// kernel of the stream launch early (it still waits in its own griddep_wait()).  Without
// the attribute both are no-ops.
__device__ __forceinline__ void griddep_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}
// 2-D tiled load global -> shared, completion counted on `bar` in bytes.
// Every CTA loads its own tiles; no copy is shared between CTAs.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* tmap, uint64_t* bar,
                                            int32_t c0, int32_t c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}
// 1-D bulk copy global -> shared of `bytes` (a multiple of 16; both addresses
// 16-byte aligned), completion counted on `bar` in bytes; this CTA only.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes),
        "r"(smem_u32(bar))
        : "memory");
}
// Ampere-style asynchronous copy of 4 or 8 bytes global -> shared; `src_bytes` = 0
// writes zeros instead of reading.  cp_async_arrive makes `bar` receive one
// arrival once all of this thread's earlier cp.async copies have landed (the
// barrier's expected count must include it).
template <int BYTES>
__device__ __forceinline__ void cp_async(void* smem_dst, const void* src, uint32_t src_bytes) {
    static_assert(BYTES == 4 || BYTES == 8, "cp.async.ca copies 4, 8 or 16 bytes");
    asm volatile("cp.async.ca.shared.global [%0], [%1], %2, %3;" ::"r"(smem_u32(smem_dst)),
                 "l"(reinterpret_cast<uint64_t>(src)), "n"(BYTES), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.wait_all;" ::: "memory");
}
// L2 eviction-priority policies for the cache_hint operand.
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// ---------------------------------------------------------------- tcgen05
// TMEM address: bits [31:16] lane, [15:0] column (32-bit cells).
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(smem_slot)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D(tmem) (+)= A(tmem) . B(smem desc)^T, kind::f16 (bf16 inputs, f32 accumulate).
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Warp-collective forms: the whole (converged) warp executes these, so every
// operand is warp-uniform; elect.sync picks one lane (always the same one in a
// converged warp) to issue the instruction.
__device__ __forceinline__ void tc_mma_ts_elect(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                                uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// SS form: A and B both from shared memory through descriptors; one elected lane issues.
__device__ __forceinline__ void tc_mma_ss_elect(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                                uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void tc_commit_elect(uint64_t* bar) {
    asm volatile(
        "{\n\t.reg .pred e;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(
            smem_u32(bar))
        : "memory");
}
// Arrive once on `bar` when every tcgen05.mma issued so far by this thread completes.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tc_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tc_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 2-D tiled store shared -> global (bulk async group); out-of-range rows and
// columns of the box are not written.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* tmap, const void* smem_src, int32_t c0,
                                             int32_t c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
            reinterpret_cast<uint64_t>(tmap)),
        "r"(smem_u32(smem_src)), "r"(c0), "r"(c1)
        : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until every committed bulk store of this thread has finished READING shared memory.
__device__ __forceinline__ void bulk_wait_group_read0() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// ... all but the most recent one.
__device__ __forceinline__ void bulk_wait_group_read1() {
    asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
// Wait until every committed bulk store of this thread has completed.
__device__ __forceinline__ void bulk_wait_group0() {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void named_barrier_sync(uint32_t id, uint32_t nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
// Zero, computed from four registers: an address offset by it cannot be used
// until the loads that produced those registers have returned.  Used before
// releasing a ring slot whose contents were loaded but are consumed only by
// plain arithmetic (an arrive issued while such loads are in flight lets the
// slot's next fill overwrite the data before they read it).
__device__ __forceinline__ uint32_t zero_after(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    uint32_t z;
    asm volatile(
        "{\n\t.reg .b32 t;\n\t"
        "or.b32 t, %1, %2;\n\t"
        "or.b32 t, t, %3;\n\t"
        "or.b32 t, t, %4;\n\t"
        "and.b32 %0, t, 0;\n\t}"
        : "=r"(z)
        : "r"(a), "r"(b), "r"(c), "r"(d));
    return z;
}

// Named barrier that also returns the AND of `pred` over the participating threads.
__device__ __forceinline__ bool named_barrier_and(uint32_t id, uint32_t nthreads, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)pred), "r"(id), "r"(nthreads)
        : "memory");
    return r != 0;
}

// Warp-collective: lane i writes 32 consecutive 32-bit columns of TMEM lane
// (taddr.lane + i) starting at taddr.column.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
        "%28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
        "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
        "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
        "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
// Warp-collective: lane i reads 16 consecutive 32-bit columns of TMEM lane (taddr.lane + i).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}
// Make this thread's generic-proxy shared-memory writes visible to the async
// proxy (TMA and the tensor core's shared-memory operand reads).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Warp-collective: lane i reads 32 consecutive 32-bit columns of TMEM lane (taddr.lane + i).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
        "%28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr)
        : "memory");
}

// Shared-memory matrix descriptor (tcgen05 format) for a K-major operand tile
// written by TMA with 128-byte swizzle: rows of 128 bytes, 8-row atoms of
// 1024 bytes.  LBO = 16 B (unused for swizzled K-major), SBO = 1024 B,
// version 1 (bits 46-47), layout SWIZZLE_128B = 2 (bits 61-63).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1u) << 16;
    d |= static_cast<uint64_t>(1024u >> 4) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= static_cast<uint64_t>(2u) << 61;
    return d;
}

// Instruction descriptor for kind::f16: bf16 A and B, f32 accumulator, both
// K-major, shape M x N.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N) {
    return (1u << 4)                                  // D format F32
           | (1u << 7)                                // A format BF16
           | (1u << 10)                               // B format BF16
           | (static_cast<uint32_t>(N >> 3) << 17)    // N / 8
           | (static_cast<uint32_t>(M >> 4) << 24);   // M / 16
}

}  // namespace sdq
