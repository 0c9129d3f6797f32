// sdq_shard.cu -- the column-sharded quantised linear over NCCL.
//
// Each rank holds a contiguous block of output features (rows of the packed
// weight), runs the single-GPU kernel on it, and the [m, n_local] results are
// exchanged over NVLink / NVSwitch into [world, m, n_local] on every rank; a
// permute kernel turns that into [m, n].
//
// When the output is wanted as [m, n] on two to eight ranks and M > 8, the exchange is
// fused into the compute kernel.  Every rank owns a symmetric output buffer ([m, n]
// bf16, IPC-mapped on every peer).  The tensor-core kernel writes this rank's column
// block of it in place (rows world * n_local apart) and, as each output tile is staged in
// shared memory, also stores it (16-byte stores over NVLink) at the same place of every
// peer's buffer, so the exchange runs tile by tile beside the math and uses no copy
// engine.  The ranks synchronise through flag words, IPC-mapped like the buffers, that
// need no SM: once the caller's stream has drained, a stream write (cuStreamWriteValue32)
// tells every peer that this rank's buffer may be written, and the kernel is preceded by
// stream waits (cuStreamWaitValue32) for every peer's word.  Each CTA, when done, fences
// at system scope and adds 1 to a count in every peer's memory; a one-thread kernel then
// waits (acquire loads at system scope, bounded) until every peer's count has grown by
// the peers' CTA count, after which the buffer holds [m, n] and is copied to the caller's
// y unless y is that buffer (sdq_comm_output).  Earlier forms of this path pushed
// finished chunks of rows with the copy engines (one stream per peer) behind NCCL
// barrier all-reduces; at eight ranks the copies reached about 300 GB/s per GPU and the
// barrier kernels waited for the compute kernel's SMs.  A kernel that gives up still
// counts, so no peer waits for it beyond its bound.  The buffer is allocated on first use
// and grows collectively (every rank calls with the same shapes).
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include <cuda.h>
#include <cuda_runtime.h>
#include <nccl.h>

#include "../../include/sdq.h"
#include "sdq_internal.h"

namespace sdq {
namespace {

thread_local std::string t_shard_msg;

constexpr int kMaxWorld = 64;

struct Comm {
    ncclComm_t nccl = nullptr;
    int rank = 0;
    int world = 1;
    int device = 0;
    // Overlapped exchange (set up when world > 1; the plain path runs without it).  The side
    // stream carries the collective set-up (handle exchanges); the calls run on the caller's.
    cudaStream_t side = nullptr;
    // Barrier words: this rank's [2][kMaxWorld], IPC-exported.  [0][p] receives peer p's
    // "ready" epoch (p's output may be written: its readers are done); [1][p] counts the
    // CTAs of p's kernels that have finished storing into this rank's output.  peer_flags[p]
    // is peer p's array as mapped here.  epoch counts overlapped calls and landed_target the
    // CTAs each sender has run in them; every rank makes the same calls, so both agree.
    uint32_t* flags = nullptr;
    uint32_t* peer_flags[kMaxWorld] = {};
    uint32_t epoch = 0;
    uint32_t landed_target = 0;
    // The symmetric output: this rank's [m, n] bf16 buffer, into whose column blocks the
    // kernel and the peers write, and the peers' buffers as mapped here.
    void* xbuf = nullptr;
    size_t xbuf_cap = 0;
    void* peer_xbuf[kMaxWorld] = {};
    cudaIpcMemHandle_t* handles_dev = nullptr;   // world handles, for the one-off exchange
};

using ValueFn = CUresult (*)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);

ValueFn driver_value_fn(const char* name) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
        return reinterpret_cast<ValueFn>(p);
    return nullptr;
}
ValueFn wait_value_fn() {
    static ValueFn fn = driver_value_fn("cuStreamWaitValue32");
    return fn;
}
ValueFn write_value_fn() {
    static ValueFn fn = driver_value_fn("cuStreamWriteValue32");
    return fn;
}

// Status word of the landed-flag wait (read and cleared by sdq_device_status).
__device__ unsigned int g_shard_status = 0;

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// One thread per peer waits until the peer's landed count has reached `target` (a cyclic
// comparison, as CU_STREAM_WAIT_VALUE_GEQ makes), reading it with acquire semantics at
// system scope: each of the peer's CTAs added to it with release semantics after its
// stores into this rank's output, so the work after this kernel sees those stores.
// Gives up after 2 s (bit 1 of the status word; the output is then incomplete).
__global__ void wait_landed(const uint32_t* __restrict__ landed, int world, int rank, uint32_t target) {
    const int p = threadIdx.x;
    if (p >= world || p == rank) return;
    const unsigned long long t0 = globaltimer_ns();
    for (;;) {
        uint32_t v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(landed + p) : "memory");
        if (static_cast<int32_t>(v - target) >= 0) return;
        if (globaltimer_ns() - t0 > 2000000000ull) {
            atomicOr(&g_shard_status, 1u);
            return;
        }
        __nanosleep(200);
    }
}

// Allocate this rank's barrier words, export them, and map every peer's (collective).
bool setup_flags(Comm* c) {
    const size_t bytes = 2 * kMaxWorld * sizeof(uint32_t);
    if (cudaMalloc(reinterpret_cast<void**>(&c->flags), bytes) != cudaSuccess) return false;
    cudaIpcMemHandle_t mine;
    if (cudaMemset(c->flags, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&mine, c->flags) != cudaSuccess ||
        cudaMemcpyAsync(c->handles_dev + c->rank, &mine, sizeof mine, cudaMemcpyHostToDevice, c->side) !=
            cudaSuccess)
        return false;
    if (ncclAllGather(c->handles_dev + c->rank, c->handles_dev, sizeof(cudaIpcMemHandle_t), ncclUint8, c->nccl,
                      c->side) != ncclSuccess)
        return false;
    std::vector<cudaIpcMemHandle_t> all(c->world);
    if (cudaMemcpyAsync(all.data(), c->handles_dev, c->world * sizeof(cudaIpcMemHandle_t), cudaMemcpyDeviceToHost,
                        c->side) != cudaSuccess ||
        cudaStreamSynchronize(c->side) != cudaSuccess)
        return false;
    for (int p = 0; p < c->world; ++p) {
        if (p == c->rank) continue;
        void* q = nullptr;
        if (cudaIpcOpenMemHandle(&q, all[p], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return false;
        c->peer_flags[p] = static_cast<uint32_t*>(q);
    }
    return true;
}

void release_flags(Comm* c) {
    for (int p = 0; p < kMaxWorld; ++p)
        if (c->peer_flags[p]) {
            cudaIpcCloseMemHandle(c->peer_flags[p]);
            c->peer_flags[p] = nullptr;
        }
    if (c->flags) cudaFree(c->flags);
    c->flags = nullptr;
}


// y[t, r * nl + j] = shards[r, t, j] for rows t in [m0, m0 + mc) of an m-row output;
// 8 bf16 (16 bytes) per thread when n_local % 8 == 0, else one element per thread.
__global__ void permute_shards_v8(const uint4* __restrict__ shards, uint4* __restrict__ y,
                                  int64_t m, int64_t m0, int64_t mc, int64_t nl8, int world) {
    const int64_t total = (int64_t)world * mc * nl8;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t j = i % nl8;
        const int64_t t = m0 + (i / nl8) % mc;
        const int64_t r = i / (nl8 * mc);
        y[t * (world * nl8) + r * nl8 + j] = shards[(r * m + t) * nl8 + j];
    }
}
__global__ void permute_shards_v1(const uint16_t* __restrict__ shards, uint16_t* __restrict__ y,
                                  int64_t m, int64_t m0, int64_t mc, int64_t nl, int world) {
    const int64_t total = (int64_t)world * mc * nl;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t j = i % nl;
        const int64_t t = m0 + (i / nl) % mc;
        const int64_t r = i / (nl * mc);
        y[t * (world * nl) + r * nl + j] = shards[(r * m + t) * nl + j];
    }
}

cudaError_t launch_permute(const void* shards, void* y, int64_t m, int64_t m0, int64_t mc,
                           int64_t nl, int world, cudaStream_t st) {
    const int threads = 256;
    if (nl % 8 == 0) {
        const int64_t total = static_cast<int64_t>(world) * mc * (nl / 8);
        int64_t grid = (total + threads - 1) / threads;
        if (grid > 4096) grid = 4096;
        permute_shards_v8<<<(int)grid, threads, 0, st>>>(static_cast<const uint4*>(shards),
                                                         static_cast<uint4*>(y), m, m0, mc, nl / 8, world);
    } else {
        const int64_t total = static_cast<int64_t>(world) * mc * nl;
        int64_t grid = (total + threads - 1) / threads;
        if (grid > 4096) grid = 4096;
        permute_shards_v1<<<(int)grid, threads, 0, st>>>(static_cast<const uint16_t*>(shards),
                                                         static_cast<uint16_t*>(y), m, m0, mc, nl, world);
    }
    return cudaGetLastError();
}

}  // namespace

cudaError_t read_and_clear_shard_status(unsigned int* out, cudaStream_t st) {
    cudaError_t e = cudaMemcpyFromSymbolAsync(out, g_shard_status, sizeof(unsigned int), 0,
                                              cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e == cudaSuccess && *out != 0) {
        const unsigned int zero = 0;
        e = cudaMemcpyToSymbolAsync(g_shard_status, &zero, sizeof(unsigned int), 0, cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    }
    return e;
}
}  // namespace sdq

using namespace sdq;

// Reported through the same per-thread message as the rest of the ABI.
extern "C" const char* sdq_last_error(void);
namespace sdq {
int set_error_message(int code, const char* msg);
}

static int nccl_fail(const char* what, ncclResult_t r) {
    t_shard_msg = std::string(what) + ": " + ncclGetErrorString(r);
    return sdq::set_error_message(SDQ_ERR_NCCL, t_shard_msg.c_str());
}

constexpr int kNotOverlapped = -1;

// Make this rank's exchange buffer hold `bytes` and map every peer's (collective: all ranks
// call it with the same size).  Allocates only when the buffer must grow.
static int ensure_exchange_buffer(Comm* c, size_t bytes, const char* fn) {
    if (c->xbuf_cap >= bytes) return SDQ_OK;
    auto fail_cuda = [&](const char* what, cudaError_t e) {
        t_shard_msg = std::string(fn) + ": exchange buffer: " + what + ": " + cudaGetErrorString(e);
        return sdq::set_error_message(SDQ_ERR_CUDA, t_shard_msg.c_str());
    };
    if (c->side == nullptr) {             // one rank, or no overlap resources: plain memory
        cudaError_t e = cudaDeviceSynchronize();
        if (e != cudaSuccess) return fail_cuda("synchronise", e);
        if (c->xbuf) cudaFree(c->xbuf);
        c->xbuf = nullptr;
        c->xbuf_cap = 0;
        if ((e = cudaMalloc(&c->xbuf, bytes)) != cudaSuccess) return fail_cuda("cudaMalloc", e);
        c->xbuf_cap = bytes;
        return SDQ_OK;
    }
    // Kernels of earlier calls may still store into the peers' buffers through the mappings
    // about to be closed, and the peers' into this one: wait for this device's work (a
    // peer's stores into this buffer have landed once this rank's wait for them is done).
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return fail_cuda("synchronise", e);
    for (int p = 0; p < c->world; ++p)
        if (c->peer_xbuf[p]) {
            cudaIpcCloseMemHandle(c->peer_xbuf[p]);
            c->peer_xbuf[p] = nullptr;
        }
    if (c->xbuf) cudaFree(c->xbuf);
    c->xbuf = nullptr;
    c->xbuf_cap = 0;
    const size_t cap = (bytes + (size_t(64) << 20) - 1) / (size_t(64) << 20) * (size_t(64) << 20);
    if ((e = cudaMalloc(&c->xbuf, cap)) != cudaSuccess) return fail_cuda("cudaMalloc", e);
    cudaIpcMemHandle_t mine;
    if ((e = cudaIpcGetMemHandle(&mine, c->xbuf)) != cudaSuccess) return fail_cuda("cudaIpcGetMemHandle", e);
    if ((e = cudaMemcpyAsync(c->handles_dev + c->rank, &mine, sizeof mine, cudaMemcpyHostToDevice,
                             c->side)) != cudaSuccess)
        return fail_cuda("handle copy", e);
    ncclResult_t r = ncclAllGather(c->handles_dev + c->rank, c->handles_dev, sizeof(cudaIpcMemHandle_t),
                                   ncclUint8, c->nccl, c->side);
    if (r != ncclSuccess) return nccl_fail("ncclAllGather (exchange-buffer handles)", r);
    std::vector<cudaIpcMemHandle_t> all(c->world);
    if ((e = cudaMemcpyAsync(all.data(), c->handles_dev, c->world * sizeof(cudaIpcMemHandle_t),
                             cudaMemcpyDeviceToHost, c->side)) != cudaSuccess ||
        (e = cudaStreamSynchronize(c->side)) != cudaSuccess)
        return fail_cuda("handle gather", e);
    for (int p = 0; p < c->world; ++p) {
        if (p == c->rank) continue;
        if ((e = cudaIpcOpenMemHandle(&c->peer_xbuf[p], all[p], cudaIpcMemLazyEnablePeerAccess)) !=
            cudaSuccess)
            return fail_cuda("cudaIpcOpenMemHandle", e);
    }
    c->xbuf_cap = cap;
    return SDQ_OK;
}

// Contiguous bf16 copy, 16 bytes per thread: the symmetric output -> the caller's y.
__global__ void copy_v8(const uint4* __restrict__ src, uint4* __restrict__ dst, int64_t n8) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8;
         i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = src[i];
}
__global__ void copy_v1(const uint16_t* __restrict__ src, uint16_t* __restrict__ dst, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = src[i];
}

// The overlapped form of sdq_quantized_matmul_sharded (see the file comment).  Returns
// kNotOverlapped, having enqueued nothing, when the shape or the world does not suit it.
static int sharded_overlapped(Comm* c, const void* x, sdq_dtype x_dtype, int64_t m, int64_t k,
                              const uint32_t* wq, const void* scales, const void* biases,
                              sdq_dtype sb_dtype, int64_t n_local, int group_size, int bits,
                              const void* bias_local, void* y, sdq_dtype y_dtype, void* stream) {
    const char* fn = "sdq_quantized_matmul_sharded";
    const int64_t ldy = static_cast<int64_t>(c->world) * n_local;      // row pitch of [m, n]
    int rc = sdq::validate_qmm(x, x_dtype, m, k, wq, scales, biases, sb_dtype, n_local, 1, group_size,
                               bits, "affine", bias_local, y, y_dtype, fn);
    if (rc != SDQ_OK) return rc;
    // The epilogue stores 16-byte pieces of rows into the peers' copies; one kernel reaches
    // at most kTcMaxPeers peers.
    if (n_local % 8 != 0 || c->world - 1 > sdq::kTcMaxPeers) return kNotOverlapped;
    const ValueFn wait = wait_value_fn(), write = write_value_fn();
    if (wait == nullptr || write == nullptr || c->flags == nullptr) return kNotOverlapped;
    const size_t total = static_cast<size_t>(m) * ldy;   // elements of [m, n]
    if ((rc = ensure_exchange_buffer(c, total * sizeof(uint16_t), fn)) != SDQ_OK) return rc;
    uint16_t* out = static_cast<uint16_t*>(c->xbuf);     // this rank's copy of [m, n]
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    auto cuda_err = [&](const char* what, cudaError_t e) {
        t_shard_msg = std::string(fn) + ": " + what + ": " + cudaGetErrorString(e);
        return sdq::set_error_message(SDQ_ERR_CUDA, t_shard_msg.c_str());
    };
    const uint32_t epoch = ++c->epoch;
    // Ready: the stream write runs once everything before it on the caller's stream is done
    // (the readers of the previous result among it), and tells every peer that its stores
    // into this rank's output may begin.  The kernel then waits for every peer's word.
    for (int p = 0; p < c->world; ++p) {
        if (p == c->rank) continue;
        if (write(reinterpret_cast<CUstream>(st), reinterpret_cast<CUdeviceptr>(c->peer_flags[p] + c->rank),
                  epoch, 0) != CUDA_SUCCESS)
            return cuda_err("ready flag", cudaErrorUnknown);
    }
    for (int p = 0; p < c->world; ++p) {
        if (p == c->rank) continue;
        if (wait(reinterpret_cast<CUstream>(st), reinterpret_cast<CUdeviceptr>(c->flags + p), epoch,
                 0 /* GEQ */) != CUDA_SUCCESS)
            return cuda_err("ready wait", cudaErrorUnknown);
    }
    // The kernel writes this rank's block in place and stores every tile of it into the
    // same place of each peer's output as it finishes.  Each rank walks its peers starting
    // from the next rank up, so that the ranks' first stores of a chunk go to different GPUs
    // rather than all to the lowest rank.
    uint16_t* peers[sdq::kTcMaxPeers];
    uint32_t* landed[sdq::kTcMaxPeers];
    int np = 0;
    for (int j = 1; j < c->world; ++j) {
        const int p = (c->rank + j) % c->world;
        peers[np] = static_cast<uint16_t*>(c->peer_xbuf[p]) + static_cast<size_t>(c->rank) * n_local;
        landed[np] = c->peer_flags[p] + kMaxWorld + c->rank;
        ++np;
    }
    const char* msg = nullptr;
    int grid = 0;
    cudaError_t e = sdq::launch_qmm_tc_push(x, m, k, wq, scales, biases, n_local, bits, sdq::bias_only(bias_local),
                                            out + static_cast<size_t>(c->rank) * n_local, ldy, st, &msg, peers,
                                            landed, np, 0, &grid);
    if (e != cudaSuccess) {
        if (msg) {
            t_shard_msg = std::string(fn) + ": " + msg;
            return sdq::set_error_message(SDQ_ERR_CUDA, t_shard_msg.c_str());
        }
        return cuda_err("tensor-core kernel", e);
    }
    // Every peer runs as many CTAs as this rank (the same shapes on the same parts); the
    // output is whole once every peer's count has grown by that many.
    c->landed_target += static_cast<uint32_t>(grid);
    wait_landed<<<1, kMaxWorld, 0, st>>>(c->flags + kMaxWorld, c->world, c->rank, c->landed_target);
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_err("landed wait", e);
    if (y != out) {
        const int threads = 256;
        const bool v8 = (reinterpret_cast<uintptr_t>(y) % 16) == 0 && total % 8 == 0;
        const int64_t work = v8 ? static_cast<int64_t>(total / 8) : static_cast<int64_t>(total);
        int64_t g = (work + threads - 1) / threads;
        if (g > 4096) g = 4096;
        if (v8)
            copy_v8<<<(int)g, threads, 0, st>>>(reinterpret_cast<const uint4*>(out), static_cast<uint4*>(y), work);
        else
            copy_v1<<<(int)g, threads, 0, st>>>(out, static_cast<uint16_t*>(y), work);
        if ((e = cudaGetLastError()) != cudaSuccess) return cuda_err("output copy", e);
    }
    return sdq::set_error_message(SDQ_OK, "");
}

extern "C" {

int sdq_comm_unique_id(uint8_t out_id[128]) {
    if (!out_id) return sdq::set_error_message(SDQ_ERR_INVALID, "sdq_comm_unique_id: null output");
    static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id is 128 bytes");
    ncclUniqueId id;
    ncclResult_t r = ncclGetUniqueId(&id);
    if (r != ncclSuccess) return nccl_fail("ncclGetUniqueId", r);
    std::memcpy(out_id, &id, 128);
    return sdq::set_error_message(SDQ_OK, "");
}

int sdq_comm_init(const uint8_t id[128], int world, int rank, void** comm_out) {
    if (!id || !comm_out) return sdq::set_error_message(SDQ_ERR_INVALID, "sdq_comm_init: null argument");
    if (world < 1 || rank < 0 || rank >= world)
        return sdq::set_error_message(SDQ_ERR_INVALID, "sdq_comm_init: need 0 <= rank < world");
    ncclUniqueId uid;
    std::memcpy(&uid, id, 128);
    Comm* c = new Comm;
    c->rank = rank;
    c->world = world;
    cudaGetDevice(&c->device);
    ncclResult_t r = ncclCommInitRank(&c->nccl, world, uid, rank);
    if (r != ncclSuccess) {
        delete c;
        return nccl_fail("ncclCommInitRank", r);
    }
    if (world > 1) {
        // Resources of the overlapped exchange; if any is missing the plain path runs.
        bool okr = world <= kMaxWorld &&
                   cudaStreamCreateWithFlags(&c->side, cudaStreamNonBlocking) == cudaSuccess &&
                   cudaMalloc(reinterpret_cast<void**>(&c->handles_dev), world * sizeof(cudaIpcMemHandle_t)) ==
                       cudaSuccess;
        okr = okr && wait_value_fn() != nullptr && write_value_fn() != nullptr && setup_flags(c);
        if (!okr) {
            cudaGetLastError();
            release_flags(c);
            if (c->handles_dev) cudaFree(c->handles_dev);
            if (c->side) cudaStreamDestroy(c->side);
            c->handles_dev = nullptr;
            c->side = nullptr;
        }
    }
    *comm_out = c;
    return sdq::set_error_message(SDQ_OK, "");
}

int sdq_comm_output(void* comm, int64_t m, int64_t n, void** out) {
    if (!comm || !out || m <= 0 || n <= 0)
        return sdq::set_error_message(SDQ_ERR_INVALID, "sdq_comm_output: null argument or empty shape");
    Comm* c = static_cast<Comm*>(comm);
    const int rc = ensure_exchange_buffer(c, static_cast<size_t>(m) * static_cast<size_t>(n) * sizeof(uint16_t),
                                          "sdq_comm_output");
    if (rc != SDQ_OK) return rc;
    *out = c->xbuf;
    return sdq::set_error_message(SDQ_OK, "");
}

int sdq_comm_destroy(void* comm) {
    if (!comm) return sdq::set_error_message(SDQ_OK, "");
    Comm* c = static_cast<Comm*>(comm);
    if (c->side) {
        // This rank's kernels may still store into the peers' outputs through the mappings.
        cudaDeviceSynchronize();
        for (int p = 0; p < c->world; ++p)
            if (c->peer_xbuf[p]) cudaIpcCloseMemHandle(c->peer_xbuf[p]);
        if (c->xbuf) cudaFree(c->xbuf);
        release_flags(c);
        cudaFree(c->handles_dev);
        cudaStreamDestroy(c->side);
    } else if (c->xbuf) {
        cudaDeviceSynchronize();
        cudaFree(c->xbuf);
    }
    ncclResult_t r = ncclCommDestroy(c->nccl);
    delete c;
    if (r != ncclSuccess) return nccl_fail("ncclCommDestroy", r);
    return sdq::set_error_message(SDQ_OK, "");
}

static int sharded_impl(const void* x, sdq_dtype x_dtype, int64_t m, int64_t k, const uint32_t* wq,
                        const void* scales, const void* biases, sdq_dtype sb_dtype, int64_t n_local,
                        int group_size, int bits, const void* bias_local, void* y_shards, void* y,
                        sdq_dtype y_dtype, void* comm, void* stream, bool may_overlap) {
    if (!comm || !y_shards)
        return sdq::set_error_message(SDQ_ERR_INVALID,
                                      "sdq_quantized_matmul_sharded: comm and y_shards must be non-null");
    if (x_dtype != SDQ_BF16 || sb_dtype != SDQ_BF16 || y_dtype != SDQ_BF16)
        return sdq::set_error_message(SDQ_ERR_UNSUPPORTED,
                                      "sdq_quantized_matmul_sharded: x, y, scales and biases must be bf16");
    if (reinterpret_cast<uintptr_t>(y_shards) % 16 != 0 ||
        (y && reinterpret_cast<uintptr_t>(y) % 16 != 0))
        return sdq::set_error_message(SDQ_ERR_INVALID,
                                      "sdq_quantized_matmul_sharded: y_shards and y need 16-byte alignment");
    Comm* c = static_cast<Comm*>(comm);
    if (m <= 0 || n_local <= 0)
        return sdq::set_error_message(SDQ_ERR_INVALID,
                                      "sdq_quantized_matmul_sharded: m and n_local must be >= 1");
    // y inside the communicator's output buffer must fit in it: growing the buffer would
    // free the memory y points to.
    const uintptr_t yb = reinterpret_cast<uintptr_t>(y), xb = reinterpret_cast<uintptr_t>(c->xbuf);
    if (y && c->xbuf && yb >= xb && yb < xb + c->xbuf_cap &&
        yb + static_cast<size_t>(m) * n_local * c->world * sizeof(uint16_t) > xb + c->xbuf_cap)
        return sdq::set_error_message(SDQ_ERR_INVALID,
                                      "sdq_quantized_matmul_sharded: y lies in the communicator's output "
                                      "buffer, which is smaller than the output; call sdq_comm_output "
                                      "with this shape first");
    const size_t chunk = static_cast<size_t>(m) * static_cast<size_t>(n_local);
    uint16_t* mine = static_cast<uint16_t*>(y_shards) + static_cast<size_t>(c->rank) * chunk;
    if (may_overlap && c->world > 1 && y != nullptr && c->side != nullptr && m > 8) {
        const int rc = sharded_overlapped(c, x, x_dtype, m, k, wq, scales, biases, sb_dtype, n_local,
                                          group_size, bits, bias_local, y, y_dtype, stream);
        if (rc != kNotOverlapped) return rc;
    }
    int rc = sdq_quantized_matmul(x, x_dtype, m, k, wq, scales, biases, sb_dtype, n_local, 1,
                                  group_size, bits, "affine", bias_local, mine, y_dtype, stream);
    if (rc != SDQ_OK) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (c->world > 1) {
        ncclResult_t r = ncclAllGather(mine, y_shards, chunk, ncclBfloat16, c->nccl, st);
        if (r != ncclSuccess) return nccl_fail("ncclAllGather", r);
    }
    if (y) {
        cudaError_t e = launch_permute(y_shards, y, m, 0, m, n_local, c->world, st);
        if (e != cudaSuccess) {
            t_shard_msg = std::string("sdq_quantized_matmul_sharded: permute kernel: ") +
                          cudaGetErrorString(e);
            return sdq::set_error_message(SDQ_ERR_CUDA, t_shard_msg.c_str());
        }
    }
    return sdq::set_error_message(SDQ_OK, "");
}

int sdq_quantized_matmul_sharded(const void* x, sdq_dtype x_dtype, int64_t m, int64_t k,
                                 const uint32_t* wq, const void* scales, const void* biases,
                                 sdq_dtype sb_dtype, int64_t n_local, int group_size, int bits,
                                 const void* bias_local, void* y_shards, void* y,
                                 sdq_dtype y_dtype, void* comm, void* stream) {
    return sharded_impl(x, x_dtype, m, k, wq, scales, biases, sb_dtype, n_local, group_size, bits,
                        bias_local, y_shards, y, y_dtype, comm, stream, true);
}

}  // extern "C"

// ---------------------------------------------------------------- no-allocation variant
// Some callers cannot allocate device memory when they call the sharded linear: an
// engine that hands all of HBM to its own arena at start-up (cudaMalloc would then
// fail, or escape its accounting), or a host loop that must not stall (cudaFree
// synchronises the whole device).  For them the [world, m, n_local] all-gather
// buffer lives in this file-scope array instead of a caller buffer.  It costs
// kStaticShardBytes of device memory on every GPU that loads the library, for as
// long as the process runs, and bounds world * m * n_local.
namespace sdq {
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

unsigned long long current_context_id() {
    static CtxGetIdFn get_id = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            return reinterpret_cast<CtxGetIdFn>(p);
        return static_cast<CtxGetIdFn>(nullptr);
    }();
    unsigned long long id = 0;
    if (get_id == nullptr || get_id(nullptr, &id) != CUDA_SUCCESS) return 0;
    return id;
}
}  // namespace sdq

namespace {

constexpr size_t kStaticShardBytes = size_t(8) << 20;                // 8 MiB
constexpr size_t kStaticShardElems = kStaticShardBytes / sizeof(uint16_t);

static __device__ __align__(256) uint16_t g_static_shards[kStaticShardElems];

// The array's device address on each device, fetched once with that device current.
// In host code the name g_static_shards is only a host-side stand-in; kernels and
// NCCL must be given this address.  The address belongs to the device's context: a
// cudaDeviceReset replaces the context (and reloads the module), so the cache also
// keeps the context's unique id and fetches the address again when it changes.
constexpr int kMaxDevices = 64;
std::mutex g_static_mu;
void* g_static_ptr[kMaxDevices] = {};
unsigned long long g_static_ctx[kMaxDevices] = {};

cudaError_t static_shards_on_current_device(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    // Id 0: no context is current yet (or the driver cannot tell); the lookup below makes
    // the primary context current, and without an id the address is looked up every call.
    const unsigned long long ctx = sdq::current_context_id();
    std::lock_guard<std::mutex> lock(g_static_mu);
    if (!g_static_ptr[dev] || ctx == 0 || g_static_ctx[dev] != ctx) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_static_shards);
        if (e != cudaSuccess) return e;
        g_static_ptr[dev] = p;
        g_static_ctx[dev] = sdq::current_context_id();
    }
    *out = g_static_ptr[dev];
    return cudaSuccess;
}

thread_local char t_static_msg[256];

}  // namespace

extern "C" {

int sdq_quantized_matmul_sharded_static(const void* x, sdq_dtype x_dtype, int64_t m, int64_t k,
                                        const uint32_t* wq, const void* scales, const void* biases,
                                        sdq_dtype sb_dtype, int64_t n_local, int group_size,
                                        int bits, const void* bias_local, void* y,
                                        sdq_dtype y_dtype, void* comm, void* stream) {
    const char* fn = "sdq_quantized_matmul_sharded_static";
    if (!comm || !y) {
        std::snprintf(t_static_msg, sizeof t_static_msg, "%s: comm and y must be non-null", fn);
        return sdq::set_error_message(SDQ_ERR_INVALID, t_static_msg);
    }
    if (m <= 0 || n_local <= 0) {
        std::snprintf(t_static_msg, sizeof t_static_msg, "%s: m and n_local must be >= 1", fn);
        return sdq::set_error_message(SDQ_ERR_INVALID, t_static_msg);
    }
    const Comm* c = static_cast<const Comm*>(comm);
    const double need = static_cast<double>(c->world) * static_cast<double>(m) *
                        static_cast<double>(n_local);
    if (need > static_cast<double>(kStaticShardElems)) {
        std::snprintf(t_static_msg, sizeof t_static_msg,
                      "%s: world*m*n_local = %.0f bf16 values exceeds the static scratch of %zu "
                      "(%zu MiB); use sdq_quantized_matmul_sharded with a caller buffer",
                      fn, need, kStaticShardElems, kStaticShardBytes >> 20);
        return sdq::set_error_message(SDQ_ERR_INVALID, t_static_msg);
    }
    // Every GPU holds its own copy of the array: a call made with another device current
    // would hand NCCL (bound to the communicator's device) another GPU's copy.
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess && dev != c->device) {
        std::snprintf(t_static_msg, sizeof t_static_msg,
                      "%s: the current device is %d but the communicator belongs to device %d", fn, dev,
                      c->device);
        return sdq::set_error_message(SDQ_ERR_INVALID, t_static_msg);
    }
    void* scratch = nullptr;
    if (e == cudaSuccess) e = static_shards_on_current_device(&scratch);
    if (e != cudaSuccess) {
        std::snprintf(t_static_msg, sizeof t_static_msg,
                      "%s: cudaGetSymbolAddress of the static scratch: %s", fn, cudaGetErrorString(e));
        return sdq::set_error_message(SDQ_ERR_CUDA, t_static_msg);
    }
    // The plain exchange: the overlapped one may allocate its exchange buffer.
    return sharded_impl(x, x_dtype, m, k, wq, scales, biases, sb_dtype, n_local, group_size, bits,
                        bias_local, scratch, y, y_dtype, comm, stream, false);
}

}  // extern "C"
