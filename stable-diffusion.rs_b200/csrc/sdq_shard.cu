// sdq_shard.cu -- the column-sharded quantised linear over NCCL.
//
// Each rank holds a contiguous block of output features (rows of the packed
// weight), runs the single-GPU kernel on it, and the [m, n_local] results are
// exchanged over NVLink / NVSwitch into [world, m, n_local] on every rank; a
// permute kernel turns that into [m, n].
//
// When the output is wanted as [m, n] on two or more ranks and M spans several
// token tiles, the exchange overlaps the compute and uses no SMs: the tensor-core
// kernel counts, per chunk of token tiles, the output tiles it has finished; a
// library-owned side stream waits on each chunk's count (cuStreamWaitValue32) and
// pushes that chunk's rows with the copy engines straight into every peer's
// exchange buffer (IPC-mapped device memory, over NVLink) while the kernel computes
// the next chunk -- without SMs.  A small NCCL all-reduce then tells each rank that
// all pushes into its buffer have landed, and one permute kernel builds [m, n].
// (NCCL's send / receive kernels did not start until the compute kernel had
// finished, so they could not overlap it; per-chunk arrival flags with strided
// copies into Y were slower than the single permute.)  A kernel that gives up
// raises every count to its maximum, so the side stream never waits for ever.  The
// exchange buffer is allocated on the first overlapped call and grows collectively
// (every rank calls with the same shapes); a second small all-reduce at the start
// of each call keeps a fast rank from pushing into a buffer that a slower one is
// still permuting.
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

constexpr int kMaxChunks = 16;     // chunk counters per communicator
constexpr int kChunks = 8;         // chunks the overlapped path aims for
constexpr int kMaxWorld = 64;

struct Comm {
    ncclComm_t nccl = nullptr;
    int rank = 0;
    int world = 1;
    int device = 0;
    // Overlapped exchange (set up when world > 1; the plain path runs without it).
    cudaStream_t side = nullptr;
    cudaEvent_t ev_start = nullptr, ev_end = nullptr, ev_bar = nullptr;
    // One push stream per peer, so that the pushes to different peers run concurrently
    // on different copy engines (one stream runs its copies one after another).
    cudaStream_t push[kMaxWorld] = {};
    cudaEvent_t push_done[kMaxWorld] = {};
    uint32_t* counters = nullptr;          // kMaxChunks completion counts + 1 barrier word
    // This rank's exchange buffer ([world, m, n_local] bf16; peers push into it) and the
    // peers' buffers as mapped here.
    void* xbuf = nullptr;
    size_t xbuf_cap = 0;
    void* peer_xbuf[kMaxWorld] = {};
    cudaIpcMemHandle_t* handles_dev = nullptr;   // world handles, for the one-off exchange
};

void destroy_push_streams(Comm* c) {
    for (int p = 0; p < kMaxWorld; ++p) {
        if (c->push[p]) {
            cudaStreamSynchronize(c->push[p]);
            cudaStreamDestroy(c->push[p]);
        }
        if (c->push_done[p]) cudaEventDestroy(c->push_done[p]);
        c->push[p] = nullptr;
        c->push_done[p] = nullptr;
    }
}

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

// A zero-byte-payload barrier over the communicator on `st`: an all-reduce of one word.
static ncclResult_t side_barrier(Comm* c, cudaStream_t st) {
    uint32_t* w = c->counters + kMaxChunks;
    return ncclAllReduce(w, w, 1, ncclUint32, ncclMax, c->nccl, st);
}

// Make this rank's exchange buffer hold `bytes` and map every peer's (collective: all ranks
// call it with the same size).  Allocates only when the buffer must grow.
static int ensure_exchange_buffer(Comm* c, size_t bytes, const char* fn) {
    if (c->xbuf_cap >= bytes) return SDQ_OK;
    auto fail_cuda = [&](const char* what, cudaError_t e) {
        t_shard_msg = std::string(fn) + ": exchange buffer: " + what + ": " + cudaGetErrorString(e);
        return sdq::set_error_message(SDQ_ERR_CUDA, t_shard_msg.c_str());
    };
    cudaError_t e = cudaStreamSynchronize(c->side);
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

// y[t, p * nl + j] = (p == rank ? own : xbuf[p])[t, j]: the permute of the overlapped path,
// which reads this rank's block from y_shards and the peers' blocks from the exchange buffer.
__global__ void permute_exchange_v8(const uint4* __restrict__ xbuf, const uint4* __restrict__ own,
                                    uint4* __restrict__ y, int64_t m, int64_t nl8, int world, int rank) {
    const int64_t total = (int64_t)world * m * nl8;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t j = i % nl8;
        const int64_t t = (i / nl8) % m;
        const int64_t r = i / (nl8 * m);
        const uint4 v = r == rank ? own[t * nl8 + j] : xbuf[(r * m + t) * nl8 + j];
        y[t * (world * nl8) + r * nl8 + j] = v;
    }
}
__global__ void permute_exchange_v1(const uint16_t* __restrict__ xbuf, const uint16_t* __restrict__ own,
                                    uint16_t* __restrict__ y, int64_t m, int64_t nl, int world, int rank) {
    const int64_t total = (int64_t)world * m * nl;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t j = i % nl;
        const int64_t t = (i / nl) % m;
        const int64_t r = i / (nl * m);
        const uint16_t v = r == rank ? own[t * nl + j] : xbuf[(r * m + t) * nl + j];
        y[t * (world * nl) + r * nl + j] = v;
    }
}

// The overlapped form of sdq_quantized_matmul_sharded (see the file comment).  Returns
// kNotOverlapped, having enqueued nothing, when the shape does not split into chunks.
static int sharded_overlapped(Comm* c, const void* x, sdq_dtype x_dtype, int64_t m, int64_t k,
                              const uint32_t* wq, const void* scales, const void* biases,
                              sdq_dtype sb_dtype, int64_t n_local, int group_size, int bits,
                              const void* bias_local, void* y_shards, void* y, sdq_dtype y_dtype,
                              void* stream) {
    const char* fn = "sdq_quantized_matmul_sharded";
    uint16_t* mine = static_cast<uint16_t*>(y_shards) + static_cast<size_t>(c->rank) * m * n_local;
    int rc = sdq::validate_qmm(x, x_dtype, m, k, wq, scales, biases, sb_dtype, n_local, 1, group_size,
                               bits, "affine", bias_local, mine, y_dtype, fn);
    if (rc != SDQ_OK) return rc;
    const int64_t bt = sdq::qmm_tc_tile_tokens(m, k, n_local, bits, 0);
    const int64_t ntt = (m + bt - 1) / bt;
    if (ntt < 2) return kNotOverlapped;
    // Fewer, larger chunks when there are many peers: every chunk costs a wait and a copy
    // per peer to enqueue.
    const int64_t want_chunks = c->world <= 2 ? kChunks : kChunks / 2;
    int64_t nch = ntt < want_chunks ? ntt : want_chunks;
    const int64_t tpc = (ntt + nch - 1) / nch;           // token tiles per chunk
    nch = (ntt + tpc - 1) / tpc;
    const int64_t nft = (n_local + 127) / 128;
    const size_t block = static_cast<size_t>(m) * n_local;   // elements of one rank's block
    if ((rc = ensure_exchange_buffer(c, c->world * block * sizeof(uint16_t), fn)) != SDQ_OK) return rc;
    uint16_t* xb = static_cast<uint16_t*>(c->xbuf);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    auto cuda_err = [&](const char* what, cudaError_t e) {
        t_shard_msg = std::string(fn) + ": " + what + ": " + cudaGetErrorString(e);
        return sdq::set_error_message(SDQ_ERR_CUDA, t_shard_msg.c_str());
    };
    const ValueFn wait = wait_value_fn();
    // Every rank has finished permuting out of its buffer from the previous call before
    // anyone pushes into it again.
    ncclResult_t r = side_barrier(c, c->side);
    if (r != ncclSuccess) return nccl_fail("ncclAllReduce (barrier)", r);
    cudaError_t e = cudaEventRecord(c->ev_bar, c->side);
    if (e == cudaSuccess) e = cudaMemsetAsync(c->counters, 0, nch * sizeof(uint32_t), st);
    if (e == cudaSuccess) e = cudaEventRecord(c->ev_start, st);
    // The pushes follow the barrier (side) and the counters' reset (st).
    for (int p = 0; e == cudaSuccess && p < c->world; ++p) {
        if (p == c->rank) continue;
        e = cudaStreamWaitEvent(c->push[p], c->ev_bar, 0);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(c->push[p], c->ev_start, 0);
    }
    if (e != cudaSuccess) return cuda_err("stream set-up", e);
    const char* msg = nullptr;
    e = sdq::launch_qmm_tc_signal(x, m, k, wq, scales, biases, n_local, bits,
                                  sdq::bias_only(bias_local), mine, st,
                                  &msg, c->counters, (int)tpc, (int)nch, 0);
    if (e != cudaSuccess) {
        if (msg) {
            t_shard_msg = std::string(fn) + ": " + msg;
            return sdq::set_error_message(SDQ_ERR_CUDA, t_shard_msg.c_str());
        }
        return cuda_err("tensor-core kernel", e);
    }
    // Without stream memory operations every push waits for the whole kernel instead.
    if (wait == nullptr) {
        if ((e = cudaEventRecord(c->ev_start, st)) != cudaSuccess) return cuda_err("stream wait", e);
        for (int p = 0; p < c->world; ++p)
            if (p != c->rank && (e = cudaStreamWaitEvent(c->push[p], c->ev_start, 0)) != cudaSuccess)
                return cuda_err("stream wait", e);
    }
    for (int64_t i = 0; i < nch; ++i) {
        const int64_t t0 = i * tpc, t1 = (i + 1) * tpc < ntt ? (i + 1) * tpc : ntt;
        const int64_t m0 = t0 * bt, m1 = t1 * bt < m ? t1 * bt : m;
        const cuuint32_t target = static_cast<cuuint32_t>((t1 - t0) * nft);
        const size_t off = static_cast<size_t>(m0) * n_local;
        const size_t bytes = static_cast<size_t>(m1 - m0) * n_local * sizeof(uint16_t);
        for (int p = 0; p < c->world; ++p) {
            if (p == c->rank) continue;
            if (wait != nullptr &&
                wait(reinterpret_cast<CUstream>(c->push[p]), reinterpret_cast<CUdeviceptr>(c->counters + i),
                     target, 0 /* GEQ */) != CUDA_SUCCESS)
                return cuda_err("stream wait on a chunk count", cudaErrorUnknown);
            uint16_t* dst = static_cast<uint16_t*>(c->peer_xbuf[p]) + c->rank * block + off;
            if ((e = cudaMemcpyAsync(dst, mine + off, bytes, cudaMemcpyDeviceToDevice, c->push[p])) !=
                cudaSuccess)
                return cuda_err("push to a peer", e);
        }
    }
    for (int p = 0; p < c->world; ++p) {
        if (p == c->rank) continue;
        if ((e = cudaEventRecord(c->push_done[p], c->push[p])) != cudaSuccess ||
            (e = cudaStreamWaitEvent(c->side, c->push_done[p], 0)) != cudaSuccess)
            return cuda_err("push join", e);
    }
    // All pushes into this rank's buffer have landed once every rank has passed here.
    if ((r = side_barrier(c, c->side)) != ncclSuccess) return nccl_fail("ncclAllReduce (barrier)", r);
    const int threads = 256;
    if (n_local % 8 == 0) {
        const int64_t total = static_cast<int64_t>(c->world) * m * (n_local / 8);
        int64_t grid = (total + threads - 1) / threads;
        if (grid > 4096) grid = 4096;
        permute_exchange_v8<<<(int)grid, threads, 0, c->side>>>(
            reinterpret_cast<const uint4*>(xb), reinterpret_cast<const uint4*>(mine),
            static_cast<uint4*>(y), m, n_local / 8, c->world, c->rank);
    } else {
        const int64_t total = static_cast<int64_t>(c->world) * m * n_local;
        int64_t grid = (total + threads - 1) / threads;
        if (grid > 4096) grid = 4096;
        permute_exchange_v1<<<(int)grid, threads, 0, c->side>>>(xb, mine, static_cast<uint16_t*>(y), m,
                                                                n_local, c->world, c->rank);
    }
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_err("permute kernel", e);
    e = cudaEventRecord(c->ev_end, c->side);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(st, c->ev_end, 0);
    if (e != cudaSuccess) return cuda_err("stream join", e);
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
                   cudaEventCreateWithFlags(&c->ev_start, cudaEventDisableTiming) == cudaSuccess &&
                   cudaEventCreateWithFlags(&c->ev_end, cudaEventDisableTiming) == cudaSuccess &&
                   cudaEventCreateWithFlags(&c->ev_bar, cudaEventDisableTiming) == cudaSuccess &&
                   cudaMalloc(reinterpret_cast<void**>(&c->counters), (kMaxChunks + 1) * sizeof(uint32_t)) ==
                       cudaSuccess &&
                   world <= kMaxWorld &&
                   cudaMalloc(reinterpret_cast<void**>(&c->handles_dev), world * sizeof(cudaIpcMemHandle_t)) ==
                       cudaSuccess;
        for (int p = 0; okr && p < world; ++p)
            okr = p == rank ||
                  (cudaStreamCreateWithFlags(&c->push[p], cudaStreamNonBlocking) == cudaSuccess &&
                   cudaEventCreateWithFlags(&c->push_done[p], cudaEventDisableTiming) == cudaSuccess);
        if (!okr) {
            cudaGetLastError();
            destroy_push_streams(c);
            if (c->ev_bar) cudaEventDestroy(c->ev_bar);
            c->ev_bar = nullptr;
            if (c->handles_dev) cudaFree(c->handles_dev);
            if (c->counters) cudaFree(c->counters);
            if (c->ev_end) cudaEventDestroy(c->ev_end);
            if (c->ev_start) cudaEventDestroy(c->ev_start);
            if (c->side) cudaStreamDestroy(c->side);
            c->counters = nullptr;
            c->handles_dev = nullptr;
            c->ev_start = c->ev_end = nullptr;
            c->side = nullptr;
        }
    }
    *comm_out = c;
    return sdq::set_error_message(SDQ_OK, "");
}

int sdq_comm_destroy(void* comm) {
    if (!comm) return sdq::set_error_message(SDQ_OK, "");
    Comm* c = static_cast<Comm*>(comm);
    if (c->side) {
        cudaStreamSynchronize(c->side);
        for (int p = 0; p < c->world; ++p)
            if (c->peer_xbuf[p]) cudaIpcCloseMemHandle(c->peer_xbuf[p]);
        if (c->xbuf) cudaFree(c->xbuf);
        cudaFree(c->handles_dev);
        cudaFree(c->counters);
        destroy_push_streams(c);
        cudaEventDestroy(c->ev_bar);
        cudaEventDestroy(c->ev_end);
        cudaEventDestroy(c->ev_start);
        cudaStreamDestroy(c->side);
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
    if (reinterpret_cast<uintptr_t>(y_shards) % 16 != 0 ||
        (y && reinterpret_cast<uintptr_t>(y) % 16 != 0))
        return sdq::set_error_message(SDQ_ERR_INVALID,
                                      "sdq_quantized_matmul_sharded: y_shards and y need 16-byte alignment");
    Comm* c = static_cast<Comm*>(comm);
    if (m <= 0 || n_local <= 0)
        return sdq::set_error_message(SDQ_ERR_INVALID,
                                      "sdq_quantized_matmul_sharded: m and n_local must be >= 1");
    const size_t chunk = static_cast<size_t>(m) * static_cast<size_t>(n_local);
    uint16_t* mine = static_cast<uint16_t*>(y_shards) + static_cast<size_t>(c->rank) * chunk;
    if (may_overlap && c->world > 1 && y != nullptr && c->side != nullptr && m > 8) {
        const int rc = sharded_overlapped(c, x, x_dtype, m, k, wq, scales, biases, sb_dtype, n_local,
                                          group_size, bits, bias_local, y_shards, y, y_dtype, stream);
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
namespace {

constexpr size_t kStaticShardBytes = size_t(8) << 20;                // 8 MiB
constexpr size_t kStaticShardElems = kStaticShardBytes / sizeof(uint16_t);

static __device__ __align__(256) uint16_t g_static_shards[kStaticShardElems];

// The array's device address on each device, fetched once with that device current.
// In host code the name g_static_shards is only a host-side stand-in; kernels and
// NCCL must be given this address.
constexpr int kMaxDevices = 64;
std::mutex g_static_mu;
void* g_static_ptr[kMaxDevices] = {};

cudaError_t static_shards_on_current_device(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_static_mu);
    if (!g_static_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_static_shards);
        if (e != cudaSuccess) return e;
        g_static_ptr[dev] = p;
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
    void* scratch = nullptr;
    const cudaError_t e = static_shards_on_current_device(&scratch);
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
