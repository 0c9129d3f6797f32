// sdq_shard.cu -- the column-sharded quantised linear over NCCL.
//
// Each rank holds a contiguous block of output features (rows of the packed
// weight), runs the single-GPU kernel on it, and the [m, n_local] results are
// all-gathered over NVLink / NVSwitch.  NCCL's all-gather concatenates rank
// chunks, so a permute kernel turns [world, m, n_local] into [m, n].
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include <cuda_runtime.h>
#include <nccl.h>

#include "../../include/sdq.h"

namespace sdq {
namespace {

thread_local std::string t_shard_msg;

struct Comm {
    ncclComm_t nccl = nullptr;
    int rank = 0;
    int world = 1;
    int device = 0;
};

// y[t, r * nl + j] = shards[r, t, j]; 8 bf16 (16 bytes) per thread when
// n_local % 8 == 0, else one element per thread.
__global__ void permute_shards_v8(const uint4* __restrict__ shards, uint4* __restrict__ y,
                                  int64_t m, int64_t nl8, int world) {
    const int64_t total = (int64_t)world * m * nl8;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t j = i % nl8;
        const int64_t t = (i / nl8) % m;
        const int64_t r = i / (nl8 * m);
        y[t * (world * nl8) + r * nl8 + j] = shards[i];
    }
}
__global__ void permute_shards_v1(const uint16_t* __restrict__ shards, uint16_t* __restrict__ y,
                                  int64_t m, int64_t nl, int world) {
    const int64_t total = (int64_t)world * m * nl;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t j = i % nl;
        const int64_t t = (i / nl) % m;
        const int64_t r = i / (nl * m);
        y[t * (world * nl) + r * nl + j] = shards[i];
    }
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
    *comm_out = c;
    return sdq::set_error_message(SDQ_OK, "");
}

int sdq_comm_destroy(void* comm) {
    if (!comm) return sdq::set_error_message(SDQ_OK, "");
    Comm* c = static_cast<Comm*>(comm);
    ncclResult_t r = ncclCommDestroy(c->nccl);
    delete c;
    if (r != ncclSuccess) return nccl_fail("ncclCommDestroy", r);
    return sdq::set_error_message(SDQ_OK, "");
}

int sdq_quantized_matmul_sharded(const void* x, sdq_dtype x_dtype, int64_t m, int64_t k,
                                 const uint32_t* wq, const void* scales, const void* biases,
                                 sdq_dtype sb_dtype, int64_t n_local, int group_size, int bits,
                                 const void* bias_local, void* y_shards, void* y,
                                 sdq_dtype y_dtype, void* comm, void* stream) {
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
    int rc = sdq_quantized_matmul(x, x_dtype, m, k, wq, scales, biases, sb_dtype, n_local, 1,
                                  group_size, bits, "affine", bias_local, mine, y_dtype, stream);
    if (rc != SDQ_OK) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (c->world > 1) {
        ncclResult_t r = ncclAllGather(mine, y_shards, chunk, ncclBfloat16, c->nccl, st);
        if (r != ncclSuccess) return nccl_fail("ncclAllGather", r);
    }
    if (y) {
        const int threads = 256;
        if (n_local % 8 == 0) {
            const int64_t total = static_cast<int64_t>(c->world) * m * (n_local / 8);
            int64_t grid = (total + threads - 1) / threads;
            if (grid > 4096) grid = 4096;
            permute_shards_v8<<<(int)grid, threads, 0, st>>>(static_cast<const uint4*>(y_shards),
                                                             static_cast<uint4*>(y), m, n_local / 8,
                                                             c->world);
        } else {
            const int64_t total = static_cast<int64_t>(c->world) * m * n_local;
            int64_t grid = (total + threads - 1) / threads;
            if (grid > 4096) grid = 4096;
            permute_shards_v1<<<(int)grid, threads, 0, st>>>(static_cast<const uint16_t*>(y_shards),
                                                             static_cast<uint16_t*>(y), m, n_local,
                                                             c->world);
        }
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) {
            t_shard_msg = std::string("sdq_quantized_matmul_sharded: permute kernel: ") +
                          cudaGetErrorString(e);
            return sdq::set_error_message(SDQ_ERR_CUDA, t_shard_msg.c_str());
        }
    }
    return sdq::set_error_message(SDQ_OK, "");
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
    return sdq_quantized_matmul_sharded(x, x_dtype, m, k, wq, scales, biases, sb_dtype, n_local,
                                        group_size, bits, bias_local, scratch, y, y_dtype, comm,
                                        stream);
}

}  // extern "C"
