// sdq_api.cu -- the C ABI (include/sdq.h): argument validation, per-thread
// error messages, and kernel selection.  No CPU fallback: without an sm_100
// device every compute entry point fails with SDQ_ERR_CUDA.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include <cuda_runtime.h>

#include "../../include/sdq.h"
#include "sdq_internal.h"

namespace sdq {
namespace {

thread_local std::string t_last_error;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return code;
}

int ok() {
    t_last_error.clear();
    return SDQ_OK;
}

int cuda_fail(const char* what, cudaError_t e) {
    return fail(SDQ_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

struct DevInfo {
    bool probed = false;
    bool supported = false;
    int sms = 0;
    int major = 0, minor = 0;
};
DevInfo g_dev[64];

// Ensure the current device is an sm_100 part (the library carries sm_100a
// code only).  Returns SDQ_OK or an error code with the message set.
int check_device() {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail("no CUDA device", e);
    if (dev < 0 || dev >= 64) return fail(SDQ_ERR_CUDA, "device ordinal %d out of range", dev);
    DevInfo& d = g_dev[dev];
    if (!d.probed) {
        if ((e = cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess ||
            (e = cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev)) != cudaSuccess ||
            (e = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
            return cuda_fail("cudaDeviceGetAttribute", e);
        d.supported = d.major == 10 && d.minor == 0;
        d.probed = true;
    }
    if (!d.supported)
        return fail(SDQ_ERR_CUDA, "device %d is sm_%d%d; libsdq carries sm_100a code only", dev,
                    d.major, d.minor);
    return SDQ_OK;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Shared checks of the quantisation parameters; resolves defaults in place.
int check_qparams(int& group_size, int& bits, const char* mode, const char* fn) {
    if (group_size <= 0) group_size = 64;
    if (bits <= 0) bits = 4;
    if (mode != nullptr && std::strcmp(mode, "affine") != 0)
        return fail(SDQ_ERR_UNSUPPORTED, "%s: mode \"%s\" is not supported (only \"affine\")", fn,
                    mode);
    if (group_size != 64)
        return fail(SDQ_ERR_UNSUPPORTED, "%s: group_size %d is not supported (only 64)", fn,
                    group_size);
    if (bits == 2 || bits == 3 || bits == 5 || bits == 6)
        return fail(SDQ_ERR_UNSUPPORTED, "%s: bits %d is not supported (only 4 and 8)", fn, bits);
    if (bits != 4 && bits != 8)
        return fail(SDQ_ERR_INVALID, "%s: bits must be one of 2, 3, 4, 5, 6, 8; got %d", fn, bits);
    return SDQ_OK;
}

int check_nk(int64_t n, int64_t k, const char* fn) {
    if (n <= 0) return fail(SDQ_ERR_INVALID, "%s: n (rows, out features) must be >= 1; got %lld", fn, (long long)n);
    if (k <= 0) return fail(SDQ_ERR_INVALID, "%s: k (in features) must be >= 1; got %lld", fn, (long long)k);
    if (k % 64 != 0)
        return fail(SDQ_ERR_INVALID,
                    "%s: k = %lld is not a multiple of the group size 64 (such weights stay dense)",
                    fn, (long long)k);
    if (n > INT32_MAX || k > INT32_MAX)
        return fail(SDQ_ERR_INVALID, "%s: n and k must each be < 2^31", fn);
    return SDQ_OK;
}

}  // namespace

int set_error_message(int code, const char* msg) {
    if (code == SDQ_OK) t_last_error.clear();
    else t_last_error = msg ? msg : "";
    return code;
}

int num_sms() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    DevInfo& d = g_dev[dev];
    if (!d.probed) check_device();
    return d.sms > 0 ? d.sms : 148;
}

}  // namespace sdq

using namespace sdq;

namespace sdq {
// The argument checks of sdq_quantized_matmul, shared with the overlapped sharded path.
int validate_qmm(const void* x, sdq_dtype x_dtype, int64_t m, int64_t k, const uint32_t* wq,
                 const void* scales, const void* biases, sdq_dtype sb_dtype, int64_t n,
                 int transpose, int& group_size, int& bits, const char* mode, const void* bias,
                 const void* y, sdq_dtype y_dtype, const char* fn) {
    int rc;
    if ((rc = check_qparams(group_size, bits, mode, fn))) return rc;
    if ((rc = check_nk(n, k, fn))) return rc;
    if (m <= 0) return fail(SDQ_ERR_INVALID, "%s: m (rows of x) must be >= 1; got %lld", fn, (long long)m);
    if (m > INT32_MAX) return fail(SDQ_ERR_INVALID, "%s: m must be < 2^31", fn);
    if (!transpose)
        return fail(SDQ_ERR_UNSUPPORTED,
                    "%s: transpose=false is not supported (weights are [out, in]; pass true)", fn);
    if (!x || !wq || !scales || !biases || !y)
        return fail(SDQ_ERR_INVALID, "%s: x, wq, scales, biases and y must be non-null", fn);
    auto bf_or_f32 = [](sdq_dtype d) { return d == SDQ_BF16 || d == SDQ_F32; };
    if (!bf_or_f32(x_dtype) || !bf_or_f32(y_dtype) || !bf_or_f32(sb_dtype))
        return fail(SDQ_ERR_UNSUPPORTED, "%s: x, y, scales and biases must be bf16 or f32", fn);
    const size_t ye = y_dtype == SDQ_F32 ? 4 : 2, se = sb_dtype == SDQ_F32 ? 4 : 2;
    if (!aligned(x, 16) || !aligned(wq, 16) || !aligned(y, ye) || !aligned(scales, se) ||
        !aligned(biases, se) || (bias && !aligned(bias, ye)))
        return fail(SDQ_ERR_INVALID, "%s: misaligned pointer (x and wq need 16 bytes)", fn);
    return check_device();
}

// The dispatch shared by the matmul entry points: the small-M weight stream where it
// serves the shape, the tensor-core kernel otherwise.
int run_qmm(const void* x, int64_t m, int64_t k, const uint32_t* wq, const void* scales,
            const void* biases, int64_t n, int bits, const EpiArgs& epi, void* y, void* stream,
            const char* fn) {
    const char* msg = nullptr;
    bool taken = false;
    cudaError_t e = launch_qmv(x, false, m, k, wq, scales, biases, false, n, bits, epi, y, epi.f32,
                               static_cast<cudaStream_t>(stream), &msg, &taken);
    if (e == cudaSuccess && !taken)
        e = launch_qmm_tc(x, m, k, wq, scales, biases, n, bits, epi, y,
                          static_cast<cudaStream_t>(stream), &msg);
    if (e != cudaSuccess) {
        if (msg) return fail(SDQ_ERR_CUDA, "%s: %s", fn, msg);
        return fail(SDQ_ERR_CUDA, "%s: kernel launch: %s (%s)", fn, cudaGetErrorString(e),
                    cudaGetErrorName(e));
    }
    return ok();
}

// sdq_quantized_matmul after its argument checks: the bf16 kernels directly, or, for f32
// activations or scales, after rounding them to bf16 (nearest even) into stream-ordered
// temporaries -- the one place the library allocates on the compute path, through the
// stream's memory pool.  Scales and biases from sdq_quantize are bf16 values already and stay
// exact; an f32 result is the f32 accumulator.
int qmm_any_dtype(const void* x, sdq_dtype x_dtype, int64_t m, int64_t k, const uint32_t* wq,
                  const void* scales, const void* biases, sdq_dtype sb_dtype, int64_t n, int bits,
                  const void* bias, void* y, sdq_dtype y_dtype, cudaStream_t st, const char* fn) {
    EpiArgs epi = bias_only(bias);
    epi.f32 = y_dtype == SDQ_F32;
    if (x_dtype == SDQ_BF16 && sb_dtype == SDQ_BF16)
        return run_qmm(x, m, k, wq, scales, biases, n, bits, epi, y, st, fn);
    const size_t xb = x_dtype == SDQ_F32 ? ((size_t)m * k * 2 + 255) & ~(size_t)255 : 0;
    const size_t sbb = sb_dtype == SDQ_F32 ? ((size_t)n * (k / 64) * 2 + 255) & ~(size_t)255 : 0;
    uint8_t* tmp = nullptr;
    cudaError_t e = cudaMallocAsync(reinterpret_cast<void**>(&tmp), xb + 2 * sbb, st);
    if (e != cudaSuccess) return fail(SDQ_ERR_CUDA, "%s: cudaMallocAsync (f32 inputs): %s", fn,
                                      cudaGetErrorString(e));
    const void* xk = x;
    const void* sk = scales;
    const void* bk = biases;
    if (x_dtype == SDQ_F32) {
        e = launch_f32_to_bf16(static_cast<const float*>(x), tmp, m * k, st);
        xk = tmp;
    }
    if (e == cudaSuccess && sb_dtype == SDQ_F32) {
        e = launch_f32_to_bf16(static_cast<const float*>(scales), tmp + xb, n * (k / 64), st);
        if (e == cudaSuccess) e = launch_f32_to_bf16(static_cast<const float*>(biases), tmp + xb + sbb, n * (k / 64), st);
        sk = tmp + xb;
        bk = tmp + xb + sbb;
    }
    if (e != cudaSuccess) {
        cudaFreeAsync(tmp, st);
        return fail(SDQ_ERR_CUDA, "%s: f32 -> bf16 conversion: %s", fn, cudaGetErrorString(e));
    }
    int rc = run_qmm(xk, m, k, wq, sk, bk, n, bits, epi, y, st, fn);
    e = cudaFreeAsync(tmp, st);
    if (rc == SDQ_OK && e != cudaSuccess) return fail(SDQ_ERR_CUDA, "%s: cudaFreeAsync: %s", fn,
                                                      cudaGetErrorString(e));
    return rc;
}

// ---------------------------------------------------------------- host-buffer pipeline
// Each device keeps two copy streams (upload, download) and a ring of events, made once per
// CUDA context.  A call records an event on the caller's stream; both copy streams wait for
// it, so the call is ordered after the caller's earlier work on x_dev / y_dev / the host
// buffers.  Then, per row chunk c: the upload stream copies x rows into x_dev and records
// up[c]; the caller's stream waits for up[c] and runs the product of those rows into y_dev,
// recording mm[c]; the download stream waits for mm[c] and copies the rows of y out.  The
// caller's stream finally waits for the download stream.  Uploads run back to back on one
// copy engine, downloads on the other (PCIe is full duplex), and each chunk's product runs
// while later chunks upload, so the call costs about the upload of x plus one chunk's
// product and download.  The events are re-recorded by the next call; a wait uses the
// record current when the wait was issued, and the lock keeps calls from interleaving
// their records and waits.
constexpr int kPipeChunks = 64;
struct HostPipe {
    unsigned long long ctx = 0;
    cudaStream_t up = nullptr, down = nullptr;
    cudaEvent_t start = nullptr, done = nullptr;
    cudaEvent_t up_ev[kPipeChunks] = {}, mm_ev[kPipeChunks] = {};
};
std::mutex g_pipe_mu;
HostPipe g_pipe[64];

cudaError_t pipe_for_current_device(HostPipe** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    HostPipe& p = g_pipe[dev];
    const unsigned long long ctx = current_context_id();
    if (p.up == nullptr || ctx == 0 || p.ctx != ctx) {
        // A new context (first use, or after a cudaDeviceReset, which destroyed the old
        // streams and events with their context): make them anew.
        p = HostPipe{};
        const unsigned fl = cudaEventDisableTiming;
        if ((e = cudaStreamCreateWithFlags(&p.up, cudaStreamNonBlocking)) != cudaSuccess ||
            (e = cudaStreamCreateWithFlags(&p.down, cudaStreamNonBlocking)) != cudaSuccess ||
            (e = cudaEventCreateWithFlags(&p.start, fl)) != cudaSuccess ||
            (e = cudaEventCreateWithFlags(&p.done, fl)) != cudaSuccess)
            return e;
        for (int i = 0; i < kPipeChunks; ++i)
            if ((e = cudaEventCreateWithFlags(&p.up_ev[i], fl)) != cudaSuccess ||
                (e = cudaEventCreateWithFlags(&p.mm_ev[i], fl)) != cudaSuccess)
                return e;
        p.ctx = ctx;
    }
    *out = &p;
    return cudaSuccess;
}

// Row counts of the chunks, into rows[kPipeChunks]; returns how many.  Chunks of `asked`
// rows, or with `asked` = 0 of about m / 8 rows (a multiple of 64, 128 to 1024: a product
// that still fills the SMs, few enough calls that the host keeps ahead of the copies); more
// rows when m would need over kPipeChunks chunks.  On a B200 over PCIe 5 (cfg2: 100.7 MB up,
// 25.2 MB down) 384- and 512-row chunks both took 2.02-2.03 ms, 128-row chunks 2.39 ms;
// splitting the last chunk into halves and quarters to shorten the tail (2.04 ms) and
// alternating two upload streams (2.10-2.19 ms) measured slower.
int pipe_chunks(int64_t m, int64_t asked, int64_t* rows) {
    int64_t r = asked;
    if (r <= 0) {
        r = ((m + 7) / 8 + 63) / 64 * 64;
        r = r < 128 ? 128 : (r > 1024 ? 1024 : r);
    }
    const int64_t floor_rows = (m + kPipeChunks - 1) / kPipeChunks;
    if (r < floor_rows) r = floor_rows;
    int n = 0;
    for (int64_t r0 = 0; r0 < m; r0 += r) rows[n++] = m - r0 < r ? m - r0 : r;
    return n;
}

int qmm_host_pipeline(const void* x_host, sdq_dtype x_dtype, int64_t m, int64_t k, const uint32_t* wq,
                      const void* scales, const void* biases, sdq_dtype sb_dtype, int64_t n, int bits,
                      const void* bias, void* y_host, sdq_dtype y_dtype, void* x_dev, void* y_dev,
                      int64_t chunk_rows, cudaStream_t st, const char* fn) {
    const size_t xe = x_dtype == SDQ_F32 ? 4 : 2, ye = y_dtype == SDQ_F32 ? 4 : 2;
    int64_t rows[kPipeChunks];
    const int nch = pipe_chunks(m, chunk_rows, rows);
    std::lock_guard<std::mutex> lock(g_pipe_mu);
    HostPipe* p = nullptr;
    cudaError_t e = pipe_for_current_device(&p);
    if (e != cudaSuccess) return fail(SDQ_ERR_CUDA, "%s: copy streams: %s", fn, cudaGetErrorString(e));
    if ((e = cudaEventRecord(p->start, st)) != cudaSuccess ||
        (e = cudaStreamWaitEvent(p->up, p->start, 0)) != cudaSuccess ||
        (e = cudaStreamWaitEvent(p->down, p->start, 0)) != cudaSuccess)
        return fail(SDQ_ERR_CUDA, "%s: stream fork: %s", fn, cudaGetErrorString(e));
    int rc = SDQ_OK;
    int64_t r0 = 0;
    for (int c = 0; c < nch && rc == SDQ_OK; r0 += rows[c], ++c) {
        const int64_t mc = rows[c];
        uint8_t* xd = static_cast<uint8_t*>(x_dev) + (size_t)r0 * k * xe;
        uint8_t* yd = static_cast<uint8_t*>(y_dev) + (size_t)r0 * n * ye;
        e = cudaMemcpyAsync(xd, static_cast<const uint8_t*>(x_host) + (size_t)r0 * k * xe,
                            (size_t)mc * k * xe, cudaMemcpyHostToDevice, p->up);
        if (e == cudaSuccess) e = cudaEventRecord(p->up_ev[c], p->up);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(st, p->up_ev[c], 0);
        if (e != cudaSuccess) { rc = fail(SDQ_ERR_CUDA, "%s: upload: %s", fn, cudaGetErrorString(e)); break; }
        rc = qmm_any_dtype(xd, x_dtype, mc, k, wq, scales, biases, sb_dtype, n, bits, bias, yd, y_dtype,
                           st, fn);
        if (rc != SDQ_OK) break;
        e = cudaEventRecord(p->mm_ev[c], st);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(p->down, p->mm_ev[c], 0);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(static_cast<uint8_t*>(y_host) + (size_t)r0 * n * ye, yd, (size_t)mc * n * ye,
                                cudaMemcpyDeviceToHost, p->down);
        if (e != cudaSuccess) rc = fail(SDQ_ERR_CUDA, "%s: download: %s", fn, cudaGetErrorString(e));
    }
    // Join the copy streams back into the caller's stream, also after a failure, so that
    // nothing the call enqueued outlives the caller's view of it.
    cudaError_t j = cudaEventRecord(p->done, p->down);
    if (j == cudaSuccess) j = cudaStreamWaitEvent(st, p->done, 0);
    if (j == cudaSuccess) j = cudaEventRecord(p->done, p->up);
    if (j == cudaSuccess) j = cudaStreamWaitEvent(st, p->done, 0);
    if (rc != SDQ_OK) return rc;
    if (j != cudaSuccess) return fail(SDQ_ERR_CUDA, "%s: stream join: %s", fn, cudaGetErrorString(j));
    return ok();
}
}  // namespace sdq

extern "C" {

const char* sdq_last_error(void) { return t_last_error.c_str(); }

int sdq_abi_version(void) { return SDQ_ABI_VERSION; }

size_t sdq_resident_bytes(int64_t n, int64_t k, int group_size, int bits, int sb_bytes) {
    if (group_size <= 0) group_size = 64;
    if (bits <= 0) bits = 4;
    if (n < 0 || k <= 0 || k % group_size != 0 || (32 % bits) != 0 || sb_bytes <= 0) return 0;
    const size_t packed = static_cast<size_t>(n) * static_cast<size_t>(k) * bits / 32 * 4;
    const size_t sb = static_cast<size_t>(n) * static_cast<size_t>(k / group_size) * 2 * sb_bytes;
    return packed + sb;
}

int sdq_quantize(const void* w, sdq_dtype w_dtype, int64_t n, int64_t k, int group_size, int bits,
                 const char* mode, uint32_t* wq, void* scales, void* biases, sdq_dtype sb_dtype,
                 void* stream) {
    const char* fn = "sdq_quantize";
    int rc;
    if ((rc = check_qparams(group_size, bits, mode, fn))) return rc;
    if ((rc = check_nk(n, k, fn))) return rc;
    if (!w || !wq || !scales || !biases)
        return fail(SDQ_ERR_INVALID, "%s: w, wq, scales and biases must be non-null", fn);
    if (w_dtype != SDQ_F32 && w_dtype != SDQ_BF16)
        return fail(SDQ_ERR_UNSUPPORTED, "%s: weights must be f32 or bf16 (dtype %d)", fn, (int)w_dtype);
    if (sb_dtype != SDQ_BF16 && sb_dtype != SDQ_F32)
        return fail(SDQ_ERR_UNSUPPORTED, "%s: scales/biases are stored bf16 or f32 (dtype %d)", fn,
                    (int)sb_dtype);
    const size_t se = sb_dtype == SDQ_F32 ? 4 : 2;
    if (!aligned(w, w_dtype == SDQ_F32 ? 8 : 4) || !aligned(wq, 4) || !aligned(scales, se) ||
        !aligned(biases, se))
        return fail(SDQ_ERR_INVALID, "%s: misaligned pointer (w needs %d bytes, wq 4, scales/biases %d)",
                    fn, w_dtype == SDQ_F32 ? 8 : 4, (int)se);
    if ((rc = check_device())) return rc;
    cudaError_t e = launch_quantize(w, w_dtype == SDQ_BF16, n, k, bits, wq, scales, biases,
                                    sb_dtype == SDQ_F32, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail("sdq_quantize: kernel launch", e);
    return ok();
}

int sdq_dequantize(const uint32_t* wq, const void* scales, const void* biases, sdq_dtype sb_dtype,
                   int64_t n, int64_t k, int group_size, int bits, const char* mode, void* out,
                   sdq_dtype out_dtype, void* stream) {
    const char* fn = "sdq_dequantize";
    int rc;
    if ((rc = check_qparams(group_size, bits, mode, fn))) return rc;
    if ((rc = check_nk(n, k, fn))) return rc;
    if (!wq || !scales || !biases || !out)
        return fail(SDQ_ERR_INVALID, "%s: wq, scales, biases and out must be non-null", fn);
    if (sb_dtype != SDQ_BF16 && sb_dtype != SDQ_F32)
        return fail(SDQ_ERR_UNSUPPORTED, "%s: scales/biases must be bf16 or f32", fn);
    if (out_dtype != SDQ_BF16 && out_dtype != SDQ_F32)
        return fail(SDQ_ERR_UNSUPPORTED, "%s: output must be bf16 or f32", fn);
    const size_t se = sb_dtype == SDQ_F32 ? 4 : 2;
    if (!aligned(wq, 4) || !aligned(out, 16) || !aligned(scales, se) || !aligned(biases, se))
        return fail(SDQ_ERR_INVALID, "%s: misaligned pointer (out needs 16 bytes)", fn);
    if ((rc = check_device())) return rc;
    cudaError_t e = launch_dequantize(wq, scales, biases, sb_dtype == SDQ_F32, n, k, bits, out,
                                      out_dtype == SDQ_F32, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail("sdq_dequantize: kernel launch", e);
    return ok();
}

int sdq_quantized_matmul(const void* x, sdq_dtype x_dtype, int64_t m, int64_t k, const uint32_t* wq,
                         const void* scales, const void* biases, sdq_dtype sb_dtype, int64_t n,
                         int transpose, int group_size, int bits, const char* mode, const void* bias,
                         void* y, sdq_dtype y_dtype, void* stream) {
    const char* fn = "sdq_quantized_matmul";
    int rc;
    if ((rc = sdq::validate_qmm(x, x_dtype, m, k, wq, scales, biases, sb_dtype, n, transpose,
                                group_size, bits, mode, bias, y, y_dtype, fn)))
        return rc;
    return qmm_any_dtype(x, x_dtype, m, k, wq, scales, biases, sb_dtype, n, bits, bias, y, y_dtype,
                         static_cast<cudaStream_t>(stream), fn);
}

int sdq_quantized_matmul_host(const void* x_host, sdq_dtype x_dtype, int64_t m, int64_t k,
                              const uint32_t* wq, const void* scales, const void* biases,
                              sdq_dtype sb_dtype, int64_t n, int group_size, int bits,
                              const void* bias, void* y_host, sdq_dtype y_dtype, void* x_dev,
                              void* y_dev, int64_t chunk_rows, void* stream) {
    const char* fn = "sdq_quantized_matmul_host";
    int rc;
    if (!x_host || !y_host) return fail(SDQ_ERR_INVALID, "%s: x_host and y_host must be non-null", fn);
    if ((rc = sdq::validate_qmm(x_dev, x_dtype, m, k, wq, scales, biases, sb_dtype, n, 1, group_size,
                                bits, "affine", bias, y_dev, y_dtype, fn)))
        return rc;
    if (chunk_rows < 0) return fail(SDQ_ERR_INVALID, "%s: chunk_rows must be >= 0 (0: automatic)", fn);
    for (const void* p : {x_host, static_cast<const void*>(y_host)}) {
        cudaPointerAttributes a{};
        cudaError_t e = cudaPointerGetAttributes(&a, p);
        if (e != cudaSuccess) return cuda_fail("sdq_quantized_matmul_host: cudaPointerGetAttributes", e);
        if (a.type == cudaMemoryTypeDevice)
            return fail(SDQ_ERR_INVALID,
                        "%s: x_host / y_host is device memory; call sdq_quantized_matmul instead", fn);
    }
    return qmm_host_pipeline(x_host, x_dtype, m, k, wq, scales, biases, sb_dtype, n, bits, bias, y_host,
                             y_dtype, x_dev, y_dev, chunk_rows, static_cast<cudaStream_t>(stream), fn);
}

int sdq_quantized_matmul_epilogue(const void* x, sdq_dtype x_dtype, int64_t m, int64_t k,
                                  const uint32_t* wq, const void* scales, const void* biases,
                                  sdq_dtype sb_dtype, int64_t n, int group_size, int bits,
                                  const void* bias, int act, const void* gate,
                                  const void* residual, void* y, sdq_dtype y_dtype,
                                  void* stream) {
    const char* fn = "sdq_quantized_matmul_epilogue";
    int rc;
    if (act != SDQ_ACT_NONE && act != SDQ_ACT_GELU_TANH && act != SDQ_ACT_SILU)
        return fail(SDQ_ERR_INVALID, "%s: act must be SDQ_ACT_NONE, _GELU_TANH or _SILU; got %d", fn, act);
    if ((gate && !aligned(gate, 2)) || (residual && !aligned(residual, 2)))
        return fail(SDQ_ERR_INVALID, "%s: misaligned gate or residual (bf16 needs 2 bytes)", fn);
    if (residual && residual != y && m > 0 && n > 0) {     // bad shapes: validate_qmm reports them
        // Partial overlap would let one tile read what another already wrote.
        const uintptr_t r0 = reinterpret_cast<uintptr_t>(residual), y0 = reinterpret_cast<uintptr_t>(y);
        const uintptr_t bytes = static_cast<uintptr_t>(m) * static_cast<uintptr_t>(n) * 2;
        if (r0 < y0 + bytes && y0 < r0 + bytes)
            return fail(SDQ_ERR_INVALID, "%s: residual overlaps y without being y", fn);
    }
    if ((rc = sdq::validate_qmm(x, x_dtype, m, k, wq, scales, biases, sb_dtype, n, 1, group_size,
                                bits, "affine", bias, y, y_dtype, fn)))
        return rc;
    if (x_dtype != SDQ_BF16 || y_dtype != SDQ_BF16 || sb_dtype != SDQ_BF16)
        return fail(SDQ_ERR_UNSUPPORTED, "%s: x, y, scales and biases must be bf16", fn);
    EpiArgs epi = bias_only(bias);
    epi.act = act;
    epi.gate = static_cast<const uint16_t*>(gate);
    epi.resid = static_cast<const uint16_t*>(residual);
    return run_qmm(x, m, k, wq, scales, biases, n, bits, epi, y, stream, fn);
}

size_t sdq_gguf_bytes(int ggml_type, int64_t elems) {
    int values = 0, bytes = 0;
    if (!sdq::gguf_block(ggml_type, values, bytes) || elems <= 0 || elems % values != 0) return 0;
    return static_cast<size_t>(elems / values) * static_cast<size_t>(bytes);
}

int sdq_gguf_quantize(const void* raw, int ggml_type, int64_t n, int64_t k, int group_size, int bits,
                      uint32_t* wq, void* scales, void* biases, sdq_dtype sb_dtype, void* stream) {
    const char* fn = "sdq_gguf_quantize";
    int rc;
    if ((rc = check_qparams(group_size, bits, "affine", fn))) return rc;
    if ((rc = check_nk(n, k, fn))) return rc;
    int values = 0, bytes = 0;
    if (!sdq::gguf_block(ggml_type, values, bytes))
        return fail(SDQ_ERR_UNSUPPORTED,
                    "%s: GGML type %d is not supported (F32, F16, BF16, Q4_0, Q8_0, Q4_K, Q5_K, Q6_K)", fn,
                    ggml_type);
    if (k % values != 0)
        return fail(SDQ_ERR_INVALID, "%s: rows of %lld values are not whole blocks of %d", fn, (long long)k,
                    values);
    if (!raw || !wq || !scales || !biases)
        return fail(SDQ_ERR_INVALID, "%s: raw, wq, scales and biases must be non-null", fn);
    if (sb_dtype != SDQ_BF16)
        return fail(SDQ_ERR_UNSUPPORTED, "%s: scales/biases are stored bf16 only (dtype %d)", fn, (int)sb_dtype);
    if (!aligned(raw, 4) || !aligned(wq, 4) || !aligned(scales, 2) || !aligned(biases, 2))
        return fail(SDQ_ERR_INVALID, "%s: misaligned pointer (raw and wq need 4 bytes)", fn);
    if ((rc = check_device())) return rc;
    cudaError_t e = launch_gguf_quantize(raw, ggml_type, n, k, bits, wq, scales, biases,
                                         static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail("sdq_gguf_quantize: kernel launch", e);
    return ok();
}

int sdq_gguf_dequantize(const void* raw, int ggml_type, int64_t count, void* out, sdq_dtype out_dtype,
                        void* stream) {
    const char* fn = "sdq_gguf_dequantize";
    int values = 0, bytes = 0;
    if (!sdq::gguf_block(ggml_type, values, bytes))
        return fail(SDQ_ERR_UNSUPPORTED,
                    "%s: GGML type %d is not supported (F32, F16, BF16, Q4_0, Q8_0, Q4_K, Q5_K, Q6_K)", fn,
                    ggml_type);
    if (count <= 0 || count % values != 0)
        return fail(SDQ_ERR_INVALID, "%s: %lld values are not a whole number of blocks of %d", fn,
                    (long long)count, values);
    if (!raw || !out) return fail(SDQ_ERR_INVALID, "%s: raw and out must be non-null", fn);
    if (out_dtype != SDQ_F32 && out_dtype != SDQ_BF16)
        return fail(SDQ_ERR_UNSUPPORTED, "%s: out must be f32 or bf16 (dtype %d)", fn, (int)out_dtype);
    if (!aligned(raw, 4) || !aligned(out, out_dtype == SDQ_F32 ? 4 : 2))
        return fail(SDQ_ERR_INVALID, "%s: misaligned pointer (raw needs 4 bytes)", fn);
    int rc;
    if ((rc = check_device())) return rc;
    cudaError_t e = launch_gguf_dequantize(raw, ggml_type, count, out, out_dtype == SDQ_F32,
                                           static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail("sdq_gguf_dequantize: kernel launch", e);
    return ok();
}

int sdq_seeded_normals(uint64_t seed, int64_t count, float* out, void* stream) {
    if (count < 0 || (count > 0 && !out))
        return fail(SDQ_ERR_INVALID, "sdq_seeded_normals: need count >= 0 and a non-null out");
    if (!aligned(out, 4)) return fail(SDQ_ERR_INVALID, "sdq_seeded_normals: misaligned out");
    if (count == 0) return ok();
    int rc;
    if ((rc = check_device())) return rc;
    cudaError_t e = launch_seeded_normals(seed, count, out, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail("sdq_seeded_normals: kernel launch", e);
    return ok();
}

int sdq_debug_wait_hook(uint64_t wait_limit_ns, int withhold_first_copy, void* stream) {
    if (wait_limit_ns != 0 && (wait_limit_ns < 1000000ull || wait_limit_ns > 2000000000ull))
        return fail(SDQ_ERR_INVALID, "sdq_debug_wait_hook: wait_limit_ns must be 0 or in [1 ms, 2 s], got %llu",
                    (unsigned long long)wait_limit_ns);
    int rc;
    if ((rc = check_device())) return rc;
    const unsigned long long lim = wait_limit_ns == 0 ? 2000000000ull : wait_limit_ns;
    const int wh = withhold_first_copy != 0;
    cudaError_t e = set_wait_hook_tc(lim, wh, static_cast<cudaStream_t>(stream));
    if (e == cudaSuccess) e = set_wait_hook_qmv(lim, wh, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail("sdq_debug_wait_hook", e);
    return ok();
}

int sdq_device_status(void* stream) {
    int rc;
    if ((rc = check_device())) return rc;
    unsigned int st = 0, sv = 0, ss = 0;
    cudaError_t e = read_and_clear_status(&st, static_cast<cudaStream_t>(stream));
    if (e == cudaSuccess) e = read_and_clear_qmv_status(&sv, static_cast<cudaStream_t>(stream));
    if (e == cudaSuccess) e = read_and_clear_shard_status(&ss, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail("sdq_device_status", e);
    if (st != 0 || sv != 0 || ss != 0) {
        return fail(SDQ_ERR_TIMEOUT,
                    "a device-side wait gave up (tensor-core kernel bits 0x%x: 1 producer, 2 MMA, "
                    "4 dequant, 8 epilogue; small-M kernel bits 0x%x: 1 producer, 2 activations, "
                    "4 weights; sharded exchange bits 0x%x: 1 a peer's pushes never landed); the "
                    "kernel returned early and its output is incomplete",
                    st, sv, ss);
    }
    return ok();
}

}  // extern "C"
