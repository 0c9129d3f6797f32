// sdq_api.cu -- the C ABI (include/sdq.h): argument validation, per-thread
// error messages, and kernel selection.  No CPU fallback: without an sm_100
// device every compute entry point fails with SDQ_ERR_CUDA.
#include <cstdarg>
#include <cstdio>
#include <cstring>
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
    EpiArgs epi = bias_only(bias);
    epi.f32 = y_dtype == SDQ_F32;
    if (x_dtype == SDQ_BF16 && sb_dtype == SDQ_BF16)
        return run_qmm(x, m, k, wq, scales, biases, n, bits, epi, y, stream, fn);
    // f32 activations or scales: the tensor cores take bf16, so they are rounded (nearest
    // even) into stream-ordered temporaries first -- the one place the library allocates on
    // the compute path, through the stream's memory pool.  Scales and biases from
    // sdq_quantize are bf16 values already and stay exact.
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const size_t xb = x_dtype == SDQ_F32 ? ((size_t)m * k * 2 + 255) & ~(size_t)255 : 0;
    const size_t sbb = sb_dtype == SDQ_F32 ? ((size_t)n * (k / 64) * 2 + 255) & ~(size_t)255 : 0;
    uint8_t* tmp = nullptr;
    cudaError_t e = cudaMallocAsync(reinterpret_cast<void**>(&tmp), xb + 2 * sbb, st);
    if (e != cudaSuccess) return cuda_fail("sdq_quantized_matmul: cudaMallocAsync (f32 inputs)", e);
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
        return cuda_fail("sdq_quantized_matmul: f32 -> bf16 conversion", e);
    }
    rc = run_qmm(xk, m, k, wq, sk, bk, n, bits, epi, y, stream, fn);
    e = cudaFreeAsync(tmp, st);
    if (rc == SDQ_OK && e != cudaSuccess) return cuda_fail("sdq_quantized_matmul: cudaFreeAsync", e);
    return rc;
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
    unsigned int st = 0, sv = 0;
    cudaError_t e = read_and_clear_status(&st, static_cast<cudaStream_t>(stream));
    if (e == cudaSuccess) e = read_and_clear_qmv_status(&sv, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail("sdq_device_status", e);
    if (st != 0 || sv != 0) {
        return fail(SDQ_ERR_TIMEOUT,
                    "a device-side wait gave up (tensor-core kernel bits 0x%x: 1 producer, 2 MMA, "
                    "4 dequant, 8 epilogue; small-M kernel bits 0x%x: 1 producer, 2 activations, "
                    "4 weights); the kernel returned early and its output is incomplete",
                    st, sv);
    }
    return ok();
}

}  // extern "C"
