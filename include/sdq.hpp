// sdq.hpp -- C++17 host mirror of the reference's `sd-tensor` quantised-weight
// interface over the libsdq C ABI (sdq.h).
//
// The reference's Rust surface (crates/sd-tensor/src/mlx.rs:1846-1986):
//
//   QuantizedArray::quantize(w: &Array, group_size, bits, &Stream) -> Result<Self>
//   QuantizedArray::dequantize(&self, &Stream) -> Result<Array>
//   QuantizedArray::matmul(&self, x: &Array, &Stream) -> Result<Array>
//   QuantizedArray::resident_bytes(&self) -> usize
//   pub weight, scales, biases, group_size, bits
//
// is mirrored here with the same names and argument meaning.  `Result<T>` is
// a value-or-error type; the error text is the library's per-thread message,
// prefixed with the operation as mlx.rs:448-470 does ("mlx: quantize: ...").
// Arrays own device memory (cudaMalloc / cudaFree, as MLX arrays own theirs
// and free on Drop, mlx.rs:1448-1451).  Calls are asynchronous on the stream;
// Stream::synchronize() (or Array::to_host_*) is the `eval` sync point.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <memory>
#include <string>
#include <utility>
#include <vector>

#include "sdq.h"

namespace sdq {

// ---------------------------------------------------------------- Result
struct Error {
    int code = SDQ_OK;
    std::string message;
};

template <class T>
class Result {
public:
    Result(T v) : ok_(true), v_(std::move(v)) {}
    Result(Error e) : ok_(false), e_(std::move(e)) {}
    bool is_ok() const { return ok_; }
    bool is_err() const { return !ok_; }
    T& value() { return v_; }
    const T& value() const { return v_; }
    const Error& error() const { return e_; }
    T unwrap() && { return std::move(v_); }

private:
    bool ok_;
    T v_{};
    Error e_;
};

inline Error error_from(int code, const char* what) {
    std::string msg = sdq_last_error();
    Error e;
    e.code = code;
    e.message = std::string("sdq: ") + what + (msg.empty() ? " failed with status " + std::to_string(code)
                                                           : ": " + msg);
    return e;
}

// ---------------------------------------------------------------- Stream
// A CUDA stream, passed per call like the reference's `Stream` (mlx.rs:478-510).
class Stream {
public:
    static Stream gpu() { return Stream(nullptr); }         // the legacy default stream
    explicit Stream(cudaStream_t s) : s_(s) {}
    cudaStream_t raw() const { return s_; }
    void synchronize() const { cudaStreamSynchronize(s_); }

private:
    cudaStream_t s_;
};

// ---------------------------------------------------------------- Array
// A contiguous device tensor (row-major) with an element type.
class Array {
public:
    Array() = default;
    static Result<Array> empty(std::vector<int64_t> shape, sdq_dtype dtype) {
        Array a;
        a.shape_ = std::move(shape);
        a.dtype_ = dtype;
        void* p = nullptr;
        const size_t bytes = a.nbytes();
        if (bytes) {
            cudaError_t e = cudaMalloc(&p, bytes);
            if (e != cudaSuccess) return Error{SDQ_ERR_CUDA, std::string("sdq: cudaMalloc: ") + cudaGetErrorString(e)};
        }
        a.buf_ = std::shared_ptr<void>(p, [](void* q) { if (q) cudaFree(q); });
        return a;
    }
    // f32 host data -> device array of `dtype` (f32 kept, bf16 rounded to nearest even).
    static Result<Array> from_slice_f32(const std::vector<float>& v, std::vector<int64_t> shape,
                                        sdq_dtype dtype = SDQ_F32) {
        auto r = empty(std::move(shape), dtype);
        if (r.is_err()) return r;
        Array a = std::move(r).unwrap();
        if ((int64_t)v.size() != a.elem_count()) return Error{SDQ_ERR_INVALID, "sdq: from_slice_f32: size mismatch"};
        cudaError_t e;
        if (dtype == SDQ_F32) {
            e = cudaMemcpy(a.data(), v.data(), v.size() * 4, cudaMemcpyHostToDevice);
        } else {
            std::vector<uint16_t> h(v.size());
            for (size_t i = 0; i < v.size(); ++i) h[i] = f32_to_bf16(v[i]);
            e = cudaMemcpy(a.data(), h.data(), h.size() * 2, cudaMemcpyHostToDevice);
        }
        if (e != cudaSuccess) return Error{SDQ_ERR_CUDA, std::string("sdq: cudaMemcpy: ") + cudaGetErrorString(e)};
        return a;
    }
    // Device -> host as f32 (waits for the array's producers on `s`, like to_vec_f32 + eval).
    Result<std::vector<float>> to_vec_f32(const Stream& s) const {
        s.synchronize();
        std::vector<float> out((size_t)elem_count());
        cudaError_t e;
        if (dtype_ == SDQ_F32) {
            e = cudaMemcpy(out.data(), data(), out.size() * 4, cudaMemcpyDeviceToHost);
        } else {
            std::vector<uint16_t> h(out.size());
            e = cudaMemcpy(h.data(), data(), h.size() * 2, cudaMemcpyDeviceToHost);
            for (size_t i = 0; i < h.size(); ++i) {
                uint32_t u = (uint32_t)h[i] << 16;
                std::memcpy(&out[i], &u, 4);
            }
        }
        if (e != cudaSuccess) return Error{SDQ_ERR_CUDA, std::string("sdq: cudaMemcpy: ") + cudaGetErrorString(e)};
        return out;
    }
    void* data() const { return buf_.get(); }
    const std::vector<int64_t>& shape() const { return shape_; }
    sdq_dtype dtype() const { return dtype_; }
    int64_t elem_count() const {
        int64_t n = 1;
        for (auto d : shape_) n *= d;
        return shape_.empty() ? 0 : n;
    }
    size_t elem_bytes() const { return dtype_ == SDQ_F32 ? 4 : (dtype_ == 100 ? 4 : 2); }
    size_t nbytes() const { return (size_t)elem_count() * elem_bytes(); }

    static uint16_t f32_to_bf16(float f) {
        uint32_t u;
        std::memcpy(&u, &f, 4);
        if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fff;
        u += 0x7fffu + ((u >> 16) & 1u);
        return (uint16_t)(u >> 16);
    }

private:
    std::shared_ptr<void> buf_;
    std::vector<int64_t> shape_;
    sdq_dtype dtype_ = SDQ_F32;
};

// u32 packed words are held as 4-byte elements; SDQ_F32 has the width we need.
constexpr sdq_dtype kPackedWords = SDQ_F32;

// ---------------------------------------------------------------- QuantizedArray
struct QuantizedArray {
    Array weight;  // packed u32 words, 32 / bits values each
    Array scales;
    Array biases;
    size_t group_size = 64;
    size_t bits = 4;

    // `[out, in]` in, packed `[out, in * bits / 32]` out (mlx.rs:1861-1911).  The scales and
    // biases take the weight's dtype, as MLX's do: f32 for the reference's f32 weights.
    static Result<QuantizedArray> quantize(const Array& w, size_t group_size, size_t bits,
                                           const Stream& s) {
        if (w.shape().size() != 2) return Error{SDQ_ERR_INVALID, "sdq: quantize: weight must be 2-D"};
        const int64_t n = w.shape()[0], k = w.shape()[1];
        if (bits == 0 || 32 % bits != 0 || group_size == 0 || k % (int64_t)group_size != 0) {
            int rc = sdq_quantize(w.data(), w.dtype(), n, k, (int)group_size, (int)bits, "affine",
                                  nullptr, nullptr, nullptr, SDQ_BF16, s.raw());
            return error_from(rc, "quantize");
        }
        auto wq = Array::empty({n, k * (int64_t)bits / 32}, kPackedWords);
        const sdq_dtype sbt = w.dtype() == SDQ_F32 ? SDQ_F32 : SDQ_BF16;
        auto sc = Array::empty({n, k / (int64_t)group_size}, sbt);
        auto bi = Array::empty({n, k / (int64_t)group_size}, sbt);
        if (wq.is_err()) return wq.error();
        if (sc.is_err()) return sc.error();
        if (bi.is_err()) return bi.error();
        QuantizedArray q{std::move(wq).unwrap(), std::move(sc).unwrap(), std::move(bi).unwrap(),
                         group_size, bits};
        int rc = sdq_quantize(w.data(), w.dtype(), n, k, (int)group_size, (int)bits, "affine",
                              static_cast<uint32_t*>(q.weight.data()), q.scales.data(), q.biases.data(),
                              sbt, s.raw());
        if (rc != SDQ_OK) return error_from(rc, "quantize");
        return q;
    }

    // Reconstruct the dense array in the scales' dtype, as MLX does (tests and dense-only
    // layers; mlx.rs:1913-1945).
    Result<Array> dequantize(const Stream& s) const {
        const int64_t n = weight.shape()[0], k = weight.shape()[1] * 32 / (int64_t)bits;
        auto out = Array::empty({n, k}, scales.dtype());
        if (out.is_err()) return out;
        Array o = std::move(out).unwrap();
        int rc = sdq_dequantize(static_cast<const uint32_t*>(weight.data()), scales.data(), biases.data(),
                                scales.dtype(), n, k, (int)group_size, (int)bits, "affine", o.data(), o.dtype(),
                                s.raw());
        if (rc != SDQ_OK) return error_from(rc, "dequantize");
        return o;
    }

    // x @ weight.T, dequantising inside the kernel (mlx.rs:1947-1975).  x is [.., in] bf16 or
    // f32; the result has x's dtype (f32 in, f32 out, as the reference's f32 activations get).
    Result<Array> matmul(const Array& x, const Stream& s, const Array* bias = nullptr) const {
        const int64_t k = x.shape().back();
        int64_t m = 1;
        for (size_t i = 0; i + 1 < x.shape().size(); ++i) m *= x.shape()[i];
        const int64_t n = weight.shape()[0];
        std::vector<int64_t> oshape(x.shape().begin(), x.shape().end() - 1);
        oshape.push_back(n);
        auto out = Array::empty(oshape, x.dtype());
        if (out.is_err()) return out;
        Array y = std::move(out).unwrap();
        int rc = sdq_quantized_matmul(x.data(), x.dtype(), m, k, static_cast<const uint32_t*>(weight.data()),
                                      scales.data(), biases.data(), scales.dtype(), n, 1, (int)group_size,
                                      (int)bits, "affine", bias ? bias->data() : nullptr, y.data(), y.dtype(),
                                      s.raw());
        if (rc != SDQ_OK) return error_from(rc, "quantized_matmul");
        return y;
    }

    // Packed words plus both scale tensors, counted at 4 bytes each whatever they are stored as
    // (mlx.rs:1981-1985).
    size_t resident_bytes() const {
        return (size_t)weight.elem_count() * 4 + (size_t)(scales.elem_count() + biases.elem_count()) * 4;
    }
};

}  // namespace sdq
