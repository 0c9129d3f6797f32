// The reference's quantised-weight tests (crates/sd-models/tests/mlx_quantized.rs:53-146),
// restated through the C++ host mirror include/sdq.hpp: the same deterministic inputs
// (weight() / activation(), mlx_quantized.rs:27-39), the same thresholds.  Exit status 0
// when every check holds; one line per check on stdout.
#include <cmath>
#include <cstdio>
#include <vector>

#include "sdq.hpp"

namespace {

std::vector<float> weight_values(size_t out, size_t inp) {
    std::vector<float> v(out * inp);
    for (size_t i = 0; i < v.size(); ++i) v[i] = (float(i % 97) - 48.0f) / 96.0f;
    return v;
}
std::vector<float> activation_values(size_t rows, size_t inp) {
    std::vector<float> v(rows * inp);
    for (size_t i = 0; i < v.size(); ++i) v[i] = (float(i % 31) - 15.0f) / 15.0f;
    return v;
}
double cosine(const std::vector<float>& a, const std::vector<float>& b) {
    double dot = 0, na = 0, nb = 0;
    for (size_t i = 0; i < a.size(); ++i) {
        dot += double(a[i]) * b[i];
        na += double(a[i]) * a[i];
        nb += double(b[i]) * b[i];
    }
    return dot / std::sqrt(na * nb);
}

int failures = 0;
void check(bool ok, const char* what, double value) {
    std::printf("%s %s %.6f\n", ok ? "ok  " : "FAIL", what, value);
    if (!ok) ++failures;
}

template <class T>
T must(sdq::Result<T> r, const char* what) {
    if (r.is_err()) {
        std::printf("FAIL %s: %s\n", what, r.error().message.c_str());
        std::exit(2);
    }
    return std::move(r).unwrap();
}

}  // namespace

int main() {
    const sdq::Stream s = sdq::Stream::gpu();
    {   // the round-trip cost is what the bit width says (mlx_quantized.rs:53-76)
        const auto dense = weight_values(256, 512);
        auto w = must(sdq::Array::from_slice_f32(dense, {256, 512}), "weight");
        double previous = 0;
        for (size_t bits : {4u, 8u}) {
            auto q = must(sdq::QuantizedArray::quantize(w, 64, bits, s), "quantize");
            auto back = must(q.dequantize(s), "dequantize");
            const double c = cosine(dense, must(back.to_vec_f32(s), "to_vec_f32"));
            check(back.shape() == w.shape() && c > 0.99 && c > previous,
                  bits == 4 ? "round trip 4-bit cosine" : "round trip 8-bit cosine", c);
            previous = c;
        }
    }
    {   // the quantised matmul agrees with the dense one (mlx_quantized.rs:85-120)
        const size_t out = 256, inp = 512, rows = 8;
        const auto wv = weight_values(out, inp);
        const auto xv = activation_values(rows, inp);
        std::vector<float> want(rows * out);
        for (size_t r = 0; r < rows; ++r)
            for (size_t o = 0; o < out; ++o) {
                double acc = 0;
                for (size_t i = 0; i < inp; ++i) acc += double(xv[r * inp + i]) * wv[o * inp + i];
                want[r * out + o] = float(acc);
            }
        auto w = must(sdq::Array::from_slice_f32(wv, {(int64_t)out, (int64_t)inp}), "weight");
        // f32 activations, f32 weights, f32 result: the reference's dtypes.
        auto x = must(sdq::Array::from_slice_f32(xv, {(int64_t)rows, (int64_t)inp}), "x");
        for (size_t bits : {4u, 8u}) {
            auto q = must(sdq::QuantizedArray::quantize(w, 64, bits, s), "quantize");
            auto y = must(q.matmul(x, s), "matmul");
            const double c = cosine(want, must(y.to_vec_f32(s), "to_vec_f32"));
            check(y.shape() == std::vector<int64_t>{(int64_t)rows, (int64_t)out} && y.dtype() == SDQ_F32 &&
                      q.scales.dtype() == SDQ_F32 && c > 0.999,
                  bits == 4 ? "matmul vs dense 4-bit cosine" : "matmul vs dense 8-bit cosine", c);
        }
    }
    {   // quantising shrinks the weight by what it claims (mlx_quantized.rs:123-146)
        const size_t out = 1024, inp = 1024;
        auto w = must(sdq::Array::from_slice_f32(weight_values(out, inp), {(int64_t)out, (int64_t)inp}), "weight");
        for (auto [bits, most] : {std::pair<size_t, double>{4, 0.20}, {8, 0.35}}) {
            auto q = must(sdq::QuantizedArray::quantize(w, 64, bits, s), "quantize");
            const double ratio = double(q.resident_bytes()) / double(out * inp * 4);
            check(ratio < most, bits == 4 ? "footprint 4-bit ratio" : "footprint 8-bit ratio", ratio);
        }
    }
    {   // errors carry the library's message (a width that is not a multiple of 64)
        auto w = must(sdq::Array::from_slice_f32(weight_values(4, 96), {4, 96}), "weight");
        auto r = sdq::QuantizedArray::quantize(w, 64, 4, s);
        const bool ok = r.is_err() && r.error().code == SDQ_ERR_INVALID &&
                        r.error().message.find("quantize") != std::string::npos;
        check(ok, "quantize rejects K % 64 != 0 with a message", ok ? 1.0 : 0.0);
    }
    std::printf("%d failure(s)\n", failures);
    return failures == 0 ? 0 : 1;
}
