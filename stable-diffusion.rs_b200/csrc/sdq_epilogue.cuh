// sdq_epilogue.cuh -- the elementwise output stage shared by the matmul kernels.
//
//   y = resid + gate * act(acc + bias)        (f32, rounded to bf16 once by the caller)
//
// The activations are the two the reference applies right after a linear:
//   gelu_approx  0.5 a (1 + tanh(sqrt(2/pi) (a + 0.044715 a^3)))
//                (crates/sd-tensor/src/mlx.rs:1033-1052)
//   silu         a * sigmoid(a) = a / (1 + e^-a)   (mlx.rs:697-705)
// The epilogue runs while the tile's accumulator is held, so its per-element cost delays
// the next tile's MMAs: tanh is the hardware approximation (PTX tanh.approx.f32, maximum
// relative error about 2^-11, below bf16's 2^-9 rounding step) and the sigmoid uses
// __expf and a fast divide.  The reference itself evaluates both chains op by op in bf16.
#pragma once

#include <cstdint>

#include "../../include/sdq.h"

namespace sdq {

__device__ __forceinline__ float tanh_approx(float x) {
    float y;
    asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float epi_activation(float a, int act) {
    if (act == SDQ_ACT_GELU_TANH) {
        const float c = 0.7978845608028654f;              // sqrt(2 / pi)
        const float h = 0.5f * a;
        return fmaf(h, tanh_approx(c * fmaf(0.044715f * a, a * a, a)), h);
    }
    if (act == SDQ_ACT_SILU) return __fdividef(a, 1.f + __expf(-a));
    return a;
}

}  // namespace sdq
