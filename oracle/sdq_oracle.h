/*
 * sdq_oracle.h -- CPU restatement of the affine group-wise quantiser used by
 * andreinknv/stable-diffusion.rs, for tests and the CPU baseline only.
 *
 * This is test infrastructure.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference legs of bench.py may load it, and only as the
 * checker or the timed CPU baseline.  The product (libsdq.so) never calls it
 * and has no CPU fallback.
 *
 * What it restates (reference paths are inside the reference project):
 *   - crates/sd-tensor/src/mlx.rs:1828-1911  QuantizedArray::quantize, mode
 *     "affine": [out,in] -> packed [out, in*bits/32] u32 + scales + biases.
 *   - crates/sd-tensor/src/mlx.rs:1913-1945  QuantizedArray::dequantize.
 *   - crates/sd-tensor/src/mlx.rs:1947-1975  QuantizedArray::matmul,
 *     x @ dequant(w).T (transpose=true).
 *   - crates/sd-tensor/src/mlx.rs:1977-1985  resident_bytes.
 *   - crates/sd-models/src/mlx/quantized.rs:45-49, 168-174  group 64 and the
 *     K % 64 rule.
 *   - crates/sd-tensor/src/lib.rs:104-145  SeededRng (splitmix64 +
 *     Box-Muller), the reference's documented synthetic draw.
 *
 * The arithmetic itself lives in MLX / mlx-c (ml-explore/mlx), an external
 * system library that the reference links at build time
 * (crates/sd-tensor/build.rs:14-45) with NO pinned version (Cargo.lock has no
 * mlx entry; docs cite MLX 0.29.3 and 0.32).  MLX is absent here, so the rule
 * restated is the one the build's brief states -- scale = (max-min)/(2^bits-1),
 * bias = min, both stored bf16, little-end packing -- with every rounding
 * choice written down below.
 *
 * PARITY UNPINNED at the bit level against MLX itself: no reference test pins
 * packed words, scales or biases, and MLX cannot run in this container.  The
 * oracle IS pinned against every known-answer property the reference's own
 * tests hold for this path (crates/sd-models/tests/mlx_quantized.rs:53-228:
 * round-trip cosine, 8-bit better than 4-bit, qmm-vs-dense cosine, footprint
 * ratios, dense/quantised split), re-run in tests/test_oracle.py on the same
 * deterministic inputs.
 *
 * Rounding rules (the kernels follow the same IEEE-754 binary32 steps):
 *   per row n, group g of 64 consecutive k:
 *     mn, mx  = min / max of the 64 f32 values under a total order in which
 *               -0 < +0 and NaN is ignored (order-independent)
 *     scale   = (mx - mn) / (2^bits - 1)      binary32 sub then binary32 div
 *     s, b    = bf16_rne(scale), bf16_rne(mn)
 *     q       = 0 if s == 0, else clamp(rint((w - b) / s), 0, 2^bits - 1)
 *               (binary32 sub, binary32 div, round-half-even; NaN -> 0)
 *     dequant = bf16_rne(fmaf(s, q, b))  -- s*q is exact in binary32, so this
 *               is the correctly rounded bf16 of the exact s*q + b
 *   packing: element k of a row sits in word k / (32/bits) at bit offset
 *   bits * (k % (32/bits)).
 */
#ifndef SDQ_ORACLE_H
#define SDQ_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

uint16_t oracle_f32_to_bf16(float f);
float oracle_bf16_to_f32(uint16_t h);

/* W f32 [n,k] row-major -> wq u32 [n, k*bits/32], scales/biases bf16 [n, k/64].
 * Returns 0, or -1 on invalid arguments (bits not 4/8, k % 64 != 0). */
int oracle_quantize_f32(const float* w, int64_t n, int64_t k, int bits,
                        uint32_t* wq, uint16_t* scales, uint16_t* biases);
/* Same rule with bf16 weights (widened exactly to f32 first). */
int oracle_quantize_bf16(const uint16_t* w, int64_t n, int64_t k, int bits,
                         uint32_t* wq, uint16_t* scales, uint16_t* biases);

/* Reconstruct [n,k] as bf16 bits (bit-exact target for the kernels). */
int oracle_dequantize_bf16(const uint32_t* wq, const uint16_t* scales, const uint16_t* biases,
                           int64_t n, int64_t k, int bits, uint16_t* out);

/* y[m,n] = x_bf16[m,k] . dequant(w)[n,k]^T (+ bias_bf16[n] if non-null),
 * accumulated in f64 over the bf16 dequantised weights, rounded to f32.
 * threads <= 0 uses every OpenMP thread. */
int oracle_qmatmul(const uint16_t* x, int64_t m, int64_t k, const uint32_t* wq,
                   const uint16_t* scales, const uint16_t* biases, int64_t n, int bits,
                   const uint16_t* bias, float* y, int threads);

/* Bytes a quantised [n,k] weight occupies, counting 4 bytes per scale and per
 * bias as the reference does (mlx.rs:1981-1985). */
size_t oracle_resident_bytes(int64_t n, int64_t k, int group_size, int bits);

/* SeededRng (lib.rs:104-145): `count` standard normals from `seed`. */
void oracle_seeded_normals(uint64_t seed, int64_t count, float* out);

/* Threads OpenMP would use. */
int oracle_max_threads(void);

#ifdef __cplusplus
}
#endif
#endif
