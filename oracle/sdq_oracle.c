/*
 * sdq_oracle.c -- CPU restatement of the affine group-wise quantiser (test
 * infrastructure only; see sdq_oracle.h for scope, citations and the exact
 * rounding rules).  Compiled by oracle/Makefile with -O2 -fopenmp and
 * -ffp-contract=off so that no multiply-add is fused behind the source's back.
 */
#include "sdq_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define GROUP 64

uint16_t oracle_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fffu; /* canonical NaN */
    u += 0x7fffu + ((u >> 16) & 1u);                        /* round half to even */
    return (uint16_t)(u >> 16);
}

float oracle_bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* Total order for the group extrema: NaN ignored, -0 below +0.  The result
 * does not depend on the order the 64 values are visited in, which is what
 * lets a warp-tree reduction on the GPU agree with this sequential loop. */
static inline float qmin(float a, float b) {
    if (isnan(a)) return b;
    if (isnan(b)) return a;
    if (a < b) return a;
    if (b < a) return b;
    return signbit(a) ? a : b;
}
static inline float qmax(float a, float b) {
    if (isnan(a)) return b;
    if (isnan(b)) return a;
    if (a > b) return a;
    if (b > a) return b;
    return signbit(a) ? b : a;
}

/* One group of 64 widened values -> packed words, scale and bias bits. */
static void quantize_group(const float* v, int bits, uint32_t* words, uint16_t* s_out,
                           uint16_t* b_out) {
    float mn = INFINITY, mx = -INFINITY;
    for (int i = 0; i < GROUP; ++i) {
        mn = qmin(mn, v[i]);
        mx = qmax(mx, v[i]);
    }
    const unsigned qmax_i = (1u << bits) - 1u;
    const float range = mx - mn;
    const float scale = range / (float)qmax_i;
    const uint16_t sb = oracle_f32_to_bf16(scale);
    const uint16_t bb = oracle_f32_to_bf16(mn);
    const float s = oracle_bf16_to_f32(sb);
    const float b = oracle_bf16_to_f32(bb);
    const int per_word = 32 / bits;
    for (int w = 0; w < GROUP / per_word; ++w) words[w] = 0u;
    for (int i = 0; i < GROUP; ++i) {
        unsigned q = 0u;
        if (s != 0.0f) {
            const float t = (v[i] - b) / s;
            const float r = rintf(t);
            if (!(r > 0.0f)) q = 0u;                 /* also NaN */
            else if (r > (float)qmax_i) q = qmax_i;
            else q = (unsigned)r;
        }
        words[i / per_word] |= (uint32_t)q << (bits * (i % per_word));
    }
    *s_out = sb;
    *b_out = bb;
}

static int check_shape(int64_t n, int64_t k, int bits) {
    if (bits != 4 && bits != 8) return -1;
    if (n < 0 || k <= 0 || k % GROUP != 0) return -1;
    return 0;
}

int oracle_quantize_f32(const float* w, int64_t n, int64_t k, int bits, uint32_t* wq,
                        uint16_t* scales, uint16_t* biases) {
    if (check_shape(n, k, bits)) return -1;
    const int64_t groups = k / GROUP;
    const int64_t wpr = k * bits / 32; /* words per row */
    const int gw = GROUP * bits / 32;  /* words per group */
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < n; ++r) {
        for (int64_t g = 0; g < groups; ++g) {
            quantize_group(w + r * k + g * GROUP, bits, wq + r * wpr + g * gw,
                           scales + r * groups + g, biases + r * groups + g);
        }
    }
    return 0;
}

int oracle_quantize_bf16(const uint16_t* w, int64_t n, int64_t k, int bits, uint32_t* wq,
                         uint16_t* scales, uint16_t* biases) {
    if (check_shape(n, k, bits)) return -1;
    const int64_t groups = k / GROUP;
    const int64_t wpr = k * bits / 32;
    const int gw = GROUP * bits / 32;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < n; ++r) {
        float v[GROUP];
        for (int64_t g = 0; g < groups; ++g) {
            for (int i = 0; i < GROUP; ++i) v[i] = oracle_bf16_to_f32(w[r * k + g * GROUP + i]);
            quantize_group(v, bits, wq + r * wpr + g * gw, scales + r * groups + g,
                           biases + r * groups + g);
        }
    }
    return 0;
}

static inline float dequant_one(uint32_t word, int j, int bits, float s, float b) {
    const unsigned q = (word >> (bits * j)) & ((1u << bits) - 1u);
    return oracle_bf16_to_f32(oracle_f32_to_bf16(fmaf(s, (float)q, b)));
}

static void dequant_row_f32(const uint32_t* wq_row, const uint16_t* s_row, const uint16_t* b_row,
                            int64_t k, int bits, float* out) {
    const int per_word = 32 / bits;
    for (int64_t i = 0; i < k; ++i) {
        const int64_t g = i / GROUP;
        out[i] = dequant_one(wq_row[i / per_word], (int)(i % per_word), bits,
                             oracle_bf16_to_f32(s_row[g]), oracle_bf16_to_f32(b_row[g]));
    }
}

int oracle_dequantize_bf16(const uint32_t* wq, const uint16_t* scales, const uint16_t* biases,
                           int64_t n, int64_t k, int bits, uint16_t* out) {
    if (check_shape(n, k, bits)) return -1;
    const int64_t groups = k / GROUP;
    const int64_t wpr = k * bits / 32;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < n; ++r) {
        const int per_word = 32 / bits;
        for (int64_t i = 0; i < k; ++i) {
            const int64_t g = i / GROUP;
            const unsigned q = (wq[r * wpr + i / per_word] >> (bits * (i % per_word))) &
                               ((1u << bits) - 1u);
            const float s = oracle_bf16_to_f32(scales[r * groups + g]);
            const float b = oracle_bf16_to_f32(biases[r * groups + g]);
            out[r * k + i] = oracle_f32_to_bf16(fmaf(s, (float)q, b));
        }
    }
    return 0;
}

int oracle_qmatmul(const uint16_t* x, int64_t m, int64_t k, const uint32_t* wq,
                   const uint16_t* scales, const uint16_t* biases, int64_t n, int bits,
                   const uint16_t* bias, float* y, int threads) {
    if (check_shape(n, k, bits) || m < 0) return -1;
    const int64_t groups = k / GROUP;
    const int64_t wpr = k * bits / 32;
    enum { NB = 8 };
    const int64_t nblocks = (n + NB - 1) / NB;
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#else
    (void)threads;
#endif
    float* xf = (float*)malloc(sizeof(float) * (size_t)(m * k > 0 ? m * k : 1));
    if (!xf) return -1;
    for (int64_t i = 0; i < m * k; ++i) xf[i] = oracle_bf16_to_f32(x[i]);
#pragma omp parallel num_threads(threads)
    {
        float* wrows = (float*)malloc(sizeof(float) * (size_t)(NB * k));
#pragma omp for schedule(dynamic, 1)
        for (int64_t nb = 0; nb < nblocks; ++nb) {
            const int64_t n0 = nb * NB;
            const int rows = (int)((n - n0) < NB ? (n - n0) : NB);
            for (int r = 0; r < rows; ++r)
                dequant_row_f32(wq + (n0 + r) * wpr, scales + (n0 + r) * groups,
                                biases + (n0 + r) * groups, k, bits, wrows + (int64_t)r * k);
            for (int64_t i = 0; i < m; ++i) {
                const float* xr = xf + i * k;
                for (int r = 0; r < rows; ++r) {
                    const float* wr = wrows + (int64_t)r * k;
                    double acc = 0.0;
                    /* each product of two binary32 values is exact in binary64 */
                    for (int64_t kk = 0; kk < k; ++kk) acc += (double)xr[kk] * (double)wr[kk];
                    if (bias) acc += (double)oracle_bf16_to_f32(bias[n0 + r]);
                    y[i * n + n0 + r] = (float)acc;
                }
            }
        }
        free(wrows);
    }
    free(xf);
    return 0;
}

size_t oracle_resident_bytes(int64_t n, int64_t k, int group_size, int bits) {
    const size_t packed = (size_t)(n * k * bits / 32) * 4u;
    const size_t sb = (size_t)(n * (k / group_size)) * 2u * 4u;
    return packed + sb;
}

/* splitmix64 step and Box-Muller pair, in the order lib.rs:115-144 draws them:
 * u1 then u2, cos value first, sin value second, each narrowed to f32. */
static inline uint64_t splitmix64_next(uint64_t* state) {
    *state += 0x9E3779B97F4A7C15ull;
    uint64_t z = *state;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
static inline double next_open_unit(uint64_t* state) {
    const uint64_t bits = splitmix64_next(state) >> 11;
    return ((double)bits + 1.0) / (9007199254740992.0 + 1.0);
}

void oracle_seeded_normals(uint64_t seed, int64_t count, float* out) {
    uint64_t state = seed;
    const double tau = 6.283185307179586476925286766559;
    int64_t i = 0;
    while (i < count) {
        const double u1 = next_open_unit(&state);
        const double u2 = next_open_unit(&state);
        const double r = sqrt(-2.0 * log(u1));
        const double theta = tau * u2;
        out[i++] = (float)(r * cos(theta));
        if (i < count) out[i++] = (float)(r * sin(theta));
    }
}

int oracle_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
