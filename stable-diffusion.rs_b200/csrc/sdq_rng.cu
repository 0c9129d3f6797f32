// sdq_rng.cu -- the reference's synthetic-input generator on the GPU.
//
// SeededRng (crates/sd-tensor/src/lib.rs:104-145) is splitmix64 feeding Box-Muller: draw j
// advances the state to seed + (j + 1) * 0x9E3779B97F4A7C15 and mixes it, two uniform draws in
// (0, 1] make one pair of normals (r cos t, r sin t) in f64, each rounded to f32.  Every draw
// depends only on its index, so one thread makes one pair.  The benchmark's inputs are drawn
// with it (X first, then W), as the reference documents for its synthetic data.
#include <cstdint>
#include <cuda_runtime.h>

#include "sdq_internal.h"

namespace sdq {
namespace {

__device__ __forceinline__ uint64_t splitmix64_at(uint64_t seed, uint64_t j) {
    uint64_t z = seed + (j + 1) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// Uniform in (0, 1]: 53 significant bits shifted off zero (lib.rs:121-126).
__device__ __forceinline__ double uniform_at(uint64_t seed, uint64_t j) {
    return ((double)(splitmix64_at(seed, j) >> 11) + 1.0) / (9007199254740992.0 + 1.0);
}

__global__ void seeded_normals_kernel(uint64_t seed, int64_t count, float* __restrict__ out) {
    const int64_t pairs = (count + 1) / 2;
    for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < pairs;
         p += (int64_t)gridDim.x * blockDim.x) {
        const double u1 = uniform_at(seed, 2 * (uint64_t)p), u2 = uniform_at(seed, 2 * (uint64_t)p + 1);
        const double r = sqrt(-2.0 * log(u1));
        const double t = 6.283185307179586 * u2;          // TAU
        double sn, cs;
        sincos(t, &sn, &cs);
        out[2 * p] = (float)(r * cs);
        if (2 * p + 1 < count) out[2 * p + 1] = (float)(r * sn);
    }
}

}  // namespace

cudaError_t launch_seeded_normals(uint64_t seed, int64_t count, float* out, cudaStream_t st) {
    const int64_t pairs = (count + 1) / 2;
    int64_t grid = (pairs + 255) / 256;
    const int64_t cap = (int64_t)num_sms() * 32;
    if (grid > cap) grid = cap;
    seeded_normals_kernel<<<(int)(grid > 0 ? grid : 1), 256, 0, st>>>(seed, count, out);
    return cudaGetLastError();
}

}  // namespace sdq
