// sdq_internal.h -- declarations shared between the kernel files and the C ABI.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace sdq {

// Streaming multiprocessors of the current device (cached per device).
int num_sms();

cudaError_t launch_quantize(const void* w, bool w_bf16, int64_t n, int64_t k, int bits,
                            uint32_t* wq, void* scales, void* biases, cudaStream_t st);
cudaError_t launch_dequantize(const uint32_t* wq, const void* scales, const void* biases,
                              int64_t n, int64_t k, int bits, void* out, bool out_f32,
                              cudaStream_t st);

// Quantised matmul on the tensor cores (TMA + tcgen05 / TMEM), every M.  Returns a CUDA error
// or cudaSuccess; `msg` receives a description when tensor-map encoding fails.
cudaError_t launch_qmm_tc(const void* x, int64_t m, int64_t k, const uint32_t* wq,
                          const void* scales, const void* biases, int64_t n, int bits,
                          const void* bias, void* y, cudaStream_t st, const char** msg);

// Device status word (see sdq_ptx.cuh).
cudaError_t read_and_clear_status(unsigned int* out, cudaStream_t st);

}  // namespace sdq
