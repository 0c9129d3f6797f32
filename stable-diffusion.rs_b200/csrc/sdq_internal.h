// sdq_internal.h -- declarations shared between the kernel files and the C ABI.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include "../../include/sdq.h"

namespace sdq {

// Streaming multiprocessors of the current device (cached per device).
int num_sms();

// cuTensorMapEncodeTiled from the driver (nullptr when unavailable).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

// Peers one tensor-core kernel can store its output tiles to (one 8-GPU node).
constexpr int kTcMaxPeers = 7;

// Opt-in dynamic shared memory per block on sm_100 (227 KB).
constexpr size_t kQmvMaxSmem = 232448;

// The output stage of the matmul kernels: y = resid + gate[f] * act(acc + bias[f]),
// computed in f32 and rounded to bf16 once.  Null pointers drop their term; act is one
// of SDQ_ACT_*.  resid is [M, N] and may be y itself.
struct EpiArgs {
    const uint16_t* bias = nullptr;
    const uint16_t* gate = nullptr;
    const uint16_t* resid = nullptr;
    int act = SDQ_ACT_NONE;
    // The output y is f32 (written from the f32 accumulator, not rounded) and bias holds f32
    // values; only the plain output stage (bias alone) has this form.
    bool f32 = false;
    // Whether anything beyond the bias is asked for.
    bool fused() const { return gate != nullptr || resid != nullptr || act != SDQ_ACT_NONE; }
};
inline EpiArgs bias_only(const void* bias) {
    EpiArgs e;
    e.bias = static_cast<const uint16_t*>(bias);
    return e;
}

cudaError_t launch_quantize(const void* w, bool w_bf16, int64_t n, int64_t k, int bits,
                            uint32_t* wq, void* scales, void* biases, bool sb_f32, cudaStream_t st);
cudaError_t launch_dequantize(const uint32_t* wq, const void* scales, const void* biases, bool sb_f32,
                              int64_t n, int64_t k, int bits, void* out, bool out_f32,
                              cudaStream_t st);
// f32 -> bf16, round to nearest even (in 16-byte aligned when count >= 8, out 16-byte aligned).
cudaError_t launch_f32_to_bf16(const float* in, void* out, int64_t count, cudaStream_t st);

// Quantised matmul on the tensor cores (TMA + tcgen05 / TMEM), every M.  Returns a CUDA error
// or cudaSuccess; `msg` receives a description when tensor-map encoding fails.
cudaError_t launch_qmm_tc(const void* x, int64_t m, int64_t k, const uint32_t* wq,
                          const void* scales, const void* biases, int64_t n, int bits,
                          const EpiArgs& epi, void* y, cudaStream_t st, const char** msg);

// The unique id of the calling thread's current CUDA context (0 when the driver cannot say).
// A cudaDeviceReset replaces the context; caches of per-context objects compare this id.
unsigned long long current_context_id();

// The argument and device checks of sdq_quantized_matmul (status, message set on failure).
int validate_qmm(const void* x, sdq_dtype x_dtype, int64_t m, int64_t k, const uint32_t* wq,
                 const void* scales, const void* biases, sdq_dtype sb_dtype, int64_t n,
                 int transpose, int& group_size, int& bits, const char* mode, const void* bias,
                 const void* y, sdq_dtype y_dtype, const char* fn);

// The tensor-core matmul of the overlapped sharded linear: the same kernel, on at most
// grid_cap CTAs (0: every SM), writing rows ldy elements apart, whose epilogue also stores
// every output tile at the same place of each of the npeers (<= kTcMaxPeers) peers' copies
// (peers[i]: this rank's column block in peer i's output) and, once a CTA is done, adds 1
// to the word landed[i] in peer i's memory.  *grid_out receives the CTA count.
// qmm_tc_tile_tokens is the token-tile height the dispatcher picks for the shape.
int qmm_tc_tile_tokens(int64_t m, int64_t k, int64_t n, int bits, int grid_cap);
cudaError_t launch_qmm_tc_push(const void* x, int64_t m, int64_t k, const uint32_t* wq,
                               const void* scales, const void* biases, int64_t n, int bits,
                               const EpiArgs& epi, void* y, int64_t ldy, cudaStream_t st,
                               const char** msg, uint16_t* const* peers, uint32_t* const* landed,
                               int npeers, int grid_cap, int* grid_out);

// Small-M quantised matmul (1 <= M <= 8; TMA weight stream, register-fed m16n8k16 MMAs,
// programmatic dependent launch).  Sets *taken = false, launching nothing, for what it does
// not serve (M > 8, X too large to stay resident beside the weight ring, misaligned scales,
// f32 activations / scales / output); the caller then uses launch_qmm_tc.
cudaError_t launch_qmv(const void* x, bool x_f32, int64_t m, int64_t k, const uint32_t* wq,
                       const void* scales, const void* biases, bool sb_f32, int64_t n, int bits,
                       const EpiArgs& epi, void* y, bool y_f32, cudaStream_t st, const char** msg,
                       bool* taken);

// GGUF block types (sdq_gguf.cu): values and bytes per block (0 for an unknown type), and
// the fused dequantise-quantise / the dense dequantise kernels.
int gguf_block(int type, int& values, int& bytes);
cudaError_t launch_gguf_quantize(const void* raw, int type, int64_t n, int64_t k, int bits, uint32_t* wq,
                                 void* scales, void* biases, cudaStream_t st);
cudaError_t launch_gguf_dequantize(const void* raw, int type, int64_t count, void* out, bool out_f32,
                                   cudaStream_t st);

// SeededRng::normals (sdq_rng.cu).
cudaError_t launch_seeded_normals(uint64_t seed, int64_t count, float* out, cudaStream_t st);

// Device status words of the two matmul kernels (see sdq_ptx.cuh): read, then cleared.
cudaError_t read_and_clear_status(unsigned int* out, cudaStream_t st);
cudaError_t read_and_clear_qmv_status(unsigned int* out, cudaStream_t st);
// Status word of the sharded linear's landed-flag wait (sdq_shard.cu): read, then cleared.
cudaError_t read_and_clear_shard_status(unsigned int* out, cudaStream_t st);
// Testing hooks of the two matmul files (wait limit, withheld first copy); synchronise `st`.
cudaError_t set_wait_hook_tc(unsigned long long limit_ns, int withhold, cudaStream_t st);
cudaError_t set_wait_hook_qmv(unsigned long long limit_ns, int withhold, cudaStream_t st);

}  // namespace sdq
