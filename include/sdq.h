/*
 * sdq.h -- C ABI of libsdq, a B200 (sm_100a) CUDA library for the affine
 * group-wise quantised linear of andreinknv/stable-diffusion.rs.
 *
 * This ABI replaces the three mlx-c entry points that the reference's
 * `sd-tensor` seam binds for `QuantizedArray` (crates/sd-tensor/src/mlx.rs:
 * 361-397) -- mlx_quantize, mlx_dequantize and mlx_quantized_matmul -- with
 * plain pointers and sizes.  Conventions mirror the reference's FFI:
 *
 *   - every entry point returns an int status, 0 = success (mlx.rs:448-470);
 *   - on failure the message is kept per thread and read with
 *     sdq_last_error() (the thread-local handler of mlx.rs:419-446);
 *   - no C++ exception crosses the boundary;
 *   - the library never frees caller memory; all tensors are caller-allocated
 *     DEVICE buffers (cudaMalloc'd or equivalent);
 *   - every call takes an explicit CUDA stream (`void*` = cudaStream_t, NULL =
 *     legacy default stream), mirroring the per-call mlx_stream, and is
 *     asynchronous on it.  The caller synchronises, as the reference's
 *     `eval` does (mlx.rs:1531-1544).
 *
 * There is no CPU fallback: a call on a machine without an sm_100 device
 * fails with SDQ_ERR_CUDA.
 *
 * Tensor layouts (row-major, contiguous):
 *   W   [n, k]                   dense weight, `[out, in]` (diffusers Linear)
 *   Wq  [n, k * bits / 32] u32   element k of a row in word k / (32/bits) at
 *                                bit offset bits * (k % (32/bits)) (little-end)
 *   S,B [n, k / group_size]      per-group scale and bias
 *   X   [m, k]                   activations
 *   Y   [m, n]                   Y = X . dequant(W)^T (+ bias[n])
 *
 * Supported today: group_size 64, bits 4 or 8, mode "affine", transpose true,
 * k % 64 == 0; W, S, B, X and Y bf16 or f32 in sdq_quantize, sdq_dequantize
 * and sdq_quantized_matmul (the reference's own tensors are f32), bf16 in the
 * fused-epilogue and sharded entry points.  Scales and biases hold bf16 values
 * either way (the quantiser rounds them to bf16 and widens them exactly when
 * stored as f32); f32 scales passed in are rounded to bf16.  Anything else is
 * rejected with SDQ_ERR_UNSUPPORTED or SDQ_ERR_INVALID and a message.
 */
#ifndef SDQ_H
#define SDQ_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SDQ_ABI_VERSION 1

/* Status codes. */
#define SDQ_OK 0
#define SDQ_ERR_INVALID 1     /* bad argument: null pointer, shape, alignment */
#define SDQ_ERR_UNSUPPORTED 2 /* valid in MLX but not provided here (bits 2/3/5/6, f16 ...) */
#define SDQ_ERR_CUDA 3        /* a CUDA runtime / driver call failed */
#define SDQ_ERR_TIMEOUT 4     /* a device-side wait exceeded its limit (kernel returned early) */
#define SDQ_ERR_NCCL 5        /* an NCCL call failed */

/* Element types (values fixed; they are part of the ABI). */
typedef enum sdq_dtype {
    SDQ_F32 = 0,
    SDQ_BF16 = 1,
    SDQ_F16 = 2
} sdq_dtype;

/* The last error message on this thread, or "" when the last call succeeded.
 * Replaces the error-handler trampoline of mlx.rs:432-446. */
const char* sdq_last_error(void);

/* ABI version (SDQ_ABI_VERSION) the library was built with. */
int sdq_abi_version(void);

/*
 * Quantise a dense weight.
 * Replaces mlx_quantize (mlx.rs:362-370) as called by QuantizedArray::quantize
 * (mlx.rs:1861-1911): w [n,k] (w_dtype) -> wq, scales, biases (sb_dtype).
 * group_size / bits <= 0 select the defaults 64 / 4, as an absent
 * mlx_optional_int does.  mode NULL means "affine".
 */
int sdq_quantize(const void* w, sdq_dtype w_dtype, int64_t n, int64_t k, int group_size,
                 int bits, const char* mode, uint32_t* wq, void* scales, void* biases,
                 sdq_dtype sb_dtype, void* stream);

/*
 * Reconstruct the dense weight: out[n,k] = s * q + b, rounded once to
 * out_dtype.  Replaces mlx_dequantize (mlx.rs:373-384) as called by
 * QuantizedArray::dequantize (mlx.rs:1918-1945).  For tests and for layers
 * without a quantised kernel; not the hot path.
 */
int sdq_dequantize(const uint32_t* wq, const void* scales, const void* biases,
                   sdq_dtype sb_dtype, int64_t n, int64_t k, int group_size, int bits,
                   const char* mode, void* out, sdq_dtype out_dtype, void* stream);

/*
 * y[m,n] = x[m,k] . dequant(wq, scales, biases)[n,k]^T (+ bias[n] when bias is
 * non-NULL), dequantising inside the kernel.  Replaces mlx_quantized_matmul
 * (mlx.rs:386-397) as called by QuantizedArray::matmul (mlx.rs:1952-1975) and,
 * with `bias`, the separate `y.add(bias)` of quantized::linear
 * (crates/sd-models/src/mlx/quantized.rs:314-317).  x, scales/biases and y
 * are each bf16 or f32 (bias has y's dtype).  f32 x or scales are rounded to
 * bf16 by a conversion pass on `stream` (stream-ordered scratch from the
 * device's default memory pool) before the product; an f32 y is the f32
 * accumulator plus bias, not rounded to bf16.  `transpose` must be true
 * (the reference always passes true).  m >= 1.  For m <= 8 a weight-stream
 * kernel (TMA ring of packed words, mma.sync on the raw codes, HBM-bound)
 * runs when k * bits / 8 is a multiple of 128; every other shape runs the
 * tcgen05 tensor-core kernel, whose token tile (16 .. 256 rows of x) follows
 * m and the SM count, and for m <= 16 keeps the activations resident in
 * shared memory while the packed weight streams from HBM.  x and wq must be
 * 16-byte aligned.
 */
int sdq_quantized_matmul(const void* x, sdq_dtype x_dtype, int64_t m, int64_t k,
                         const uint32_t* wq, const void* scales, const void* biases,
                         sdq_dtype sb_dtype, int64_t n, int transpose, int group_size, int bits,
                         const char* mode, const void* bias, void* y, sdq_dtype y_dtype,
                         void* stream);

/*
 * sdq_quantized_matmul with the activations and the result in HOST memory, as
 * the reference's callers hold them around QuantizedArray::matmul (mlx.rs:
 * 1952-1975, on MLX's unified memory): x_host [m,k] goes to the device
 * workspace x_dev, the product into the workspace y_dev, and y_dev back to
 * y_host [m,n].  The rows go in chunks of chunk_rows (0: automatic -- about
 * m/8 rows, 128 to 1024; at most 64 chunks) so that one chunk uploads while the
 * previous one's product runs and the one before downloads: the call costs
 * about the upload of x plus one chunk's product and download.  Page-locked
 * host memory (cudaHostAlloc / cudaHostRegister) lets the copies overlap;
 * pageable memory works, without the overlap.  Asynchronous on `stream` like
 * the other entry points: y_host is complete once `stream` has caught up.
 * x_dev holds m*k and y_dev m*n values of x_dtype / y_dtype; the other
 * arguments are sdq_quantized_matmul's (transpose true, mode "affine").
 */
int sdq_quantized_matmul_host(const void* x_host, sdq_dtype x_dtype, int64_t m, int64_t k,
                              const uint32_t* wq, const void* scales, const void* biases,
                              sdq_dtype sb_dtype, int64_t n, int group_size, int bits,
                              const void* bias, void* y_host, sdq_dtype y_dtype, void* x_dev,
                              void* y_dev, int64_t chunk_rows, void* stream);

/* Activations for sdq_quantized_matmul_epilogue (values fixed; part of the ABI). */
#define SDQ_ACT_NONE 0
#define SDQ_ACT_GELU_TANH 1 /* 0.5 a (1 + tanh(sqrt(2/pi) (a + 0.044715 a^3))), mlx.rs:1033-1052 */
#define SDQ_ACT_SILU 2      /* a * sigmoid(a), mlx.rs:697-705 */

/*
 * The quantised linear with its elementwise consumers fused into the output
 * stage:
 *
 *   y[t,f] = residual[t,f] + gate[f] * act(x[t,:] . dequant(w)[f,:] + bias[f])
 *
 * computed in f32 from the accumulator and rounded to bf16 once.  Every term
 * is optional: bias, gate and residual may be NULL (then 0, 1 and 0), act is
 * one of SDQ_ACT_*.  No single reference function does this; it replaces the
 * chains the reference's Flux model builds around a linear, each op a
 * separate pass over [m, n]:
 *   x.add(linear(a).mul(gate))   crates/sd-models/src/mlx/flux.rs:389-398,
 *                                408-414 and 470 (residual + gate, "m[2]" /
 *                                "m[5]" of the block's modulation)
 *   linear(a).gelu_approx()      flux.rs:400-407 (the MLP's first layer)
 *   linear(a).silu()             flux.rs:491-495 (the conditioning MLPs)
 * with the linear being quantized::linear (quantized.rs:298-318).
 * gate and bias are [n] bf16, residual [m, n] bf16 (row-major, contiguous).
 * residual may be y itself (in-place update of a residual stream) but must
 * not otherwise overlap y.  The other arguments and the dispatch (small-M
 * weight stream for m <= 8, tensor cores otherwise) are those of
 * sdq_quantized_matmul with transpose = 1 and mode "affine".
 */
int sdq_quantized_matmul_epilogue(const void* x, sdq_dtype x_dtype, int64_t m, int64_t k,
                                  const uint32_t* wq, const void* scales, const void* biases,
                                  sdq_dtype sb_dtype, int64_t n, int group_size, int bits,
                                  const void* bias, int act, const void* gate,
                                  const void* residual, void* y, sdq_dtype y_dtype,
                                  void* stream);

/*
 * Bytes a quantised [n,k] weight occupies, packed words plus scales and
 * biases, with sb_bytes per scale/bias element (the reference counts 4,
 * mlx.rs:1981-1985; this library stores bf16, 2).  Returns 0 on invalid
 * arguments.
 */
size_t sdq_resident_bytes(int64_t n, int64_t k, int group_size, int bits, int sb_bytes);

/* GGML block types of GGUF tensors (the file's type ids, crates/sd-tensor/src/mlx_gguf.rs:
 * 61-78): the set the reference's checkpoints use. */
#define SDQ_GGML_F32 0
#define SDQ_GGML_F16 1
#define SDQ_GGML_Q4_0 2
#define SDQ_GGML_Q8_0 8
#define SDQ_GGML_Q4_K 12
#define SDQ_GGML_Q5_K 13
#define SDQ_GGML_Q6_K 14
#define SDQ_GGML_BF16 30

/*
 * Bytes of GGUF data for `elems` values of block type ggml_type, or 0 when the type is
 * not one of SDQ_GGML_* or elems is not a whole number of blocks (mlx_gguf.rs:80-93,
 * 237-244).
 */
size_t sdq_gguf_bytes(int ggml_type, int64_t elems);

/*
 * Quantise a GGUF tensor's raw data (device memory, 4-byte aligned, sdq_gguf_bytes(type,
 * n*k) bytes; the tensor's row-major [n, k]) straight into wq / scales / biases, as
 * sdq_quantize would quantise its f32 dequantisation -- bit for bit -- without
 * materialising it.  Replaces, per tensor, the reference's Gguf::dequantize followed by
 * QuantizedArray::quantize in quantized::from_gguf (crates/sd-models/src/mlx/
 * quantized.rs:180-211; mlx_gguf.rs:235-435).  k must be a multiple of 64 and of the
 * type's block size; the other arguments are sdq_quantize's.
 */
int sdq_gguf_quantize(const void* raw, int ggml_type, int64_t n, int64_t k, int group_size, int bits,
                      uint32_t* wq, void* scales, void* biases, sdq_dtype sb_dtype, void* stream);

/*
 * Dequantise a GGUF tensor's raw data (device memory, as above) to `count` values of
 * out_dtype (SDQ_F32: the reference's f32 values exactly; SDQ_BF16: those rounded to
 * nearest even).  Replaces Gguf::dequantize (mlx_gguf.rs:235-283) for the tensors that stay
 * dense.
 */
int sdq_gguf_dequantize(const void* raw, int ggml_type, int64_t count, void* out, sdq_dtype out_dtype,
                        void* stream);

/*
 * `count` f32 standard normals of SeededRng::new(seed).normals(count) (crates/sd-tensor/src/
 * lib.rs:104-145: splitmix64, Box-Muller in f64, cos then sin), into device memory `out`:
 * the reference's documented draw for synthetic inputs.  Not on the quantised path; the
 * benchmark draws its inputs with it.
 */
int sdq_seeded_normals(uint64_t seed, int64_t count, float* out, void* stream);

/*
 * Read back and clear the device-side status word that the kernels set when a
 * bounded wait gives up.  Synchronises `stream`.  Returns SDQ_OK or
 * SDQ_ERR_TIMEOUT (with a message naming the wait).  No counterpart in the
 * reference (MLX kernels have no device-side waits).
 */
int sdq_device_status(void* stream);

/*
 * Testing hook for the bounded waits; not for production use.  wait_limit_ns
 * replaces the 2 s limit of every device-side wait of the matmul kernels (0
 * restores it; otherwise 1 ms .. 2 s).  With withhold_first_copy non-zero the
 * weight producer of every CTA of the tensor-core and small-M kernels skips its
 * first copy and the arrival that goes with it, so the consumers' wait on that
 * stage runs out: the kernel then records its status bit, lets the copies it
 * did start land, frees its tensor memory and returns, and sdq_device_status
 * reports SDQ_ERR_TIMEOUT.  Settings hold for the current device until changed.
 * Synchronises `stream`.  No counterpart in the reference.
 */
int sdq_debug_wait_hook(uint64_t wait_limit_ns, int withhold_first_copy, void* stream);

/*
 * Communicators for the column-sharded linear.  The library owns its NCCL
 * communicator, so no NCCL type crosses the ABI: rank 0 calls
 * sdq_comm_unique_id, shares the 128 bytes with the other ranks by any means
 * (a store, a file, MPI), then every rank calls sdq_comm_init on its own
 * device.  No counterpart in the reference (single-device; crates/sd-tensor
 * has no collectives).
 */
int sdq_comm_unique_id(uint8_t out_id[128]);
int sdq_comm_init(const uint8_t id[128], int world, int rank, void** comm_out);
int sdq_comm_destroy(void* comm);

/*
 * Column-sharded quantised linear: this rank holds rows
 * [rank*n_local, (rank+1)*n_local) of the weight (wq/scales/biases/bias_local
 * are the local shard).  It computes y_local[m, n_local] into
 * y_shards + rank*m*n_local, all-gathers in place over NVLink so that every
 * rank's y_shards holds [world, m, n_local], and, when y is non-NULL,
 * permutes that into y[m, world*n_local].  y_shards is caller-provided
 * (world*m*n_local elements, 16-byte aligned).  The compute step is
 * sdq_quantized_matmul; the exchange is one ncclAllGather on `stream`.
 * When y is non-NULL, 2 <= world <= 8, n_local % 8 == 0 and m > 8, the
 * exchange is instead fused into the compute: the tensor-core kernel writes
 * this rank's column block of the communicator's output buffer (see
 * sdq_comm_output) and stores each finished output tile at the same place of
 * every peer's buffer over NVLink; flag words in IPC-mapped memory, written and
 * waited on by stream memory operations, order the calls across ranks without
 * using an SM.  The assembled [m, world*n_local] is then copied to y, unless y
 * is that buffer.  y_shards is not written on this path.  Every rank must make
 * the same calls, in the same order; a rank that never makes its call leaves
 * the others' streams waiting, as an NCCL collective would.
 */
int sdq_quantized_matmul_sharded(const void* x, sdq_dtype x_dtype, int64_t m, int64_t k,
                                 const uint32_t* wq, const void* scales, const void* biases,
                                 sdq_dtype sb_dtype, int64_t n_local, int group_size, int bits,
                                 const void* bias_local, void* y_shards, void* y,
                                 sdq_dtype y_dtype, void* comm, void* stream);

/*
 * The communicator's output buffer: device memory of at least m*n bf16 values
 * on this rank, mapped into every peer (IPC), which the overlapped sharded call
 * assembles its [m, n] result in.  Passing it as that call's y leaves the
 * result there with no final copy.  Collective: every rank calls it with the
 * same m, n.  The pointer stays valid until a later call needs a larger buffer
 * (sdq_comm_output or a sharded call with a larger output, which reallocates)
 * or the communicator is destroyed; each sharded call overwrites its contents.
 * A sharded call whose y lies in the buffer but does not fit in it fails with
 * SDQ_ERR_INVALID.  No counterpart in the reference (single-device).
 */
int sdq_comm_output(void* comm, int64_t m, int64_t n, void** out);

/*
 * sdq_quantized_matmul_sharded without the caller's y_shards buffer, for callers
 * that cannot allocate device memory when they call it (an engine whose arena
 * owns all of HBM from start-up, a loop that may not stall on cudaFree).  The
 * [world, m, n_local] all-gather buffer is a static 8 MiB device array inside
 * the library, held on every GPU that loads it until the process exits, so
 * world*m*n_local must not exceed 4 Mi bf16 values (larger calls return
 * SDQ_ERR_INVALID naming the limit).  y must be non-NULL.  The call itself
 * allocates nothing; NCCL's buffers belong to the communicator.  The first call
 * on a device looks up the array's device address (cudaGetSymbolAddress); make
 * that first call before any stream capture.  The address is cached per device
 * together with the context's id and looked up again after a cudaDeviceReset.
 * The call must be made with the communicator's device current (otherwise
 * SDQ_ERR_INVALID): each GPU has its own copy of the array.  All calls share the array: each
 * call writes every element it reads, so nothing needs clearing, but calls whose
 * work overlaps on the GPU (other streams, other host threads) race on it.
 * No counterpart in the reference: its matmul allocates through MLX.
 */
int sdq_quantized_matmul_sharded_static(const void* x, sdq_dtype x_dtype, int64_t m, int64_t k,
                                        const uint32_t* wq, const void* scales, const void* biases,
                                        sdq_dtype sb_dtype, int64_t n_local, int group_size,
                                        int bits, const void* bias_local, void* y,
                                        sdq_dtype y_dtype, void* comm, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* SDQ_H */
