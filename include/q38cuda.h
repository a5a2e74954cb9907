/* q38cuda.h - C ABI of the B200 (sm_100a) quantized-kernel library.
 *
 * Drop-in device counterpart of the upstream engine's kernel API
 * (include/qwen38/qwen38_quant.h).  Every entry point takes plain pointers,
 * sizes and a CUDA stream passed as `void *` (a cudaStream_t; NULL = legacy
 * default stream), never a framework type.
 *
 * Conventions shared with the upstream API:
 *   - matrices use GGUF order: shape[0] is the input width K, shape[1] the
 *     number of output rows N (qwen38_quant.h:33);
 *   - GEMM outputs are batch-major, out[token * N + row] (qwen38_quant.h:44-46);
 *   - return 1 on success and 0 on bad arguments, shape or unsupported type
 *     (qwen38_quant.c:2837-2857).  The reason for a 0 is available from
 *     q38cu_last_error().
 * Differences forced by the device:
 *   - all buffers are device pointers owned by the caller;
 *   - calls are asynchronous on `stream`; a kernel that gives up a bounded
 *     wait records a code readable with q38cu_device_status();
 *   - tensor data must start on a 16-byte boundary and its allocation must
 *     extend to the next multiple of 16 bytes past nbytes (weights are moved
 *     with 16-byte bulk copies); q38cu_tensor_upload() guarantees both.
 */
#ifndef Q38CUDA_H
#define Q38CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define Q38CU_Q8_K_BLOCK_SIZE 256

/* Same layout as the upstream Q38Q8KBlock (qwen38_quant.h:14-18): 292 bytes. */
typedef struct {
    float scale;
    int8_t quants[Q38CU_Q8_K_BLOCK_SIZE];
    int16_t sums[Q38CU_Q8_K_BLOCK_SIZE / 16];
} Q38CuQ8KBlock;

/* Tensor data layouts on the device. */
#define Q38CU_LAYOUT_GGUF 0u   /* the GGUF bytes as in the file (row-major blocks) */
#define Q38CU_LAYOUT_TILED 1u  /* the same blocks regrouped for streaming: rows in tiles of
                                  tile_rows, block (r, b) at
                                  (((r / T) * nb + b) * T + r % T) * B with T = tile_rows,
                                  rows padded with zero blocks to whole tiles */

/* Device view of a GGUF tensor.  Mirrors the fields of the upstream
 * Q38GGUFTensor (qwen38_gguf.h:186-195) that the kernels read: `data` is the
 * device copy of the tensor's GGUF bytes, optionally in the streaming layout
 * (the upstream `iq1_s_repack` side view, qwen38_gguf.h:194, is the precedent
 * for a load-time repack hanging off the tensor).  Tensors in the tiled layout
 * carry `scratch`: per-tensor device memory for the partial sums of row tiles
 * that several CTAs share (zeroed counters at the start); calls that use the
 * same tensor concurrently on two streams race. */
typedef struct {
    uint32_t type;      /* GGML type id (GGUF value) */
    uint32_t n_dims;    /* 2 for matrices, 1 for vectors */
    uint64_t shape[2];  /* shape[0] = K (input width), shape[1] = N (rows) */
    uint64_t nbytes;    /* bytes of device data (padded rows included) */
    const void *data;   /* device pointer, 16-byte aligned */
    uint32_t layout;    /* Q38CU_LAYOUT_* */
    uint32_t tile_rows; /* tiled layout: rows per tile (a multiple of 8); else 0 */
    void *scratch;      /* tiled layout only: device scratch */
    uint64_t scratch_bytes;
} Q38CuTensor;

/* fp16 bits -> float (replaces q38_f16_to_f32, qwen38_quant.h:20). Host only. */
float q38cu_f16_to_f32(uint16_t value);

/* Quantize `length` fp32 values (a multiple of 256) into length/256 Q8_K
 * blocks, bit-exact with q38_quantize_q8_k (qwen38_quant.h:24-25,
 * qwen38_quant.c:50-88). */
int q38cu_quantize_q8_k(Q38CuQ8KBlock *output, const float *input, uint64_t length,
                        void *stream);

/* Integer GEMV against a Q8_K activation row (replaces q38_tensor_gemv_q8_k,
 * qwen38_quant.h:37-39). */
int q38cu_tensor_gemv_q8_k(float *output, const Q38CuQ8KBlock *input, uint64_t input_length,
                           const Q38CuTensor *tensor, void *stream);

/* Batch-major integer GEMM, output [batch][N] (replaces q38_tensor_gemm_q8_k,
 * qwen38_quant.h:47-49).  Each weight superblock is read from HBM once for
 * all batch_size tokens. */
int q38cu_tensor_gemm_q8_k(float *output, const Q38CuQ8KBlock *input, uint32_t batch_size,
                           uint64_t input_length, const Q38CuTensor *tensor, void *stream);

/* Parity probe: the same GEMM kernel additionally stores, for every
 * (token, row, superblock), the two integer sums the upstream code folds into
 * its float result: w = the scaled quant dot, x = the min term (Q2_K, Q4_K,
 * Q5_K) or the delta correction (IQ1_S, IQ1_M), else 0.  Arrays are
 * [batch][N][K/256].  IQ4_NL (float sums per 32 elements) is refused.  No upstream counterpart (the upstream kernels keep these
 * sums in registers); used to prove the sums bit-exact. */
int q38cu_tensor_gemm_q8_k_sums(float *output, int32_t *w_out, int32_t *x_out,
                                const Q38CuQ8KBlock *input, uint32_t batch_size,
                                uint64_t input_length, const Q38CuTensor *tensor, void *stream);

/* Float-activation GEMV/GEMM (replaces q38_tensor_gemv_f32 and
 * q38_tensor_gemm_f32, qwen38_quant.h:33-35, 44-46).  Types: F32, F16, BF16,
 * Q8_0 (the Q8_0 tensors of the Q4_K_M mix only take this path), Q2_K..Q6_K,
 * IQ4_NL. */
int q38cu_tensor_gemv_f32(float *output, const float *input, const Q38CuTensor *tensor,
                          void *stream);
int q38cu_tensor_gemm_f32(float *output, const float *input, uint32_t batch_size,
                          uint64_t input_length, const Q38CuTensor *tensor, void *stream);

/* Dequantize one row (replaces q38_tensor_row_f32, qwen38_quant.h:28-29);
 * bit-exact with the upstream basis-vector evaluation for finite weights. */
int q38cu_tensor_row_f32(float *output, const Q38CuTensor *tensor, uint64_t row, void *stream);

/* Dot product of one row with a float vector (replaces q38_tensor_dot_row_f32,
 * qwen38_quant.h:31-32): *output (device memory) = row . input (device, width
 * floats), the same value as that row of q38cu_tensor_gemv_f32.  As upstream,
 * returns 1 only when the result is finite: the call waits for the stream to
 * read it back (the one synchronizing entry of this header besides
 * q38cu_device_status). */
int q38cu_tensor_dot_row_f32(float *output, const float *input, const Q38CuTensor *tensor, uint64_t row,
                             void *stream);

/* Allocate device memory for a tensor (16-byte aligned, padded), copy
 * `host_data` (GGUF bytes, may be NULL to only allocate) into it in the given
 * layout and, for the tiled layout, choose its tile height for this device and
 * allocate its scratch.  The
 * library counterpart of binding an mmapped tensor (qwen38_gguf.h:186-195,
 * qwen38_model.c:1370-1406). */
int q38cu_tensor_upload(Q38CuTensor *tensor, uint32_t type, uint64_t width, uint64_t rows,
                        const void *host_data, uint32_t layout, void *stream);
/* Build a tiled copy (plus scratch) of a GGUF-layout device tensor
 * (counterpart of q38_prepare_iq1_s_repacks, qwen38_quant.h:53-56). */
int q38cu_tensor_repack(Q38CuTensor *dst, const Q38CuTensor *src, void *stream);
void q38cu_tensor_free(Q38CuTensor *tensor);

/* Bytes per GGUF block / elements per block (replaces q38_ggml_block_bytes and
 * q38_ggml_block_elements, qwen38_gguf.h:228-229). */
uint32_t q38cu_block_bytes(uint32_t type);
uint32_t q38cu_block_elements(uint32_t type);

/* GEMM over a tiled tensor that allocates no device memory.  No counterpart
 * in the upstream engine (its CPU kernels need no scratch).
 *
 * For callers that cannot call cudaMalloc: an engine that hands out device
 * memory only from a pre-planned arena (cudaMalloc/cudaFree synchronize the
 * whole device, which a serving loop cannot afford), or code handed a tiled
 * tensor whose weights were placed without the scratch buffer
 * q38cu_tensor_upload/q38cu_tensor_repack would allocate.  Same arguments,
 * result and bit-exactness as q38cu_tensor_gemm_q8_k for a tensor in the tiled
 * layout (tensor->scratch is ignored and may be NULL).
 *
 * Its scratch is one file-scope device array of Q38CU_NOALLOC_SCRATCH_BYTES,
 * which every GPU that loads the library holds until the process exits.  The
 * first call on a device looks up that array's device address (set-up, once
 * per device); make that first call before any stream capture (a first call
 * on a capturing stream is refused), and do not call it again after ending the
 * device's context (cudaDeviceReset) in the same process.  Shapes whose
 * scratch exceeds the maximum are rejected (return 0, reason in
 * q38cu_last_error).  All calls share the one array and each clears its tile
 * counters first, so calls whose kernels overlap on the GPU (two streams, or
 * two host threads on one device) race; serialize them. */
#define Q38CU_NOALLOC_SCRATCH_BYTES (16u << 20)
int q38cu_tensor_gemm_q8_k_noalloc(float *output, const Q38CuQ8KBlock *input, uint32_t batch_size,
                                   uint64_t input_length, const Q38CuTensor *tensor, void *stream);

/* Batch GEMM on the tensor cores, for prefill-sized batches (replaces
 * q38_tensor_gemm_q8_k, qwen38_quant.h:47-49, when M is large: the upstream
 * layer-major prefill calls it with M = prompt tokens, qwen38_model.c:1519-1560).
 * Same arguments and batch-major output [batch_size][N] as
 * q38cu_tensor_gemm_q8_k, for Q4_K and Q6_K tensors in either layout; the
 * weights and the Q8_K activations are dequantized to fp16 in `workspace`
 * (device memory, 256-byte aligned, at least
 * q38cu_tensor_gemm_q8_k_tc_workspace() bytes) and multiplied by tcgen05.mma
 * with fp32 accumulation.  Results agree with the integer path within 1e-3
 * relative (fp16 operand rounding); they are not bit-identical to it. */
uint64_t q38cu_tensor_gemm_q8_k_tc_workspace(uint32_t batch_size, uint64_t input_length, const Q38CuTensor *tensor);
int q38cu_tensor_gemm_q8_k_tc(float *output, const Q38CuQ8KBlock *input, uint32_t batch_size, uint64_t input_length,
                              const Q38CuTensor *tensor, void *workspace, uint64_t workspace_bytes, void *stream);

/* Diagnostics: the message behind the last 0 return on this host thread, and
 * the device status word (0 = ok, else a bounded wait gave up) which is read
 * after synchronizing `stream` and then cleared. */
const char *q38cu_last_error(void);
int q38cu_device_status(void *stream);

/* Host only, no device work: parses the GGUF file at `path` with the device
 * model's reader, which accepts what the upstream q38_gguf_open accepts
 * (src/io/qwen38_gguf.c:326-413: header, metadata, tensor table, every
 * tensor's bytes inside the file).  Returns the tensor count, or 0 with the
 * reason in q38cu_last_error() for a missing, truncated or corrupt file. */
uint64_t q38cu_gguf_check(const char *path);

/* Failure-path check (no upstream counterpart): launches one kernel whose
 * bounded mbarrier wait - the same wait every streaming kernel uses, with
 * limit_ns (1 .. 1e9) instead of the 2 s default - has nothing to wait for, so
 * it gives up, records the wait-timeout status (1) and returns; the context
 * stays usable.  q38cu_device_status then reports 1 once. */
int q38cu_debug_wait_probe(uint64_t limit_ns, void *stream);

#ifdef __cplusplus
}
#endif

#endif
