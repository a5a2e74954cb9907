/* q38_oracle.h - CPU restatement of the upstream engine's quantized kernels.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA path:
 * only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
 * load it.  The product (libq38cuda.so) never links or calls it.
 *
 * Each function restates the scalar branch of the upstream C kernels in
 * src/qwen38/qwen38_quant.c (file:line cited per function in q38_oracle.c)
 * and additionally exposes the per-superblock integer sums that the upstream
 * code only folds into floats.  It is pinned against the upstream library
 * built from its own sources (oracle/Makefile -> oracle/_ref/) and against
 * committed golden vectors (tests/golden/).
 */
#ifndef Q38_ORACLE_H
#define Q38_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGML tensor type ids (GGUF on-disk values). */
enum {
    Q38O_F32 = 0, Q38O_F16 = 1, Q38O_Q8_0 = 8, Q38O_Q2_K = 10, Q38O_Q3_K = 11,
    Q38O_Q4_K = 12, Q38O_Q5_K = 13, Q38O_Q6_K = 14, Q38O_IQ2_XXS = 16,
    Q38O_IQ2_XS = 17, Q38O_IQ3_XXS = 18, Q38O_IQ1_S = 19, Q38O_IQ4_NL = 20,
    Q38O_IQ3_S = 21, Q38O_IQ2_S = 22, Q38O_IQ4_XS = 23, Q38O_IQ1_M = 29,
    Q38O_BF16 = 30
};

/* Same layout as the upstream Q38Q8KBlock (qwen38_quant.h:14-18): 292 bytes. */
typedef struct {
    float scale;
    int8_t quants[256];
    int16_t sums[16];
} Q38OQ8KBlock;

float q38o_f16_to_f32(uint16_t value);
uint32_t q38o_block_elements(uint32_t type);
uint32_t q38o_block_bytes(uint32_t type);
/* 1 when the type has an integer Q8_K kernel (upstream q38_matrix_type_q8_k). */
int q38o_type_q8_k(uint32_t type);

int q38o_quantize_q8_k(Q38OQ8KBlock *output, const float *input, uint64_t length);

/* Integer sums of one 256-element superblock against one Q8_K block.
 * w: the scaled integer dot; x: the second integer term (Q4_K/Q5_K/Q2_K min
 * term, IQ1_S/IQ1_M delta correction; 0 for other types). */
int q38o_block_sums(uint32_t type, const uint8_t *block, const Q38OQ8KBlock *act,
                    int32_t *w, int32_t *x);
/* The per-superblock float contribution, formed from (w, x) exactly as the
 * upstream scalar path forms it. */
float q38o_block_value(uint32_t type, const uint8_t *block, const Q38OQ8KBlock *act);

/* Batch-major GEMM over Q8_K activations, output [batch][rows]; batch 1 is
 * GEMV.  Per-block values are summed in block order (scalar upstream path). */
int q38o_gemm_q8_k(float *output, const Q38OQ8KBlock *input, uint32_t batch,
                   uint64_t width, uint32_t type, const uint8_t *data, uint64_t rows);
/* Per-superblock integer sums for every (token, row, block):
 * w_out/x_out are [batch][rows][width/256]. */
int q38o_gemm_q8_k_sums(int32_t *w_out, int32_t *x_out, const Q38OQ8KBlock *input,
                        uint32_t batch, uint64_t width, uint32_t type,
                        const uint8_t *data, uint64_t rows);

/* Float path: fp32 activations, sequential fmaf per row (upstream q38_dot_row). */
float q38o_dot_row_f32(uint32_t type, const uint8_t *row, const float *input, uint64_t width);
int q38o_gemm_f32(float *output, const float *input, uint32_t batch, uint64_t width,
                  uint32_t type, const uint8_t *data, uint64_t rows);
/* Dequantize one row (upstream q38_tensor_row_f32, basis-vector semantics). */
int q38o_row_f32(float *output, uint32_t type, const uint8_t *data, uint64_t width,
                 uint64_t rows, uint64_t row);

#ifdef __cplusplus
}
#endif

#endif
