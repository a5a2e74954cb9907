// q38_internal.h - host-side interfaces between the C ABI (q38_api.cu) and
// the kernel launchers (q38_kernels.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace q38 {

// How one weight-streaming GEMM launch walks a tensor.
struct GemmPlan {
    uint64_t row_bytes;   // GGUF bytes of one weight row
    int rows;             // N
    int nb;               // 256-element superblocks per row (K / 256)
    int rows_per_pass;    // rows decoded concurrently by one CTA (one superblock per thread)
    int rows_per_stage;   // rows moved per bulk copy (a multiple of rows_per_pass)
    int units;            // ceil(rows / rows_per_stage)
    int stages;           // bulk-copy pipeline depth
    uint32_t stage_bytes; // shared memory reserved per stage
    int threads;          // CTA size
    int max_ctas_per_sm;  // 0 = as many as fit
};

struct LaunchGemm {
    const void *weights;
    const void *act;
    int batch;
    float *out;
    int32_t *dbg_w;  // optional per-superblock integer sums
    int32_t *dbg_x;
};

// Tiled-layout streaming GEMM (q38_stream.cu).
struct StreamPlan {
    int rows, rows_pad, nb, block_bytes;
    int tile_rows, tiles, groups, chunk;
    int parts, group_threads;  // threads per (row, superblock); threads per group
    int mt, token_group;  // kernel token capacity / tokens handled per launch
    int stages;
    uint32_t stage_bytes;
    int threads, grid;
    long long units;
    int max_slots;
    uint64_t counter_bytes, scratch_bytes;
};

struct StreamLaunch {
    const void *weights;  // tiled-layout bytes
    const void *act;      // Q8_K blocks of this launch's tokens
    int tokens;
    float *out;           // rows of this launch's first token
    void *scratch;
    int32_t *dbg_w;
    int32_t *dbg_x;
    int out_ld = 0;       // output row stride between tokens (0: rows)
    int accumulate = 0;   // 1: add the result to the output rows
    // Activation prologue: kActQ8K reads Q8_K blocks from `act`; the fused
    // modes form them from floats inside the kernel (see q38_stream.cu).
    int act_mode = 0;
    const float *act_x = nullptr;  // RMSNorm: x rows; SwiGLU: gate rows ([tokens][act_ld])
    const float *act_y = nullptr;  // RMSNorm: norm weight; SwiGLU: up rows
    int act_ld = 0;
    float *act_f_out = nullptr;    // optional float copy of the activation [tokens][width]
    // Replicas (see q38_stream.cu): inputs read from copy blockIdx % act_reps,
    // outputs stored out_reps times; strides in bytes.
    int act_reps = 1;
    long long act_rep_bytes = 0, act_y_rep_bytes = 0;
    int out_reps = 1;
    long long out_rep_bytes = 0;
    // L2 prefetch, after the last bulk copy, of the first nx_cta_bytes of each
    // of the next GEMV's CTA ranges (see q38_stream.cu); null = none
    const void *nx_weights = nullptr;
    long long nx_units = 0;
    int nx_grid = 0;
    int nx_unit_bytes = 0;
    long long nx_cta_bytes = 0;
    // SwiGLU epilogue for interleaved (gate, up) rows in 256-row tiles (see
    // q38_stream.cu): floats to sw_act, Q8_K blocks to sw_q8 (sw_q_reps copies)
    float *sw_act = nullptr;
    void *sw_q8 = nullptr;
    int *sw_counters = nullptr;
    int sw_q_reps = 1;
    long long sw_q_rep_bytes = 0;
    unsigned long long *trace = nullptr;  // optional launch timeline record (q38_device.cuh)
    // RMSNorm input only: side_rows (<= grid) Q8_0 rows of width `width`
    // (GGUF layout) dotted with the normalized floats into
    // side_out[tok * side_ld + row] (see q38_stream.cu)
    const void *side_w = nullptr;
    int side_rows = 0, side_ld = 0;
    float *side_out = nullptr;
    // optional: the staged activation exported as Q8_K [tokens][width / 256],
    // export_reps copies export_rep_bytes apart (see q38_stream.cu)
    void *act_export = nullptr;
    int export_reps = 1;
    long long export_rep_bytes = 0;
    // Tensor-parallel exchange of a row-parallel projection's final rows over
    // peer memory, fused into the GEMV (see q38_stream.cu): xc_bufs[r] is rank
    // r's exchange buffer ([2][world][kXcTokens][xc_rows] 8-byte words, zero
    // at the start), mapped in this process; xc_counter is this rank's [2]
    // call counter (zero at the start).  The rows go to out (+= with
    // accumulate) once all ranks' partials are in.
    int xc_world = 0, xc_rank = 0, xc_rows = 0;
    unsigned long long *xc_bufs[8] = {};
    unsigned int *xc_counter = nullptr;
};

constexpr int kXcMaxWorld = 8, kXcTokens = 8;

enum : int { kActQ8K = 0, kActRmsNorm = 1, kActSwiGLU = 2 };

// RMSNorm of `tokens` rows -> Q8_K blocks (q_reps copies), optional floats
// and optional Q8_0 side rows, computed exactly as a stream GEMV's fused
// RMSNorm prologue with `warps` consumer warps computes them (see
// q38_stream.cu); a batch whose Q8_K input comes from here is bit-identical,
// row for row, to single-token launches with the fused prologue.
struct RmsPrologue {
    const float *x;       // [tokens][ld]
    int ld;
    const float *w;       // norm weight [width]
    int width, tokens, warps;
    void *out_q;          // [tokens][width / 256] Q8_K, q_reps copies q_rep_bytes apart
    int q_reps;
    long long q_rep_bytes;
    float *out_f;         // optional [tokens][f_ld]
    int f_ld;
    const void *side_w;   // optional Q8_0 rows [side_rows][width] (GGUF layout)
    int side_rows, side_ld;
    float *side_out;      // [tokens][side_ld]
};
cudaError_t launch_rms_prologue(const RmsPrologue &a, cudaStream_t s);
// Consumer warps of a stream GEMV launch of this shape and token count.
int stream_consumer_warps(const StreamPlan &p);

int stream_tile_rows(int rows);
cudaError_t stream_plan(int type, int rows, int width, int tile_rows, int tokens, StreamPlan *p);
cudaError_t launch_stream_gemm(int type, const StreamPlan &p, const StreamLaunch &l, cudaStream_t s);
cudaError_t launch_repack_tiled(void *dst, const void *src, uint64_t rows, uint64_t nb, uint32_t tile_rows,
                                uint32_t block_bytes, cudaStream_t s);
// q38cu_tensor_repack with a given tile height (a multiple of 8, 8..256).
int repack_tiled_with(void *dst_tensor, const void *src_tensor, uint32_t tile_rows, void *stream);

// Tensor-core batch GEMM (q38_tc.cu): out[t * ld + row] (+)= row_scale[row]
// sum_sb b_scale[sb][t] sum_{k in sb} A[row][k] B[t][k], A = A_hi + A_lo with
// A_hi fp16 [n][k] followed by A_lo [n][k], B fp16 [m][k] (K-major, k a
// multiple of 256, 16-byte aligned); sb = k / 256.
struct TcGemm {
    float *out;
    int ld;
    int n, m, k;
    const float *b_scale;  // [k / 256][b_scale_ld], b_scale_ld a multiple of tc_token_tile
    int b_scale_ld;
    const float *row_scale;
    int accumulate;
};
bool tc_weight_type(int type);
int tc_token_tile(int m);
// Quantized rows (tiled layout when tile_rows != 0) -> fp16 hi/lo [2][rows][width]
// scaled by 1 / row_scale[row] (a power of two per row, written here too);
// split: rows interleaved (gate i, up i) are written as [gate rows | up rows].
cudaError_t launch_dequant_f16(const void *w, int type, uint64_t rows, uint64_t width, uint32_t tile_rows, int bb,
                               void *out, float *row_scale, int split, cudaStream_t s);
// Q8_K [m][nb] -> the quants as fp16 [m][nb * 256] and the block scales
// b_scale[b][t] (t < ld, 0 past m; ld a multiple of tc_token_tile).
cudaError_t launch_q8k_to_f16(const void *q8, int nb, int m, int ld, void *out, float *b_scale, cudaStream_t s);
cudaError_t launch_tc_gemm(const void *a16, const void *b16, const TcGemm &p, cudaStream_t s);
cudaError_t read_and_clear_tc_status(int *status);

int device_sm_count();
// Message returned by q38cu_last_error() on this host thread.
void set_last_error(const char *message);
int superblock_bytes(int type);
size_t gemm_smem_for(int type, const GemmPlan &plan, int batch);
cudaError_t launch_q8k_gemm(int type, const GemmPlan &plan, const LaunchGemm &l, cudaStream_t s);
cudaError_t launch_quantize_q8k(void *out, const float *in, uint64_t blocks, cudaStream_t s);
// `tile_rows` != 0 selects the tiled layout for block addressing.
cudaError_t launch_f32_gemm(float *out, const float *x, int batch, uint64_t width, const void *w, uint64_t rows,
                            uint32_t tile_rows, int type, int be, int bb, cudaStream_t s);
// PDL launch with strides: out[tok * out_ld + row] (+)= row . x[tok * x_ld ..]
// One row's dot product with x (the f32 GEMV's arithmetic for that row).
cudaError_t launch_dot_row_f32(float *out, const float *x, const void *w, uint64_t width, uint32_t tile_rows,
                               uint64_t row, int type, int be, int bb, cudaStream_t s);
cudaError_t launch_f32_gemm_ex(float *out, uint64_t out_ld, int accumulate, const float *x, uint64_t x_ld, int batch,
                               uint64_t width, const void *w, uint64_t rows, uint32_t tile_rows, int type, int be,
                               int bb, cudaStream_t s);
cudaError_t launch_row_f32(float *out, const void *w, uint64_t width, uint32_t tile_rows, uint64_t row, int type,
                           int be, int bb, cudaStream_t s);
// Output row y (and its reps - 1 replicas, rep_floats apart) = row row_index[y].
cudaError_t launch_row_f32_indexed(float *out, const void *w, uint64_t width, uint32_t tile_rows, uint64_t rows,
                                   const uint32_t *row_index, int count, int type, int be, int bb, cudaStream_t s,
                                   int reps = 1, long long rep_floats = 0);
cudaError_t read_and_clear_status(int *status, cudaStream_t s);
// One bounded mbarrier wait that nothing completes, abandoned after limit_ns.
cudaError_t launch_wait_probe(unsigned long long limit_ns, cudaStream_t s);
cudaError_t read_and_clear_stream_status(int *status);

}  // namespace q38
