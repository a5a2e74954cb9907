// q38_model_internal.h - launch interfaces of the decode-step kernels
// (q38_model_kernels.cu) used by the device model (q38_model.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace q38 {

// Attention: the CTAs (one thread-block cluster) that share one (token, head),
// and the positions per CTA below which fewer of them take part.
constexpr int kAttnSplits = 8;
constexpr int kAttnSplitPositions = 64;
constexpr int kArgmaxCtas = 148;

// The device control block every captured step reads: ctl[0] = input token
// id, ctl[1] = position of the first token of the step, ctl[2] = number of
// tokens appended to the greedy history.
struct DeltaArgs {
    const float *qkvz;  // per token: q | k | v (10240), z at z_off (6144)
    int qkvz_ld, z_off;
    const float *beta, *alpha;  // raw projections, per token at stride ba_ld (ba_fused == 0)
    int ba_ld;
    // ba_fused: beta/alpha formed in the kernel from the Q8_0 rows ba_w
    // ([beta 48 rows | alpha 48 rows], GGUF layout) and RMSNorm(hidden, attn_norm)
    int ba_fused;
    const uint8_t *ba_w;
    const float *hidden, *attn_norm;  // [tokens][5120], [5120]
    // replicas: hidden is read from copy blockIdx % reps (hidden_rep_bytes
    // apart); out_q is written to all reps copies (q_rep_bytes apart)
    int reps;
    long long hidden_rep_bytes, q_rep_bytes;
    const float *conv_w;  // [10240][4]
    float *conv_ring;     // [10240][16]
    const float *dt, *a;  // [48]
    const float *norm_w;  // [128]
    float *state;         // [48][128][128], column-major per head
    // optional: the state after token t (t < tokens - 1) also goes to
    // snap + t * snap_stride (same layout), for speculative rollback
    float *snap;
    long long snap_stride;
    const int *ctl;
    int tokens;
    float *out_f;  // optional [tokens][6144]
    void *out_q;   // [tokens][24] Q8_K
    const void *pf_ptr;   // L2 prefetch of the next kernel's leading weights
    long long pf_bytes;
    unsigned long long *trace;  // optional launch timeline record (q38_device.cuh)
    // Head layout (0 = the whole model: 16 key heads, 24 output blocks).  A
    // tensor-parallel shard holds n_kh key heads and 3 n_kh value heads in
    // its own order (qkv rows q | k | v, the value heads of local output
    // block b being 2b and 2b + 1, key head = value head % n_kh), its output
    // rows n_kh * 384 floats and n_kh * 3 / 2 Q8_K blocks wide.
    int n_kh;
};

// A whole prefill chunk of one DeltaNet layer (deltanet_prefill_kernel): the
// same layer arguments as DeltaArgs, the chunk's first position `base`, any
// number of tokens, beta / alpha precomputed per token, and o_raw [tokens][o_ld]
// for the heads' outputs before their RMSNorm.
struct DeltaPrefillArgs {
    const float *qkvz;  // [tokens][qkvz_ld]: q | k | v, z at z_off
    int qkvz_ld, z_off;
    const float *beta, *alpha;  // [tokens][ba_ld]
    int ba_ld;
    const float *conv_w;  // [channels][4]
    float *conv_ring;     // [channels][16]
    const float *dt, *a;  // [value heads]
    const float *norm_w;  // [128]
    float *state;         // [value heads][128][128], column-major per head
    int base, tokens;
    float *o_raw;         // [tokens][o_ld]
    int o_ld;             // value heads * 128
    float *out_f;         // optional [tokens][o_ld]
    void *out_q;          // [tokens][o_ld / 256] Q8_K
    int n_kh;             // key heads (0: 16)
    float *rec;           // state-independent records of the chunk (16-byte aligned)
    int rec_tokens;       // token stride of `rec`: >= tokens, a multiple of 32
};

// Floats of the DeltaNet prefill records for `rec_tokens` tokens (key heads n_kh).
inline size_t delta_prefill_rec_floats(int n_kh, int rec_tokens)
{
    return static_cast<size_t>(rec_tokens) * (static_cast<size_t>(n_kh) * 260 + static_cast<size_t>(3 * n_kh) * 130);
}

struct AttnArgs {
    const float *qkv;  // per token: q|gate interleaved per head (12288), k at k_off, v at v_off
    int qkv_ld, k_off, v_off;
    const float *q_norm, *k_norm;  // [256]
    void *k_cache, *v_cache;       // this layer's [context][kv_ld], fp32 or (kv_half) fp16
    int kv_half;
    const int *ctl;
    float theta_scale;  // powf(1e7, -2 / 64), computed on the host as upstream
    int tokens;
    float *out_f;     // optional [tokens][6144]
    void *out_q;      // [tokens][24] Q8_K, written to all reps copies q_rep_bytes apart
    int reps;
    long long q_rep_bytes;
    const void *pf_ptr;   // L2 prefetch of the next kernel's leading weights
    long long pf_bytes;
    unsigned long long *trace;  // optional launch timeline record (q38_device.cuh)
    // Head layout (heads = 0: all 24 query heads, 4 KV heads).  A
    // tensor-parallel shard holds query heads head0 .. head0 + heads - 1
    // (rows h * 512 of qkv, local h) and KV heads kv0 .. (global KV head =
    // global query head / 6), its caches kv_ld floats per position and its
    // output heads * 256 floats (heads Q8_K blocks) per token.
    int heads, head0, kv0, kv_ld;
};

// The residual add after a row-parallel projection with the partial sums
// exchanged over NVLink (tensor parallelism without NCCL): every rank writes
// its partial [tokens][n] into slot `rank` of every rank's exchange buffer
// (peer pointers from CUDA IPC), raises per-CTA flags there, waits for the
// other ranks' flags and adds all slots in rank order into hidden (and its
// replicas).  Slots alternate between two halves by call parity; the call
// number comes from a device counter every rank advances identically.
struct TpReduceArgs {
    const float *partial;           // this rank's [tokens][n]
    float *hidden;                  // [tokens][n], reps copies rep_floats apart
    int reps;
    long long rep_floats;
    int n, tokens, rank, world;
    float *bufs[8];                 // every rank's exchange buffer: [2][world][8][n] floats
    unsigned long long *flags[8];   // every rank's flags: [world][kTpReduceCtas]
    unsigned long long *counter;    // [2]: the call number, and the CTAs done with this call
};
constexpr int kTpReduceCtas = 40;
cudaError_t launch_tp_reduce(const TpReduceArgs &args, cudaStream_t s);

// Full attention over a whole prefill chunk (launch_attention_prefill): the
// queries of tokens 0 .. tokens - 1 at positions base .. base + tokens - 1
// attend to the cached positions up to their own; this chunk's keys and
// values are written into the caches first.
struct AttnPrefillArgs {
    const float *qkv;  // [tokens][qkv_ld]: q|gate interleaved per head (512), k at k_off, v at v_off
    int qkv_ld, k_off, v_off;
    const float *q_norm, *k_norm;
    void *k_cache, *v_cache;  // this layer's [context][kv_ld], fp32 or (kv_half) fp16
    int kv_half;
    int kv_ld;                 // 256 * KV heads held
    int heads, head0, kv0;     // query heads held (global head0 ..), first KV head held
    float theta_scale;
    int base, tokens;
    float *qbuf;     // [tokens][heads][256]: the normed, rotated queries
    float *out_f;    // [tokens][out_ld]
    int out_ld;      // heads * 256
    void *out_q;     // [tokens][heads] Q8_K
};

struct ArgmaxArgs {
    const float *logits;
    int ld, n;
    float *part_v;  // [tokens][kArgmaxCtas]
    int *part_i;
    int *counters;  // [tokens], zero between launches
    uint32_t *out;  // [tokens]
    int *ctl;       // optional: fed with the last token's argmax
    int advance;    // added to ctl[1]
    uint32_t *history;
    int history_len;  // appends stop at this many tokens
    const void *pf_ptr;   // L2 prefetch of the next kernel's leading weights
    long long pf_bytes;
    unsigned long long *trace;  // optional launch timeline record (q38_device.cuh)
};

// RMSNorm of `tokens` rows of n floats, written as floats (out_f, optional)
// and as Q8_K blocks (out_q, optional; q_ld blocks per token, 0 = n / 256).
cudaError_t launch_rmsnorm_quant(const float *in, int in_ld, const float *weight, int n, int tokens, float *out_f,
                                 int out_ld, void *out_q, cudaStream_t s, int q_ld = 0);
cudaError_t launch_swiglu_quant(const float *gate, const float *up, int ld, int n, int tokens, float *out_f,
                                void *out_q, cudaStream_t s);
cudaError_t launch_add(float *out, const float *branch, int n, int tokens, cudaStream_t s);
// hidden[t][i] = hidden[t][i] + branch[t][i] in copy 0 and its reps - 1
// replicas (rep_floats apart): the residual add after a collective.
cudaError_t launch_add_replicated(float *hidden, const float *branch, int n, int tokens, int reps,
                                  long long rep_floats, cudaStream_t s);
cudaError_t launch_deltanet(const DeltaArgs &args, cudaStream_t s);
// The recurrence over the chunk, the head norm + gate + Q8_K, the conv ring.
cudaError_t launch_deltanet_prefill(const DeltaPrefillArgs &args, cudaStream_t s);
cudaError_t launch_attention(const AttnArgs &args, cudaStream_t s);
cudaError_t launch_attention_prefill(const AttnPrefillArgs &args, cudaStream_t s);
cudaError_t launch_argmax(const ArgmaxArgs &args, int tokens, cudaStream_t s);
cudaError_t read_and_clear_model_status(int *status);
// Sets `count` timeline records (q38_device.cuh) to their initial values.
cudaError_t launch_trace_reset(unsigned long long *records, int count, cudaStream_t s);
// Copies rows [0, bytes) of `base` to its replicas 1 .. reps - 1 (stride bytes apart).
cudaError_t launch_replicate(void *base, size_t bytes, int reps, long long stride, cudaStream_t s);

}  // namespace q38
