/* q38cuda_model.h - the device-resident model behind the upstream model API.
 *
 * The q38_model_* entry points have the names, signatures, argument meaning
 * and error behaviour of include/qwen38/qwen38_model.h (upstream), so the
 * upstream CLI and probes link against libq38cuda.so in place of
 * src/qwen38/qwen38_model.c and keep their loader, tokenizer and sampler:
 *
 *   Q38Model *q38_model_open_gguf     qwen38_model.h:12   (qwen38_model.c:1370-1414)
 *   q38_model_attach_mtp_gguf          qwen38_model.h:13   (qwen38_model.c:1416-1434)
 *   q38_model_close / q38_model_reset  qwen38_model.h:14-15
 *   q38_model_forward_token            qwen38_model.h:19-20 (qwen38_model.c:1494-1517)
 *   q38_model_prefill                  qwen38_model.h:24-25 (qwen38_model.c:1519-1560)
 *   q38_model_enable_mtp / _mtp_forward qwen38_model.h:29-31 (qwen38_model.c:1562-1612)
 *   q38_model_speculative_greedy       qwen38_model.h:37-42 (qwen38_model.c:1614-1714)
 *   q38_model_forward_token_layers     qwen38_model.h:46-47 (qwen38_model.c:1476-1492)
 *   q38_model_vocab_size / _position / _context_length  qwen38_model.h:49-51
 *
 * Differences a caller can see: the model lives on the CUDA device that is
 * current when q38_model_open_gguf is called; logits pointers are pinned host
 * buffers owned by the model (replaced by the next call, as upstream).
 * Failures return 0 / NULL, print a diagnostic on stderr as upstream does, and
 * leave the reason in q38cu_last_error().
 */
#ifndef Q38CUDA_MODEL_H
#define Q38CUDA_MODEL_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct Q38Model Q38Model;

Q38Model *q38_model_open_gguf(const char *path, uint32_t context_length);
int q38_model_attach_mtp_gguf(Q38Model *model, const char *path);
void q38_model_close(Q38Model *model);
void q38_model_reset(Q38Model *model);
int q38_model_forward_token(Q38Model *model, uint32_t token_id, const float **logits);
int q38_model_prefill(Q38Model *model, const uint32_t *tokens, uint32_t token_count, const float **logits);
int q38_model_enable_mtp(Q38Model *model);
int q38_model_mtp_forward(Q38Model *model, uint32_t token_id, const float **logits);
int q38_model_speculative_greedy(Q38Model *model, uint32_t token_id, uint32_t stop_token, uint32_t draft_count,
                                 uint32_t *accepted_tokens, uint32_t *accepted_count, const float **next_logits);
int q38_model_forward_token_layers(Q38Model *model, uint32_t token_id, uint32_t layer_count, float *hidden_out);
uint32_t q38_model_vocab_size(const Q38Model *model);
uint32_t q38_model_position(const Q38Model *model);
uint32_t q38_model_context_length(const Q38Model *model);

/* Greedy decoding without logits on the host (no upstream counterpart; the
 * upstream loop is q38_model_forward_token + q38_sampler argmax,
 * src/cli/qwen38_main.c:545-578).  Evaluates token_id at the current position,
 * then feeds each step's argmax back as the next input on the device, for
 * `count` steps; tokens_out[i] is the argmax of step i.  The position advances
 * by `count`; the last token is pending, as after the upstream loop. */
int q38cu_model_generate_greedy(Q38Model *model, uint32_t token_id, uint32_t count, uint32_t *tokens_out);

/* Tensor-parallel decode over 1, 2, 4 or 8 GPUs of one node (no upstream
 * counterpart: the upstream engine's only parallelism is OpenMP over output
 * rows, qwen38_model.c:724-739).  One process per GPU; each opens its shard
 * with the same path, context length, world size and communicator id (from
 * q38cu_nccl_unique_id on one rank, sent to the others by the caller), with
 * its own rank, on the CUDA device current at the call.  The returned model
 * takes every q38_model_* call above, which every rank must make in the same
 * order with the same arguments; all ranks compute identical logits and
 * tokens.  Column-parallel projections keep this shard's output rows (DeltaNet
 * key-head pairs with the value heads that read them, attention query heads
 * with their KV heads, a slice of the FFN and of the LM head); row-parallel
 * ones (ssm_out, attn_output, ffn_down) keep this shard's input superblocks
 * and their partial sums are added by an NCCL all-reduce; the LM head's rows
 * are gathered.  The MTP head and the tensor-core prefill are single-GPU only
 * (a tensor-parallel prefill runs the 8-token batch path).  The NCCL library
 * is loaded at run time (libnccl.so.2). */
typedef struct {
    uint32_t rank, world;
    uint32_t key_heads[16], n_key_heads;        /* DeltaNet key heads, local order */
    uint32_t value_blocks[24], n_value_blocks;  /* DeltaNet output blocks (value heads 2b, 2b + 1), local order */
    uint32_t attn_head0, attn_heads;            /* full-attention query heads */
    uint32_t kv_head0, kv_heads;                /* full-attention KV heads */
    uint32_t ffn0, ffn;                         /* FFN outputs [ffn0, ffn0 + ffn) */
    uint32_t vocab0, vocab;                     /* LM head rows */
} Q38CuTPShard;
/* What rank `rank` of `world` holds (host only).  1 = ok, 0 = bad arguments. */
int q38cu_tp_shard(uint32_t rank, uint32_t world, Q38CuTPShard *out);
/* 128 bytes of communicator id into id_out.  1 = ok. */
int q38cu_nccl_unique_id(void *id_out);
Q38Model *q38cu_model_open_tp(const char *path, uint32_t context_length, uint32_t rank, uint32_t world,
                              const void *nccl_id);

/* The cudaStream_t the model runs on (for event timing by a caller). */
void *q38cu_model_stream(Q38Model *model);

/* Number of kernels one decode step launches (the kernel nodes of the captured
 * decode graph; builds the graph if needed).  0 on failure. */
int q38cu_model_step_kernels(Q38Model *model);

/* Launch timeline of the decode step (profiling; no upstream counterpart, the
 * upstream's closest is its QWEN38_TRACE_LAYERS stderr trace).  Active only
 * when the environment has Q38CU_TRACE=1 at q38_model_open_gguf.  Each kernel
 * of the captured decode graph (and, into the same records, of the
 * speculative verification graphs) keeps one record of eleven %globaltimer stamps
 * in ns, each the earliest or latest over the kernel's CTAs: earliest start,
 * earliest return from the grid-dependency wait, latest end; for the
 * weight-streaming GEMVs also the latest CTA to finish staging its activation
 * and to finish decoding its weights, the latest start, the latest return from
 * the wait, the earliest to finish staging, and for an RMSNorm input the
 * earliest to know its sum of squares, to receive its first activation floats
 * and to finish quantizing in warp 0 (0 for other kernels, or ~0 when
 * unused).  Records accumulate over the replays since the last call.  Copies
 * up to max_records records (11 uint64 each, launch order) and clears them; returns the number
 * copied, 0 when tracing is off, -1 on error. */
int q38cu_model_trace(Q38Model *model, uint64_t *records, int max_records);

#ifdef __cplusplus
}
#endif

#endif
