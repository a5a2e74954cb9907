// q38_model.cu - the device-resident Qwen3.8-27B model behind the upstream
// model API (include/qwen38/qwen38_model.h, implemented upstream in
// src/qwen38/qwen38_model.c).
//
// Weights, recurrent state, KV cache and activations live in HBM; a token step
// is one stream of kernels (weight-streaming GEMVs and the fused kernels of
// q38_model_kernels.cu) that reads the token id and the position from a small
// device control block, so the whole step is captured once as a CUDA graph
// and replayed for every token.  Greedy decoding feeds the argmax back into
// the control block on the device; no logits cross PCIe unless the caller
// asks for them.
//
// Projections that share an input are merged when their types allow it
// (attn_qkv | attn_gate, attn_q | attn_k, ffn_gate | ffn_up, ssm_beta |
// ssm_alpha): their rows are concatenated into one tiled tensor, so one launch
// streams them all.  Results are unchanged by the merge: every output row is
// computed by the same per-row arithmetic.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/q38cuda.h"
#include "../../include/q38cuda_model.h"
#include "q38_device.cuh"
#include "q38_gguf_file.h"
#include "q38_internal.h"
#include "q38_model_internal.h"

namespace {

constexpr int kHidden = 5120, kFfn = 17408, kLayers = 64, kTotalLayers = 65;
constexpr int kRecurrent = 48, kFull = 17;
constexpr int kLinQkv = 10240, kLinV = 6144, kLinHeads = 48, kLinDim = 128;
constexpr int kAttnQg = 12288, kAttnQ = 6144, kAttnKv = 1024, kAttnDim = 256;
constexpr int kVocab = 248320;
constexpr int kMaxTokens = 8;    // tokens per launch of the batch kernels
constexpr int kMaxDrafts = 64;   // speculative drafts per call
constexpr int kConvRing = 16;
// Copies of each freshly written activation (hidden rows, gate/up outputs, the
// mixers' Q8_K blocks) and of the RMSNorm weights: every GEMV CTA reads its
// input right after the previous kernel finishes, and 148 CTAs loading the
// same lines at once queue at the L2 slices that hold them; CTA c reads copy
// c % kReps instead.  The producers store all copies.
constexpr int kReps = 8;

enum : uint32_t { kF32 = 0, kF16 = 1, kQ8_0 = 8, kBF16 = 30 };

bool q8k_type(uint32_t t)  // upstream q38_matrix_type_q8_k (qwen38_model.c:172-182)
{
    return t == 10 || t == 11 || t == 12 || t == 13 || t == 14 || t == 16 || t == 17 || t == 18 || t == 20 ||
           t == 21 || t == 22 || t == 23 || t == 19 || t == 29;
}
bool float_type(uint32_t t) { return t == kF32 || t == kF16 || t == kBF16 || t == kQ8_0; }

int fail(const char *fmt, const std::string &detail = std::string())
{
    char buffer[512];
    std::snprintf(buffer, sizeof(buffer), fmt, detail.c_str());
    q38::set_last_error(buffer);
    std::fprintf(stderr, "qwen38: %s\n", buffer);
    return 0;
}

bool cuda_ok(cudaError_t e, const char *what)
{
    if (e == cudaSuccess) return true;
    fail("%s", std::string(what) + ": " + cudaGetErrorString(e));
    return false;
}

// One projection: one or more weight tensors whose output rows are placed
// side by side.  A part is either a tiled tensor on the Q8_K integer path or
// a GGUF-layout tensor on the float path (upstream q38_project,
// qwen38_model.c:599-606).
struct Part {
    Q38CuTensor t{};
    bool int_path = false;
    int rows = 0, offset = 0;
};

struct Proj {
    std::vector<Part> parts;
    int rows = 0, width = 0;
};

struct Layer {
    bool full = false;
    int index = 0;  // recurrent index (DeltaNet) or full-attention index
    float *attn_norm = nullptr, *post_norm = nullptr;
    Proj in_proj;  // DeltaNet: qkv | z     full: q | k | v
    Proj ba;       // DeltaNet: beta | alpha
    Proj out;      // ssm_out / attn_output
    Proj gate_up;  // ffn_gate | ffn_up (rows interleaved gate 0, up 0, gate 1, ... when swiglu_fused)
    bool swiglu_fused = false;  // gate_up's epilogue forms silu(gate) * up and its Q8_K blocks
    Proj down;
    float *conv_w = nullptr, *dt = nullptr, *a = nullptr, *ssm_norm = nullptr;
    float *q_norm = nullptr, *k_norm = nullptr;
};

template <typename T>
bool dalloc(T **p, size_t count, std::vector<void *> &owned)
{
    void *q = nullptr;
    if (!cuda_ok(cudaMalloc(&q, std::max<size_t>(count * sizeof(T), 16)), "cudaMalloc")) return false;
    owned.push_back(q);
    *p = static_cast<T *>(q);
    return cuda_ok(cudaMemset(q, 0, std::max<size_t>(count * sizeof(T), 16)), "cudaMemset");
}

// ---------------------------------------------------------------------------
// Tensor-parallel partition (world GPUs, 1, 2, 4 or 8).  Rank r holds:
//  * DeltaNet: the key-head pairs p = r, r + world, ... of the 8 pairs (key
//    heads 2p, 2p + 1) and the value heads that read them (value head v reads
//    key head v % 16, qwen38_model.c:764): value-head pairs (output Q8_K
//    blocks) p, p + 8, p + 16.  Local order: key heads 2i, 2i + 1 for the
//    i-th local pair; output block i + n j for pair i and j = 0, 1, 2, so a
//    local value head still reads local key head (value head % local key
//    heads) and every output block stays a whole Q8_K block;
//  * full attention: query heads [24 r / world, 24 (r + 1) / world) and the
//    KV heads they read (KV head = query head / 6, qwen38_model.c:851);
//  * FFN: the 256-wide blocks [68 r / world, 68 (r + 1) / world) of the 17408
//    outputs;
//  * LM head: rows [248320 r / world, 248320 (r + 1) / world).
// Column-parallel projections (qkv, z, beta, alpha, q, k, v, gate, up, LM
// head) keep their local output rows; row-parallel ones (ssm_out,
// attn_output, ffn_down) keep their local input superblocks, and their
// partial outputs are summed across the GPUs (one all-reduce of [tokens][5120]
// after each, two per layer).
struct Shard {
    int rank = 0, world = 1;
    std::vector<int> key_heads;     // local key head -> global
    std::vector<int> value_blocks;  // local output block -> global (value heads 2b, 2b + 1)
    int head0 = 0, heads = 24, kv0 = 0, kv_heads = 4;
    int ffn0 = 0, ffn = kFfn;
    int vocab0 = 0, vocab = kVocab;
    int n_kh() const { return static_cast<int>(key_heads.size()); }
    int n_vh() const { return 2 * static_cast<int>(value_blocks.size()); }
    int value_head(int local) const { return 2 * value_blocks[local / 2] + local % 2; }
};

bool make_shard(int rank, int world, Shard *out)
{
    if (world != 1 && world != 2 && world != 4 && world != 8) return false;
    if (rank < 0 || rank >= world) return false;
    Shard s;
    s.rank = rank;
    s.world = world;
    std::vector<int> pairs;
    for (int p = rank; p < 8; p += world) pairs.push_back(p);
    for (int p : pairs) {
        s.key_heads.push_back(2 * p);
        s.key_heads.push_back(2 * p + 1);
    }
    for (int j = 0; j < 3; ++j)
        for (int p : pairs) s.value_blocks.push_back(p + 8 * j);
    s.head0 = 24 * rank / world;
    s.heads = 24 * (rank + 1) / world - s.head0;
    s.kv0 = s.head0 / 6;
    s.kv_heads = (s.head0 + s.heads - 1) / 6 - s.kv0 + 1;
    const int b0 = (kFfn / 256) * rank / world, b1 = (kFfn / 256) * (rank + 1) / world;
    s.ffn0 = 256 * b0;
    s.ffn = 256 * (b1 - b0);
    s.vocab0 = static_cast<int>(static_cast<long long>(kVocab) * rank / world);
    s.vocab = static_cast<int>(static_cast<long long>(kVocab) * (rank + 1) / world) - s.vocab0;
    *out = s;
    return true;
}

// A (possibly partial) view of a GGUF tensor: the rows in `rows` and, in each
// row, the blocks in `cols` (half-open ranges; empty = all), gathered on the
// host in that order.
using Ranges = std::vector<std::pair<uint64_t, uint64_t>>;

struct View {
    const q38::GGUFTensorInfo *info = nullptr;
    uint32_t type = 0;
    uint64_t width = 0, rows = 0, nbytes = 0;
    const uint8_t *data = nullptr;
    std::vector<uint8_t> owned;
};

View full_view(const q38::GGUFTensorInfo *t)
{
    View v;
    v.info = t;
    v.type = t->type;
    v.width = t->shape[0];
    v.rows = t->n_dims > 1 ? t->shape[1] : 1;
    v.nbytes = t->nbytes;
    v.data = t->data;
    return v;
}

View gather_view(const q38::GGUFTensorInfo *t, const Ranges &rows, const Ranges &cols)
{
    if (rows.empty() && cols.empty()) return full_view(t);
    View v = full_view(t);
    const uint64_t be = q38::ggml_block_elements(t->type), bb = q38::ggml_block_bytes(t->type);
    const uint64_t all_rows = v.rows, row_bytes = t->nbytes / all_rows;
    Ranges rr = rows.empty() ? Ranges{{0, all_rows}} : rows;
    Ranges cc = cols.empty() ? Ranges{{0, t->shape[0] / be}} : cols;
    uint64_t n_rows = 0, n_blocks = 0;
    for (const auto &r : rr) n_rows += r.second - r.first;
    for (const auto &c : cc) n_blocks += c.second - c.first;
    v.owned.resize(n_rows * n_blocks * bb);
    uint8_t *dst = v.owned.data();
    for (const auto &r : rr)
        for (uint64_t row = r.first; row < r.second; ++row)
            for (const auto &c : cc) {
                const uint64_t n = (c.second - c.first) * bb;
                std::memcpy(dst, t->data + row * row_bytes + c.first * bb, n);
                dst += n;
            }
    v.rows = n_rows;
    v.width = n_blocks * be;
    v.nbytes = v.owned.size();
    v.data = v.owned.data();
    return v;
}

}  // namespace

struct Q38Model {
    q38::GGUFFile gguf, mtp_gguf;
    int device = 0;
    cudaStream_t stream = nullptr;
    uint32_t context_length = 0, position = 0, mtp_position = 0;
    bool mtp_loaded = false, mtp_enabled = false;
    float theta_scale = 0.0f;

    Q38CuTensor embedding{}, mtp_embedding{};  // GGUF layout, row lookups
    Proj output, mtp_output;                   // LM heads
    float *output_norm = nullptr;
    Layer layers[kTotalLayers];
    Proj eh_proj;
    float *enorm = nullptr, *hnorm = nullptr, *shared_head_norm = nullptr;

    // state
    float *conv_ring = nullptr, *delta_state = nullptr;
    uint8_t *k_cache = nullptr, *v_cache = nullptr;  // [17][context][kv_ld] of kv_bytes each
    int kv_bytes = 4;                                // 4: fp32 (the upstream's), 2: fp16 (Q38CU_KV_F16=1)
    float *ck_conv_ring = nullptr, *ck_delta_state = nullptr, *mtp_hidden = nullptr, *ck_mtp_hidden = nullptr;
    float *target_norm = nullptr;  // [kMaxDrafts][kHidden]: output-normed hidden of verified tokens
    uint32_t ck_position = 0, ck_mtp_position = 0;

    // activations, [kMaxTokens] rows each
    float *hidden = nullptr, *normf = nullptr, *wide = nullptr, *ba = nullptr, *act_f = nullptr, *logits = nullptr;
    void *q8 = nullptr;
    void *q8_norm = nullptr;  // batched launches: RMSNorm inputs as Q8_K (kReps copies)
    int wide_ld = 0, ba_ld = 0;
    int *ctl = nullptr;  // [0] token, [1] position, [2] history count
    uint32_t *ids = nullptr, *argmax_out = nullptr, *history = nullptr;
    float *argmax_part_v = nullptr;
    int *argmax_part_i = nullptr, *argmax_counters = nullptr;
    int *swiglu_counters = nullptr;  // one per Q8_K block of the FFN activation

    // host staging
    float *host_logits = nullptr;
    int *host_ctl = nullptr;
    uint32_t *host_ids = nullptr;

    cudaGraphExec_t decode_graph = nullptr;
    int step_kernels = 0;  // kernel nodes of the decode graph
    // Speculative decoding: one MTP draft step that feeds its argmax back
    // into the control block (replayed once per draft), and the target's
    // verification of n tokens with per-token DeltaNet state snapshots.
    cudaGraphExec_t mtp_draft_graph = nullptr;
    cudaGraphExec_t verify_graph[kMaxTokens + 1] = {};
    float *delta_snap = nullptr;  // [kMaxTokens - 1][48][48][128][128]
    bool snapping = false;        // set while a verification is captured
    // Launch timeline of the decode graph (Q38CU_TRACE=1 at open): one record
    // of q38::kTraceFields timestamps per traced kernel, in launch order.
    unsigned long long *trace = nullptr;
    int trace_cap = 0, trace_slots = 0;
    bool tracing = false;  // set while the decode step is captured
    std::vector<void *> owned;
    std::vector<Q38CuTensor> tensors;  // every uploaded tensor, freed at close
    void *staging = nullptr;
    size_t staging_bytes = 0;

    // Tensor-core prefill (prefill_tc): activations of up to pf_cap tokens,
    // the fp16 operands of one projection and per-sub-chunk control blocks.
    // Tensor parallelism (q38cu_model_open_tp): this process's shard and
    // the communicator of the GPUs that hold the others.
    Shard shard;
    ncclComm_t comm = nullptr;
    float *partial = nullptr;       // [kMaxTokens][kHidden]: a row-parallel projection's partial sums
    float *logits_local = nullptr;  // [kMaxTokens][shard.vocab]
    // How the row-parallel sums are added up across the GPUs:
    //   Q38CU_TP_P2P=0: NCCL's all-reduce, then a residual-add kernel;
    //   Q38CU_TP_P2P=1: tp_reduce_kernel over CUDA IPC buffers (NVLink);
    //   Q38CU_TP_P2P=2: inside the projection's own GEMV, tile by tile, over
    //                   the same buffers (the exchange fused with the GEMV).
    int tp_mode = 0;
    bool p2p = false;            // tp_mode 1
    bool xc = false;             // tp_mode 2
    uint8_t *ar_base = nullptr;  // this rank's [flags][exchange flags][exchange buffer]
    unsigned long long *ar_counter = nullptr;
    unsigned int *xc_counter = nullptr;
    float *ar_bufs[8] = {};
    unsigned long long *ar_flags[8] = {};
    std::vector<void *> ipc_opened;
    int kv_ld = kAttnKv;            // floats per position of this shard's KV cache rows
    int lin_qkv = kLinQkv, lin_heads = kLinHeads;  // this shard's DeltaNet channels and value heads

    int pf_cap = 0;
    float *pf_hidden = nullptr, *pf_normf = nullptr, *pf_wide = nullptr, *pf_act = nullptr, *pf_ba = nullptr;
    float *pf_scale = nullptr, *pf_row_scale = nullptr, *pf_oraw = nullptr, *pf_rec = nullptr;
    float *pf_part = nullptr;  // tensor parallel: a row-parallel projection's partial sums [cap][kHidden]
    void *pf_q8 = nullptr, *pf_q8mix = nullptr, *pf_a16 = nullptr, *pf_b16 = nullptr;
    uint32_t *pf_ids = nullptr, *host_pf_ids = nullptr;
    std::vector<void *> pf_owned;
};

namespace {

// ---------------------------------------------------------------------------
// loading
// ---------------------------------------------------------------------------
const q38::GGUFTensorInfo *find_layer(const q38::GGUFFile &f, int layer, const char *suffix)
{
    char name[128];
    std::snprintf(name, sizeof(name), "blk.%d.%s", layer, suffix);
    const q38::GGUFTensorInfo *t = f.find_tensor(name);
    if (!t) fail("missing tensor %s", name);
    return t;
}

// upstream q38_expect_tensor (qwen38_model.c:184-205)
bool expect(const q38::GGUFTensorInfo *t, uint64_t width, uint64_t rows, bool f32_only)
{
    if (!t) return false;
    const uint32_t dims = rows ? 2u : 1u;
    const bool shape_ok = t->n_dims == dims && t->shape[0] == width && (!rows || t->shape[1] == rows);
    const bool type_ok = f32_only ? t->type == kF32 : (float_type(t->type) || q8k_type(t->type));
    if (shape_ok && type_ok) return true;
    return fail("incompatible tensor %s", t->name);
}

bool ensure_staging(Q38Model *m, size_t bytes)
{
    if (m->staging_bytes >= bytes) return true;
    if (m->staging) cudaFree(m->staging);
    m->staging = nullptr;
    m->staging_bytes = 0;
    if (!cuda_ok(cudaMalloc(&m->staging, bytes), "cudaMalloc staging")) return false;
    m->staging_bytes = bytes;
    return true;
}

// Upload a group of tensors that share the input width.  Consecutive members
// of one type on the Q8_K integer path are concatenated into one tiled tensor;
// float-path members of one type into one GGUF-layout tensor.
// Tile height of a tiled projection, by shape (measured on the decode step):
// large projections (64 or more rows per SM) take whole warps per tile,
// rounded up (fewer, fuller CTAs: qkvz 16,384 rows -> 128); the 5120-row
// projections of the 6144-wide mixer output take 64 (80 CTAs: the next
// gate|up launch starts early on the SMs left free); the others the library's
// choice (ffn_down 40, attn_v 8).
uint32_t tile_rows_for(uint64_t rows, uint64_t width)
{
    const uint64_t sms = static_cast<uint64_t>(q38::device_sm_count());
    const uint64_t per_sm = (rows + sms - 1) / sms;
    if (per_sm >= 64) return static_cast<uint32_t>(std::min<uint64_t>(256, (per_sm + 31) / 32 * 32));
    if (rows == kHidden && width == kLinV) return 64;
    return 0;
}

bool upload_proj(Q38Model *m, Proj *p, const std::vector<View> &members)
{
    p->parts.clear();
    p->rows = 0;
    p->width = static_cast<int>(members[0].width);
    size_t i = 0;
    while (i < members.size()) {
        size_t j = i + 1;
        while (j < members.size() && members[j].type == members[i].type) ++j;
        const uint32_t type = members[i].type;
        const bool int_path = q8k_type(type);
        if (int_path && !q38::superblock_bytes(static_cast<int>(type)))
            return fail("tensor %s: this quantization type has no device kernel yet", members[i].info->name);
        uint64_t rows = 0, bytes = 0;
        for (size_t k = i; k < j; ++k) {
            rows += members[k].rows;
            bytes += members[k].nbytes;
        }
        if (!ensure_staging(m, bytes + 256)) return false;
        uint64_t at = 0;
        for (size_t k = i; k < j; ++k) {
            if (!cuda_ok(cudaMemcpy(static_cast<uint8_t *>(m->staging) + at, members[k].data, members[k].nbytes,
                                    cudaMemcpyHostToDevice),
                         "weight upload"))
                return false;
            at += members[k].nbytes;
        }
        Q38CuTensor src{};
        src.type = type;
        src.n_dims = 2;
        src.shape[0] = members[i].width;
        src.shape[1] = rows;
        src.nbytes = bytes;
        src.data = m->staging;
        src.layout = Q38CU_LAYOUT_GGUF;
        Part part;
        part.int_path = int_path;
        part.rows = static_cast<int>(rows);
        part.offset = p->rows;
        if (int_path) {
            const uint32_t tile = tile_rows_for(rows, src.shape[0]);
            const bool ok = tile ? q38::repack_tiled_with(&part.t, &src, tile, m->stream) != 0
                                 : q38cu_tensor_repack(&part.t, &src, m->stream) != 0;
            if (!ok) return fail("%s", q38cu_last_error());
        } else {
            void *dev = nullptr;
            if (!cuda_ok(cudaMalloc(&dev, bytes + 256), "cudaMalloc")) return false;
            if (!cuda_ok(cudaMemcpyAsync(dev, m->staging, bytes, cudaMemcpyDeviceToDevice, m->stream), "copy"))
                return false;
            part.t = src;
            part.t.data = dev;
        }
        if (!cuda_ok(cudaStreamSynchronize(m->stream), "upload")) return false;
        m->tensors.push_back(part.t);
        p->parts.push_back(part);
        p->rows += part.rows;
        i = j;
    }
    return true;
}

// A norm weight vector read by GEMV prologues: kReps copies, nbytes apart.
bool upload_norm(Q38Model *m, float **dst, const q38::GGUFTensorInfo *t)
{
    if (!dalloc(dst, t->nbytes / 4 * kReps, m->owned)) return false;
    for (int k = 0; k < kReps; ++k)
        if (!cuda_ok(cudaMemcpy(*dst + k * (t->nbytes / 4), t->data, t->nbytes, cudaMemcpyHostToDevice), "upload"))
            return false;
    return true;
}

// ffn_gate | ffn_up.  When both are one Q8_K integer-path type, their rows are
// interleaved (gate i, up i) and tiled 256 rows high, so each CTA's tile
// yields 128 SwiGLU outputs and the GEMV epilogue forms the FFN activation
// and its Q8_K blocks itself (q38_stream.cu); otherwise a plain projection.
bool upload_gate_up(Q38Model *m, Layer *L, const View &gate, const View &up)
{
    const uint64_t rows = gate.rows;
    // Fused only on one GPU: a shard's slice of the FFN has too few 256-row
    // tiles to occupy the GPU, so it streams as a plain projection in smaller
    // tiles and ffn_down forms SwiGLU in its prologue instead.
    const bool fusable = m->shard.world == 1 && gate.type == up.type && q8k_type(gate.type) &&
                         q38::superblock_bytes(static_cast<int>(gate.type)) && gate.width == up.width &&
                         rows == up.rows && (2 * rows) % 512 == 0 &&
                         static_cast<int>(2 * rows / 256) <= q38::device_sm_count();
    L->swiglu_fused = false;
    if (!fusable) {
        std::vector<View> members(2);
        members[0] = gate;
        members[1] = up;
        members[0].owned.clear();
        members[1].owned.clear();
        return upload_proj(m, &L->gate_up, members);
    }
    const uint64_t row_bytes = gate.nbytes / rows;
    if (!ensure_staging(m, 2 * gate.nbytes + 256)) return false;
    uint8_t *st = static_cast<uint8_t *>(m->staging);
    if (!cuda_ok(cudaMemcpy2D(st, 2 * row_bytes, gate.data, row_bytes, row_bytes, rows, cudaMemcpyHostToDevice),
                 "gate upload") ||
        !cuda_ok(cudaMemcpy2D(st + row_bytes, 2 * row_bytes, up.data, row_bytes, row_bytes, rows,
                              cudaMemcpyHostToDevice),
                 "up upload"))
        return false;
    Q38CuTensor src{};
    src.type = gate.type;
    src.n_dims = 2;
    src.shape[0] = gate.width;
    src.shape[1] = 2 * rows;
    src.nbytes = 2 * gate.nbytes;
    src.data = st;
    src.layout = Q38CU_LAYOUT_GGUF;
    Part part;
    part.int_path = true;
    part.rows = static_cast<int>(2 * rows);
    if (!q38::repack_tiled_with(&part.t, &src, 256, m->stream)) return fail("%s", q38cu_last_error());
    if (!cuda_ok(cudaStreamSynchronize(m->stream), "upload")) return false;
    m->tensors.push_back(part.t);
    L->gate_up.parts.clear();
    L->gate_up.parts.push_back(part);
    L->gate_up.rows = part.rows;
    L->gate_up.width = static_cast<int>(gate.width);
    L->swiglu_fused = true;
    return true;
}

bool upload_vec(Q38Model *m, float **dst, const View &v)
{
    if (!dalloc(dst, v.nbytes / 4, m->owned)) return false;
    return cuda_ok(cudaMemcpy(*dst, v.data, v.nbytes, cudaMemcpyHostToDevice), "vector upload");
}

bool upload_vec(Q38Model *m, float **dst, const q38::GGUFTensorInfo *t) { return upload_vec(m, dst, full_view(t)); }

std::vector<View> views(std::initializer_list<const q38::GGUFTensorInfo *> ts)
{
    std::vector<View> out;
    for (const auto *t : ts) out.push_back(full_view(t));
    return out;
}

// The rows of a DeltaNet layer's projections a shard keeps (qkv channels in
// local order q | k | v, then value rows for z, beta and alpha), see Shard.
Ranges qkv_rows(const Shard &sh)
{
    Ranges r;
    for (int kh : sh.key_heads) r.push_back({128ull * kh, 128ull * kh + 128});
    for (int kh : sh.key_heads) r.push_back({2048ull + 128 * kh, 2048ull + 128 * kh + 128});
    for (int v = 0; v < sh.n_vh(); ++v) r.push_back({4096ull + 128 * sh.value_head(v), 4096ull + 128 * sh.value_head(v) + 128});
    return r;
}

Ranges value_rows(const Shard &sh, uint64_t per_head)
{
    Ranges r;
    for (int v = 0; v < sh.n_vh(); ++v)
        r.push_back({per_head * sh.value_head(v), per_head * sh.value_head(v) + per_head});
    return r;
}

bool load_layer(Q38Model *m, const q38::GGUFFile &f, int l)
{
    Layer &L = m->layers[l];
    const Shard &sh = m->shard;
    const bool split = sh.world > 1 && l < kLayers;  // the MTP layer is never split
    L.full = (l + 1) % 4 == 0 || l == kLayers;
    L.index = L.full ? l / 4 : l - (l + 1) / 4;
    auto T = [&](const char *s) { return find_layer(f, l, s); };
    const auto *attn_norm = T("attn_norm.weight"), *post_norm = T("post_attention_norm.weight");
    const auto *gate = T("ffn_gate.weight"), *up = T("ffn_up.weight"), *down = T("ffn_down.weight");
    bool ok = expect(attn_norm, kHidden, 0, true) && expect(post_norm, kHidden, 0, true) &&
              expect(gate, kHidden, kFfn, false) && expect(up, kHidden, kFfn, false) &&
              expect(down, kFfn, kHidden, false);
    if (!ok) return false;
    const Ranges none;
    if (L.full) {
        const auto *q = T("attn_q.weight"), *k = T("attn_k.weight"), *v = T("attn_v.weight");
        const auto *o = T("attn_output.weight"), *qn = T("attn_q_norm.weight"), *kn = T("attn_k_norm.weight");
        ok = expect(q, kHidden, kAttnQg, false) && expect(k, kHidden, kAttnKv, false) &&
             expect(v, kHidden, kAttnKv, false) && expect(o, kAttnQ, kHidden, false) &&
             expect(qn, kAttnDim, 0, true) && expect(kn, kAttnDim, 0, true);
        if (!ok) return false;
        std::vector<View> in;
        std::vector<View> out;
        if (split) {
            const Ranges qr{{512ull * sh.head0, 512ull * (sh.head0 + sh.heads)}};
            const Ranges kvr{{256ull * sh.kv0, 256ull * (sh.kv0 + sh.kv_heads)}};
            in.push_back(gather_view(q, qr, none));
            in.push_back(gather_view(k, kvr, none));
            in.push_back(gather_view(v, kvr, none));
            out.push_back(gather_view(o, none, Ranges{{static_cast<uint64_t>(sh.head0),
                                                      static_cast<uint64_t>(sh.head0 + sh.heads)}}));
        } else {
            in = views({q, k, v});
            out = views({o});
        }
        if (!upload_proj(m, &L.in_proj, in) || !upload_proj(m, &L.out, out) || !upload_vec(m, &L.q_norm, qn) ||
            !upload_vec(m, &L.k_norm, kn))
            return false;
    } else {
        const auto *qkv = T("attn_qkv.weight"), *z = T("attn_gate.weight"), *al = T("ssm_alpha.weight");
        const auto *be = T("ssm_beta.weight"), *conv = T("ssm_conv1d.weight"), *dt = T("ssm_dt.bias");
        const auto *a = T("ssm_a"), *nrm = T("ssm_norm.weight"), *o = T("ssm_out.weight");
        ok = expect(qkv, kHidden, kLinQkv, false) && expect(z, kHidden, kLinV, false) &&
             expect(al, kHidden, kLinHeads, false) && expect(be, kHidden, kLinHeads, false) &&
             expect(conv, 4, kLinQkv, true) && expect(dt, kLinHeads, 0, true) && expect(a, kLinHeads, 0, true) &&
             expect(nrm, kLinDim, 0, true) && expect(o, kLinV, kHidden, false);
        if (!ok) return false;
        std::vector<View> in, ba, out;
        View conv_v, dt_v, a_v;
        if (split) {
            in.push_back(gather_view(qkv, qkv_rows(sh), none));
            in.push_back(gather_view(z, value_rows(sh, 128), none));
            ba.push_back(gather_view(be, value_rows(sh, 1), none));
            ba.push_back(gather_view(al, value_rows(sh, 1), none));
            Ranges blocks;
            for (int b : sh.value_blocks) blocks.push_back({static_cast<uint64_t>(b), static_cast<uint64_t>(b) + 1});
            out.push_back(gather_view(o, none, blocks));
            conv_v = gather_view(conv, qkv_rows(sh), none);
            // 1-D vectors: one "row" of 48 single-element blocks
            Ranges vh;
            for (int v = 0; v < sh.n_vh(); ++v)
                vh.push_back({static_cast<uint64_t>(sh.value_head(v)), static_cast<uint64_t>(sh.value_head(v)) + 1});
            dt_v = gather_view(dt, none, vh);
            a_v = gather_view(a, none, vh);
        } else {
            in = views({qkv, z});
            ba = views({be, al});
            out = views({o});
            conv_v = full_view(conv);
            dt_v = full_view(dt);
            a_v = full_view(a);
        }
        if (!upload_proj(m, &L.in_proj, in) || !upload_proj(m, &L.ba, ba) || !upload_proj(m, &L.out, out) ||
            !upload_vec(m, &L.conv_w, conv_v) || !upload_vec(m, &L.dt, dt_v) || !upload_vec(m, &L.a, a_v) ||
            !upload_vec(m, &L.ssm_norm, nrm))
            return false;
    }
    View gv, uv, dv;
    if (split) {
        const Ranges fr{{static_cast<uint64_t>(sh.ffn0), static_cast<uint64_t>(sh.ffn0 + sh.ffn)}};
        gv = gather_view(gate, fr, none);
        uv = gather_view(up, fr, none);
        dv = gather_view(down, none, Ranges{{static_cast<uint64_t>(sh.ffn0 / 256),
                                             static_cast<uint64_t>((sh.ffn0 + sh.ffn) / 256)}});
    } else {
        gv = full_view(gate);
        uv = full_view(up);
        dv = full_view(down);
    }
    std::vector<View> dvs;
    dvs.push_back(std::move(dv));
    return upload_norm(m, &L.attn_norm, attn_norm) && upload_norm(m, &L.post_norm, post_norm) &&
           upload_gate_up(m, &L, gv, uv) && upload_proj(m, &L.down, dvs);
}

bool meta_is_qwen38(const q38::GGUFFile &f, uint32_t *blocks, uint32_t *nextn)
{
    auto u32 = [&](const char *k, uint32_t v) {
        uint32_t x = 0;
        return f.meta_u32(k, &x) && x == v;
    };
    return f.meta_u32("qwen35.block_count", blocks) && f.meta_u32("qwen35.nextn_predict_layers", nextn) &&
           ((*blocks == kLayers && *nextn == 0) || (*blocks == kTotalLayers && *nextn == 1)) &&
           f.meta_string_is("general.architecture", "qwen35") && u32("qwen35.embedding_length", kHidden) &&
           u32("qwen35.feed_forward_length", kFfn) && u32("qwen35.attention.head_count", 24) &&
           u32("qwen35.attention.head_count_kv", 4) && u32("qwen35.full_attention_interval", 4) &&
           u32("qwen35.ssm.state_size", kLinDim) && u32("qwen35.ssm.group_count", 16) &&
           u32("qwen35.ssm.time_step_rank", kLinHeads) && u32("qwen35.ssm.inner_size", kLinV);
}

bool upload_embedding(Q38Model *m, Q38CuTensor *dst, const q38::GGUFTensorInfo *t)
{
    if (!q38cu_tensor_upload(dst, t->type, t->shape[0], t->shape[1], t->data, Q38CU_LAYOUT_GGUF, m->stream))
        return fail("%s", q38cu_last_error());
    m->tensors.push_back(*dst);
    return true;
}

bool load_mtp(Q38Model *m, const q38::GGUFFile &f)
{
    const auto *emb = f.find_tensor("token_embd.weight"), *out = f.find_tensor("output.weight");
    const auto *eh = find_layer(f, kLayers, "nextn.eh_proj.weight");
    const auto *en = find_layer(f, kLayers, "nextn.enorm.weight");
    const auto *hn = find_layer(f, kLayers, "nextn.hnorm.weight");
    const auto *sh = find_layer(f, kLayers, "nextn.shared_head_norm.weight");
    if (!emb || !out || !expect(emb, kHidden, kVocab, false) || !expect(out, kHidden, kVocab, false) ||
        !expect(eh, 2u * kHidden, kHidden, false) || !expect(en, kHidden, 0, true) || !expect(hn, kHidden, 0, true) ||
        !expect(sh, kHidden, 0, true))
        return false;
    if (&f == &m->gguf) {
        m->mtp_embedding = m->embedding;  // same tensors as the target model's
        m->mtp_output = m->output;
    } else if (!upload_embedding(m, &m->mtp_embedding, emb) || !upload_proj(m, &m->mtp_output, views({out}))) {
        return false;
    }
    if (!load_layer(m, f, kLayers) || !upload_proj(m, &m->eh_proj, views({eh})) || !upload_vec(m, &m->enorm, en) ||
        !upload_vec(m, &m->hnorm, hn) || !upload_norm(m, &m->shared_head_norm, sh))
        return false;
    m->mtp_loaded = true;
    return true;
}

bool alloc_runtime(Q38Model *m)
{
    auto &o = m->owned;
    const size_t ctx = m->context_length;
    m->wide_ld = std::max({kLinQkv + kLinV, kAttnQg + 2 * kAttnKv, 2 * kFfn});
    m->ba_ld = 2 * kLinHeads;
    const size_t q8_blocks = kMaxTokens * static_cast<size_t>(kFfn / 256);
    const Shard &sh = m->shard;
    m->lin_heads = sh.n_vh();
    m->lin_qkv = 5 * sh.n_kh() * kLinDim;
    m->kv_ld = 256 * sh.kv_heads;
    if (sh.world > 1 && (!dalloc(&m->partial, kMaxTokens * kHidden, o) ||
                         !dalloc(&m->logits_local, kMaxTokens * static_cast<size_t>(sh.vocab), o)))
        return false;
    return dalloc(&m->conv_ring, static_cast<size_t>(kRecurrent) * m->lin_qkv * kConvRing, o) &&
           dalloc(&m->delta_state, static_cast<size_t>(kRecurrent) * m->lin_heads * kLinDim * kLinDim, o) &&
           dalloc(&m->k_cache, kFull * ctx * m->kv_ld * m->kv_bytes, o) &&
           dalloc(&m->v_cache, kFull * ctx * m->kv_ld * m->kv_bytes, o) &&
           dalloc(&m->mtp_hidden, kHidden, o) && dalloc(&m->hidden, kReps * kMaxTokens * kHidden, o) &&
           dalloc(&m->normf, kMaxTokens * 2 * kHidden, o) &&
           dalloc(&m->wide, kReps * kMaxTokens * static_cast<size_t>(m->wide_ld), o) &&
           dalloc(&m->ba, kMaxTokens * m->ba_ld, o) && dalloc(&m->act_f, kMaxTokens * kFfn, o) &&
           dalloc(&m->logits, kMaxTokens * static_cast<size_t>(kVocab), o) &&
           dalloc(reinterpret_cast<uint8_t **>(&m->q8), kReps * q8_blocks * sizeof(Q38CuQ8KBlock), o) &&
           dalloc(reinterpret_cast<uint8_t **>(&m->q8_norm), kReps * q8_blocks * sizeof(Q38CuQ8KBlock), o) &&
           dalloc(&m->target_norm, kMaxDrafts * static_cast<size_t>(kHidden), o) &&
           dalloc(&m->ctl, 4, o) && dalloc(&m->ids, kMaxTokens, o) && dalloc(&m->argmax_out, kMaxDrafts, o) &&
           dalloc(&m->history, ctx + 1, o) &&
           dalloc(&m->swiglu_counters, kFfn / 256, o) &&
           dalloc(&m->argmax_part_v, kMaxTokens * q38::kArgmaxCtas, o) &&
           dalloc(&m->argmax_part_i, kMaxTokens * q38::kArgmaxCtas, o) &&
           dalloc(&m->argmax_counters, kMaxTokens, o) &&
           cuda_ok(cudaMallocHost(&m->host_logits, kMaxTokens * static_cast<size_t>(kVocab) * sizeof(float)),
                   "cudaMallocHost") &&
           cuda_ok(cudaMallocHost(&m->host_ctl, 4 * sizeof(int)), "cudaMallocHost") &&
           cuda_ok(cudaMallocHost(&m->host_ids, kMaxTokens * sizeof(uint32_t)), "cudaMallocHost");
}

// ---------------------------------------------------------------------------
// the token step
// ---------------------------------------------------------------------------
// The input of a projection: Q8_K blocks already formed (kActQ8K, with the
// float rows for float-path parts), or floats that the GEMV normalizes /
// gates and quantizes in its prologue (kActRmsNorm: RMSNorm(x) * y;
// kActSwiGLU: silu(x) * y).
struct ActIn {
    int mode = q38::kActQ8K;
    const void *q8 = nullptr;   // kActQ8K
    const float *f = nullptr;   // kActQ8K: float rows for float-path parts
    int f_ld = 0;
    const float *x = nullptr, *y = nullptr;  // fused modes
    int ld = 0;
    float *f_out = nullptr;     // fused modes: optional float copy of the activation
    int reps = 1;               // copies of q8 / x (and y for SwiGLU), rep_bytes apart
    long long rep_bytes = 0, y_rep_bytes = 0;  // y_rep_bytes: copies of the RMSNorm weight
    // kActRmsNorm: Q8_0 side rows formed in the first launch's prologue (see
    // q38_stream.cu), e.g. ssm_beta | ssm_alpha beside attn_qkv | attn_gate
    const void *side_w = nullptr;
    int side_rows = 0, side_ld = 0;
    float *side_out = nullptr;
};

// Copies of an output: the producer stores `reps` copies, `bytes` apart.
struct OutReps {
    int reps = 1;
    long long bytes = 0;
};

// L2 prefetch of the weights streamed next (see q38_stream.cu): a GEMV's
// producer, once its last bulk copy is issued, may prefetch the first
// Q38CU_PREFETCH_KB KiB of each of the next GEMV's CTA ranges, and the
// latency-bound mixer kernels the first Q38CU_MIXER_PREFETCH_MB MiB of the
// projection that follows them.  Both default to 0 (off): measured on B200,
// the decode step is faster without them (the consumers, not HBM, limit the
// launches they would feed).
struct Prefetch {
    const Part *next = nullptr;
};

long long env_bytes(const char *name, long long fallback, int shift)
{
    const char *v = std::getenv(name);
    return (v && *v ? std::atoll(v) : fallback) << shift;
}

Prefetch prefetch_of(const Part *p)
{
    Prefetch f;
    f.next = p && p->int_path ? p : nullptr;
    return f;
}

// The launch fields of a GEMV's prefetch of `pf.next`.
void set_next_prefetch(q38::StreamLaunch &l, const Prefetch &pf)
{
    static const long long per_cta = env_bytes("Q38CU_PREFETCH_KB", 0, 10);
    if (!pf.next || per_cta <= 0) return;
    const Part &n = *pf.next;
    q38::StreamPlan plan;
    if (q38::stream_plan(static_cast<int>(n.t.type), n.rows, static_cast<int>(n.t.shape[0]),
                         static_cast<int>(n.t.tile_rows), 1, &plan) != cudaSuccess)
        return;
    l.nx_weights = n.t.data;
    l.nx_units = plan.units;
    l.nx_grid = plan.grid;
    l.nx_unit_bytes = plan.tile_rows * plan.block_bytes;
    l.nx_cta_bytes = per_cta;
}

// The contiguous prefetch a mixer kernel issues: the leading bytes of `p`.
void mixer_prefetch(const Part *p, const void **ptr, long long *bytes)
{
    static const long long limit = env_bytes("Q38CU_MIXER_PREFETCH_MB", 0, 20);
    *ptr = nullptr;
    *bytes = 0;
    if (!p || limit <= 0) return;
    *ptr = p->t.data;
    *bytes = std::min<long long>(limit, static_cast<long long>(p->t.nbytes)) & ~15LL;
}

const Part *first_part(const Proj &p) { return p.parts.empty() ? nullptr : &p.parts[0]; }

// The timeline record of the next traced launch (null when tracing is off or full).
unsigned long long *next_trace(Q38Model *m)
{
    if (!m->tracing || m->trace_slots >= m->trace_cap) return nullptr;
    return m->trace + q38::kTraceFields * m->trace_slots++;
}

long long hidden_rep_bytes() { return static_cast<long long>(kMaxTokens) * kHidden * 4; }
long long q8_rep_bytes() { return static_cast<long long>(kMaxTokens) * (kFfn / 256) * sizeof(Q38CuQ8KBlock); }
long long norm_rep_bytes() { return static_cast<long long>(kHidden) * 4; }

// Stream GEMM with an output stride and optional accumulation.
// The gate_up SwiGLU epilogue's outputs (see upload_gate_up).
struct SwigluOut {
    float *act = nullptr;
    void *q8 = nullptr;
    int *counters = nullptr;
    int reps = 1;
    long long rep_bytes = 0;
};

bool stream_project(const Part &p, const ActIn &in, int tokens, float *out, int out_ld, int accumulate,
                    const OutReps &orep, const Prefetch &pf, cudaStream_t s, const SwigluOut *sw = nullptr,
                    Q38Model *tm = nullptr, void *export_q8 = nullptr, bool exchange = false)
{
    const int width = static_cast<int>(p.t.shape[0]), nb = width / 256;
    for (int tok0 = 0; tok0 < tokens;) {
        q38::StreamPlan plan;
        cudaError_t e = q38::stream_plan(static_cast<int>(p.t.type), p.rows, width, static_cast<int>(p.t.tile_rows),
                                         tokens - tok0, &plan);
        if (!cuda_ok(e, "stream plan")) return false;
        q38::StreamLaunch l;
        l.weights = p.t.data;
        l.act = in.q8 ? static_cast<const Q38CuQ8KBlock *>(in.q8) + static_cast<size_t>(tok0) * nb : nullptr;
        l.tokens = plan.token_group;
        l.out = out + static_cast<size_t>(tok0) * out_ld;
        l.scratch = p.t.scratch;
        l.dbg_w = nullptr;
        l.dbg_x = nullptr;
        l.out_ld = out_ld;
        l.accumulate = accumulate;
        l.act_mode = in.mode;
        l.act_reps = in.reps;
        l.act_rep_bytes = in.rep_bytes;
        l.act_y_rep_bytes = in.y_rep_bytes;
        l.out_reps = orep.reps;
        l.out_rep_bytes = orep.bytes;
        if (tok0 + plan.token_group >= tokens) set_next_prefetch(l, pf);
        if (tm) l.trace = next_trace(tm);
        if (exchange) {
            // the all-reduce of a row-parallel projection, fused into its GEMV
            l.xc_world = tm->shard.world;
            l.xc_rank = tm->shard.rank;
            l.xc_rows = kHidden;
            for (int r = 0; r < l.xc_world; ++r) l.xc_bufs[r] = reinterpret_cast<unsigned long long *>(tm->ar_bufs[r]);
            l.xc_counter = tm->xc_counter;
        }
        if (export_q8) {
            l.act_export = static_cast<Q38CuQ8KBlock *>(export_q8) + static_cast<size_t>(tok0) * nb;
            l.export_reps = kReps;
            l.export_rep_bytes = q8_rep_bytes();
        }
        if (in.side_w) {
            l.side_w = in.side_w;
            l.side_rows = in.side_rows;
            l.side_ld = in.side_ld;
            l.side_out = in.side_out + static_cast<size_t>(tok0) * in.side_ld;
        }
        if (sw) {
            const int width_out = p.rows / 2;
            l.sw_act = sw->act + static_cast<size_t>(tok0) * width_out;
            l.sw_q8 = static_cast<Q38CuQ8KBlock *>(sw->q8) + static_cast<size_t>(tok0) * (width_out / 256);
            l.sw_counters = sw->counters;
            l.sw_q_reps = sw->reps;
            l.sw_q_rep_bytes = sw->rep_bytes;
        }
        if (in.mode != q38::kActQ8K) {
            l.act_x = in.x + static_cast<size_t>(tok0) * in.ld;
            l.act_y = in.mode == q38::kActSwiGLU ? in.y + static_cast<size_t>(tok0) * in.ld : in.y;
            l.act_ld = in.ld;
            l.act_f_out = in.f_out ? in.f_out + static_cast<size_t>(tok0) * width : nullptr;
        }
        if (!cuda_ok(q38::launch_stream_gemm(static_cast<int>(p.t.type), plan, l, s), "stream gemm launch"))
            return false;
        tok0 += plan.token_group;
    }
    return true;
}

bool has_float_part(const Proj &p)
{
    for (const Part &part : p.parts)
        if (!part.int_path) return true;
    return false;
}

// out[tok * out_ld + part.offset + row] (+)= projection of this token's input.
// A fused input that a float-path part cannot take is materialized first
// (RMSNorm / SwiGLU kernels into the float rows and m->q8).
bool batch_rmsnorm_input(Q38Model *m, const Part &part, const ActIn &in, int tokens, ActIn *out);
ActIn q8_input(const void *q8, const float *f, int f_ld, bool replicated);

// Whether an RMSNorm input of `tokens` tokens is formed by the separate
// prologue kernel (always for batches; for single tokens when
// Q38CU_SPLIT_NORM=1, else inside every CTA of the GEMV).  Both give the same
// bits.
bool split_norm(int tokens)
{
    static const bool single = [] {
        const char *v = std::getenv("Q38CU_SPLIT_NORM");
        return v && *v == '1';
    }();
    return tokens > 1 || single;
}

bool project(Q38Model *m, const Proj &p, ActIn in, int tokens, float *out, int out_ld, int accumulate,
             const OutReps &orep = OutReps(), const Part *next_after = nullptr, bool exchange = false)
{
    const cudaStream_t s = m->stream;
    if (exchange && (p.parts.size() != 1 || !p.parts[0].int_path))
        return fail("the fused exchange takes one integer-path matrix%s", "");
    const int width = p.width;
    if (in.mode != q38::kActQ8K && has_float_part(p)) {
        float *f = in.f_out ? in.f_out : m->act_f;
        const bool ok = in.mode == q38::kActRmsNorm
                            ? cuda_ok(q38::launch_rmsnorm_quant(in.x, in.ld, in.y, width, tokens, f, width, m->q8, s),
                                      "rmsnorm")
                            : cuda_ok(q38::launch_swiglu_quant(in.x, in.y, in.ld, width, tokens, f, m->q8, s),
                                      "swiglu");
        if (!ok) return false;
        in = ActIn();
        in.q8 = m->q8;
        in.f = f;
        in.f_ld = width;
    }
    // Several integer-path parts on one RMSNorm input (attn_q|attn_k and
    // attn_v) normalize it once: the first part's launch exports its Q8_K input
    // (a batch: one prologue kernel with the first part's warp count) and the
    // other parts stage that.
    const bool share = in.mode == q38::kActRmsNorm && p.parts.size() > 1 && !has_float_part(p);
    if (share && split_norm(tokens) && !batch_rmsnorm_input(m, p.parts[0], in, tokens, &in)) return false;
    bool float_part = false;
    for (size_t i = 0; i < p.parts.size(); ++i) {
        const Part &part = p.parts[i];
        const Part *next = i + 1 < p.parts.size() ? &p.parts[i + 1] : next_after;
        if (part.int_path) {
            ActIn pin = in;
            if (i > 0) pin.side_w = nullptr;  // side rows come with the first launch only
            if (share && i > 0) pin = q8_input(m->q8_norm, in.f_out, width, true);
            if (pin.mode == q38::kActRmsNorm && split_norm(tokens) && !batch_rmsnorm_input(m, part, pin, tokens, &pin))
                return false;
            const bool exporting = share && i == 0 && pin.mode == q38::kActRmsNorm;
            if (!stream_project(part, pin, tokens, out + part.offset, out_ld, accumulate, orep, prefetch_of(next), s,
                                nullptr, m, exporting ? m->q8_norm : nullptr, exchange))
                return false;
        } else {
            float_part = true;
            const uint32_t be = q38cu_block_elements(part.t.type), bb = q38cu_block_bytes(part.t.type);
            if (!cuda_ok(q38::launch_f32_gemm_ex(out + part.offset, out_ld, accumulate, in.f, in.f_ld, tokens,
                                                 part.t.shape[0], part.t.data, part.rows, 0,
                                                 static_cast<int>(part.t.type), static_cast<int>(be),
                                                 static_cast<int>(bb), s),
                         "f32 gemm launch"))
                return false;
        }
    }
    // float-path parts store one copy: copy the rows to the replicas
    if (float_part && orep.reps > 1 &&
        !cuda_ok(q38::launch_replicate(out, static_cast<size_t>(tokens) * out_ld * 4, orep.reps, orep.bytes, s),
                 "replicate"))
        return false;
    return true;
}

// Q8_K blocks as input; `replicated` when their producer stored kReps copies.
ActIn q8_input(const void *q8, const float *f, int f_ld, bool replicated = false)
{
    ActIn in;
    in.q8 = q8;
    in.f = f;
    in.f_ld = f_ld;
    if (replicated) {
        in.reps = kReps;
        in.rep_bytes = q8_rep_bytes();
    }
    return in;
}

// A batch (more than one token) with an RMSNorm input takes it as Q8_K from
// the prologue kernel (q38_stream.cu: rms_prologue_kernel) rather than from
// the GEMV's fused prologue, which would normalize and quantize the tokens one
// after another in every CTA.  The kernel runs with the warp count of the
// single-token launch of `part`, so every token's input - and so its output
// row - is bit-identical to what a single-token launch computes; side rows
// (beta | alpha) come with it.
bool batch_rmsnorm_input(Q38Model *m, const Part &part, const ActIn &in, int tokens, ActIn *out)
{
    const int width = static_cast<int>(part.t.shape[0]);
    q38::StreamPlan one;
    if (!cuda_ok(q38::stream_plan(static_cast<int>(part.t.type), part.rows, width, static_cast<int>(part.t.tile_rows),
                                  1, &one),
                 "stream plan"))
        return false;
    q38::RmsPrologue a{};
    a.x = in.x;
    a.ld = in.ld;
    a.w = in.y;
    a.width = width;
    a.tokens = tokens;
    a.warps = q38::stream_consumer_warps(one);
    a.out_q = m->q8_norm;
    a.q_reps = kReps;
    a.q_rep_bytes = q8_rep_bytes();
    a.out_f = in.f_out;
    a.f_ld = width;
    if (in.side_w) {
        a.side_w = in.side_w;
        a.side_rows = in.side_rows;
        a.side_ld = in.side_ld;
        a.side_out = in.side_out;
    }
    if (!cuda_ok(q38::launch_rms_prologue(a, m->stream), "rms prologue")) return false;
    *out = q8_input(m->q8_norm, in.f_out, width, true);
    return true;
}

// RMSNorm(hidden rows) * weight, both replicated.
ActIn rmsnorm_input(const float *hidden, const float *weight, float *f_out = nullptr)
{
    ActIn in;
    in.mode = q38::kActRmsNorm;
    in.x = hidden;
    in.y = weight;
    in.ld = kHidden;
    in.f_out = f_out;
    in.reps = kReps;
    in.rep_bytes = hidden_rep_bytes();
    in.y_rep_bytes = norm_rep_bytes();
    return in;
}

// silu(gate) * up from the replicated gate/up rows.
ActIn swiglu_input(const Q38Model *m)
{
    ActIn in;
    in.mode = q38::kActSwiGLU;
    in.x = m->wide;
    in.y = m->wide + m->shard.ffn;
    in.ld = m->wide_ld;
    in.reps = kReps;
    in.rep_bytes = static_cast<long long>(kMaxTokens) * m->wide_ld * 4;
    return in;
}

OutReps hidden_out() { return OutReps{kReps, hidden_rep_bytes()}; }

// ssm_beta | ssm_alpha as one Q8_0 tensor: the DeltaNet kernel forms both
// projections itself.
bool fusable_ba(const Proj &p, int n_vh)
{
    return p.parts.size() == 1 && !p.parts[0].int_path && p.parts[0].t.type == kQ8_0 && p.rows == 2 * n_vh &&
           p.width == kHidden;
}

// beta | alpha can ride on the input projection's prologue: one Q8_0 tensor
// of 2 x 48 rows over the hidden width, the projection's first part on the
// integer path with at least one CTA per side row.
bool side_ba_ok(const Q38Model *m, const Layer &L)
{
    if (!fusable_ba(L.ba, m->lin_heads) || L.in_proj.parts.empty() || !L.in_proj.parts[0].int_path) return false;
    const Part &p = L.in_proj.parts[0];
    q38::StreamPlan plan;
    if (q38::stream_plan(static_cast<int>(p.t.type), p.rows, static_cast<int>(p.t.shape[0]),
                         static_cast<int>(p.t.tile_rows), 1, &plan) != cudaSuccess)
        return false;
    (void)m;
    return plan.grid >= L.ba.rows && m->ba_ld >= L.ba.rows;
}

bool reduce_into_hidden(Q38Model *m, int tokens);
bool gather_logits(Q38Model *m, int tokens);

bool enqueue_layer(Q38Model *m, int l, int tokens, uint32_t base_hint)
{
    (void)base_hint;
    const Layer &L = m->layers[l];
    const Shard &sh = m->shard;
    const bool tp = sh.world > 1 && l < kLayers;
    const cudaStream_t s = m->stream;
    const ActIn attn_in = rmsnorm_input(m->hidden, L.attn_norm);
    // the weight tensor streamed after this layer's ffn_down
    const Part *after = l + 1 < kLayers ? first_part(m->layers[l + 1].in_proj) : first_part(m->output);
    const void *mixer_pf_ptr = nullptr;
    long long mixer_pf_bytes = 0;
    mixer_prefetch(first_part(L.out), &mixer_pf_ptr, &mixer_pf_bytes);
    // DeltaNet beta | alpha (Q8_0, float path) as side rows of the input
    // projection's prologue, which has RMSNorm(hidden) at hand
    const bool ba_side = !L.full && side_ba_ok(m, L);
    ActIn in_proj_in = attn_in;
    if (ba_side) {
        in_proj_in.side_w = L.ba.parts[0].t.data;
        in_proj_in.side_rows = L.ba.rows;
        in_proj_in.side_ld = m->ba_ld;
        in_proj_in.side_out = m->ba;
    }
    if (!project(m, L.in_proj, in_proj_in, tokens, m->wide, m->wide_ld, 0, OutReps(), first_part(L.out)))
        return false;
    const int mix_width = L.full ? (tp ? sh.heads * kAttnDim : kAttnQ) : (tp ? m->lin_heads * kLinDim : kLinV);
    const ActIn mixed = q8_input(m->q8, m->act_f, mix_width, true);
    if (L.full) {
        q38::AttnArgs a{};
        a.qkv = m->wide;
        a.qkv_ld = m->wide_ld;
        a.k_off = tp ? sh.heads * 2 * kAttnDim : kAttnQg;
        a.v_off = a.k_off + (tp ? sh.kv_heads * kAttnDim : kAttnKv);
        if (tp) {
            a.heads = sh.heads;
            a.head0 = sh.head0;
            a.kv0 = sh.kv0;
            a.kv_ld = m->kv_ld;
        }
        a.q_norm = L.q_norm;
        a.k_norm = L.k_norm;
        a.k_cache = m->k_cache + static_cast<size_t>(L.index) * m->context_length * m->kv_ld * m->kv_bytes;
        a.v_cache = m->v_cache + static_cast<size_t>(L.index) * m->context_length * m->kv_ld * m->kv_bytes;
        a.kv_half = m->kv_bytes == 2;
        a.ctl = m->ctl;
        a.theta_scale = m->theta_scale;
        a.tokens = tokens;
        a.out_f = m->act_f;
        a.out_q = m->q8;
        a.reps = kReps;
        a.q_rep_bytes = q8_rep_bytes();
        a.pf_ptr = mixer_pf_ptr;
        a.pf_bytes = mixer_pf_bytes;
        a.trace = next_trace(m);
        if (!cuda_ok(q38::launch_attention(a, s), "attention")) return false;
    } else {
        q38::DeltaArgs d{};
        if (tp) d.n_kh = sh.n_kh();
        if (ba_side) {
            d.beta = m->ba;
            d.alpha = m->ba + m->lin_heads;
            d.ba_ld = m->ba_ld;
        } else if (fusable_ba(L.ba, m->lin_heads)) {
            d.ba_fused = 1;
            d.ba_w = static_cast<const uint8_t *>(L.ba.parts[0].t.data);
            d.hidden = m->hidden;
            d.attn_norm = L.attn_norm;
            d.hidden_rep_bytes = hidden_rep_bytes();
        } else {
            if (!project(m, L.ba, attn_in, tokens, m->ba, m->ba_ld, 0)) return false;
            d.beta = m->ba;
            d.alpha = m->ba + m->lin_heads;
            d.ba_ld = m->ba_ld;
        }
        d.qkvz = m->wide;
        d.qkvz_ld = m->wide_ld;
        d.z_off = m->lin_qkv;
        d.conv_w = L.conv_w;
        d.conv_ring = m->conv_ring + static_cast<size_t>(L.index) * m->lin_qkv * kConvRing;
        d.dt = L.dt;
        d.a = L.a;
        d.norm_w = L.ssm_norm;
        d.state = m->delta_state + static_cast<size_t>(L.index) * m->lin_heads * kLinDim * kLinDim;
        if (m->snapping && m->delta_snap && L.index < kRecurrent) {
            d.snap = m->delta_snap + static_cast<size_t>(L.index) * m->lin_heads * kLinDim * kLinDim;
            d.snap_stride = static_cast<long long>(kRecurrent) * m->lin_heads * kLinDim * kLinDim;
        }
        d.ctl = m->ctl;
        d.tokens = tokens;
        d.out_f = m->act_f;
        d.out_q = m->q8;
        d.reps = kReps;
        d.q_rep_bytes = q8_rep_bytes();
        d.pf_ptr = mixer_pf_ptr;
        d.pf_bytes = mixer_pf_bytes;
        d.trace = next_trace(m);
        if (!cuda_ok(q38::launch_deltanet(d, s), "deltanet")) return false;
    }
    if (tp && m->xc) {
        // row-parallel, the exchange fused into the GEMV: hidden += the sum over the GPUs
        if (!project(m, L.out, mixed, tokens, m->hidden, kHidden, 1, hidden_out(), first_part(L.gate_up), true))
            return false;
    } else if (tp) {
        // row-parallel: this shard's partial sums, added up across the GPUs
        if (!project(m, L.out, mixed, tokens, m->partial, kHidden, 0, OutReps(), first_part(L.gate_up)) ||
            !reduce_into_hidden(m, tokens))
            return false;
    } else if (!project(m, L.out, mixed, tokens, m->hidden, kHidden, 1, hidden_out(), first_part(L.gate_up))) {
        return false;
    }
    if (L.swiglu_fused) {
        // gate_up's epilogue leaves silu(gate) * up in act_f and its Q8_K blocks in q8
        SwigluOut sw;
        sw.act = m->act_f;
        sw.q8 = m->q8;
        sw.counters = m->swiglu_counters;
        sw.reps = kReps;
        sw.rep_bytes = q8_rep_bytes();
        ActIn gin = rmsnorm_input(m->hidden, L.post_norm);
        if (split_norm(tokens) && !batch_rmsnorm_input(m, L.gate_up.parts[0], gin, tokens, &gin)) return false;
        if (!stream_project(L.gate_up.parts[0], gin, tokens, nullptr, 0, 0, OutReps(), prefetch_of(first_part(L.down)),
                            s, &sw, m))
            return false;
        return project(m, L.down, q8_input(m->q8, m->act_f, kFfn, true), tokens, m->hidden, kHidden, 1,
                       hidden_out(), after);
    }
    const OutReps wide_out{kReps, static_cast<long long>(kMaxTokens) * m->wide_ld * 4};
    if (!project(m, L.gate_up, rmsnorm_input(m->hidden, L.post_norm), tokens, m->wide, m->wide_ld, 0, wide_out,
                 first_part(L.down)))
        return false;
    if (tp && m->xc) return project(m, L.down, swiglu_input(m), tokens, m->hidden, kHidden, 1, hidden_out(), after, true);
    if (tp)
        return project(m, L.down, swiglu_input(m), tokens, m->partial, kHidden, 0, OutReps(), after) &&
               reduce_into_hidden(m, tokens);
    return project(m, L.down, swiglu_input(m), tokens, m->hidden, kHidden, 1, hidden_out(), after);
}

// Embedding rows of `tokens` ids held in device memory.
bool enqueue_embed(Q38Model *m, const Q38CuTensor &emb, const uint32_t *d_ids, int tokens, float *out)
{
    const uint32_t be = q38cu_block_elements(emb.type), bb = q38cu_block_bytes(emb.type);
    return cuda_ok(q38::launch_row_f32_indexed(out, emb.data, kHidden, 0, emb.shape[1], d_ids, tokens,
                                               static_cast<int>(emb.type), static_cast<int>(be),
                                               static_cast<int>(bb), m->stream, kReps,
                                               hidden_rep_bytes() / 4),
                   "embedding");
}

// Final norm + LM head + greedy argmax.  The normed hidden rows go to
// `norm_out` (the MTP head's input); argmax results to argmax_out + out_at;
// with `feed` the last token's argmax also feeds the control block.
bool enqueue_head(Q38Model *m, const float *norm_w, const Proj &head, int tokens, float *norm_out, int out_at,
                  bool feed, int advance)
{
    const cudaStream_t s = m->stream;
    // the next step starts with layer 0's input projection
    if (m->shard.world > 1) {
        // this shard's rows of the LM head, then every GPU gathers all rows
        if (!project(m, head, rmsnorm_input(m->hidden, norm_w, norm_out), tokens, m->logits_local, m->shard.vocab, 0,
                     OutReps(), first_part(m->layers[0].in_proj)) ||
            !gather_logits(m, tokens))
            return false;
    } else if (!project(m, head, rmsnorm_input(m->hidden, norm_w, norm_out), tokens, m->logits, kVocab, 0, OutReps(),
                        first_part(m->layers[0].in_proj))) {
        return false;
    }
    q38::ArgmaxArgs a{};
    a.logits = m->logits;
    a.ld = kVocab;
    a.n = kVocab;
    a.part_v = m->argmax_part_v;
    a.part_i = m->argmax_part_i;
    a.counters = m->argmax_counters;
    a.out = m->argmax_out + out_at;
    a.ctl = feed ? m->ctl : nullptr;
    a.advance = advance;
    a.history = m->history;
    a.history_len = static_cast<int>(m->context_length);
    a.trace = next_trace(m);
    return cuda_ok(q38::launch_argmax(a, tokens, s), "argmax");
}

// One decode step of the target model for the token in ctl[0] at ctl[1].
bool enqueue_decode_step(Q38Model *m)
{
    if (!enqueue_embed(m, m->embedding, reinterpret_cast<const uint32_t *>(m->ctl), 1, m->hidden)) return false;
    for (int l = 0; l < kLayers; ++l)
        if (!enqueue_layer(m, l, 1, 0)) return false;
    // the normed hidden is also the MTP head's next input (qwen38_model.c:1507-1509)
    return enqueue_head(m, m->output_norm, m->output, 1, m->mtp_hidden, 0, true, 1);
}

bool set_ctl(Q38Model *m, uint32_t token, uint32_t position);

// MTP head over `n` tokens whose ids are in d_ids (qwen38_model.c:1268-1294
// for a batch, 1588-1612 for one token): its input is
// [RMSNorm(embedding, enorm) | RMSNorm(previous normed hidden, hnorm)], the
// previous hidden being the MTP state for the first token and the target's
// normed hidden of the token before for the others (rows of `prev_rows`).
// Leaves the MTP layer's output in m->hidden.
bool enqueue_mtp_body(Q38Model *m, const uint32_t *d_ids, int n, const float *prev_rows)
{
    const cudaStream_t s = m->stream;
    const int w2 = 2 * kHidden, nb2 = w2 / 256, nb = kHidden / 256;
    Q38CuQ8KBlock *q8 = static_cast<Q38CuQ8KBlock *>(m->q8);
    if (!enqueue_embed(m, m->mtp_embedding, d_ids, n, m->hidden)) return false;
    bool ok = cuda_ok(q38::launch_rmsnorm_quant(m->hidden, kHidden, m->enorm, kHidden, n, m->normf, w2, q8, s, nb2),
                      "rmsnorm") &&
              cuda_ok(q38::launch_rmsnorm_quant(m->mtp_hidden, kHidden, m->hnorm, kHidden, 1, m->normf + kHidden, w2,
                                                q8 + nb, s, nb2),
                      "rmsnorm");
    if (ok && n > 1)
        ok = cuda_ok(q38::launch_rmsnorm_quant(prev_rows, kHidden, m->hnorm, kHidden, n - 1, m->normf + w2 + kHidden,
                                               w2, q8 + nb2 + nb, s, nb2),
                     "rmsnorm");
    return ok && project(m, m->eh_proj, q8_input(m->q8, m->normf, w2), n, m->hidden, kHidden, 0, hidden_out()) &&
           enqueue_layer(m, kLayers, n, 0);
}

// MTP catch-up of n verified tokens (ids in d_ids, normed target hidden rows
// in target_rows): advances the MTP layer's KV cache and leaves the MTP state
// at the last token's normed hidden.
bool enqueue_mtp_catchup(Q38Model *m, const uint32_t *d_ids, int n, const float *target_rows)
{
    return enqueue_mtp_body(m, d_ids, n, target_rows) &&
           cuda_ok(cudaMemcpyAsync(m->mtp_hidden, target_rows + static_cast<size_t>(n - 1) * kHidden,
                                   kHidden * sizeof(float), cudaMemcpyDeviceToDevice, m->stream),
                   "copy");
}

bool upload_ids(Q38Model *m, const uint32_t *tokens, int n, uint32_t position)
{
    std::memcpy(m->host_ids, tokens, n * sizeof(uint32_t));
    return set_ctl(m, tokens[0], position) &&
           cuda_ok(cudaMemcpyAsync(m->ids, m->host_ids, n * sizeof(uint32_t), cudaMemcpyHostToDevice, m->stream),
                   "ids upload");
}

bool check_status(Q38Model *m);

// Target model over `count` tokens from the current position, in chunks of
// kMaxTokens (upstream q38_batch_target_eval, qwen38_model.c:1241-1266):
// argmax of every token to argmax_host, logits of the last token to the host
// buffer, normed hidden rows to m->target_norm.  count <= kMaxDrafts.
bool target_eval(Q38Model *m, const uint32_t *tokens, uint32_t count, uint32_t *argmax_host)
{
    const uint32_t base = m->position;
    int last_n = 0;
    for (uint32_t c0 = 0; c0 < count; c0 += kMaxTokens) {
        const int n = static_cast<int>(std::min<uint32_t>(kMaxTokens, count - c0));
        bool ok = upload_ids(m, tokens + c0, n, base + c0) && enqueue_embed(m, m->embedding, m->ids, n, m->hidden);
        for (int l = 0; ok && l < kLayers; ++l) ok = enqueue_layer(m, l, n, 0);
        ok = ok && enqueue_head(m, m->output_norm, m->output, n, m->target_norm + static_cast<size_t>(c0) * kHidden,
                                static_cast<int>(c0), false, 0);
        if (!ok || !check_status(m)) return false;
        last_n = n;
    }
    const bool ok =
        cuda_ok(cudaMemcpyAsync(argmax_host, m->argmax_out, count * sizeof(uint32_t), cudaMemcpyDeviceToHost,
                                m->stream),
                "argmax copy") &&
        cuda_ok(cudaMemcpyAsync(m->host_logits, m->logits + static_cast<size_t>(last_n - 1) * kVocab,
                                static_cast<size_t>(kVocab) * sizeof(float), cudaMemcpyDeviceToHost, m->stream),
                "logits copy") &&
        check_status(m);
    if (ok) m->position = base + count;
    return ok;
}

// MTP catch-up over `count` tokens starting at MTP position `base`, in chunks
// (the target rows are m->target_norm, as target_eval left them).
bool mtp_catchup(Q38Model *m, const uint32_t *tokens, uint32_t count, uint32_t base)
{
    for (uint32_t c0 = 0; c0 < count; c0 += kMaxTokens) {
        const int n = static_cast<int>(std::min<uint32_t>(kMaxTokens, count - c0));
        if (!upload_ids(m, tokens + c0, n, base + c0) ||
            !enqueue_mtp_catchup(m, m->ids, n, m->target_norm + static_cast<size_t>(c0) * kHidden) ||
            !check_status(m))
            return false;
    }
    m->mtp_position = base + count;
    return true;
}

// One MTP draft step for `token` at the MTP position; its argmax is left in
// argmax_out[0] and its logits in m->logits.
bool mtp_step(Q38Model *m, uint32_t token)
{
    if (!set_ctl(m, token, m->mtp_position) ||
        !enqueue_mtp_body(m, reinterpret_cast<const uint32_t *>(m->ctl), 1, nullptr) ||
        !enqueue_head(m, m->shared_head_norm, m->mtp_output, 1, m->mtp_hidden, 0, false, 0))
        return false;
    ++m->mtp_position;
    return true;
}

size_t conv_ring_bytes(const Q38Model *m)
{
    return static_cast<size_t>(kRecurrent) * m->lin_qkv * kConvRing * sizeof(float);
}
size_t delta_state_bytes(const Q38Model *m)
{
    return static_cast<size_t>(kRecurrent) * m->lin_heads * kLinDim * kLinDim * sizeof(float);
}

// qwen38_model.c:1200-1226
bool checkpoint_state(Q38Model *m)
{
    const cudaStream_t s = m->stream;
    m->ck_position = m->position;
    m->ck_mtp_position = m->mtp_position;
    return cuda_ok(cudaMemcpyAsync(m->ck_conv_ring, m->conv_ring, conv_ring_bytes(m), cudaMemcpyDeviceToDevice, s),
                   "checkpoint") &&
           cuda_ok(cudaMemcpyAsync(m->ck_delta_state, m->delta_state, delta_state_bytes(m), cudaMemcpyDeviceToDevice,
                                   s),
                   "checkpoint") &&
           cuda_ok(cudaMemcpyAsync(m->ck_mtp_hidden, m->mtp_hidden, kHidden * sizeof(float), cudaMemcpyDeviceToDevice,
                                   s),
                   "checkpoint");
}

bool restore_target_state(Q38Model *m)
{
    const cudaStream_t s = m->stream;
    m->position = m->ck_position;
    return cuda_ok(cudaMemcpyAsync(m->conv_ring, m->ck_conv_ring, conv_ring_bytes(m), cudaMemcpyDeviceToDevice, s),
                   "restore") &&
           cuda_ok(cudaMemcpyAsync(m->delta_state, m->ck_delta_state, delta_state_bytes(m), cudaMemcpyDeviceToDevice,
                                   s),
                   "restore");
}

bool restore_mtp_state(Q38Model *m)
{
    m->mtp_position = m->ck_mtp_position;
    return cuda_ok(cudaMemcpyAsync(m->mtp_hidden, m->ck_mtp_hidden, kHidden * sizeof(float), cudaMemcpyDeviceToDevice,
                                   m->stream),
                   "restore");
}

bool set_ctl(Q38Model *m, uint32_t token, uint32_t position)
{
    m->host_ctl[0] = static_cast<int>(token);
    m->host_ctl[1] = static_cast<int>(position);
    return cuda_ok(cudaMemcpyAsync(m->ctl, m->host_ctl, 2 * sizeof(int), cudaMemcpyHostToDevice, m->stream),
                   "control upload");
}

bool build_decode_graph(Q38Model *m)
{
    if (m->decode_graph) return true;
    cudaGraph_t graph = nullptr;
    if (!cuda_ok(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal), "begin capture")) return false;
    m->trace_slots = 0;
    m->tracing = m->trace != nullptr;
    const bool ok = enqueue_decode_step(m);
    m->tracing = false;
    const cudaError_t e = cudaStreamEndCapture(m->stream, &graph);
    if (!ok || !cuda_ok(e, "end capture")) {
        if (graph) cudaGraphDestroy(graph);
        return false;
    }
    size_t n_nodes = 0;
    if (cudaGraphGetNodes(graph, nullptr, &n_nodes) == cudaSuccess && n_nodes) {
        std::vector<cudaGraphNode_t> nodes(n_nodes);
        if (cudaGraphGetNodes(graph, nodes.data(), &n_nodes) == cudaSuccess) {
            m->step_kernels = 0;
            for (size_t i = 0; i < n_nodes; ++i) {
                cudaGraphNodeType type;
                if (cudaGraphNodeGetType(nodes[i], &type) == cudaSuccess && type == cudaGraphNodeTypeKernel)
                    ++m->step_kernels;
            }
        }
    }
    const cudaError_t ei = cudaGraphInstantiate(&m->decode_graph, graph, 0);
    cudaGraphDestroy(graph);
    return cuda_ok(ei, "graph instantiate");
}

// Capture `enqueue` on the model stream into an executable graph.
template <typename F>
bool capture_graph(Q38Model *m, cudaGraphExec_t *exec, F enqueue)
{
    if (*exec) return true;
    cudaGraph_t graph = nullptr;
    if (!cuda_ok(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal), "begin capture")) return false;
    const bool ok = enqueue();
    const cudaError_t e = cudaStreamEndCapture(m->stream, &graph);
    if (!ok || !cuda_ok(e, "end capture")) {
        if (graph) cudaGraphDestroy(graph);
        return false;
    }
    const cudaError_t ei = cudaGraphInstantiate(exec, graph, 0);
    cudaGraphDestroy(graph);
    return cuda_ok(ei, "graph instantiate");
}

// One MTP draft step for the token in ctl[0] at MTP position ctl[1]
// (qwen38_model.c:1588-1612): its argmax becomes ctl[0], ctl[1] advances and
// the draft is appended to history[ctl[2]++].
bool build_mtp_draft_graph(Q38Model *m)
{
    return capture_graph(m, &m->mtp_draft_graph, [&] {
        return enqueue_mtp_body(m, reinterpret_cast<const uint32_t *>(m->ctl), 1, nullptr) &&
               enqueue_head(m, m->shared_head_norm, m->mtp_output, 1, m->mtp_hidden, 0, true, 1);
    });
}

// The target model over the n tokens in m->ids from position ctl[1], with
// the DeltaNet state after each but the last token kept in m->delta_snap;
// argmax of every token to argmax_out, normed hidden rows to target_norm,
// logits of every token to m->logits.
bool build_verify_graph(Q38Model *m, int n)
{
    return capture_graph(m, &m->verify_graph[n], [&] {
        // traced like the decode step (the same records; read them after
        // speculative calls only)
        m->snapping = true;
        m->trace_slots = 0;
        m->tracing = m->trace != nullptr;
        bool ok = enqueue_embed(m, m->embedding, m->ids, n, m->hidden);
        for (int l = 0; ok && l < kLayers; ++l) ok = enqueue_layer(m, l, n, 0);
        m->snapping = false;
        ok = ok && enqueue_head(m, m->output_norm, m->output, n, m->target_norm, 0, false, 0);
        m->tracing = false;
        return ok;
    });
}

bool check_status(Q38Model *m)
{
    if (!cuda_ok(cudaStreamSynchronize(m->stream), "step")) return false;
    int a = 0, b = 0, c = 0, d = 0;
    if (!cuda_ok(q38::read_and_clear_model_status(&a), "status") ||
        !cuda_ok(q38::read_and_clear_stream_status(&b), "status") ||
        !cuda_ok(q38::read_and_clear_status(&c, m->stream), "status") ||
        !cuda_ok(q38::read_and_clear_tc_status(&d), "status"))
        return false;
    if (a | b | c | d) return fail("a kernel reported status %s", std::to_string(a | b | c | d));
    return true;
}

bool use_device(const Q38Model *m) { return cuda_ok(cudaSetDevice(m->device), "cudaSetDevice"); }

// NCCL, loaded at run time: the process that uses PyTorch already holds its
// libnccl.so.2, any other process gets the system one.
struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*group_start)() = nullptr;
    ncclResult_t (*group_end)() = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    const char *(*error_string)(ncclResult_t) = nullptr;
};

const NcclApi *nccl()
{
    static NcclApi api;
    static bool ok = false;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        auto sym = [&](const char *n) { return dlsym(h, n); };
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(sym("ncclCommInitRank"));
        api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(sym("ncclAllReduce"));
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(sym("ncclAllGather"));
        api.group_start = reinterpret_cast<decltype(api.group_start)>(sym("ncclGroupStart"));
        api.group_end = reinterpret_cast<decltype(api.group_end)>(sym("ncclGroupEnd"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
        ok = api.get_unique_id && api.comm_init_rank && api.all_reduce && api.all_gather && api.group_start &&
             api.group_end && api.comm_destroy && api.error_string;
    });
    return ok ? &api : nullptr;
}

bool nccl_ok(ncclResult_t r, const char *what)
{
    if (r == ncclSuccess) return true;
    const NcclApi *api = nccl();
    return fail("%s", std::string(what) + ": " + (api ? api->error_string(r) : "NCCL unavailable"));
}

constexpr size_t kArFlagBytes = 4096;  // tp_reduce_kernel's flags

// Exchange buffers for the NVLink all-reduce: one allocation per rank
// ([tp_reduce flags][2 halves x world slots x 8 tokens x 5120 words of 8
// bytes: the fused exchange's tagged values, or tp_reduce_kernel's floats]),
// its IPC handle all-gathered over the NCCL communicator, the peers'
// allocations opened.  `mode` 1: tp_reduce_kernel, 2: fused into the GEMVs.
bool setup_p2p(Q38Model *m, int mode)
{
    const int world = m->shard.world, rank = m->shard.rank;
    const size_t bytes = kArFlagBytes + static_cast<size_t>(2) * world * kMaxTokens * kHidden * sizeof(uint64_t);
    static_assert(8 * q38::kTpReduceCtas * sizeof(unsigned long long) <= kArFlagBytes, "flags area");
    static_assert(kMaxTokens == q38::kXcTokens, "exchange slots");
    // Every rank reaches both collectives below whatever failed locally, and
    // all ranks take the same decision (a rank that went its own way would
    // leave the others waiting in a collective).
    struct Entry {
        cudaIpcMemHandle_t handle;
        int ok;
        int pad[3];
    };
    Entry mine{};
    mine.ok = dalloc(&m->ar_base, bytes, m->owned) && dalloc(&m->ar_counter, 2, m->owned) &&
              dalloc(&m->xc_counter, 2, m->owned) &&
              cuda_ok(cudaIpcGetMemHandle(&mine.handle, m->ar_base), "cudaIpcGetMemHandle");
    uint8_t *dev = nullptr;
    if (!dalloc(&dev, sizeof(Entry) * world + 16, m->owned)) return false;  // every rank needs this to go on
    std::vector<Entry> all(world);
    const NcclApi *api = nccl();
    if (!cuda_ok(cudaMemcpy(dev + rank * sizeof(Entry), &mine, sizeof(Entry), cudaMemcpyHostToDevice),
                 "handle copy") ||
        !nccl_ok(api->all_gather(dev + rank * sizeof(Entry), dev, sizeof(Entry), ncclChar, m->comm, m->stream),
                 "handle all-gather") ||
        !cuda_ok(cudaStreamSynchronize(m->stream), "handle all-gather") ||
        !cuda_ok(cudaMemcpy(all.data(), dev, sizeof(Entry) * world, cudaMemcpyDeviceToHost), "handle copy"))
        return false;
    int opened = 1;
    for (int r = 0; r < world; ++r) opened = opened && all[r].ok;
    for (int r = 0; opened && r < world; ++r) {
        uint8_t *base = m->ar_base;
        if (r != rank) {
            void *p = nullptr;
            if (!cuda_ok(cudaIpcOpenMemHandle(&p, all[r].handle, cudaIpcMemLazyEnablePeerAccess),
                         "cudaIpcOpenMemHandle")) {
                opened = 0;
                break;
            }
            m->ipc_opened.push_back(p);
            base = static_cast<uint8_t *>(p);
        }
        m->ar_flags[r] = reinterpret_cast<unsigned long long *>(base);
        m->ar_bufs[r] = reinterpret_cast<float *>(base + kArFlagBytes);
    }
    // the smallest outcome over the ranks
    int *flag = reinterpret_cast<int *>(dev + sizeof(Entry) * world);
    int agreed = 0;
    if (!cuda_ok(cudaMemcpy(flag, &opened, sizeof(int), cudaMemcpyHostToDevice), "flag copy") ||
        !nccl_ok(api->all_reduce(flag, flag, 1, ncclInt32, ncclMin, m->comm, m->stream), "flag all-reduce") ||
        !cuda_ok(cudaStreamSynchronize(m->stream), "flag all-reduce") ||
        !cuda_ok(cudaMemcpy(&agreed, flag, sizeof(int), cudaMemcpyDeviceToHost), "flag copy"))
        return false;
    if (!agreed) {
        for (void *p : m->ipc_opened) cudaIpcCloseMemHandle(p);
        m->ipc_opened.clear();
        return fail("a rank could not map its peers' exchange buffers%s", "");
    }
    m->p2p = mode == 1;
    m->xc = mode == 2;
    m->tp_mode = mode;
    return true;
}

// The residual add after a row-parallel projection: the partial sums of all
// GPUs are added up (all-reduce) and into the hidden rows and their replicas.
bool reduce_into_hidden(Q38Model *m, int tokens)
{
    if (m->p2p) {
        q38::TpReduceArgs a{};
        a.partial = m->partial;
        a.hidden = m->hidden;
        a.reps = kReps;
        a.rep_floats = hidden_rep_bytes() / 4;
        a.n = kHidden;
        a.tokens = tokens;
        a.rank = m->shard.rank;
        a.world = m->shard.world;
        for (int r = 0; r < a.world; ++r) {
            a.bufs[r] = m->ar_bufs[r];
            a.flags[r] = m->ar_flags[r];
        }
        a.counter = m->ar_counter;
        return cuda_ok(q38::launch_tp_reduce(a, m->stream), "NVLink all-reduce");
    }
    const NcclApi *api = nccl();
    return nccl_ok(api->all_reduce(m->partial, m->partial, static_cast<size_t>(tokens) * kHidden, ncclFloat, ncclSum,
                                   m->comm, m->stream),
                   "all-reduce") &&
           cuda_ok(q38::launch_add_replicated(m->hidden, m->partial, kHidden, tokens, kReps, hidden_rep_bytes() / 4,
                                              m->stream),
                   "residual add");
}

// LM head shards -> the full logits rows of every token on every GPU.
bool gather_logits(Q38Model *m, int tokens)
{
    const NcclApi *api = nccl();
    const size_t n = static_cast<size_t>(m->shard.vocab);
    if (!nccl_ok(api->group_start(), "group start")) return false;
    for (int t = 0; t < tokens; ++t)
        if (!nccl_ok(api->all_gather(m->logits_local + t * n, m->logits + static_cast<size_t>(t) * kVocab, n, ncclFloat,
                                     m->comm, m->stream),
                     "all-gather"))
            return false;
    return nccl_ok(api->group_end(), "group end");
}

// ---------------------------------------------------------------------------
// Tensor-core prefill
// ---------------------------------------------------------------------------
// Prompts of at least kTcPrefillMin tokens (without MTP) run layer-major over
// chunks of up to kTcChunk tokens, as the upstream prefill does
// (qwen38_model.c:1519-1560): every projection of a layer is one tensor-core
// GEMM over the whole chunk (q38_tc.cu: the weights dequantized to fp16 once
// per chunk, the Q8_K input to fp16, tcgen05.mma with fp32 accumulation);
// the recurrent mixers run over the chunk's tokens in order, 8 per launch.
// Results agree with token-by-token decoding to the fp16 operand rounding of
// the GEMMs (about 1e-4 relative per projection), not bit for bit.
constexpr int kTcPrefillMin = 64;
constexpr int kTcChunk = 4096;

// Token stride of the tensor-core GEMM's block-scale rows for n tokens.
int tc_scale_ld(int n)
{
    const int tile = q38::tc_token_tile(n);
    return (n + tile - 1) / tile * tile;
}

size_t tc_a16_elements(const Q38Model *m)
{
    size_t most = 0;
    auto see = [&](const Proj &p) {
        for (const Part &part : p.parts)
            most = std::max(most, static_cast<size_t>(part.rows) * static_cast<size_t>(part.t.shape[0]));
    };
    for (int l = 0; l < kLayers; ++l) {
        const Layer &L = m->layers[l];
        see(L.in_proj);
        see(L.out);
        see(L.gate_up);
        see(L.down);
    }
    return most;
}

template <typename T>
bool pf_alloc(Q38Model *m, T **p, size_t count)
{
    void *q = nullptr;
    if (!cuda_ok(cudaMalloc(&q, std::max<size_t>(count * sizeof(T), 256)), "cudaMalloc prefill")) return false;
    m->pf_owned.push_back(q);
    *p = static_cast<T *>(q);
    return true;
}

bool ensure_prefill_buffers(Q38Model *m, int cap)
{
    if (m->pf_cap >= cap) return true;
    for (void *p : m->pf_owned) cudaFree(p);
    m->pf_owned.clear();
    m->pf_cap = 0;
    const size_t n = static_cast<size_t>(cap);
    const size_t q8 = sizeof(Q38CuQ8KBlock);
    bool ok = pf_alloc(m, &m->pf_hidden, n * kHidden) && pf_alloc(m, &m->pf_normf, n * kHidden) &&
              pf_alloc(m, &m->pf_wide, n * m->wide_ld) && pf_alloc(m, &m->pf_act, n * kFfn) &&
              pf_alloc(m, &m->pf_ba, n * m->ba_ld) && pf_alloc(m, &m->pf_scale, (kFfn / 256) * tc_scale_ld(cap)) &&
              pf_alloc(m, reinterpret_cast<uint8_t **>(&m->pf_q8), n * (kFfn / 256) * q8) &&
              pf_alloc(m, reinterpret_cast<uint8_t **>(&m->pf_q8mix), n * (kLinV / 256) * q8) &&
              pf_alloc(m, reinterpret_cast<uint16_t **>(&m->pf_a16), 2 * tc_a16_elements(m)) &&
              pf_alloc(m, reinterpret_cast<uint16_t **>(&m->pf_b16), 2 * n * kFfn) &&
              pf_alloc(m, &m->pf_row_scale, static_cast<size_t>(m->wide_ld)) && pf_alloc(m, &m->pf_ids, n) &&
              pf_alloc(m, &m->pf_oraw, n * kLinV) &&
              pf_alloc(m, &m->pf_rec, q38::delta_prefill_rec_floats(m->lin_heads / 3, (cap + 31) / 32 * 32)) &&
              (m->shard.world == 1 || pf_alloc(m, &m->pf_part, n * kHidden));
    if (ok && m->host_pf_ids) {
        cudaFreeHost(m->host_pf_ids);
        m->host_pf_ids = nullptr;
    }
    ok = ok && cuda_ok(cudaMallocHost(&m->host_pf_ids, n * sizeof(uint32_t)), "cudaMallocHost");
    if (ok) m->pf_cap = cap;
    return ok;
}

// out[t * out_ld + part.offset + row] (+)= projection of tokens 0..n-1, whose
// input is `q8` (Q8_K [n][width / 256]) and, for float-path parts, the float
// rows xf.  Q4_K / Q6_K parts run on the tensor cores; other Q8_K types on
// the streaming batch GEMM; float-path parts on the float kernel.
bool tc_project(Q38Model *m, const Proj &p, const void *q8, const float *xf, int xf_ld, int n, float *out,
                int out_ld, int accumulate, bool split_pairs)
{
    const cudaStream_t s = m->stream;
    const int width = p.width;
    bool staged = false;
    for (const Part &part : p.parts) {
        const int type = static_cast<int>(part.t.type);
        if (part.int_path && q38::tc_weight_type(type)) {
            if (!staged &&
                !cuda_ok(q38::launch_q8k_to_f16(q8, width / 256, n, tc_scale_ld(n), m->pf_b16, m->pf_scale, s),
                         "q8k to f16"))
                return false;
            staged = true;
            const uint32_t bb = q38cu_block_bytes(part.t.type);
            if (!cuda_ok(q38::launch_dequant_f16(part.t.data, type, static_cast<uint64_t>(part.rows),
                                                 static_cast<uint64_t>(width), part.t.tile_rows,
                                                 static_cast<int>(bb), m->pf_a16, m->pf_row_scale,
                                                 split_pairs ? 1 : 0, s),
                         "dequant f16"))
                return false;
            q38::TcGemm g;
            g.out = out + part.offset;
            g.ld = out_ld;
            g.n = part.rows;
            g.m = n;
            g.k = width;
            g.b_scale = m->pf_scale;
            g.b_scale_ld = tc_scale_ld(n);
            g.row_scale = m->pf_row_scale;
            g.accumulate = accumulate;
            if (!cuda_ok(q38::launch_tc_gemm(m->pf_a16, m->pf_b16, g, s), "tensor-core gemm")) return false;
        } else if (part.int_path) {
            if (split_pairs) return fail("interleaved gate|up rows need the tensor-core GEMM%s");
            if (!stream_project(part, q8_input(q8, xf, xf_ld), n, out + part.offset, out_ld, accumulate, OutReps(),
                                Prefetch(), s))
                return false;
        } else {
            const uint32_t be = q38cu_block_elements(part.t.type), bb = q38cu_block_bytes(part.t.type);
            if (!cuda_ok(q38::launch_f32_gemm_ex(out + part.offset, out_ld, accumulate, xf, xf_ld, n, width,
                                                 part.t.data, part.rows, 0, type, static_cast<int>(be),
                                                 static_cast<int>(bb), s),
                         "f32 gemm launch"))
                return false;
        }
    }
    return true;
}

// One layer over the n tokens of the chunk at positions base .. base + n - 1.
// Tensor parallel: the row-parallel projection's partial sums (in pf_part)
// added up across the GPUs (NCCL all-reduce) and into the hidden rows.
bool tc_reduce_into_hidden(Q38Model *m, int n)
{
    const NcclApi *api = nccl();
    return nccl_ok(api->all_reduce(m->pf_part, m->pf_part, static_cast<size_t>(n) * kHidden, ncclFloat, ncclSum,
                                   m->comm, m->stream),
                   "prefill all-reduce") &&
           cuda_ok(q38::launch_add(m->pf_hidden, m->pf_part, kHidden, n, m->stream), "residual add");
}

bool tc_layer(Q38Model *m, int l, int n, uint32_t base)
{
    const Layer &L = m->layers[l];
    const Shard &sh = m->shard;
    const bool tp = sh.world > 1;
    const cudaStream_t s = m->stream;
    const int nb = kHidden / 256;
    Q38CuQ8KBlock *q8 = static_cast<Q38CuQ8KBlock *>(m->pf_q8);
    if (!cuda_ok(q38::launch_rmsnorm_quant(m->pf_hidden, kHidden, L.attn_norm, kHidden, n, m->pf_normf, kHidden, q8,
                                           s, nb),
                 "rmsnorm") ||
        !tc_project(m, L.in_proj, q8, m->pf_normf, kHidden, n, m->pf_wide, m->wide_ld, 0, false))
        return false;
    if (!L.full && !tc_project(m, L.ba, q8, m->pf_normf, kHidden, n, m->pf_ba, m->ba_ld, 0, false)) return false;
    Q38CuQ8KBlock *mix = static_cast<Q38CuQ8KBlock *>(m->pf_q8mix);
    if (!L.full) {
        // the DeltaNet recurrence over the whole chunk in one launch
        q38::DeltaPrefillArgs d{};
        d.qkvz = m->pf_wide;
        d.qkvz_ld = m->wide_ld;
        d.z_off = m->lin_qkv;
        d.beta = m->pf_ba;
        d.alpha = m->pf_ba + m->lin_heads;
        d.ba_ld = m->ba_ld;
        d.conv_w = L.conv_w;
        d.conv_ring = m->conv_ring + static_cast<size_t>(L.index) * m->lin_qkv * kConvRing;
        d.dt = L.dt;
        d.a = L.a;
        d.norm_w = L.ssm_norm;
        d.state = m->delta_state + static_cast<size_t>(L.index) * m->lin_heads * kLinDim * kLinDim;
        d.base = static_cast<int>(base);
        d.tokens = n;
        d.o_raw = m->pf_oraw;
        d.o_ld = m->lin_heads * kLinDim;
        d.out_f = has_float_part(L.out) ? m->pf_act : nullptr;  // floats only for a float-path out projection
        d.out_q = mix;
        d.n_kh = m->lin_heads / 3;
        d.rec = m->pf_rec;
        d.rec_tokens = (n + 31) / 32 * 32;
        if (!cuda_ok(q38::launch_deltanet_prefill(d, s), "deltanet prefill")) return false;
    }
    if (L.full) {
        // full attention of the whole chunk (its keys and values join the caches first)
        q38::AttnPrefillArgs a{};
        a.qkv = m->pf_wide;
        a.qkv_ld = m->wide_ld;
        a.k_off = kAttnQg;
        a.v_off = kAttnQg + kAttnKv;
        a.q_norm = L.q_norm;
        a.k_norm = L.k_norm;
        a.k_cache = m->k_cache + static_cast<size_t>(L.index) * m->context_length * m->kv_ld * m->kv_bytes;
        a.v_cache = m->v_cache + static_cast<size_t>(L.index) * m->context_length * m->kv_ld * m->kv_bytes;
        a.kv_half = m->kv_bytes == 2;
        a.kv_ld = m->kv_ld;
        a.heads = tp ? sh.heads : 24;
        a.head0 = tp ? sh.head0 : 0;
        a.kv0 = tp ? sh.kv0 : 0;
        if (tp) {
            a.k_off = sh.heads * 2 * kAttnDim;
            a.v_off = a.k_off + sh.kv_heads * kAttnDim;
        }
        a.theta_scale = m->theta_scale;
        a.base = static_cast<int>(base);
        a.tokens = n;
        a.qbuf = m->pf_oraw;
        a.out_f = m->pf_act;
        a.out_ld = a.heads * kAttnDim;
        a.out_q = mix;
        if (!cuda_ok(q38::launch_attention_prefill(a, s), "attention prefill")) return false;
    }
    const int mix_width = L.full ? (tp ? sh.heads * kAttnDim : kAttnQ) : (tp ? m->lin_heads * kLinDim : kLinV);
    if (tp ? !tc_project(m, L.out, mix, m->pf_act, mix_width, n, m->pf_part, kHidden, 0, false) ||
                 !tc_reduce_into_hidden(m, n)
           : !tc_project(m, L.out, mix, m->pf_act, mix_width, n, m->pf_hidden, kHidden, 1, false))
        return false;
    const int ffn = tp ? sh.ffn : kFfn;
    if (!cuda_ok(q38::launch_rmsnorm_quant(m->pf_hidden, kHidden, L.post_norm, kHidden, n, m->pf_normf, kHidden, q8,
                                           s, nb),
                 "rmsnorm") ||
        !tc_project(m, L.gate_up, q8, m->pf_normf, kHidden, n, m->pf_wide, m->wide_ld, 0, L.swiglu_fused) ||
        !cuda_ok(q38::launch_swiglu_quant(m->pf_wide, m->pf_wide + ffn, m->wide_ld, ffn, n,
                                          has_float_part(L.down) ? m->pf_act : nullptr, q8, s),
                 "swiglu"))
        return false;
    if (tp)
        return tc_project(m, L.down, q8, m->pf_act, ffn, n, m->pf_part, kHidden, 0, false) &&
               tc_reduce_into_hidden(m, n);
    return tc_project(m, L.down, q8, m->pf_act, ffn, n, m->pf_hidden, kHidden, 1, false);
}

// The widest tensor-parallel model whose shards take the tensor-core prefill:
// the world sizes it has been checked on against one GPU (wider models prefill
// on the 8-token path, which is checked at every world size).
constexpr int kTcPrefillMaxWorld = 2;

bool tc_prefill_enabled()
{
    const char *v = std::getenv("Q38CU_TC_PREFILL");
    return !(v && *v == '0');
}

// The tensor-core prefill takes models whose integer-path matrices are all
// Q4_K or Q6_K (the tensor-core GEMM's types); others (the IQ1_M-typed
// variant) prefill through the 8-token path.
bool tc_prefill_types(const Q38Model *m)
{
    auto ok = [](const Proj &p) {
        for (const Part &part : p.parts)
            if (part.int_path && !q38::tc_weight_type(static_cast<int>(part.t.type))) return false;
        return true;
    };
    for (int l = 0; l < kLayers; ++l) {
        const Layer &L = m->layers[l];
        if (!ok(L.in_proj) || !ok(L.out) || !ok(L.gate_up) || !ok(L.down)) return false;
    }
    return true;
}

// Prefill of `count` tokens from the current position with the tensor-core
// layer-major path; leaves the last token's logits in m->host_logits.
bool prefill_tc(Q38Model *m, const uint32_t *tokens, uint32_t count)
{
    const uint32_t base = m->position;
    const cudaStream_t s = m->stream;
    // buffers for a whole chunk (or the context) on the first call, so a later
    // longer prompt does not reallocate them (cudaMalloc synchronizes the device)
    if (!ensure_prefill_buffers(m, static_cast<int>(std::min<uint32_t>(m->context_length, kTcChunk)))) return false;
    const Q38CuTensor &emb = m->embedding;
    const uint32_t be = q38cu_block_elements(emb.type), bb = q38cu_block_bytes(emb.type);
    for (uint32_t done = 0; done < count;) {
        const int n = static_cast<int>(std::min<uint32_t>(kTcChunk, count - done));
        std::memcpy(m->host_pf_ids, tokens + done, n * sizeof(uint32_t));
        bool ok = cuda_ok(cudaMemcpyAsync(m->pf_ids, m->host_pf_ids, n * sizeof(uint32_t), cudaMemcpyHostToDevice, s),
                          "ids upload") &&
                  cuda_ok(q38::launch_row_f32_indexed(m->pf_hidden, emb.data, kHidden, 0, emb.shape[1], m->pf_ids, n,
                                                      static_cast<int>(emb.type), static_cast<int>(be),
                                                      static_cast<int>(bb), s),
                          "embedding");
        for (int l = 0; ok && l < kLayers; ++l) ok = tc_layer(m, l, n, base + done);
        if (ok && done + n == count) {
            // logits of the last token (upstream: output norm, LM head)
            const float *last = m->pf_hidden + static_cast<size_t>(n - 1) * kHidden;
            ok = cuda_ok(q38::launch_rmsnorm_quant(last, kHidden, m->output_norm, kHidden, 1, m->target_norm, kHidden,
                                                   m->q8, s),
                         "rmsnorm") &&
                 (m->shard.world > 1
                      ? project(m, m->output, q8_input(m->q8, m->target_norm, kHidden), 1, m->logits_local,
                                m->shard.vocab, 0) &&
                            gather_logits(m, 1)
                      : project(m, m->output, q8_input(m->q8, m->target_norm, kHidden), 1, m->logits, kVocab, 0)) &&
                 cuda_ok(cudaMemcpyAsync(m->host_logits, m->logits, static_cast<size_t>(kVocab) * sizeof(float),
                                         cudaMemcpyDeviceToHost, s),
                         "logits copy");
        }
        // the pinned ids are rewritten by the next chunk
        if (!ok || !check_status(m)) return false;
        done += static_cast<uint32_t>(n);
    }
    m->position = base + count;
    return true;
}

Q38Model *open_model(const char *path, uint32_t context_length, int rank, int world, const ncclUniqueId *id)
{
    if (!path || context_length == 0) return nullptr;
    Shard shard;
    if (!make_shard(rank, world, &shard)) {
        fail("tensor-parallel world must be 1, 2, 4 or 8 and rank below it%s");
        return nullptr;
    }
    if (world > 1 && !nccl()) {
        fail("libnccl.so.2 could not be loaded%s");
        return nullptr;
    }
    Q38Model *m = new Q38Model();
    m->shard = shard;
    // KV cache precision: fp32 as upstream, or fp16 with Q38CU_KV_F16=1 at open
    const char *kv16 = std::getenv("Q38CU_KV_F16");
    m->kv_bytes = kv16 && *kv16 == '1' ? 2 : 4;
    m->context_length = context_length;
    // the RoPE frequency step, evaluated by the host libm as upstream does
    // (qwen38_model.c:699)
    m->theta_scale = powf(10000000.0f, -2.0f / 64.0f);
    uint32_t blocks = 0, nextn = 0;
    bool ok = cuda_ok(cudaGetDevice(&m->device), "cudaGetDevice") &&
              cuda_ok(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking), "cudaStreamCreate");
    if (ok && !m->gguf.open(path)) ok = fail("%s", m->gguf.error());
    if (ok && !meta_is_qwen38(m->gguf, &blocks, &nextn)) ok = fail("checkpoint metadata is not Qwen3.8-27B%s");
    if (ok) {
        const auto *emb = m->gguf.find_tensor("token_embd.weight"), *on = m->gguf.find_tensor("output_norm.weight");
        const auto *out = m->gguf.find_tensor("output.weight");
        ok = emb && on && out && expect(emb, kHidden, kVocab, false) && expect(on, kHidden, 0, true) &&
             expect(out, kHidden, kVocab, false);
        if (!ok && !(emb && on && out)) fail("missing token_embd, output_norm or output tensor%s");
        std::vector<View> head;
        head.push_back(world > 1 ? gather_view(out, Ranges{{static_cast<uint64_t>(shard.vocab0),
                                                             static_cast<uint64_t>(shard.vocab0 + shard.vocab)}},
                                               Ranges())
                                 : full_view(out));
        ok = ok && upload_embedding(m, &m->embedding, emb) && upload_norm(m, &m->output_norm, on) &&
             upload_proj(m, &m->output, head);
    }
    for (int l = 0; ok && l < kLayers; ++l) ok = load_layer(m, m->gguf, l);
    // the MTP head runs on one GPU only (tensor-parallel models decode without it)
    if (ok && world == 1 && blocks == kTotalLayers && nextn == 1) ok = load_mtp(m, m->gguf);
    ok = ok && alloc_runtime(m);
    if (ok && world > 1) {
        const NcclApi *api = nccl();
        ok = nccl_ok(api->comm_init_rank(&m->comm, world, *id, rank), "ncclCommInitRank");
        // default: the exchange fused into the GEMVs (measured fastest on 2
        // GPUs); NCCL alone when the peers' memory cannot be mapped
        const char *p2p = std::getenv("Q38CU_TP_P2P");
        const int mode = p2p && *p2p >= '0' && *p2p <= '2' ? *p2p - '0' : 2;
        if (ok && mode && !setup_p2p(m, mode)) {
            if (p2p) {
                ok = false;
            } else {
                std::fprintf(stderr, "q38cuda: peer-memory exchange unavailable (%s); using NCCL's all-reduce\n",
                             q38cu_last_error());
                m->p2p = m->xc = false;
                m->tp_mode = 0;
            }
        }
    }
    if (ok) {
        const char *tv = std::getenv("Q38CU_TRACE");
        if (tv && *tv && *tv != '0') {
            m->trace_cap = 1024;
            ok = dalloc(&m->trace, q38::kTraceFields * static_cast<size_t>(m->trace_cap), m->owned) &&
                 cuda_ok(q38::launch_trace_reset(m->trace, m->trace_cap, m->stream), "trace reset");
        }
    }
    if (m->staging) {
        cudaFree(m->staging);
        m->staging = nullptr;
        m->staging_bytes = 0;
    }
    if (!ok) {
        q38_model_close(m);
        return nullptr;
    }
    return m;
}

}  // namespace

extern "C" {

Q38Model *q38_model_open_gguf(const char *path, uint32_t context_length)
{
    return open_model(path, context_length, 0, 1, nullptr);
}

int q38cu_tp_shard(uint32_t rank, uint32_t world, Q38CuTPShard *out)
{
    Shard sh;
    if (!out || !make_shard(static_cast<int>(rank), static_cast<int>(world), &sh))
        return fail("tensor-parallel world must be 1, 2, 4 or 8 and rank below it%s");
    std::memset(out, 0, sizeof(*out));
    out->rank = rank;
    out->world = world;
    out->n_key_heads = static_cast<uint32_t>(sh.key_heads.size());
    for (size_t i = 0; i < sh.key_heads.size(); ++i) out->key_heads[i] = static_cast<uint32_t>(sh.key_heads[i]);
    out->n_value_blocks = static_cast<uint32_t>(sh.value_blocks.size());
    for (size_t i = 0; i < sh.value_blocks.size(); ++i) out->value_blocks[i] = static_cast<uint32_t>(sh.value_blocks[i]);
    out->attn_head0 = static_cast<uint32_t>(sh.head0);
    out->attn_heads = static_cast<uint32_t>(sh.heads);
    out->kv_head0 = static_cast<uint32_t>(sh.kv0);
    out->kv_heads = static_cast<uint32_t>(sh.kv_heads);
    out->ffn0 = static_cast<uint32_t>(sh.ffn0);
    out->ffn = static_cast<uint32_t>(sh.ffn);
    out->vocab0 = static_cast<uint32_t>(sh.vocab0);
    out->vocab = static_cast<uint32_t>(sh.vocab);
    return 1;
}

int q38cu_nccl_unique_id(void *id_out)
{
    if (!id_out) return fail("id_out is NULL%s");
    const NcclApi *api = nccl();
    if (!api) return fail("libnccl.so.2 could not be loaded%s");
    ncclUniqueId id;
    if (!nccl_ok(api->get_unique_id(&id), "ncclGetUniqueId")) return 0;
    std::memcpy(id_out, &id, sizeof(id));
    return 1;
}

Q38Model *q38cu_model_open_tp(const char *path, uint32_t context_length, uint32_t rank, uint32_t world,
                              const void *nccl_id)
{
    if (world > 1 && !nccl_id) {
        fail("a tensor-parallel open needs the communicator id from q38cu_nccl_unique_id%s");
        return nullptr;
    }
    ncclUniqueId id;
    if (nccl_id) std::memcpy(&id, nccl_id, sizeof(id));
    return open_model(path, context_length, static_cast<int>(rank), static_cast<int>(world), nccl_id ? &id : nullptr);
}

void q38_model_close(Q38Model *m)
{
    if (!m) return;
    cudaSetDevice(m->device);
    if (m->stream) cudaStreamSynchronize(m->stream);
    if (m->decode_graph) cudaGraphExecDestroy(m->decode_graph);
    if (m->mtp_draft_graph) cudaGraphExecDestroy(m->mtp_draft_graph);
    for (auto &g : m->verify_graph)
        if (g) cudaGraphExecDestroy(g);
    // tensors shared between the target and the MTP head are listed once
    for (void *p : m->ipc_opened) cudaIpcCloseMemHandle(p);
    if (m->comm) nccl()->comm_destroy(m->comm);
    for (auto &t : m->tensors) q38cu_tensor_free(&t);
    for (void *p : m->owned) cudaFree(p);
    for (void *p : m->pf_owned) cudaFree(p);
    if (m->host_pf_ids) cudaFreeHost(m->host_pf_ids);
    if (m->staging) cudaFree(m->staging);
    if (m->host_logits) cudaFreeHost(m->host_logits);
    if (m->host_ctl) cudaFreeHost(m->host_ctl);
    if (m->host_ids) cudaFreeHost(m->host_ids);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
}

void q38_model_reset(Q38Model *m)
{
    if (!m || !use_device(m)) return;
    const size_t ctx = m->context_length;
    cudaMemsetAsync(m->conv_ring, 0, conv_ring_bytes(m), m->stream);
    cudaMemsetAsync(m->delta_state, 0, delta_state_bytes(m), m->stream);
    cudaMemsetAsync(m->k_cache, 0, kFull * ctx * m->kv_ld * m->kv_bytes, m->stream);
    cudaMemsetAsync(m->v_cache, 0, kFull * ctx * m->kv_ld * m->kv_bytes, m->stream);
    cudaMemsetAsync(m->mtp_hidden, 0, kHidden * 4, m->stream);
    cudaMemsetAsync(m->ctl, 0, 4 * sizeof(int), m->stream);
    cudaStreamSynchronize(m->stream);
    m->position = 0;
    m->mtp_position = 0;
}

int q38_model_forward_token(Q38Model *m, uint32_t token_id, const float **logits)
{
    if (!m || !logits || token_id >= kVocab || m->position >= m->context_length) return 0;
    if (!use_device(m) || !build_decode_graph(m)) return 0;
    if (!set_ctl(m, token_id, m->position)) return 0;
    if (!cuda_ok(cudaGraphLaunch(m->decode_graph, m->stream), "graph launch")) return 0;
    if (!cuda_ok(cudaMemcpyAsync(m->host_logits, m->logits, static_cast<size_t>(kVocab) * sizeof(float),
                                 cudaMemcpyDeviceToHost, m->stream),
                 "logits copy"))
        return 0;
    if (!check_status(m)) return 0;
    ++m->position;
    *logits = m->host_logits;
    return 1;
}

int q38_model_forward_token_layers(Q38Model *m, uint32_t token_id, uint32_t layer_count, float *hidden_out)
{
    if (!m || !hidden_out || token_id >= kVocab || layer_count > kLayers || m->position >= m->context_length)
        return 0;
    if (!use_device(m) || !set_ctl(m, token_id, m->position)) return 0;
    bool ok = enqueue_embed(m, m->embedding, reinterpret_cast<const uint32_t *>(m->ctl), 1, m->hidden);
    for (uint32_t l = 0; ok && l < layer_count; ++l) ok = enqueue_layer(m, static_cast<int>(l), 1, 0);
    ok = ok && cuda_ok(cudaMemcpyAsync(hidden_out, m->hidden, kHidden * sizeof(float), cudaMemcpyDeviceToHost,
                                       m->stream),
                       "hidden copy");
    if (!ok || !check_status(m)) return 0;
    ++m->position;
    return 1;
}

int q38_model_prefill(Q38Model *m, const uint32_t *tokens, uint32_t token_count, const float **logits)
{
    if (!m || !tokens || !token_count || !logits || token_count > m->context_length - m->position) return 0;
    for (uint32_t i = 0; i < token_count; ++i)
        if (tokens[i] >= kVocab) return 0;
    if (!use_device(m)) return 0;
    if (token_count >= static_cast<uint32_t>(kTcPrefillMin) && !m->mtp_enabled && tc_prefill_enabled() &&
        m->shard.world <= kTcPrefillMaxWorld && tc_prefill_types(m)) {
        if (!prefill_tc(m, tokens, token_count)) return 0;
        *logits = m->host_logits;
        return 1;
    }
    // Chunks of kMaxTokens tokens go through all layers in turn; the result is
    // the upstream layer-major batch's (qwen38_model.c:1519-1560), since every
    // token only depends on the tokens before it.
    const uint32_t base = m->position;
    const int nb = kHidden / 256;
    for (uint32_t done = 0; done < token_count;) {
        const int n = static_cast<int>(std::min<uint32_t>(kMaxTokens, token_count - done));
        const bool last = done + n == token_count;
        bool ok = upload_ids(m, tokens + done, n, base + done) && enqueue_embed(m, m->embedding, m->ids, n, m->hidden);
        for (int l = 0; ok && l < kLayers; ++l) ok = enqueue_layer(m, l, n, 0);
        if (ok && (last || m->mtp_enabled))
            ok = cuda_ok(q38::launch_rmsnorm_quant(m->hidden, kHidden, m->output_norm, kHidden, n, m->target_norm,
                                                   kHidden, m->q8, m->stream),
                         "rmsnorm");
        if (ok && last) {
            // logits of the last token only
            const Q38CuQ8KBlock *q8 = static_cast<const Q38CuQ8KBlock *>(m->q8) + static_cast<size_t>(n - 1) * nb;
            const ActIn last = q8_input(q8, m->target_norm + static_cast<size_t>(n - 1) * kHidden, kHidden);
            ok = (m->shard.world > 1
                      ? project(m, m->output, last, 1, m->logits_local, m->shard.vocab, 0) && gather_logits(m, 1)
                      : project(m, m->output, last, 1, m->logits, kVocab, 0)) &&
                 cuda_ok(cudaMemcpyAsync(m->host_logits, m->logits, static_cast<size_t>(kVocab) * sizeof(float),
                                         cudaMemcpyDeviceToHost, m->stream),
                         "logits copy");
        }
        if (ok && m->mtp_enabled) ok = enqueue_mtp_catchup(m, m->ids, n, m->target_norm);
        if (!ok || !check_status(m)) return 0;
        done += static_cast<uint32_t>(n);
    }
    m->position = base + token_count;
    if (m->mtp_enabled) m->mtp_position = base + token_count;
    *logits = m->host_logits;
    return 1;
}

int q38_model_attach_mtp_gguf(Q38Model *m, const char *path)
{
    if (!m || !path || m->position != 0 || m->mtp_position != 0 || m->mtp_enabled || m->mtp_loaded ||
        m->mtp_gguf.is_open())
        return 0;
    if (m->shard.world > 1) return fail("the MTP head is not available on a tensor-parallel model%s");
    if (!use_device(m)) return 0;
    uint32_t v = 0;
    bool ok = m->mtp_gguf.open(path);
    if (!ok) fail("%s", m->mtp_gguf.error());
    ok = ok && m->mtp_gguf.meta_string_is("general.architecture", "qwen35") &&
         m->mtp_gguf.meta_u32("qwen35.block_count", &v) && v == kTotalLayers &&
         m->mtp_gguf.meta_u32("qwen35.nextn_predict_layers", &v) && v == 1 &&
         m->mtp_gguf.meta_u32("qwen35.embedding_length", &v) && v == kHidden &&
         m->mtp_gguf.meta_u32("qwen35.feed_forward_length", &v) && v == kFfn;
    if (!ok) {
        if (m->mtp_gguf.is_open()) fail("MTP checkpoint metadata is not Qwen3.8-27B%s");
        m->mtp_gguf.close();
        return 0;
    }
    ok = load_mtp(m, m->mtp_gguf);
    if (m->staging) {
        cudaFree(m->staging);
        m->staging = nullptr;
        m->staging_bytes = 0;
    }
    if (!ok) {
        m->mtp_loaded = false;
        m->mtp_gguf.close();
    }
    return ok ? 1 : 0;
}

int q38_model_enable_mtp(Q38Model *m)
{
    if (!m || m->position != 0 || m->mtp_position != 0) return 0;
    if (m->shard.world > 1) return fail("the MTP head is not available on a tensor-parallel model%s");
    if (!m->mtp_loaded) return fail("MTP weights are unavailable; attach the MTP GGUF first%s");
    if (!use_device(m)) return 0;
    if (!m->ck_conv_ring &&
        (!dalloc(reinterpret_cast<uint8_t **>(&m->ck_conv_ring), conv_ring_bytes(m), m->owned) ||
         !dalloc(reinterpret_cast<uint8_t **>(&m->ck_delta_state), delta_state_bytes(m), m->owned) ||
         !dalloc(&m->ck_mtp_hidden, kHidden, m->owned)))
        return fail("unable to allocate speculative checkpoint%s");
    if (!m->delta_snap &&
        !dalloc(reinterpret_cast<uint8_t **>(&m->delta_snap), (kMaxTokens - 1) * delta_state_bytes(m), m->owned))
        return fail("unable to allocate the speculative state snapshots%s");
    m->mtp_enabled = true;
    return 1;
}

int q38_model_mtp_forward(Q38Model *m, uint32_t token_id, const float **logits)
{
    if (!m || !m->mtp_enabled || !logits || token_id >= kVocab || m->mtp_position >= m->context_length) return 0;
    if (!use_device(m) || !mtp_step(m, token_id)) return 0;
    if (!cuda_ok(cudaMemcpyAsync(m->host_logits, m->logits, static_cast<size_t>(kVocab) * sizeof(float),
                                 cudaMemcpyDeviceToHost, m->stream),
                 "logits copy") ||
        !check_status(m)) {
        --m->mtp_position;
        return 0;
    }
    *logits = m->host_logits;
    return 1;
}

// Speculative greedy decoding for more than kMaxTokens drafts: drafts one
// by one with a host round trip each, verifies in chunks, and on a mismatch
// restores the checkpointed state and replays the consumed prefix.
static int speculative_greedy_replay(Q38Model *m, uint32_t token_id, uint32_t stop_token, uint32_t draft_count,
                                     uint32_t *accepted_tokens, uint32_t *accepted_count, const float **next_logits)
{
    if (!checkpoint_state(m)) return 0;

    // drafts from the MTP head, greedy (qwen38_model.c:1636-1650)
    uint32_t drafts[kMaxDrafts], inputs[kMaxDrafts], target[kMaxDrafts];
    uint32_t actual = 0, draft_input = token_id;
    while (actual < draft_count) {
        uint32_t next = 0;
        if (!mtp_step(m, draft_input) ||
            !cuda_ok(cudaMemcpyAsync(&m->host_ids[0], m->argmax_out, sizeof(uint32_t), cudaMemcpyDeviceToHost,
                                     m->stream),
                     "argmax copy") ||
            !check_status(m)) {
            restore_mtp_state(m);
            cudaStreamSynchronize(m->stream);
            return 0;
        }
        next = m->host_ids[0];
        drafts[actual++] = next;
        draft_input = next;
        if (next == stop_token) break;
    }

    // verify on the target model; replay the consumed prefix on a mismatch
    inputs[0] = token_id;
    for (uint32_t i = 1; i < actual; ++i) inputs[i] = drafts[i - 1];
    bool ok = target_eval(m, inputs, actual, target);
    uint32_t matched = 0, next = 0;
    if (ok) {
        while (matched < actual && target[matched] == drafts[matched]) ++matched;
        next = matched < actual ? target[matched] : drafts[actual - 1];
    }
    const uint32_t consumed = matched < actual ? matched + 1 : actual;
    if (ok && consumed < actual) ok = restore_target_state(m) && target_eval(m, inputs, consumed, target);
    if (ok) ok = restore_mtp_state(m) && mtp_catchup(m, inputs, consumed, m->ck_mtp_position);
    if (!ok) {
        restore_target_state(m);
        restore_mtp_state(m);
        cudaStreamSynchronize(m->stream);
        return 0;
    }
    for (uint32_t i = 0; i < matched; ++i) accepted_tokens[i] = drafts[i];
    if (matched < actual) accepted_tokens[matched] = next;
    *accepted_count = consumed;
    *next_logits = m->host_logits;
    return 1;
}

int q38_model_speculative_greedy(Q38Model *m, uint32_t token_id, uint32_t stop_token, uint32_t draft_count,
                                 uint32_t *accepted_tokens, uint32_t *accepted_count, const float **next_logits)
{
    if (!m || !m->mtp_enabled || !accepted_tokens || !accepted_count || !next_logits || token_id >= kVocab ||
        draft_count == 0 || m->position != m->mtp_position || draft_count > m->context_length - m->position)
        return 0;
    if (draft_count > kMaxDrafts) return fail("draft_count above %s is not supported", std::to_string(kMaxDrafts));
    if (!use_device(m)) return 0;
    if (draft_count > kMaxTokens)
        return speculative_greedy_replay(m, token_id, stop_token, draft_count, accepted_tokens, accepted_count,
                                         next_logits);
    // Up to kMaxTokens drafts (upstream qwen38_model.c:1614-1714, same
    // accepted tokens): the draft chain runs on the device (each MTP step feeds
    // its argmax to the next), the target verifies all drafts in one captured
    // pass that keeps the DeltaNet state after each token, and a mismatch rolls
    // the state back to the consumed prefix instead of replaying it.  The conv
    // ring and the KV caches are indexed by position, so the rejected tail is
    // simply overwritten later.  Drafts past a stop token are verified too but
    // never accepted.
    const int n = static_cast<int>(draft_count);
    const uint32_t base = m->position, mbase = m->mtp_position;
    const cudaStream_t s = m->stream;
    if (!build_mtp_draft_graph(m) || !build_verify_graph(m, n)) return 0;
    m->host_ctl[0] = static_cast<int>(token_id);
    m->host_ctl[1] = static_cast<int>(mbase);
    m->host_ctl[2] = 0;
    m->host_ids[0] = token_id;
    bool ok = cuda_ok(cudaMemcpyAsync(m->ck_mtp_hidden, m->mtp_hidden, kHidden * sizeof(float),
                                      cudaMemcpyDeviceToDevice, s),
                      "checkpoint") &&
              cuda_ok(cudaMemcpyAsync(m->ctl, m->host_ctl, 3 * sizeof(int), cudaMemcpyHostToDevice, s), "control");
    for (int i = 0; ok && i < n; ++i) ok = cuda_ok(cudaGraphLaunch(m->mtp_draft_graph, s), "draft graph");
    // verification inputs: the token, then drafts 0 .. n - 2
    ok = ok && cuda_ok(cudaMemcpyAsync(m->ids, m->host_ids, sizeof(uint32_t), cudaMemcpyHostToDevice, s), "ids");
    if (ok && n > 1)
        ok = cuda_ok(cudaMemcpyAsync(m->ids + 1, m->history, (n - 1) * sizeof(uint32_t), cudaMemcpyDeviceToDevice, s),
                     "ids");
    ok = ok && set_ctl(m, token_id, base) && cuda_ok(cudaGraphLaunch(m->verify_graph[n], s), "verify graph");
    uint32_t *target = m->host_ids, drafts[kMaxTokens];
    ok = ok &&
         cuda_ok(cudaMemcpyAsync(target, m->argmax_out, n * sizeof(uint32_t), cudaMemcpyDeviceToHost, s),
                 "argmax copy") &&
         // the drafts, through the pinned logits buffer (rewritten below)
         cuda_ok(cudaMemcpyAsync(m->host_logits, m->history, n * sizeof(uint32_t), cudaMemcpyDeviceToHost, s),
                 "draft copy") &&
         check_status(m);
    if (!ok) {
        cudaStreamSynchronize(s);
        return 0;
    }
    std::memcpy(drafts, m->host_logits, n * sizeof(uint32_t));
    uint32_t actual = static_cast<uint32_t>(n);
    for (uint32_t i = 0; i < actual; ++i)
        if (drafts[i] == stop_token) actual = i + 1;
    uint32_t matched = 0;
    while (matched < actual && target[matched] == drafts[matched]) ++matched;
    const uint32_t next = matched < actual ? target[matched] : drafts[actual - 1];
    const uint32_t consumed = matched < actual ? matched + 1 : actual;
    uint32_t inputs[kMaxTokens];
    inputs[0] = token_id;
    for (uint32_t i = 1; i < consumed; ++i) inputs[i] = drafts[i - 1];
    if (consumed < static_cast<uint32_t>(n))
        ok = cuda_ok(cudaMemcpyAsync(m->delta_state, m->delta_snap + (consumed - 1) * (delta_state_bytes(m) / 4),
                                     delta_state_bytes(m), cudaMemcpyDeviceToDevice, s),
                     "state rollback");
    ok = ok &&
         cuda_ok(cudaMemcpyAsync(m->host_logits, m->logits + static_cast<size_t>(consumed - 1) * kVocab,
                                 static_cast<size_t>(kVocab) * sizeof(float), cudaMemcpyDeviceToHost, s),
                 "logits copy") &&
         cuda_ok(cudaMemcpyAsync(m->mtp_hidden, m->ck_mtp_hidden, kHidden * sizeof(float), cudaMemcpyDeviceToDevice, s),
                 "restore");
    m->position = base + consumed;
    m->mtp_position = mbase;
    ok = ok && mtp_catchup(m, inputs, consumed, mbase);
    if (!ok) {
        cudaStreamSynchronize(s);
        return 0;
    }
    for (uint32_t i = 0; i < matched; ++i) accepted_tokens[i] = drafts[i];
    if (matched < actual) accepted_tokens[matched] = next;
    *accepted_count = consumed;
    *next_logits = m->host_logits;
    return 1;
}

uint32_t q38_model_vocab_size(const Q38Model *m) { return m ? kVocab : 0; }
uint32_t q38_model_position(const Q38Model *m) { return m ? m->position : 0; }
uint32_t q38_model_context_length(const Q38Model *m) { return m ? m->context_length : 0; }

int q38cu_model_generate_greedy(Q38Model *m, uint32_t token_id, uint32_t count, uint32_t *tokens_out)
{
    if (!m || !tokens_out || token_id >= kVocab || !count || count > m->context_length - m->position) return 0;
    if (!use_device(m) || !build_decode_graph(m)) return 0;
    m->host_ctl[2] = 0;
    if (!set_ctl(m, token_id, m->position) ||
        !cuda_ok(cudaMemcpyAsync(m->ctl + 2, m->host_ctl + 2, sizeof(int), cudaMemcpyHostToDevice, m->stream),
                 "control upload"))
        return 0;
    for (uint32_t i = 0; i < count; ++i)
        if (!cuda_ok(cudaGraphLaunch(m->decode_graph, m->stream), "graph launch")) return 0;
    if (!cuda_ok(cudaMemcpyAsync(tokens_out, m->history, count * sizeof(uint32_t), cudaMemcpyDeviceToHost, m->stream),
                 "token copy") ||
        !check_status(m))
        return 0;
    m->position += count;
    return 1;
}

void *q38cu_model_stream(Q38Model *m) { return m ? m->stream : nullptr; }

int q38cu_model_trace(Q38Model *m, uint64_t *records, int max_records)
{
    if (!m || !records || max_records < 0) return -1;
    if (!m->trace || !use_device(m)) return 0;
    const int n = std::min(m->trace_slots, max_records);
    if (!cuda_ok(cudaStreamSynchronize(m->stream), "trace") ||
        !cuda_ok(cudaMemcpy(records, m->trace, q38::kTraceFields * sizeof(uint64_t) * n, cudaMemcpyDeviceToHost),
                 "trace copy") ||
        !cuda_ok(q38::launch_trace_reset(m->trace, m->trace_cap, m->stream), "trace reset") ||
        !cuda_ok(cudaStreamSynchronize(m->stream), "trace reset"))
        return -1;
    return n;
}

int q38cu_model_step_kernels(Q38Model *m)
{
    if (!m || !use_device(m) || !build_decode_graph(m)) return 0;
    return m->step_kernels;
}

}  // extern "C"
