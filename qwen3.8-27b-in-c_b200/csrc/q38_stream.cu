// q38_stream.cu - weight-streaming GEMV/GEMM over a tiled device repack.
//
// Layout (Q38CU_LAYOUT_TILED).  Rows are cut into tiles of T rows (T a
// multiple of 8, chosen from the row count and the SM count); the blocks are
// stored tile by tile, column by column: superblock (row r, column b) sits at
// (((r / T) * nb + b) * T + r % T) * B.  Rows are padded with zero blocks to a
// whole number of tiles.  A "unit" (one column of one tile, T*B bytes) is a
// multiple of 16 bytes, and consecutive units of a tile are adjacent, so any
// run of units moves with one 1-D TMA bulk copy.  The bytes are the GGUF
// bytes, only permuted (the upstream engine's IQ1_S repack,
// src/qwen38/qwen38_quant.c:1255-1377, is the precedent for a load-time view).
//
// Kernel.  Units in memory order are split into G contiguous ranges, one per
// CTA; when the tiles fit on the GPU at once each CTA owns exactly one tile.
// Inside a CTA:
//   * warp (consumers / 32) is the producer: one lane cuts the CTA's range into
//     chunks of up to C units that do not cross a tile, and issues each chunk
//     as one cp.async.bulk into the ring of its consumer group (chunk q goes to
//     group q % J; each group's ring has S stages and one in-order consumer);
//   * J consumer groups, each a whole number of warps covering the T rows:
//     thread rt of a group owns row rt of the tile and, for every column of
//     the group's chunks, decodes its row's superblock against that Q8_K
//     activation column (staged once in shared memory; all threads read the
//     same column - a broadcast).  The superblock's integer sums form inside
//     one thread; its float contribution is added to the thread's row sum.
//     For Q6_K tiles whose height leaves lanes of the groups idle (40 rows:
//     the 5120-row tensors; 8 rows: attn_v), a row's superblock is instead
//     split over L = 4 consecutive lanes that form parts of its integer sums,
//     added exactly with warp shuffles before the float formula: the split
//     changes no result.
// At the end of a tile (or of the CTA's range) the groups' row sums are added
// in group order; a tile shared between CTAs is finished by the last CTA to
// deposit its sums (per-tile counter, deposits added in CTA order).  T, J, C
// and G depend only on the tensor's shape (the ring depth S does not change
// the arithmetic), so a row's float sum is associated the same way for any
// batch size: a batched row is bit-identical
// to the single-token GEMV (the upstream property,
// tests/unit/test_qwen38_quant.c:637-684).  Kernels launch with programmatic
// dependent launch: weight prefetch starts while the previous kernel of the
// stream finishes; activations, deposits, counters and outputs are touched only
// after griddepcontrol.wait.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <type_traits>

#include "../../include/q38cuda.h"
#include "q38_device.cuh"
#include "q38_grid.cuh"
#include "q38_internal.h"
#include "q38_act.cuh"
#include "q38_types.cuh"

namespace q38 {

__device__ int g_stream_status;  // status word of this file's kernels

#ifndef Q38_STREAM_COLUMNS_IN_FLIGHT
#define Q38_STREAM_COLUMNS_IN_FLIGHT 1
#endif
// Superblock columns a thread decodes at once (1 or 2): two give independent
// dependency chains, one keeps the decode loop's code smaller - measured
// slightly faster on B200 (instruction fetch is the kernel's top stall
// reason), so one is the default.  Results are the same either way.
constexpr int kColumnsInFlight = Q38_STREAM_COLUMNS_IN_FLIGHT;
constexpr int kStreamMaxStages = 32;            // stages of all groups together
constexpr size_t kChunkBudget = 112 * 1024;     // one ring pass of all groups (sets the chunk)
constexpr size_t kActBudget = 96 * 1024;        // shared memory for activation columns
constexpr int kMaxConsumers = 256;              // CTA bound for 8 tokens: 288 threads
constexpr size_t kOverlapSmem = 112 * 1024;     // short launches: half an SM's shared memory
constexpr size_t kLongLaunchBytes = 2u << 20;   // per-CTA bytes above which a launch is long

struct StreamArgs {
    const uint8_t *weights;
    int block_bytes;   // B
    int rows;          // N
    int nb;
    int tile_rows;     // T
    int tiles;
    int units;         // tiles * nb
    int groups;        // J
    int parts;         // L: threads per (row, superblock); 1 = one thread decodes a whole superblock
    int group_threads; // threads of one group: T * L rounded up to whole warps
    int stages;        // S, per group
    int chunk;         // C, units per copy
    uint32_t stage_bytes;
    const Q8KBlock *act;  // [tokens][nb]
    int tokens;
    float *out;           // out[tok * out_ld + row]
    int out_ld;
    int accumulate;       // 1: out += result (the residual add of the caller)
    // activation prologue (kActQ8K: `act` holds Q8_K blocks already)
    int act_mode;
    const float *act_x;   // kActRmsNorm: x rows; kActSwiGLU: gate rows  [tokens][act_ld]
    const float *act_y;   // kActRmsNorm: norm weight [width]; kActSwiGLU: up rows
    int act_ld;
    float *act_f_out;     // optional: CTA 0 stores the float activation [tokens][width]
    // Replicated inputs: act / act_x (and act_y in SwiGLU mode) exist act_reps
    // times, act_rep_bytes apart, and so do the RMSNorm weights
    // (act_y_rep_bytes apart); CTA c reads copy c % act_reps, so fewer CTAs
    // load the same freshly written lines at the same time.
    int act_reps;
    long long act_rep_bytes, act_y_rep_bytes;
    // Replicated output: each final row value is also stored out_reps - 1
    // more times, out_rep_bytes apart, for the next kernel's readers.
    int out_reps;
    long long out_rep_bytes;
    // L2 prefetch of the next GEMV's weights, issued by the producer after its
    // last bulk copy: HBM keeps streaming through this kernel's last decode,
    // its epilogue and the next kernel's activation prologue, and the next
    // kernel's first ring fills hit L2.  CTA c prefetches the first
    // nx_cta_bytes of the unit ranges of the next kernel's CTAs c, c + G, ...
    // (the next kernel has nx_grid CTAs over nx_units units of nx_unit_bytes).
    const uint8_t *nx_weights;
    long long nx_units;
    int nx_grid;
    int nx_unit_bytes;
    long long nx_cta_bytes;
    // 1: the CTA has one more warp, after the producer, that runs the shared
    // Q8_K quantizer once on dummy values into a private slot while the
    // consumers load the activation, so that the quantizer's instructions
    // are cached on the SM when the fused RMSNorm prologue reaches it.
    int warm_warp;
    // SwiGLU epilogue (sw_act != nullptr): rows come in (gate i, up i) pairs,
    // 2i and 2i + 1, and a tile is 256 rows = 128 outputs = half a Q8_K
    // block.  Instead of the rows, the kernel stores sw_act[tok][i] =
    // silu(gate) * up, and the second CTA to finish a Q8_K block quantizes it
    // into sw_q8[tok][block] (sw_q_reps copies, sw_q_rep_bytes apart).
    float *sw_act;
    Q8KBlock *sw_q8;
    int *sw_counters;  // one per Q8_K block, zero between launches
    int sw_width;      // outputs per token (rows / 2)
    int sw_q_reps;
    long long sw_q_rep_bytes;
    float *partials;
    int *counters;
    int max_slots;
    int32_t *dbg_w;       // optional [tokens][rows][nb]
    int32_t *dbg_x;
    unsigned long long *trace;  // optional launch timeline record
    // Side rows (RMSNorm input only): CTA c < side_rows also forms the dot
    // product of Q8_0 row c of side_w (GGUF layout, width nb * 256) with the
    // normalized floats of each token, as the upstream float path does
    // (q38_dot_q8_0: fmaf(d * q, x, acc)), into side_out[tok * side_ld + c].
    const uint8_t *side_w;
    int side_rows, side_ld;
    float *side_out;
    // Optional export of the staged activation as Q8_K blocks [tokens][nb]:
    // CTA c < export_reps writes copy c (export_rep_bytes apart), so a later
    // launch on the same input stages it instead of normalizing it again.
    Q8KBlock *act_export;
    int export_reps;
    long long export_rep_bytes;
    // Tensor-parallel exchange (xc_world > 1, a row-parallel projection; see
    // xc_rows): each rank's buffer is [2 halves][world][kXcTokens][rows] words
    // of (call tag << 32 | float bits); xc_counter[0] counts the calls,
    // xc_counter[1] the CTAs done with the current one.
    int xc_world, xc_rank;
    unsigned long long *xc_bufs[kXcMaxWorld];
    unsigned int *xc_counter;
};

// Final store of one output row; with `accumulate` the value is added to what
// the row holds (one rounding, as `hidden[i] += branch[i]` upstream).
__device__ __forceinline__ void store_row(const StreamArgs &g, int tok, int row, float v)
{
    float *dst = g.out + static_cast<size_t>(tok) * g.out_ld + row;
    const float r = g.accumulate ? __fadd_rn(*dst, v) : v;
    *dst = r;
    for (int k = 1; k < g.out_reps; ++k)
        *reinterpret_cast<float *>(reinterpret_cast<char *>(dst) + k * g.out_rep_bytes) = r;
}

__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long *p, unsigned long long v)
{
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long *p)
{
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Tensor-parallel exchange of finished rows of a row-parallel projection,
// fused with the GEMV: a tile crosses NVLink as soon as its sums are final,
// while other CTAs still stream weights.  Each `writer` thread holds row
// `row`'s partial sums vals[tok] on this rank.  It stores every value into
// slot `rank` of every rank's buffer (peer memory) as one 8-byte word
// (call tag << 32 | float bits, tag = call + 1), so the value and the proof
// that it belongs to this call arrive together - no fence and no separate
// flag; then it reads its row's word from every rank's slot in its own
// buffer, waiting (bounded) until each carries this call's tag, adds them in
// rank order and stores out[tok][row] (+)= sum - the all-reduce and the
// residual add of the upstream's row-parallel projection.  The tag compare
// is wrap-safe.  Buffers alternate halves by call parity: a rank writes a
// half again only two calls later, after every rank has finished the call
// that read it.  An abandoned wait records the status word and leaves the
// row unstored; so does `keep` false (this CTA's own sums are void after an
// abandoned wait, but the peers still get words to end their waits).
// xs[1]: the call number.
template <int MT>
__device__ void xc_rows(const StreamArgs &g, int row, bool writer, bool keep, const float *vals, volatile int *xs)
{
    if (!writer) return;
    const unsigned int tag = static_cast<unsigned int>(xs[1]) + 1u;
    const size_t slot = static_cast<size_t>(kXcTokens) * g.rows;
    const size_t half = static_cast<size_t>((tag - 1u) & 1u) * g.xc_world * slot;
#pragma unroll
    for (int tok = 0; tok < MT; ++tok) {
        if (tok >= g.tokens) break;
        const unsigned long long word =
            (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(vals[tok]);
        for (int r = 0; r < g.xc_world; ++r)
            st_relaxed_sys_u64(g.xc_bufs[r] + half + g.xc_rank * slot + static_cast<size_t>(tok) * g.rows + row, word);
    }
    const unsigned long long *mine = g.xc_bufs[g.xc_rank] + half;
    const unsigned long long start = global_timer_ns();
#pragma unroll
    for (int tok = 0; tok < MT; ++tok) {
        if (tok >= g.tokens) break;
        float sum = 0.0f;
        bool ok = true;
        for (int r = 0; r < g.xc_world && ok; ++r) {
            const unsigned long long *p = mine + r * slot + static_cast<size_t>(tok) * g.rows + row;
            unsigned long long w = ld_relaxed_sys_u64(p);
            while (static_cast<int>(static_cast<unsigned int>(w >> 32) - tag) < 0) {
                if (global_timer_ns() - start > kWaitLimitNs) {
                    atomicExch(&g_stream_status, kStatusWaitTimeout);
                    ok = false;
                    break;
                }
                w = ld_relaxed_sys_u64(p);
            }
            const float v = __uint_as_float(static_cast<unsigned int>(w));
            sum = r == 0 ? v : __fadd_rn(sum, v);
        }
        if (ok && keep) store_row(g, tok, row, sum);
    }
}

template <typename T>
__device__ __forceinline__ const T *replica(const T *p, long long bytes, int reps)
{
    return reps > 1 ? reinterpret_cast<const T *>(reinterpret_cast<const char *>(p) + (blockIdx.x % reps) * bytes)
                    : p;
}

__host__ __device__ __forceinline__ int cta_of_unit(long long u, long long units, int grid)
{
    // inverse of first_unit(c) = floor(units * c / grid)
    return static_cast<int>(((u + 1) * grid - 1) / units);
}

__device__ __forceinline__ void consumer_barrier(int consumers)
{
    asm volatile("bar.sync 1, %0;" ::"r"(consumers) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Chunk walker shared by the producer and the consumers: the CTA's range of
// units [u0, u1) cut at tile ends and every C units.
struct ChunkWalk {
    int u, u_end, nb, chunk;
    int t, b;  // tile and column of `u`
    __device__ void init(int u0, int u1, int nb_, int chunk_)
    {
        u = u0;
        u_end = u1;
        nb = nb_;
        chunk = chunk_;
        t = u0 / nb_;
        b = u0 - t * nb_;
    }
    __device__ bool done() const { return u >= u_end; }
    __device__ int len() const { return min(chunk, min(nb - b, u_end - u)); }
    __device__ void next(int n)
    {
        u += n;
        b += n;
        if (b == nb) { b = 0; ++t; }
    }
};

// CTA size bound: 416 threads (157 registers) for up to 2 tokens, 288 threads
// (227 registers) for 4 and 8; 672 threads (97 registers) for one token with
// superblocks split across threads.
template <int MT, int L = 1> struct StreamThreads {
    static constexpr int kValue = L > 1 ? 672 : (MT <= 2 ? 416 : 288);
};

// Threads per superblock a decoder supports (block_part / finish).
template <typename Dec> struct SplitParts { static constexpr int kMax = 1; };
template <> struct SplitParts<DecQ4K> { static constexpr int kMax = 4; };
template <> struct SplitParts<DecQ6K> { static constexpr int kMax = 4; };
// IQ1_M can split too (block_part / finish), but measured slower on B200
// (17408 x 5120: 24.2 us at 4 lanes against 18.1 us at one), so the planner
// only splits it when Q38CU_STREAM_PARTS asks.
template <> struct SplitParts<DecIQ1M> { static constexpr int kMax = 4; };

// Activation prologues.  They run after the grid dependency, so their global
// loads are the latency every launch pays before its first decode: each
// thread issues all the loads of a batch (ActBatch blocks per warp) before
// using any of them, instead of one L2 round trip per loop iteration.  The
// batch is shallower when several tokens share the kernel's registers.
template <int MT, int L = 1> struct ActBatch { static constexpr int kValue = L > 1 ? 1 : (MT == 1 ? 4 : 2); };

__device__ __forceinline__ void load8(const float *p, float (&v)[8])
{
    const float4 a = *reinterpret_cast<const float4 *>(p);
    const float4 b = *reinterpret_cast<const float4 *>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

__device__ __forceinline__ void ldg8(const float *p, float (&v)[8])
{
    const float4 a = __ldg(reinterpret_cast<const float4 *>(p));
    const float4 b = __ldg(reinterpret_cast<const float4 *>(p + 4));
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// Q8_K of one 256-element block held 8 per lane, into an activation slot
// (raw bsums in aux[8..15], as the Q8_K staging path leaves them).  One
// out-of-line copy serves every kernel of this file: the prologue runs once
// per launch, so its code is fetched cold unless the launches share it.
__device__ __noinline__ void quantize_to_slot(Act *slot, float v0, float v1, float v2, float v3, float v4,
                                              float v5, float v6, float v7)
{
    const int lane = threadIdx.x & 31;
    const float v[8] = {v0, v1, v2, v3, v4, v5, v6, v7};
    const WarpQ8K r = act_quantize_warp(v);
    slot->q[lane * 2] = r.q0;
    slot->q[lane * 2 + 1] = r.q1;
    if ((lane & 3) == 0) slot->aux[8 + (lane >> 2)] = r.sums_word;
    if (lane == 0) slot->xs = r.scale;
}

__device__ __forceinline__ void store_block(Act &slot, const float (&v)[8])
{
    quantize_to_slot(&slot, v[0], v[1], v[2], v[3], v[4], v[5], v[6], v[7]);
}

__device__ __forceinline__ void store_floats(const StreamArgs &g, int tok, int e, const float (&v)[8])
{
    if (g.act_f_out && blockIdx.x == 0) {
        float *o = g.act_f_out + static_cast<size_t>(tok) * g.nb * 256 + e;
        *reinterpret_cast<float4 *>(o) = make_float4(v[0], v[1], v[2], v[3]);
        *reinterpret_cast<float4 *>(o + 4) = make_float4(v[4], v[5], v[6], v[7]);
    }
}

// Fused modes: the consumer warps form the Q8_K blocks of this launch's
// input in shared memory themselves (the upstream q38_rmsnorm or q38_swiglu
// followed by q38_quantize_q8_k) while the producer warp is already streaming
// weights.  Warp w owns blocks w, w + warps, ...; lane l holds elements
// 8l .. 8l + 7 of each.  Every CTA computes the same values in the same order
// (the order depends only on the shape); CTA 0 also stores the floats when
// asked.
// The RMSNorm weights do not depend on the previous kernel: when a warp's
// blocks fit one batch they are loaded before the grid dependency resolves.
template <int MT, int L>
__device__ __forceinline__ bool preload_norm_weights(const StreamArgs &g, int consumers,
                                                     float (&wv)[ActBatch<MT, L>::kValue][8])
{
    constexpr int kActBatch = ActBatch<MT, L>::kValue;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = consumers >> 5;
    if (g.act_mode != kActRmsNorm || (g.nb + warps - 1) / warps > kActBatch) return false;
    const float *w = replica(g.act_y, g.act_y_rep_bytes, g.act_reps);
#pragma unroll
    for (int j = 0; j < kActBatch; ++j) {
        const int b = warp + j * warps;
        if (b < g.nb) ldg8(w + b * 256 + lane * 8, wv[j]);
    }
    return true;
}

// Shared-memory slots of the side rows' per-warp partials: past the RMS sum's
// doubles in `red`, [token][warp] (red holds consumers * MT floats).
__device__ __forceinline__ float *side_slots(double *red) { return reinterpret_cast<float *>(red) + 64; }

__device__ __forceinline__ void finish_side_rows(const StreamArgs &g, double *red, int consumers, int tokens)
{
    if (!g.side_w || static_cast<int>(blockIdx.x) >= g.side_rows || threadIdx.x >= tokens) return;
    const int warps = consumers >> 5, tok = threadIdx.x;
    const float *slot = side_slots(red) + tok * warps;
    float total = 0.0f;
    for (int w = 0; w < warps; ++w) total = __fadd_rn(total, slot[w]);
    g.side_out[static_cast<size_t>(tok) * g.side_ld + blockIdx.x] = total;
}

template <int MT, int L>
__device__ void stage_fused_activation(const StreamArgs &g, Act *acts, double *red, int consumers,
                                       const float (&wpre)[ActBatch<MT, L>::kValue][8], bool preloaded)
{
    constexpr int kActBatch = ActBatch<MT, L>::kValue;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, warps = consumers >> 5;
    const int per_warp = (g.nb + warps - 1) / warps;
    const float *act_x = replica(g.act_x, g.act_rep_bytes, g.act_reps);
    const float *act_y = g.act_mode == kActSwiGLU ? replica(g.act_y, g.act_rep_bytes, g.act_reps)
                                                  : replica(g.act_y, g.act_y_rep_bytes, g.act_reps);
    for (int tok = 0; tok < MT; ++tok) {
        Act *slots = acts + tok * g.nb;
        if (tok >= g.tokens) {
            for (int b = warp; b < g.nb; b += warps) {
                slots[b].q[lane * 2] = slots[b].q[lane * 2 + 1] = 0u;
                if (lane < 8) slots[b].aux[8 + lane] = 0u;
                if (lane == 0) slots[b].xs = 0.0f;
            }
            continue;
        }
        const float *x = act_x + static_cast<size_t>(tok) * g.act_ld;
        if (g.act_mode == kActSwiGLU) {
            const float *u = act_y + static_cast<size_t>(tok) * g.act_ld;
            for (int j0 = 0; j0 < per_warp; j0 += kActBatch) {
                float xv[kActBatch][8], uv[kActBatch][8];
#pragma unroll
                for (int j = 0; j < kActBatch; ++j) {
                    const int b = warp + (j0 + j) * warps;
                    if (b < g.nb) {
                        load8(x + b * 256 + lane * 8, xv[j]);
                        load8(u + b * 256 + lane * 8, uv[j]);
                    }
                }
#pragma unroll
                for (int j = 0; j < kActBatch; ++j) {
                    const int b = warp + (j0 + j) * warps;
                    if (b >= g.nb) break;
                    float v[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(act_silu(xv[j][i]), uv[j][i]);
                    store_floats(g, tok, b * 256 + lane * 8, v);
                    store_block(slots[b], v);
                }
            }
            continue;
        }
        // RMSNorm: sum of squares (double, per thread in block and element
        // order, then the warp tree, then warps in order), scale, quantize.
        float xv[kActBatch][8], wv[kActBatch][8];
        const bool one_batch = per_warp <= kActBatch;
        // side row of this CTA: lane l of block b takes Q8_0 block 8b + l / 4,
        // elements 8 (l % 4) .. + 7, loaded with the activation
        const bool side = g.side_w && static_cast<int>(blockIdx.x) < g.side_rows;
        const uint8_t *side_row = side ? g.side_w + static_cast<size_t>(blockIdx.x) * g.nb * 8 * 34 : nullptr;
        float sd[kActBatch];
        uint32_t sq[kActBatch][2];
        auto load_side = [&](int j, int b) {
            const uint8_t *blk = side_row + static_cast<size_t>(b * 8 + (lane >> 2)) * 34;
            const unsigned short *h = reinterpret_cast<const unsigned short *>(blk);
            const unsigned short *qp = reinterpret_cast<const unsigned short *>(blk + 2 + (lane & 3) * 8);
            sd[j] = __half2float(__ushort_as_half(__ldg(h)));
            sq[j][0] = static_cast<uint32_t>(__ldg(qp)) | static_cast<uint32_t>(__ldg(qp + 1)) << 16;
            sq[j][1] = static_cast<uint32_t>(__ldg(qp + 2)) | static_cast<uint32_t>(__ldg(qp + 3)) << 16;
        };
        float side_acc = 0.0f;
        double part = 0.0;
        for (int j0 = 0; j0 < per_warp; j0 += kActBatch) {
#pragma unroll
            for (int j = 0; j < kActBatch; ++j) {
                const int b = warp + (j0 + j) * warps;
                if (b < g.nb) {
                    load8(x + b * 256 + lane * 8, xv[j]);
                    if (side && one_batch) load_side(j, b);
                    if (one_batch) {
                        if (preloaded) {
#pragma unroll
                            for (int i = 0; i < 8; ++i) wv[j][i] = wpre[j][i];
                        } else {
                            ldg8(act_y + b * 256 + lane * 8, wv[j]);  // in the same round trip
                        }
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < kActBatch; ++j) {
                const int b = warp + (j0 + j) * warps;
                if (b >= g.nb) break;
#pragma unroll
                for (int i = 0; i < 8; ++i) part += static_cast<double>(__fmul_rn(xv[j][i], xv[j][i]));
            }
            if (tok == 0 && j0 == 0 && g.trace && threadIdx.x == 0 && part >= 0.0) trace_mark(g.trace, kTraceXLoaded);
        }
        part = act_warp_sum_d(part);
        if (lane == 0) red[warp] = part;
        consumer_barrier(consumers);
        double sum = 0.0;
        for (int w = 0; w < warps; ++w) sum += red[w];
        consumer_barrier(consumers);  // red is reused by the next token
        if (tok == 0) trace_mark(g.trace, kTraceNormed);
        const float mean = static_cast<float>(sum / static_cast<double>(g.nb * 256));
        const float scale = __fdiv_rn(1.0f, sqrtf(__fadd_rn(mean, kRmsEps)));
        for (int j0 = 0; j0 < per_warp; j0 += kActBatch) {
            // a single batch keeps x and the weights in registers from the first pass
            if (!one_batch) {
#pragma unroll
                for (int j = 0; j < kActBatch; ++j) {
                    const int b = warp + (j0 + j) * warps;
                    if (b < g.nb) {
                        load8(x + b * 256 + lane * 8, xv[j]);
                        ldg8(act_y + b * 256 + lane * 8, wv[j]);
                        if (side) load_side(j, b);
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < kActBatch; ++j) {
                const int b = warp + (j0 + j) * warps;
                if (b >= g.nb) break;
                float v[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(__fmul_rn(xv[j][i], scale), wv[j][i]);
                store_floats(g, tok, b * 256 + lane * 8, v);
                store_block(slots[b], v);
                if (side) {
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int qv = static_cast<int8_t>((sq[j][i >> 2] >> (8 * (i & 3))) & 0xFFu);
                        side_acc = fmaf(__fmul_rn(sd[j], static_cast<float>(qv)), v[i], side_acc);
                    }
                }
            }
        }
        if (side) {
            // the warp's partial (lane tree); the warps' partials are added in
            // warp order after staging's closing barrier (finish_side_rows)
            const float r = act_warp_sum_f(side_acc);
            if (lane == 0) side_slots(red)[tok * warps + warp] = r;
        }
        if (tok == 0) {
            __syncwarp();
            trace_mark(g.trace, kTraceQuantized);
        }
    }
}

// Q8_K staging: the blocks' words (scale, 64 quant words, 8 bsum words) are
// copied into the activation slots.  Each global load round trip costs about
// a microsecond between dependent kernels, so all words are loaded in one
// round trip where possible: 16-byte loads (when each token's blocks start on
// a 16-byte boundary), kBatch of them in flight per thread; 4-byte loads
// otherwise.  Tokens beyond g.tokens stage zeros.
template <int MT>
__device__ void stage_q8k_activation(const StreamArgs &g, Act *acts, int consumers)
{
    constexpr int kWords = 73;
    const int tid = threadIdx.x;
    const Q8KBlock *act = replica(g.act, g.act_rep_bytes, g.act_reps);
    const int row_words = g.nb * kWords;
    auto put = [&](int tok, int w4, uint32_t v) {
        const int blk = w4 / kWords, w = w4 - blk * kWords;
        Act &slot = acts[tok * g.nb + blk];
        if (w == 0) slot.xs = __uint_as_float(v);
        else if (w <= 64) slot.q[w - 1] = v;      // quants
        else slot.aux[8 + (w - 65)] = v;          // bsums
    };
    if (row_words % 4 == 0 && (reinterpret_cast<uintptr_t>(act) & 15u) == 0) {
        constexpr int kBatch = 8;
        const int row_vecs = row_words / 4, total = MT * row_vecs;
        for (int i0 = tid; i0 < total; i0 += consumers * kBatch) {
            uint4 v[kBatch];
#pragma unroll
            for (int k = 0; k < kBatch; ++k) {
                const int i = i0 + k * consumers;
                v[k] = make_uint4(0u, 0u, 0u, 0u);
                const int tok = i / row_vecs;
                if (i < total && tok < g.tokens)
                    v[k] = __ldcg(reinterpret_cast<const uint4 *>(act + static_cast<size_t>(tok) * g.nb) +
                                  (i - tok * row_vecs));
            }
#pragma unroll
            for (int k = 0; k < kBatch; ++k) {
                const int i = i0 + k * consumers;
                if (i >= total) break;
                const int tok = i / row_vecs, w4 = (i - tok * row_vecs) * 4;
                put(tok, w4, v[k].x);
                put(tok, w4 + 1, v[k].y);
                put(tok, w4 + 2, v[k].z);
                put(tok, w4 + 3, v[k].w);
            }
        }
        return;
    }
    constexpr int kBatchWords = 8;
    const int total = MT * row_words;
    for (int i0 = tid; i0 < total; i0 += consumers * kBatchWords) {
        uint32_t v[kBatchWords];
#pragma unroll
        for (int k = 0; k < kBatchWords; ++k) {
            const int i = i0 + k * consumers;
            v[k] = 0u;
            const int tok = i / row_words;
            if (i < total && tok < g.tokens)
                v[k] = __ldcg(reinterpret_cast<const uint32_t *>(act + static_cast<size_t>(tok) * g.nb) +
                              (i - tok * row_words));
        }
#pragma unroll
        for (int k = 0; k < kBatchWords; ++k) {
            const int i = i0 + k * consumers;
            if (i >= total) break;
            const int tok = i / row_words;
            put(tok, i - tok * row_words, v[k]);
        }
    }
}
// SwiGLU epilogue of a whole 256-row tile t (see StreamArgs::sw_act): rows
// 2i and 2i + 1 (lanes `parts` apart) hold gate and up of one output (the upstream q38_swiglu,
// qwen38_model.c:523-541); the Q8_K block of outputs 256 (t / 2) .. + 255 is
// quantized (qwen38_quant.c:50-88) by whichever of its two CTAs finishes last.
template <int MT>
__device__ void swiglu_epilogue(const StreamArgs &g, int t, int rt, int grp, int part, bool failed,
                                const float (&total)[MT], int consumers, volatile int *last_flag)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const bool pair_lead = (rt & 1) == 0;
    const int i = (t * 256 + rt) >> 1;  // output index
#pragma unroll
    for (int tok = 0; tok < MT; ++tok) {
        const float up = __shfl_xor_sync(0xffffffffu, total[tok], g.parts);
        if (grp == 0 && part == 0 && pair_lead && !failed && tok < g.tokens)
            g.sw_act[static_cast<size_t>(tok) * g.sw_width + i] = __fmul_rn(act_silu(total[tok]), up);
    }
    __threadfence();
    consumer_barrier(consumers);
    const int block = t >> 1;
    // Every CTA counts itself in, failed or not, so the block counter always
    // returns to zero and a later launch never sees a stale count; a CTA
    // that abandoned a wait (its sums are unusable, the status word says
    // so) only skips the quantization.
    if (threadIdx.x == 0) *last_flag = atomicAdd(&g.sw_counters[block], 1) == 1 ? (failed ? 2 : 1) : 0;
    consumer_barrier(consumers);
    const int last = *last_flag;
    if (!last) return;
    if (threadIdx.x == 0) g.sw_counters[block] = 0;
    if (last != 1 || failed) return;
    __threadfence();
    if (warp < MT && warp < g.tokens) {
        const float *src = g.sw_act + static_cast<size_t>(warp) * g.sw_width + block * 256 + lane * 8;
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = __ldcg(src + k);
        const WarpQ8K r = act_quantize_warp(v);
        for (int k = 0; k < g.sw_q_reps; ++k) {
            Q8KBlock *d = reinterpret_cast<Q8KBlock *>(reinterpret_cast<char *>(
                              g.sw_q8 + static_cast<size_t>(warp) * (g.sw_width / 256) + block) +
                          k * g.sw_q_rep_bytes);
            uint32_t *q = reinterpret_cast<uint32_t *>(d->quants);
            q[lane * 2] = r.q0;
            q[lane * 2 + 1] = r.q1;
            if ((lane & 3) == 0) reinterpret_cast<uint32_t *>(d->sums)[lane >> 2] = r.sums_word;
            if (lane == 0) d->scale = r.scale;
        }
    }
}

template <typename Dec, int MT, bool kDbg>
__device__ __forceinline__ void decode_column(const StreamArgs &g, const uint8_t *blk, const Act *acts, int b,
                                              int row, float (&acc)[MT], const uint2 *grid)
{
    SmemActs<MT> a;
#pragma unroll
    for (int tok = 0; tok < MT; ++tok) a.p[tok] = acts + tok * g.nb + b;
    int w[MT], x[MT];
    float val[MT];
    run_block<Dec, MT>(blk, a, w, x, val, grid);
#pragma unroll
    for (int tok = 0; tok < MT; ++tok) acc[tok] += val[tok];
    if constexpr (kDbg) {
        if (row < g.rows) {
#pragma unroll
            for (int tok = 0; tok < MT; ++tok) {
                if (tok < g.tokens) {
                    const size_t o = (static_cast<size_t>(tok) * g.rows + row) * g.nb + b;
                    g.dbg_w[o] = w[tok];
                    g.dbg_x[o] = x[tok];
                }
            }
        }
    }
}

// The producer's L2 prefetch of the next GEMV's leading weights (see
// StreamArgs::nx_weights).  Unit ranges start on 16-byte boundaries.
__device__ __forceinline__ void prefetch_next_ranges(const StreamArgs &g)
{
    if (!g.nx_weights || g.nx_cta_bytes <= 0) return;
    for (long long cn = blockIdx.x; cn < g.nx_grid; cn += gridDim.x) {
        const long long u0 = g.nx_units * cn / g.nx_grid, u1 = g.nx_units * (cn + 1) / g.nx_grid;
        long long bytes = (u1 - u0) * g.nx_unit_bytes;
        if (bytes > g.nx_cta_bytes) bytes = g.nx_cta_bytes & ~15LL;
        const uint8_t *p = g.nx_weights + u0 * g.nx_unit_bytes;
        for (long long off = 0; off < bytes; off += 1 << 20) {
            const long long take = bytes - off < (1 << 20) ? bytes - off : (1 << 20);
            bulk_prefetch_l2(p + off, static_cast<uint32_t>(take));
        }
    }
}

// One superblock decoded by the L threads of a row (lanes `mask`), thread
// `part` taking part `part` of the integer sums; the parts are added across
// the lanes (exact integer adds) and every lane forms the same float value.
template <typename Dec, int MT, int L, bool kDbg>
__device__ __forceinline__ void decode_column_part(const StreamArgs &g, const uint8_t *blk, const Act *acts, int b,
                                                   int row, float (&acc)[MT], int part, unsigned mask,
                                                   const uint2 *grid)
{
    SmemActs<MT> a;
#pragma unroll
    for (int tok = 0; tok < MT; ++tok) a.p[tok] = acts + tok * g.nb + b;
    int w[MT], x[MT];
    float val[MT];
    if constexpr (NeedsGrid<Dec>::kEntries > 0) Dec::template block_part<MT, L>(blk, a, part, w, x, grid);
    else Dec::template block_part<MT, L>(blk, a, part, w, x);
#pragma unroll
    for (int o = 1; o < L; o <<= 1) {
#pragma unroll
        for (int tok = 0; tok < MT; ++tok) {
            w[tok] += __shfl_xor_sync(mask, w[tok], o);
            x[tok] += __shfl_xor_sync(mask, x[tok], o);
        }
    }
    Dec::template finish<MT>(blk, a, w, x, val);
#pragma unroll
    for (int tok = 0; tok < MT; ++tok) acc[tok] += val[tok];
    if constexpr (kDbg) {
        if (part == 0 && row < g.rows) {
#pragma unroll
            for (int tok = 0; tok < MT; ++tok) {
                if (tok < g.tokens) {
                    const size_t o = (static_cast<size_t>(tok) * g.rows + row) * g.nb + b;
                    g.dbg_w[o] = w[tok];
                    g.dbg_x[o] = x[tok];
                }
            }
        }
    }
}

template <typename Dec, int MT, int L, bool kDbg>
__global__ void __launch_bounds__(StreamThreads<MT, L>::kValue, 1) stream_gemm_kernel(StreamArgs g)
{
    extern __shared__ __align__(128) uint8_t smem[];
    const int consumers = static_cast<int>(blockDim.x) - 32 - 32 * g.warm_warp;
    const int n_stages = g.groups * g.stages;
    uint8_t *stage_mem = smem;
    Act *acts = reinterpret_cast<Act *>(smem + static_cast<size_t>(n_stages) * g.stage_bytes);
    uint2 *grid = reinterpret_cast<uint2 *>(acts + MT * g.nb);
    float *red = reinterpret_cast<float *>(grid + NeedsGrid<Dec>::kEntries);  // [groups][MT][row threads]
    uint64_t *full = reinterpret_cast<uint64_t *>(red + consumers * MT);
    uint64_t *empty = full + kStreamMaxStages;
    volatile int *issued = reinterpret_cast<volatile int *>(empty + kStreamMaxStages);
    volatile int *last_flag = issued + 1;
    Act *warm_slot = reinterpret_cast<Act *>(const_cast<int *>(issued) + 4);  // 16-byte aligned, past the flags

    const int tid = threadIdx.x;
    trace_mark(g.trace, kTraceStart);
    trace_mark(g.trace, kTraceLastStart);
    const int G = gridDim.x, c = blockIdx.x;
    const int u0 = static_cast<int>(static_cast<long long>(g.units) * c / G);
    const int u1 = static_cast<int>(static_cast<long long>(g.units) * (c + 1) / G);
    // Group k is threads [k * group_threads, (k + 1) * group_threads): row rt
    // of the tile is decoded by its L consecutive threads (part = tid % L);
    // threads past the tile's rows, and past the last group, only keep step.
    const int group_threads = g.group_threads;
    const int row_slots = group_threads / L;  // >= tile_rows

    if (tid == 0) {
        for (int s = 0; s < n_stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], group_threads / 32);  // the owning group's warps free a stage
        }
        *issued = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (tid >= consumers) {
        // ---------------- producer warp ----------------
        if (tid == consumers) {
            ChunkWalk w;
            w.init(u0, u1, g.nb, g.chunk);
            int q = 0, grp = 0, slot = 0, wrap = 0;
            const uint64_t stream_policy = l2_evict_first_policy();  // weights are read once per step
            const size_t unit_bytes = static_cast<size_t>(g.tile_rows) * g.block_bytes;
            for (; !w.done(); ++q) {
                const int n = w.len();
                const int s = grp * g.stages + slot;
                if (wrap > 0) {
                    if (!mbar_wait_bounded(&empty[s], static_cast<uint32_t>(wrap - 1) & 1u, &g_stream_status)) break;
                    fence_proxy_async_shared();
                }
                const uint32_t bytes = static_cast<uint32_t>(n * unit_bytes);
                mbar_arrive_expect_tx(&full[s], bytes);
                bulk_copy_g2s_hint(stage_mem + static_cast<size_t>(s) * g.stage_bytes,
                                   g.weights + static_cast<size_t>(w.u) * unit_bytes, bytes, &full[s], stream_policy);
                *issued = q + 1;
                w.next(n);
                if (++grp == g.groups) {
                    grp = 0;
                    if (++slot == g.stages) { slot = 0; ++wrap; }
                }
            }
            prefetch_next_ranges(g);
        } else if (tid >= consumers + 32) {
            // ---------------- code warm-up warp ----------------
            const float d = static_cast<float>((tid & 31) + 1);
            quantize_to_slot(warm_slot, d, -d, d, -d, d, -d, d, -d);
        }
        return;
    }

    // ---------------- consumer warps ----------------
    const int lane = tid & 31;
    // Codebook expansion (constant tables only) may precede the grid dependency.
    fill_grid<Dec>(grid, tid, consumers);
    float wpre[ActBatch<MT, L>::kValue][8];
    const bool preloaded = preload_norm_weights<MT, L>(g, consumers, wpre);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    trace_mark(g.trace, kTraceReady);
    trace_mark(g.trace, kTraceLastReady);
    volatile int *xs = issued + 2;  // exchange state (see xc_rows)
    if (g.xc_world > 1 && tid == 0) xs[1] = static_cast<int>(__ldcg(g.xc_counter));

    const int slots = MT * g.nb;
    if (g.act_mode == kActQ8K) {
        // Activation columns -> shared memory: quants, raw bsums (into
        // aux[8..15]) and scale; tokens beyond g.tokens are zero.  The
        // per-format sums are then derived from shared memory only.
        stage_q8k_activation<MT>(g, acts, consumers);
    } else {
        stage_fused_activation<MT, L>(g, acts, reinterpret_cast<double *>(red), consumers, wpre, preloaded);
    }
    consumer_barrier(consumers);
    for (int slot = tid; slot < slots; slot += consumers) Dec::aux_from_raw(acts[slot]);
    if (g.act_mode == kActRmsNorm) finish_side_rows(g, reinterpret_cast<double *>(red), consumers, g.tokens);
    consumer_barrier(consumers);
    if (g.act_export && static_cast<int>(blockIdx.x) < g.export_reps) {
        // scale, 64 quant words and the 8 raw bsum words (aux[8..15]) of each slot
        Q8KBlock *dst = reinterpret_cast<Q8KBlock *>(reinterpret_cast<char *>(g.act_export) +
                                                     blockIdx.x * g.export_rep_bytes);
        const int words = g.tokens * g.nb * 73;
        for (int i = tid; i < words; i += consumers) {
            const int slot = i / 73, w = i - slot * 73;
            uint32_t *d = reinterpret_cast<uint32_t *>(dst + slot);
            const Act &a = acts[slot];
            d[w] = w == 0 ? __float_as_uint(a.xs) : w <= 64 ? a.q[w - 1] : a.aux[8 + (w - 65)];
        }
    }
    trace_mark(g.trace, kTraceStaged);
    trace_mark(g.trace, kTraceFirstStaged);
    // Only now let the next kernel in the stream launch and start its weight
    // prefetch: launched earlier, its bulk copies queue ahead of this kernel's
    // activation loads in the memory system and stall the prologue.  It still
    // waits for our completion before it touches anything we write.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    const int grp = tid / group_threads, rt = (tid - grp * group_threads) / L;
    const int part = L > 1 ? tid % L : 0;
    const unsigned part_mask = L > 1 ? ((1u << L) - 1u) << (lane & ~(L - 1)) : 0xFFFFFFFFu;
    const bool in_group = grp < g.groups;
    const bool mine_row = in_group && rt < g.tile_rows;
    const size_t unit_bytes = static_cast<size_t>(g.tile_rows) * g.block_bytes;
    bool failed = false;
    int slot = 0, wrap = 0;  // this group's ring position
    ChunkWalk w;
    w.init(u0, u1, g.nb, g.chunk);
    int q = 0;  // CTA chunk index
    while (!w.done()) {
        // One tile segment: the chunks of tile w.t inside [u0, u1).
        const int t = w.t;
        const bool seg_whole = w.b == 0 && (t + 1) * g.nb <= u1;
        const int row = t * g.tile_rows + rt;
        float acc[MT];
#pragma unroll
        for (int tok = 0; tok < MT; ++tok) acc[tok] = 0.0f;
        do {
            const int n = w.len();
            if (q % g.groups == grp) {
                const int s = grp * g.stages + slot;
                if (!failed) failed = !mbar_wait_bounded(&full[s], static_cast<uint32_t>(wrap) & 1u, &g_stream_status);
                if constexpr (L > 1) failed = __any_sync(part_mask, failed);  // a row's lanes decode together
                if (!failed && mine_row) {
                    const uint8_t *base = stage_mem + static_cast<size_t>(s) * g.stage_bytes +
                                          static_cast<size_t>(rt) * g.block_bytes;
                    int k = 0;
                    if constexpr (L > 1) {
                        for (; k < n; ++k)
                            decode_column_part<Dec, MT, L, kDbg>(g, base + k * unit_bytes, acts, w.b + k, row, acc,
                                                                 part, part_mask, grid);
                    }
                    if constexpr (MT <= 2 && !kDbg && L == 1 && kColumnsInFlight == 2) {
                        // two columns in flight: independent decode chains,
                        // the earlier column still added first
                        for (; k + 1 < n; k += 2) {
                            float a0[MT], a1[MT];
#pragma unroll
                            for (int tok = 0; tok < MT; ++tok) a0[tok] = a1[tok] = 0.0f;
                            decode_column<Dec, MT, kDbg>(g, base + k * unit_bytes, acts, w.b + k, row, a0, grid);
                            decode_column<Dec, MT, kDbg>(g, base + (k + 1) * unit_bytes, acts, w.b + k + 1, row, a1,
                                                         grid);
#pragma unroll
                            for (int tok = 0; tok < MT; ++tok) {
                                acc[tok] += a0[tok];
                                acc[tok] += a1[tok];
                            }
                        }
                    }
                    for (; k < n; ++k) {
                        float a0[MT];
#pragma unroll
                        for (int tok = 0; tok < MT; ++tok) a0[tok] = 0.0f;
                        decode_column<Dec, MT, kDbg>(g, base + k * unit_bytes, acts, w.b + k, row, a0, grid);
#pragma unroll
                        for (int tok = 0; tok < MT; ++tok) acc[tok] += a0[tok];
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
                if (++slot == g.stages) { slot = 0; ++wrap; }
            }
            ++q;
            w.next(n);
        } while (!w.done() && w.t == t);

        if (w.done()) trace_mark(g.trace, kTraceDecoded);
        // Combine the groups' row sums in group order.
        if (in_group && part == 0) {
#pragma unroll
            for (int tok = 0; tok < MT; ++tok) red[(grp * MT + tok) * row_slots + rt] = acc[tok];
        }
        consumer_barrier(consumers);
        float total[MT];
#pragma unroll
        for (int tok = 0; tok < MT; ++tok) {
            float sum = 0.0f;
            if (grp == 0)
                for (int k = 0; k < g.groups; ++k) sum += red[(k * MT + tok) * row_slots + rt];
            total[tok] = sum;
        }
        if (seg_whole && g.sw_act) {
            swiglu_epilogue<MT>(g, t, rt, grp, part, failed, total, consumers, last_flag);
        } else if (seg_whole) {
            if (g.xc_world > 1) {
                // (also after a failure, so that the peers' waits end; the
                // status word already says the results are void)
                xc_rows<MT>(g, row, grp == 0 && part == 0 && mine_row && row < g.rows, !failed, total, xs);
            } else if (grp == 0 && part == 0 && !failed && mine_row && row < g.rows) {
#pragma unroll
                for (int tok = 0; tok < MT; ++tok)
                    if (tok < g.tokens) store_row(g, tok, row, total[tok]);
            }
        } else {
            // The tile is shared with other CTAs: deposit this segment's sums;
            // the last CTA to arrive adds all deposits in CTA order.
            const long long tu = static_cast<long long>(t) * g.nb;
            const int cf = cta_of_unit(tu, g.units, G);
            const int cl = cta_of_unit(tu + g.nb - 1, g.units, G);
            const int n_dep = cl - cf + 1, dep = c - cf;
            if (grp == 0 && part == 0 && mine_row) {
                float *mine = g.partials + (static_cast<size_t>(t) * g.max_slots + dep) * MT * g.tile_rows;
#pragma unroll
                for (int tok = 0; tok < MT; ++tok) __stcg(mine + tok * g.tile_rows + rt, total[tok]);
            }
            __threadfence();
            consumer_barrier(consumers);
            // Failed or not, every CTA counts its deposit, so the last to
            // arrive always resets the counter for the next launch; after an
            // abandoned wait (recorded in the status word) the row is not
            // stored.
            if (tid == 0) *last_flag = atomicAdd(&g.counters[t], 1) == n_dep - 1 ? (failed ? 2 : 1) : 0;
            consumer_barrier(consumers);
            const bool finisher = *last_flag == 1 && !failed && grp == 0 && part == 0 && mine_row;
            float fin[MT];
#pragma unroll
            for (int tok = 0; tok < MT; ++tok) fin[tok] = 0.0f;
            if (finisher) {
                __threadfence();
                const float *base = g.partials + static_cast<size_t>(t) * g.max_slots * MT * g.tile_rows;
#pragma unroll
                for (int tok = 0; tok < MT; ++tok) {
                    if (tok >= g.tokens) break;
                    for (int k = 0; k < n_dep; ++k)
                        fin[tok] += __ldcg(base + (static_cast<size_t>(k) * MT + tok) * g.tile_rows + rt);
                }
            }
            if (*last_flag && tid == 0) atomicExch(&g.counters[t], 0);
            if (*last_flag && g.xc_world > 1) {
                // the tile's last CTA exchanges it (also after a failure, so
                // that the peers' waits end)
                xc_rows<MT>(g, row, grp == 0 && part == 0 && mine_row && row < g.rows, finisher, fin, xs);
            } else if (finisher && row < g.rows) {
#pragma unroll
                for (int tok = 0; tok < MT; ++tok)
                    if (tok < g.tokens) store_row(g, tok, row, fin[tok]);
            }
        }
        consumer_barrier(consumers);  // `red` and the flag are reused by the next segment
    }
    if (g.xc_world > 1 && tid == 0) {
        // the CTA is done with this call; the last one advances the call number
        __threadfence();
        if (atomicAdd(g.xc_counter + 1, 1u) == gridDim.x - 1) {
            g.xc_counter[1] = 0;
            __threadfence();
            atomicExch(g.xc_counter, static_cast<unsigned int>(xs[1]) + 1u);
        }
    }
    if (failed && tid == 0) {
        // Drain the bulk copies still in flight before shared memory goes away:
        // the last copy issued into each stage completes after all earlier ones,
        // and the last (groups * stages) chunks cover every stage's last copy.
        const int n_issued = *issued;
        const int from = n_issued - n_stages;
        for (int j = from < 0 ? 0 : from; j < n_issued; ++j) {
            const int k = j / g.groups;
            const int st = (j % g.groups) * g.stages + k % g.stages;
            mbar_wait_bounded(&full[st], static_cast<uint32_t>(k / g.stages) & 1u, nullptr);
        }
    }
    trace_mark(g.trace, kTraceEnd);
}

// GGUF row-major -> tiled layout (padding rows stay zero).
__global__ void repack_tiled_kernel(uint8_t *dst, const uint8_t *src, uint64_t rows, uint64_t nb, uint32_t tile_rows,
                                    uint32_t block_bytes)
{
    const uint64_t total = rows * nb * block_bytes;
    for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint64_t blk = i / block_bytes, k = i - blk * block_bytes;
        const uint64_t r = blk / nb, b = blk - r * nb;
        const uint64_t t = r / tile_rows, rr = r - t * tile_rows;
        dst[((t * nb + b) * tile_rows + rr) * block_bytes + k] = src[i];
    }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
namespace {

// Tuning overrides read from the environment (for sweeps; unset = the
// built-in plan).
int env_knob(const char *name, int fallback)
{
    const char *v = std::getenv(name);
    return v && *v ? std::atoi(v) : fallback;
}

template <typename Dec>
size_t stream_smem(const StreamPlan &p)
{
    return static_cast<size_t>(p.groups) * p.stages * p.stage_bytes + static_cast<size_t>(p.mt) * p.nb * sizeof(Act) +
           static_cast<size_t>(NeedsGrid<Dec>::kEntries) * 8 + static_cast<size_t>(p.threads - 32) * p.mt * 4 +
           2 * kStreamMaxStages * 8 + 16 + sizeof(Act);  // + the warm-up warp's slot
}

template <typename Dec, int MT, bool kDbg, int L = 1>
const void *stream_kernel_ptr()
{
    return reinterpret_cast<const void *>(stream_gemm_kernel<Dec, MT, L, kDbg>);
}

template <typename Dec>
const void *select_kernel(int mt, bool dbg, int parts)
{
    if constexpr (SplitParts<Dec>::kMax >= 4) {
        if (mt == 1 && parts == 4)
            return dbg ? stream_kernel_ptr<Dec, 1, true, 4>() : stream_kernel_ptr<Dec, 1, false, 4>();
        if (mt == 1 && parts == 2)
            return dbg ? stream_kernel_ptr<Dec, 1, true, 2>() : stream_kernel_ptr<Dec, 1, false, 2>();
    }
    if (parts != 1) return nullptr;
    switch (mt) {
    case 1: return dbg ? stream_kernel_ptr<Dec, 1, true>() : stream_kernel_ptr<Dec, 1, false>();
    case 2: return dbg ? stream_kernel_ptr<Dec, 2, true>() : stream_kernel_ptr<Dec, 2, false>();
    case 4: return dbg ? stream_kernel_ptr<Dec, 4, true>() : stream_kernel_ptr<Dec, 4, false>();
    default: return dbg ? stream_kernel_ptr<Dec, 8, true>() : stream_kernel_ptr<Dec, 8, false>();
    }
}

// Opt a kernel in to the device's full dynamic shared memory, once per device.
cudaError_t opt_in(const void *kernel)
{
    struct Entry { const void *kernel; int device; };
    static Entry done[256];
    static int used = 0;
    static std::mutex lock;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> guard(lock);
    for (int i = 0; i < used; ++i)
        if (done[i].kernel == kernel && done[i].device == dev) return cudaSuccess;
    int optin = 0;
    e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, optin);
    if (e == cudaSuccess && used < 256) done[used++] = Entry{kernel, dev};
    return e;
}

template <typename Dec>
cudaError_t plan_t(int rows, int width, int tile_rows, int tokens, StreamPlan *p)
{
    StreamPlan q{};
    q.rows = rows;
    q.nb = width / 256;
    q.block_bytes = Dec::kBytes;
    q.tile_rows = tile_rows;
    q.tiles = (rows + tile_rows - 1) / tile_rows;
    q.rows_pad = q.tiles * tile_rows;
    q.units = static_cast<long long>(q.tiles) * q.nb;
    if (q.units >= (1LL << 31)) return cudaErrorInvalidValue;
    // tokens per launch: the activation columns of a launch fit kActBudget
    int tg = 8;
    while (tg > 1 && static_cast<size_t>(tg) * q.nb * sizeof(Act) > kActBudget) tg >>= 1;
    q.token_group = std::min(tg, tokens);
    q.mt = 1;
    while (q.mt < q.token_group) q.mt <<= 1;
    // Shape-only structure (identical for every token count):
    const int sms = device_sm_count();
    const int row_threads = (tile_rows + 31) / 32 * 32;
    q.groups = std::max(1, std::min(q.nb, kMaxConsumers / row_threads));
    const int env_groups = env_knob("Q38CU_STREAM_GROUPS", 0);
    if (env_groups > 0) q.groups = std::max(1, std::min({q.nb, env_groups, kMaxConsumers / row_threads}));
    const size_t unit_bytes = static_cast<size_t>(tile_rows) * q.block_bytes;
    // Chunk (units per bulk copy; decides which columns each group sums, so
    // shape-only): the groups' stages of one ring pass share kChunkBudget.
    q.chunk = static_cast<int>(std::max<size_t>(1, kChunkBudget / (unit_bytes * q.groups)));
    const int env_chunk = env_knob("Q38CU_STREAM_CHUNK", 0);
    if (env_chunk > 0) q.chunk = env_chunk;
    q.chunk = std::max(1, std::min(q.chunk, q.nb));
    q.stage_bytes = static_cast<uint32_t>((q.chunk * unit_bytes + 16 + 15) / 16 * 16);  // +16: decoder over-read
    // Threads per superblock (no effect on the arithmetic: a superblock's
    // integer sums are exact however they are split).  One token per launch
    // takes as many as the CTA bound allows, so that enough warps decode.
    q.parts = 1;
    q.group_threads = row_threads;
    // Split only Q6_K tiles whose height leaves lanes of a whole-warp group
    // idle (measured: splitting costs more than it gains elsewhere, and a
    // split CTA holds too many registers for the next launch's CTA to be
    // resident beside it).  Q38CU_STREAM_PARTS=n overrides the choice (1: off).
    int max_parts = env_knob("Q38CU_STREAM_PARTS", 0);
    if (max_parts <= 0) max_parts = std::is_same<Dec, DecQ6K>::value && tile_rows % 32 != 0 ? 4 : 1;
    if (q.mt == 1 && SplitParts<Dec>::kMax > 1 && max_parts > 1) {
        for (int parts = std::min(4, SplitParts<Dec>::kMax); parts > 1; parts >>= 1) {
            const int gt = (tile_rows * parts + 31) / 32 * 32;
            if (parts <= max_parts && q.groups * gt + 32 <= StreamThreads<1, 4>::kValue) {
                q.parts = parts;
                q.group_threads = gt;
                break;
            }
        }
    }
    q.threads = q.groups * q.group_threads + 32;
    q.grid = q.tiles <= sms ? q.tiles : sms;
    const int env_grid = env_knob("Q38CU_STREAM_GRID", 0);
    if (env_grid > 0) q.grid = static_cast<int>(std::min<long long>(q.units, env_grid));
    // Ring depth (no effect on the arithmetic).  A short launch keeps its CTA
    // under half of an SM's shared memory, so that shared memory does not keep
    // the next launch of the stream (programmatic dependent launch) from being
    // resident beside it; a long launch takes what it can.  (At 128 registers
    // per thread the register file still does: two CTAs of 288 threads need
    // 72 K registers.)
    int optin = 0, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (optin <= 0) optin = 227 * 1024;
    const size_t cta_bytes = static_cast<size_t>((q.units + q.grid - 1) / q.grid) * unit_bytes;
    size_t budget = static_cast<size_t>(optin);
    const int env_budget = env_knob("Q38CU_STREAM_SMEM_KB", 0);
    if (env_budget > 0) budget = std::min(budget, static_cast<size_t>(env_budget) * 1024);
    else if (cta_bytes < kLongLaunchBytes) budget = std::min(budget, kOverlapSmem);
    StreamPlan no_stages = q;
    no_stages.stages = 0;
    const size_t fixed = stream_smem<Dec>(no_stages);
    const size_t ring_pass = static_cast<size_t>(q.groups) * q.stage_bytes;
    if (fixed + 2 * ring_pass > budget && env_budget <= 0) budget = static_cast<size_t>(optin);  // too tight to share
    if (fixed >= budget) return cudaErrorInvalidConfiguration;
    q.stages = static_cast<int>(std::min<size_t>(kStreamMaxStages / q.groups, (budget - fixed) / ring_pass));
    const int env_stages = env_knob("Q38CU_STREAM_STAGES", 0);
    if (env_stages > 0) q.stages = std::min(q.stages, env_stages);
    if (q.stages < 1) return cudaErrorInvalidConfiguration;
    // deposits per shared tile
    int max_slots = 1;
    for (int t = 0; t < q.tiles; ++t) {
        const long long tu = static_cast<long long>(t) * q.nb;
        const int n = cta_of_unit(tu + q.nb - 1, q.units, q.grid) - cta_of_unit(tu, q.units, q.grid) + 1;
        max_slots = std::max(max_slots, n);
    }
    q.max_slots = max_slots;
    // scratch = [tile counters, fixed position for the tensor][deposits]
    q.counter_bytes = (static_cast<uint64_t>(q.tiles) * sizeof(int) + 255) / 256 * 256;
    q.scratch_bytes = q.counter_bytes + static_cast<uint64_t>(q.tiles) * max_slots * q.mt * tile_rows * sizeof(float);
    *p = q;
    return cudaSuccess;
}

template <typename Dec>
cudaError_t launch_t(const StreamPlan &p, const StreamLaunch &l, cudaStream_t stream)
{
    StreamArgs g;
    g.weights = static_cast<const uint8_t *>(l.weights);
    g.block_bytes = p.block_bytes;
    g.rows = p.rows;
    g.nb = p.nb;
    g.tile_rows = p.tile_rows;
    g.tiles = p.tiles;
    g.units = static_cast<int>(p.units);
    g.groups = p.groups;
    g.parts = p.parts;
    g.group_threads = p.group_threads;
    g.stages = p.stages;
    g.chunk = p.chunk;
    g.stage_bytes = p.stage_bytes;
    g.act = static_cast<const Q8KBlock *>(l.act);
    g.tokens = l.tokens;
    g.out = l.out;
    g.out_ld = l.out_ld ? l.out_ld : p.rows;
    g.accumulate = l.accumulate;
    g.act_mode = l.act_mode;
    g.act_x = l.act_x;
    g.act_y = l.act_y;
    g.act_ld = l.act_ld;
    g.act_f_out = l.act_f_out;
    g.act_reps = l.act_reps > 1 ? l.act_reps : 1;
    g.act_rep_bytes = l.act_rep_bytes;
    g.act_y_rep_bytes = l.act_y_rep_bytes;
    g.out_reps = l.out_reps > 1 ? l.out_reps : 1;
    g.out_rep_bytes = l.out_rep_bytes;
    g.nx_weights = static_cast<const uint8_t *>(l.nx_weights);
    g.nx_units = l.nx_units;
    g.nx_grid = l.nx_grid;
    g.nx_unit_bytes = l.nx_unit_bytes;
    g.nx_cta_bytes = l.nx_cta_bytes;
    g.sw_act = l.sw_act;
    g.sw_q8 = static_cast<Q8KBlock *>(l.sw_q8);
    g.sw_counters = l.sw_counters;
    g.sw_width = p.rows / 2;
    g.sw_q_reps = l.sw_q_reps > 1 ? l.sw_q_reps : 1;
    g.sw_q_rep_bytes = l.sw_q_rep_bytes;
    if (l.sw_act && (p.tile_rows != 256 || p.tiles > p.grid || p.rows % 512)) return cudaErrorInvalidValue;
    g.counters = static_cast<int *>(l.scratch);
    g.partials = reinterpret_cast<float *>(static_cast<uint8_t *>(l.scratch) + p.counter_bytes);
    g.max_slots = p.max_slots;
    g.dbg_w = l.dbg_w;
    g.dbg_x = l.dbg_x;
    g.trace = l.trace;
    g.side_w = static_cast<const uint8_t *>(l.side_w);
    g.side_rows = l.side_w ? l.side_rows : 0;
    g.side_ld = l.side_ld;
    g.side_out = l.side_out;
    g.act_export = static_cast<Q8KBlock *>(l.act_export);
    g.export_reps = l.act_export ? std::max(1, l.export_reps) : 0;
    g.export_rep_bytes = l.export_rep_bytes;
    if (l.act_export && g.export_reps > p.grid) return cudaErrorInvalidValue;
    if (l.side_w && (l.act_mode != kActRmsNorm || l.side_rows > p.grid)) return cudaErrorInvalidValue;
    g.xc_world = l.xc_world > 1 ? l.xc_world : 0;
    g.xc_rank = l.xc_rank;
    for (int r = 0; r < kXcMaxWorld; ++r) g.xc_bufs[r] = r < g.xc_world ? l.xc_bufs[r] : nullptr;
    g.xc_counter = l.xc_counter;
    // the exchange waits on the peers' CTAs inside the kernel: every CTA must
    // be resident at once (one per SM)
    if (g.xc_world > 1 &&
        (g.xc_world > kXcMaxWorld || l.xc_rank < 0 || l.xc_rank >= g.xc_world || !l.xc_counter ||
         l.tokens > kXcTokens || p.rows > l.xc_rows || p.grid > device_sm_count() || l.sw_act))
        return cudaErrorInvalidValue;
    const void *kernel = select_kernel<Dec>(p.mt, l.dbg_w != nullptr, p.parts);
    if (!kernel) return cudaErrorInvalidValue;
    cudaError_t e = opt_in(kernel);
    if (e != cudaSuccess) return e;

    // The warm-up warp serves the single-token fused RMSNorm prologue, when
    // the kernel's thread bound leaves room for it (Q38CU_WARM_WARP=0: off).
    // Measured on the decode step: the prologue's quantize step 0.3-1.1 us
    // shorter, 193.2 vs 192.2 tok/s.
    static const int warm_knob = env_knob("Q38CU_WARM_WARP", 1);
    const int max_threads = p.parts > 1 ? StreamThreads<1, 4>::kValue
                                        : (p.mt <= 2 ? StreamThreads<1, 1>::kValue : StreamThreads<4, 1>::kValue);
    g.warm_warp = warm_knob && l.act_mode == kActRmsNorm && p.mt == 1 && p.threads + 32 <= max_threads ? 1 : 0;

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.grid);
    cfg.blockDim = dim3(p.threads + 32 * g.warm_warp);
    cfg.dynamicSmemBytes = stream_smem<Dec>(p);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = env_knob("Q38CU_NO_PDL", 0) ? 0 : 1;
    void *args[] = {&g};
    return cudaLaunchKernelExC(&cfg, kernel, args);
}

}  // namespace

int stream_tile_rows(int rows)
{
    const int env_tile = env_knob("Q38CU_STREAM_TILE", 0);
    if (env_tile > 0) return std::max(8, std::min(256, env_tile / 8 * 8));
    // the smallest multiple of 8 that gives at most one tile per SM
    const int sms = device_sm_count();
    const int per_sm = (rows + sms - 1) / sms;
    return std::max(8, std::min(256, (per_sm + 7) / 8 * 8));
}

cudaError_t stream_plan(int type, int rows, int width, int tile_rows, int tokens, StreamPlan *p)
{
    switch (type) {
    case kQ4_K: return plan_t<DecQ4K>(rows, width, tile_rows, tokens, p);
    case kQ6_K: return plan_t<DecQ6K>(rows, width, tile_rows, tokens, p);
    case kIQ2_S: return plan_t<DecIQ2S>(rows, width, tile_rows, tokens, p);
    case kIQ1_S: return plan_t<DecIQ1S>(rows, width, tile_rows, tokens, p);
    case kIQ1_M: return plan_t<DecIQ1M>(rows, width, tile_rows, tokens, p);
    case kQ2_K: return plan_t<DecQ2K>(rows, width, tile_rows, tokens, p);
    case kQ3_K: return plan_t<DecQ3K>(rows, width, tile_rows, tokens, p);
    case kQ5_K: return plan_t<DecQ5K>(rows, width, tile_rows, tokens, p);
    case kIQ2_XXS: return plan_t<DecIQ2XXS>(rows, width, tile_rows, tokens, p);
    case kIQ2_XS: return plan_t<DecIQ2XS>(rows, width, tile_rows, tokens, p);
    case kIQ3_XXS: return plan_t<DecIQ3XXS>(rows, width, tile_rows, tokens, p);
    case kIQ3_S: return plan_t<DecIQ3S>(rows, width, tile_rows, tokens, p);
    case kIQ4_XS: return plan_t<DecIQ4XS>(rows, width, tile_rows, tokens, p);
    default: return cudaErrorInvalidValue;
    }
}

// The fused RMSNorm prologue of stage_fused_activation, as a kernel of its
// own: CTA (0, t) forms token t's Q8_K blocks and floats, CTA (1 + r, t) the
// side row r.  Warp w takes blocks w, w + warps, ... and lane l elements
// 8l .. 8l + 7 of each; every sum runs in the prologue's order.
__global__ void __launch_bounds__(1024) rms_prologue_kernel(RmsPrologue a)
{
    __shared__ double red_d[32];
    __shared__ float red_f[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
    const int tok = blockIdx.y, nb = a.width / 256;
    const int per_warp = (nb + warps - 1) / warps;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const float *x = a.x + static_cast<size_t>(tok) * a.ld;
    double part = 0.0;
    for (int j = 0; j < per_warp; ++j) {
        const int b = warp + j * warps;
        if (b >= nb) break;
        float xv[8];
        load8(x + b * 256 + lane * 8, xv);
#pragma unroll
        for (int i = 0; i < 8; ++i) part += static_cast<double>(__fmul_rn(xv[i], xv[i]));
    }
    part = act_warp_sum_d(part);
    if (lane == 0) red_d[warp] = part;
    __syncthreads();
    double sum = 0.0;
    for (int w = 0; w < warps; ++w) sum += red_d[w];
    const float mean = static_cast<float>(sum / static_cast<double>(nb * 256));
    const float scale = __fdiv_rn(1.0f, sqrtf(__fadd_rn(mean, kRmsEps)));
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int row = static_cast<int>(blockIdx.x) - 1;
    const uint8_t *side_row = row >= 0 ? static_cast<const uint8_t *>(a.side_w) + static_cast<size_t>(row) * nb * 8 * 34
                                       : nullptr;
    float side_acc = 0.0f;
    for (int j = 0; j < per_warp; ++j) {
        const int b = warp + j * warps;
        if (b >= nb) break;
        float xv[8], wv[8], v[8];
        load8(x + b * 256 + lane * 8, xv);
        ldg8(a.w + b * 256 + lane * 8, wv);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(__fmul_rn(xv[i], scale), wv[i]);
        if (row < 0) {
            if (a.out_f) {
                float *o = a.out_f + static_cast<size_t>(tok) * a.f_ld + b * 256 + lane * 8;
                *reinterpret_cast<float4 *>(o) = make_float4(v[0], v[1], v[2], v[3]);
                *reinterpret_cast<float4 *>(o + 4) = make_float4(v[4], v[5], v[6], v[7]);
            }
            const WarpQ8K r = act_quantize_warp(v);
            for (int k = 0; k < a.q_reps; ++k) {
                Q8KBlock *d = reinterpret_cast<Q8KBlock *>(static_cast<char *>(a.out_q) + k * a.q_rep_bytes) +
                              static_cast<size_t>(tok) * nb + b;
                uint32_t *q = reinterpret_cast<uint32_t *>(d->quants);
                q[lane * 2] = r.q0;
                q[lane * 2 + 1] = r.q1;
                if ((lane & 3) == 0) reinterpret_cast<uint32_t *>(d->sums)[lane >> 2] = r.sums_word;
                if (lane == 0) d->scale = r.scale;
            }
        } else {
            const uint8_t *blk = side_row + static_cast<size_t>(b * 8 + (lane >> 2)) * 34;
            const unsigned short *h = reinterpret_cast<const unsigned short *>(blk);
            const unsigned short *qp = reinterpret_cast<const unsigned short *>(blk + 2 + (lane & 3) * 8);
            const float sd = __half2float(__ushort_as_half(__ldg(h)));
            const uint32_t sq[2] = {static_cast<uint32_t>(__ldg(qp)) | static_cast<uint32_t>(__ldg(qp + 1)) << 16,
                                    static_cast<uint32_t>(__ldg(qp + 2)) | static_cast<uint32_t>(__ldg(qp + 3)) << 16};
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int qv = static_cast<int8_t>((sq[i >> 2] >> (8 * (i & 3))) & 0xFFu);
                side_acc = fmaf(__fmul_rn(sd, static_cast<float>(qv)), v[i], side_acc);
            }
        }
    }
    if (row < 0) return;
    const float r = act_warp_sum_f(side_acc);
    if (lane == 0) red_f[warp] = r;
    __syncthreads();
    if (threadIdx.x == 0) {
        float total = 0.0f;
        for (int w = 0; w < warps; ++w) total = __fadd_rn(total, red_f[w]);
        a.side_out[static_cast<size_t>(tok) * a.side_ld + row] = total;
    }
}

cudaError_t launch_rms_prologue(const RmsPrologue &a, cudaStream_t s)
{
    if (a.width % 256 || a.tokens < 1 || a.warps < 1 || a.warps > 32 || a.q_reps < 1 || (a.side_w && !a.side_out))
        return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1 + (a.side_w ? a.side_rows : 0), a.tokens);
    cfg.blockDim = dim3(a.warps * 32);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, rms_prologue_kernel, a);
}

int stream_consumer_warps(const StreamPlan &p) { return (p.threads - 32) / 32; }

cudaError_t launch_stream_gemm(int type, const StreamPlan &p, const StreamLaunch &l, cudaStream_t s)
{
    switch (type) {
    case kQ4_K: return launch_t<DecQ4K>(p, l, s);
    case kQ6_K: return launch_t<DecQ6K>(p, l, s);
    case kIQ2_S: return launch_t<DecIQ2S>(p, l, s);
    case kIQ1_S: return launch_t<DecIQ1S>(p, l, s);
    case kIQ1_M: return launch_t<DecIQ1M>(p, l, s);
    case kQ2_K: return launch_t<DecQ2K>(p, l, s);
    case kQ3_K: return launch_t<DecQ3K>(p, l, s);
    case kQ5_K: return launch_t<DecQ5K>(p, l, s);
    case kIQ2_XXS: return launch_t<DecIQ2XXS>(p, l, s);
    case kIQ2_XS: return launch_t<DecIQ2XS>(p, l, s);
    case kIQ3_XXS: return launch_t<DecIQ3XXS>(p, l, s);
    case kIQ3_S: return launch_t<DecIQ3S>(p, l, s);
    case kIQ4_XS: return launch_t<DecIQ4XS>(p, l, s);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t read_and_clear_stream_status(int *status)
{
    cudaError_t e = cudaMemcpyFromSymbol(status, g_stream_status, sizeof(int));
    if (e != cudaSuccess) return e;
    const int zero = 0;
    return cudaMemcpyToSymbol(g_stream_status, &zero, sizeof(int));
}

cudaError_t launch_repack_tiled(void *dst, const void *src, uint64_t rows, uint64_t nb, uint32_t tile_rows,
                                uint32_t block_bytes, cudaStream_t s)
{
    const uint64_t total = rows * nb * block_bytes;
    if (!total) return cudaSuccess;
    const unsigned grid = static_cast<unsigned>(std::min<uint64_t>((total + 255) / 256, 65535ull * 16));
    repack_tiled_kernel<<<grid, 256, 0, s>>>(static_cast<uint8_t *>(dst), static_cast<const uint8_t *>(src), rows, nb,
                                             tile_rows, block_bytes);
    return cudaGetLastError();
}

}  // namespace q38
