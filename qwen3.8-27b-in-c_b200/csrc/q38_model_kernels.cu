// q38_model_kernels.cu - the decode-step kernels around the weight-streaming
// GEMV: norms and activation quantization, the Gated-DeltaNet mixer, full
// attention over the KV cache, and greedy argmax.
//
// Every kernel here is launched with programmatic dependent launch: it calls
// pdl_wait() before touching activations or state and lets its successor
// start early.  Token ids and the position come from device memory (the
// model's control block) so that one captured CUDA graph serves every step.
//
// Float semantics follow the upstream C compiled with -ffp-contract=off
// (src/qwen38/qwen38_model.c): every product and sum is rounded separately
// (__fmul_rn / __fadd_rn), except where the upstream itself uses fmaf or its
// AVX2 FMA kernels.  Reductions run as trees rather than left to right, and
// expf/logf/cosf/sinf are CUDA's (within 2 ulp of glibc's), so the results
// agree with the upstream to rounding, not bit for bit.
#include <cooperative_groups.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "q38_device.cuh"
#include "q38_act.cuh"
#include "q38_model_internal.h"
#include "q38_types.cuh"

namespace cg = cooperative_groups;

namespace q38 {

__device__ int g_model_status;

namespace {

constexpr float kRmsEps = 1e-6f;

__device__ __forceinline__ double warp_sum_d(double v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_sum_f(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}


// Sum of a double over the CTA (all threads get the result).  `red` holds one
// double per warp; the warps' partials are added in warp order.
__device__ double block_sum_d(double v, double *red)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
    v = warp_sum_d(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    double t = 0.0;
    for (int w = 0; w < warps; ++w) t += red[w];
    return t;
}

__device__ __forceinline__ float silu(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x))); }
__device__ __forceinline__ float sigmoid(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x))); }
__device__ __forceinline__ float softplus(float x) { return x > 20.0f ? x : logf(__fadd_rn(1.0f, expf(x))); }

// upstream q38_nearest_int (qwen38_quant.c:42-48)
__device__ __forceinline__ int nearest_int(float v)
{
    const float shifted = __fadd_rn(v, 12582912.0f);
    return static_cast<int>(__float_as_uint(shifted) & 0x007fffffu) - 0x00400000;
}

// Largest |v| with the smallest index among equals: the element the upstream
// quantizer's strict `>` scan keeps (qwen38_quant.c:58-65).
struct AbsMax {
    float a;
    int i;
    float v;
};

__device__ __forceinline__ AbsMax better(AbsMax x, AbsMax y)
{
    return (y.a > x.a || (y.a == x.a && y.i < x.i)) ? y : x;
}

__device__ __forceinline__ AbsMax warp_absmax(AbsMax m)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        AbsMax other;
        other.a = __shfl_xor_sync(0xffffffffu, m.a, o);
        other.i = __shfl_xor_sync(0xffffffffu, m.i, o);
        other.v = __shfl_xor_sync(0xffffffffu, m.v, o);
        m = better(m, other);
    }
    return m;
}

// KV cache elements: fp32 (the upstream's precision, qwen38_model.c:1391-1396)
// or fp16 (half the bytes a long-context step reads).  `idx` counts elements;
// a 4-element load starts on a multiple of 4.
__device__ __forceinline__ float4 kv_load4(const void *base, size_t idx, int half)
{
    if (!half) return *reinterpret_cast<const float4 *>(static_cast<const float *>(base) + idx);
    const uint2 raw = *reinterpret_cast<const uint2 *>(static_cast<const __half *>(base) + idx);
    const float2 lo = __half22float2(*reinterpret_cast<const __half2 *>(&raw.x));
    const float2 hi = __half22float2(*reinterpret_cast<const __half2 *>(&raw.y));
    return make_float4(lo.x, lo.y, hi.x, hi.y);
}

__device__ __forceinline__ void kv_store(void *base, size_t idx, float v, int half)
{
    if (half) static_cast<__half *>(base)[idx] = __float2half_rn(v);
    else static_cast<float *>(base)[idx] = v;
}

// Q8_K quantization of 256 values held one per thread by a 256-thread CTA
// (qwen38_quant.c:50-88, bit-exact): thread i owns element i.
__device__ void quantize_block_256(float v, Q8KBlock *dst, AbsMax *red, int reps = 1, long long rep_bytes = 0)
{
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    AbsMax m{fabsf(v), tid, v};
    m = warp_absmax(m);
    __syncthreads();
    if (lane == 0) red[warp] = m;
    __syncthreads();
    AbsMax best = red[0];
    for (int w = 1; w < 8; ++w) best = better(best, red[w]);
    int q = 0;
    float inverse = 0.0f;
    if (best.a != 0.0f) {
        inverse = __fdiv_rn(-127.0f, best.v);
        q = min(nearest_int(__fmul_rn(inverse, v)), 127);
    }
    int sum = q;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    for (int k = 0; k < (reps > 1 ? reps : 1); ++k) {  // the block and its replicas
        Q8KBlock *d = reinterpret_cast<Q8KBlock *>(reinterpret_cast<char *>(dst) + k * rep_bytes);
        reinterpret_cast<int8_t *>(d->quants)[tid] = static_cast<int8_t>(q);
        if ((lane & 15) == 0) d->sums[tid >> 4] = static_cast<int16_t>(sum);
        if (tid == 0) d->scale = best.a != 0.0f ? __fdiv_rn(1.0f, inverse) : 0.0f;
    }
}

// ---------------------------------------------------------------------------
// RMSNorm -> (float, Q8_K).  Grid (n / 256, tokens), 256 threads.
// qwen38_model.c:426-435 (q38_rmsnorm) followed by q38_quantize_q8_k.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) rmsnorm_quant_kernel(const float *in, int in_ld, const float *weight, int n,
                                                            float *out_f, int out_ld, Q8KBlock *out_q, int q_ld)
{
    __shared__ double red_d[8];
    __shared__ AbsMax red_m[8];
    pdl_wait();
    pdl_launch_dependents();
    const int tok = blockIdx.y;
    const float *x = in + static_cast<size_t>(tok) * in_ld;
    double part = 0.0;
    for (int i = threadIdx.x; i < n; i += 256) {
        const float v = x[i];
        part += static_cast<double>(__fmul_rn(v, v));
    }
    const double sum = block_sum_d(part, red_d);
    const float mean = static_cast<float>(sum / static_cast<double>(n));
    const float scale = __fdiv_rn(1.0f, sqrtf(__fadd_rn(mean, kRmsEps)));
    const int e = blockIdx.x * 256 + threadIdx.x;
    const float v = __fmul_rn(__fmul_rn(x[e], scale), weight[e]);
    if (out_f) out_f[static_cast<size_t>(tok) * out_ld + e] = v;
    if (out_q) quantize_block_256(v, out_q + static_cast<size_t>(tok) * q_ld + blockIdx.x, red_m);
}

// A Q8_K block from act_quantize_warp (lane l: quants 8l .. 8l + 7; lanes 4j:
// the bsums of 16-element groups 2j, 2j + 1; the scale).
__device__ __forceinline__ void store_q8k_warp(const WarpQ8K &r, Q8KBlock *dst)
{
    const int lane = threadIdx.x & 31;
    uint32_t *qw = reinterpret_cast<uint32_t *>(dst->quants);
    qw[2 * lane] = r.q0;
    qw[2 * lane + 1] = r.q1;
    if ((lane & 3) == 0) reinterpret_cast<uint32_t *>(dst->sums)[lane >> 2] = r.sums_word;
    if (lane == 0) dst->scale = r.scale;
}

// The same for prompt-sized batches: one CTA per token forms the row's sum
// of squares once (the same per-thread partials and warp order as above, so
// the same bits), then each warp quantizes whole blocks (act_quantize_warp:
// the same Q8_K bits as quantize_block_256).
__global__ void __launch_bounds__(256) rmsnorm_quant_rows_kernel(const float *in, int in_ld, const float *weight,
                                                                 int n, float *out_f, int out_ld, Q8KBlock *out_q,
                                                                 int q_ld)
{
    __shared__ double red_d[8];
    pdl_wait();
    pdl_launch_dependents();
    const int tok = blockIdx.x;
    const float *x = in + static_cast<size_t>(tok) * in_ld;
    double part = 0.0;
    for (int i = threadIdx.x; i < n; i += 256) {
        const float v = x[i];
        part += static_cast<double>(__fmul_rn(v, v));
    }
    const double sum = block_sum_d(part, red_d);
    const float mean = static_cast<float>(sum / static_cast<double>(n));
    const float scale = __fdiv_rn(1.0f, sqrtf(__fadd_rn(mean, kRmsEps)));
    // warp w quantizes blocks w, w + 8, ...; lane l holds elements 8l .. 8l + 7
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int b = warp; b < n / 256; b += 8) {
        const int e0 = b * 256 + lane * 8;
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; i += 4) {
            const float4 xv = *reinterpret_cast<const float4 *>(x + e0 + i);
            const float4 wv = *reinterpret_cast<const float4 *>(weight + e0 + i);
            v[i] = __fmul_rn(__fmul_rn(xv.x, scale), wv.x);
            v[i + 1] = __fmul_rn(__fmul_rn(xv.y, scale), wv.y);
            v[i + 2] = __fmul_rn(__fmul_rn(xv.z, scale), wv.z);
            v[i + 3] = __fmul_rn(__fmul_rn(xv.w, scale), wv.w);
        }
        if (out_f) {
            float *of = out_f + static_cast<size_t>(tok) * out_ld + e0;
            *reinterpret_cast<float4 *>(of) = make_float4(v[0], v[1], v[2], v[3]);
            *reinterpret_cast<float4 *>(of + 4) = make_float4(v[4], v[5], v[6], v[7]);
        }
        if (out_q) store_q8k_warp(act_quantize_warp(v), out_q + static_cast<size_t>(tok) * q_ld + b);
    }
}

// ---------------------------------------------------------------------------
// SwiGLU -> (float, Q8_K).  gate_up[tok] = [gate n | up n] at stride ld.
// qwen38_model.c:523-541 (scalar q38_swiglu) followed by q38_quantize_q8_k.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) swiglu_quant_kernel(const float *gate, const float *up, int ld, int n,
                                                           float *out_f, Q8KBlock *out_q)
{
    __shared__ AbsMax red_m[8];
    pdl_wait();
    pdl_launch_dependents();
    const int tok = blockIdx.y;
    const int e = blockIdx.x * 256 + threadIdx.x;
    const float g = gate[static_cast<size_t>(tok) * ld + e];
    const float u = up[static_cast<size_t>(tok) * ld + e];
    const float v = __fmul_rn(silu(g), u);
    if (out_f) out_f[static_cast<size_t>(tok) * n + e] = v;
    quantize_block_256(v, out_q + static_cast<size_t>(tok) * (n / 256) + blockIdx.x, red_m);
}

// The same for prompt-sized batches: one warp per (token, block), lane l
// holding elements 8l .. 8l + 7 (act_quantize_warp: the same Q8_K bits).
__global__ void __launch_bounds__(256) swiglu_quant_warp_kernel(const float *gate, const float *up, int ld, int n,
                                                                int tokens, float *out_f, Q8KBlock *out_q)
{
    pdl_wait();
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int nb = n / 256;
    const long long gw = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    if (gw >= static_cast<long long>(tokens) * nb) return;
    const int tok = static_cast<int>(gw / nb), b = static_cast<int>(gw % nb);
    const size_t o = static_cast<size_t>(tok) * ld + b * 256 + lane * 8;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; i += 4) {
        const float4 g = *reinterpret_cast<const float4 *>(gate + o + i);
        const float4 u = *reinterpret_cast<const float4 *>(up + o + i);
        v[i] = __fmul_rn(silu(g.x), u.x);
        v[i + 1] = __fmul_rn(silu(g.y), u.y);
        v[i + 2] = __fmul_rn(silu(g.z), u.z);
        v[i + 3] = __fmul_rn(silu(g.w), u.w);
    }
    if (out_f) {
        float *of = out_f + static_cast<size_t>(tok) * n + b * 256 + lane * 8;
        *reinterpret_cast<float4 *>(of) = make_float4(v[0], v[1], v[2], v[3]);
        *reinterpret_cast<float4 *>(of + 4) = make_float4(v[4], v[5], v[6], v[7]);
    }
    store_q8k_warp(act_quantize_warp(v), out_q + static_cast<size_t>(tok) * nb + b);
}

// ---------------------------------------------------------------------------
// out[tok][i] += branch[tok][i]  (the residual add, for float-path projections)
// ---------------------------------------------------------------------------
__global__ void add_kernel(float *out, const float *branch, int n)
{
    pdl_wait();
    pdl_launch_dependents();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const size_t o = static_cast<size_t>(blockIdx.y) * n + i;
    if (i < n) out[o] = __fadd_rn(out[o], branch[o]);
}

// hidden[t][i] += branch[t][i] (one rounding, as upstream), stored into copy 0
// and the replicas of the hidden rows.
__global__ void add_replicated_kernel(float *hidden, const float *branch, int n, int reps, long long rep_floats)
{
    pdl_wait();
    pdl_launch_dependents();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const size_t o = static_cast<size_t>(blockIdx.y) * n + i;
    const float v = __fadd_rn(hidden[o], branch[o]);
    for (int k = 0; k < reps; ++k) hidden[o + k * rep_floats] = v;
}

// ---------------------------------------------------------------------------
// Gated-DeltaNet step (qwen38_model.c:715-792), one token after another for
// `tokens` tokens at positions base .. base + tokens - 1.
//
// Grid: 24 clusters of 8 CTAs, 128 threads each.  Cluster c covers value
// heads 2c and 2c + 1 (= Q8_K block c of the 6144-wide output); CTA rank r
// covers head 2c + r / 4, value columns [32 (r % 4), 32 (r % 4) + 32).  Each
// CTA recomputes the causal conv, SiLU and L2 norm of its key head's q and k
// (key head = value head % 16), keeps its 32 columns of the 128 x 128 state
// private, and exchanges through distributed shared memory only the per-head
// sum of squares (the head RMSNorm) and the block's absolute maximum (Q8_K).
//
// Conv state is a 16-slot ring per channel: the input of position p lives in
// slot p % 16.  Taps of positions before `base` come from the ring, taps of
// this launch's tokens straight from their projections, and each channel's
// ring is written by one CTA only (q/k channels by the quarter-0 CTA of value
// heads 0..15).  A launch writes positions >= base and reads positions in
// [base - 3, base), so with at most 8 tokens the two never share a slot.
// ---------------------------------------------------------------------------
constexpr int kDeltaCluster = 8;
constexpr int kConvRing = 16;

struct __align__(16) DeltaShared {
    float q[128], k[128];
    float v[32], o[32];
    double red[4][2];
    double ss[4];
    float ba_part[4];
    float beta, decay;
    double head_part;   // exchanged: this CTA's sum of squares
    AbsMax block_part;  // exchanged: this CTA's absolute maximum
};

// The four conv inputs of one channel at position pos (taps pos-3 .. pos-1
// and the new input) and its kernel, loaded together: a tap before `base`
// comes from the ring, later ones from this launch's projections, chosen by
// address so the loads do not wait on one another.
struct ConvTaps {
    float t0, t1, t2, x;
};

__device__ __forceinline__ const float *conv_tap_ptr(const DeltaArgs &a, int ch, int p, int base)
{
    return p >= base ? a.qkvz + static_cast<size_t>(p - base) * a.qkvz_ld + ch
                     : a.conv_ring + static_cast<size_t>(ch) * kConvRing + (p & (kConvRing - 1));
}

__device__ __forceinline__ ConvTaps load_taps(const DeltaArgs &a, int ch, int pos, int base)
{
    ConvTaps c;
    c.t0 = *conv_tap_ptr(a, ch, pos - 3, base);
    c.t1 = *conv_tap_ptr(a, ch, pos - 2, base);
    c.t2 = *conv_tap_ptr(a, ch, pos - 1, base);
    c.x = a.qkvz[static_cast<size_t>(pos - base) * a.qkvz_ld + ch];
    return c;
}

__device__ __forceinline__ float4 conv_kernel(const DeltaArgs &a, int ch)
{
    return __ldg(reinterpret_cast<const float4 *>(a.conv_w + static_cast<size_t>(ch) * 4));
}

// ((s0 k0 + s1 k1) + s2 k2) + x k3, then SiLU (qwen38_model.c:722-737).
__device__ __forceinline__ float conv_silu(const ConvTaps &c, const float4 w)
{
    float v = __fmul_rn(c.t0, w.x);
    v = __fadd_rn(v, __fmul_rn(c.t1, w.y));
    v = __fadd_rn(v, __fmul_rn(c.t2, w.z));
    v = __fadd_rn(v, __fmul_rn(c.x, w.w));
    return silu(v);
}

// Fused beta/alpha (upstream q38_dot_q8_0, qwen38_quant.c:496-507:
// fmaf(d * q, x, acc), on RMSNorm(hidden, attn_norm)).  Threads 0..63 form
// beta, 64..127 alpha; thread k of a row takes Q8_0 blocks k, k + 64, k + 128.
// Phase 1 loads the hidden row and the norm weights; phase 2 (after the
// caller's barrier publishes the sum of squares) writes the normed row to
// shared memory and loads the thread's Q8_0 blocks; phase 3 forms the dots.
struct BaLoads {
    float4 h[10], w[10];  // hidden row (per token), norm weights (loaded once, before the grid dependency)
};

__device__ __forceinline__ void ba_load_weights(const DeltaArgs &a, BaLoads &l)
{
    const float4 *w4 = reinterpret_cast<const float4 *>(a.attn_norm);
#pragma unroll
    for (int j = 0; j < 10; ++j) l.w[j] = __ldg(w4 + threadIdx.x + 128 * j);
}

__device__ __forceinline__ void ba_load_row(const DeltaArgs &a, int t, BaLoads &l)
{
    const float *hidden = a.reps > 1 ? reinterpret_cast<const float *>(reinterpret_cast<const char *>(a.hidden) +
                                                                       (blockIdx.x % a.reps) * a.hidden_rep_bytes)
                                     : a.hidden;
    const float4 *h4 = reinterpret_cast<const float4 *>(hidden + static_cast<size_t>(t) * 5120);
#pragma unroll
    for (int j = 0; j < 10; ++j) l.h[j] = h4[threadIdx.x + 128 * j];
}

__device__ __forceinline__ double ba_sum_squares(const BaLoads &l)
{
    double part = 0.0;
#pragma unroll
    for (int j = 0; j < 10; ++j) {
        part += static_cast<double>(__fmul_rn(l.h[j].x, l.h[j].x));
        part += static_cast<double>(__fmul_rn(l.h[j].y, l.h[j].y));
        part += static_cast<double>(__fmul_rn(l.h[j].z, l.h[j].z));
        part += static_cast<double>(__fmul_rn(l.h[j].w, l.h[j].w));
    }
    return part;
}

__device__ __forceinline__ void ba_store_normed(const BaLoads &l, float scale, float *xs)
{
    const int tid = threadIdx.x;
#pragma unroll
    for (int j = 0; j < 10; ++j) {
        float4 x;
        x.x = __fmul_rn(__fmul_rn(l.h[j].x, scale), l.w[j].x);
        x.y = __fmul_rn(__fmul_rn(l.h[j].y, scale), l.w[j].y);
        x.z = __fmul_rn(__fmul_rn(l.h[j].z, scale), l.w[j].z);
        x.w = __fmul_rn(__fmul_rn(l.h[j].w, scale), l.w[j].w);
        reinterpret_cast<float4 *>(xs)[tid + 128 * j] = x;
    }
}

struct BaBlocks {
    unsigned short raw[3][17];  // fp16 d + 32 int8 quants per 34-byte block
};

__device__ __forceinline__ void ba_load_blocks(const DeltaArgs &a, int vh, BaBlocks &b)
{
    const int tid = threadIdx.x, which = tid >> 6, k = tid & 63;
    const uint8_t *row = a.ba_w + static_cast<size_t>(which * 3 * (a.n_kh > 0 ? a.n_kh : 16) + vh) * 5440;
#pragma unroll
    for (int n = 0; n < 3; ++n) {
        const int blk = k + 64 * n;
        const unsigned short *b16 = reinterpret_cast<const unsigned short *>(row + (blk < 160 ? blk : 0) * 34);
#pragma unroll
        for (int i = 0; i < 17; ++i) b.raw[n][i] = blk < 160 ? __ldg(b16 + i) : static_cast<unsigned short>(0);
    }
}

__device__ __forceinline__ float ba_dot(const BaBlocks &b, const float *xs)
{
    const int k = threadIdx.x & 63;
    float acc = 0.0f;
#pragma unroll
    for (int n = 0; n < 3; ++n) {
        const int blk = k + 64 * n;
        if (blk >= 160) break;
        const float d = __half2float(__ushort_as_half(b.raw[n][0]));
        const float *x = xs + blk * 32;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const float q0 = static_cast<float>(static_cast<int8_t>(b.raw[n][1 + i] & 0xFF));
            const float q1 = static_cast<float>(static_cast<int8_t>(b.raw[n][1 + i] >> 8));
            acc = fmaf(__fmul_rn(d, q0), x[2 * i], acc);
            acc = fmaf(__fmul_rn(d, q1), x[2 * i + 1], acc);
        }
    }
    return acc;
}

__global__ void __cluster_dims__(kDeltaCluster, 1, 1) __launch_bounds__(128)
    deltanet_kernel(DeltaArgs a)
{
    __shared__ DeltaShared sh;
    __shared__ __align__(16) float xs[5120];  // RMSNorm(hidden) for the fused beta/alpha rows
    trace_mark(a.trace, kTraceStart);
    cg::cluster_group cluster = cg::this_cluster();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int rank = static_cast<int>(cluster.block_rank());
    const int cidx = blockIdx.x / kDeltaCluster;
    const int n_kh = a.n_kh > 0 ? a.n_kh : 16;           // key heads of this layout
    const int out_ld = n_kh * 384, out_nb = n_kh * 3 / 2;  // 6144 floats, 24 blocks for the whole model
    const int vh = 2 * cidx + rank / 4, quarter = rank & 3, kh = vh % n_kh;
    const int col0 = quarter * 32;
    const bool qk_writer = vh < n_kh && quarter == 0;
    const int ch_q = kh * 128 + tid, ch_k = n_kh * 128 + kh * 128 + tid;
    const int ch_v = 2 * n_kh * 128 + vh * 128 + col0 + (tid & 31);
    // Nothing below depends on the previous kernel, so it loads before the
    // grid-dependency wait: the weights, the control block and the recurrent
    // state (written only by launches that completed before the previous
    // kernel passed its own wait; read through L2, past this SM's L1).  The
    // warp's 8 state columns (128 floats each, 4 per lane) stay in registers
    // for all tokens of the launch and are stored once at the end.
    const float4 wq = conv_kernel(a, ch_q), wk = conv_kernel(a, ch_k), wvv = conv_kernel(a, ch_v);
    BaLoads bl;
    BaBlocks bb;
    if (a.ba_fused) {
        ba_load_weights(a, bl);
        ba_load_blocks(a, vh, bb);
    }
    const int base = __ldcg(a.ctl + 1);
    float *state = a.state + (static_cast<size_t>(vh) * 128 + col0 + warp * 8) * 128 + lane * 4;
    float4 s[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j] = __ldcg(reinterpret_cast<const float4 *>(state + j * 128));
    const float norm_wc = tid < 32 ? __ldg(a.norm_w + col0 + tid) : 0.0f;  // this lane's column of ssm_norm
    if (tid == 0) prefetch_share_l2(a.pf_ptr, a.pf_bytes);  // keeps HBM busy through this latency-bound step

    pdl_wait();
    trace_mark(a.trace, kTraceReady);

    for (int t = 0; t < a.tokens; ++t) {
        const int pos = base + t;
        // The conv inputs of q, k (the key head's 128 channels) and v (this
        // CTA's 32 channels) and the hidden row for the fused beta/alpha.
        // the gate z of this lane's output column, needed after the delta rule
        const float zc = tid < 32 ? a.qkvz[static_cast<size_t>(t) * a.qkvz_ld + a.z_off + vh * 128 + col0 + tid] : 0.0f;
        const ConvTaps cq = load_taps(a, ch_q, pos, base);
        const ConvTaps ck = load_taps(a, ch_k, pos, base);
        const ConvTaps cv = load_taps(a, ch_v, pos, base);
        if (a.ba_fused) ba_load_row(a, t, bl);
        float beta_raw = 0.0f, alpha_raw = 0.0f;
        if (!a.ba_fused && tid == 0) {
            const size_t bo = static_cast<size_t>(t) * a.ba_ld + vh;
            beta_raw = a.beta[bo];
            alpha_raw = a.alpha[bo];
        }

        // conv ring: this position's inputs, one writer per channel
        if (qk_writer) {
            a.conv_ring[static_cast<size_t>(ch_q) * kConvRing + (pos & (kConvRing - 1))] = cq.x;
            a.conv_ring[static_cast<size_t>(ch_k) * kConvRing + (pos & (kConvRing - 1))] = ck.x;
        }
        if (tid < 32) a.conv_ring[static_cast<size_t>(ch_v) * kConvRing + (pos & (kConvRing - 1))] = cv.x;

        // causal conv + SiLU, then the L2 norms of q and k (qwen38_model.c:608-614)
        const float qv = conv_silu(cq, wq), kv = conv_silu(ck, wk);
        if (tid < 32) sh.v[tid] = conv_silu(cv, wvv);
        const double pq = warp_sum_d(static_cast<double>(__fmul_rn(qv, qv)));
        const double pk = warp_sum_d(static_cast<double>(__fmul_rn(kv, kv)));
        const double ph = a.ba_fused ? warp_sum_d(ba_sum_squares(bl)) : 0.0;
        if (lane == 0) {
            sh.red[warp][0] = pq;
            sh.red[warp][1] = pk;
            sh.ss[warp] = ph;
        }
        __syncthreads();
        if (t == 0) trace_mark(a.trace, kTraceXLoaded);  // taps loaded, conv and norms reduced
        double sq = 0.0, sk = 0.0;
        for (int w = 0; w < 4; ++w) {
            sq += sh.red[w][0];
            sk += sh.red[w][1];
        }
        const float scale_q = __fdiv_rn(1.0f, fmaxf(sqrtf(static_cast<float>(sq)), kRmsEps));
        const float scale_k = __fdiv_rn(1.0f, fmaxf(sqrtf(static_cast<float>(sk)), kRmsEps));
        sh.q[tid] = __fmul_rn(qv, scale_q);
        sh.k[tid] = __fmul_rn(kv, scale_k);

        // beta and alpha (qwen38_model.c:748-752)
        if (a.ba_fused) {
            const double sum = ((sh.ss[0] + sh.ss[1]) + sh.ss[2]) + sh.ss[3];
            const float mean = static_cast<float>(sum / 5120.0);
            ba_store_normed(bl, __fdiv_rn(1.0f, sqrtf(__fadd_rn(mean, kRmsEps))), xs);
            __syncthreads();  // the normed row is complete
            const float acc = warp_sum_f(ba_dot(bb, xs));
            if (lane == 0) sh.ba_part[warp] = acc;
            __syncthreads();
            if (tid == 0) {
                beta_raw = __fadd_rn(sh.ba_part[0], sh.ba_part[1]);
                alpha_raw = __fadd_rn(sh.ba_part[2], sh.ba_part[3]);
            }
        }
        if (tid == 0) {
            sh.beta = sigmoid(beta_raw);
            sh.decay = expf(__fmul_rn(a.a[vh], softplus(__fadd_rn(alpha_raw, a.dt[vh]))));
        }
        __syncthreads();
        if (t == 0) trace_mark(a.trace, kTraceStaged);  // beta, decay ready
        // the next kernel's weight prefetch may start once this step's loads
        // are in (earlier, its bulk copies would queue ahead of them)
        if (t == a.tokens - 1) pdl_launch_dependents();

        // delta rule on this warp's 8 columns (qwen38_model.c:758-781)
        const float4 k4 = *reinterpret_cast<const float4 *>(&sh.k[lane * 4]);
        const float4 q4 = *reinterpret_cast<const float4 *>(&sh.q[lane * 4]);
        const float decay = sh.decay, beta = sh.beta;
        const float query_scale = __fdiv_rn(1.0f, sqrtf(128.0f));
        // The 8 columns are independent: their dot products reduce across the
        // warp together (one shuffle round for all 8), not one column after
        // another; every column keeps the upstream's arithmetic.
        float red[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            float4 &x = s[j];
            x.x = __fmul_rn(x.x, decay);
            x.y = __fmul_rn(x.y, decay);
            x.z = __fmul_rn(x.z, decay);
            x.w = __fmul_rn(x.w, decay);
            red[j] = fmaf(x.w, k4.w, fmaf(x.z, k4.z, fmaf(x.y, k4.y, __fmul_rn(x.x, k4.x))));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
            for (int j = 0; j < 8; ++j) red[j] = __fadd_rn(red[j], __shfl_xor_sync(0xffffffffu, red[j], o));
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            float4 &x = s[j];
            const float delta = __fmul_rn(__fsub_rn(sh.v[warp * 8 + j], red[j]), beta);
            x.x = fmaf(k4.x, delta, x.x);
            x.y = fmaf(k4.y, delta, x.y);
            x.z = fmaf(k4.z, delta, x.z);
            x.w = fmaf(k4.w, delta, x.w);
            red[j] = fmaf(x.w, q4.w, fmaf(x.z, q4.z, fmaf(x.y, q4.y, __fmul_rn(x.x, q4.x))));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
            for (int j = 0; j < 8; ++j) red[j] = __fadd_rn(red[j], __shfl_xor_sync(0xffffffffu, red[j], o));
        }
        if (lane == 0) {
#pragma unroll
            for (int j = 0; j < 8; ++j) sh.o[warp * 8 + j] = __fmul_rn(red[j], query_scale);
        }
        if (a.snap && t + 1 < a.tokens) {
            // the state after this token, kept for a speculative rollback
            float *snap = a.snap + t * a.snap_stride + (state - a.state);
#pragma unroll
            for (int j = 0; j < 8; ++j) *reinterpret_cast<float4 *>(snap + j * 128) = s[j];
        }
        __syncthreads();
        if (t == 0) trace_mark(a.trace, kTraceNormed);  // delta rule done

        // head RMSNorm across the head's 4 CTAs (qwen38_model.c:783-789)
        float o = 0.0f;
        if (tid < 32) {
            o = sh.o[tid];
            const double p = warp_sum_d(static_cast<double>(__fmul_rn(o, o)));
            if (tid == 0) sh.head_part = p;
        }
        cluster.sync();
        if (t == 0) trace_mark(a.trace, kTraceQuantized);  // head norm exchanged
        if (tid < 32) {
            // the head's 4 partial sums: one remote read per lane, added in rank order
            const double mine = lane < 4 ? cluster.map_shared_rank(&sh, (rank & ~3) + lane)->head_part : 0.0;
            double sum = __shfl_sync(0xffffffffu, mine, 0);
#pragma unroll
            for (int r = 1; r < 4; ++r) sum += __shfl_sync(0xffffffffu, mine, r);
            const float mean = static_cast<float>(sum / 128.0);
            const float scale = __fdiv_rn(1.0f, sqrtf(__fadd_rn(mean, kRmsEps)));
            const int col = col0 + tid;
            o = __fmul_rn(__fmul_rn(o, scale), norm_wc);
            o = __fmul_rn(o, silu(zc));
            if (a.out_f) a.out_f[static_cast<size_t>(t) * out_ld + vh * 128 + col] = o;
            const int e = (rank / 4) * 128 + col;  // index inside the Q8_K block
            AbsMax m = warp_absmax(AbsMax{fabsf(o), e, o});
            if (tid == 0) sh.block_part = m;
        }
        cluster.sync();
        if (t == 0) trace_mark(a.trace, kTraceFirstStaged);  // block max exchanged
        if (tid < 32) {
            // the block's 8 partial maxima: one remote read per lane, folded in rank order
            AbsMax part{0.0f, 0, 0.0f};
            if (lane < kDeltaCluster) part = cluster.map_shared_rank(&sh, lane)->block_part;
            AbsMax best{__shfl_sync(0xffffffffu, part.a, 0), __shfl_sync(0xffffffffu, part.i, 0),
                        __shfl_sync(0xffffffffu, part.v, 0)};
#pragma unroll
            for (int r = 1; r < kDeltaCluster; ++r)
                best = better(best, AbsMax{__shfl_sync(0xffffffffu, part.a, r), __shfl_sync(0xffffffffu, part.i, r),
                                           __shfl_sync(0xffffffffu, part.v, r)});
            Q8KBlock *dst = static_cast<Q8KBlock *>(a.out_q) + static_cast<size_t>(t) * out_nb + cidx;
            int q = 0;
            float inverse = 0.0f;
            if (best.a != 0.0f) {
                inverse = __fdiv_rn(-127.0f, best.v);
                q = min(nearest_int(__fmul_rn(inverse, o)), 127);
            }
            const int e = (rank / 4) * 128 + col0 + tid;
            int sum = q;
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
            const int reps = a.reps > 1 ? a.reps : 1;
            for (int k = 0; k < reps; ++k) {
                Q8KBlock *d = reinterpret_cast<Q8KBlock *>(reinterpret_cast<char *>(dst) + k * a.q_rep_bytes);
                reinterpret_cast<int8_t *>(d->quants)[e] = static_cast<int8_t>(q);
                if ((tid & 15) == 0) d->sums[e >> 4] = static_cast<int16_t>(sum);
                if (rank == 0 && tid == 0) d->scale = best.a != 0.0f ? __fdiv_rn(1.0f, inverse) : 0.0f;
            }
        }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) *reinterpret_cast<float4 *>(state + j * 128) = s[j];
    cluster.sync();  // peers may still read this CTA's exchange slots
    trace_mark(a.trace, kTraceEnd);
}

// ---------------------------------------------------------------------------
// Gated-DeltaNet over a whole prefill chunk (qwen38_model.c:715-792 for each
// token of the chunk in order, as q38_batch_layer runs it, :1078-1085), in
// four launches:
//
//  1. deltanet_prefill_prep_kernel (token-parallel): everything that does not
//     depend on the recurrent state - the causal conv + SiLU of every q, k and
//     v channel, the L2 norms of q and k, beta and the decay - written as
//     records laid out for the serial kernel's bulk copies:
//       qk  [key head][token][260]    q (128), k (128), normalized; q.k; 3 pad
//       v   [value head][8][token][16] the 128 v channels, 16 per column block
//       gb  [value head][token][2]    beta, decay
//     (token stride rec_tokens, a multiple of kDeltaChunk).
//  2. deltanet_prefill_kernel (serial in tokens): each warp owns 8 columns of
//     one value head's state; lane l holds rows 32 (l / 8) .. + 31 of column
//     l % 8, in registers for the whole chunk, so a column's dot products
//     reduce over 4 lanes (2 shuffle levels).  A CTA's 2 warps share the
//     records of one 16-column block (384 CTAs: small enough that every SM
//     gets two or three), streamed into a ring of shared-memory stages by
//     cp.async.bulk kDeltaChunk tokens at a time, so the token loop reads only
//     shared memory.  It stores the raw head output (before the
//     RMSNorm).  With a = k.S and b = q.S of the state before the token, the
//     upstream's
//       S <- decay S;  kv = k.S;  delta = (v - kv) beta;  S <- S + k delta;
//       out = q.S
//     is evaluated as kv = decay a, out = decay b + (q.k) delta: one
//     reduction per token (the same quantities, rounded differently: about
//     1e-7 relative).
//  3. deltanet_prefill_post_kernel: head RMSNorm, the gate, Q8_K.
//  4. deltanet_ring_store_kernel: the conv ring, once every reader is done.
// ---------------------------------------------------------------------------
constexpr int kDeltaChunk = 32;   // tokens per bulk-copy stage
constexpr int kDeltaStages = 2;
constexpr int kDeltaCols = 16;    // state columns per CTA (2 warps of 8)
constexpr int kDeltaQkLd = 260;  // floats per token of the q|k record
constexpr uint32_t kDeltaQkBytes = kDeltaChunk * kDeltaQkLd * 4, kDeltaVBytes = kDeltaChunk * kDeltaCols * 4,
                   kDeltaGbBytes = kDeltaChunk * 2 * 4;
constexpr uint32_t kDeltaStageBytes = kDeltaQkBytes + kDeltaVBytes + kDeltaGbBytes;
constexpr size_t kDeltaSmem = static_cast<size_t>(kDeltaStages) * kDeltaStageBytes + 64;

// Conv + SiLU of channels ch .. ch + 3 at position p (qwen38_model.c:722-737):
// ((x[p-3] w0 + x[p-2] w1) + x[p-1] w2) + x[p] w3, positions before 0 read 0,
// positions before the chunk read the conv ring.  The four inputs of a
// position come in one 16-byte load when the rows allow it (ch a multiple of 4).
__device__ __forceinline__ void prefill_conv4(const DeltaPrefillArgs &a, int ch, int p, float (&out)[4])
{
    float x[4][4];  // [position p - 3 + d][channel]
#pragma unroll
    for (int d = 0; d < 4; ++d) {
        const int q = p - 3 + d;
        if (q < 0) {
#pragma unroll
            for (int i = 0; i < 4; ++i) x[d][i] = 0.0f;
        } else if (q >= a.base && (a.qkvz_ld & 3) == 0) {
            const float4 v =
                *reinterpret_cast<const float4 *>(a.qkvz + static_cast<size_t>(q - a.base) * a.qkvz_ld + ch);
            x[d][0] = v.x;
            x[d][1] = v.y;
            x[d][2] = v.z;
            x[d][3] = v.w;
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i)
                x[d][i] = q >= a.base ? a.qkvz[static_cast<size_t>(q - a.base) * a.qkvz_ld + ch + i]
                                      : a.conv_ring[static_cast<size_t>(ch + i) * 16 + (q & 15)];
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float4 w = __ldg(reinterpret_cast<const float4 *>(a.conv_w) + ch + i);
        float c = __fmul_rn(x[0][i], w.x);
        c = __fadd_rn(c, __fmul_rn(x[1][i], w.y));
        c = __fadd_rn(c, __fmul_rn(x[2][i], w.z));
        out[i] = silu(__fadd_rn(c, __fmul_rn(x[3][i], w.w)));
    }
}

// One CTA of 256 threads per token; warp w takes tasks w, w + 8, ...: tasks
// 0 .. n_kh - 1 are key heads (q and k), the rest value heads (v, beta,
// decay).  Lane l holds channels 4l .. 4l + 3.
__global__ void __launch_bounds__(256) deltanet_prefill_prep_kernel(DeltaPrefillArgs a)
{
    pdl_wait();
    const int t = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int n_kh = a.n_kh > 0 ? a.n_kh : 16, n_vh = 3 * n_kh;
    const int p = a.base + t;
    const size_t rt = static_cast<size_t>(a.rec_tokens);
    float *rec_qk = a.rec, *rec_v = a.rec + static_cast<size_t>(n_kh) * rt * kDeltaQkLd,
          *rec_gb = rec_v + static_cast<size_t>(n_vh) * rt * 128;
    for (int task = warp; task < n_kh + n_vh; task += 8) {
        if (task < n_kh) {
            const int kh = task;
            const int ch_q = kh * 128 + lane * 4, ch_k = n_kh * 128 + kh * 128 + lane * 4;
            float qv[4], kv[4];
            double pq = 0.0, pk = 0.0;
            prefill_conv4(a, ch_q, p, qv);
            prefill_conv4(a, ch_k, p, kv);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                pq += static_cast<double>(__fmul_rn(qv[i], qv[i]));
                pk += static_cast<double>(__fmul_rn(kv[i], kv[i]));
            }
            // L2 norms (qwen38_model.c:608-614)
            const double sq = warp_sum_d(pq), sk = warp_sum_d(pk);
            const float scale_q = __fdiv_rn(1.0f, fmaxf(sqrtf(static_cast<float>(sq)), kRmsEps));
            const float scale_k = __fdiv_rn(1.0f, fmaxf(sqrtf(static_cast<float>(sk)), kRmsEps));
            float *dst = rec_qk + (static_cast<size_t>(kh) * rt + t) * kDeltaQkLd;
            const float4 q4 = make_float4(__fmul_rn(qv[0], scale_q), __fmul_rn(qv[1], scale_q),
                                          __fmul_rn(qv[2], scale_q), __fmul_rn(qv[3], scale_q));
            const float4 k4 = make_float4(__fmul_rn(kv[0], scale_k), __fmul_rn(kv[1], scale_k),
                                          __fmul_rn(kv[2], scale_k), __fmul_rn(kv[3], scale_k));
            reinterpret_cast<float4 *>(dst)[lane] = q4;
            reinterpret_cast<float4 *>(dst + 128)[lane] = k4;
            const float qk = warp_sum_f(fmaf(q4.w, k4.w, fmaf(q4.z, k4.z, fmaf(q4.y, k4.y, __fmul_rn(q4.x, k4.x)))));
            if (lane == 0) *reinterpret_cast<float4 *>(dst + 256) = make_float4(qk, 0.0f, 0.0f, 0.0f);
        } else {
            const int vh = task - n_kh;
            const int ch = 2 * n_kh * 128 + vh * 128 + lane * 4;
            float v[4];
            prefill_conv4(a, ch, p, v);
            // channel 4l + i sits in column block l / 4, slot 4 (l % 4) + i
            float *dst = rec_v + ((static_cast<size_t>(vh) * 8 + lane / 4) * rt + t) * kDeltaCols + (lane % 4) * 4;
            *reinterpret_cast<float4 *>(dst) = make_float4(v[0], v[1], v[2], v[3]);
            if (lane == 0) {
                // beta and the decay (qwen38_model.c:748-752)
                const float br = a.beta[static_cast<size_t>(t) * a.ba_ld + vh];
                const float ar = a.alpha[static_cast<size_t>(t) * a.ba_ld + vh];
                float2 gb;
                gb.x = sigmoid(br);
                gb.y = expf(__fmul_rn(a.a[vh], softplus(__fadd_rn(ar, a.dt[vh]))));
                reinterpret_cast<float2 *>(rec_gb)[static_cast<size_t>(vh) * rt + t] = gb;
            }
        }
    }
    pdl_launch_dependents();
}

// The serial recurrence.  Grid: value heads x 8 column blocks, 64 threads;
// thread 0 also issues the stage copies.  A stage holds kDeltaChunk tokens:
// [token][260] q|k|q.k of the head's key head, [token][16] v of the column
// block, [token][2] beta, decay.
__global__ void __launch_bounds__(64) deltanet_prefill_kernel(DeltaPrefillArgs a)
{
    extern __shared__ __align__(128) uint8_t dsm[];
    uint64_t *full = reinterpret_cast<uint64_t *>(dsm + static_cast<size_t>(kDeltaStages) * kDeltaStageBytes);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int n_kh = a.n_kh > 0 ? a.n_kh : 16, n_vh = 3 * n_kh;
    const int vh = blockIdx.x >> 3, cb = blockIdx.x & 7, col0 = cb * kDeltaCols + warp * 8;
    const int kh = vh % n_kh;
    const size_t rt = static_cast<size_t>(a.rec_tokens);
    const float *rec_qk = a.rec + static_cast<size_t>(kh) * rt * kDeltaQkLd;
    const float *rec_v = a.rec + static_cast<size_t>(n_kh) * rt * kDeltaQkLd +
                         (static_cast<size_t>(vh) * 8 + cb) * rt * kDeltaCols;
    const float *rec_gb = a.rec + static_cast<size_t>(n_kh) * rt * kDeltaQkLd + static_cast<size_t>(n_vh) * rt * 128 +
                          static_cast<size_t>(vh) * rt * 2;
    const int chunks = (a.tokens + kDeltaChunk - 1) / kDeltaChunk;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kDeltaStages; ++i) mbar_init(&full[i], 1);
        fence_mbar_init();
    }
    // this lane's state column (col0 + lane % 8), rows 32 rg .. 32 rg + 31
    const int jc = lane & 7, rg = lane >> 3;
    float *state = a.state + (static_cast<size_t>(vh) * 128 + col0 + jc) * 128 + rg * 32;
    float4 s[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j] = *reinterpret_cast<const float4 *>(state + j * 4);
    const float query_scale = __fdiv_rn(1.0f, sqrtf(128.0f));
    __syncthreads();
    pdl_wait();
    auto issue = [&](int c) {
        uint8_t *st = dsm + static_cast<size_t>(c % kDeltaStages) * kDeltaStageBytes;
        uint64_t *bar = &full[c % kDeltaStages];
        const size_t t0 = static_cast<size_t>(c) * kDeltaChunk;
        mbar_arrive_expect_tx(bar, kDeltaStageBytes);
        bulk_copy_g2s(st, rec_qk + t0 * kDeltaQkLd, kDeltaQkBytes, bar);
        bulk_copy_g2s(st + kDeltaQkBytes, rec_v + t0 * kDeltaCols, kDeltaVBytes, bar);
        bulk_copy_g2s(st + kDeltaQkBytes + kDeltaVBytes, rec_gb + t0 * 2, kDeltaGbBytes, bar);
    };
    if (threadIdx.x == 0)
        for (int c = 0; c < kDeltaStages && c < chunks; ++c) issue(c);
    int issued = min(chunks, kDeltaStages);  // chunks whose copies were issued (same in every thread)
    bool failed = false;
    for (int c = 0; c < chunks && !failed; ++c) {
        const uint8_t *st = dsm + static_cast<size_t>(c % kDeltaStages) * kDeltaStageBytes;
        const bool arrived =
            mbar_wait_bounded(&full[c % kDeltaStages], static_cast<uint32_t>(c / kDeltaStages) & 1u, &g_model_status);
        if (__syncthreads_or(!arrived)) {
            failed = true;
            break;
        }
        const float *sqk = reinterpret_cast<const float *>(st);
        const float *sv = reinterpret_cast<const float *>(st + kDeltaQkBytes);
        const float *sgb = reinterpret_cast<const float *>(st + kDeltaQkBytes + kDeltaVBytes);
        const int n = min(kDeltaChunk, a.tokens - c * kDeltaChunk);
        for (int i = 0; i < n; ++i) {
            const int t = c * kDeltaChunk + i;
            const float *rq = sqk + i * kDeltaQkLd;
            const float4 *q4 = reinterpret_cast<const float4 *>(rq + rg * 32);
            const float4 *k4 = reinterpret_cast<const float4 *>(rq + 128 + rg * 32);
            const float qk = rq[256];
            const float vj = sv[i * kDeltaCols + warp * 8 + jc];
            const float2 gb = reinterpret_cast<const float2 *>(sgb)[i];
            const float beta = gb.x, decay = gb.y;
            // k.S and q.S of the state before this token: the lane's 32 rows
            // (two chains each), then the column's 4 lanes
            float ka = 0.0f, kb = 0.0f, qa = 0.0f, qb = 0.0f;
            float4 kk[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                kk[j] = k4[j];
                const float4 qq = q4[j];
                const float4 &x = s[j];
                float &kacc = j & 1 ? kb : ka;
                float &qacc = j & 1 ? qb : qa;
                kacc = fmaf(x.w, kk[j].w, fmaf(x.z, kk[j].z, fmaf(x.y, kk[j].y, fmaf(x.x, kk[j].x, kacc))));
                qacc = fmaf(x.w, qq.w, fmaf(x.z, qq.z, fmaf(x.y, qq.y, fmaf(x.x, qq.x, qacc))));
            }
            float kd = __fadd_rn(ka, kb), qd = __fadd_rn(qa, qb);
            kd = __fadd_rn(kd, __shfl_xor_sync(0xffffffffu, kd, 8));
            qd = __fadd_rn(qd, __shfl_xor_sync(0xffffffffu, qd, 8));
            kd = __fadd_rn(kd, __shfl_xor_sync(0xffffffffu, kd, 16));
            qd = __fadd_rn(qd, __shfl_xor_sync(0xffffffffu, qd, 16));
            // delta rule on the column (qwen38_model.c:758-781)
            const float delta = __fmul_rn(__fsub_rn(vj, __fmul_rn(decay, kd)), beta);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                float4 &x = s[j];
                x.x = fmaf(kk[j].x, delta, __fmul_rn(x.x, decay));
                x.y = fmaf(kk[j].y, delta, __fmul_rn(x.y, decay));
                x.z = fmaf(kk[j].z, delta, __fmul_rn(x.z, decay));
                x.w = fmaf(kk[j].w, delta, __fmul_rn(x.w, decay));
            }
            if (rg == 0) {
                const float out = fmaf(qk, delta, __fmul_rn(decay, qd));
                a.o_raw[static_cast<size_t>(t) * a.o_ld + vh * 128 + col0 + jc] = __fmul_rn(out, query_scale);
            }
        }
        // every warp is done with this stage: refill it with chunk c + kDeltaStages
        __syncthreads();
        if (c + kDeltaStages < chunks) {
            if (threadIdx.x == 0) {
                fence_proxy_async_shared();
                issue(c + kDeltaStages);
            }
            issued = c + kDeltaStages + 1;
        }
    }
    if (failed && threadIdx.x == 0) {
        // copies still in flight land before the CTA's shared memory is released:
        // wait (bounded) for the last issued chunk of every stage
        for (int c = max(0, issued - kDeltaStages); c < issued; ++c)
            mbar_wait_bounded(&full[c % kDeltaStages], static_cast<uint32_t>(c / kDeltaStages) & 1u, nullptr);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) *reinterpret_cast<float4 *>(state + j * 4) = s[j];
    pdl_launch_dependents();
}

// Head RMSNorm (qwen38_model.c:783-789), the gate silu(z) and the Q8_K block of
// each (token, output block): one CTA of 256 threads per (block, token);
// threads 0..127 hold value head 2b, 128..255 head 2b + 1.
__global__ void __launch_bounds__(256) deltanet_prefill_post_kernel(DeltaPrefillArgs a)
{
    __shared__ double red_d[8];
    __shared__ AbsMax red_m[8];
    pdl_wait();
    const int b = blockIdx.x, t = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int col = b * 256 + tid;  // value head col / 128, column col % 128
    float o = a.o_raw[static_cast<size_t>(t) * a.o_ld + col];
    const float z = a.qkvz[static_cast<size_t>(t) * a.qkvz_ld + a.z_off + col];
    // the head's sum of squares: 4 warps per head, warp partials in order
    double part = warp_sum_d(static_cast<double>(__fmul_rn(o, o)));
    if (lane == 0) red_d[warp] = part;
    __syncthreads();
    const int h0 = (tid >> 7) * 4;
    const double sum = ((red_d[h0] + red_d[h0 + 1]) + red_d[h0 + 2]) + red_d[h0 + 3];
    const float mean = static_cast<float>(sum / 128.0);
    const float scale = __fdiv_rn(1.0f, sqrtf(__fadd_rn(mean, kRmsEps)));
    o = __fmul_rn(__fmul_rn(o, scale), a.norm_w[tid & 127]);
    o = __fmul_rn(o, silu(z));
    if (a.out_f) a.out_f[static_cast<size_t>(t) * a.o_ld + col] = o;
    quantize_block_256(o, static_cast<Q8KBlock *>(a.out_q) + static_cast<size_t>(t) * (a.o_ld / 256) + b, red_m);
    pdl_launch_dependents();
}

// The conv ring after a chunk: slot p % 16 of every channel takes the input of
// position p for the chunk's last 16 positions (those inside the chunk).
__global__ void deltanet_ring_store_kernel(DeltaPrefillArgs a, int channels)
{
    pdl_wait();
    const int ch = blockIdx.x * blockDim.x + threadIdx.x;
    if (ch < channels) {
        const int first = a.tokens > 16 ? a.tokens - 16 : 0;
        for (int t = first; t < a.tokens; ++t)
            a.conv_ring[static_cast<size_t>(ch) * 16 + ((a.base + t) & 15)] =
                a.qkvz[static_cast<size_t>(t) * a.qkvz_ld + ch];
    }
    pdl_launch_dependents();
}

// ---------------------------------------------------------------------------
// Full attention (qwen38_model.c:697-713, 816-885) for `tokens` tokens at
// positions base .. base + tokens - 1.
//
// Grid: tokens x 24 heads x kAttnSplits CTAs of 256 threads; the kAttnSplits
// CTAs of one (token, head) form a thread-block cluster.  The positions
// [0, len) of the token are cut into `active` = min(kAttnSplits, ceil(len /
// kAttnSplitPositions)) contiguous ranges, one per CTA of the cluster (the
// others only keep the cluster's barriers); the cut depends on len alone, so
// a token's result does not depend on how many tokens share the launch.
// In a CTA, warp w scores positions in groups of four (all K and V rows of a
// group loaded before any is used) and keeps a running softmax: its maximum,
// its sum of exponentials and the weighted V of its lane's 8 dimensions.  The
// warps' states merge in warp order in shared memory, the CTAs' states merge
// in rank order in the cluster's rank 0 through distributed shared memory,
// which applies the sigmoid gate and quantizes the head (one Q8_K block).
// Keys and values of this launch's own tokens are recomputed where needed
// rather than read back from the cache; CTA (t, 6g, rank 0) writes token t's
// key and value rows of KV head g into the cache, which no CTA of the launch
// reads.
// ---------------------------------------------------------------------------
constexpr int kAttnHeads = 24, kAttnDim = 256, kMaxTokens = 8;

struct AttnShared {
    float q[kAttnDim];
    float knew[kMaxTokens][kAttnDim];
    float vnew[kMaxTokens][kAttnDim];
    float tmp[kAttnDim];
    float wacc[8][kAttnDim];  // per-warp weighted values
    float wm[8], wl[8];       // per-warp running maximum and sum
    float acc[kAttnDim];      // this CTA's merged state, read by the cluster's rank 0
    float m, l;
    double red_d[8];
    float red_f[8];
    AbsMax red_m[8];
};

// Normalize (RMSNorm with `norm`) and rotate (first 64 dims, pairs (j, j + 32))
// one 256-wide head vector held one element per thread; returns the result.
__device__ float norm_rope(float x, const float *norm, int pos, float theta_scale, float *tmp, double *red)
{
    const int d = threadIdx.x;
    const double sum = block_sum_d(static_cast<double>(__fmul_rn(x, x)), red);
    const float mean = static_cast<float>(sum / 256.0);
    const float scale = __fdiv_rn(1.0f, sqrtf(__fadd_rn(mean, kRmsEps)));
    const float v = __fmul_rn(__fmul_rn(x, scale), norm[d]);
    __syncthreads();
    tmp[d] = v;
    __syncthreads();
    if (d >= 64) return v;
    const int j = d & 31;
    float theta = static_cast<float>(pos);
    for (int i = 0; i < j; ++i) theta = __fmul_rn(theta, theta_scale);
    const float c = cosf(theta), sn = sinf(theta);
    const float x0 = tmp[j], x1 = tmp[j + 32];
    return d < 32 ? __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn)) : __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
}

__device__ __forceinline__ float dot8(const float4 qa, const float4 qb, const float4 ka, const float4 kb)
{
    float part = fmaf(qa.x, ka.x, fmaf(qa.y, ka.y, fmaf(qa.z, ka.z, __fmul_rn(qa.w, ka.w))));
    return fmaf(qb.x, kb.x, fmaf(qb.y, kb.y, fmaf(qb.z, kb.z, fmaf(qb.w, kb.w, part))));
}

__device__ __forceinline__ void scale_add(float4 &acc, float c, float w, const float4 v)
{
    acc.x = fmaf(w, v.x, __fmul_rn(acc.x, c));
    acc.y = fmaf(w, v.y, __fmul_rn(acc.y, c));
    acc.z = fmaf(w, v.z, __fmul_rn(acc.z, c));
    acc.w = fmaf(w, v.w, __fmul_rn(acc.w, c));
}

__global__ void __launch_bounds__(256) attention_kernel(AttnArgs a)
{
    __shared__ AttnShared sh;
    trace_mark(a.trace, kTraceStart);
    cg::cluster_group cluster = cg::this_cluster();
    const int d = threadIdx.x, lane = d & 31, warp = d >> 5;
    const int split = static_cast<int>(cluster.block_rank());
    const int th = blockIdx.x / kAttnSplits;
    const int heads = a.heads > 0 ? a.heads : kAttnHeads;
    const int kv_ld = a.heads > 0 ? a.kv_ld : 1024, out_ld = heads * 256;
    const int h = th % heads, t = th / heads;
    const int gh = (a.heads > 0 ? a.head0 : 0) + h;                          // global query head
    const int g = gh / (kAttnHeads / 4) - (a.heads > 0 ? a.kv0 : 0);         // local KV head
    if (d == 0) prefetch_share_l2(a.pf_ptr, a.pf_bytes);  // keeps HBM busy through this latency-bound step

    pdl_wait();
    trace_mark(a.trace, kTraceReady);
    const int base = a.ctl[1];
    const int pos = base + t, len = pos + 1;
    const int active = min(kAttnSplits, (len + kAttnSplitPositions - 1) / kAttnSplitPositions);
    const int chunk = (len + active - 1) / active;
    const int p0 = min(len, split * chunk), p1 = min(len, p0 + chunk);
    const float *row = a.qkv + static_cast<size_t>(t) * a.qkv_ld;
    // one writer per KV head: the first of its query heads held here
    const bool writer = (h == 0 || gh % (kAttnHeads / 4) == 0) && split == 0;

    if (split < active) {
        const float gate = row[h * 512 + 256 + d];  // loaded with the query, used by rank 0
        // query: RMSNorm + RoPE
        const float q = norm_rope(row[h * 512 + d], a.q_norm, pos, a.theta_scale, sh.tmp, sh.red_d);
        __syncthreads();
        trace_mark(a.trace, kTraceXLoaded);  // query normalized and rotated
        sh.q[d] = q;
        // keys/values of this launch's tokens that fall in [p0, p1), and the
        // cache rows of token t (written by one CTA per KV head)
        for (int tt = 0; tt <= t; ++tt) {
            const int pp = base + tt;
            const bool needed = pp >= p0 && pp < p1;
            if (!needed && !(writer && tt == t)) continue;
            const float *r2 = a.qkv + static_cast<size_t>(tt) * a.qkv_ld;
            __syncthreads();
            const float kx = norm_rope(r2[a.k_off + g * 256 + d], a.k_norm, pp, a.theta_scale, sh.tmp, sh.red_d);
            const float vx = r2[a.v_off + g * 256 + d];
            // with an fp16 cache, this launch's own keys and values take the
            // cache's rounding too, so a token's result does not depend on
            // whether its neighbours share the launch
            sh.knew[tt][d] = a.kv_half ? __half2float(__float2half_rn(kx)) : kx;
            sh.vnew[tt][d] = a.kv_half ? __half2float(__float2half_rn(vx)) : vx;
            if (writer && tt == t) {
                kv_store(a.k_cache, static_cast<size_t>(pp) * kv_ld + g * 256 + d, kx, a.kv_half);
                kv_store(a.v_cache, static_cast<size_t>(pp) * kv_ld + g * 256 + d, vx, a.kv_half);
            }
        }
        __syncthreads();
        trace_mark(a.trace, kTraceNormed);  // this launch's keys and values ready

        // Running softmax over the warp's positions: group i covers positions
        // p0 + 32 i + 4 warp + k, k = 0..3.  Lane l holds dimensions 4l..4l+3
        // and 128 + 4l..+3 of q, of each K and V row and of the weighted sum.
        const float4 qa = *reinterpret_cast<const float4 *>(&sh.q[lane * 4]);
        const float4 qb = *reinterpret_cast<const float4 *>(&sh.q[128 + lane * 4]);
        float m_run = -INFINITY, l_run = 0.0f;
        float4 acc_a = make_float4(0.f, 0.f, 0.f, 0.f), acc_b = acc_a;
        for (int p = p0 + 4 * warp; p < p1; p += 32) {
            float4 ka[4], kb[4], va[4], vb[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int pk = min(p + k, p1 - 1);  // past the range: a valid row, masked below
                if (pk < base) {
                    const size_t row = static_cast<size_t>(pk) * kv_ld + g * 256 + lane * 4;
                    ka[k] = kv_load4(a.k_cache, row, a.kv_half);
                    kb[k] = kv_load4(a.k_cache, row + 128, a.kv_half);
                    va[k] = kv_load4(a.v_cache, row, a.kv_half);
                    vb[k] = kv_load4(a.v_cache, row + 128, a.kv_half);
                } else {
                    const float *kr = sh.knew[pk - base], *vr = sh.vnew[pk - base];
                    ka[k] = *reinterpret_cast<const float4 *>(kr + lane * 4);
                    kb[k] = *reinterpret_cast<const float4 *>(kr + 128 + lane * 4);
                    va[k] = *reinterpret_cast<const float4 *>(vr + lane * 4);
                    vb[k] = *reinterpret_cast<const float4 *>(vr + 128 + lane * 4);
                }
            }
            float sc[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) sc[k] = dot8(qa, qb, ka[k], kb[k]);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
                for (int k = 0; k < 4; ++k) sc[k] = __fadd_rn(sc[k], __shfl_xor_sync(0xffffffffu, sc[k], o));
            }
            float m_new = m_run;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                sc[k] = p + k < p1 ? __fmul_rn(sc[k], 0.0625f) : -INFINITY;  // 1 / sqrt(256)
                m_new = fmaxf(m_new, sc[k]);
            }
            const float c = expf(__fsub_rn(m_run, m_new));
            l_run = __fmul_rn(l_run, c);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float w = p + k < p1 ? expf(__fsub_rn(sc[k], m_new)) : 0.0f;
                l_run = __fadd_rn(l_run, w);
                scale_add(acc_a, k == 0 ? c : 1.0f, w, va[k]);
                scale_add(acc_b, k == 0 ? c : 1.0f, w, vb[k]);
            }
            m_run = m_new;
        }
        trace_mark(a.trace, kTraceQuantized);  // this warp's positions done
        // warps -> CTA state (warp order)
        *reinterpret_cast<float4 *>(&sh.wacc[warp][lane * 4]) = acc_a;
        *reinterpret_cast<float4 *>(&sh.wacc[warp][128 + lane * 4]) = acc_b;
        __syncthreads();
        if (lane == 0) {
            sh.wm[warp] = m_run;
            sh.wl[warp] = l_run;
        }
        __syncthreads();
        float mx = -INFINITY;
        for (int w = 0; w < 8; ++w) mx = fmaxf(mx, sh.wm[w]);
        float acc = 0.0f, l = 0.0f;
        for (int w = 0; w < 8; ++w) {
            if (sh.wm[w] == -INFINITY) continue;
            const float c = expf(__fsub_rn(sh.wm[w], mx));
            acc = fmaf(sh.wacc[w][d], c, acc);
            l = fmaf(sh.wl[w], c, l);
        }
        sh.acc[d] = acc;
        if (d == 0) {
            sh.m = mx;
            sh.l = l;
        }
        // the keys and values are read: the next kernel's weight prefetch may start
        pdl_launch_dependents();
        trace_mark(a.trace, kTraceFirstStaged);  // CTA state ready
        trace_mark(a.trace, kTraceStaged);
        cluster.sync();
        if (split == 0) {
            // merge the active ranks in rank order; gate; Q8_K
            float M = -INFINITY;
            for (int r = 0; r < active; ++r) M = fmaxf(M, cluster.map_shared_rank(&sh, r)->m);
            float num = 0.0f, den = 0.0f;
            for (int r = 0; r < active; ++r) {
                const AttnShared *peer = cluster.map_shared_rank(&sh, r);
                const float mr = peer->m;
                if (mr == -INFINITY) continue;
                const float c = expf(__fsub_rn(mr, M));
                den = fmaf(peer->l, c, den);
                num = fmaf(peer->acc[d], c, num);
            }
            float o = __fdiv_rn(num, den);
            o = __fmul_rn(o, sigmoid(gate));
            if (a.out_f) a.out_f[static_cast<size_t>(t) * out_ld + h * 256 + d] = o;
            quantize_block_256(o, static_cast<Q8KBlock *>(a.out_q) + static_cast<size_t>(t) * heads + h, sh.red_m,
                               a.reps, a.q_rep_bytes);
        }
    } else {
        pdl_launch_dependents();
        cluster.sync();
    }
    cluster.sync();  // rank 0 has read every peer's state
    trace_mark(a.trace, kTraceEnd);
}

// ---------------------------------------------------------------------------
// Full attention over a whole prefill chunk (qwen38_model.c:816-885 for each
// token of the chunk): three kernels.
//  1. attn_prefill_qk_kernel: per (token, head) the query's RMSNorm + RoPE into
//     qbuf, and per (token, KV head) the key's RMSNorm + RoPE and the value into
//     the KV cache at the token's position (one CTA of 256 threads each).
//  2. attn_prefill_kernel: a CTA takes 64 consecutive query tokens of one
//     head and walks the cached positions 0 .. its last query's position in
//     tiles of 64 keys (Q, K and V rows staged in shared memory, fp32).  Thread
//     (qg, kg) of the 16 x 16 grid scores queries qg + 16i against keys
//     kg + 16j (16 fp32 dot products, dimensions in order), the scores go
//     through shared memory to a running softmax per query (4 threads a row),
//     and the thread accumulates dimensions 4kg + 64j .. + 3 of the weighted
//     values of its 4 queries; positions past a query's own are masked.  Then
//     the sigmoid gate, into out_f.  Query tiles run heaviest (latest) first.
//  3. attn_prefill_quant_kernel: the Q8_K block of each (token, head).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) attn_prefill_qk_kernel(AttnPrefillArgs a)
{
    __shared__ float tmp[kAttnDim];
    __shared__ double red[8];
    pdl_wait();
    const int t = blockIdx.y, which = blockIdx.x, d = threadIdx.x;
    const int pos = a.base + t;
    const float *row = a.qkv + static_cast<size_t>(t) * a.qkv_ld;
    if (which < a.heads) {
        const float q = norm_rope(row[which * 512 + d], a.q_norm, pos, a.theta_scale, tmp, red);
        a.qbuf[(static_cast<size_t>(t) * a.heads + which) * kAttnDim + d] = q;
    } else {
        const int g = which - a.heads;
        const float k = norm_rope(row[a.k_off + g * kAttnDim + d], a.k_norm, pos, a.theta_scale, tmp, red);
        kv_store(a.k_cache, static_cast<size_t>(pos) * a.kv_ld + g * kAttnDim + d, k, a.kv_half);
        kv_store(a.v_cache, static_cast<size_t>(pos) * a.kv_ld + g * kAttnDim + d, row[a.v_off + g * kAttnDim + d],
                 a.kv_half);
    }
    pdl_launch_dependents();
}

// ---- attn_prefill_kernel: tensor cores (mma.sync m16n8k16, fp16 in, fp32
// accumulate) on two-term operands ----
//
// Every fp32 operand x is split into hi = fp16(x) and lo = fp16(x - hi) (22
// significant bits), and a product is hi.hi + hi.lo + lo.hi (the lo.lo term is
// below 2^-22 of it): scores S = Q K^T and the weighted values P V carry the
// rounding of fp32 products with 22-bit operands, not fp16's 11 bits.  V is
// scaled by 2^-4 before the split (exact; undone at the end) so that values up
// to 2^20 stay in fp16 range.
//
// A CTA takes 64 queries of one head (8 warps); per tile of 64 keys:
//   1. all threads load the K and V rows (fp32 or fp16 cache) and split them
//      into hi/lo fp16 in shared memory (rows padded to 528 bytes: the eight
//      16-byte rows of an ldmatrix land in distinct bank groups);
//   2. warp w scores query rows 16 (w % 4) .. + 15 against keys 32 (w / 4) ..
//      + 31 (4 n-tiles of 8, 16 k-steps of 16 dimensions, 3 MMAs each);
//   3. running softmax per query row: each warp's partial row maxima and sums
//      go through shared memory so the two warps of a row agree; P (hi/lo fp16)
//      goes to shared memory;
//   4. warp w accumulates P V for rows 16 (w % 4) .. and dimensions 128 (w / 4)
//      .. + 127 (16 n-tiles, 4 k-steps of 16 keys, 3 MMAs each), after scaling
//      its accumulators by the rows' softmax correction.
// Then O / l times the sigmoid gate, into out_f.  Query tiles run latest-first.
constexpr int kPfQueries = 64, kPfKeys = 64;
constexpr int kPfRow = kAttnDim + 8;  // halves per padded Q / K / V row (528 bytes)
constexpr int kPfPRow = kPfKeys + 8;  // halves per padded P row (144 bytes)
constexpr size_t kPfTile = static_cast<size_t>(64) * kPfRow * 2;  // bytes of one hi or lo tile
constexpr size_t kPfSmem = 6 * kPfTile + 2 * static_cast<size_t>(kPfQueries) * kPfPRow * 2 +
                           4 * static_cast<size_t>(kPfQueries) * sizeof(float);
constexpr float kPfVScale = 0.0625f;  // 2^-4

__device__ __forceinline__ void split_half(float x, __half &hi, __half &lo)
{
    hi = __float2half_rn(x);
    lo = __float2half_rn(__fsub_rn(x, __half2float(hi)));
}

// Store 4 fp32 values split into the hi and lo rows at half offset `o`.
__device__ __forceinline__ void store_split4(__half *hi, __half *lo, int o, float4 v, float scale)
{
    __half h[4], l[4];
    split_half(__fmul_rn(v.x, scale), h[0], l[0]);
    split_half(__fmul_rn(v.y, scale), h[1], l[1]);
    split_half(__fmul_rn(v.z, scale), h[2], l[2]);
    split_half(__fmul_rn(v.w, scale), h[3], l[3]);
    *reinterpret_cast<uint2 *>(hi + o) = *reinterpret_cast<const uint2 *>(h);
    *reinterpret_cast<uint2 *>(lo + o) = *reinterpret_cast<const uint2 *>(l);
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4])
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&r)[4])
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

// D (16 x 8 fp32) += A (16 x 16 fp16, row) x B (16 x 8 fp16, col)
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
                 "{%8, %9}, {%0, %1, %2, %3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__global__ void __launch_bounds__(256, 1) attn_prefill_kernel(AttnPrefillArgs a)
{
    extern __shared__ __align__(128) uint8_t pf_raw[];
    __half *qh = reinterpret_cast<__half *>(pf_raw);
    __half *ql = qh + 64 * kPfRow;
    __half *kh = ql + 64 * kPfRow;
    __half *kl = kh + 64 * kPfRow;
    __half *vh = kl + 64 * kPfRow;
    __half *vl = vh + 64 * kPfRow;
    __half *ph = vl + 64 * kPfRow;
    __half *pl = ph + kPfQueries * kPfPRow;
    float *rmax = reinterpret_cast<float *>(pl + kPfQueries * kPfPRow);  // [2][64] partial row maxima
    float *rsum = rmax + 2 * kPfQueries;                                  // [2][64] partial row sums
    pdl_wait();
    const int tiles = (a.tokens + kPfQueries - 1) / kPfQueries;
    const int h = blockIdx.y, t0 = (tiles - 1 - static_cast<int>(blockIdx.x)) * kPfQueries;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, tq = lane & 3;
    const int rb = (warp & 3) * 16, half_sel = warp >> 2;  // row block; key half (scores) / dim half (P V)
    const int kvh = (a.head0 + h) / (kAttnHeads / 4) - a.kv0;
    const int last = a.base + min(t0 + kPfQueries - 1, a.tokens - 1);
    // the query tile, split (8 loads in flight per thread)
    for (int i0 = tid; i0 < kPfQueries * kAttnDim / 4; i0 += 8 * 256) {
        float4 q[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = i0 + u * 256, r = i / (kAttnDim / 4), c4 = i % (kAttnDim / 4);
            const int t = min(t0 + r, a.tokens - 1);
            q[u] = *reinterpret_cast<const float4 *>(a.qbuf + (static_cast<size_t>(t) * a.heads + h) * kAttnDim +
                                                     c4 * 4);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = i0 + u * 256, r = i / (kAttnDim / 4), c4 = i % (kAttnDim / 4);
            store_split4(qh, ql, r * kPfRow + c4 * 4, q[u], 1.0f);
        }
    }
    // this lane's two query rows (g and g + 8 of the row block) and their positions
    const int row0 = rb + g, row1 = rb + g + 8;
    const int pos0 = a.base + min(t0 + row0, a.tokens - 1), pos1 = a.base + min(t0 + row1, a.tokens - 1);
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;  // running max / sum (l: warps of half 0)
    float o[16][4];
#pragma unroll
    for (int j = 0; j < 16; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[j][e] = 0.0f;
    const uint32_t s_qh = smem_addr(qh), s_ql = smem_addr(ql), s_kh = smem_addr(kh), s_kl = smem_addr(kl);
    const uint32_t s_vh = smem_addr(vh), s_vl = smem_addr(vl), s_ph = smem_addr(ph), s_pl = smem_addr(pl);
    for (int p0 = 0; p0 <= last; p0 += kPfKeys) {
        __syncthreads();  // the previous tile's K, V and P are consumed (and Q is written)
        // 8 K and 8 V loads in flight per thread before any is converted
        for (int i0 = tid; i0 < kPfKeys * kAttnDim / 4; i0 += 8 * 256) {
            float4 kq[8], vq[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int i = i0 + u * 256, key = i / (kAttnDim / 4), d4 = i % (kAttnDim / 4);
                const int p = min(p0 + key, last);  // past `last`: a valid row, masked below
                const size_t off = static_cast<size_t>(p) * a.kv_ld + kvh * kAttnDim + d4 * 4;
                kq[u] = kv_load4(a.k_cache, off, a.kv_half);
                vq[u] = kv_load4(a.v_cache, off, a.kv_half);
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int i = i0 + u * 256, key = i / (kAttnDim / 4), d4 = i % (kAttnDim / 4);
                store_split4(kh, kl, key * kPfRow + d4 * 4, kq[u], 1.0f);
                store_split4(vh, vl, key * kPfRow + d4 * 4, vq[u], kPfVScale);
            }
        }
        __syncthreads();
        // 2. scores of rows rb .. rb + 15 against keys 32 half_sel .. + 31
        float sc[4][4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) sc[j][e] = 0.0f;
        const uint32_t a_off = static_cast<uint32_t>(((rb + (lane & 15)) * kPfRow + (lane >> 4) * 8) * 2);
        const int key_l = 32 * half_sel + (lane & 7) + ((lane >> 4) << 3);
        const uint32_t b_off = static_cast<uint32_t>((key_l * kPfRow + ((lane >> 3) & 1) * 8) * 2);
#pragma unroll 4
        for (int kk = 0; kk < kAttnDim / 16; ++kk) {
            uint32_t ah[4], al[4];
            ldsm_x4(s_qh + a_off + kk * 32, ah);
            ldsm_x4(s_ql + a_off + kk * 32, al);
#pragma unroll
            for (int jp = 0; jp < 2; ++jp) {  // n-tile pairs (16 keys)
                uint32_t bh[4], bl[4];
                const uint32_t o2 = b_off + jp * 16 * kPfRow * 2 + kk * 32;
                ldsm_x4(s_kh + o2, bh);
                ldsm_x4(s_kl + o2, bl);
                mma16816(sc[2 * jp], ah, bh[0], bh[1]);
                mma16816(sc[2 * jp], ah, bl[0], bl[1]);
                mma16816(sc[2 * jp], al, bh[0], bh[1]);
                mma16816(sc[2 * jp + 1], ah, bh[2], bh[3]);
                mma16816(sc[2 * jp + 1], ah, bl[2], bl[3]);
                mma16816(sc[2 * jp + 1], al, bh[2], bh[3]);
            }
        }
        // 3. running softmax: mask, scale, partial maxima of this warp's 32 keys
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int kp = p0 + 32 * half_sel + 8 * j + 2 * tq;  // position of column c0 / c2
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                sc[j][e] = kp + e <= pos0 ? __fmul_rn(sc[j][e], 0.0625f) : -INFINITY;
                sc[j][2 + e] = kp + e <= pos1 ? __fmul_rn(sc[j][2 + e], 0.0625f) : -INFINITY;
                mx0 = fmaxf(mx0, sc[j][e]);
                mx1 = fmaxf(mx1, sc[j][2 + e]);
            }
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        if (tq == 0) {
            rmax[half_sel * kPfQueries + row0] = mx0;
            rmax[half_sel * kPfQueries + row1] = mx1;
        }
        __syncthreads();
        const float n0 = fmaxf(m0, fmaxf(rmax[row0], rmax[kPfQueries + row0]));
        const float n1 = fmaxf(m1, fmaxf(rmax[row1], rmax[kPfQueries + row1]));
        const float c0 = m0 == -INFINITY ? 0.0f : expf(__fsub_rn(m0, n0));
        const float c1 = m1 == -INFINITY ? 0.0f : expf(__fsub_rn(m1, n1));
        float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float w[4];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                w[e] = sc[j][e] == -INFINITY ? 0.0f : expf(__fsub_rn(sc[j][e], n0));
                w[2 + e] = sc[j][2 + e] == -INFINITY ? 0.0f : expf(__fsub_rn(sc[j][2 + e], n1));
            }
            s0 = __fadd_rn(s0, __fadd_rn(w[0], w[1]));
            s1 = __fadd_rn(s1, __fadd_rn(w[2], w[3]));
            const int col = 32 * half_sel + 8 * j + 2 * tq;
            __half hh[2], hl[2];
            split_half(w[0], hh[0], hl[0]);
            split_half(w[1], hh[1], hl[1]);
            *reinterpret_cast<__half2 *>(ph + row0 * kPfPRow + col) = __halves2half2(hh[0], hh[1]);
            *reinterpret_cast<__half2 *>(pl + row0 * kPfPRow + col) = __halves2half2(hl[0], hl[1]);
            split_half(w[2], hh[0], hl[0]);
            split_half(w[3], hh[1], hl[1]);
            *reinterpret_cast<__half2 *>(ph + row1 * kPfPRow + col) = __halves2half2(hh[0], hh[1]);
            *reinterpret_cast<__half2 *>(pl + row1 * kPfPRow + col) = __halves2half2(hl[0], hl[1]);
        }
        s0 = __fadd_rn(s0, __shfl_xor_sync(0xffffffffu, s0, 1));
        s0 = __fadd_rn(s0, __shfl_xor_sync(0xffffffffu, s0, 2));
        s1 = __fadd_rn(s1, __shfl_xor_sync(0xffffffffu, s1, 1));
        s1 = __fadd_rn(s1, __shfl_xor_sync(0xffffffffu, s1, 2));
        if (tq == 0) {
            rsum[half_sel * kPfQueries + row0] = s0;
            rsum[half_sel * kPfQueries + row1] = s1;
        }
        m0 = n0;
        m1 = n1;
        __syncthreads();  // P and the partial sums are complete
        l0 = __fadd_rn(__fmul_rn(l0, c0), __fadd_rn(rsum[row0], rsum[kPfQueries + row0]));
        l1 = __fadd_rn(__fmul_rn(l1, c1), __fadd_rn(rsum[row1], rsum[kPfQueries + row1]));
        // 4. O = O c + P V for rows rb .., dimensions 128 half_sel ..
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            o[j][0] = __fmul_rn(o[j][0], c0);
            o[j][1] = __fmul_rn(o[j][1], c0);
            o[j][2] = __fmul_rn(o[j][2], c1);
            o[j][3] = __fmul_rn(o[j][3], c1);
        }
        const uint32_t pa_off = static_cast<uint32_t>(((rb + (lane & 15)) * kPfPRow + (lane >> 4) * 8) * 2);
        const int vkey = (lane & 7) + ((lane >> 3) & 1) * 8;
        const uint32_t vb_off = static_cast<uint32_t>((vkey * kPfRow + 128 * half_sel + (lane >> 4) * 8) * 2);
#pragma unroll
        for (int ks = 0; ks < kPfKeys / 16; ++ks) {
            uint32_t ah[4], al[4];
            ldsm_x4(s_ph + pa_off + ks * 32, ah);
            ldsm_x4(s_pl + pa_off + ks * 32, al);
#pragma unroll
            for (int jp = 0; jp < 8; ++jp) {  // n-tile pairs (16 dimensions)
                uint32_t bh[4], bl[4];
                const uint32_t o2 = vb_off + (ks * 16 * kPfRow + jp * 16) * 2;
                ldsm_x4_trans(s_vh + o2, bh);
                ldsm_x4_trans(s_vl + o2, bl);
                mma16816(o[2 * jp], ah, bh[0], bh[1]);
                mma16816(o[2 * jp], ah, bl[0], bl[1]);
                mma16816(o[2 * jp], al, bh[0], bh[1]);
                mma16816(o[2 * jp + 1], ah, bh[2], bh[3]);
                mma16816(o[2 * jp + 1], ah, bl[2], bl[3]);
                mma16816(o[2 * jp + 1], al, bh[2], bh[3]);
            }
        }
    }
    // O / l times the sigmoid gate (qwen38_model.c:870-878), V's 2^4 restored
    const float inv0 = __fdiv_rn(1.0f / kPfVScale, l0), inv1 = __fdiv_rn(1.0f / kPfVScale, l1);
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int t = t0 + (r ? row1 : row0);
        if (t >= a.tokens) continue;
        const float inv = r ? inv1 : inv0;
        const float *gate = a.qkv + static_cast<size_t>(t) * a.qkv_ld + h * 512 + kAttnDim;
        float *dst = a.out_f + static_cast<size_t>(t) * a.out_ld + h * kAttnDim;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const int d = 128 * half_sel + 8 * j + 2 * tq;
#pragma unroll
            for (int e = 0; e < 2; ++e)
                dst[d + e] = __fmul_rn(__fmul_rn(o[j][2 * r + e], inv), sigmoid(gate[d + e]));
        }
    }
    pdl_launch_dependents();
}

__global__ void __launch_bounds__(256) attn_prefill_quant_kernel(AttnPrefillArgs a)
{
    __shared__ AbsMax red_m[8];
    pdl_wait();
    const int h = blockIdx.x, t = blockIdx.y;
    const float v = a.out_f[static_cast<size_t>(t) * a.out_ld + h * kAttnDim + threadIdx.x];
    quantize_block_256(v, static_cast<Q8KBlock *>(a.out_q) + static_cast<size_t>(t) * a.heads + h, red_m);
    pdl_launch_dependents();
}

// ---------------------------------------------------------------------------
// The all-reduce of a row-parallel projection over peer memory (TpReduceArgs).
// CTA c owns columns [n c / C, n (c + 1) / C) of every token: it stores them to
// slot `rank` of every rank's buffer, publishes flag (rank, c) on every rank
// after a system-scope fence, waits (bounded) until every rank's flag c here
// shows this call, then adds the world slots in rank order to the hidden rows.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void st_release_sys(unsigned long long *p, unsigned long long v)
{
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *p)
{
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(128) tp_reduce_kernel(TpReduceArgs a)
{
    __shared__ unsigned long long call_s;
    __shared__ int failed_s;
    pdl_wait();
    // the next GEMV may start streaming its weights now; it waits for this
    // kernel's completion before it reads the hidden rows
    pdl_launch_dependents();
    const int c = blockIdx.x, tid = threadIdx.x;
    if (tid == 0) {
        call_s = __ldcg(a.counter);
        failed_s = 0;
    }
    __syncthreads();
    const unsigned long long call = call_s;
    const int half = static_cast<int>(call & 1);
    const int c0 = a.n * c / kTpReduceCtas, c1 = a.n * (c + 1) / kTpReduceCtas;
    const size_t slot = static_cast<size_t>(8) * a.n;                // floats of one rank's slot
    const size_t half_floats = static_cast<size_t>(a.world) * slot;  // floats of one half
    // 1. this rank's partial into slot `rank` of every rank
    for (int t = 0; t < a.tokens; ++t)
        for (int i = c0 + tid; i < c1; i += blockDim.x) {
            const float v = a.partial[static_cast<size_t>(t) * a.n + i];
            for (int r = 0; r < a.world; ++r)
                a.bufs[r][half * half_floats + a.rank * slot + static_cast<size_t>(t) * a.n + i] = v;
        }
    __syncthreads();
    // 2. publish, 3. wait for every rank's slice c of this call
    if (tid == 0) {
        __threadfence_system();
        for (int r = 0; r < a.world; ++r) st_release_sys(a.flags[r] + a.rank * kTpReduceCtas + c, call + 1);
        const unsigned long long start = global_timer_ns();
        for (int r = 0; r < a.world; ++r) {
            const unsigned long long *f = a.flags[a.rank] + r * kTpReduceCtas + c;
            while (ld_acquire_sys(f) < call + 1) {
                if (global_timer_ns() - start > kWaitLimitNs) {
                    atomicExch(&g_model_status, kStatusWaitTimeout);
                    failed_s = 1;
                    break;
                }
            }
            if (failed_s) break;
        }
    }
    __syncthreads();
    // 4. hidden += the slots in rank order (the same sum on every rank)
    if (!failed_s) {
        const float *mine = a.bufs[a.rank] + half * half_floats;
        for (int t = 0; t < a.tokens; ++t)
            for (int i = c0 + tid; i < c1; i += blockDim.x) {
                const size_t o = static_cast<size_t>(t) * a.n + i;
                float sum = __ldcg(mine + o);
                for (int r = 1; r < a.world; ++r) sum = __fadd_rn(sum, __ldcg(mine + r * slot + o));
                const float h = __fadd_rn(a.hidden[o], sum);
                for (int k = 0; k < a.reps; ++k) a.hidden[o + k * a.rep_floats] = h;
            }
    }
    // the last CTA advances the call number for the next reduction
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(a.counter + 1, 1ull) == kTpReduceCtas - 1) {
            a.counter[1] = 0;
            __threadfence();
            atomicExch(a.counter, call + 1);
        }
    }
}

// ---------------------------------------------------------------------------
// Greedy argmax over each token's logits (upstream q38_argmax: the first index
// of the maximum, qwen38_model.c:1228-1239).  Grid (kArgmaxCtas, tokens); the
// last CTA of a token merges the CTA results in order and, for the last token
// of the launch, feeds the control block: ctl[0] = token, ctl[1] += tokens,
// history[ctl[2]++] = token.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) argmax_kernel(ArgmaxArgs a)
{
    __shared__ float sv[8];
    __shared__ int si[8];
    __shared__ int last;
    trace_mark(a.trace, kTraceStart);
    pdl_wait();
    trace_mark(a.trace, kTraceReady);
    pdl_launch_dependents();
    const int tok = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float *x = a.logits + static_cast<size_t>(tok) * a.ld;
    const int per = (a.n + gridDim.x - 1) / gridDim.x;
    const int i0 = blockIdx.x * per, i1 = min(a.n, i0 + per);
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = i0 + tid; i < i1; i += 256) {
        const float v = x[i];
        if (v > best) { best = v; bi = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    if (lane == 0) { sv[warp] = best; si[warp] = bi; }
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < 8; ++w)
            if (sv[w] > best || (sv[w] == best && si[w] < bi)) { best = sv[w]; bi = si[w]; }
        a.part_v[tok * gridDim.x + blockIdx.x] = best;
        a.part_i[tok * gridDim.x + blockIdx.x] = bi;
        __threadfence();
        last = atomicAdd(&a.counters[tok], 1) == static_cast<int>(gridDim.x) - 1;
    }
    __syncthreads();
    if (!last || warp != 0) {
        trace_mark(a.trace, kTraceEnd);
        return;
    }
    __threadfence();
    // Warp 0 merges the CTA results: lane l scans CTAs l, l + 32, ... in
    // order (strict >: the earliest of equal maxima), then the lanes combine
    // with ties going to the lower index (CTA ranges are in index order).
    float bv = -INFINITY;
    int bidx = 0x7fffffff;
    for (unsigned c = lane; c < gridDim.x; c += 32) {
        const float v = __ldcg(&a.part_v[tok * gridDim.x + c]);
        const int i = __ldcg(&a.part_i[tok * gridDim.x + c]);
        if (v > bv) { bv = v; bidx = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bidx, o);
        if (ov > bv || (ov == bv && oi < bidx)) { bv = ov; bidx = oi; }
    }
    if (lane != 0) return;
    if (bidx == 0x7fffffff) bidx = 0;  // all NaN / -inf: the upstream scan keeps index 0
    a.out[tok] = static_cast<uint32_t>(bidx);
    a.counters[tok] = 0;
    trace_mark(a.trace, kTraceEnd);
    if (a.ctl && tok == static_cast<int>(gridDim.y) - 1) {
        a.ctl[0] = bidx;
        a.ctl[1] += a.advance;
        if (a.history && a.ctl[2] >= 0 && a.ctl[2] < a.history_len) a.history[a.ctl[2]++] = static_cast<uint32_t>(bidx);
    }
}

template <typename Kernel, typename... Args>
cudaError_t launch_pdl(Kernel kernel, dim3 grid, dim3 block, cudaStream_t s, Args... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

}  // namespace

cudaError_t launch_rmsnorm_quant(const float *in, int in_ld, const float *weight, int n, int tokens, float *out_f,
                                 int out_ld, void *out_q, cudaStream_t s, int q_ld)
{
    if (n % 256) return cudaErrorInvalidValue;
    if (tokens >= 64)  // a prompt: one CTA per token (same results)
        return launch_pdl(rmsnorm_quant_rows_kernel, dim3(tokens), dim3(256), s, in, in_ld, weight, n, out_f, out_ld,
                          static_cast<Q8KBlock *>(out_q), q_ld ? q_ld : n / 256);
    return launch_pdl(rmsnorm_quant_kernel, dim3(n / 256, tokens), dim3(256), s, in, in_ld, weight, n, out_f, out_ld,
                      static_cast<Q8KBlock *>(out_q), q_ld ? q_ld : n / 256);
}

cudaError_t launch_swiglu_quant(const float *gate, const float *up, int ld, int n, int tokens, float *out_f,
                                void *out_q, cudaStream_t s)
{
    if (n % 256) return cudaErrorInvalidValue;
    if (tokens >= 64 && ld % 4 == 0) {
        // a prompt: one warp per (token, block) (same results)
        const long long warps = static_cast<long long>(tokens) * (n / 256);
        return launch_pdl(swiglu_quant_warp_kernel, dim3(static_cast<unsigned>((warps + 7) / 8)), dim3(256), s, gate,
                          up, ld, n, tokens, out_f, static_cast<Q8KBlock *>(out_q));
    }
    return launch_pdl(swiglu_quant_kernel, dim3(n / 256, tokens), dim3(256), s, gate, up, ld, n, out_f,
                      static_cast<Q8KBlock *>(out_q));
}

cudaError_t launch_add_replicated(float *hidden, const float *branch, int n, int tokens, int reps,
                                  long long rep_floats, cudaStream_t s)
{
    return launch_pdl(add_replicated_kernel, dim3((n + 255) / 256, tokens), dim3(256), s, hidden, branch, n,
                      reps < 1 ? 1 : reps, rep_floats);
}

cudaError_t launch_add(float *out, const float *branch, int n, int tokens, cudaStream_t s)
{
    return launch_pdl(add_kernel, dim3((n + 255) / 256, tokens), dim3(256), s, out, branch, n);
}

cudaError_t launch_deltanet(const DeltaArgs &args, cudaStream_t s)
{
    if (args.tokens < 1 || args.tokens > kMaxTokens) return cudaErrorInvalidValue;
    const int n_kh = args.n_kh > 0 ? args.n_kh : 16;
    if (n_kh % 2 || n_kh > 16) return cudaErrorInvalidValue;
    return launch_pdl(deltanet_kernel, dim3(n_kh * 3 / 2 * kDeltaCluster), dim3(128), s, args);
}

cudaError_t launch_deltanet_prefill(const DeltaPrefillArgs &args, cudaStream_t s)
{
    const int n_kh = args.n_kh > 0 ? args.n_kh : 16;
    if (args.tokens < 1 || n_kh % 2 || n_kh > 16 || args.o_ld != n_kh * 384) return cudaErrorInvalidValue;
    const int n_vh = 3 * n_kh, channels = 5 * n_kh * 128;
    if (!args.rec || args.rec_tokens < args.tokens || args.rec_tokens % kDeltaChunk ||
        reinterpret_cast<uintptr_t>(args.rec) % 16)
        return cudaErrorInvalidValue;
    static cudaError_t attr = cudaFuncSetAttribute(deltanet_prefill_kernel,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   static_cast<int>(kDeltaSmem));
    if (attr != cudaSuccess) return attr;
    cudaError_t e = launch_pdl(deltanet_prefill_prep_kernel, dim3(args.tokens), dim3(256), s, args);
    if (e == cudaSuccess) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(n_vh * (128 / kDeltaCols));
        cfg.blockDim = dim3(64);
        cfg.dynamicSmemBytes = kDeltaSmem;
        cfg.stream = s;
        cudaLaunchAttribute pdl[1];
        pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        pdl[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = pdl;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, deltanet_prefill_kernel, args);
    }
    if (e == cudaSuccess)
        e = launch_pdl(deltanet_prefill_post_kernel, dim3(n_vh / 2, args.tokens), dim3(256), s, args);
    if (e == cudaSuccess)
        e = launch_pdl(deltanet_ring_store_kernel, dim3((channels + 127) / 128), dim3(128), s, args, channels);
    return e;
}

cudaError_t launch_attention_prefill(const AttnPrefillArgs &args, cudaStream_t s)
{
    if (args.tokens < 1 || args.heads < 1 || args.heads > kAttnHeads || args.kv_ld % 256 ||
        args.out_ld != args.heads * kAttnDim)
        return cudaErrorInvalidValue;
    static cudaError_t attr = cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   static_cast<int>(kPfSmem));
    if (attr != cudaSuccess) return attr;
    const int kv_heads = args.kv_ld / 256;
    cudaError_t e = launch_pdl(attn_prefill_qk_kernel, dim3(args.heads + kv_heads, args.tokens), dim3(256), s, args);
    if (e == cudaSuccess) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((args.tokens + kPfQueries - 1) / kPfQueries, args.heads);
        cfg.blockDim = dim3(256);
        cfg.dynamicSmemBytes = kPfSmem;
        cfg.stream = s;
        cudaLaunchAttribute attr1[1];
        attr1[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr1[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr1;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, attn_prefill_kernel, args);
    }
    if (e == cudaSuccess) e = launch_pdl(attn_prefill_quant_kernel, dim3(args.heads, args.tokens), dim3(256), s, args);
    return e;
}

cudaError_t launch_tp_reduce(const TpReduceArgs &args, cudaStream_t s)
{
    if (args.world < 2 || args.world > 8 || args.rank < 0 || args.rank >= args.world || args.tokens < 1 ||
        args.tokens > kMaxTokens || args.n < kTpReduceCtas)
        return cudaErrorInvalidValue;
    return launch_pdl(tp_reduce_kernel, dim3(kTpReduceCtas), dim3(128), s, args);
}

cudaError_t launch_attention(const AttnArgs &args, cudaStream_t s)
{
    if (args.tokens < 1 || args.tokens > kMaxTokens) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    if (args.heads < 0 || args.heads > kAttnHeads || (args.heads > 0 && args.kv_ld % 256)) return cudaErrorInvalidValue;
    cfg.gridDim = dim3(args.tokens * (args.heads > 0 ? args.heads : kAttnHeads) * kAttnSplits);
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = kAttnSplits;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, attention_kernel, args);
}

cudaError_t launch_argmax(const ArgmaxArgs &args, int tokens, cudaStream_t s)
{
    return launch_pdl(argmax_kernel, dim3(kArgmaxCtas, tokens), dim3(256), s, args);
}

namespace {
__global__ void replicate_kernel(char *base, size_t words, int reps, long long stride)
{
    pdl_wait();
    pdl_launch_dependents();
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= words) return;
    const uint32_t v = reinterpret_cast<const uint32_t *>(base)[i];
    for (int k = 1; k < reps; ++k) reinterpret_cast<uint32_t *>(base + k * stride)[i] = v;
}
}  // namespace

namespace {
__global__ void trace_reset_kernel(unsigned long long *rec, int count)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= count) return;
    unsigned long long *r = rec + static_cast<size_t>(kTraceFields) * i;
    for (int f = 0; f < kTraceFields; ++f) r[f] = trace_is_min(f) ? ~0ull : 0ull;
}
}  // namespace

cudaError_t launch_trace_reset(unsigned long long *records, int count, cudaStream_t s)
{
    if (count <= 0) return cudaSuccess;
    trace_reset_kernel<<<(count + 255) / 256, 256, 0, s>>>(records, count);
    return cudaGetLastError();
}

cudaError_t launch_replicate(void *base, size_t bytes, int reps, long long stride, cudaStream_t s)
{
    if (reps <= 1 || bytes == 0) return cudaSuccess;
    const size_t words = bytes / 4;
    return launch_pdl(replicate_kernel, dim3(static_cast<unsigned>((words + 255) / 256)), dim3(256), s,
                      static_cast<char *>(base), words, reps, stride);
}

cudaError_t read_and_clear_model_status(int *status)
{
    cudaError_t e = cudaMemcpyFromSymbol(status, g_model_status, sizeof(int));
    if (e != cudaSuccess) return e;
    const int zero = 0;
    return cudaMemcpyToSymbol(g_model_status, &zero, sizeof(int));
}

}  // namespace q38
