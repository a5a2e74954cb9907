// q38_kernels.cu - sm_100a kernels of the quantized hot path.
//
//  * q8k_gemm_kernel: weight-streaming GEMV/GEMM over Q8_K activations
//    (upstream q38_tensor_gemv_q8_k / q38_tensor_gemm_q8_k,
//    src/qwen38/qwen38_quant.c:2833-2922, 2950-3169).
//  * quantize_q8k_kernel: fp32 -> Q8_K (qwen38_quant.c:50-88), bit-exact.
//  * f32_gemm_kernel: float-activation path (qwen38_quant.c:2768-2831, 2924-2948).
//  * row_f32_kernel: one-row dequantization (qwen38_quant.c:3186-3222).
//
// Weight streaming design: a persistent grid of CTAs walks "units" of
// consecutive weight rows.  Each unit's bytes are one contiguous range of the
// GGUF tensor; a single thread moves it into a shared-memory stage with a 1-D
// TMA bulk copy (cp.async.bulk) signalled on an mbarrier, several stages deep,
// so HBM always has whole units in flight.  Thread t of a CTA owns superblock
// column b = t % nb of row (t / nb) within each pass over the stage; its Q8_K
// activation block for column b is loaded into registers once per kernel, so
// the integer sums of a (row, superblock) are formed inside one thread, the way
// the upstream per-row loop forms them, and only the per-superblock floats are
// reduced across threads (in a fixed order, hence deterministic).
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/q38cuda.h"
#include "q38_device.cuh"
#include "q38_grid.cuh"
#include "q38_internal.h"
#include "q38_types.cuh"

namespace q38 {

__device__ int g_status;  // device status word (see q38cu_device_status)

constexpr int kMaxStages = 4;

struct GemmArgs {
    const uint8_t *weights;
    uint64_t row_bytes;
    uint64_t total_bytes;
    int rows;       // N
    int nb;         // superblocks per row
    const Q8KBlock *act;  // [batch][nb]
    int batch;
    float *out;     // [batch][rows]
    int32_t *dbg_w;  // optional [batch][rows][nb]
    int32_t *dbg_x;
    int rows_per_pass;
    int rows_per_stage;
    int units;
    int stages;
    uint32_t stage_bytes;  // bytes reserved per stage (>= data + 32 slack)
};

// Issue the bulk copy of unit `unit` into stage `s`.  Returns the byte offset
// of the unit's first row inside the stage.
__device__ __forceinline__ void issue_unit(const GemmArgs &g, uint8_t *stage, uint64_t *bar, int unit)
{
    const uint64_t first = static_cast<uint64_t>(unit) * g.rows_per_stage * g.row_bytes;
    uint64_t last = static_cast<uint64_t>(min(g.rows, (unit + 1) * g.rows_per_stage)) * g.row_bytes;
    const uint64_t a0 = first & ~uint64_t(15);
    const uint64_t a1 = (last + 15) & ~uint64_t(15);
    const uint32_t bytes = static_cast<uint32_t>(a1 - a0);
    mbar_arrive_expect_tx(bar, bytes);
    bulk_copy_g2s(stage, g.weights + a0, bytes, bar);
}

// CTA size bound per token tile: MT = 1 leaves 170 registers a thread, MT = 2
// leaves 255 (two activation blocks in registers).
template <int MT> struct MaxThreads { static constexpr int kValue = MT == 1 ? 384 : 256; };

template <typename Dec, int MT, bool kDbg>
__global__ void __launch_bounds__(MaxThreads<MT>::kValue) q8k_gemm_kernel(GemmArgs g)
{
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t *stages = smem;
    float *red = reinterpret_cast<float *>(smem + static_cast<size_t>(g.stages) * g.stage_bytes);
    const int red_floats = g.rows_per_stage * g.nb * MT;
    uint2 *grid = reinterpret_cast<uint2 *>(red + ((red_floats + 3) & ~3));
    uint64_t *bars = reinterpret_cast<uint64_t *>(grid + NeedsGrid<Dec>::kEntries);

    const int tid = threadIdx.x;
    const int active = g.rows_per_pass * g.nb;
    const int my_row = tid / g.nb;
    const int my_col = tid - my_row * g.nb;
    const int passes = g.rows_per_stage / g.rows_per_pass;
    const int nwarps = blockDim.x >> 5;
    const int lane = tid & 31, warp = tid >> 5;

    if (tid == 0) {
        for (int s = 0; s < g.stages; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) {
        for (int s = 0; s < g.stages; ++s) {
            const int unit = blockIdx.x + s * gridDim.x;
            if (unit < g.units) issue_unit(g, stages + static_cast<size_t>(s) * g.stage_bytes, &bars[s], unit);
        }
    }
    build_grid<Dec>(grid);

    Act a[MT];
    const bool single_pass = g.batch <= MT;
    if (single_pass && tid < active) {
#pragma unroll
        for (int t = 0; t < MT; ++t) {
            if (t < g.batch) Dec::load(a[t], g.act + static_cast<size_t>(t) * g.nb + my_col);
            else Dec::zero(a[t]);
        }
    }
    __syncthreads();

    bool failed = false;
    int it = 0;
    for (int unit = blockIdx.x; unit < g.units; unit += gridDim.x, ++it) {
        const int s = it % g.stages;
        const uint32_t parity = static_cast<uint32_t>(it / g.stages) & 1u;
        // Every thread waits; the give-up decision is made CTA-uniform so no
        // thread is left behind at a later __syncthreads.
        const bool arrived = mbar_wait_bounded(&bars[s], parity, &g_status);
        if (__syncthreads_or(!arrived)) { failed = true; break; }
        const uint64_t first = static_cast<uint64_t>(unit) * g.rows_per_stage * g.row_bytes;
        const uint8_t *base = stages + static_cast<size_t>(s) * g.stage_bytes + (first & 15);
        const int row0 = unit * g.rows_per_stage;
        const int nrows = min(g.rows_per_stage, g.rows - row0);

        for (int tok0 = 0; tok0 < g.batch; tok0 += MT) {
            if (!single_pass && tid < active) {
#pragma unroll
                for (int t = 0; t < MT; ++t) {
                    if (tok0 + t < g.batch)
                        Dec::load(a[t], g.act + static_cast<size_t>(tok0 + t) * g.nb + my_col);
                    else
                        Dec::zero(a[t]);
                }
            }
            if (tid < active) {
                for (int p = 0; p < passes; ++p) {
                    const int r = p * g.rows_per_pass + my_row;
                    if (r < nrows) {
                        const uint8_t *blk = base + static_cast<size_t>(r) * g.row_bytes +
                                             static_cast<size_t>(my_col) * Dec::kBytes;
                        int w[MT], x[MT];
                        float v[MT];
                        run_block<Dec, MT>(blk, RegActs<MT>{a}, w, x, v, grid);
#pragma unroll
                        for (int t = 0; t < MT; ++t) {
                            red[(r * g.nb + my_col) * MT + t] = v[t];
                            if constexpr (kDbg) {
                                if (tok0 + t < g.batch) {
                                    const size_t o = (static_cast<size_t>(tok0 + t) * g.rows + row0 + r) * g.nb + my_col;
                                    g.dbg_w[o] = w[t];
                                    g.dbg_x[o] = x[t];
                                }
                            }
                        }
                    }
                }
            }
            __syncthreads();
            // Row totals: sum the nb superblock contributions in column order.
            for (int r = warp; r < nrows; r += nwarps) {
#pragma unroll
                for (int t = 0; t < MT; ++t) {
                    if (tok0 + t >= g.batch) break;
                    float sum = 0.0f;
                    for (int b = lane; b < g.nb; b += 32) sum += red[(r * g.nb + b) * MT + t];
#pragma unroll
                    for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
                    if (lane == 0) g.out[static_cast<size_t>(tok0 + t) * g.rows + row0 + r] = sum;
                }
            }
            __syncthreads();
        }
        if (tid == 0) {
            const int next = unit + g.stages * gridDim.x;
            if (next < g.units) {
                fence_proxy_async_shared();
                issue_unit(g, stages + static_cast<size_t>(s) * g.stage_bytes, &bars[s], next);
            }
        }
    }
    if (failed && tid == 0) {
        // Drain copies this CTA still has in flight before its shared memory
        // is released (bounded, like every wait here).
        int j = it;
        for (int unit = blockIdx.x + it * gridDim.x; unit < g.units && j < it + g.stages;
             unit += gridDim.x, ++j) {
            mbar_wait_bounded(&bars[j % g.stages], static_cast<uint32_t>(j / g.stages) & 1u, nullptr);
        }
    }
}

// ---------------------------------------------------------------------------
// fp32 -> Q8_K.  One warp per 256-element block; lane l owns elements
// 8l..8l+7.  The max-abs element is the first index holding the largest
// |value| (the upstream scan keeps the first strict maximum).
// ---------------------------------------------------------------------------
__global__ void quantize_q8k_kernel(Q8KBlock *out, const float *in, uint64_t blocks)
{
    const uint64_t block = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (block >= blocks) return;
    const float4 *src = reinterpret_cast<const float4 *>(in + block * 256 + lane * 8);
    const float4 u0 = __ldg(src), u1 = __ldg(src + 1);
    const float x[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
    float amax = 0.0f;
    int idx = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float av = fabsf(x[i]);
        if (av > amax) { amax = av; idx = lane * 8 + i; }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float oa = __shfl_xor_sync(0xffffffffu, amax, off);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, off);
        if (oa > amax || (oa == amax && oi < idx)) { amax = oa; idx = oi; }
    }
    Q8KBlock *q = out + block;
    uint32_t *qw = reinterpret_cast<uint32_t *>(q->quants) + lane * 2;
    if (amax == 0.0f) {
        qw[0] = qw[1] = 0u;
        if (lane < 16) q->sums[lane] = 0;
        if (lane == 0) q->scale = 0.0f;
        return;
    }
    const float maximum = __ldg(in + block * 256 + idx);
    const float inverse = __fdiv_rn(-127.0f, maximum);
    int qv[8];
    int partial = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float shifted = __fadd_rn(__fmul_rn(inverse, x[i]), 12582912.0f);
        int v = static_cast<int>(__float_as_uint(shifted) & 0x007fffffu) - 0x00400000;
        if (v > 127) v = 127;
        qv[i] = v;
        partial += static_cast<int8_t>(v);
    }
    qw[0] = (qv[0] & 0xFF) | (qv[1] & 0xFF) << 8 | (qv[2] & 0xFF) << 16 | static_cast<uint32_t>(qv[3] & 0xFF) << 24;
    qw[1] = (qv[4] & 0xFF) | (qv[5] & 0xFF) << 8 | (qv[6] & 0xFF) << 16 | static_cast<uint32_t>(qv[7] & 0xFF) << 24;
    const int pair = partial + __shfl_xor_sync(0xffffffffu, partial, 1);
    if ((lane & 1) == 0) q->sums[lane >> 1] = static_cast<int16_t>(pair);
    if (lane == 0) q->scale = __fdiv_rn(1.0f, inverse);
}

// ---------------------------------------------------------------------------
// Float path: element decode (exact upstream float formulas) ...
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t ld_u16(const uint8_t *p) { return p[0] | (p[1] << 8); }

__device__ __forceinline__ void k4_scale_min(int j, const uint8_t *p, int &sc, int &m)
{
    if (j < 4) {
        sc = p[j] & 63;
        m = p[j + 4] & 63;
    } else {
        sc = (p[j + 4] & 15) | ((p[j - 4] >> 6) << 4);
        m = (p[j + 4] >> 4) | ((p[j] >> 6) << 4);
    }
}

__device__ __forceinline__ int q3_scale(const uint8_t *p, int i)
{
    const int low = i < 8 ? (p[i] & 15) : (p[i - 8] >> 4);
    const int high = (p[8 + i % 4] >> (2 * (i / 4))) & 3;
    return (low | high << 4) - 32;
}

// Weight i (0 <= i < block elements) of the block at `b`, rounded exactly as
// the upstream float path forms it (qwen38_quant.c:330-508, 2768-2810).
__device__ float element_weight(int type, const uint8_t *b, int i)
{
    switch (type) {
    case kF32: return __ldg(reinterpret_cast<const float *>(b));
    case kF16: return f16_bits_to_f32(ld_u16(b));
    case kBF16: return __uint_as_float(ld_u16(b) << 16);
    case kQ8_0: return __fmul_rn(f16_bits_to_f32(ld_u16(b)), static_cast<float>(static_cast<int8_t>(b[2 + i])));
    case kIQ4_NL: {
        static constexpr int8_t lv[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};
        const uint8_t pk = b[2 + (i & 15)];
        const int q = lv[i < 16 ? (pk & 15) : (pk >> 4)];
        return __fmul_rn(f16_bits_to_f32(ld_u16(b)), static_cast<float>(q));
    }
    case kQ4_K: {
        const int chunk = i >> 6, j = (i >> 5) & 1, e = i & 31;
        int sc, m;
        k4_scale_min(chunk * 2 + j, b + 4, sc, m);
        const uint8_t qb = b[16 + chunk * 32 + e];
        const int q = j ? (qb >> 4) : (qb & 15);
        const float d = f16_bits_to_f32(ld_u16(b)), dmin = f16_bits_to_f32(ld_u16(b + 2));
        return __fsub_rn(__fmul_rn(__fmul_rn(d, static_cast<float>(sc)), static_cast<float>(q)),
                         __fmul_rn(dmin, static_cast<float>(m)));
    }
    case kQ5_K: {
        const int chunk = i >> 6, j = (i >> 5) & 1, e = i & 31;
        int sc, m;
        k4_scale_min(chunk * 2 + j, b + 4, sc, m);
        const uint8_t lb = b[48 + chunk * 32 + e];
        const int hbit = (b[16 + e] >> (2 * chunk + j)) & 1;
        const int q = (j ? (lb >> 4) : (lb & 15)) + 16 * hbit;
        const float d = f16_bits_to_f32(ld_u16(b)), dmin = f16_bits_to_f32(ld_u16(b + 2));
        return __fsub_rn(__fmul_rn(__fmul_rn(d, static_cast<float>(sc)), static_cast<float>(q)),
                         __fmul_rn(dmin, static_cast<float>(m)));
    }
    case kQ6_K: {
        const int half = i >> 7, r = i & 127, qq = r >> 5, e = r & 31;
        const uint8_t lb = b[half * 64 + (qq & 1) * 32 + e];
        const uint8_t hb = b[128 + half * 32 + e];
        const int q = ((qq < 2 ? (lb & 15) : (lb >> 4)) | (((hb >> (2 * qq)) & 3) << 4)) - 32;
        const int sc = static_cast<int8_t>(b[192 + half * 8 + qq * 2 + e / 16]);
        const float d = f16_bits_to_f32(ld_u16(b + 208));
        return __fmul_rn(__fmul_rn(d, static_cast<float>(sc)), static_cast<float>(q));
    }
    case kQ2_K: {
        const int half = i >> 7, field = (i >> 5) & 3, group = (i >> 4) & 1, lane = i & 15;
        const int si = half * 8 + field * 2 + group;
        const uint8_t ps = b[si];
        const int q = (b[16 + half * 32 + group * 16 + lane] >> (field * 2)) & 3;
        const float d = f16_bits_to_f32(ld_u16(b + 80)), dmin = f16_bits_to_f32(ld_u16(b + 82));
        return __fsub_rn(__fmul_rn(__fmul_rn(d, static_cast<float>(ps & 15)), static_cast<float>(q)),
                         __fmul_rn(dmin, static_cast<float>(ps >> 4)));
    }
    case kQ3_K: {
        const int half = i >> 7, field = (i >> 5) & 3, lane = i & 31, group = half * 4 + field;
        const int q = ((b[32 + half * 32 + lane] >> (field * 2)) & 3) - ((b[lane] & (1 << group)) ? 0 : 4);
        const int s = q3_scale(b + 96, group * 2 + lane / 16);
        const float d = f16_bits_to_f32(ld_u16(b + 108));
        return __fmul_rn(__fmul_rn(d, static_cast<float>(s)), static_cast<float>(q));
    }
    default: return __int_as_float(0x7fc00000);
    }
}

// One warp per (row, token).  Lanes take blocks lane, lane+32, ... and the
// partials are reduced with shuffles (fixed order).
// Address of block `blk` of row `row`: GGUF row-major, or the tiled layout
// when tile_rows != 0.
__device__ __forceinline__ const uint8_t *block_at(const uint8_t *w, uint64_t row, uint64_t blk, uint64_t nblocks,
                                                   uint32_t tile_rows, int bb)
{
    if (!tile_rows) return w + (row * nblocks + blk) * bb;
    const uint64_t t = row / tile_rows, r = row - t * tile_rows;
    return w + ((t * nblocks + blk) * tile_rows + r) * bb;
}

// out[tok * out_ld + row] (+)= row . x[tok * x_ld ..]; one warp per (token, row).
__global__ void f32_gemm_kernel(float *out, const float *x, int batch, uint64_t width, const uint8_t *w,
                                uint64_t rows, uint32_t tile_rows, int type, int be, int bb, uint64_t x_ld,
                                uint64_t out_ld, int accumulate)
{
    pdl_wait();
    pdl_launch_dependents();
    const uint64_t gw = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (gw >= rows * static_cast<uint64_t>(batch)) return;
    const uint64_t row = gw % rows;
    const int tok = static_cast<int>(gw / rows);
    const uint64_t nblocks = width / be;
    const float *xx = x + static_cast<uint64_t>(tok) * x_ld;
    float total = 0.0f;
    for (uint64_t blk = lane; blk < nblocks; blk += 32) {
        const uint8_t *b = block_at(w, row, blk, nblocks, tile_rows, bb);
        for (int i = 0; i < be; ++i) total = fmaf(element_weight(type, b, i), __ldg(xx + blk * be + i), total);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) total += __shfl_xor_sync(0xffffffffu, total, off);
    if (lane == 0) {
        float *dst = out + static_cast<uint64_t>(tok) * out_ld + row;
        *dst = accumulate ? __fadd_rn(*dst, total) : total;
    }
}

// The same products for prompt-sized batches: one warp per (kF32Rows rows,
// kF32Toks tokens), so that each decoded weight serves kF32Toks tokens and
// each activation kF32Rows rows.  Every output keeps f32_gemm_kernel's
// summation order (a lane's blocks in order, the same shuffle tree), so the
// two kernels agree bit for bit.
constexpr int kF32Rows = 4;
constexpr int kF32Toks = 8;

__global__ void __launch_bounds__(256) f32_gemm_tile_kernel(float *out, const float *x, int batch, uint64_t width,
                                                            const uint8_t *w, uint64_t rows, uint32_t tile_rows,
                                                            int type, int be, int bb, uint64_t x_ld, uint64_t out_ld,
                                                            int accumulate)
{
    pdl_wait();
    pdl_launch_dependents();
    const uint64_t gw = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const uint64_t row_groups = (rows + kF32Rows - 1) / kF32Rows;
    if (gw >= row_groups * static_cast<uint64_t>((batch + kF32Toks - 1) / kF32Toks)) return;
    const uint64_t row0 = (gw % row_groups) * kF32Rows;
    const int tok0 = static_cast<int>(gw / row_groups) * kF32Toks;
    const uint64_t nblocks = width / be;
    float acc[kF32Rows][kF32Toks];
#pragma unroll
    for (int r = 0; r < kF32Rows; ++r)
#pragma unroll
        for (int t = 0; t < kF32Toks; ++t) acc[r][t] = 0.0f;
    for (uint64_t blk = lane; blk < nblocks; blk += 32) {
        const uint8_t *b[kF32Rows];
#pragma unroll
        for (int r = 0; r < kF32Rows; ++r)
            b[r] = row0 + r < rows ? block_at(w, row0 + r, blk, nblocks, tile_rows, bb) : nullptr;
        for (int i = 0; i < be; ++i) {
            float wv[kF32Rows], xv[kF32Toks];
#pragma unroll
            for (int r = 0; r < kF32Rows; ++r) wv[r] = b[r] ? element_weight(type, b[r], i) : 0.0f;
#pragma unroll
            for (int t = 0; t < kF32Toks; ++t)
                xv[t] = tok0 + t < batch ? __ldg(x + static_cast<uint64_t>(tok0 + t) * x_ld + blk * be + i) : 0.0f;
#pragma unroll
            for (int r = 0; r < kF32Rows; ++r)
#pragma unroll
                for (int t = 0; t < kF32Toks; ++t) acc[r][t] = fmaf(wv[r], xv[t], acc[r][t]);
        }
    }
#pragma unroll
    for (int r = 0; r < kF32Rows; ++r)
#pragma unroll
        for (int t = 0; t < kF32Toks; ++t) {
            float total = acc[r][t];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) total += __shfl_xor_sync(0xffffffffu, total, off);
            if (lane == 0 && row0 + r < rows && tok0 + t < batch) {
                float *dst = out + static_cast<uint64_t>(tok0 + t) * out_ld + row0 + r;
                *dst = accumulate ? __fadd_rn(*dst, total) : total;
            }
        }
}

// The same for 32-element blocks (Q8_0, IQ4_NL): a lane's activation
// elements are 32 floats apart in memory, so the CTA (8 warps = 32 rows, 8
// tokens) first copies 32 blocks' worth of each token's activation into
// shared memory with coalesced loads (rows padded to 33 floats: lane l reads
// bank (l + i) % 32), then every warp walks them as f32_gemm_tile_kernel
// does - same order, same results.  Q8_0 weights take the scale once per
// block (the same product per element).
constexpr int kF32Chunk = 32;  // blocks per shared-memory pass

__global__ void __launch_bounds__(256) f32_gemm_tile32_kernel(float *out, const float *x, int batch, uint64_t width,
                                                              const uint8_t *w, uint64_t rows, uint32_t tile_rows,
                                                              int type, int bb, uint64_t x_ld, uint64_t out_ld,
                                                              int accumulate)
{
    __shared__ float xs[kF32Toks][kF32Chunk * 33];
    pdl_wait();
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint64_t row0 = (static_cast<uint64_t>(blockIdx.x) * 8 + warp) * kF32Rows;
    const int tok0 = static_cast<int>(blockIdx.y) * kF32Toks;
    const uint64_t nblocks = width / 32;
    float acc[kF32Rows][kF32Toks];
#pragma unroll
    for (int r = 0; r < kF32Rows; ++r)
#pragma unroll
        for (int t = 0; t < kF32Toks; ++t) acc[r][t] = 0.0f;
    for (uint64_t c0 = 0; c0 < nblocks; c0 += kF32Chunk) {
        __syncthreads();  // the previous pass is consumed
        const int n_el = static_cast<int>(nblocks - c0 < kF32Chunk ? nblocks - c0 : kF32Chunk) * 32;
        for (int i = threadIdx.x; i < kF32Toks * kF32Chunk * 32; i += blockDim.x) {
            const int t = i / (kF32Chunk * 32), e = i % (kF32Chunk * 32);
            xs[t][(e >> 5) * 33 + (e & 31)] =
                tok0 + t < batch && e < n_el ? __ldg(x + static_cast<uint64_t>(tok0 + t) * x_ld + c0 * 32 + e) : 0.0f;
        }
        __syncthreads();
        const uint64_t blk = c0 + lane;
        if (blk >= nblocks) continue;
        const uint8_t *b[kF32Rows];
#pragma unroll
        for (int r = 0; r < kF32Rows; ++r)
            b[r] = row0 + r < rows ? block_at(w, row0 + r, blk, nblocks, tile_rows, bb) : nullptr;
        const float *xl = &xs[0][lane * 33];
        if (type == kQ8_0) {
            float d[kF32Rows];
#pragma unroll
            for (int r = 0; r < kF32Rows; ++r) d[r] = b[r] ? f16_bits_to_f32(ld_u16(b[r])) : 0.0f;
            for (int i = 0; i < 32; ++i) {
                float wv[kF32Rows];
#pragma unroll
                for (int r = 0; r < kF32Rows; ++r)
                    wv[r] = b[r] ? __fmul_rn(d[r], static_cast<float>(static_cast<int8_t>(b[r][2 + i]))) : 0.0f;
#pragma unroll
                for (int t = 0; t < kF32Toks; ++t) {
                    const float xv = xl[t * kF32Chunk * 33 + i];
#pragma unroll
                    for (int r = 0; r < kF32Rows; ++r) acc[r][t] = fmaf(wv[r], xv, acc[r][t]);
                }
            }
        } else {
            for (int i = 0; i < 32; ++i) {
                float wv[kF32Rows];
#pragma unroll
                for (int r = 0; r < kF32Rows; ++r) wv[r] = b[r] ? element_weight(type, b[r], i) : 0.0f;
#pragma unroll
                for (int t = 0; t < kF32Toks; ++t) {
                    const float xv = xl[t * kF32Chunk * 33 + i];
#pragma unroll
                    for (int r = 0; r < kF32Rows; ++r) acc[r][t] = fmaf(wv[r], xv, acc[r][t]);
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < kF32Rows; ++r)
#pragma unroll
        for (int t = 0; t < kF32Toks; ++t) {
            float total = acc[r][t];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) total += __shfl_xor_sync(0xffffffffu, total, off);
            if (lane == 0 && row0 + r < rows && tok0 + t < batch) {
                float *dst = out + static_cast<uint64_t>(tok0 + t) * out_ld + row0 + r;
                *dst = accumulate ? __fadd_rn(*dst, total) : total;
            }
        }
}

// Row `row` . x by one warp, in f32_gemm_kernel's order (the same value).
__global__ void dot_row_f32_kernel(float *out, const float *x, const uint8_t *w, uint64_t width, uint32_t tile_rows,
                                   uint64_t row, int type, int be, int bb)
{
    const int lane = threadIdx.x & 31;
    const uint64_t nblocks = width / be;
    float total = 0.0f;
    for (uint64_t blk = lane; blk < nblocks; blk += 32) {
        const uint8_t *b = block_at(w, row, blk, nblocks, tile_rows, bb);
        for (int i = 0; i < be; ++i) total = fmaf(element_weight(type, b, i), __ldg(x + blk * be + i), total);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) total += __shfl_xor_sync(0xffffffffu, total, off);
    if (lane == 0) *out = total;
}

// Element i of row `row`.  The upstream evaluates fma(w, 1, 0) against a
// basis vector, which equals w for finite w except that -0 becomes +0.
__global__ void row_f32_kernel(float *out, const uint8_t *w, uint64_t width, uint32_t tile_rows, uint64_t row,
                               int type, int be, int bb)
{
    const uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= width) return;
    const uint64_t nblocks = width / be;
    const uint8_t *b = block_at(w, row, i / be, nblocks, tile_rows, bb);
    const float v = element_weight(type, b, static_cast<int>(i % be));
    out[i] = type == kF32 || type == kF16 || type == kBF16 ? v : __fadd_rn(v, 0.0f);
}

// Rows selected by token ids held in device memory (the model's embedding
// lookup inside a captured decode step): output row y is row row_index[y].
// An id outside the tensor yields NaN and the kStatusBadToken status.
__global__ void row_f32_indexed_kernel(float *out, const uint8_t *w, uint64_t width, uint32_t tile_rows,
                                       uint64_t rows, const uint32_t *row_index, int type, int be, int bb,
                                       int reps, long long rep_floats)
{
    pdl_wait();
    pdl_launch_dependents();
    const uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= width) return;
    const uint64_t row = row_index[blockIdx.y];
    float *o = out + static_cast<uint64_t>(blockIdx.y) * width;
    float v = __int_as_float(0x7fc00000);
    if (row >= rows) {
        if (i == 0) atomicExch(&g_status, kStatusBadToken);
    } else {
        const uint64_t nblocks = width / be;
        const uint8_t *b = block_at(w, row, i / be, nblocks, tile_rows, bb);
        v = element_weight(type, b, static_cast<int>(i % be));
        if (!(type == kF32 || type == kF16 || type == kBF16)) v = __fadd_rn(v, 0.0f);
    }
    for (int k = 0; k < reps; ++k) o[i + k * rep_floats] = v;  // the row and its replicas
}

// ---------------------------------------------------------------------------
// Host-side launchers
// ---------------------------------------------------------------------------
// Occupancy cache for the weight-streaming kernels (see launch_gemm_t).
static cudaError_t cached_occupancy(const void *kernel, int threads, size_t smem, int *per_sm)
{
    struct Entry { const void *kernel; int device; int threads; size_t smem; int per_sm; };
    static Entry cache[256];
    static int used = 0;
    static std::mutex lock;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> guard(lock);
    for (int i = 0; i < used; ++i) {
        const Entry &c = cache[i];
        if (c.kernel == kernel && c.device == dev && c.threads == threads && c.smem == smem) {
            *per_sm = c.per_sm;
            return cudaSuccess;
        }
    }
    // Opt in to the device's full dynamic shared memory once per kernel, so a
    // later (smaller) configuration never lowers the limit a cached one uses.
    bool opted = false;
    for (int i = 0; i < used; ++i) opted |= cache[i].kernel == kernel && cache[i].device == dev;
    if (!opted) {
        int optin = 0;
        e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, optin);
        if (e != cudaSuccess) return e;
    }
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(per_sm, kernel, threads, smem);
    if (e != cudaSuccess) return e;
    if (used < 256) cache[used++] = Entry{kernel, dev, threads, smem, *per_sm};
    return cudaSuccess;
}

template <typename Dec>
static size_t gemm_smem_bytes(const GemmPlan &p, int mt)
{
    const size_t red = (static_cast<size_t>(p.rows_per_stage) * p.nb * mt + 3) & ~size_t(3);
    return static_cast<size_t>(p.stages) * p.stage_bytes + red * 4 +
           static_cast<size_t>(NeedsGrid<Dec>::kEntries) * 8 + kMaxStages * 8;
}

template <typename Dec, int MT, bool kDbg>
static cudaError_t launch_gemm_t(const GemmPlan &p, const LaunchGemm &l, cudaStream_t stream)
{
    GemmArgs g;
    g.weights = static_cast<const uint8_t *>(l.weights);
    g.row_bytes = p.row_bytes;
    g.total_bytes = p.row_bytes * static_cast<uint64_t>(p.rows);
    g.rows = p.rows;
    g.nb = p.nb;
    g.act = static_cast<const Q8KBlock *>(l.act);
    g.batch = l.batch;
    g.out = l.out;
    g.dbg_w = l.dbg_w;
    g.dbg_x = l.dbg_x;
    g.rows_per_pass = p.rows_per_pass;
    g.rows_per_stage = p.rows_per_stage;
    g.units = p.units;
    g.stages = p.stages;
    g.stage_bytes = p.stage_bytes;
    const size_t smem = gemm_smem_bytes<Dec>(p, MT);
    auto kernel = q8k_gemm_kernel<Dec, MT, kDbg>;
    // The shared-memory opt-in and the occupancy query are host API calls;
    // they are made once per (device, configuration) and cached, so a launch
    // inside CUDA-graph capture issues nothing but the kernel itself.
    int per_sm = 0;
    cudaError_t e = cached_occupancy(reinterpret_cast<const void *>(kernel), p.threads, smem, &per_sm);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    if (p.max_ctas_per_sm > 0 && per_sm > p.max_ctas_per_sm) per_sm = p.max_ctas_per_sm;
    const int grid = min(p.units, per_sm * device_sm_count());
    kernel<<<grid, p.threads, smem, stream>>>(g);
    return cudaGetLastError();
}

template <typename Dec>
static cudaError_t dispatch_mt(const GemmPlan &p, const LaunchGemm &l, cudaStream_t s)
{
    const bool dbg = l.dbg_w != nullptr;
    if (l.batch == 1) return dbg ? launch_gemm_t<Dec, 1, true>(p, l, s) : launch_gemm_t<Dec, 1, false>(p, l, s);
    return dbg ? launch_gemm_t<Dec, 2, true>(p, l, s) : launch_gemm_t<Dec, 2, false>(p, l, s);
}

int superblock_bytes(int type)
{
    switch (type) {
    case kQ4_K: return DecQ4K::kBytes;
    case kQ6_K: return DecQ6K::kBytes;
    case kIQ2_S: return DecIQ2S::kBytes;
    case kIQ1_S: return DecIQ1S::kBytes;
    case kIQ1_M: return DecIQ1M::kBytes;
    case kQ2_K: return DecQ2K::kBytes;
    case kQ3_K: return DecQ3K::kBytes;
    case kQ5_K: return DecQ5K::kBytes;
    case kIQ2_XXS: return DecIQ2XXS::kBytes;
    case kIQ2_XS: return DecIQ2XS::kBytes;
    case kIQ3_XXS: return DecIQ3XXS::kBytes;
    case kIQ3_S: return DecIQ3S::kBytes;
    case kIQ4_XS: return DecIQ4XS::kBytes;
    case kIQ4_NL: return DecIQ4NL::kBytes;
    default: return 0;
    }
}

size_t gemm_smem_for(int type, const GemmPlan &p, int batch)
{
    const int mt = batch == 1 ? 1 : 2;
    switch (type) {
    case kQ4_K: return gemm_smem_bytes<DecQ4K>(p, mt);
    case kQ6_K: return gemm_smem_bytes<DecQ6K>(p, mt);
    case kIQ2_S: return gemm_smem_bytes<DecIQ2S>(p, mt);
    case kIQ1_S: return gemm_smem_bytes<DecIQ1S>(p, mt);
    case kIQ1_M: return gemm_smem_bytes<DecIQ1M>(p, mt);
    case kQ2_K: return gemm_smem_bytes<DecQ2K>(p, mt);
    case kQ3_K: return gemm_smem_bytes<DecQ3K>(p, mt);
    case kQ5_K: return gemm_smem_bytes<DecQ5K>(p, mt);
    case kIQ2_XXS: return gemm_smem_bytes<DecIQ2XXS>(p, mt);
    case kIQ2_XS: return gemm_smem_bytes<DecIQ2XS>(p, mt);
    case kIQ3_XXS: return gemm_smem_bytes<DecIQ3XXS>(p, mt);
    case kIQ3_S: return gemm_smem_bytes<DecIQ3S>(p, mt);
    case kIQ4_XS: return gemm_smem_bytes<DecIQ4XS>(p, mt);
    case kIQ4_NL: return gemm_smem_bytes<DecIQ4NL>(p, mt);
    default: return 0;
    }
}

cudaError_t launch_q8k_gemm(int type, const GemmPlan &p, const LaunchGemm &l, cudaStream_t s)
{
    switch (type) {
    case kQ4_K: return dispatch_mt<DecQ4K>(p, l, s);
    case kQ6_K: return dispatch_mt<DecQ6K>(p, l, s);
    case kIQ2_S: return dispatch_mt<DecIQ2S>(p, l, s);
    case kIQ1_S: return dispatch_mt<DecIQ1S>(p, l, s);
    case kIQ1_M: return dispatch_mt<DecIQ1M>(p, l, s);
    case kQ2_K: return dispatch_mt<DecQ2K>(p, l, s);
    case kQ3_K: return dispatch_mt<DecQ3K>(p, l, s);
    case kQ5_K: return dispatch_mt<DecQ5K>(p, l, s);
    case kIQ2_XXS: return dispatch_mt<DecIQ2XXS>(p, l, s);
    case kIQ2_XS: return dispatch_mt<DecIQ2XS>(p, l, s);
    case kIQ3_XXS: return dispatch_mt<DecIQ3XXS>(p, l, s);
    case kIQ3_S: return dispatch_mt<DecIQ3S>(p, l, s);
    case kIQ4_XS: return dispatch_mt<DecIQ4XS>(p, l, s);
    case kIQ4_NL: return dispatch_mt<DecIQ4NL>(p, l, s);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_quantize_q8k(void *out, const float *in, uint64_t blocks, cudaStream_t s)
{
    if (blocks == 0) return cudaSuccess;
    const uint64_t threads = blocks * 32;
    const unsigned grid = static_cast<unsigned>((threads + 255) / 256);
    quantize_q8k_kernel<<<grid, 256, 0, s>>>(static_cast<Q8KBlock *>(out), in, blocks);
    return cudaGetLastError();
}

cudaError_t launch_dot_row_f32(float *out, const float *x, const void *w, uint64_t width, uint32_t tile_rows,
                               uint64_t row, int type, int be, int bb, cudaStream_t s)
{
    dot_row_f32_kernel<<<1, 32, 0, s>>>(out, x, static_cast<const uint8_t *>(w), width, tile_rows, row, type, be, bb);
    return cudaGetLastError();
}

cudaError_t launch_f32_gemm(float *out, const float *x, int batch, uint64_t width, const void *w, uint64_t rows,
                            uint32_t tile_rows, int type, int be, int bb, cudaStream_t s)
{
    return launch_f32_gemm_ex(out, rows, 0, x, width, batch, width, w, rows, tile_rows, type, be, bb, s);
}

cudaError_t launch_f32_gemm_ex(float *out, uint64_t out_ld, int accumulate, const float *x, uint64_t x_ld, int batch,
                               uint64_t width, const void *w, uint64_t rows, uint32_t tile_rows, int type, int be,
                               int bb, cudaStream_t s)
{
    const uint64_t warps = rows * static_cast<uint64_t>(batch);
    if (warps == 0) return cudaSuccess;
    // batches of a prompt take the register-tiled forms (same results)
    const bool tiled = batch >= 2 * kF32Toks;
    if (tiled && be == 32) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(static_cast<unsigned>((rows + 8 * kF32Rows - 1) / (8 * kF32Rows)),
                           static_cast<unsigned>((batch + kF32Toks - 1) / kF32Toks));
        cfg.blockDim = dim3(256);
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        return cudaLaunchKernelEx(&cfg, f32_gemm_tile32_kernel, out, x, batch, width,
                                  static_cast<const uint8_t *>(w), rows, tile_rows, type, bb, x_ld, out_ld,
                                  accumulate);
    }
    const uint64_t launch_warps =
        tiled ? (rows + kF32Rows - 1) / kF32Rows * static_cast<uint64_t>((batch + kF32Toks - 1) / kF32Toks) : warps;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>((launch_warps * 32 + 255) / 256));
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, tiled ? f32_gemm_tile_kernel : f32_gemm_kernel, out, x, batch, width,
                              static_cast<const uint8_t *>(w), rows, tile_rows, type, be, bb, x_ld, out_ld,
                              accumulate);
}

cudaError_t launch_row_f32(float *out, const void *w, uint64_t width, uint32_t tile_rows, uint64_t row, int type,
                           int be, int bb, cudaStream_t s)
{
    const unsigned grid = static_cast<unsigned>((width + 255) / 256);
    row_f32_kernel<<<grid, 256, 0, s>>>(out, static_cast<const uint8_t *>(w), width, tile_rows, row, type, be, bb);
    return cudaGetLastError();
}

cudaError_t launch_row_f32_indexed(float *out, const void *w, uint64_t width, uint32_t tile_rows, uint64_t rows,
                                   const uint32_t *row_index, int count, int type, int be, int bb, cudaStream_t s,
                                   int reps, long long rep_floats)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>((width + 255) / 256), static_cast<unsigned>(count));
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, row_f32_indexed_kernel, out, static_cast<const uint8_t *>(w), width, tile_rows,
                              rows, row_index, type, be, bb, reps < 1 ? 1 : reps, rep_floats);
}

// Failure-path probe: one thread waits on an mbarrier that nothing arrives
// at, with the bounded wait every kernel of the library uses, so the wait
// runs out after `limit_ns` and records kStatusWaitTimeout in the status word.
__global__ void wait_probe_kernel(unsigned long long limit_ns)
{
    __shared__ __align__(8) uint64_t bar;
    mbar_init(&bar, 1);
    fence_mbar_init();
    mbar_wait_bounded(&bar, 0u, &g_status, limit_ns);
}

cudaError_t launch_wait_probe(unsigned long long limit_ns, cudaStream_t s)
{
    wait_probe_kernel<<<1, 1, 0, s>>>(limit_ns);
    return cudaGetLastError();
}

cudaError_t read_and_clear_status(int *status, cudaStream_t s)
{
    cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return e;
    e = cudaMemcpyFromSymbol(status, g_status, sizeof(int));
    if (e != cudaSuccess) return e;
    const int zero = 0;
    return cudaMemcpyToSymbol(g_status, &zero, sizeof(int));
}

}  // namespace q38
