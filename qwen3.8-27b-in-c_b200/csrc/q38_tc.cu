// q38_tc.cu - tensor-core batch GEMM for prefill (sm_100a tcgen05).
//
// Prefill multiplies every weight matrix by a whole prompt chunk (the
// upstream layer-major batch, src/qwen38/qwen38_model.c:1519-1560, which calls
// q38_tensor_gemm_q8_k, src/qwen38/qwen38_quant.c:2950-3169, with M = prompt
// tokens).  At M in the hundreds or thousands this is a dense contraction, so
// it runs on the 5th-generation tensor cores with dequant-staged operands:
//
//   A (weights)     each row dequantized with the upstream float formula of
//                   its type, times a power of two 2^-e per row that puts
//                   the row's bound on |w| just below 2^15, split into
//                   hi = fp16(w) and lo = fp16(w - hi): 22 significant bits;
//   B (activations) the int8 quants of the M tokens' Q8_K blocks, as fp16
//                   (exact); each block's scale d[t][sb] stays fp32;
//   D               per 256-wide superblock (one Q8_K block), fp32 in tensor
//                   memory: A_hi.B + A_lo.B over its sixteen 16-wide K steps
//                   (products exact in fp32); the epilogue promotes it into
//                   fp32 registers as sum += D x d[t][sb] (the upstream's
//                   per-block scale of the integer dot), then times the
//                   row's power of two, stored batch-major out[token][row]
//                   (+= with `accumulate`, the residual add of the caller).
//
// So the result carries the rounding of an fp32 dot product with 22-bit
// weights and exact activations: about 1e-6 relative, the same order as the
// float combination of the integer path, instead of the 1e-3 of single fp16
// operands (which the chaotic 64-layer random-init models amplify into
// different logits).  Per-block integer sums are not formed here - the M <= 8
// decode and verification path keeps the exact integer sums.
//
// Kernel: one CTA per 128 x BN output tile (128 weight rows, BN = 128 or 256
// tokens), 2 + BN / 32 warps: warp 0 lane 0 issues the TMA tile loads (3-D
// boxes: the hi and lo tiles of A, 2 x 128 x 64 fp16, and B, BN x 64,
// 128-byte swizzle) into a ring of stages; warp 1 allocates 2 BN
// tensor-memory columns (two superblock buffers) and its lane 0 issues
// tcgen05.mma (M = 128, N = BN, K = 16, two per K step) and commits each stage
// back to the producer; the other warps read the accumulator (warp w reads
// TMEM lanes 32 (w % 4) .., 128 columns each) and store it.  Every mbarrier
// wait is bounded (2 s): a wait that runs out records the status word, the
// MMA issuer still commits the accumulator barrier, the producer waits for
// the copies it issued, and the CTA frees its tensor memory and exits.
#include <cuda.h>  // CUtensorMap and its enums; the encoder comes from the driver at run time
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "../../include/q38cuda.h"
#include "q38_device.cuh"
#include "q38_internal.h"
#include "q38_types.cuh"

namespace q38 {

__device__ int g_tc_status;  // status word of this file's kernels

namespace {

constexpr int kTcRows = 128;   // UMMA M: weight rows per tile
constexpr int kTcK = 64;       // fp16 elements per stage row: one 128-byte swizzle span

template <int BN> struct TcCfg {
    static constexpr int kEpiWarps = BN / 32;             // 128 accumulator columns each
    static constexpr int kThreads = 64 + 32 * kEpiWarps;  // producer, MMA issuer, epilogue
    // declared thread bound: 320 also for BN = 128 (192 threads), which caps
    // registers at 204 a thread - enough for the 128 sums without spilling
    static constexpr int kLaunchBound = 320;
    static constexpr int kStages = BN == 256 ? 3 : 4;
    static constexpr uint32_t kATile = kTcRows * kTcK * 2;   // one of A hi / A lo
    static constexpr uint32_t kBTile = BN * kTcK * 2;
    static constexpr uint32_t kStage = 2 * kATile + kBTile;  // a multiple of 1024
};

// ---- TMA, tensor memory and tcgen05 primitives ----------------------------

// Box (64, rows, 2) at (x, y, 0): the hi tile, then the lo tile.
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar)
{
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_addr(dst)),
        "l"(map), "r"(x), "r"(y), "r"(0), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t cols)
{
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)),
                 "r"(cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols)
{
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] x B[smem]^T, kind::f16 (fp16 inputs, fp32 accumulate).
__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on `bar` once every tcgen05.mma this thread issued so far completes.
__device__ __forceinline__ void mma_commit(uint64_t *bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns of tensor memory.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor of a K-major operand tile stored as the TMA
// writes it with 128-byte swizzling: rows of 128 bytes, 8-row groups 1024
// bytes apart (stride byte offset), the leading byte offset unused for this
// layout (1), descriptor version 1, layout type 2 = 128-byte swizzle.  A
// K-step of 16 fp16 inside the 128-byte row advances the start address by 32
// bytes; the swizzle is applied to the absolute address, so the tile must
// start 1024-byte aligned.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr)
{
    return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(1) << 16) |
           (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
           (static_cast<uint64_t>(2) << 61);
}

// Instruction descriptor: fp32 accumulator (bits 4-5 = 1), A and B fp16
// (bits 7-9, 10-12 = 0), both K-major (bits 15, 16 = 0), N >> 3 at bits
// 17-22, M >> 4 at bits 24-28.
template <int BN> __host__ __device__ constexpr uint32_t f16_idesc()
{
    return (1u << 4) | (static_cast<uint32_t>(BN >> 3) << 17) | (static_cast<uint32_t>(kTcRows >> 4) << 24);
}

struct TcArgs {
    float *out;             // [m][ld]
    int ld;
    int n, m, k;            // weight rows, tokens, width
    const float *b_scale;   // [k / 256][b_scale_ld]: Q8_K block scales (0 past m)
    int b_scale_ld;         // a multiple of BN
    const float *row_scale; // [n]: 2^e of each weight row
    int accumulate;
};

// K steps (64 wide) per accumulation segment: one 256-element superblock.
constexpr int kTcSegment = 4;

template <int BN>
__global__ void __launch_bounds__(TcCfg<BN>::kLaunchBound, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, TcArgs g)
{
    using C = TcCfg<BN>;
    constexpr int kStages = C::kStages;
    // a stage: A hi, A lo, B (each tile 1024-byte aligned)
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + kStages * C::kStage);
    uint64_t *empty = full + kStages;
    uint64_t *acc_full = empty + kStages;  // [2]: a segment's sums are in tensor-memory buffer b
    uint64_t *acc_empty = acc_full + 2;    // [2]: the epilogue has read buffer b
    uint64_t *drained = acc_empty + 2;     // the MMA issuer's last MMA has completed
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drained + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tok_tiles = (g.m + BN - 1) / BN;
    const int row0 = (blockIdx.x / tok_tiles) * kTcRows, tok0 = (blockIdx.x % tok_tiles) * BN;
    const int nk = g.k / kTcK;
    const int segments = (nk + kTcSegment - 1) / kTcSegment;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], C::kEpiWarps);  // one arrival per epilogue warp
        }
        mbar_init(drained, 1);
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, 2 * BN);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();  // A and B were written by the preceding kernels of the stream

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            int issued = 0;
            for (int k = 0; k < nk; ++k) {
                const int s = k % kStages;
                if (k >= kStages &&
                    !mbar_wait_bounded(&empty[s], static_cast<uint32_t>((k / kStages) - 1) & 1u, &g_tc_status))
                    break;
                uint8_t *stage = smem + s * C::kStage;
                mbar_arrive_expect_tx(&full[s], C::kStage);
                tma_load_3d(stage, &map_a, k * kTcK, row0, &full[s]);
                tma_load_3d(stage + 2 * C::kATile, &map_b, k * kTcK, tok0, &full[s]);
                issued = k + 1;
            }
            // The copies issued last must land before shared memory goes away.
            for (int k = issued > kStages ? issued - kStages : 0; k < issued; ++k)
                mbar_wait_bounded(&full[k % kStages], static_cast<uint32_t>(k / kStages) & 1u, &g_tc_status);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            // Segment sg accumulates K steps [4 sg, 4 sg + 4) (superblock sg)
            // into tensor-memory buffer sg % 2, which the epilogue must have
            // emptied first.
            bool ok = true;
            for (int sg = 0; ok && sg < segments; ++sg) {
                const int b = sg & 1;
                const uint32_t acc = tmem + static_cast<uint32_t>(b * BN);
                if (sg >= 2 && !mbar_wait_bounded(&acc_empty[b], static_cast<uint32_t>((sg >> 1) - 1) & 1u, &g_tc_status)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const int k1 = min(nk, (sg + 1) * kTcSegment);
                for (int k = sg * kTcSegment; k < k1; ++k) {
                    const int s = k % kStages;
                    if (!mbar_wait_bounded(&full[s], static_cast<uint32_t>(k / kStages) & 1u, &g_tc_status)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_hi = smem_addr(smem + s * C::kStage), a_lo = a_hi + C::kATile;
                    const uint32_t bq = a_hi + 2 * C::kATile;
#pragma unroll
                    for (int kk = 0; kk < kTcK / 16; ++kk) {
                        const uint32_t o = kk * 32;
                        mma_f16(acc, sw128_desc(a_hi + o), sw128_desc(bq + o), f16_idesc<BN>(),
                                (k > sg * kTcSegment || kk > 0) ? 1u : 0u);
                        mma_f16(acc, sw128_desc(a_lo + o), sw128_desc(bq + o), f16_idesc<BN>(), 1u);
                    }
                    mma_commit(&empty[s]);  // the stage is free once these MMAs have read it
                }
                if (ok) mma_commit(&acc_full[b]);
            }
            mma_commit(drained);  // every MMA issued has completed when this arrives
            mbar_wait_bounded(drained, 0u, &g_tc_status);
        }
        __syncwarp();
    } else {
        // ---------------- epilogue ----------------
        // Thread (quarter, lane) of epilogue warp ew owns weight row
        // 32 quarter + lane of the tile and accumulator columns (tokens)
        // col0 .. col0 + 127; each segment's sums are scaled by the tokens'
        // block scales and added into fp32 registers (IEEE rounding; the
        // tensor core's own accumulation is only trusted over one superblock).
        const int ew = warp - 2, quarter = warp & 3, col0 = (ew >> 2) * 128;
        const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
        float sum[128];
#pragma unroll
        for (int c = 0; c < 128; ++c) sum[c] = 0.0f;
        bool ok = true;
        for (int sg = 0; sg < segments; ++sg) {
            const int b = sg & 1;
            const float4 *sc = reinterpret_cast<const float4 *>(g.b_scale + static_cast<size_t>(sg) * g.b_scale_ld +
                                                                tok0 + col0);
            ok = ok && mbar_wait_bounded(&acc_full[b], static_cast<uint32_t>(sg >> 1) & 1u, &g_tc_status);
            if (!ok) break;
            __syncwarp();
            tc_fence_after();
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                uint32_t v[16];
                tmem_ld16(tmem + lane_addr + static_cast<uint32_t>(b * BN + col0 + c * 16), v);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float4 d = __ldg(sc + c * 4 + q);
                    float *s4 = sum + c * 16 + q * 4;
                    s4[0] = fmaf(__uint_as_float(v[q * 4 + 0]), d.x, s4[0]);
                    s4[1] = fmaf(__uint_as_float(v[q * 4 + 1]), d.y, s4[1]);
                    s4[2] = fmaf(__uint_as_float(v[q * 4 + 2]), d.z, s4[2]);
                    s4[3] = fmaf(__uint_as_float(v[q * 4 + 3]), d.w, s4[3]);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[b]);
        }
        const int row = row0 + quarter * 32 + lane;
        if (ok && row < g.n) {
            const float rs = __ldg(g.row_scale + row);
#pragma unroll
            for (int c = 0; c < 128; ++c) {
                const int tok = tok0 + col0 + c;
                if (tok < g.m) {
                    float *dst = g.out + static_cast<size_t>(tok) * g.ld + row;
                    const float r = __fmul_rn(sum[c], rs);
                    *dst = g.accumulate ? __fadd_rn(*dst, r) : r;
                }
            }
        }
    }
    pdl_launch_dependents();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 2 * BN);
    }
}

template <int BN> constexpr size_t tc_smem_bytes()
{
    return 1024 + static_cast<size_t>(TcCfg<BN>::kStages) * TcCfg<BN>::kStage +
           (2 * TcCfg<BN>::kStages + 5) * 8 + 16;
}

// ---- operand staging --------------------------------------------------------

__device__ __forceinline__ uint32_t ld_u16(const uint8_t *p) { return p[0] | (p[1] << 8); }

// Weights 8 l .. 8 l + 7 of one superblock (lane l of a warp), dequantized
// with the upstream float formula of the type (qwen38_quant.c:330-508):
// Q4_K w = (d sc) q - dmin m per 32-weight sub-block, Q6_K w = (d sc) q.
// The block's 16-byte header (d, dmin, 12 scale bytes) and this lane's 8
// quant bytes, as two loads (Q4_K blocks of 144 bytes start on 16-byte
// boundaries in either layout).
struct Q4KLane {
    uint4 hdr;
    uint2 q;
};

__device__ __forceinline__ Q4KLane q4k_load(const uint8_t *b, int lane)
{
    Q4KLane r;
    r.hdr = *reinterpret_cast<const uint4 *>(b);
    r.q = *reinterpret_cast<const uint2 *>(b + 16 + (lane >> 3) * 32 + (lane & 3) * 8);
    return r;
}

__device__ __forceinline__ void q4k_eight(const Q4KLane &in, int lane, float (&w)[8])
{
    const int grp = lane >> 2, hi = grp & 1;
    auto byte = [&](int k) -> int {  // header byte k (selects, no indexed array)
        const uint32_t wd = k < 4 ? in.hdr.x : k < 8 ? in.hdr.y : k < 12 ? in.hdr.z : in.hdr.w;
        return static_cast<int>((wd >> (8 * (k & 3))) & 0xFFu);
    };
    int sc, m;
    if (grp < 4) {  // header bytes 4 + i are the scale bytes p[i]
        sc = byte(4 + grp) & 63;
        m = byte(8 + grp) & 63;
    } else {
        sc = (byte(8 + grp) & 15) | ((byte(grp) >> 6) << 4);
        m = (byte(8 + grp) >> 4) | ((byte(4 + grp) >> 6) << 4);
    }
    const float d = f16_bits_to_f32(in.hdr.x & 0xFFFFu), dmin = f16_bits_to_f32(in.hdr.x >> 16);
    const float ds = __fmul_rn(d, static_cast<float>(sc)), dm = __fmul_rn(dmin, static_cast<float>(m));
    const uint2 q = in.q;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const uint32_t byte = ((e < 4 ? q.x : q.y) >> (8 * (e & 3))) & 0xFFu;
        const int qv = hi ? static_cast<int>(byte >> 4) : static_cast<int>(byte & 15u);
        w[e] = __fsub_rn(__fmul_rn(ds, static_cast<float>(qv)), dm);
    }
}

__device__ __forceinline__ void q6k_eight(const uint8_t *b, int lane, float (&w)[8])
{
    const int half = lane >> 4, qq = (lane >> 2) & 3, el0 = (lane & 3) * 8;
    const float d = f16_bits_to_f32(ld_u16(b + 208));
    const int sc = static_cast<int8_t>(b[192 + half * 8 + qq * 2 + el0 / 16]);
    const float dsc = __fmul_rn(d, static_cast<float>(sc));
    // Q6_K blocks are 210 bytes: only 2-byte alignment holds
    const uint8_t *lbp = b + half * 64 + (qq & 1) * 32 + el0;
    const uint8_t *hbp = b + 128 + half * 32 + el0;
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
        const uint32_t l2 = ld_u16(lbp + e), h2 = ld_u16(hbp + e);
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const uint32_t lb = (l2 >> (8 * k)) & 0xFFu, hb = (h2 >> (8 * k)) & 0xFFu;
            const int q = static_cast<int>((qq < 2 ? (lb & 15u) : (lb >> 4)) | (((hb >> (2 * qq)) & 3u) << 4)) - 32;
            w[e + k] = __fmul_rn(dsc, static_cast<float>(q));
        }
    }
}

// The power of two 2^e of each weight row: e is chosen so that a bound on
// the row's |w| (Q4_K: |d| 63 15 + |dmin| 63 per superblock; Q6_K: |d| 127 32)
// times 2^-e lies in [2^14, 2^15).  One warp per row.
__global__ void row_scale_kernel(const uint8_t *w, int type, uint64_t rows, uint64_t nb, uint32_t tile_rows, int bb,
                                 float *row_scale, int split)
{
    pdl_wait();
    const uint64_t row = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    float bound = 0.0f;
    for (uint64_t blk = lane; blk < nb; blk += 32) {
        const uint8_t *b;
        if (tile_rows) {
            const uint64_t t = row / tile_rows, r = row - t * tile_rows;
            b = w + ((t * nb + blk) * tile_rows + r) * bb;
        } else {
            b = w + (row * nb + blk) * bb;
        }
        const float v = type == 12 ? fabsf(f16_bits_to_f32(ld_u16(b))) * 945.0f +
                                         fabsf(f16_bits_to_f32(ld_u16(b + 2))) * 63.0f
                                   : fabsf(f16_bits_to_f32(ld_u16(b + 208))) * 4064.0f;
        bound = fmaxf(bound, v);
    }
    for (int o = 16; o; o >>= 1) bound = fmaxf(bound, __shfl_xor_sync(0xffffffffu, bound, o));
    const uint64_t orow = split ? ((row & 1) ? rows / 2 + row / 2 : row / 2) : row;  // the written row
    if (lane == 0) row_scale[orow] = bound > 0.0f ? ldexpf(1.0f, ilogbf(bound) - 14) : 1.0f;
}

// hi = fp16(v), lo = fp16(v - hi)
__device__ __forceinline__ void split2(float a, float b, __half2 &hi, __half2 &lo)
{
    hi = __floats2half2_rn(a, b);
    const float2 h = __half22float2(hi);
    lo = __floats2half2_rn(__fsub_rn(a, h.x), __fsub_rn(b, h.y));
}

// Weights -> fp16 hi [rows][width] and lo (rows * width further), times
// 1 / row_scale.  One warp per (row, NB consecutive superblocks): lane l forms
// weights 8 l .. 8 l + 7 of each and stores them as one 16-byte vector of each
// half, so a warp writes 512 contiguous bytes of hi and of lo per superblock;
// the blocks' loads are all issued before any is decoded.  Rows are read in
// the tiled layout when tile_rows != 0.  With `split`, the rows come
// interleaved in pairs (gate i, up i) and are written as [gate rows | up
// rows] (row_scale is indexed by the written row).
template <int NB>
__global__ void __launch_bounds__(256) dequant_f16_kernel(const uint8_t *w, int type, uint64_t rows, uint64_t width,
                                                          uint32_t tile_rows, int bb, __half *out,
                                                          const float *row_scale, int split)
{
    pdl_wait();
    const uint64_t nb = width / 256, per_row = nb / NB;
    const uint64_t gw = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (gw < rows * per_row) {
        const uint64_t row = gw / per_row, blk0 = (gw - row * per_row) * NB;
        const uint8_t *b[NB];
#pragma unroll
        for (int k = 0; k < NB; ++k) {
            const uint64_t blk = blk0 + k;
            if (tile_rows) {
                const uint64_t t = row / tile_rows, r = row - t * tile_rows;
                b[k] = w + ((t * nb + blk) * tile_rows + r) * bb;
            } else {
                b[k] = w + (row * nb + blk) * bb;
            }
        }
        float v[NB][8];
        if (type == 12) {
            Q4KLane in[NB];
#pragma unroll
            for (int k = 0; k < NB; ++k) in[k] = q4k_load(b[k], lane);
#pragma unroll
            for (int k = 0; k < NB; ++k) q4k_eight(in[k], lane, v[k]);
        } else {
#pragma unroll
            for (int k = 0; k < NB; ++k) q6k_eight(b[k], lane, v[k]);
        }
        const uint64_t orow = split ? ((row & 1) ? rows / 2 + row / 2 : row / 2) : row;
        const float inv = __frcp_rn(__ldg(row_scale + orow));  // a power of two: exact
#pragma unroll
        for (int k = 0; k < NB; ++k) {
            __half2 hi[4], lo[4];
#pragma unroll
            for (int e = 0; e < 4; ++e)
                split2(__fmul_rn(v[k][2 * e], inv), __fmul_rn(v[k][2 * e + 1], inv), hi[e], lo[e]);
            const size_t o = orow * width + (blk0 + k) * 256 + lane * 8;
            *reinterpret_cast<uint4 *>(out + o) = *reinterpret_cast<const uint4 *>(hi);
            *reinterpret_cast<uint4 *>(out + rows * width + o) = *reinterpret_cast<const uint4 *>(lo);
        }
    }
    pdl_launch_dependents();
}

// Q8_K blocks [m][nb] -> B = the quants as fp16 [m][nb * 256] (exact) and
// b_scale[b][t] = the scale of token t's block b, for t < ld (0 past m).
// One CTA per token of [0, ld).
__global__ void __launch_bounds__(256) q8k_to_f16_kernel(const Q8KBlock *in, int nb, int m, int ld, __half *out,
                                                         float *b_scale)
{
    pdl_wait();
    const int t = blockIdx.x, tid = threadIdx.x;
    const Q8KBlock *row = in + static_cast<size_t>(t) * nb;
    for (int b = tid; b < nb; b += blockDim.x) b_scale[static_cast<size_t>(b) * ld + t] = t < m ? row[b].scale : 0.0f;
    if (t < m) {
        const int width = nb * 256;
        __half2 *dst = reinterpret_cast<__half2 *>(out + static_cast<size_t>(t) * width);
        for (int i = tid; i < width / 4; i += blockDim.x) {
            const int k = 4 * i, b = k >> 8, j = k & 255;
            const char4 q = *reinterpret_cast<const char4 *>(row[b].quants + j);
            dst[2 * i] = __floats2half2_rn(static_cast<float>(q.x), static_cast<float>(q.y));
            dst[2 * i + 1] = __floats2half2_rn(static_cast<float>(q.z), static_cast<float>(q.w));
        }
    }
    pdl_launch_dependents();
}

// ---- host side ------------------------------------------------------------

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encoder()
{
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// 3-D fp16 tensor map [depth][outer][inner] (A: the hi matrix, then the lo
// matrix, depth 2; B: depth 1), box 64 x box_outer x depth, 128-byte swizzle.
bool make_map(CUtensorMap *map, const void *base, uint64_t inner, uint64_t outer, uint32_t box_outer, uint32_t depth)
{
    EncodeTiledFn enc = encoder();
    if (!enc || (reinterpret_cast<uintptr_t>(base) & 15u) || inner % 64) return false;
    const cuuint64_t dims[3] = {inner, outer, depth};
    const cuuint64_t strides[2] = {inner * 2, inner * outer * 2};
    const cuuint32_t box[3] = {static_cast<cuuint32_t>(kTcK), box_outer, depth};
    const cuuint32_t estr[3] = {1, 1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN>
cudaError_t launch_tc_bn(const void *a16, const void *b16, const TcGemm &p, cudaStream_t s)
{
    CUtensorMap ma, mb;
    if (!make_map(&ma, a16, p.k, p.n, kTcRows, 2) || !make_map(&mb, b16, p.k, p.m, BN, 1)) return cudaErrorInvalidValue;
    static std::once_flag once;
    static cudaError_t attr = cudaSuccess;
    std::call_once(once, [] {
        attr = cudaFuncSetAttribute(tc_gemm_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(tc_smem_bytes<BN>()));
    });
    if (attr != cudaSuccess) return attr;
    TcArgs g;
    g.out = p.out;
    g.ld = p.ld;
    g.n = p.n;
    g.m = p.m;
    g.k = p.k;
    g.b_scale = p.b_scale;
    g.b_scale_ld = p.b_scale_ld;
    g.row_scale = p.row_scale;
    g.accumulate = p.accumulate;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(((p.n + kTcRows - 1) / kTcRows) * ((p.m + BN - 1) / BN)));
    cfg.blockDim = dim3(TcCfg<BN>::kThreads);
    cfg.dynamicSmemBytes = tc_smem_bytes<BN>();
    cfg.stream = s;
    cudaLaunchAttribute la[1];
    la[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    la[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = la;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, tc_gemm_kernel<BN>, ma, mb, g);
}

}  // namespace

int tc_token_tile(int) { return 256; }  // b_scale rows are padded to a multiple of this

bool tc_weight_type(int type) { return type == 12 || type == 14; }  // Q4_K, Q6_K

cudaError_t launch_dequant_f16(const void *w, int type, uint64_t rows, uint64_t width, uint32_t tile_rows, int bb,
                               void *out, float *row_scale, int split, cudaStream_t s)
{
    if (!tc_weight_type(type) || width % 256 || (split && rows % 2)) return cudaErrorInvalidValue;
    {
        // the rows' powers of two first, in the order the rows are written
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(static_cast<unsigned>((rows * 32 + 255) / 256));
        cfg.blockDim = dim3(256);
        cfg.stream = s;
        cudaLaunchAttribute la[1];
        la[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        la[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = la;
        cfg.numAttrs = 1;
        const cudaError_t e = cudaLaunchKernelEx(&cfg, row_scale_kernel, static_cast<const uint8_t *>(w), type, rows,
                                                 width / 256, tile_rows, bb, row_scale, split);
        if (e != cudaSuccess) return e;
    }
    const bool four = (width / 256) % 4 == 0;  // four superblocks a warp where they divide the row
    const uint64_t warps = rows * (width / 256) / (four ? 4 : 1);
    const unsigned grid = static_cast<unsigned>((warps * 32 + 255) / 256);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute la[1];
    la[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    la[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = la;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, four ? dequant_f16_kernel<4> : dequant_f16_kernel<1>,
                              static_cast<const uint8_t *>(w), type, rows, width, tile_rows,
                              bb, static_cast<__half *>(out), static_cast<const float *>(row_scale), split);
}

cudaError_t launch_q8k_to_f16(const void *q8, int nb, int m, int ld, void *out, float *b_scale, cudaStream_t s)
{
    if (m < 1 || ld < m || ld % tc_token_tile(m)) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(ld));
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute la[1];
    la[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    la[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = la;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, q8k_to_f16_kernel, static_cast<const Q8KBlock *>(q8), nb, m, ld,
                              static_cast<__half *>(out), b_scale);
}

cudaError_t launch_tc_gemm(const void *a16, const void *b16, const TcGemm &p, cudaStream_t s)
{
    if (p.k % 256 || p.n < 1 || p.m < 1 || !p.out || !p.b_scale || p.b_scale_ld < p.m ||
        p.b_scale_ld % tc_token_tile(p.m))
        return cudaErrorInvalidValue;
    // 256-token tiles for prompts (twice the MMA work per staged A tile),
    // 128 for short batches (less padding)
    return p.m > 128 ? launch_tc_bn<256>(a16, b16, p, s) : launch_tc_bn<128>(a16, b16, p, s);
}

cudaError_t read_and_clear_tc_status(int *status)
{
    cudaError_t e = cudaMemcpyFromSymbol(status, g_tc_status, sizeof(int));
    if (e != cudaSuccess) return e;
    const int zero = 0;
    return cudaMemcpyToSymbol(g_tc_status, &zero, sizeof(int));
}

}  // namespace q38
