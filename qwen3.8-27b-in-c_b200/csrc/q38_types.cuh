// q38_types.cuh - per-format superblock decoders for the Q8_K integer path.
//
// A decoder works on one 256-element superblock of one weight row that sits
// in shared memory, against MT Q8_K activation blocks held in registers (one
// per token).  For each token it produces the two integer sums the upstream
// kernels form (w, x) and the superblock's float contribution v, using the
// same per-block formula as the upstream scalar code (src/qwen38/
// qwen38_quant.c, cited per type).  Activation words are indexed with
// compile-time constants only, so they stay in registers.
#pragma once

#include "q38_device.cuh"

namespace q38 {

enum : int {
    kF32 = 0, kF16 = 1, kQ8_0 = 8, kQ2_K = 10, kQ3_K = 11, kQ4_K = 12, kQ5_K = 13, kQ6_K = 14,
    kIQ2_XXS = 16, kIQ2_XS = 17, kIQ3_XXS = 18, kIQ1_S = 19, kIQ4_NL = 20, kIQ3_S = 21,
    kIQ2_S = 22, kIQ4_XS = 23, kIQ1_M = 29, kBF16 = 30
};

// Device copy of an upstream Q38Q8KBlock (292 bytes, 4-byte aligned).
struct Q8KBlock {
    float scale;
    int8_t quants[256];
    int16_t sums[16];
};

// Activation block: 64 words of int8 quants, up to 16 words of per-format
// precomputed sums ("aux", see each decoder's load) and the block scale.  The
// same layout is used in registers (one block per thread) and in shared memory
// (one block per column, read by every thread of a CTA).
struct Act {
    uint32_t q[64];
    uint32_t aux[16];
    float xs;
    uint32_t pad[3];
};
static_assert(sizeof(Act) == 336, "shared-memory activation slot is 336 bytes");

__device__ __forceinline__ void load_act_base(Act &a, const Q8KBlock *g)
{
    const uint32_t *w = reinterpret_cast<const uint32_t *>(g->quants);
#pragma unroll
    for (int i = 0; i < 64; ++i) a.q[i] = __ldg(w + i);
    a.xs = __ldg(&g->scale);
}

__device__ __forceinline__ void zero_act(Act &a)
{
#pragma unroll
    for (int i = 0; i < 64; ++i) a.q[i] = 0u;
#pragma unroll
    for (int i = 0; i < 16; ++i) a.aux[i] = 0u;
    a.xs = 0.0f;
}

// Accessors over MT activation blocks: registers (RegActs) or shared memory
// (SmemActs, one pointer per token).  Indices are compile-time constants.
template <int MT>
struct RegActs {
    const Act (&a)[MT];
    __device__ __forceinline__ uint4 q4(int t, int j) const
    {
        return make_uint4(a[t].q[4 * j], a[t].q[4 * j + 1], a[t].q[4 * j + 2], a[t].q[4 * j + 3]);
    }
    __device__ __forceinline__ uint4 aux4(int t, int j) const
    {
        return make_uint4(a[t].aux[4 * j], a[t].aux[4 * j + 1], a[t].aux[4 * j + 2], a[t].aux[4 * j + 3]);
    }
    __device__ __forceinline__ uint32_t q(int t, int i) const { return a[t].q[i]; }
    __device__ __forceinline__ uint32_t aux(int t, int i) const { return a[t].aux[i]; }
    __device__ __forceinline__ float xs(int t) const { return a[t].xs; }
};

template <int MT>
struct SmemActs {
    const Act *p[MT];  // 16-byte aligned slots in shared memory
    __device__ __forceinline__ uint4 q4(int t, int j) const { return reinterpret_cast<const uint4 *>(p[t]->q)[j]; }
    __device__ __forceinline__ uint4 aux4(int t, int j) const
    {
        return reinterpret_cast<const uint4 *>(p[t]->aux)[j];
    }
    __device__ __forceinline__ uint32_t q(int t, int i) const { return p[t]->q[i]; }
    __device__ __forceinline__ uint32_t aux(int t, int i) const { return p[t]->aux[i]; }
    __device__ __forceinline__ float xs(int t) const { return p[t]->xs; }
};

// Sixteen int16 bsums of a Q8_K block.
__device__ __forceinline__ int bsum(const Q8KBlock *g, int k) { return __ldg(&g->sums[k]); }

__device__ __forceinline__ int lo16(uint32_t p) { return static_cast<int>(static_cast<int16_t>(p & 0xFFFFu)); }
__device__ __forceinline__ int hi16(uint32_t p) { return static_cast<int>(static_cast<int16_t>(p >> 16)); }

__device__ __forceinline__ uint32_t pack16(int lo, int hi)
{
    return (static_cast<uint32_t>(lo) & 0xFFFFu) | (static_cast<uint32_t>(hi) << 16);
}

// ===========================================================================
// Q4_K (144 B: fp16 d, fp16 dmin, 12 B packed 6-bit scales/mins, 128 B quants)
// qwen38_quant.c:1546-1634 (integer path), :131-143 (scale unpack).
// ===========================================================================
struct DecQ4K {
    static constexpr int kBytes = 144;
    static constexpr int kAlign = 16;
    // aux[j] = int16 pair (bsum[4j] + bsum[4j+1], bsum[4j+2] + bsum[4j+3]): the
    // activation sums of sub-blocks 2j and 2j+1, weighted by the 6-bit mins.
    __device__ static void aux(Act &a, const Q8KBlock *g)
    {
#pragma unroll
        for (int j = 0; j < 4; ++j)
            a.aux[j] = pack16(bsum(g, 4 * j) + bsum(g, 4 * j + 1), bsum(g, 4 * j + 2) + bsum(g, 4 * j + 3));
    }
    // Same, from the raw bsums staged in aux[8..15] (int16 pairs).
    __device__ static void aux_from_raw(Act &a)
    {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t p0 = a.aux[8 + 2 * j], p1 = a.aux[9 + 2 * j];
            a.aux[j] = pack16(lo16(p0) + hi16(p0), lo16(p1) + hi16(p1));
        }
    }
    __device__ static void load(Act &a, const Q8KBlock *g) { load_act_base(a, g); aux(a, g); }
    __device__ static void zero(Act &a) { zero_act(a); }
    template <int MT, class A>
    __device__ static void block(const uint8_t *blk, const A &a, int (&w)[MT], int (&x)[MT], float (&v)[MT])
    {
        const uint4 *p = reinterpret_cast<const uint4 *>(blk);
        const uint4 h = p[0];
        const uint32_t s0 = h.y, s1 = h.z, s2 = h.w;
        const uint32_t sc_lo = s0 & 0x3F3F3F3Fu;
        const uint32_t m_lo = s1 & 0x3F3F3F3Fu;
        const uint32_t sc_hi = (s2 & 0x0F0F0F0Fu) | ((s0 >> 2) & 0x30303030u);
        const uint32_t m_hi = ((s2 >> 4) & 0x0F0F0F0Fu) | ((s1 >> 2) & 0x30303030u);
        int wl[MT], wh[MT];
#pragma unroll
        for (int t = 0; t < MT; ++t) wl[t] = wh[t] = 0;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const uint4 qa = p[1 + 2 * c], qb = p[2 + 2 * c];
            const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
            const uint32_t scw = c < 2 ? sc_lo : sc_hi;
            const int sc0 = static_cast<int>(byte_of(scw, (2 * c) & 3));
            const int sc1 = static_cast<int>(byte_of(scw, (2 * c + 1) & 3));
#pragma unroll
            for (int t = 0; t < MT; ++t) {
                const uint4 x0 = a.q4(t, 4 * c), x1 = a.q4(t, 4 * c + 1);
                const uint4 x2 = a.q4(t, 4 * c + 2), x3 = a.q4(t, 4 * c + 3);
                const uint32_t xl[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
                const uint32_t xh[8] = {x2.x, x2.y, x2.z, x2.w, x3.x, x3.y, x3.z, x3.w};
                // two independent chains per half for instruction-level parallelism
                int dl0 = 0, dl1 = 0, dh0 = 0, dh1 = 0;
#pragma unroll
                for (int i = 0; i < 8; i += 2) {
                    dl0 = dp4a_ss(q[i] & 0x0F0F0F0Fu, xl[i], dl0);
                    dl1 = dp4a_ss(q[i + 1] & 0x0F0F0F0Fu, xl[i + 1], dl1);
                    // high nibbles kept in place: unsigned bytes 16*q
                    dh0 = dp4a_us(q[i] & 0xF0F0F0F0u, xh[i], dh0);
                    dh1 = dp4a_us(q[i + 1] & 0xF0F0F0F0u, xh[i + 1], dh1);
                }
                wl[t] += sc0 * (dl0 + dl1);
                wh[t] += sc1 * (dh0 + dh1);
            }
        }
        const float d = f16_bits_to_f32(h.x & 0xFFFFu);
        const float dmin = f16_bits_to_f32(h.x >> 16);
#pragma unroll
        for (int t = 0; t < MT; ++t) {
            w[t] = wl[t] + (wh[t] >> 4);  // wh is an exact multiple of 16
            const uint4 pm = a.aux4(t, 0);
            int m = dp2a_lo_ss(pm.x, m_lo, 0);
            m = dp2a_hi_ss(pm.y, m_lo, m);
            m = dp2a_lo_ss(pm.z, m_hi, m);
            m = dp2a_hi_ss(pm.w, m_hi, m);
            x[t] = m;
            const float dd = __fmul_rn(d, a.xs(t)), dm = __fmul_rn(dmin, a.xs(t));
            v[t] = __fsub_rn(__fmul_rn(dd, static_cast<float>(w[t])), __fmul_rn(dm, static_cast<float>(m)));
        }
    }
    // Part j of L (L = 2 or 4) of `block`: the integer sums of sub-block pairs
    // c = j * 4 / L .. (j + 1) * 4 / L - 1 only.  Integer sums add exactly, so
    // the parts of a row, added and passed to `finish`, give bit for bit what
    // `block` gives.
    template <int MT, int L, class A>
    __device__ static void block_part(const uint8_t *blk, const A &a, int j, int (&w)[MT], int (&x)[MT])
    {
        constexpr int kC = 4 / L;
        const uint4 *p = reinterpret_cast<const uint4 *>(blk);
        const uint4 h = p[0];
        const uint32_t s0 = h.y, s1 = h.z, s2 = h.w;
        const uint32_t sc_lo = s0 & 0x3F3F3F3Fu;
        const uint32_t m_lo = s1 & 0x3F3F3F3Fu;
        const uint32_t sc_hi = (s2 & 0x0F0F0F0Fu) | ((s0 >> 2) & 0x30303030u);
        const uint32_t m_hi = ((s2 >> 4) & 0x0F0F0F0Fu) | ((s1 >> 2) & 0x30303030u);
#pragma unroll
        for (int t = 0; t < MT; ++t) w[t] = x[t] = 0;
#pragma unroll
        for (int cc = 0; cc < kC; ++cc) {
            const int c = j * kC + cc;
            const uint4 qa = p[1 + 2 * c], qb = p[2 + 2 * c];
            const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
            const uint32_t scw = c < 2 ? sc_lo : sc_hi;
            const int sc0 = static_cast<int>(byte_of(scw, (2 * c) & 3));
            const int sc1 = static_cast<int>(byte_of(scw, (2 * c + 1) & 3));
            // mins of sub-blocks 2c, 2c + 1 moved to bytes 0, 1
            const uint32_t mw = (c < 2 ? m_lo : m_hi) >> (16 * (c & 1));
#pragma unroll
            for (int t = 0; t < MT; ++t) {
                const uint4 x0 = a.q4(t, 4 * c), x1 = a.q4(t, 4 * c + 1);
                const uint4 x2 = a.q4(t, 4 * c + 2), x3 = a.q4(t, 4 * c + 3);
                const uint32_t xl[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
                const uint32_t xh[8] = {x2.x, x2.y, x2.z, x2.w, x3.x, x3.y, x3.z, x3.w};
                int dl0 = 0, dl1 = 0, dh0 = 0, dh1 = 0;
#pragma unroll
                for (int i = 0; i < 8; i += 2) {
                    dl0 = dp4a_ss(q[i] & 0x0F0F0F0Fu, xl[i], dl0);
                    dl1 = dp4a_ss(q[i + 1] & 0x0F0F0F0Fu, xl[i + 1], dl1);
                    dh0 = dp4a_us(q[i] & 0xF0F0F0F0u, xh[i], dh0);
                    dh1 = dp4a_us(q[i + 1] & 0xF0F0F0F0u, xh[i + 1], dh1);
                }
                // the high-nibble sum is an exact multiple of 16
                w[t] += sc0 * (dl0 + dl1) + ((sc1 * (dh0 + dh1)) >> 4);
                x[t] = dp2a_lo_ss(a.aux(t, c), mw, x[t]);
            }
        }
    }
    // The float value of a superblock from its whole integer sums.
    template <int MT, class A>
    __device__ static void finish(const uint8_t *blk, const A &a, const int (&w)[MT], const int (&x)[MT],
                                  float (&v)[MT])
    {
        const uint32_t hx = *reinterpret_cast<const uint32_t *>(blk);
        const float d = f16_bits_to_f32(hx & 0xFFFFu);
        const float dmin = f16_bits_to_f32(hx >> 16);
#pragma unroll
        for (int t = 0; t < MT; ++t) {
            const float dd = __fmul_rn(d, a.xs(t)), dm = __fmul_rn(dmin, a.xs(t));
            v[t] = __fsub_rn(__fmul_rn(dd, static_cast<float>(w[t])), __fmul_rn(dm, static_cast<float>(x[t])));
        }
    }
};

// ===========================================================================
// Q6_K (210 B: 128 B low nibbles, 64 B high 2-bit pairs, 16 int8 scales, fp16 d)
// qwen38_quant.c:1727-1833 (the AVX2 form: unsigned q, minus 32*sum(sc*bsum)).
// ===========================================================================
struct DecQ6K {
    static constexpr int kBytes = 210;
    static constexpr int kAlign = 2;
    // aux[j] = int16 pair (bsum[2j], bsum[2j+1]).
    __device__ static void aux(Act &a, const Q8KBlock *g)
    {
#pragma unroll
        for (int j = 0; j < 8; ++j) a.aux[j] = pack16(bsum(g, 2 * j), bsum(g, 2 * j + 1));
    }
    __device__ static void aux_from_raw(Act &a)
    {
#pragma unroll
        for (int j = 0; j < 8; ++j) a.aux[j] = a.aux[8 + j];
    }
    __device__ static void load(Act &a, const Q8KBlock *g) { load_act_base(a, g); aux(a, g); }
    __device__ static void zero(Act &a) { zero_act(a); }
    template <int MT, class A>
    __device__ static void block(const uint8_t *blk, const A &a, int (&w)[MT], int (&x)[MT], float (&v)[MT])
    {
        uint32_t tail[5];  // bytes 192..211: 16 int8 scales, fp16 d (+2 past the end)
        lds_words<5>(blk + 192, tail);
        int acc[MT];
#pragma unroll
        for (int t = 0; t < MT; ++t) acc[t] = 0;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            uint32_t ql[16], qh[8];
            lds_words<16>(blk + 64 * h, ql);
            lds_words<8>(blk + 128 + 32 * h, qh);
#pragma unroll
            for (int qq = 0; qq < 4; ++qq) {
                const int s = 4 * h + qq;
                uint32_t val[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const uint32_t lw = ql[(qq & 1) * 8 + i];
                    const uint32_t nib = qq < 2 ? (lw & 0x0F0F0F0Fu) : ((lw >> 4) & 0x0F0F0F0Fu);
                    val[i] = nib | (((qh[i] >> (2 * qq)) & 0x03030303u) << 4);
                }
                const int g0 = 8 * h + 2 * qq;
                const int sc0 = sbyte_of(tail[g0 / 4], g0 & 3);
                const int sc1 = sbyte_of(tail[(g0 + 1) / 4], (g0 + 1) & 3);
#pragma unroll
                for (int t = 0; t < MT; ++t) {
                    const uint4 x0 = a.q4(t, 2 * s), x1 = a.q4(t, 2 * s + 1);
                    const int da = dp4a_us(val[0], x0.x, 0) + dp4a_us(val[1], x0.y, 0) +
                                   (dp4a_us(val[2], x0.z, 0) + dp4a_us(val[3], x0.w, 0));
                    const int db = dp4a_us(val[4], x1.x, 0) + dp4a_us(val[5], x1.y, 0) +
                                   (dp4a_us(val[6], x1.z, 0) + dp4a_us(val[7], x1.w, 0));
                    acc[t] += sc0 * da + sc1 * db;
                }
            }
        }
        const float d = f16_bits_to_f32(tail[4] & 0xFFFFu);
#pragma unroll
        for (int t = 0; t < MT; ++t) {
            const uint4 b0 = a.aux4(t, 0), b1 = a.aux4(t, 1);
            const uint32_t bs[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
            int off = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                off = dp2a_lo_ss(bs[2 * j], tail[j], off);
                off = dp2a_hi_ss(bs[2 * j + 1], tail[j], off);
            }
            w[t] = acc[t] - 32 * off;
            x[t] = 0;
            v[t] = __fmul_rn(__fmul_rn(d, a.xs(t)), static_cast<float>(w[t]));
        }
    }
    // Part j of L (L = 2 or 4) of `block`: L = 2 takes half h = j (sub-blocks
    // 8h .. 8h + 7), L = 4 half h = j / 2 and quarter groups qq = j % 2 and
    // j % 2 + 2 (both read low-bit words 8 (j % 2) .. + 7 of the half).  The
    // 32 * sum(sc * bsum) offset is split the same way; parts add exactly.
    template <int MT, int L, class A>
    __device__ static void block_part(const uint8_t *blk, const A &a, int j, int (&w)[MT], int (&x)[MT])
    {
        static_assert(L == 2 || L == 4, "Q6_K splits in 2 or 4 parts");
        constexpr int kQq = L == 4 ? 2 : 4;
        const int h = L == 4 ? (j >> 1) : j;
        const int qsel = L == 4 ? (j & 1) : 0;
        const int8_t *scales = reinterpret_cast<const int8_t *>(blk + 192);
        uint32_t ql[L == 4 ? 8 : 16], qh[8];
        lds_words<L == 4 ? 8 : 16>(blk + 64 * h + 32 * qsel, ql);
        lds_words<8>(blk + 128 + 32 * h, qh);
        int acc[MT], off[MT];
#pragma unroll
        for (int t = 0; t < MT; ++t) acc[t] = off[t] = 0;
#pragma unroll
        for (int k = 0; k < kQq; ++k) {
            const int qq = L == 4 ? qsel + 2 * k : k;
            const bool high = L == 4 ? k == 1 : k >= 2;  // nibble of the low-bit words
            const int lw0 = L == 4 ? 0 : (k & 1) * 8;
            uint32_t val[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint32_t lw = ql[lw0 + i];
                const uint32_t nib = high ? ((lw >> 4) & 0x0F0F0F0Fu) : (lw & 0x0F0F0F0Fu);
                val[i] = nib | (((qh[i] >> (2 * qq)) & 0x03030303u) << 4);
            }
            const int s = 4 * h + qq;
            const int sc0 = scales[2 * s], sc1 = scales[2 * s + 1];
#pragma unroll
            for (int t = 0; t < MT; ++t) {
                const uint4 x0 = a.q4(t, 2 * s), x1 = a.q4(t, 2 * s + 1);
                const int da = dp4a_us(val[0], x0.x, 0) + dp4a_us(val[1], x0.y, 0) +
                               (dp4a_us(val[2], x0.z, 0) + dp4a_us(val[3], x0.w, 0));
                const int db = dp4a_us(val[4], x1.x, 0) + dp4a_us(val[5], x1.y, 0) +
                               (dp4a_us(val[6], x1.z, 0) + dp4a_us(val[7], x1.w, 0));
                acc[t] += sc0 * da + sc1 * db;
                const uint32_t bw = a.aux(t, s);  // bsums of sub-blocks 2s, 2s + 1
                off[t] += sc0 * lo16(bw) + sc1 * hi16(bw);
            }
        }
#pragma unroll
        for (int t = 0; t < MT; ++t) {
            w[t] = acc[t] - 32 * off[t];
            x[t] = 0;
        }
    }
    template <int MT, class A>
    __device__ static void finish(const uint8_t *blk, const A &a, const int (&w)[MT], const int (&)[MT],
                                  float (&v)[MT])
    {
        const float d = f16_bits_to_f32(*reinterpret_cast<const unsigned short *>(blk + 208));
#pragma unroll
        for (int t = 0; t < MT; ++t) v[t] = __fmul_rn(__fmul_rn(d, a.xs(t)), static_cast<float>(w[t]));
    }
};

// ===========================================================================
// IQ2_S (82 B: fp16 d, 32 B grid index low bytes, 32 B signs, 8 B index high
// bits, 8 B 4-bit scales).  qwen38_quant.c:664-756.  `grid` is the 1024-entry
// magnitude table expanded into shared memory (8 bytes per entry).
// ===========================================================================
struct DecIQ2S {
    static constexpr int kBytes = 82;
    static constexpr int kAlign = 2;
    __device__ static void aux(Act &, const Q8KBlock *) {}
    __device__ static void aux_from_raw(Act &) {}
    __device__ static void load(Act &a, const Q8KBlock *g) { load_act_base(a, g); }
    __device__ static void zero(Act &a) { zero_act(a); }
    template <int MT, class A>
    __device__ static void block(const uint8_t *blk, const A &a, int (&w)[MT], int (&x)[MT], float (&v)[MT],
                                 const uint2 *grid)
    {
        uint32_t raw[21];  // bytes 0..83
        lds_words<21>(blk, raw);
        // byte k of the block
#define Q38_B(k) byte_of(raw[(k) >> 2], (k) & 3)
        int acc[MT];
#pragma unroll
        for (int t = 0; t < MT; ++t) acc[t] = 0;
#pragma unroll
        for (int g = 0; g < 8; ++g) {
            const uint32_t qh = Q38_B(66 + g);
            const uint32_t scb = Q38_B(74 + g);
            const int s0 = 1 + 2 * static_cast<int>(scb & 15u);
            const int s1 = 1 + 2 * static_cast<int>(scb >> 4);
            int part[MT][2];
#pragma unroll
            for (int t = 0; t < MT; ++t) part[t][0] = part[t][1] = 0;
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                const uint32_t gi = Q38_B(2 + 4 * g + s) | ((qh << (8 - 2 * s)) & 0x300u);
                const uint2 e = grid[gi];
                const uint32_t sg = Q38_B(34 + 4 * g + s);
                const uint32_t lo = apply_signs(e.x, sign_mask4(sg & 15u));
                const uint32_t hi = apply_signs(e.y, sign_mask4(sg >> 4));
#pragma unroll
                for (int t = 0; t < MT; ++t) {
                    int d = dp4a_ss(lo, a.q(t, 8 * g + 2 * s), part[t][s / 2]);
                    part[t][s / 2] = dp4a_ss(hi, a.q(t, 8 * g + 2 * s + 1), d);
                }
            }
#pragma unroll
            for (int t = 0; t < MT; ++t) acc[t] += s0 * part[t][0] + s1 * part[t][1];
        }
#undef Q38_B
        const float d = __fmul_rn(0.125f, f16_bits_to_f32(raw[0] & 0xFFFFu));
#pragma unroll
        for (int t = 0; t < MT; ++t) {
            w[t] = acc[t];
            x[t] = 0;
            v[t] = __fmul_rn(__fmul_rn(d, a.xs(t)), static_cast<float>(acc[t]));
        }
    }
};

// ===========================================================================
// IQ1_S (50 B: fp16 d, 32 B grid index low bytes, 8 x u16 {3-bit index highs,
// 3-bit scale, delta sign}).  qwen38_quant.c:1177-1253.  `grid` is the
// 2048-entry {-1,0,1} table expanded into shared memory.
// ===========================================================================
struct DecIQ1S {
    static constexpr int kBytes = 50;
    static constexpr int kAlign = 2;
    // aux[g] = bsum[2g] + bsum[2g+1] (the 32-element group sums).
    __device__ static void aux(Act &a, const Q8KBlock *g)
    {
#pragma unroll
        for (int j = 0; j < 8; ++j) a.aux[j] = static_cast<uint32_t>(bsum(g, 2 * j) + bsum(g, 2 * j + 1));
    }
    __device__ static void aux_from_raw(Act &a)
    {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t p = a.aux[8 + j];
            a.aux[j] = static_cast<uint32_t>(lo16(p) + hi16(p));
        }
    }
    __device__ static void load(Act &a, const Q8KBlock *g) { load_act_base(a, g); aux(a, g); }
    __device__ static void zero(Act &a) { zero_act(a); }
    template <int MT, class A>
    __device__ static void block(const uint8_t *blk, const A &a, int (&w)[MT], int (&x)[MT], float (&v)[MT],
                                 const uint2 *grid)
    {
        uint32_t raw[13];  // bytes 0..51
        lds_words<13>(blk, raw);
#define Q38_B(k) byte_of(raw[(k) >> 2], (k) & 3)
        int acc[MT], cor[MT];
#pragma unroll
        for (int t = 0; t < MT; ++t) acc[t] = cor[t] = 0;
#pragma unroll
        for (int g = 0; g < 8; ++g) {
            const uint32_t qh = Q38_B(34 + 2 * g) | (Q38_B(35 + 2 * g) << 8);
            const int scale = 1 + 2 * static_cast<int>((qh >> 12) & 7u);
            const int sd = (qh & 0x8000u) ? -scale : scale;
            int dot[MT];
#pragma unroll
            for (int t = 0; t < MT; ++t) dot[t] = 0;
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                const uint32_t gi = Q38_B(2 + 4 * g + s) | (((qh >> (3 * s)) & 7u) << 8);
                const uint2 e = grid[gi];
#pragma unroll
                for (int t = 0; t < MT; ++t) {
                    dot[t] = dp4a_ss(e.x, a.q(t, 8 * g + 2 * s), dot[t]);
                    dot[t] = dp4a_ss(e.y, a.q(t, 8 * g + 2 * s + 1), dot[t]);
                }
            }
#pragma unroll
            for (int t = 0; t < MT; ++t) {
                acc[t] += scale * dot[t];
                cor[t] += sd * static_cast<int>(a.aux(t, g));
            }
        }
#undef Q38_B
        const float d = f16_bits_to_f32(raw[0] & 0xFFFFu);
#pragma unroll
        for (int t = 0; t < MT; ++t) {
            w[t] = acc[t];
            x[t] = cor[t];
            const float dd = __fmul_rn(d, a.xs(t));
            v[t] = __fmul_rn(dd, __fadd_rn(static_cast<float>(acc[t]),
                                           __fmul_rn(0.125f, static_cast<float>(cor[t]))));
        }
    }
};

// ===========================================================================
// IQ1_M (56 B: 32 B grid index low bytes, 16 B {3-bit index highs, delta
// signs}, 8 B {3-bit scales, fp16 super-scale in the top nibbles}).
// qwen38_quant.c:1388-1544.  The correction uses 8-element activation sums.
// ===========================================================================
struct DecIQ1M {
    static constexpr int kBytes = 56;
    static constexpr int kAlign = 8;
    // aux[j] = int16 pair of the eight-element quant sums of sections 2j, 2j+1
    // (computed from the quants, which must already be in `a`).
    __device__ static void aux(Act &a, const Q8KBlock *)
    {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const int lo = dp4a_ss(a.q[4 * j], 0x01010101u, dp4a_ss(a.q[4 * j + 1], 0x01010101u, 0));
            const int hi = dp4a_ss(a.q[4 * j + 2], 0x01010101u, dp4a_ss(a.q[4 * j + 3], 0x01010101u, 0));
            a.aux[j] = pack16(lo, hi);
        }
    }
    __device__ static void aux_from_raw(Act &a) { aux(a, nullptr); }
    __device__ static void load(Act &a, const Q8KBlock *g) { load_act_base(a, g); aux(a, g); }
    __device__ static void zero(Act &a) { zero_act(a); }
    __device__ static void load_raw(const uint8_t *blk, uint32_t (&raw)[14])
    {
        const uint2 *p = reinterpret_cast<const uint2 *>(blk);
#pragma unroll
        for (int i = 0; i < 7; ++i) {
            const uint2 u = p[i];
            raw[2 * i] = u.x;
            raw[2 * i + 1] = u.y;
        }
    }
    // The integer sums of groups g0 .. g1 - 1 (32 elements each): acc = the
    // scaled grid dot products, cor = the scaled +-1 delta corrections.
    template <int MT, int G0, int G1, class A>
    __device__ static void groups(const uint32_t (&raw)[14], const A &a, int (&acc)[MT], int (&cor)[MT],
                                  const uint2 *grid)
    {
#define Q38_B(k) byte_of(raw[(k) >> 2], (k) & 3)
#pragma unroll
        for (int g = G0; g < G1; ++g) {
            const uint32_t scw = (g < 4 ? raw[12] : raw[13]) >> (16 * ((g / 2) & 1));
            const int shift = 6 * (g % 2);
            const int sc[2] = {1 + 2 * static_cast<int>((scw >> shift) & 7u),
                               1 + 2 * static_cast<int>((scw >> (shift + 3)) & 7u)};
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                const uint32_t hb = Q38_B(32 + 2 * g + s / 2);
                const uint32_t gi = Q38_B(4 * g + s) | ((hb << (8 - 4 * (s % 2))) & 0x700u);
                const bool neg = (hb & (s % 2 ? 0x80u : 0x08u)) != 0;
                const int scl = sc[s / 2];
                const uint2 e = grid[gi];
#pragma unroll
                for (int t = 0; t < MT; ++t) {
                    int d = dp4a_ss(e.x, a.q(t, 8 * g + 2 * s), 0);
                    d = dp4a_ss(e.y, a.q(t, 8 * g + 2 * s + 1), d);
                    acc[t] += scl * d;
                    const uint32_t pair = a.aux(t, (4 * g + s) >> 1);
                    const int sec = ((4 * g + s) & 1) ? static_cast<int>(static_cast<int16_t>(pair >> 16))
                                                      : static_cast<int>(static_cast<int16_t>(pair & 0xFFFFu));
                    cor[t] += neg ? -scl * sec : scl * sec;
                }
            }
        }
#undef Q38_B
    }
    template <int MT, class A>
    __device__ static void combine(const uint32_t (&raw)[14], const A &a, const int (&acc)[MT], const int (&cor)[MT],
                                   float (&v)[MT])
    {
        const uint32_t sb = ((raw[12] & 0xFFFFu) >> 12) | (((raw[12] >> 16) >> 8) & 0x00F0u) |
                            (((raw[13] & 0xFFFFu) >> 4) & 0x0F00u) | ((raw[13] >> 16) & 0xF000u);
        const float d = f16_bits_to_f32(sb);
#pragma unroll
        for (int t = 0; t < MT; ++t) {
            const float dd = __fmul_rn(d, a.xs(t));
            v[t] = __fmul_rn(dd, __fadd_rn(static_cast<float>(acc[t]),
                                           __fmul_rn(0.125f, static_cast<float>(cor[t]))));
        }
    }
    template <int MT, class A>
    __device__ static void block(const uint8_t *blk, const A &a, int (&w)[MT], int (&x)[MT], float (&v)[MT],
                                 const uint2 *grid)
    {
        uint32_t raw[14];
        load_raw(blk, raw);
        int acc[MT], cor[MT];
#pragma unroll
        for (int t = 0; t < MT; ++t) acc[t] = cor[t] = 0;
        groups<MT, 0, 8>(raw, a, acc, cor, grid);
#pragma unroll
        for (int t = 0; t < MT; ++t) {
            w[t] = acc[t];
            x[t] = cor[t];
        }
        combine<MT>(raw, a, acc, cor, v);
    }
    // Part j of L (2 or 4) of `block`: groups 8j / L .. 8(j + 1) / L; the parts'
    // integer sums add exactly, so `finish` on the totals equals `block`.
    template <int MT, int L, class A>
    __device__ static void block_part(const uint8_t *blk, const A &a, int j, int (&w)[MT], int (&x)[MT],
                                      const uint2 *grid)
    {
        static_assert(L == 2 || L == 4, "IQ1_M splits in 2 or 4 parts");
        uint32_t raw[14];
        load_raw(blk, raw);
#pragma unroll
        for (int t = 0; t < MT; ++t) w[t] = x[t] = 0;
        if constexpr (L == 2) {
            if (j == 0) groups<MT, 0, 4>(raw, a, w, x, grid);
            else groups<MT, 4, 8>(raw, a, w, x, grid);
        } else {
            if (j == 0) groups<MT, 0, 2>(raw, a, w, x, grid);
            else if (j == 1) groups<MT, 2, 4>(raw, a, w, x, grid);
            else if (j == 2) groups<MT, 4, 6>(raw, a, w, x, grid);
            else groups<MT, 6, 8>(raw, a, w, x, grid);
        }
    }
    template <int MT, class A>
    __device__ static void finish(const uint8_t *blk, const A &a, const int (&w)[MT], const int (&x)[MT],
                                  float (&v)[MT])
    {
        uint32_t raw[14];
        load_raw(blk, raw);
        combine<MT>(raw, a, w, x, v);
    }
};

}  // namespace q38
