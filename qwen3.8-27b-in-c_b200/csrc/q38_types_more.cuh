// q38_types_more.cuh - superblock decoders of the secondary Q8_K-path types
// (the upstream's Q2_K, Q3_K, Q5_K, IQ2_XXS, IQ2_XS, IQ3_XXS, IQ3_S, IQ4_XS and
// IQ4_NL kernels, src/qwen38/qwen38_quant.c), with the interface of the
// decoders in q38_types.cuh: per token the upstream's integer sums (w, x) of
// the superblock and its float contribution v by the upstream's per-block
// formula.  Integer sums are formed with dp4a on bytes rebuilt from the
// packed fields; every product and sum is exact, so the sums equal the
// upstream's whatever the order.  The codebook types read `grid`, the
// per-CTA shared-memory expansion of their table (q38_grid.cuh): 8 signed or
// unsigned byte values per entry (IQ2), or 4 in the low word (IQ3).
#pragma once

#include "q38_types.cuh"

namespace q38 {

// Raw bsums as int16 pairs in aux[8..15] (the layout the staging path leaves).
__device__ __forceinline__ void raw_bsums(Act &a, const Q8KBlock *g)
{
#pragma unroll
    for (int j = 0; j < 8; ++j) a.aux[8 + j] = pack16(bsum(g, 2 * j), bsum(g, 2 * j + 1));
}

// The 16-element activation sum e (0..15) from the raw pairs.
template <int MT, class A>
__device__ __forceinline__ int bsum16(const A &a, int t, int e)
{
    const uint32_t pair = a.aux(t, 8 + (e >> 1));
    return (e & 1) ? hi16(pair) : lo16(pair);
}

// Both nibbles of the four bytes of `w` through a 16-entry byte table held in
// four words: lo = table[low nibble of byte i] and hi = table[high nibble of
// byte i] in byte i.  Each 16-bit half of w is used as a prmt selector for
// four table lookups at once (selector nibbles masked to 3 bits: bit 3 would
// ask prmt for sign replication); a third prmt keeps, per byte, the entry
// from the upper table half where the index has bit 3 set, and two more
// regroup the lookups by nibble.
__device__ __forceinline__ void lookup16_nibbles(uint32_t w, uint32_t t0, uint32_t t1, uint32_t t2, uint32_t t3,
                                                 uint32_t &lo, uint32_t &hi)
{
    uint32_t r[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const uint32_t sel = h ? w >> 16 : w;
        const uint32_t s7 = sel & 0x7777u;
        const uint32_t pick = ((sel >> 1) & 0x4444u) | 0x3210u;
        r[h] = prmt(prmt(t0, t1, s7), prmt(t2, t3, s7), pick);
    }
    lo = prmt(r[0], r[1], 0x6420u);
    hi = prmt(r[0], r[1], 0x7531u);
}

// IQ4_NL levels (qwen38_quant.c kvalues_iq4nl) as signed bytes.
constexpr uint32_t kIq4Lv0 = 0xBFAD9881u, kIq4Lv1 = 0xF6EADDCFu, kIq4Lv2 = 0x26190D01u, kIq4Lv3 = 0x71594535u;

// 8-bit sign mask of a 7-bit index (the 8th bit makes the parity even, the
// upstream's ksigns table).
__device__ __forceinline__ uint32_t ksigns(uint32_t index7)
{
    return index7 | ((static_cast<uint32_t>(__popc(index7)) & 1u) << 7);
}

// ===========================================================================
// Q2_K (84 B: 16 scale bytes - low nibble scale, high nibble min - 64 B of
// 2-bit quants, fp16 d, fp16 dmin).  qwen38_quant.c:510-585.
// ===========================================================================
struct DecQ2K {
    static constexpr int kBytes = 84;
    static constexpr int kAlign = 4;
    __device__ static void aux(Act &a, const Q8KBlock *g) { raw_bsums(a, g); }
    __device__ static void aux_from_raw(Act &) {}
    __device__ static void load(Act &a, const Q8KBlock *g) { load_act_base(a, g); aux(a, g); }
    __device__ static void zero(Act &a) { zero_act(a); }
    template <int MT, class A>
    __device__ static void block(const uint8_t *blk, const A &a, int (&w)[MT], int (&x)[MT], float (&v)[MT])
    {
        uint32_t sc[4], q[16], tail[1];
        lds_words<4>(blk, sc);
        lds_words<16>(blk + 16, q);
        lds_words<1>(blk + 80, tail);
#pragma unroll
        for (int t = 0; t < MT; ++t) w[t] = x[t] = 0;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
#pragma unroll
            for (int field = 0; field < 4; ++field) {
#pragma unroll
                for (int group = 0; group < 2; ++group) {
                    const int si = half * 8 + field * 2 + group;
                    const int scb = static_cast<int>(byte_of(sc[si >> 2], si & 3));
#pragma unroll
                    for (int t = 0; t < MT; ++t) {
                        int dot = 0;
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            const uint32_t qw = (q[half * 8 + group * 4 + k] >> (2 * field)) & 0x03030303u;
                            dot = dp4a_us(qw, a.q(t, half * 32 + field * 8 + group * 4 + k), dot);
                        }
                        w[t] += (scb & 15) * dot;
                        x[t] += (scb >> 4) * bsum16<MT>(a, t, si);
                    }
                }
            }
        }
        const float d = f16_bits_to_f32(tail[0] & 0xFFFFu), dmin = f16_bits_to_f32(tail[0] >> 16);
#pragma unroll
        for (int t = 0; t < MT; ++t) {
            const float dd = __fmul_rn(d, a.xs(t)), dm = __fmul_rn(dmin, a.xs(t));
            v[t] = __fsub_rn(__fmul_rn(dd, static_cast<float>(w[t])), __fmul_rn(dm, static_cast<float>(x[t])));
        }
    }
};

// ===========================================================================
// Q3_K (110 B: 32 B high-bit mask, 64 B of 2-bit quants, 12 B of 6-bit
// scales, fp16 d).  qwen38_quant.c:587-662 (scales :319-329).  q = low - 4
// where the mask bit is clear: sum(q x) = sum((low + 4 bit) x) - 4 sum(x),
// the last term a bsum.
// ===========================================================================
struct DecQ3K {
    static constexpr int kBytes = 110;
    static constexpr int kAlign = 2;
    __device__ static void aux(Act &a, const Q8KBlock *g) { raw_bsums(a, g); }
    __device__ static void aux_from_raw(Act &) {}
    __device__ static void load(Act &a, const Q8KBlock *g) { load_act_base(a, g); aux(a, g); }
    __device__ static void zero(Act &a) { zero_act(a); }
    template <int MT, class A>
    __device__ static void block(const uint8_t *blk, const A &a, int (&w)[MT], int (&x)[MT], float (&v)[MT])
    {
        uint32_t hm[8], lw[16], sw[4];
        lds_words<8>(blk, hm);
        lds_words<16>(blk + 32, lw);
        lds_words<4>(blk + 96, sw);  // 12 scale bytes, then d in the low half of word 3
#pragma unroll
        for (int t = 0; t < MT; ++t) w[t] = x[t] = 0;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
#pragma unroll
            for (int field = 0; field < 4; ++field) {
                const int group = half * 4 + field;
#pragma unroll
                for (int k2 = 0; k2 < 2; ++k2) {
                    const int si = group * 2 + k2;
                    const int low = si < 8 ? static_cast<int>(byte_of(sw[si >> 2], si & 3) & 15u)
                                           : static_cast<int>(byte_of(sw[(si - 8) >> 2], (si - 8) & 3) >> 4);
                    const int high = static_cast<int>((byte_of(sw[2], si & 3) >> (2 * (si >> 2))) & 3u);
                    const int s = (low | (high << 4)) - 32;
#pragma unroll
                    for (int t = 0; t < MT; ++t) {
                        int dot = 0;
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            const int wi = k2 * 4 + k;
                            const uint32_t lo = (lw[half * 8 + wi] >> (2 * field)) & 0x03030303u;
                            const uint32_t hb = (hm[wi] >> group) & 0x01010101u;
                            dot = dp4a_us(lo | (hb << 2), a.q(t, half * 32 + field * 8 + wi), dot);
                        }
                        w[t] += s * (dot - 4 * bsum16<MT>(a, t, half * 8 + field * 2 + k2));
                    }
                }
            }
        }
        const float d = f16_bits_to_f32(sw[3] & 0xFFFFu);
#pragma unroll
        for (int t = 0; t < MT; ++t) v[t] = __fmul_rn(__fmul_rn(d, a.xs(t)), static_cast<float>(w[t]));
    }
};

// ===========================================================================
// Q5_K (176 B: fp16 d, fp16 dmin, 12 B packed 6-bit scales/mins, 32 B high
// bits, 128 B low nibbles).  qwen38_quant.c:1636-1725.  Same scales, mins
// and activation sums as Q4_K (DecQ4K::aux).
// ===========================================================================
struct DecQ5K {
    static constexpr int kBytes = 176;
    static constexpr int kAlign = 16;
    __device__ static void aux(Act &a, const Q8KBlock *g) { DecQ4K::aux(a, g); }
    __device__ static void aux_from_raw(Act &a) { DecQ4K::aux_from_raw(a); }
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
        const uint4 qa = p[1], qb = p[2];
        const uint32_t hw[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
        for (int t = 0; t < MT; ++t) w[t] = 0;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const uint4 la = p[3 + 2 * c], lb = p[4 + 2 * c];
            const uint32_t lq[8] = {la.x, la.y, la.z, la.w, lb.x, lb.y, lb.z, lb.w};
            const uint32_t scw = c < 2 ? sc_lo : sc_hi;
            const int sc0 = static_cast<int>(byte_of(scw, (2 * c) & 3));
            const int sc1 = static_cast<int>(byte_of(scw, (2 * c + 1) & 3));
#pragma unroll
            for (int t = 0; t < MT; ++t) {
                int d0 = 0, d1 = 0;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const uint32_t q0 = (lq[i] & 0x0F0F0F0Fu) | (((hw[i] >> (2 * c)) & 0x01010101u) << 4);
                    const uint32_t q1 = ((lq[i] >> 4) & 0x0F0F0F0Fu) | (((hw[i] >> (2 * c + 1)) & 0x01010101u) << 4);
                    d0 = dp4a_us(q0, a.q(t, 16 * c + i), d0);
                    d1 = dp4a_us(q1, a.q(t, 16 * c + 8 + i), d1);
                }
                w[t] += sc0 * d0 + sc1 * d1;
            }
        }
        const float d = f16_bits_to_f32(h.x & 0xFFFFu);
        const float dmin = f16_bits_to_f32(h.x >> 16);
#pragma unroll
        for (int t = 0; t < MT; ++t) {
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
};

// ===========================================================================
// IQ4_XS (136 B: fp16 d, 16-bit high scale pairs, 4 B low scale nibbles,
// 128 B of 4-bit level indices).  qwen38_quant.c:1063-1127.
// ===========================================================================
struct DecIQ4XS {
    static constexpr int kBytes = 136;
    static constexpr int kAlign = 8;
    __device__ static void aux(Act &, const Q8KBlock *) {}
    __device__ static void aux_from_raw(Act &) {}
    __device__ static void load(Act &a, const Q8KBlock *g) { load_act_base(a, g); }
    __device__ static void zero(Act &a) { zero_act(a); }
    template <int MT, class A>
    __device__ static void block(const uint8_t *blk, const A &a, int (&w)[MT], int (&x)[MT], float (&v)[MT])
    {
        const uint2 *p = reinterpret_cast<const uint2 *>(blk);
        const uint2 h = p[0];
        const uint32_t sh = h.x >> 16, sl = h.y;
#pragma unroll
        for (int t = 0; t < MT; ++t) w[t] = x[t] = 0;
#pragma unroll
        for (int g = 0; g < 8; ++g) {
            const int scale = static_cast<int>(((byte_of(sl, g >> 1) >> (4 * (g & 1))) & 15u) |
                                               (((sh >> (2 * g)) & 3u) << 4)) - 32;
            const uint2 qa = p[1 + 2 * g], qb = p[2 + 2 * g];
            const uint32_t qw[4] = {qa.x, qa.y, qb.x, qb.y};
            uint32_t lv[8];  // levels of elements 4k.. (lv[k]) and 16 + 4k.. (lv[4 + k])
#pragma unroll
            for (int k = 0; k < 4; ++k) lookup16_nibbles(qw[k], kIq4Lv0, kIq4Lv1, kIq4Lv2, kIq4Lv3, lv[k], lv[4 + k]);
#pragma unroll
            for (int t = 0; t < MT; ++t) {
                int sub = 0;
#pragma unroll
                for (int k = 0; k < 8; ++k) sub = dp4a_ss(lv[k], a.q(t, 8 * g + k), sub);
                w[t] += scale * sub;
            }
        }
        const float d = f16_bits_to_f32(h.x & 0xFFFFu);
#pragma unroll
        for (int t = 0; t < MT; ++t) v[t] = __fmul_rn(__fmul_rn(d, a.xs(t)), static_cast<float>(w[t]));
    }
};

// ===========================================================================
// IQ4_NL on the Q8_K path: 8 blocks of 32 (18 B: fp16 d, 16 B of level
// index pairs) per 256 elements; the upstream adds one float per 32 elements
// (qwen38_quant.c:1129-1175), so v is that sum in order and (w, x) are 0.
// ===========================================================================
struct DecIQ4NL {
    static constexpr int kBytes = 144;
    static constexpr int kAlign = 2;
    __device__ static void aux(Act &, const Q8KBlock *) {}
    __device__ static void aux_from_raw(Act &) {}
    __device__ static void load(Act &a, const Q8KBlock *g) { load_act_base(a, g); }
    __device__ static void zero(Act &a) { zero_act(a); }
    template <int MT, class A>
    __device__ static void block(const uint8_t *blk, const A &a, int (&w)[MT], int (&x)[MT], float (&v)[MT])
    {
#pragma unroll
        for (int t = 0; t < MT; ++t) {
            w[t] = x[t] = 0;
            v[t] = 0.0f;
        }
#pragma unroll
        for (int g = 0; g < 8; ++g) {
            uint32_t raw[5];  // d and the 16 index bytes (bytes 18 g .. 18 g + 19)
            lds_words<5>(blk + 18 * g, raw);
            const float d = f16_bits_to_f32(raw[0] & 0xFFFFu);
            uint32_t qw[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) qw[k] = __funnelshift_r(raw[k], raw[k + 1], 16);
            uint32_t lv[8];
#pragma unroll
            for (int k = 0; k < 4; ++k) lookup16_nibbles(qw[k], kIq4Lv0, kIq4Lv1, kIq4Lv2, kIq4Lv3, lv[k], lv[4 + k]);
#pragma unroll
            for (int t = 0; t < MT; ++t) {
                int sub = 0;
#pragma unroll
                for (int k = 0; k < 8; ++k) sub = dp4a_ss(lv[k], a.q(t, 8 * g + k), sub);
                v[t] = __fadd_rn(v[t], __fmul_rn(__fmul_rn(d, a.xs(t)), static_cast<float>(sub)));
            }
        }
    }
};

// Signed bytes of an 8-value codebook entry `e` under the 8 sign bits `s8`.
__device__ __forceinline__ void signed_entry(uint2 e, uint32_t s8, uint32_t &lo, uint32_t &hi)
{
    lo = apply_signs(e.x, sign_mask4(s8 & 15u));
    hi = apply_signs(e.y, sign_mask4(s8 >> 4));
}

// ===========================================================================
// IQ2_XXS (66 B: fp16 d, then per 32 elements 4 grid indices and a word of
// 4 x 7 sign bits and a 4-bit scale).  qwen38_quant.c:758-822.
// ===========================================================================
struct DecIQ2XXS {
    static constexpr int kBytes = 66;
    static constexpr int kAlign = 2;
    __device__ static void aux(Act &, const Q8KBlock *) {}
    __device__ static void aux_from_raw(Act &) {}
    __device__ static void load(Act &a, const Q8KBlock *g) { load_act_base(a, g); }
    __device__ static void zero(Act &a) { zero_act(a); }
    template <int MT, class A>
    __device__ static void block(const uint8_t *blk, const A &a, int (&w)[MT], int (&x)[MT], float (&v)[MT],
                                 const uint2 *grid)
    {
        uint32_t raw[17];  // bytes 0..67: d, then the 8 groups
        lds_words<17>(blk, raw);
#pragma unroll
        for (int t = 0; t < MT; ++t) w[t] = x[t] = 0;
#pragma unroll
        for (int g = 0; g < 8; ++g) {
            const uint32_t codes = __funnelshift_r(raw[2 * g], raw[2 * g + 1], 16);
            const uint32_t meta = __funnelshift_r(raw[2 * g + 1], raw[2 * g + 2], 16);
            const int scale = 1 + 2 * static_cast<int>(meta >> 28);
            int sub[MT];
#pragma unroll
            for (int t = 0; t < MT; ++t) sub[t] = 0;
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                uint32_t lo, hi;
                signed_entry(grid[byte_of(codes, s)], ksigns((meta >> (7 * s)) & 127u), lo, hi);
#pragma unroll
                for (int t = 0; t < MT; ++t) {
                    sub[t] = dp4a_ss(lo, a.q(t, 8 * g + 2 * s), sub[t]);
                    sub[t] = dp4a_ss(hi, a.q(t, 8 * g + 2 * s + 1), sub[t]);
                }
            }
#pragma unroll
            for (int t = 0; t < MT; ++t) w[t] += scale * sub[t];
        }
        const float d = f16_bits_to_f32(raw[0] & 0xFFFFu);
#pragma unroll
        for (int t = 0; t < MT; ++t)
            v[t] = __fmul_rn(__fmul_rn(__fmul_rn(0.125f, d), a.xs(t)), static_cast<float>(w[t]));
    }
};

// ===========================================================================
// IQ2_XS (74 B: fp16 d, 32 codes of a 9-bit grid index and 7 sign bits,
// 8 bytes of 4-bit scale pairs).  qwen38_quant.c:824-893.
// ===========================================================================
struct DecIQ2XS {
    static constexpr int kBytes = 74;
    static constexpr int kAlign = 2;
    __device__ static void aux(Act &, const Q8KBlock *) {}
    __device__ static void aux_from_raw(Act &) {}
    __device__ static void load(Act &a, const Q8KBlock *g) { load_act_base(a, g); }
    __device__ static void zero(Act &a) { zero_act(a); }
    template <int MT, class A>
    __device__ static void block(const uint8_t *blk, const A &a, int (&w)[MT], int (&x)[MT], float (&v)[MT],
                                 const uint2 *grid)
    {
        uint32_t raw[19];  // bytes 0..75
        lds_words<19>(blk, raw);
#pragma unroll
        for (int t = 0; t < MT; ++t) w[t] = x[t] = 0;
#pragma unroll
        for (int g = 0; g < 8; ++g) {
            const int sb = static_cast<int>(byte_of(__funnelshift_r(raw[16 + (g >> 2)], raw[17 + (g >> 2)], 16), g & 3));
            int sub[MT][2];
#pragma unroll
            for (int t = 0; t < MT; ++t) sub[t][0] = sub[t][1] = 0;
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                const int c = 4 * g + s;  // code c sits at bytes 2 + 2c
                const uint32_t word = raw[(2 + 2 * c) >> 2];
                const uint32_t code = (c & 1) ? (word & 0xFFFFu) : (word >> 16);
                uint32_t lo, hi;
                signed_entry(grid[code & 511u], ksigns(code >> 9), lo, hi);
#pragma unroll
                for (int t = 0; t < MT; ++t) {
                    sub[t][s >> 1] = dp4a_ss(lo, a.q(t, 8 * g + 2 * s), sub[t][s >> 1]);
                    sub[t][s >> 1] = dp4a_ss(hi, a.q(t, 8 * g + 2 * s + 1), sub[t][s >> 1]);
                }
            }
#pragma unroll
            for (int t = 0; t < MT; ++t) w[t] += (1 + 2 * (sb & 15)) * sub[t][0] + (1 + 2 * (sb >> 4)) * sub[t][1];
        }
        const float d = f16_bits_to_f32(raw[0] & 0xFFFFu);
#pragma unroll
        for (int t = 0; t < MT; ++t)
            v[t] = __fmul_rn(__fmul_rn(__fmul_rn(0.125f, d), a.xs(t)), static_cast<float>(w[t]));
    }
};

// ===========================================================================
// IQ3_XXS (98 B: fp16 d, 64 grid indices (4 values each), 8 words of 4 x 7
// sign bits and a 4-bit scale).  qwen38_quant.c:895-976.
// ===========================================================================
struct DecIQ3XXS {
    static constexpr int kBytes = 98;
    static constexpr int kAlign = 2;
    __device__ static void aux(Act &, const Q8KBlock *) {}
    __device__ static void aux_from_raw(Act &) {}
    __device__ static void load(Act &a, const Q8KBlock *g) { load_act_base(a, g); }
    __device__ static void zero(Act &a) { zero_act(a); }
    template <int MT, class A>
    __device__ static void block(const uint8_t *blk, const A &a, int (&w)[MT], int (&x)[MT], float (&v)[MT],
                                 const uint2 *grid)
    {
        uint32_t idx[16], meta[8], head[1];
        lds_words<16>(blk + 2, idx);
        lds_words<8>(blk + 66, meta);
        lds_words<1>(blk, head);
#pragma unroll
        for (int t = 0; t < MT; ++t) w[t] = x[t] = 0;
#pragma unroll
        for (int g = 0; g < 8; ++g) {
            const uint32_t packed = meta[g];
            const int scale = 1 + 2 * static_cast<int>(packed >> 28);
            int sub[MT];
#pragma unroll
            for (int t = 0; t < MT; ++t) sub[t] = 0;
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                const uint32_t iw = idx[2 * g + (s >> 1)];
                const uint2 e = make_uint2(grid[byte_of(iw, (2 * s) & 3)].x, grid[byte_of(iw, (2 * s + 1) & 3)].x);
                uint32_t lo, hi;
                signed_entry(e, ksigns((packed >> (7 * s)) & 127u), lo, hi);
#pragma unroll
                for (int t = 0; t < MT; ++t) {
                    sub[t] = dp4a_ss(lo, a.q(t, 8 * g + 2 * s), sub[t]);
                    sub[t] = dp4a_ss(hi, a.q(t, 8 * g + 2 * s + 1), sub[t]);
                }
            }
#pragma unroll
            for (int t = 0; t < MT; ++t) w[t] += scale * sub[t];
        }
        const float d = f16_bits_to_f32(head[0] & 0xFFFFu);
#pragma unroll
        for (int t = 0; t < MT; ++t)
            v[t] = __fmul_rn(__fmul_rn(__fmul_rn(0.25f, d), a.xs(t)), static_cast<float>(w[t]));
    }
};

// ===========================================================================
// IQ3_S (110 B: fp16 d, 64 low index bytes, 8 bytes of index high bits,
// 32 bytes of explicit signs, 4 bytes of 4-bit scales).  qwen38_quant.c:978-1061.
// ===========================================================================
struct DecIQ3S {
    static constexpr int kBytes = 110;
    static constexpr int kAlign = 2;
    __device__ static void aux(Act &, const Q8KBlock *) {}
    __device__ static void aux_from_raw(Act &) {}
    __device__ static void load(Act &a, const Q8KBlock *g) { load_act_base(a, g); }
    __device__ static void zero(Act &a) { zero_act(a); }
    template <int MT, class A>
    __device__ static void block(const uint8_t *blk, const A &a, int (&w)[MT], int (&x)[MT], float (&v)[MT],
                                 const uint2 *grid)
    {
        uint32_t idx[16], qh[2], sg[8], tail[1], head[1];
        lds_words<16>(blk + 2, idx);
        lds_words<2>(blk + 66, qh);
        lds_words<8>(blk + 74, sg);
        lds_words<1>(blk + 106, tail);
        lds_words<1>(blk, head);
#pragma unroll
        for (int t = 0; t < MT; ++t) w[t] = x[t] = 0;
#pragma unroll
        for (int g = 0; g < 8; ++g) {
            const uint32_t hg = byte_of(qh[g >> 2], g & 3);
            const int scale = 1 + 2 * static_cast<int>((byte_of(tail[0], g >> 1) >> (4 * (g & 1))) & 15u);
            int sub[MT];
#pragma unroll
            for (int t = 0; t < MT; ++t) sub[t] = 0;
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                const uint32_t iw = idx[2 * g + (s >> 1)];
                const uint32_t i0 = byte_of(iw, (2 * s) & 3) | ((hg << (8 - 2 * s)) & 0x100u);
                const uint32_t i1 = byte_of(iw, (2 * s + 1) & 3) | ((hg << (7 - 2 * s)) & 0x100u);
                uint32_t lo, hi;
                signed_entry(make_uint2(grid[i0].x, grid[i1].x), byte_of(sg[g], s), lo, hi);
#pragma unroll
                for (int t = 0; t < MT; ++t) {
                    sub[t] = dp4a_ss(lo, a.q(t, 8 * g + 2 * s), sub[t]);
                    sub[t] = dp4a_ss(hi, a.q(t, 8 * g + 2 * s + 1), sub[t]);
                }
            }
#pragma unroll
            for (int t = 0; t < MT; ++t) w[t] += scale * sub[t];
        }
        const float d = f16_bits_to_f32(head[0] & 0xFFFFu);
#pragma unroll
        for (int t = 0; t < MT; ++t) v[t] = __fmul_rn(__fmul_rn(d, a.xs(t)), static_cast<float>(w[t]));
    }
};

}  // namespace q38
