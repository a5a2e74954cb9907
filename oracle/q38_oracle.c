/* q38_oracle.c - CPU restatement of the upstream quantized kernels.
 *
 * TEST INFRASTRUCTURE ONLY (see q38_oracle.h).  Compiled with
 * -ffp-contract=off like the upstream build (GNUmakefile:25), so every float
 * operation rounds exactly where the upstream scalar C rounds.
 *
 * Citations are to src/qwen38/qwen38_quant.c of the upstream engine unless
 * stated otherwise.  The integer sums restate the scalar (#else) branches; the
 * upstream AVX2 branches compute the same integers in SIMD lanes.
 */
#include "q38_oracle.h"

#include <math.h>
#include <string.h>

#include "../qwen3.8-27b-in-c_b200/csrc/q38_codebooks.h"

static uint16_t load_u16(const uint8_t *p) { return (uint16_t)(p[0] | p[1] << 8); }
static uint32_t load_u32(const uint8_t *p)
{
    return (uint32_t)p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24;
}

/* Exact IEEE half -> float (qwen38_quant.c:90-122, portable branch). */
float q38o_f16_to_f32(uint16_t value)
{
    const uint32_t sign = (uint32_t)(value & 0x8000u) << 16;
    const uint32_t exponent = (value >> 10) & 31u;
    uint32_t mantissa = value & 1023u;
    uint32_t bits;
    if (exponent == 0) {
        if (mantissa == 0) {
            bits = sign;
        } else {
            int e = -1;
            do { mantissa <<= 1; ++e; } while ((mantissa & 0x400u) == 0);
            bits = sign | (uint32_t)(112 - e) << 23 | (mantissa & 0x3ffu) << 13;
        }
    } else if (exponent == 31) {
        bits = sign | 0x7f800000u | mantissa << 13;
    } else {
        bits = sign | (exponent + 112u) << 23 | mantissa << 13;
    }
    float out;
    memcpy(&out, &bits, sizeof(out));
    return out;
}

static float bf16_to_f32(const uint8_t *p)
{
    uint32_t bits = (uint32_t)load_u16(p) << 16;
    float out;
    memcpy(&out, &bits, sizeof(out));
    return out;
}

/* Block geometry (src/io/qwen38_gguf.c:130-185). */
uint32_t q38o_block_elements(uint32_t type)
{
    switch (type) {
    case Q38O_F32: case Q38O_F16: case Q38O_BF16: return 1;
    case Q38O_Q8_0: case Q38O_IQ4_NL: return 32;
    case Q38O_Q2_K: case Q38O_Q3_K: case Q38O_Q4_K: case Q38O_Q5_K: case Q38O_Q6_K:
    case Q38O_IQ2_XXS: case Q38O_IQ2_XS: case Q38O_IQ3_XXS: case Q38O_IQ1_S:
    case Q38O_IQ3_S: case Q38O_IQ2_S: case Q38O_IQ4_XS: case Q38O_IQ1_M: return 256;
    default: return 0;
    }
}

uint32_t q38o_block_bytes(uint32_t type)
{
    switch (type) {
    case Q38O_F32: return 4;
    case Q38O_F16: case Q38O_BF16: return 2;
    case Q38O_Q8_0: return 34;
    case Q38O_IQ4_NL: return 18;
    case Q38O_Q2_K: return 84;
    case Q38O_Q3_K: return 110;
    case Q38O_Q4_K: return 144;
    case Q38O_Q5_K: return 176;
    case Q38O_Q6_K: return 210;
    case Q38O_IQ2_XXS: return 66;
    case Q38O_IQ2_XS: return 74;
    case Q38O_IQ3_XXS: return 98;
    case Q38O_IQ1_S: return 50;
    case Q38O_IQ3_S: return 110;
    case Q38O_IQ2_S: return 82;
    case Q38O_IQ4_XS: return 136;
    case Q38O_IQ1_M: return 56;
    default: return 0;
    }
}

/* qwen38_model.c:172-182. */
int q38o_type_q8_k(uint32_t type)
{
    switch (type) {
    case Q38O_Q2_K: case Q38O_Q3_K: case Q38O_Q4_K: case Q38O_Q5_K: case Q38O_Q6_K:
    case Q38O_IQ2_XXS: case Q38O_IQ2_XS: case Q38O_IQ3_XXS: case Q38O_IQ4_NL:
    case Q38O_IQ3_S: case Q38O_IQ2_S: case Q38O_IQ4_XS: case Q38O_IQ1_S: case Q38O_IQ1_M:
        return 1;
    default: return 0;
    }
}

/* Bytes of one 256-column superblock row segment in the Q8_K path
 * (qwen38_quant.c:2841-2857; IQ4_NL packs 8 x 18 bytes). */
static uint32_t superblock_bytes(uint32_t type)
{
    return type == Q38O_IQ4_NL ? 144u : q38o_block_bytes(type);
}

/* Round-half-even via the 1.5*2^23 magic constant (qwen38_quant.c:42-48). */
static int nearest_int(float value)
{
    const float shifted = value + 12582912.0f;
    uint32_t bits;
    memcpy(&bits, &shifted, sizeof(bits));
    return (int)(bits & 0x007fffffu) - 0x00400000;
}

/* qwen38_quant.c:50-88. */
int q38o_quantize_q8_k(Q38OQ8KBlock *output, const float *input, uint64_t length)
{
    if (!output || !input || length % 256 != 0) return 0;
    for (uint64_t block = 0; block < length / 256; ++block) {
        const float *x = input + block * 256;
        Q38OQ8KBlock *q = output + block;
        float maximum = 0.0f, absolute_maximum = 0.0f;
        for (int i = 0; i < 256; ++i) {
            const float a = fabsf(x[i]);
            if (a > absolute_maximum) { absolute_maximum = a; maximum = x[i]; }
        }
        if (absolute_maximum == 0.0f) {
            memset(q, 0, sizeof(*q));
            continue;
        }
        const float inverse = -127.0f / maximum;
        for (int i = 0; i < 256; ++i) {
            const float scaled = inverse * x[i];
            int v = nearest_int(scaled);
            if (v > 127) v = 127;
            q->quants[i] = (int8_t)v;
        }
        for (int g = 0; g < 16; ++g) {
            int s = 0;
            for (int i = 0; i < 16; ++i) s += q->quants[g * 16 + i];
            q->sums[g] = (int16_t)s;
        }
        q->scale = 1.0f / inverse;
    }
    return 1;
}

/* 6-bit scale/min unpack (qwen38_quant.c:131-143). */
static void scale_min_k4(int j, const uint8_t *p, int *sc, int *m)
{
    if (j < 4) {
        *sc = p[j] & 63;
        *m = p[j + 4] & 63;
    } else {
        *sc = (p[j + 4] & 15) | ((p[j - 4] >> 6) << 4);
        *m = (p[j + 4] >> 4) | ((p[j] >> 6) << 4);
    }
}

/* qwen38_quant.c:319-329. */
static void unpack_q3_scales(const uint8_t *p, int s[16])
{
    for (int i = 0; i < 16; ++i) {
        const int low = i < 8 ? (p[i] & 15) : (p[i - 8] >> 4);
        const int high = (p[8 + i % 4] >> (2 * (i / 4))) & 3;
        s[i] = (low | high << 4) - 32;
    }
}

/* Codebook accessors over the compact tables. */
static int iq1s_value(uint32_t index, int lane)
{
    const uint32_t e = Q38_IQ1S_GRID_NIB[index];
    const int shift = lane < 4 ? 8 * lane : 8 * (lane - 4) + 4;
    return (int)((e >> shift) & 15u) - 1;
}

static int iq2_value(const uint32_t *grid, uint32_t index, int lane)
{
    static const int magnitude[3] = {8, 25, 43};
    const uint32_t e = grid[index];
    const int shift = lane < 4 ? 8 * lane : 8 * (lane - 4) + 4;
    return magnitude[(e >> shift) & 15u];
}

static int iq3_value(const uint16_t *grid, const uint8_t *magnitudes, uint32_t index, int lane)
{
    return magnitudes[(grid[index] >> (4 * lane)) & 15u];
}

static int ksign_bits(uint32_t index7)
{
    int parity = 0;
    for (int b = 0; b < 7; ++b) parity ^= (index7 >> b) & 1;
    return (int)(index7 | (uint32_t)parity << 7);
}

int q38o_block_sums(uint32_t type, const uint8_t *b, const Q38OQ8KBlock *a,
                    int32_t *w_out, int32_t *x_out)
{
    const int8_t *q8 = a->quants;
    int32_t w = 0, x = 0;
    switch (type) {
    case Q38O_Q2_K: { /* :510-585 */
        const uint8_t *scales = b, *quants = b + 16;
        for (int half = 0; half < 2; ++half)
            for (int field = 0; field < 4; ++field)
                for (int group = 0; group < 2; ++group) {
                    const int si = half * 8 + field * 2 + group;
                    int dot = 0;
                    for (int lane = 0; lane < 16; ++lane)
                        dot += ((quants[half * 32 + group * 16 + lane] >> (2 * field)) & 3) *
                               q8[half * 128 + field * 32 + group * 16 + lane];
                    w += (scales[si] & 15) * dot;
                    x += (scales[si] >> 4) * a->sums[si];
                }
        break;
    }
    case Q38O_Q3_K: { /* :587-662 */
        const uint8_t *high = b, *low = b + 32;
        int scales[16];
        unpack_q3_scales(b + 96, scales);
        int group = 0;
        for (int half = 0; half < 2; ++half)
            for (int field = 0; field < 4; ++field, ++group) {
                const int bit = 1 << group;
                for (int lane = 0; lane < 32; ++lane) {
                    const int q = ((low[half * 32 + lane] >> (2 * field)) & 3) -
                                  ((high[lane] & bit) ? 0 : 4);
                    const int s = lane < 16 ? scales[group * 2] : scales[group * 2 + 1];
                    w += s * q * q8[half * 128 + field * 32 + lane];
                }
            }
        break;
    }
    case Q38O_Q4_K: { /* :1546-1634 */
        const uint8_t *scales = b + 4, *quants = b + 16;
        for (int chunk = 0; chunk < 4; ++chunk) {
            int sc0, m0, sc1, m1;
            scale_min_k4(chunk * 2, scales, &sc0, &m0);
            scale_min_k4(chunk * 2 + 1, scales, &sc1, &m1);
            int dot0 = 0, dot1 = 0;
            for (int i = 0; i < 32; ++i) {
                dot0 += (quants[chunk * 32 + i] & 15) * q8[chunk * 64 + i];
                dot1 += (quants[chunk * 32 + i] >> 4) * q8[chunk * 64 + 32 + i];
            }
            w += sc0 * dot0 + sc1 * dot1;
            x += m0 * (a->sums[chunk * 4] + a->sums[chunk * 4 + 1]);
            x += m1 * (a->sums[chunk * 4 + 2] + a->sums[chunk * 4 + 3]);
        }
        break;
    }
    case Q38O_Q5_K: { /* :1636-1725 */
        const uint8_t *scales = b + 4, *high = b + 16, *low = b + 48;
        for (int chunk = 0; chunk < 4; ++chunk) {
            int sc0, m0, sc1, m1;
            scale_min_k4(chunk * 2, scales, &sc0, &m0);
            scale_min_k4(chunk * 2 + 1, scales, &sc1, &m1);
            const int h0 = 1 << (2 * chunk), h1 = 2 << (2 * chunk);
            int dot0 = 0, dot1 = 0;
            for (int i = 0; i < 32; ++i) {
                dot0 += ((low[chunk * 32 + i] & 15) + ((high[i] & h0) ? 16 : 0)) * q8[chunk * 64 + i];
                dot1 += ((low[chunk * 32 + i] >> 4) + ((high[i] & h1) ? 16 : 0)) * q8[chunk * 64 + 32 + i];
            }
            w += sc0 * dot0 + sc1 * dot1;
            x += m0 * (a->sums[chunk * 4] + a->sums[chunk * 4 + 1]);
            x += m1 * (a->sums[chunk * 4 + 2] + a->sums[chunk * 4 + 3]);
        }
        break;
    }
    case Q38O_Q6_K: { /* :1727-1833; the AVX2 branch subtracts 32*sum(sc*bsum) */
        const uint8_t *low = b, *high = b + 128;
        const int8_t *scales = (const int8_t *)(b + 192);
        int offset = 0;
        for (int g = 0; g < 16; ++g) offset += scales[g] * a->sums[g];
        for (int half = 0; half < 2; ++half)
            for (int i = 0; i < 32; ++i) {
                const int si = half * 8 + i / 16;
                const int q0 = (low[half * 64 + i] & 15) | ((high[half * 32 + i] & 3) << 4);
                const int q1 = (low[half * 64 + i + 32] & 15) | (((high[half * 32 + i] >> 2) & 3) << 4);
                const int q2 = (low[half * 64 + i] >> 4) | (((high[half * 32 + i] >> 4) & 3) << 4);
                const int q3 = (low[half * 64 + i + 32] >> 4) | (((high[half * 32 + i] >> 6) & 3) << 4);
                const int base = half * 128;
                w += scales[si] * q0 * q8[base + i];
                w += scales[si + 2] * q1 * q8[base + 32 + i];
                w += scales[si + 4] * q2 * q8[base + 64 + i];
                w += scales[si + 6] * q3 * q8[base + 96 + i];
            }
        w -= 32 * offset;
        break;
    }
    case Q38O_IQ2_XXS: { /* :758-822 */
        const uint8_t *codes = b + 2;
        for (int g = 0; g < 8; ++g, codes += 8) {
            const uint32_t meta = load_u32(codes + 4);
            const int scale = 1 + 2 * (int)(meta >> 28);
            int sub = 0;
            for (int s = 0; s < 4; ++s) {
                const int signs = ksign_bits((meta >> (7 * s)) & 127u);
                for (int lane = 0; lane < 8; ++lane)
                    sub += q8[g * 32 + s * 8 + lane] * iq2_value(Q38_IQ2XXS_GRID_NIB, codes[s], lane) *
                           ((signs >> lane) & 1 ? -1 : 1);
            }
            w += scale * sub;
        }
        break;
    }
    case Q38O_IQ2_XS: { /* :824-893 */
        const uint8_t *codes = b + 2, *scales = b + 66;
        for (int g = 0; g < 8; ++g, codes += 8) {
            int sub[2] = {0, 0};
            for (int s = 0; s < 4; ++s) {
                const uint16_t code = load_u16(codes + 2 * s);
                const int signs = ksign_bits(code >> 9);
                for (int lane = 0; lane < 8; ++lane)
                    sub[s / 2] += q8[g * 32 + s * 8 + lane] *
                                  iq2_value(Q38_IQ2XS_GRID_NIB, code & 511u, lane) *
                                  ((signs >> lane) & 1 ? -1 : 1);
            }
            w += (1 + 2 * (scales[g] & 15)) * sub[0] + (1 + 2 * (scales[g] >> 4)) * sub[1];
        }
        break;
    }
    case Q38O_IQ2_S: { /* :664-756 */
        const uint8_t *idx = b + 2, *signs = b + 34, *high = b + 66, *scales = b + 74;
        for (int g = 0; g < 8; ++g) {
            int sub[2] = {0, 0};
            for (int s = 0; s < 4; ++s) {
                const uint32_t gi = idx[g * 4 + s] | ((high[g] << (8 - 2 * s)) & 0x300);
                for (int lane = 0; lane < 8; ++lane)
                    sub[s / 2] += q8[g * 32 + s * 8 + lane] * iq2_value(Q38_IQ2S_GRID_NIB, gi, lane) *
                                  ((signs[g * 4 + s] >> lane) & 1 ? -1 : 1);
            }
            w += (1 + 2 * (scales[g] & 15)) * sub[0] + (1 + 2 * (scales[g] >> 4)) * sub[1];
        }
        break;
    }
    case Q38O_IQ3_XXS: { /* :895-976 */
        const uint8_t *idx = b + 2, *meta = b + 66;
        for (int g = 0; g < 8; ++g) {
            const uint32_t packed = load_u32(meta + g * 4);
            const int scale = 1 + 2 * (int)(packed >> 28);
            const uint8_t *code = idx + g * 8;
            int sub = 0;
            for (int s = 0; s < 4; ++s) {
                const int signs = ksign_bits((packed >> (7 * s)) & 127u);
                for (int lane = 0; lane < 4; ++lane) {
                    sub += q8[g * 32 + s * 8 + lane] *
                           iq3_value(Q38_IQ3XXS_GRID_C4, Q38_IQ3XXS_MAGNITUDES, code[2 * s], lane) *
                           ((signs >> lane) & 1 ? -1 : 1);
                    sub += q8[g * 32 + s * 8 + lane + 4] *
                           iq3_value(Q38_IQ3XXS_GRID_C4, Q38_IQ3XXS_MAGNITUDES, code[2 * s + 1], lane) *
                           ((signs >> (lane + 4)) & 1 ? -1 : 1);
                }
            }
            w += scale * sub;
        }
        break;
    }
    case Q38O_IQ3_S: { /* :978-1061 */
        const uint8_t *idx = b + 2, *high = b + 66, *signs = b + 74, *scales = b + 106;
        for (int g = 0; g < 8; ++g) {
            const uint8_t *code = idx + g * 8;
            const int scale = 1 + 2 * ((scales[g / 2] >> (4 * (g % 2))) & 15);
            int sub = 0;
            for (int s = 0; s < 4; ++s) {
                const uint32_t i0 = code[2 * s] | ((high[g] << (8 - 2 * s)) & 0x100);
                const uint32_t i1 = code[2 * s + 1] | ((high[g] << (7 - 2 * s)) & 0x100);
                for (int lane = 0; lane < 4; ++lane) {
                    sub += q8[g * 32 + s * 8 + lane] *
                           iq3_value(Q38_IQ3S_GRID_C4, Q38_IQ3S_MAGNITUDES, i0, lane) *
                           ((signs[g * 4 + s] >> lane) & 1 ? -1 : 1);
                    sub += q8[g * 32 + s * 8 + lane + 4] *
                           iq3_value(Q38_IQ3S_GRID_C4, Q38_IQ3S_MAGNITUDES, i1, lane) *
                           ((signs[g * 4 + s] >> (lane + 4)) & 1 ? -1 : 1);
                }
            }
            w += scale * sub;
        }
        break;
    }
    case Q38O_IQ4_XS: { /* :1063-1127 */
        const uint16_t scale_high = load_u16(b + 2);
        const uint8_t *scale_low = b + 4, *quants = b + 8;
        for (int g = 0; g < 8; ++g) {
            const int scale = ((scale_low[g / 2] >> (4 * (g % 2))) & 15) |
                              (((scale_high >> (2 * g)) & 3) << 4);
            int sub = 0;
            for (int lane = 0; lane < 16; ++lane) {
                const uint8_t p = quants[16 * g + lane];
                sub += q8[g * 32 + lane] * Q38_IQ4NL_LEVELS[p & 15];
                sub += q8[g * 32 + lane + 16] * Q38_IQ4NL_LEVELS[p >> 4];
            }
            w += (scale - 32) * sub;
        }
        break;
    }
    case Q38O_IQ1_S: { /* :1177-1253 */
        const uint8_t *idx = b + 2, *high = b + 34;
        for (int g = 0; g < 8; ++g) {
            const uint16_t packed = load_u16(high + 2 * g);
            const int scale = 1 + 2 * ((packed >> 12) & 7);
            const int delta = (packed & 0x8000u) ? -1 : 1;
            int sub = 0;
            for (int s = 0; s < 4; ++s) {
                const uint32_t gi = idx[4 * g + s] | (((packed >> (3 * s)) & 7u) << 8);
                for (int lane = 0; lane < 8; ++lane)
                    sub += q8[g * 32 + s * 8 + lane] * iq1s_value(gi, lane);
            }
            w += scale * sub;
            x += scale * delta * (a->sums[2 * g] + a->sums[2 * g + 1]);
        }
        break;
    }
    case Q38O_IQ1_M: { /* :1388-1544 */
        const uint8_t *idx = b, *high = b + 32, *packed_scales = b + 48;
        for (int g = 0; g < 8; ++g) {
            int dot[2] = {0, 0}, corr[2] = {0, 0};
            for (int s = 0; s < 4; ++s) {
                const uint8_t h = high[2 * g + s / 2];
                const uint32_t gi = idx[4 * g + s] | (((uint32_t)h << (8 - 4 * (s % 2))) & 0x700u);
                const int delta = (h & (s % 2 ? 0x80u : 0x08u)) ? -1 : 1;
                for (int lane = 0; lane < 8; ++lane) {
                    const int act = q8[g * 32 + s * 8 + lane];
                    dot[s / 2] += act * iq1s_value(gi, lane);
                    corr[s / 2] += act * delta;
                }
            }
            const uint16_t sc = load_u16(packed_scales + (g / 2) * 2);
            const int shift = 6 * (g % 2);
            const int s0 = 1 + 2 * ((sc >> shift) & 7), s1 = 1 + 2 * ((sc >> (shift + 3)) & 7);
            w += s0 * dot[0] + s1 * dot[1];
            x += s0 * corr[0] + s1 * corr[1];
        }
        break;
    }
    default:
        return 0;
    }
    if (w_out) *w_out = w;
    if (x_out) *x_out = x;
    return 1;
}

static float iq1m_scale(const uint8_t *b)
{
    const uint8_t *ps = b + 48;
    const uint16_t bits = (uint16_t)((load_u16(ps) >> 12) | ((load_u16(ps + 2) >> 8) & 0x00f0u) |
                                     ((load_u16(ps + 4) >> 4) & 0x0f00u) | (load_u16(ps + 6) & 0xf000u));
    return q38o_f16_to_f32(bits);
}

float q38o_block_value(uint32_t type, const uint8_t *b, const Q38OQ8KBlock *a)
{
    int32_t w = 0, x = 0;
    if (type == Q38O_IQ4_NL) { /* :1129-1175: a float scale per 32 elements */
        float total = 0.0f;
        for (int g = 0; g < 8; ++g) {
            const uint8_t *blk = b + g * 18;
            const float d = q38o_f16_to_f32(load_u16(blk)) * a->scale;
            int sub = 0;
            for (int lane = 0; lane < 16; ++lane) {
                sub += a->quants[g * 32 + lane] * Q38_IQ4NL_LEVELS[blk[2 + lane] & 15];
                sub += a->quants[g * 32 + lane + 16] * Q38_IQ4NL_LEVELS[blk[2 + lane] >> 4];
            }
            total += d * (float)sub;
        }
        return total;
    }
    if (!q38o_block_sums(type, b, a, &w, &x)) return NAN;
    const float xs = a->scale;
    switch (type) {
    case Q38O_Q2_K: {
        const float d = q38o_f16_to_f32(load_u16(b + 80)) * xs;
        const float dmin = q38o_f16_to_f32(load_u16(b + 82)) * xs;
        return d * (float)w - dmin * (float)x;
    }
    case Q38O_Q3_K: return (q38o_f16_to_f32(load_u16(b + 108)) * xs) * (float)w;
    case Q38O_Q4_K: case Q38O_Q5_K: {
        const float d = q38o_f16_to_f32(load_u16(b)) * xs;
        const float dmin = q38o_f16_to_f32(load_u16(b + 2)) * xs;
        return d * (float)w - dmin * (float)x;
    }
    case Q38O_Q6_K: return (q38o_f16_to_f32(load_u16(b + 208)) * xs) * (float)w;
    case Q38O_IQ2_XXS: case Q38O_IQ2_XS: case Q38O_IQ2_S:
        return (0.125f * q38o_f16_to_f32(load_u16(b)) * xs) * (float)w;
    case Q38O_IQ3_XXS: return (0.25f * q38o_f16_to_f32(load_u16(b)) * xs) * (float)w;
    case Q38O_IQ3_S: case Q38O_IQ4_XS: return (q38o_f16_to_f32(load_u16(b)) * xs) * (float)w;
    case Q38O_IQ1_S: {
        const float d = q38o_f16_to_f32(load_u16(b)) * xs;
        return d * ((float)w + 0.125f * (float)x);
    }
    case Q38O_IQ1_M: {
        const float d = iq1m_scale(b) * xs;
        return d * ((float)w + 0.125f * (float)x);
    }
    default: return NAN;
    }
}

/* qwen38_quant.c:2833-2922 and 2950-3169 (batch-major output). */
int q38o_gemm_q8_k(float *output, const Q38OQ8KBlock *input, uint32_t batch,
                   uint64_t width, uint32_t type, const uint8_t *data, uint64_t rows)
{
    if (!output || !input || !data || !batch || width % 256 || !q38o_type_q8_k(type)) return 0;
    const uint64_t blocks = width / 256;
    const uint64_t row_bytes = blocks * superblock_bytes(type);
    for (uint64_t row = 0; row < rows; ++row)
        for (uint32_t t = 0; t < batch; ++t) {
            float total = 0.0f;
            for (uint64_t blk = 0; blk < blocks; ++blk)
                total += q38o_block_value(type, data + row * row_bytes + blk * superblock_bytes(type),
                                          input + (uint64_t)t * blocks + blk);
            output[(uint64_t)t * rows + row] = total;
        }
    return 1;
}

int q38o_gemm_q8_k_sums(int32_t *w_out, int32_t *x_out, const Q38OQ8KBlock *input,
                        uint32_t batch, uint64_t width, uint32_t type,
                        const uint8_t *data, uint64_t rows)
{
    if (!w_out || !x_out || !input || !data || !batch || width % 256 ||
        !q38o_type_q8_k(type) || type == Q38O_IQ4_NL) return 0;
    const uint64_t blocks = width / 256;
    const uint64_t row_bytes = blocks * superblock_bytes(type);
    for (uint32_t t = 0; t < batch; ++t)
        for (uint64_t row = 0; row < rows; ++row)
            for (uint64_t blk = 0; blk < blocks; ++blk) {
                const uint64_t o = ((uint64_t)t * rows + row) * blocks + blk;
                if (!q38o_block_sums(type, data + row * row_bytes + blk * superblock_bytes(type),
                                     input + (uint64_t)t * blocks + blk, &w_out[o], &x_out[o]))
                    return 0;
            }
    return 1;
}

/* Float dequant-dot (qwen38_quant.c:330-508, 2768-2810). */
float q38o_dot_row_f32(uint32_t type, const uint8_t *row, const float *x, uint64_t width)
{
    float total = 0.0f;
    switch (type) {
    case Q38O_F32:
        for (uint64_t i = 0; i < width; ++i) {
            float v;
            memcpy(&v, row + i * 4, 4);
            total = fmaf(v, x[i], total);
        }
        return total;
    case Q38O_F16:
        for (uint64_t i = 0; i < width; ++i)
            total = fmaf(q38o_f16_to_f32(load_u16(row + i * 2)), x[i], total);
        return total;
    case Q38O_BF16:
        for (uint64_t i = 0; i < width; ++i) total = fmaf(bf16_to_f32(row + i * 2), x[i], total);
        return total;
    case Q38O_Q2_K:
        for (uint64_t base = 0; base < width; base += 256, row += 84) {
            const float d = q38o_f16_to_f32(load_u16(row + 80));
            const float dmin = q38o_f16_to_f32(load_u16(row + 82));
            int si = 0;
            for (int half = 0; half < 2; ++half)
                for (int field = 0; field < 4; ++field)
                    for (int group = 0; group < 2; ++group) {
                        const uint8_t ps = row[si++];
                        const float scale = d * (float)(ps & 15u);
                        const float minimum = dmin * (float)(ps >> 4);
                        const uint64_t off = base + half * 128u + field * 32u + group * 16u;
                        const uint8_t *pk = row + 16 + half * 32 + group * 16;
                        for (int lane = 0; lane < 16; ++lane) {
                            const int q = (pk[lane] >> (field * 2)) & 3;
                            total = fmaf(scale * (float)q - minimum, x[off + lane], total);
                        }
                    }
        }
        return total;
    case Q38O_Q3_K:
        for (uint64_t base = 0; base < width; base += 256, row += 110) {
            const uint8_t *high = row, *low = row + 32;
            int scales[16];
            unpack_q3_scales(row + 96, scales);
            const float d = q38o_f16_to_f32(load_u16(row + 108));
            int group = 0;
            uint8_t bit = 1;
            for (int half = 0; half < 2; ++half)
                for (int field = 0; field < 4; ++field, ++group, bit <<= 1) {
                    const uint8_t *pk = low + half * 32;
                    for (int lane = 0; lane < 32; ++lane) {
                        const int q = ((pk[lane] >> (field * 2)) & 3) - ((high[lane] & bit) ? 0 : 4);
                        const int s = scales[group * 2 + lane / 16];
                        total = fmaf(d * (float)s * (float)q,
                                     x[base + half * 128u + field * 32u + lane], total);
                    }
                }
        }
        return total;
    case Q38O_Q4_K:
        for (uint64_t base = 0; base < width; base += 256, row += 144) {
            const float d = q38o_f16_to_f32(load_u16(row));
            const float dmin = q38o_f16_to_f32(load_u16(row + 2));
            const uint8_t *q = row + 16;
            for (int chunk = 0; chunk < 4; ++chunk, q += 32) {
                int sc0, m0, sc1, m1;
                scale_min_k4(chunk * 2, row + 4, &sc0, &m0);
                scale_min_k4(chunk * 2 + 1, row + 4, &sc1, &m1);
                const float d0 = d * (float)sc0, mm0 = dmin * (float)m0;
                const float d1 = d * (float)sc1, mm1 = dmin * (float)m1;
                const float *xx = x + base + chunk * 64u;
                for (int i = 0; i < 32; ++i) total = fmaf(d0 * (float)(q[i] & 15u) - mm0, xx[i], total);
                for (int i = 0; i < 32; ++i) total = fmaf(d1 * (float)(q[i] >> 4) - mm1, xx[i + 32], total);
            }
        }
        return total;
    case Q38O_Q5_K:
        for (uint64_t base = 0; base < width; base += 256, row += 176) {
            const float d = q38o_f16_to_f32(load_u16(row));
            const float dmin = q38o_f16_to_f32(load_u16(row + 2));
            const uint8_t *high = row + 16, *low = row + 48;
            for (int chunk = 0; chunk < 4; ++chunk, low += 32) {
                int sc0, m0, sc1, m1;
                scale_min_k4(chunk * 2, row + 4, &sc0, &m0);
                scale_min_k4(chunk * 2 + 1, row + 4, &sc1, &m1);
                const float d0 = d * (float)sc0, mm0 = dmin * (float)m0;
                const float d1 = d * (float)sc1, mm1 = dmin * (float)m1;
                const int h0 = 1 << (2 * chunk), h1 = 2 << (2 * chunk);
                const float *xx = x + base + chunk * 64u;
                for (int i = 0; i < 32; ++i) {
                    const int q = (low[i] & 15) + ((high[i] & h0) ? 16 : 0);
                    total = fmaf(d0 * (float)q - mm0, xx[i], total);
                }
                for (int i = 0; i < 32; ++i) {
                    const int q = (low[i] >> 4) + ((high[i] & h1) ? 16 : 0);
                    total = fmaf(d1 * (float)q - mm1, xx[i + 32], total);
                }
            }
        }
        return total;
    case Q38O_Q6_K:
        for (uint64_t base = 0; base < width; base += 256, row += 210) {
            const uint8_t *low = row, *high = row + 128;
            const int8_t *scales = (const int8_t *)(row + 192);
            const float d = q38o_f16_to_f32(load_u16(row + 208));
            for (int half = 0; half < 2; ++half, low += 64, high += 32, scales += 8) {
                const float *xx = x + base + half * 128u;
                for (int i = 0; i < 32; ++i) {
                    const int si = i / 16;
                    const int q0 = ((low[i] & 15) | ((high[i] & 3) << 4)) - 32;
                    const int q1 = ((low[i + 32] & 15) | (((high[i] >> 2) & 3) << 4)) - 32;
                    const int q2 = ((low[i] >> 4) | (((high[i] >> 4) & 3) << 4)) - 32;
                    const int q3 = ((low[i + 32] >> 4) | (((high[i] >> 6) & 3) << 4)) - 32;
                    total = fmaf(d * (float)scales[si] * (float)q0, xx[i], total);
                    total = fmaf(d * (float)scales[si + 2] * (float)q1, xx[i + 32], total);
                    total = fmaf(d * (float)scales[si + 4] * (float)q2, xx[i + 64], total);
                    total = fmaf(d * (float)scales[si + 6] * (float)q3, xx[i + 96], total);
                }
            }
        }
        return total;
    case Q38O_Q8_0:
        for (uint64_t base = 0; base < width; base += 32, row += 34) {
            const float d = q38o_f16_to_f32(load_u16(row));
            const int8_t *q = (const int8_t *)(row + 2);
            for (int i = 0; i < 32; ++i) total = fmaf(d * (float)q[i], x[base + i], total);
        }
        return total;
    case Q38O_IQ4_NL:
        for (uint64_t base = 0; base < width; base += 32, row += 18) {
            const float d = q38o_f16_to_f32(load_u16(row));
            for (int lane = 0; lane < 16; ++lane) {
                const uint8_t p = row[2 + lane];
                total = fmaf(d * (float)Q38_IQ4NL_LEVELS[p & 15u], x[base + lane], total);
                total = fmaf(d * (float)Q38_IQ4NL_LEVELS[p >> 4], x[base + lane + 16], total);
            }
        }
        return total;
    default:
        return NAN;
    }
}

/* qwen38_quant.c:2924-2948. */
int q38o_gemm_f32(float *output, const float *input, uint32_t batch, uint64_t width,
                  uint32_t type, const uint8_t *data, uint64_t rows)
{
    const uint32_t be = q38o_block_elements(type), bb = q38o_block_bytes(type);
    if (!output || !input || !data || !batch || !be || width % be) return 0;
    const uint64_t row_bytes = width / be * bb;
    for (uint64_t row = 0; row < rows; ++row)
        for (uint32_t t = 0; t < batch; ++t)
            output[(uint64_t)t * rows + row] =
                q38o_dot_row_f32(type, data + row * row_bytes, input + (uint64_t)t * width, width);
    return 1;
}

/* qwen38_quant.c:3186-3222: element i of a quantized row is the float dot of
 * its block against the unit basis vector e_i. */
int q38o_row_f32(float *output, uint32_t type, const uint8_t *data, uint64_t width,
                 uint64_t rows, uint64_t row)
{
    const uint32_t be = q38o_block_elements(type), bb = q38o_block_bytes(type);
    if (!output || !data || !be || width % be || row >= rows) return 0;
    const uint64_t row_bytes = width / be * bb;
    const uint8_t *r = data + row * row_bytes;
    if (type == Q38O_F32) { memcpy(output, r, width * 4); return 1; }
    if (type == Q38O_F16) { for (uint64_t i = 0; i < width; ++i) output[i] = q38o_f16_to_f32(load_u16(r + 2 * i)); return 1; }
    if (type == Q38O_BF16) { for (uint64_t i = 0; i < width; ++i) output[i] = bf16_to_f32(r + 2 * i); return 1; }
    float basis[256] = {0};
    for (uint64_t base = 0; base < width; base += be) {
        for (uint64_t i = 0; i < be; ++i) {
            basis[i] = 1.0f;
            output[base + i] = q38o_dot_row_f32(type, r + base / be * bb, basis, be);
            basis[i] = 0.0f;
        }
    }
    return 1;
}
