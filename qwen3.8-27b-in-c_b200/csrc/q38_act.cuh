// q38_act.cuh - activation math shared by the GEMV prologues and the model
// kernels: the upstream's scalar activation functions with its rounding
// (src/qwen38/qwen38_model.c:437-445, 603-614, compiled -ffp-contract=off), the
// upstream Q8_K quantizer (qwen38_quant.c:42-88, bit-exact) in warp form, and
// deterministic warp reductions.
#pragma once

#include <stdint.h>

#include "q38_types.cuh"

namespace q38 {

constexpr float kRmsEps = 1e-6f;  // Q38_RMS_EPS

__device__ __forceinline__ float act_silu(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x))); }
__device__ __forceinline__ float act_sigmoid(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x))); }
__device__ __forceinline__ float act_softplus(float x)
{
    return x > 20.0f ? x : logf(__fadd_rn(1.0f, expf(x)));
}

// upstream q38_nearest_int (qwen38_quant.c:42-48)
__device__ __forceinline__ int act_nearest_int(float v)
{
    const float shifted = __fadd_rn(v, 12582912.0f);
    return static_cast<int>(__float_as_uint(shifted) & 0x007fffffu) - 0x00400000;
}

__device__ __forceinline__ double act_warp_sum_d(double v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float act_warp_sum_f(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Largest |v| with the smallest index among equals: the element the upstream
// quantizer's strict `>` scan keeps (qwen38_quant.c:58-65).
struct AbsMax {
    float a;
    int i;
    float v;
};

__device__ __forceinline__ AbsMax act_better(AbsMax x, AbsMax y)
{
    return (y.a > x.a || (y.a == x.a && y.i < x.i)) ? y : x;
}

__device__ __forceinline__ AbsMax act_warp_absmax(AbsMax m)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        AbsMax other;
        other.a = __shfl_xor_sync(0xffffffffu, m.a, o);
        other.i = __shfl_xor_sync(0xffffffffu, m.i, o);
        other.v = __shfl_xor_sync(0xffffffffu, m.v, o);
        m = act_better(m, other);
    }
    return m;
}

// One 256-element block quantized to Q8_K by a warp, lane l holding
// elements 8l .. 8l + 7 in v[].  Outputs: the two quant words of the lane
// (elements 8l .. 8l + 7, little-endian int8), the bsum word of 16-element
// groups 2j and 2j + 1 (valid in lanes 4j; int16 pair as in Q38Q8KBlock.sums)
// and the block scale.
struct WarpQ8K {
    uint32_t q0, q1;
    uint32_t sums_word;
    float scale;
};

__device__ __forceinline__ WarpQ8K act_quantize_warp(const float (&v)[8])
{
    const int lane = threadIdx.x & 31;
    AbsMax m{0.0f, 0x7fffffff, 0.0f};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float a = fabsf(v[i]);
        if (a > m.a) m = AbsMax{a, lane * 8 + i, v[i]};
    }
    m = act_warp_absmax(m);
    WarpQ8K r;
    int q[8];
    int partial = 0;
    float inverse = 0.0f;
    if (m.a != 0.0f) inverse = __fdiv_rn(-127.0f, m.v);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        q[i] = m.a != 0.0f ? min(act_nearest_int(__fmul_rn(inverse, v[i])), 127) : 0;
        partial += q[i];
    }
    r.q0 = (q[0] & 0xFF) | (q[1] & 0xFF) << 8 | (q[2] & 0xFF) << 16 | static_cast<uint32_t>(q[3] & 0xFF) << 24;
    r.q1 = (q[4] & 0xFF) | (q[5] & 0xFF) << 8 | (q[6] & 0xFF) << 16 | static_cast<uint32_t>(q[7] & 0xFF) << 24;
    const int group = partial + __shfl_xor_sync(0xffffffffu, partial, 1);  // 16 elements (lanes 2k, 2k+1)
    const int next = __shfl_down_sync(0xffffffffu, group, 2);             // group of lanes 4j+2, 4j+3
    r.sums_word = (static_cast<uint32_t>(group) & 0xFFFFu) | static_cast<uint32_t>(next) << 16;
    r.scale = m.a != 0.0f ? __fdiv_rn(1.0f, inverse) : 0.0f;
    return r;
}

}  // namespace q38
