// q38_grid.cuh - IQ codebooks on the device and the per-CTA expansion of the
// compact tables (see gen_codebooks.py) into 8-byte shared-memory entries.
#pragma once

#define Q38_CODEBOOKS_MACROS_ONLY
#include "q38_codebooks.h"
#include "q38_types.cuh"

namespace q38 {

// Compact codebooks (see gen_codebooks.py), expanded per CTA into shared memory.
static __device__ const uint32_t d_iq1s_nib[2048] = Q38_IQ1S_GRID_NIB_INIT;
static __device__ const uint32_t d_iq2s_nib[1024] = Q38_IQ2S_GRID_NIB_INIT;

template <typename Dec>
struct NeedsGrid { static constexpr int kEntries = 0; };
template <> struct NeedsGrid<DecIQ1S> { static constexpr int kEntries = 2048; };
template <> struct NeedsGrid<DecIQ1M> { static constexpr int kEntries = 2048; };
template <> struct NeedsGrid<DecIQ2S> { static constexpr int kEntries = 1024; };

template <typename Dec, int MT, class A>
__device__ __forceinline__ void run_block(const uint8_t *blk, const A &a, int (&w)[MT], int (&x)[MT], float (&v)[MT],
                                          const uint2 *grid)
{
    if constexpr (NeedsGrid<Dec>::kEntries > 0)
        Dec::template block<MT, A>(blk, a, w, x, v, grid);
    else
        Dec::template block<MT, A>(blk, a, w, x, v);
}

template <typename Dec>
__device__ void build_grid(uint2 *grid)
{
    if constexpr (NeedsGrid<Dec>::kEntries == 2048) {
        for (int i = threadIdx.x; i < 2048; i += blockDim.x) {
            const uint32_t e = d_iq1s_nib[i];
            // nibble = value + 1  ->  signed byte value
            const uint32_t lo = e & 0x0F0F0F0Fu, hi = (e >> 4) & 0x0F0F0F0Fu;
            const uint32_t lo_v = ((lo | 0x80808080u) - 0x01010101u) ^ 0x80808080u;
            const uint32_t hi_v = ((hi | 0x80808080u) - 0x01010101u) ^ 0x80808080u;
            grid[i] = make_uint2(lo_v, hi_v);
        }
    } else if constexpr (NeedsGrid<Dec>::kEntries == 1024) {
        for (int i = threadIdx.x; i < 1024; i += blockDim.x) {
            const uint32_t e = d_iq2s_nib[i];
            // nibble = index into {8, 25, 43}: 8 + 17c + (c >> 1) per byte
            const uint32_t lo = e & 0x0F0F0F0Fu, hi = (e >> 4) & 0x0F0F0F0Fu;
            const uint32_t lo_v = lo * 17u + 0x08080808u + ((lo >> 1) & 0x01010101u);
            const uint32_t hi_v = hi * 17u + 0x08080808u + ((hi >> 1) & 0x01010101u);
            grid[i] = make_uint2(lo_v, hi_v);
        }
    }
}

}  // namespace q38
