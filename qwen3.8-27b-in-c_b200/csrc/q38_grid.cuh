// q38_grid.cuh - IQ codebooks on the device and the per-CTA expansion of the
// compact tables (see gen_codebooks.py) into 8-byte shared-memory entries.
#pragma once

#define Q38_CODEBOOKS_MACROS_ONLY
#include "q38_codebooks.h"
#include <type_traits>

#include "q38_types.cuh"
#include "q38_types_more.cuh"

namespace q38 {

// Compact codebooks (see gen_codebooks.py), expanded per CTA into shared memory.
static __device__ const uint32_t d_iq1s_nib[2048] = Q38_IQ1S_GRID_NIB_INIT;
static __device__ const uint32_t d_iq2s_nib[1024] = Q38_IQ2S_GRID_NIB_INIT;
static __device__ const uint32_t d_iq2xxs_nib[256] = Q38_IQ2XXS_GRID_NIB_INIT;
static __device__ const uint32_t d_iq2xs_nib[512] = Q38_IQ2XS_GRID_NIB_INIT;
static __device__ const uint16_t d_iq3xxs_c4[256] = Q38_IQ3XXS_GRID_C4_INIT;
static __device__ const uint16_t d_iq3s_c4[512] = Q38_IQ3S_GRID_C4_INIT;

template <typename Dec>
struct NeedsGrid { static constexpr int kEntries = 0; };
template <> struct NeedsGrid<DecIQ1S> { static constexpr int kEntries = 2048; };
template <> struct NeedsGrid<DecIQ1M> { static constexpr int kEntries = 2048; };
template <> struct NeedsGrid<DecIQ2S> { static constexpr int kEntries = 1024; };
template <> struct NeedsGrid<DecIQ2XXS> { static constexpr int kEntries = 256; };
template <> struct NeedsGrid<DecIQ2XS> { static constexpr int kEntries = 512; };
template <> struct NeedsGrid<DecIQ3XXS> { static constexpr int kEntries = 256; };
template <> struct NeedsGrid<DecIQ3S> { static constexpr int kEntries = 512; };

// IQ1: nibble = value + 1 -> signed byte value (-1, 0, 1).
__device__ __forceinline__ uint2 iq1_entry(uint32_t e)
{
    const uint32_t lo = e & 0x0F0F0F0Fu, hi = (e >> 4) & 0x0F0F0F0Fu;
    return make_uint2(((lo | 0x80808080u) - 0x01010101u) ^ 0x80808080u,
                      ((hi | 0x80808080u) - 0x01010101u) ^ 0x80808080u);
}

// IQ2: nibble = index c into the magnitudes {8, 25, 43} = 8 + 17c + (c >> 1).
__device__ __forceinline__ uint2 iq2_entry(uint32_t e)
{
    const uint32_t lo = e & 0x0F0F0F0Fu, hi = (e >> 4) & 0x0F0F0F0Fu;
    return make_uint2(lo * 17u + 0x08080808u + ((lo >> 1) & 0x01010101u),
                      hi * 17u + 0x08080808u + ((hi >> 1) & 0x01010101u));
}

// IQ3: four 4-bit indices into an 8-entry magnitude table (two words of
// bytes), picked with one byte permute; the entry's 4 bytes go in .x.
__device__ __forceinline__ uint2 iq3_entry(uint32_t c4, uint32_t m_lo, uint32_t m_hi)
{
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(m_lo), "r"(m_hi), "r"(c4 & 0x7777u));
    return make_uint2(d, 0u);
}

template <typename Dec>
__device__ __forceinline__ uint2 grid_entry(int i)
{
    if constexpr (NeedsGrid<Dec>::kEntries == 2048) return iq1_entry(d_iq1s_nib[i]);
    else if constexpr (std::is_same<Dec, DecIQ2S>::value) return iq2_entry(d_iq2s_nib[i]);
    else if constexpr (std::is_same<Dec, DecIQ2XXS>::value) return iq2_entry(d_iq2xxs_nib[i]);
    else if constexpr (std::is_same<Dec, DecIQ2XS>::value) return iq2_entry(d_iq2xs_nib[i]);
    else if constexpr (std::is_same<Dec, DecIQ3XXS>::value)
        return iq3_entry(d_iq3xxs_c4[i], 0x1C140C04u, 0x3E342C24u);  // 4, 12, ..., 52, 62
    else return iq3_entry(d_iq3s_c4[i], 0x07050301u, 0x0F0D0B09u);      // 1, 3, ..., 15
}

// Expand the codebook of Dec into `grid` with `threads` threads (thread `tid`).
template <typename Dec>
__device__ __forceinline__ void fill_grid(uint2 *grid, int tid, int threads)
{
    if constexpr (NeedsGrid<Dec>::kEntries > 0)
        for (int i = tid; i < NeedsGrid<Dec>::kEntries; i += threads) grid[i] = grid_entry<Dec>(i);
}

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
    fill_grid<Dec>(grid, threadIdx.x, blockDim.x);
}

}  // namespace q38
