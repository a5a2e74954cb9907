// q38_device.cuh - sm_100a device helpers shared by the kernels: 1-D TMA bulk
// copies with mbarrier completion, bounded barrier waits, integer dot
// instructions and exact scalar conversions.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace q38 {

// Status codes written to the device status word.
enum : int { kStatusOk = 0, kStatusWaitTimeout = 1, kStatusBadToken = 2 };

// Programmatic dependent launch: a kernel launched with the programmatic
// stream-serialization attribute may start before its predecessor finishes;
// it must call pdl_wait() before touching anything the predecessor reads or
// writes.  pdl_launch_dependents() lets the next kernel start its prologue.
// Both are no-ops for kernels launched without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents()
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Wall-clock bound for any spin on an mbarrier (ns).  A bulk copy completes
// in microseconds; hitting this means the copy was lost.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_addr(const void *p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_timer_ns()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Launch timeline (profiling; a null record disables it).  A record is
// kTraceFields %globaltimer stamps, each the earliest (min) or latest (max)
// over the launch's CTAs: [0] min start, [1] min return from the grid-
// dependency wait, [2] max end, and for the weight-streaming GEMV [3] max
// activation staged, [4] max weights decoded, [5] max start, [6] max return
// from the wait, [7] min activation staged, [8] min RMSNorm sum of squares
// known, [9] min first activation floats arrived in thread 0, [10] min warp 0
// done quantizing (the last three for a fused RMSNorm input only).  Thread 0 of every CTA marks; the host
// initializes min fields to ~0 and max fields to 0.
enum : int {
    kTraceStart = 0, kTraceReady = 1, kTraceEnd = 2, kTraceStaged = 3, kTraceDecoded = 4,
    kTraceLastStart = 5, kTraceLastReady = 6, kTraceFirstStaged = 7, kTraceNormed = 8,
    kTraceXLoaded = 9, kTraceQuantized = 10
};
constexpr int kTraceFields = 11;
__host__ __device__ constexpr bool trace_is_min(int which)
{
    return which == kTraceStart || which == kTraceReady || which >= kTraceFirstStaged;
}
__device__ __forceinline__ void trace_mark(unsigned long long *rec, int which)
{
    if (!rec || threadIdx.x != 0) return;
    const unsigned long long t = global_timer_ns();
    if (trace_is_min(which)) atomicMin(rec + which, t);
    else atomicMax(rec + which, t);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_mbar_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Order this thread's earlier generic-proxy shared-memory accesses before
// later async-proxy (bulk copy) accesses to the same buffer.
__device__ __forceinline__ void fence_proxy_async_shared()
{
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

// 1-D TMA: copy `bytes` (multiple of 16) from global `src` (16-byte aligned)
// into shared `dst` (16-byte aligned); completion is signalled on `bar`.
// Plain (non-multicast) form only.
__device__ __forceinline__ void bulk_copy_g2s(void *dst, const void *src, uint32_t bytes,
                                              uint64_t *bar)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// L2 policy for data read once: evict it before anything else.
__device__ __forceinline__ uint64_t l2_evict_first_policy()
{
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}

// bulk_copy_g2s with an L2 cache-policy hint.
__device__ __forceinline__ void bulk_copy_g2s_hint(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                                   uint64_t policy)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
            "r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// Prefetch [src, src + bytes) into L2 (16-byte aligned, a multiple of 16
// bytes); nothing waits for it.
__device__ __forceinline__ void bulk_prefetch_l2(const void *src, uint32_t bytes)
{
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// This CTA's share of an L2 prefetch of [base, base + bytes): the range is cut
// into gridDim.x 16-byte-aligned pieces issued in 1 MiB requests.
__device__ __forceinline__ void prefetch_share_l2(const void *base, long long bytes)
{
    if (!base || bytes <= 0) return;
    const long long n = bytes >> 4;  // 16-byte units
    const long long g = gridDim.x, c = blockIdx.x;
    long long lo = n * c / g, hi = n * (c + 1) / g;
    const char *p = static_cast<const char *>(base);
    while (lo < hi) {
        const long long take = hi - lo < 65536 ? hi - lo : 65536;
        bulk_prefetch_l2(p + (lo << 4), static_cast<uint32_t>(take << 4));
        lo += take;
    }
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity)
{
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Wait for phase `parity` of `bar`, giving up after `limit_ns` (default
// kWaitLimitNs).  Returns false (and records kStatusWaitTimeout) when the wait
// was abandoned.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, int *status,
                                                  unsigned long long limit_ns = kWaitLimitNs)
{
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long start = global_timer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_timer_ns() - start > limit_ns) {
            if (status) atomicExch(status, kStatusWaitTimeout);
            return false;
        }
    }
    return true;
}

// ---- integer dot products -------------------------------------------------

// signed bytes x signed bytes
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c)
{
    return __dp4a(static_cast<int>(a), static_cast<int>(b), c);
}

// unsigned bytes (a) x signed bytes (b)
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c)
{
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// two signed 16-bit lanes of a x signed bytes 0,1 (lo) or 2,3 (hi) of b
__device__ __forceinline__ int dp2a_lo_ss(uint32_t a, uint32_t b, int c)
{
    int d;
    asm("dp2a.lo.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp2a_hi_ss(uint32_t a, uint32_t b, int c)
{
    int d;
    asm("dp2a.hi.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// byte permute with the PTX default mode (selector bit 3 = sign-replicate)
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel)
{
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// Four sign bits -> four byte masks (0xFF where the bit is set).
__device__ __forceinline__ uint32_t sign_mask4(uint32_t bits4)
{
    // bit k of bits4 lands on the MSB of byte k; prmt replicates each MSB.
    return prmt(bits4 * 0x10204080u, 0u, 0xBA98u);
}

// Negate the bytes of `m` (all in 1..127) where `mask` bytes are 0xFF.
// (m ^ 0xFF) + 1 never carries for m >= 1, so whole-word arithmetic is exact.
__device__ __forceinline__ uint32_t apply_signs(uint32_t m, uint32_t mask)
{
    return (m ^ mask) + (mask & 0x01010101u);
}

// ---- exact scalar conversions ----------------------------------------------

__device__ __forceinline__ float f16_bits_to_f32(uint32_t bits16)
{
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16)));
}

__device__ __forceinline__ uint32_t byte_of(uint32_t w, int k)
{
    return (w >> (8 * k)) & 0xFFu;
}

__device__ __forceinline__ int sbyte_of(uint32_t w, int k)
{
    return static_cast<int>(static_cast<int8_t>((w >> (8 * k)) & 0xFFu));
}

// Load `N` consecutive 32-bit words starting at an arbitrary (2-byte aligned)
// shared-memory byte address.  Reads one word past the end: callers leave
// 16 bytes of slack after every buffer.
template <int N>
__device__ __forceinline__ void lds_words(const uint8_t *p, uint32_t (&out)[N])
{
    const uintptr_t addr = reinterpret_cast<uintptr_t>(p);
    const uint32_t *base = reinterpret_cast<const uint32_t *>(addr & ~uintptr_t(3));
    const uint32_t shift = static_cast<uint32_t>(addr & 3u) * 8u;
    uint32_t prev = base[0];
#pragma unroll
    for (int i = 0; i < N; ++i) {
        const uint32_t next = base[i + 1];
        out[i] = __funnelshift_r(prev, next, shift);
        prev = next;
    }
}

}  // namespace q38
