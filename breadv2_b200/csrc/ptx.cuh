// ptx.cuh -- inline-PTX helpers for sm_100a: mbarriers, 1-D bulk async copies
// (TMA, no multicast), bounded waits, integer dot products, exact small-int
// to float conversions.
#pragma once
#include <stdint.h>
#include "common.cuh"

namespace bread {

// Device-wide error word (bits DEVERR_*), read by bread_device_error().
extern __device__ unsigned g_dev_error;

__device__ __forceinline__ uint32_t smem_u32(const void *p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void flag_error(unsigned bit) { atomicOr(&g_dev_error, bit); }

// ---- mbarrier -------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t *bar, unsigned count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
// Make barrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_mbar_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, unsigned bytes)
{
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                     smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive_cnt(uint64_t *bar, unsigned count)
{
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
                 "r"(count)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, unsigned parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Wait for phase `parity` of `bar` to complete, at most SPIN_LIMIT polls.
// Returns false (and sets the device error word) when the budget runs out.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, unsigned parity)
{
    if (mbar_try_wait(bar, parity)) return true;
    for (long long i = 0; i < SPIN_LIMIT; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (i > 64) __nanosleep(64);
    }
    flag_error(DEVERR_TIMEOUT);
    return false;
}

// ---- 1-D bulk copy global -> shared (TMA engine, no multicast) ------------
// dst and src 16-byte aligned, bytes a multiple of 16.  Completion is counted
// on `bar` as transaction bytes.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, unsigned bytes, uint64_t *bar)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
// Prefetch [src, src + bytes) into L2 (bulk, no destination).  src 16-byte
// aligned, bytes a multiple of 16.
__device__ __forceinline__ void prefetch_l2(const void *src, unsigned bytes)
{
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
// Order this thread's generic-proxy shared-memory accesses before later
// async-proxy (bulk copy) accesses of the same bytes.
__device__ __forceinline__ void fence_proxy_async_smem()
{
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Order this thread's earlier generic-proxy view of global memory (e.g. data
// another CTA published and this thread acquired) before its later
// async-proxy (bulk copy) reads of it.
__device__ __forceinline__ void fence_proxy_async_global()
{
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// ---- acquire loads / release reductions on 64-bit counters -----------------
__device__ __forceinline__ unsigned long long ld_acquire_gpu(const unsigned long long *p)
{
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *p)
{
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
// Release-add at gpu scope (the grid-barrier counter).
__device__ __forceinline__ void red_release_gpu(unsigned long long *p, unsigned long long v)
{
    asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// Release-add at system scope (arrival counters in peers' memory over NVLink).
__device__ __forceinline__ void red_release_sys(unsigned long long *p, unsigned long long v)
{
    asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// Flagged exchange words: one 64-bit store / load at gpu scope (single-copy
// atomic, served by L2), payload in the low and tag in the high 32 bits.
__device__ __forceinline__ void st_flagged(unsigned long long *p, uint32_t payload, uint32_t tag)
{
    const unsigned long long w = ((unsigned long long)tag << 32) | payload;
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ld_flagged(const unsigned long long *p)
{
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p));
    return v;
}
// The same at system scope: words another GPU stores into this GPU's memory
// (or this GPU into a peer's) over NVLink.
__device__ __forceinline__ void st_flagged_sys(unsigned long long *p, uint32_t payload, uint32_t tag)
{
    const unsigned long long w = ((unsigned long long)tag << 32) | payload;
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ld_flagged_sys(const unsigned long long *p)
{
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ unsigned long long globaltimer()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ---- named barrier for a subset of warps -----------------------------------
__device__ __forceinline__ void named_sync(int id, int threads)
{
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---- programmatic dependent launch ---------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// ---- integer dot products ---------------------------------------------------
// a: two signed 16-bit values; b: four unsigned bytes.  lo uses bytes 0,1 of
// b, hi uses bytes 2,3:  c + a.h0*b.byte(0|2) + a.h1*b.byte(1|3).  Exact.
__device__ __forceinline__ int dp2a_lo(int a, unsigned b, int c)
{
    int d;
    asm("dp2a.lo.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp2a_hi(int a, unsigned b, int c)
{
    int d;
    asm("dp2a.hi.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
// Sum of the two signed 16-bit halves of a, plus c.
__device__ __forceinline__ int sum_i16x2(int a, int c) { return dp2a_lo(a, 0x0101u, c); }

// ---- exact small integer -> float ------------------------------------------
// For 0 <= u < 2^23: the float with bit pattern 0x4B000000|u is 2^23 + u, so
// subtracting 2^23 is exact.
__device__ __forceinline__ float u2f_small(uint32_t u)
{
    return __int_as_float(0x4B000000 | u) - 8388608.0f;
}
// For |s| < 2^22: 0x4B400000 is 1.5*2^23; adding s to the pattern adds s to
// the value, exactly.
__device__ __forceinline__ float s2f_small(int s)
{
    return __int_as_float(0x4B400000 + s) - 12582912.0f;
}

}  // namespace bread
