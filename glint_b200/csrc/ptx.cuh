/* Inline-PTX building blocks for the sm_100a kernels: mbarriers with bounded
 * waits, TMA bulk / tensor copies (no cluster multicast anywhere), async-proxy
 * fences and small arithmetic forms the compiler does not emit on request.
 *
 * Bounded waits: a wait that has not completed after kWaitCycles of clock64()
 * (about a second) records `err_bit` in the translation unit's error word and
 * returns false, so the kernel can stop, drain its own copies and exit instead
 * of hanging.
 */
#ifndef GLINT_B200_PTX_CUH_
#define GLINT_B200_PTX_CUH_

#include <cuda.h>
#include <stdint.h>

namespace glint {

constexpr long long kWaitCycles = 2000000000LL; /* ~1 s at 2 GHz */
constexpr int kErrTimeout = 1;

__device__ __forceinline__ uint32_t saddr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_init_fence() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}\n"
                 : "=r"(ok)
                 : "r"(saddr(bar)), "r"(parity)
                 : "memory");
    return ok != 0;
}
/* Wait for the phase of parity `parity` to complete, at most ~kWaitCycles. */
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, int *err_word)
{
    if (mbar_try_wait(bar, parity))
        return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > kWaitCycles) {
            atomicOr(err_word, kErrTimeout);
            return false;
        }
    }
    return true;
}

/* try_wait that lets the hardware suspend the warp until the phase completes or
 * about `ns` nanoseconds pass, so waiting warps do not take issue slots from the
 * warps that work. */
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t *bar, uint32_t parity, uint32_t ns)
{
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}\n"
                 : "=r"(ok)
                 : "r"(saddr(bar)), "r"(parity), "r"(ns)
                 : "memory");
    return ok != 0;
}
/* Bounded wait as mbar_wait_bounded, suspending between polls. */
__device__ __forceinline__ bool mbar_wait_suspend_bounded(uint64_t *bar, uint32_t parity, int *err_word)
{
    if (mbar_try_wait(bar, parity))
        return true;
    const long long t0 = clock64();
    while (!mbar_try_wait_suspend(bar, parity, 20000u)) {
        if (clock64() - t0 > kWaitCycles) {
            atomicOr(err_word, kErrTimeout);
            return false;
        }
    }
    return true;
}

/* 1-D bulk copy global -> this CTA's shared memory, completion on `bar`.
 * dst and src 16-byte aligned, bytes a multiple of 16. */
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     saddr(dst)),
                 "l"(src), "r"(bytes), "r"(saddr(bar))
                 : "memory");
}
/* 2-D tiled TMA load of this GPU's memory into shared memory (no multicast). */
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            saddr(dst)),
        "l"(map), "r"(saddr(bar)), "r"(x), "r"(y)
        : "memory");
}
/* 3-D tiled TMA load of this GPU's memory into shared memory (no multicast). */
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y, int z)
{
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
            "r"(saddr(dst)),
        "l"(map), "r"(saddr(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ uint2 lds64(uint32_t a)
{
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t a)
{
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
/* 16-byte shared load issued only where `p` holds (zeros elsewhere): lanes that
 * skip it take no shared-memory bandwidth. */
__device__ __forceinline__ uint4 lds128_if(uint32_t a, bool p)
{
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.u32 q, %5, 0;\n\t"
                 "@q ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];\n\t}\n"
                 : "+r"(v.x), "+r"(v.y), "+r"(v.z), "+r"(v.w)
                 : "r"(a), "r"(p ? 1u : 0u));
    return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a)
{
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}

/* RN(a*b + c) clamped to [0, 1]; NaN becomes 0. */
__device__ __forceinline__ float fma_sat(float a, float b, float c)
{
    float d;
    asm("fma.rn.sat.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

} // namespace glint

#endif
