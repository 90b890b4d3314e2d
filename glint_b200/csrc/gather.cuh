/* Column-parallel output gather over peer memory, shared by the decode kernels
 * (htile_decode.cu) and the prefill GEMM (htile_gemm.cu).
 *
 * A rank holds rows [n0, n0 + N) of a weight whose output y[M, ldy] every rank
 * needs whole.  The kernel's epilogue stores each output element into every
 * rank's y (yr[r]: rank r's buffer as mapped in this process; plain stores over
 * NVLink, no peer loads, no multicast), then the kernel counts itself in and
 * signals every rank (gather_complete).  world == 0 means a plain, ungathered
 * call.
 *
 * Counters: flag (this rank's, 9 uint32, zero-initialised) holds in [r] the calls
 * whose rows rank r has delivered here and not yet taken, and in [kMaxGather] the
 * CTAs of the running call that are done.
 */
#ifndef GLINT_B200_GATHER_CUH_
#define GLINT_B200_GATHER_CUH_

#include <cuda_bf16.h>
#include <stdint.h>

#include "ptx.cuh"

namespace glint {

constexpr int kMaxGather = 8;
struct GatherArgs {
    int world, rank, ldy, n0;
    uint32_t *flag; /* this rank's counters */
    void *yr[kMaxGather];
    uint32_t *fr[kMaxGather]; /* every rank's counters */
};

/* y[col, n0 + n] = v in every rank's y: NVLink stores to the peers, a local store
 * for this rank */
template <bool BF16OUT>
__device__ __forceinline__ void gather_store(const GatherArgs &g, int col, int n, float v)
{
    const int64_t o = (int64_t)col * g.ldy + g.n0 + n;
    for (int r = 0; r < g.world; ++r) {
        if (BF16OUT)
            static_cast<__nv_bfloat16 *>(g.yr[r])[o] = __float2bfloat16_rn(v);
        else
            static_cast<float *>(g.yr[r])[o] = v;
    }
}

/* End of a gathered call, run by every one of a CTA's `active` producing warps
 * after its last y stores.  The warp counts itself in, first in its CTA (shared
 * memory, *cta_done zero at the start of the call), the CTA's last warp then in
 * the rank (one global atomic per CTA); the rank's last warp resets the count
 * and, after a system-scope fence, adds one to its own slot in every rank's
 * counters, then waits (acquire, system scope), bounded, for one arrival from
 * every rank and takes it (subtracts one).  Each rank's arrivals come in call
 * order and a rank can be at most one call ahead (its next call cannot finish
 * before this rank's arrival), so taking one per rank per call never confuses
 * calls; nothing here depends on a call number, so the same launch can be
 * replayed (CUDA graphs).  The kernel completes only when this rank's y holds
 * every rank's rows.  Ranks run on different GPUs; inside a rank only this one
 * warp waits.  A wait that runs out ORs kErrTimeout into *err_word. */
__device__ __forceinline__ void gather_complete(const GatherArgs &a, int active, uint32_t lane, uint32_t *cta_done,
                                                int *err_word)
{
    /* the counting chain orders every warp's stores before the rank's last warp
     * with device-scope acquire-release fences (fence, count; observe the count,
     * fence); that warp's one system-scope acquire-release fence followed by the
     * signals forms a release pattern that covers them all (an sc fence, or a
     * release on every signal, cost ~5 us more per call for the same ordering) */
    __syncwarp();
    if (lane != 0)
        return;
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
    if (atomicAdd(cta_done, 1u) + 1u != (uint32_t)active)
        return;
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
    if (atomicAdd(a.flag + kMaxGather, 1u) + 1u != gridDim.x)
        return;
    atomicExch(a.flag + kMaxGather, 0u);
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    for (int r = 0; r < a.world; ++r)
        asm volatile("red.relaxed.sys.global.add.u32 [%0], 1;" ::"l"(a.fr[r] + a.rank) : "memory");
    const long long t0 = clock64();
    for (int r = 0; r < a.world; ++r) {
        while (true) {
            uint32_t v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(a.flag + r) : "memory");
            if (v != 0u) {
                atomicSub(a.flag + r, 1u);
                break;
            }
            if (clock64() - t0 > kWaitCycles) {
                atomicOr(err_word, kErrTimeout);
                return;
            }
            __nanosleep(128);
        }
    }
}

/* GatherArgs for rank `rank` of `world` from the host arrays of every rank's y
 * and counters (false for a layout the kernels do not cover). */
inline bool make_gather_args(GatherArgs *g, void *const *y_ranks, uint32_t *const *flag_ranks, int world, int rank,
                             int ldy, int n0)
{
    if (world < 1 || world > kMaxGather || rank < 0 || rank >= world)
        return false;
    *g = GatherArgs{};
    g->world = world, g->rank = rank, g->ldy = ldy, g->n0 = n0, g->flag = flag_ranks[rank];
    for (int r = 0; r < world; ++r)
        g->yr[r] = y_ranks[r], g->fr[r] = flag_ranks[r];
    return true;
}

} // namespace glint

#endif
