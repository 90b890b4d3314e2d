/* GLINT H-TILE for prefill-shaped calls (large M) on sm_100a tensor cores.
 *
 * Same contract as the reference's glint_htile_s3_f32 (cuda/glint_htile.cu:124-164):
 *   y[m, n] = sum_k GLINT_CELLS[h][p] * absmax[(n*K + k) / bs] * x[m, k].
 * The reference runs scalar f32 FMAs, one output per thread; here the GLINT
 * weights are dequantised once per CTA tile into shared memory and fed to
 * tcgen05 UMMAs with f32 accumulators in tensor memory.
 *
 * CTA tile 256 (M) x 256 (N), K step 64, three pipeline stages:
 *   warp 0      TMA producer: x tile [256 x 64] BF16 (128B swizzle) per stage;
 *   warp 1      TMEM allocator; one elected lane issues the UMMAs: per K step
 *               4 x (M=128, N=256, K=16) for each of the two 128-row halves,
 *               then tcgen05.commit to free the stage;
 *   warps 2..9  one weight row each (256 rows): stream 32 B of each plane per K
 *               step, look the 64 codes up in a per-lane replica of the codebook,
 *               scale by the row's absmax in f32, round to BF16 and store them in
 *               the UMMA K-major 128B-swizzle layout; after the K loop they move
 *               the accumulators (512 TMEM columns) to y.
 * Weights reach the MMA as RN_bf16(cell * absmax) (relative error <= 2^-9 per
 * weight), i.e. the GLINT_HTILE_FAST arithmetic.  The activation loads are plain
 * TMA loads of this GPU's memory (no cluster multicast anywhere).
 *
 * Every wait on an mbarrier is bounded (about one second of clock64 time); when
 * a wait runs out the kernel records an error in g_glint_kernel_error, skips the
 * rest of its work, waits (bounded) for its own TMA loads and releases TMEM.
 */
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "glint_internal.h"

namespace glint {

__device__ int g_glint_kernel_error = 0;

namespace {

constexpr int BM = 256, BN = 256, BK = 64, STAGES = 3;
constexpr int kThreads = 320;                   /* 10 warps */
constexpr int kStageA = BM * BK * 2;            /* 32 KB */
constexpr int kStageB = BN * BK * 2;            /* 32 KB */
constexpr int kLutBytes = 256 * 32 * 4;         /* f32 codebook, one replica per lane */
constexpr int kSmemBytes = STAGES * (kStageA + kStageB) + kLutBytes + 1024 /* barriers + align slack */;
constexpr long long kWaitCycles = 2000000000LL; /* ~1 s at 2 GHz */
constexpr int kErrTimeout = 1;

/* ---- PTX wrappers ------------------------------------------------------------ */
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}\n"
                 : "=r"(ok)
                 : "r"(smem_u32(bar)), "r"(parity)
                 : "memory");
    return ok != 0;
}
/* Bounded wait: false (and the error flag set) if the phase does not complete. */
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, bool &alive)
{
    if (!alive)
        return false;
    if (mbar_try_wait(bar, parity))
        return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > kWaitCycles) {
            atomicOr(&g_glint_kernel_error, kErrTimeout);
            alive = false;
            return false;
        }
    }
    return true;
}
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y)
{
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
                 ::"r"(smem_u32(dst)), "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
                 : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void umma_bf16(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc)
{
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d),
                 "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void umma_commit(uint64_t *bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32])
{
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 "
                 "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                 "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                   "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
                   "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
                   "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

/* UMMA shared-memory descriptor, K-major, 128-byte swizzle: 8-row atoms of
 * 1024 B (SBO), leading offset unused for swizzled K-major (field 1), version 1. */
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr)
{
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
/* instruction descriptor: f32 accumulate, BF16 A and B, both K-major, M=128, N=256 */
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);

struct GemmArgs {
    const uint8_t *hole;
    const uint8_t *plug;
    const float *absmax;
    void *y;
    int M, N, K, bs64;
    int y_bf16;
};

__global__ void __launch_bounds__(kThreads, 1) htile_gemm_kernel(const __grid_constant__ CUtensorMap xmap,
                                                                 const GemmArgs args)
{
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    /* 1024-align the operand stages (the swizzle pattern repeats every 1024 B) */
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem;
    uint8_t *sB = smem + STAGES * kStageA;
    float *lut = reinterpret_cast<float *>(sB + STAGES * kStageB);
    uint64_t *full_a = reinterpret_cast<uint64_t *>(reinterpret_cast<uint8_t *>(lut) + kLutBytes);
    uint64_t *full_b = full_a + STAGES;
    uint64_t *empty = full_b + STAGES;
    uint64_t *acc_full = empty + STAGES;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_full + 1);

    const int warp = threadIdx.x >> 5;
    const uint32_t lane = lane_id();
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int ksteps = args.K / BK;

    for (int i = threadIdx.x; i < 256 * 32; i += kThreads)
        lut[i] = (&g_cells[0][0])[i >> 5];
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full_a[s], 1);
            mbar_init(&full_b[s], 8); /* one arrive per producer warp */
            mbar_init(&empty[s], 1);  /* tcgen05.commit */
        }
        mbar_init(acc_full, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(512)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool alive = true;

    if (warp == 0) {
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(&xmap) : "memory");
            int issued = 0;
            for (int ks = 0; ks < ksteps && alive; ++ks) {
                const int s = ks % STAGES;
                const uint32_t ph = (uint32_t)(ks / STAGES) & 1u;
                if (ks >= STAGES && !mbar_wait(&empty[s], ph ^ 1u, alive))
                    break;
                mbar_expect_tx(&full_a[s], kStageA);
                tma_load_2d(sA + s * kStageA, &xmap, &full_a[s], ks * BK, m0);
                ++issued;
            }
            /* never leave the CTA with a TMA load in flight */
            bool drain = true;
            for (int ks = std::max(0, issued - STAGES); ks < issued; ++ks)
                mbar_wait(&full_a[ks % STAGES], (uint32_t)(ks / STAGES) & 1u, drain);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            for (int ks = 0; ks < ksteps && alive; ++ks) {
                const int s = ks % STAGES;
                const uint32_t ph = (uint32_t)(ks / STAGES) & 1u;
                if (!mbar_wait(&full_a[s], ph, alive) || !mbar_wait(&full_b[s], ph, alive))
                    break;
                tc_fence_after();
                const uint32_t a0 = smem_u32(sA + s * kStageA), b0 = smem_u32(sB + s * kStageB);
#pragma unroll
                for (int h = 0; h < 2; ++h) {
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
                        const uint64_t ad = sw128_desc(a0 + h * (128 * 128) + kk * 32);
                        const uint64_t bd = sw128_desc(b0 + kk * 32);
                        umma_bf16(tmem + h * BN, ad, bd, kIdesc, (ks > 0 || kk > 0) ? 1u : 0u);
                    }
                }
                umma_commit(&empty[s]);
            }
            if (alive)
                umma_commit(acc_full);
        }
    } else {
        /* ---- dequant producers: one weight row per thread */
        const int r = threadIdx.x - 64;
        const int n = n0 + r;
        const bool rv = n < args.N;
        const int K2 = args.K >> 1;
        const float *cl = lut + lane;
        const uint8_t *hrow = args.hole + (int64_t)(rv ? n : 0) * K2;
        const uint8_t *prow = args.plug + (int64_t)(rv ? n : 0) * K2;
        uint32_t am_idx = (uint32_t)(rv ? n : 0) * (uint32_t)ksteps;
        uint32_t am_rem = am_idx % (uint32_t)args.bs64;
        am_idx /= (uint32_t)args.bs64;
        uint8_t *brow_base = sB + r * 128;
        const uint32_t sw = (uint32_t)(r & 7);
        /* register ring: the planes and absmax of the next kPF K steps are in flight
         * while a step is dequantised (global latency is far above one step) */
        constexpr int kPF = 4;
        uint4 rh0[kPF], rh1[kPF], rp0[kPF], rp1[kPF];
        float rsc[kPF];
        auto fetch = [&](int ks, uint4 &h0, uint4 &h1, uint4 &p0, uint4 &p1, float &sc) {
            if (rv && ks < ksteps) {
                const uint4 *hp = reinterpret_cast<const uint4 *>(hrow + ks * 32);
                const uint4 *pp = reinterpret_cast<const uint4 *>(prow + ks * 32);
                h0 = __ldcs(hp);
                h1 = __ldcs(hp + 1);
                p0 = __ldcs(pp);
                p1 = __ldcs(pp + 1);
                sc = __ldg(args.absmax + am_idx);
            } else {
                h0 = h1 = p0 = p1 = make_uint4(0, 0, 0, 0);
                sc = 0.f;
            }
            if (++am_rem == (uint32_t)args.bs64) {
                am_rem = 0;
                ++am_idx;
            }
        };
#pragma unroll
        for (int j = 0; j < kPF; ++j)
            fetch(j, rh0[j], rh1[j], rp0[j], rp1[j], rsc[j]);
        for (int ks0 = 0; ks0 < ksteps && alive; ks0 += kPF) {
#pragma unroll
            for (int j = 0; j < kPF; ++j) {
                const int ks = ks0 + j;
                if (ks >= ksteps || !alive)
                    break;
                const int s = ks % STAGES;
                const uint32_t ph = (uint32_t)(ks / STAGES) & 1u;
                const uint32_t hw[8] = {rh0[j].x, rh0[j].y, rh0[j].z, rh0[j].w, rh1[j].x, rh1[j].y, rh1[j].z, rh1[j].w};
                const uint32_t pw[8] = {rp0[j].x, rp0[j].y, rp0[j].z, rp0[j].w, rp1[j].x, rp1[j].y, rp1[j].z, rp1[j].w};
                const float scur = rsc[j];
                fetch(ks + kPF, rh0[j], rh1[j], rp0[j], rp1[j], rsc[j]);
                if (ks >= STAGES) {
                    /* one lane waits, the warp follows its verdict (keeps the warp converged) */
                    bool go = lane == 0 ? mbar_wait(&empty[s], ph ^ 1u, alive) : true;
                    if (!__shfl_sync(0xFFFFFFFFu, go ? 1 : 0, 0)) {
                        alive = false;
                        break;
                    }
                }
                uint8_t *brow = brow_base + s * kStageB;
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    /* 8 weights: codes of elements 2b (E) and 2b+1 (O) in byte b */
                    const uint32_t E = ((hw[c] << 4) & 0xF0F0F0F0u) | (pw[c] & 0x0F0F0F0Fu);
                    const uint32_t O = (hw[c] & 0xF0F0F0F0u) | ((pw[c] >> 4) & 0x0F0F0F0Fu);
                    uint32_t o[4];
#pragma unroll
                    for (int b = 0; b < 4; ++b) {
                        const float v0 = cl[((E >> (8 * b)) & 0xFFu) * 32] * scur;
                        const float v1 = cl[((O >> (8 * b)) & 0xFFu) * 32] * scur;
                        __nv_bfloat162 h2 = __floats2bfloat162_rn(v0, v1);
                        o[b] = *reinterpret_cast<uint32_t *>(&h2);
                    }
                    *reinterpret_cast<uint4 *>(brow + (((uint32_t)c ^ sw) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
                }
                fence_proxy_async();
                __syncwarp();
                if (lane == 0)
                    mbar_arrive(&full_b[s]);
            }
        }
        /* ---- epilogue: TMEM -> y.  Warp w reads TMEM lanes 32*(w % 4); warps 2..5
         * take accumulator 0 (rows 0..127), warps 6..9 accumulator 1. */
        bool acc_ok = (lane == 0) ? mbar_wait(acc_full, 0, alive) : alive;
        acc_ok = __shfl_sync(0xFFFFFFFFu, acc_ok ? 1 : 0, 0) != 0 && __all_sync(0xFFFFFFFFu, alive);
        if (acc_ok) {
            tc_fence_after();
            const int q = warp & 3;
            const int h = (warp - 2) >> 2;
            const int m = m0 + h * 128 + q * 32 + (int)lane;
            const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(h * BN);
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t v[32];
                tmem_ld32(tbase + c * 32, v);
                tmem_ld_wait();
                const int nc = n0 + c * 32;
                if (m < args.M && nc < args.N) {
                    if (args.y_bf16) {
                        __nv_bfloat16 *yr = static_cast<__nv_bfloat16 *>(args.y) + (int64_t)m * args.N + nc;
                        if (nc + 32 <= args.N) {
#pragma unroll
                            for (int j = 0; j < 32; j += 8) {
                                uint32_t pk[4];
#pragma unroll
                                for (int t = 0; t < 4; ++t) {
                                    __nv_bfloat162 b2 = __floats2bfloat162_rn(__uint_as_float(v[j + 2 * t]),
                                                                              __uint_as_float(v[j + 2 * t + 1]));
                                    pk[t] = *reinterpret_cast<uint32_t *>(&b2);
                                }
                                *reinterpret_cast<uint4 *>(yr + j) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                            }
                        } else {
#pragma unroll
                            for (int j = 0; j < 32; ++j)
                                if (nc + j < args.N)
                                    yr[j] = __float2bfloat16_rn(__uint_as_float(v[j]));
                        }
                    } else {
                        float *yr = static_cast<float *>(args.y) + (int64_t)m * args.N + nc;
                        if (nc + 32 <= args.N) {
#pragma unroll
                            for (int j = 0; j < 32; j += 4)
                                *reinterpret_cast<uint4 *>(yr + j) = make_uint4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                        } else {
#pragma unroll
                            for (int j = 0; j < 32; ++j)
                                if (nc + j < args.N)
                                    yr[j] = __uint_as_float(v[j]);
                        }
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
    }
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder()
{
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        else
            cudaGetLastError();
    });
    return fn;
}

} // namespace

bool htile_gemm_supported(const uint8_t *hole, const uint8_t *plug, const float *am, const __nv_bfloat16 *x,
                          const void *y, bool y_bf16, int M, int N, int K, int bs)
{
    (void)am;
    return M >= 128 && K % BK == 0 && bs % 64 == 0 && aligned_to(hole, 16) && aligned_to(plug, 16) &&
           aligned_to(x, 16) && aligned_to(y, 16) && N % (y_bf16 ? 8 : 4) == 0 &&
           (int64_t)N * (K / 64) < (int64_t)0xFFFFFFFF && tensor_map_encoder() != nullptr;
}

int htile_gemm_launch(const uint8_t *hole, const uint8_t *plug, const float *am, const __nv_bfloat16 *x, void *y,
                      bool y_bf16, int M, int N, int K, int bs, cudaStream_t st)
{
    auto encode = tensor_map_encoder();
    if (!encode)
        return kLaunch;
    CUtensorMap map;
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
    cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    cuuint32_t box[2] = {BK, BM};
    cuuint32_t estr[2] = {1, 1};
    if (encode(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<__nv_bfloat16 *>(x), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return kLaunch;
    if (!ensure_smem((const void *)htile_gemm_kernel, kSmemBytes))
        return kLaunch;
    GemmArgs a{hole, plug, am, y, M, N, K, bs / 64, y_bf16 ? 1 : 0};
    dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
    htile_gemm_kernel<<<grid, kThreads, kSmemBytes, st>>>(map, a);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunch;
}

int read_kernel_error(bool clear)
{
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_glint_kernel_error, sizeof(int)) != cudaSuccess)
        return -1;
    if (clear && v) {
        const int z = 0;
        cudaMemcpyToSymbol(g_glint_kernel_error, &z, sizeof(int));
    }
    const int e = encode_error_word(clear), x = expand_error_word(clear), d = decode_error_word(clear);
    if (e < 0 || x < 0 || d < 0)
        return -1;
    return v | e | x | d;
}

} // namespace glint
