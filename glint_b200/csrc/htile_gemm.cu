/* GLINT H-TILE for prefill-shaped calls (large M) on sm_100a tensor cores.
 *
 * Same contract as the reference's glint_htile_s3_f32 (cuda/glint_htile.cu:124-164):
 *   y[m, n] = sum_k GLINT_CELLS[h][p] * absmax[(n*K + k) / bs] * x[m, k].
 * The reference runs scalar f32 FMAs, one output per thread.  Here the product
 * is computed transposed, y^T[n, m] = W[n, :] . x[m, :], so that the GLINT
 * weights are the UMMA's A operand and can live in tensor memory: dequantiser
 * warps write RN_bf16(cell * absmax) straight into TMEM with tcgen05.st, and
 * the weights never touch shared memory (no STS, no tensor-core smem reads of
 * W).  Only the activations stream through shared memory.
 *
 * Persistent CTAs (one per SM) walk tiles of 128 weight rows (n) x 256
 * activation rows (m); K steps of 64 (one absmax block) flow through a 4-stage
 * shared-memory ring and a 4-slot TMEM ring:
 *   warp 0      TMA producer: per K step the x tile [256 x 64] BF16 (128B
 *               swizzle) and the hole and plug tiles [128 rows x 32 B] (32B
 *               swizzle); every fourth step also an absmax box [128 rows x 4
 *               blocks].  Plain loads of this GPU's memory, no cluster multicast.
 *   warp 1      TMEM owner (512 columns: accumulator 0..255, weight ring
 *               256..383) and, in one lane, the UMMA issuer: per K step
 *               4 x (M=128, N=256, K=16) with A from TMEM, B = x from shared
 *               memory, then tcgen05.commit to release the stage and the slot;
 *   warps 2..9  dequantisers: warp w owns TMEM lanes 32*(w%4).. (weight rows)
 *               and half of the K step (32 weights per thread); codes are looked
 *               up in a per-lane replica of the codebook, scaled by the row's
 *               absmax in f32 and rounded to BF16 pairs;
 *   warps 10-13 epilogue: tcgen05.ld of the accumulator (lane = weight row,
 *               column = activation row) to y.
 * Weights reach the MMA as RN_bf16(cell * absmax) (relative error <= 2^-9 per
 * weight), i.e. the GLINT_HTILE_FAST arithmetic.
 *
 * Every wait on an mbarrier is bounded (about one second of clock64 time); when
 * a wait runs out the kernel records an error in g_glint_kernel_error, stops,
 * waits (bounded) for its own TMA loads and UMMAs and releases TMEM.
 */
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "glint_internal.h"
#include "ptx.cuh"

namespace glint {

__device__ int g_glint_kernel_error = 0;

namespace {

constexpr int BN = 128;      /* weight rows per tile (UMMA M) */
constexpr int BMX = 256;     /* activation rows per tile (UMMA N) */
constexpr int BK = 64;       /* one absmax block */
constexpr int STAGES = 4;    /* smem ring == TMEM weight ring depth */
constexpr int kThreads = 14 * 32;
constexpr int kDeqWarps = 8, kEpiWarps = 4;
constexpr int kStageX = BMX * BK * 2;   /* 32 KB */
constexpr int kPlaneBox = BN * BK / 2;  /* 4 KB: 128 rows x 32 B */
constexpr int kAmBox = BN * 4 * 4;      /* 2 KB: 128 rows x 4 blocks */
constexpr int kStageBytes = kStageX + 2 * kPlaneBox + kAmBox; /* 42 KB, a multiple of 1 KB */
constexpr int kLutBytes = 256 * 32 * 4; /* f32 codebook, one replica per lane */
constexpr int kSmemBytes = 1024 + STAGES * kStageBytes + kLutBytes + 256;
constexpr uint32_t kAccCol = 0, kWCol = 256; /* TMEM column bases */
constexpr uint32_t kTmemCols = 512;

__device__ __forceinline__ bool wait_or_fail(uint64_t *bar, uint32_t parity, bool &alive)
{
    if (!alive)
        return false;
    if (!mbar_wait_bounded(bar, parity, &g_glint_kernel_error))
        alive = false;
    return alive;
}
/* lane 0 waits, the warp follows its verdict (keeps the warp converged) */
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, bool &alive)
{
    bool ok = (lane_id() == 0) ? wait_or_fail(bar, parity, alive) : alive;
    ok = __shfl_sync(0xFFFFFFFFu, ok ? 1 : 0, 0) != 0;
    alive = ok;
    return ok;
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

/* D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16 (A and B both BF16) */
__device__ __forceinline__ void umma_ts_bf16(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t acc)
{
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d),
                 "r"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void umma_commit(uint64_t *bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(saddr(bar))
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
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16])
{
    asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
                 "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
                 "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
                 "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
                 : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

/* UMMA shared-memory descriptor, K-major, 128-byte swizzle: 8-row atoms of
 * 1024 B (SBO), leading offset unused for swizzled K-major (field 1), version 1. */
__device__ __forceinline__ uint64_t sw128_desc(uint32_t sa)
{
    return (uint64_t)((sa >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
/* instruction descriptor: f32 accumulate, BF16 A and B, both K-major, M=128, N=256 */
constexpr uint32_t kIdesc =
    (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BMX >> 3) << 17) | ((uint32_t)(BN >> 4) << 24);

/* (E, O) = codes of the even and odd weights of four plane bytes: code = h*16 + p */
__device__ __forceinline__ void codes4(uint32_t h, uint32_t p, uint32_t &E, uint32_t &O)
{
    E = ((h << 4) & 0xF0F0F0F0u) | (p & 0x0F0F0F0Fu);
    O = (h & 0xF0F0F0F0u) | ((p >> 4) & 0x0F0F0F0Fu);
}

struct GemmArgs {
    void *y;
    int M, N, K;
    int y_bf16;
    int mtiles, ntiles;
};

struct Maps {
    CUtensorMap x, h, p, am;
};

__global__ void __launch_bounds__(kThreads, 1) htile_gemm_kernel(const __grid_constant__ Maps maps, const GemmArgs args)
{
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float *lut = reinterpret_cast<float *>(smem + STAGES * kStageBytes);
    uint64_t *load_full = reinterpret_cast<uint64_t *>(reinterpret_cast<uint8_t *>(lut) + kLutBytes);
    uint64_t *load_empty = load_full + STAGES;
    uint64_t *w_full = load_empty + STAGES;
    uint64_t *w_empty = w_full + STAGES;
    uint64_t *acc_full = w_empty + STAGES;
    uint64_t *acc_empty = acc_full + 1;
    uint64_t *mma_done = acc_empty + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma_done + 1);

    const int warp = threadIdx.x >> 5;
    const uint32_t lane = lane_id();
    const int ksteps = args.K / BK;
    const int ntiles_total = args.mtiles * args.ntiles;

    for (int i = threadIdx.x; i < 256 * 32; i += kThreads)
        lut[i] = (&g_cells[0][0])[i >> 5];
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&load_full[s], 1);
            mbar_init(&load_empty[s], 1 + kDeqWarps); /* UMMA commit + dequantiser warps */
            mbar_init(&w_full[s], kDeqWarps);
            mbar_init(&w_empty[s], 1);
        }
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, kEpiWarps);
        mbar_init(mma_done, 1);
        mbar_init_fence();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool alive = true;

    if (warp == 0) {
        /* ---- TMA producer */
        if (lane == 0) {
            int64_t g = 0;
            for (int tile = blockIdx.x; tile < ntiles_total && alive; tile += gridDim.x) {
                const int m0 = (tile % args.mtiles) * BMX, n0 = (tile / args.mtiles) * BN;
                for (int ks = 0; ks < ksteps && alive; ++ks, ++g) {
                    const int s = (int)(g % STAGES);
                    const uint32_t ph = (uint32_t)(g / STAGES) & 1u;
                    if (g >= STAGES && !wait_or_fail(&load_empty[s], ph ^ 1u, alive))
                        break;
                    uint8_t *st = smem + s * kStageBytes;
                    const bool am = (ks & 3) == 0;
                    mbar_expect_tx(&load_full[s], kStageX + 2 * kPlaneBox + (am ? kAmBox : 0));
                    tma_load_2d(st, &maps.x, &load_full[s], ks * BK, m0);
                    tma_load_2d(st + kStageX, &maps.h, &load_full[s], ks * (BK / 2), n0);
                    tma_load_2d(st + kStageX + kPlaneBox, &maps.p, &load_full[s], ks * (BK / 2), n0);
                    if (am)
                        tma_load_2d(st + kStageX + 2 * kPlaneBox, &maps.am, &load_full[s], ks, n0);
                }
            }
            if (!alive) {
                /* let the loads already issued land before the CTA exits */
                bool drain = true;
                for (int64_t j = g > STAGES ? g - STAGES : 0; j < g && drain; ++j)
                    drain = mbar_wait_bounded(&load_full[(int)(j % STAGES)], (uint32_t)(j / STAGES) & 1u,
                                              &g_glint_kernel_error);
            }
        }
    } else if (warp == 1) {
        /* ---- UMMA issuer */
        if (lane == 0) {
            int64_t g = 0;
            int t = 0;
            for (int tile = blockIdx.x; tile < ntiles_total && alive; tile += gridDim.x, ++t) {
                if (t >= 1 && !wait_or_fail(acc_empty, (uint32_t)(t - 1) & 1u, alive))
                    break;
                tc_fence_after();
                for (int ks = 0; ks < ksteps && alive; ++ks, ++g) {
                    const int s = (int)(g % STAGES);
                    const uint32_t ph = (uint32_t)(g / STAGES) & 1u;
                    if (!wait_or_fail(&load_full[s], ph, alive) || !wait_or_fail(&w_full[s], ph, alive))
                        break;
                    tc_fence_after();
                    const uint32_t xs = saddr(smem + s * kStageBytes);
                    const uint32_t wa = tmem + kWCol + (uint32_t)s * (BK / 2);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk)
                        umma_ts_bf16(tmem + kAccCol, wa + kk * 8, sw128_desc(xs + kk * 32), kIdesc,
                                     (ks > 0 || kk > 0) ? 1u : 0u);
                    umma_commit(&load_empty[s]); /* x tile consumed */
                    umma_commit(&w_empty[s]);    /* weight slot consumed */
                }
                if (alive)
                    umma_commit(acc_full);
            }
            /* all UMMAs issued by this thread have completed before TMEM is released */
            umma_commit(mma_done);
            mbar_wait_bounded(mma_done, 0, &g_glint_kernel_error);
        }
        __syncwarp();
    } else if (warp < 2 + kDeqWarps) {
        /* ---- dequantisers: thread -> weight row r (TMEM lane), 32 weights (K half kh) */
        const int q = warp & 3, kh = (warp - 2) >> 2;
        const int r = q * 32 + (int)lane;
        const uint32_t cl = saddr(lut) + lane * 4u;
        const uint32_t pofs = (uint32_t)r * 32u + ((uint32_t)(kh ^ ((r >> 2) & 1)) << 4); /* 32B swizzle */
        const uint32_t tw = tmem + ((uint32_t)(q * 32) << 16) + kWCol + (uint32_t)kh * 16u;
        float4 sc4 = make_float4(0.f, 0.f, 0.f, 0.f);
        int64_t g = 0;
        for (int tile = blockIdx.x; tile < ntiles_total && alive; tile += gridDim.x) {
            for (int ks = 0; ks < ksteps && alive; ++ks, ++g) {
                const int s = (int)(g % STAGES);
                const uint32_t ph = (uint32_t)(g / STAGES) & 1u;
                if (!warp_wait(&load_full[s], ph, alive))
                    break;
                const uint32_t ps = saddr(smem + s * kStageBytes + kStageX);
                const uint4 H = lds128(ps + pofs);
                const uint4 P = lds128(ps + kPlaneBox + pofs);
                if ((ks & 3) == 0) {
                    const uint4 a = lds128(ps + 2 * kPlaneBox + (uint32_t)r * 16u);
                    sc4 = make_float4(__uint_as_float(a.x), __uint_as_float(a.y), __uint_as_float(a.z),
                                      __uint_as_float(a.w));
                }
                const float sc = (ks & 3) == 0 ? sc4.x : (ks & 3) == 1 ? sc4.y : (ks & 3) == 2 ? sc4.z : sc4.w;
                __syncwarp();
                if (lane == 0)
                    mbar_arrive(&load_empty[s]);
                if (g >= STAGES && !warp_wait(&w_empty[s], ph ^ 1u, alive))
                    break;
                tc_fence_after();
                const uint32_t hw[4] = {H.x, H.y, H.z, H.w}, pw[4] = {P.x, P.y, P.z, P.w};
                uint32_t o[16];
#pragma unroll
                for (int wq = 0; wq < 4; ++wq) {
                    uint32_t E, O;
                    codes4(hw[wq], pw[wq], E, O);
#pragma unroll
                    for (int b = 0; b < 4; ++b) {
                        const float v0 = __uint_as_float(lds32(cl + (((E >> (8 * b)) & 0xFFu) << 7))) * sc;
                        const float v1 = __uint_as_float(lds32(cl + (((O >> (8 * b)) & 0xFFu) << 7))) * sc;
                        __nv_bfloat162 h2 = __floats2bfloat162_rn(v0, v1);
                        o[wq * 4 + b] = *reinterpret_cast<uint32_t *>(&h2);
                    }
                }
                tmem_st16(tw + (uint32_t)s * (BK / 2), o);
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0)
                    mbar_arrive(&w_full[s]);
            }
        }
    } else {
        /* ---- epilogue: warp w reads TMEM lanes 32*(w%4): weight rows n, columns m */
        const int q = warp & 3;
        int t = 0;
        for (int tile = blockIdx.x; tile < ntiles_total && alive; tile += gridDim.x, ++t) {
            if (!warp_wait(acc_full, (uint32_t)t & 1u, alive))
                break;
            tc_fence_after();
            const int m0 = (tile % args.mtiles) * BMX, n0 = (tile / args.mtiles) * BN;
            const int n = n0 + q * 32 + (int)lane;
            const uint32_t tb = tmem + ((uint32_t)(q * 32) << 16) + kAccCol;
            const int mlim = min(BMX, args.M - m0);
#pragma unroll 1
            for (int c = 0; c < BMX / 32 && c * 32 < mlim; ++c) {
                uint32_t v[32];
                tmem_ld32(tb + c * 32, v);
                tmem_ld_wait();
                if (n < args.N) {
                    const int jl = min(32, mlim - c * 32);
                    const size_t step = (size_t)args.N;
                    if (args.y_bf16) {
                        __nv_bfloat16 *yp = static_cast<__nv_bfloat16 *>(args.y) + (size_t)(m0 + c * 32) * step + n;
#pragma unroll
                        for (int j = 0; j < 32; ++j, yp += step)
                            if (j < jl)
                                *yp = __float2bfloat16_rn(__uint_as_float(v[j]));
                    } else {
                        float *yp = static_cast<float *>(args.y) + (size_t)(m0 + c * 32) * step + n;
#pragma unroll
                        for (int j = 0; j < 32; ++j, yp += step)
                            if (j < jl)
                                *yp = __uint_as_float(v[j]);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0)
                mbar_arrive(acc_empty);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
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
    /* K % 256: the absmax rows (K/64 floats) must be a multiple of 16 bytes for TMA */
    (void)y;
    (void)y_bf16;
    return M >= 128 && K % 256 == 0 && bs == 64 && aligned_to(hole, 16) && aligned_to(plug, 16) &&
           aligned_to(am, 16) && aligned_to(x, 16) && tensor_map_encoder() != nullptr;
}

namespace {
bool encode_map(CUtensorMap *m, CUtensorMapDataType dt, const void *base, uint64_t cols, uint64_t rows,
                uint64_t row_bytes, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle sw)
{
    auto enc = tensor_map_encoder();
    if (!enc)
        return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    return enc(m, dt, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
} // namespace

int htile_gemm_launch(const uint8_t *hole, const uint8_t *plug, const float *am, const __nv_bfloat16 *x, void *y,
                      bool y_bf16, int M, int N, int K, int bs, cudaStream_t st)
{
    (void)bs;
    Maps maps;
    if (!encode_map(&maps.x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, BK, BMX,
                    CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_map(&maps.h, CU_TENSOR_MAP_DATA_TYPE_UINT8, hole, (uint64_t)K / 2, (uint64_t)N, (uint64_t)K / 2,
                    BK / 2, BN, CU_TENSOR_MAP_SWIZZLE_32B) ||
        !encode_map(&maps.p, CU_TENSOR_MAP_DATA_TYPE_UINT8, plug, (uint64_t)K / 2, (uint64_t)N, (uint64_t)K / 2,
                    BK / 2, BN, CU_TENSOR_MAP_SWIZZLE_32B) ||
        !encode_map(&maps.am, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, am, (uint64_t)K / 64, (uint64_t)N,
                    (uint64_t)K / 64 * 4, 4, BN, CU_TENSOR_MAP_SWIZZLE_NONE))
        return kLaunch;
    if (!ensure_smem((const void *)htile_gemm_kernel, kSmemBytes))
        return kLaunch;
    GemmArgs a{y, M, N, K, y_bf16 ? 1 : 0, (M + BMX - 1) / BMX, (N + BN - 1) / BN};
    const int tiles = a.mtiles * a.ntiles;
    const int grid = std::max(1, std::min(tiles, sm_count()));
    htile_gemm_kernel<<<grid, kThreads, kSmemBytes, st>>>(maps, a);
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
