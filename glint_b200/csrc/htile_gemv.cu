/* GLINT H-TILE for decode-shaped calls (small M) on sm_100a.
 *
 * Reference behaviour: cuda/glint_htile.cu:124-164 (glint_htile_s3_f32):
 *   y[m, n] = sum_k GLINT_CELLS[h][p] * absmax[(n*K + k) / bs] * bf16(x[m, k]),
 * x BF16 [M, K] row-major, W packed over the flattened [N, K] index, y f32
 * [M, N] row-major, overwritten.  The reference computes one output per thread
 * with scalar FMAs; here the dequantised weights feed the tensor cores.
 *
 * Decode is bound by reading the packed weights (1.0625 B per weight), so the
 * kernel is built around streaming them once:
 *   - swap-AB mma.sync.m16n8k16: 16 weight rows are the A operand, up to 8
 *     activation rows the B operand (MT such tiles for M <= 8*MT);
 *   - a lane streams 8 bytes of each plane (16 weights) of rows g and g+8 per
 *     64-wide k block; since a dot product does not depend on the order of k,
 *     the MMA's k positions are mapped onto the lane's own 16 weights and the
 *     activations are read with the same map (4 consecutive BF16 per step);
 *   - each 64-block's partial sums come out of a fresh accumulator and are scaled
 *     by that block's absmax in f32 (requires bs % 64 == 0 and K % 64 == 0);
 *   - the codebook sits in shared memory with one replica per lane (32 KB) as a
 *     BF16 pair hi = RN(cell), lo = RN(cell - hi); kPrecise issues one MMA for
 *     each half, so each weight carries ~17 significant bits and y agrees with an
 *     f32 dot product to ~1e-6 relative; kFast uses hi only;
 *   - the 8 warps of a CTA split K for the same 16 rows and reduce through shared
 *     memory; CTAs are persistent over 16-row tiles.
 * Other shapes (odd K, blocksize not a multiple of 64, unaligned pointers) run
 * the generic kernel: one warp per output row and 8 activation rows, f32 FMAs.
 */
#include <algorithm>

#include "common.cuh"
#include "glint_internal.h"

namespace glint {
namespace {

constexpr int kGemvWarps = 8;
constexpr int kGemvThreads = kGemvWarps * 32;

__device__ __forceinline__ void mma_bf16_16816(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
                 "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

/* BF16 hi/lo pair of a codebook value, hi in the low half. */
__device__ __forceinline__ uint32_t split_pair(float c)
{
    const uint32_t hi = f32_to_bf16_bits(c);
    const float rest = c - __uint_as_float(hi << 16);
    return hi | (f32_to_bf16_bits(rest) << 16);
}

/* shared-memory byte offset of code `idx` in this lane's replica */
__device__ __forceinline__ uint32_t lut_off(uint32_t idx, uint32_t lane4) { return (idx << 7) | lane4; }

struct Operands {
    uint2 h[2], p[2]; /* rows g and g+8: 16 nibbles each */
    float s[2];       /* absmax of the rows' current 64-block */
};

template <int MT, bool SPLIT, bool BF16OUT>
__global__ void __launch_bounds__(kGemvThreads) htile_gemv_kernel(const uint8_t *__restrict__ hole,
                                                                  const uint8_t *__restrict__ plug,
                                                                  const float *__restrict__ absmax,
                                                                  const __nv_bfloat16 *__restrict__ x, void *y, int M,
                                                                  int N, int K, int bs64, int chunks_per_warp)
{
    __shared__ uint32_t lut[256 * 32];
    __shared__ float red[kGemvWarps][16][8 * MT];
    for (int i = threadIdx.x; i < 256 * 32; i += kGemvThreads) {
        const int idx = i >> 5;
        lut[i] = split_pair(g_cells[idx >> 4][idx & 15]);
    }
    __syncthreads();

    const int warp = threadIdx.x >> 5;
    const uint32_t lane = lane_id();
    const int g = (int)(lane >> 2), t = (int)(lane & 3);
    const char *lut_base = reinterpret_cast<const char *>(lut);
    const uint32_t lane4 = lane * 4;
    const int K2 = K >> 1, K64 = K >> 6;
    const int c_begin = warp * chunks_per_warp;
    const int c_end = min(K64, c_begin + chunks_per_warp);
    const int tiles = (N + 15) >> 4;

    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
        const int n0 = tile * 16;
        const int rows[2] = {n0 + g, n0 + g + 8};
        const bool rv[2] = {rows[0] < N, rows[1] < N};
        float acc[MT][4];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
            acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;

        /* absmax index of each row's first block, advanced one 64-block at a time */
        uint32_t am_idx[2], am_rem[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const uint32_t u = (uint32_t)(rv[r] ? rows[r] : 0) * (uint32_t)K64 + (uint32_t)c_begin;
            am_idx[r] = u / (uint32_t)bs64;
            am_rem[r] = u % (uint32_t)bs64;
        }
        auto load_ops = [&](int c, Operands &o) {
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                if (rv[r]) {
                    const int64_t off = (int64_t)rows[r] * K2 + c * 32 + t * 8;
                    o.h[r] = __ldcs(reinterpret_cast<const uint2 *>(hole + off));
                    o.p[r] = __ldcs(reinterpret_cast<const uint2 *>(plug + off));
                    o.s[r] = __ldg(absmax + am_idx[r]);
                } else {
                    o.h[r] = o.p[r] = make_uint2(0, 0);
                    o.s[r] = 0.f;
                }
                if (++am_rem[r] == (uint32_t)bs64) {
                    am_rem[r] = 0;
                    ++am_idx[r];
                }
            }
        };
        auto load_x = [&](int c, uint4 xb[MT][2]) {
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                const int m = mt * 8 + g;
                if (m < M) {
                    const uint4 *src = reinterpret_cast<const uint4 *>(x + (int64_t)m * K + c * 64 + t * 16);
                    xb[mt][0] = __ldg(src);
                    xb[mt][1] = __ldg(src + 1);
                } else {
                    xb[mt][0] = xb[mt][1] = make_uint4(0, 0, 0, 0);
                }
            }
        };

        Operands cur;
        uint4 xc[MT][2];
        if (c_begin < c_end) {
            load_ops(c_begin, cur);
            load_x(c_begin, xc);
        }
        for (int c = c_begin; c < c_end; ++c) {
            Operands nxt;
            uint4 xn[MT][2];
            if (c + 1 < c_end) {
                load_ops(c + 1, nxt);
                load_x(c + 1, xn);
            }
            float part[MT][4];
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
                part[mt][0] = part[mt][1] = part[mt][2] = part[mt][3] = 0.f;
            /* byte b of E[r][w] = code of element 2b of word w, O: element 2b+1 */
            uint32_t E[2][2], O[2][2];
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const uint32_t hw[2] = {cur.h[r].x, cur.h[r].y}, pw[2] = {cur.p[r].x, cur.p[r].y};
#pragma unroll
                for (int wd = 0; wd < 2; ++wd) {
                    E[r][wd] = ((hw[wd] << 4) & 0xF0F0F0F0u) | (pw[wd] & 0x0F0F0F0Fu);
                    O[r][wd] = (hw[wd] & 0xF0F0F0F0u) | ((pw[wd] >> 4) & 0x0F0F0F0Fu);
                }
            }
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                /* step s uses the lane's weights 4s..4s+3: word s/2, bytes 2(s%2), 2(s%2)+1 */
                const int wd = s >> 1, b0 = (s & 1) * 2;
                uint32_t e[2][4];
#pragma unroll
                for (int r = 0; r < 2; ++r) {
                    const uint32_t i0 = (E[r][wd] >> (8 * b0)) & 0xFFu, i1 = (O[r][wd] >> (8 * b0)) & 0xFFu;
                    const uint32_t i2 = (E[r][wd] >> (8 * b0 + 8)) & 0xFFu, i3 = (O[r][wd] >> (8 * b0 + 8)) & 0xFFu;
                    e[r][0] = *reinterpret_cast<const uint32_t *>(lut_base + lut_off(i0, lane4));
                    e[r][1] = *reinterpret_cast<const uint32_t *>(lut_base + lut_off(i1, lane4));
                    e[r][2] = *reinterpret_cast<const uint32_t *>(lut_base + lut_off(i2, lane4));
                    e[r][3] = *reinterpret_cast<const uint32_t *>(lut_base + lut_off(i3, lane4));
                }
                uint32_t ahi[4] = {__byte_perm(e[0][0], e[0][1], 0x5410), __byte_perm(e[1][0], e[1][1], 0x5410),
                                   __byte_perm(e[0][2], e[0][3], 0x5410), __byte_perm(e[1][2], e[1][3], 0x5410)};
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    const uint32_t xw[4] = {xc[mt][wd].x, xc[mt][wd].y, xc[mt][wd].z, xc[mt][wd].w};
                    const uint32_t bb0 = xw[(s & 1) * 2], bb1 = xw[(s & 1) * 2 + 1];
                    mma_bf16_16816(part[mt], ahi, bb0, bb1);
                }
                if (SPLIT) {
                    uint32_t alo[4] = {__byte_perm(e[0][0], e[0][1], 0x7632), __byte_perm(e[1][0], e[1][1], 0x7632),
                                       __byte_perm(e[0][2], e[0][3], 0x7632), __byte_perm(e[1][2], e[1][3], 0x7632)};
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt) {
                        const uint32_t xw[4] = {xc[mt][wd].x, xc[mt][wd].y, xc[mt][wd].z, xc[mt][wd].w};
                        mma_bf16_16816(part[mt], alo, xw[(s & 1) * 2], xw[(s & 1) * 2 + 1]);
                    }
                }
            }
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                acc[mt][0] = fmaf(cur.s[0], part[mt][0], acc[mt][0]);
                acc[mt][1] = fmaf(cur.s[0], part[mt][1], acc[mt][1]);
                acc[mt][2] = fmaf(cur.s[1], part[mt][2], acc[mt][2]);
                acc[mt][3] = fmaf(cur.s[1], part[mt][3], acc[mt][3]);
            }
            if (c + 1 < c_end) {
                cur = nxt;
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    xc[mt][0] = xn[mt][0];
                    xc[mt][1] = xn[mt][1];
                }
            }
        }
        /* C fragment: c0 (row g, col 2t), c1 (g, 2t+1), c2 (g+8, 2t), c3 (g+8, 2t+1) */
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            red[warp][g][mt * 8 + 2 * t] = acc[mt][0];
            red[warp][g][mt * 8 + 2 * t + 1] = acc[mt][1];
            red[warp][g + 8][mt * 8 + 2 * t] = acc[mt][2];
            red[warp][g + 8][mt * 8 + 2 * t + 1] = acc[mt][3];
        }
        __syncthreads();
        for (int i = threadIdx.x; i < 16 * 8 * MT; i += kGemvThreads) {
            const int row = i / (8 * MT), col = i % (8 * MT);
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < kGemvWarps; ++w)
                v += red[w][row][col];
            const int n = n0 + row;
            if (col < M && n < N) {
                if (BF16OUT)
                    static_cast<__nv_bfloat16 *>(y)[(int64_t)col * N + n] = __float2bfloat16_rn(v);
                else
                    static_cast<float *>(y)[(int64_t)col * N + n] = v;
            }
        }
        __syncthreads();
    }
}

/* Generic path: warp per (n, group of 8 activation rows), lanes split k, f32 FMAs
 * in the reference's op order for the weight (cells[h][p] * absmax). */
template <bool BF16OUT>
__global__ void htile_generic_kernel(const uint8_t *hole, const uint8_t *plug, const float *absmax,
                                     const __nv_bfloat16 *x, void *y, int M, int N, int K, int bs)
{
    const int mgroups = (M + 7) / 8;
    const int64_t items = (int64_t)N * mgroups;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
    for (int64_t it = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); it < items; it += warps) {
        const int n = (int)(it / mgroups), m0 = (int)(it % mgroups) * 8;
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int k = lane_id(); k < K; k += 32) {
            const int64_t i = (int64_t)n * K + k;
            const int sh = (int)(i & 1) * 4;
            const float w = g_cells[(hole[i >> 1] >> sh) & 15][(plug[i >> 1] >> sh) & 15] * absmax[i / bs];
#pragma unroll
            for (int mm = 0; mm < 8; ++mm)
                if (m0 + mm < M)
                    acc[mm] = fmaf(w, __bfloat162float(x[(int64_t)(m0 + mm) * K + k]), acc[mm]);
        }
#pragma unroll
        for (int mm = 0; mm < 8; ++mm) {
            const float v = warp_sum(acc[mm]);
            if (lane_id() == 0 && m0 + mm < M) {
                if (BF16OUT)
                    static_cast<__nv_bfloat16 *>(y)[(int64_t)(m0 + mm) * N + n] = __float2bfloat16_rn(v);
                else
                    static_cast<float *>(y)[(int64_t)(m0 + mm) * N + n] = v;
            }
        }
    }
}

template <int MT, bool SPLIT, bool BF16OUT>
int launch_gemv_t(const uint8_t *hole, const uint8_t *plug, const float *am, const __nv_bfloat16 *x, void *y, int M,
                  int N, int K, int bs, cudaStream_t st)
{
    const int K64 = K / 64;
    const int cpw = (K64 + kGemvWarps - 1) / kGemvWarps;
    const int tiles = (N + 15) / 16;
    const int grid = std::max(1, std::min(tiles, sm_count() * 4));
    htile_gemv_kernel<MT, SPLIT, BF16OUT><<<grid, kGemvThreads, 0, st>>>(hole, plug, am, x, y, M, N, K, bs / 64, cpw);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunch;
}

template <bool SPLIT, bool BF16OUT>
int launch_gemv_slices(const uint8_t *hole, const uint8_t *plug, const float *am, const __nv_bfloat16 *x, void *y,
                       int M, int N, int K, int bs, cudaStream_t st)
{
    const size_t ysz = BF16OUT ? 2 : 4;
    for (int m0 = 0; m0 < M; m0 += 32) {
        const int mm = std::min(32, M - m0);
        const __nv_bfloat16 *xs = x + (int64_t)m0 * K;
        void *ys = static_cast<char *>(y) + (size_t)m0 * N * ysz;
        int rc;
        if (mm <= 8)
            rc = launch_gemv_t<1, SPLIT, BF16OUT>(hole, plug, am, xs, ys, mm, N, K, bs, st);
        else if (mm <= 16)
            rc = launch_gemv_t<2, SPLIT, BF16OUT>(hole, plug, am, xs, ys, mm, N, K, bs, st);
        else
            rc = launch_gemv_t<4, SPLIT, BF16OUT>(hole, plug, am, xs, ys, mm, N, K, bs, st);
        if (rc != kOk)
            return rc;
    }
    return kOk;
}

} // namespace

/* Decode-shaped H-TILE.  Exposed to htile_gemm.cu's dispatcher. */
int htile_gemv_launch(const uint8_t *hole, const uint8_t *plug, const float *am, const __nv_bfloat16 *x, void *y,
                      OutKind yk, int M, int N, int K, int bs, HtileMode mode, cudaStream_t st)
{
    const bool fast_shape = K % 64 == 0 && bs % 64 == 0 && aligned_to(hole, 8) && aligned_to(plug, 8) &&
                            aligned_to(x, 16) && aligned_to(am, 4) && (int64_t)N * (K / 64) < (int64_t)0xFFFFFFFF;
    if (htile_decode_supported(hole, plug, am, x, M, N, K, bs))
        return htile_decode_launch(hole, plug, am, x, y, yk, M, N, K, mode, st);
    if (M > 32 && htile_decode_supported(hole, plug, am, x, 32, N, K, bs)) {
        /* larger M on the TMA-streamed decode kernels, 32 activation rows per launch
         * (the precise path at prefill shapes; consecutive launches overlap through
         * programmatic dependent launch, and the planes of layers up to ~100 MB stay
         * in L2 between them) */
        const size_t ysz = yk == kOutBF16 ? 2 : 4;
        for (int m0 = 0; m0 < M; m0 += 32) {
            const int rc = htile_decode_launch(hole, plug, am, x + (int64_t)m0 * K,
                                               static_cast<char *>(y) + (size_t)m0 * N * ysz, yk,
                                               std::min(32, M - m0), N, K, mode, st);
            if (rc != kOk)
                return rc;
        }
        return kOk;
    }
    if (fast_shape) {
        if (mode == kPrecise)
            return yk == kOutBF16 ? launch_gemv_slices<true, true>(hole, plug, am, x, y, M, N, K, bs, st)
                                  : launch_gemv_slices<true, false>(hole, plug, am, x, y, M, N, K, bs, st);
        return yk == kOutBF16 ? launch_gemv_slices<false, true>(hole, plug, am, x, y, M, N, K, bs, st)
                              : launch_gemv_slices<false, false>(hole, plug, am, x, y, M, N, K, bs, st);
    }
    const int64_t items = (int64_t)N * ((M + 7) / 8);
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((items + 7) / 8, (int64_t)sm_count() * 16));
    if (yk == kOutBF16)
        htile_generic_kernel<true><<<grid, 256, 0, st>>>(hole, plug, am, x, y, M, N, K, bs);
    else
        htile_generic_kernel<false><<<grid, 256, 0, st>>>(hole, plug, am, x, y, M, N, K, bs);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunch;
}

} // namespace glint
