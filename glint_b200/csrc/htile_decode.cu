/* GLINT H-TILE for decode-shaped calls (small M), streamed at HBM speed.
 *
 * Reference behaviour: cuda/glint_htile.cu:124-164 (glint_htile_s3_f32):
 *   y[m, n] = sum_k GLINT_CELLS[h][p] * absmax[(n*K + k) / bs] * bf16(x[m, k]),
 * x BF16 [M, K] row-major, W packed over the flattened [N, K] index, y [M, N]
 * row-major, overwritten.
 *
 * Decode reads each packed weight once (1.0625 B), so the kernel is a stream:
 *   - work units of 256 weight rows x 128 k; a persistent CTA (one per SM) takes
 *     a contiguous range of units in row-block-major order (stream-K), so every
 *     SM gets the same number of units whatever N and K are;
 *   - a producer warp fetches each unit's hole and plug tiles (256 rows x 64 B,
 *     64B swizzle), its absmax tile (256 rows x 4 blocks, taken at an even unit
 *     so the TMA coordinate stays 16-byte aligned) and the activation slice
 *     (8*MT rows x 128 k, 128B swizzle, rows past M zero-filled) with 2-D TMA
 *     loads into a 3-slot shared-memory ring (~115 KB in flight per SM);
 *   - each of the 16 consumer warps owns 16 of the 256 rows and runs swap-AB
 *     mma.sync.m16n8k16: 16 weight rows are the A operand, up to 8 activation
 *     rows the B operand (MT such tiles).  A lane holds 16 weights of rows g and
 *     g+8 per 64-k block; the MMA's k positions are mapped onto those weights and
 *     the activations read with the same map (a dot product does not depend on
 *     the order of k);
 *   - each 64-block's sums come out of a fresh accumulator and are scaled by its
 *     absmax in f32; the codebook sits in shared memory as BF16 pairs
 *     hi = RN(cell), lo = RN(cell - hi), one replica per lane with a 256-byte
 *     entry stride, so a lookup address is one byte permute: precise mode
 *     issues an MMA for each half (~17 significant bits per weight, f32-class
 *     results), fast mode uses hi only;
 *   - a row block split between CTAs is finished by whichever part arrives
 *     last: each CTA's warp writes its 16 rows' partial sums to a workspace slot
 *     and bumps a counter for (row block, warp); the last one adds the slots in
 *     k order (so results do not depend on timing) and writes y.  The workspace
 *     is allocated once per (device, stream) and reused.
 * Requires bs == 64, K % 256 == 0, 16-byte aligned planes and absmax; other
 * shapes use htile_gemv.cu.  Every barrier wait is bounded (~1 s); a timeout
 * sets this file's error word and the kernel stops.
 */
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "gather.cuh"
#include "glint_internal.h"
#include "ptx.cuh"

namespace glint {

__device__ int g_decode_error = 0;
__device__ int g_decode_error_taken = 0; /* read_error_word's result slot */

namespace {

constexpr int kRows = 256;                 /* weight rows per unit */
/* k per unit: 256 (128-byte plane rows, 128B swizzle, two ring slots) while the
 * activation slice is small, else 128 (64-byte rows, 64B swizzle, three slots).
 * Wide rows matter: a TMA row request carries the row, and the bytes in flight
 * per SM grow with it. */
template <int MT>
constexpr int ku_of() { return MT <= 2 ? 256 : 128; }
template <int MT>
constexpr int plane_tile() { return kRows * ku_of<MT>() / 2; } /* 32 or 16 KB */
constexpr int kAmTile = kRows * 4 * 4; /* 256 rows x 4 blocks x f32: the unit's blocks (k 256) or its pair's (k 128) */
constexpr int kConsumers = 16;             /* 16 rows each */
constexpr int kThreads = (kConsumers + 1) * 32;
/* codebook hi|lo pairs, one replica per lane, entry stride 256 B: the lookup address
 * of code byte b of a word is one byte permute, (code << 8) | (lane << 2) */
constexpr int kLutBytes = 256 * 256;
/* x tile of a unit: 2 boxes of 64 k x 8*MT rows (128B swizzle), 1 KB per 8 rows */
template <int MT>
constexpr int x_tile() { return (ku_of<MT>() / 64) * 8 * MT * 128; }
template <int MT>
constexpr int slot_bytes() { return 2 * plane_tile<MT>() + kAmTile + x_tile<MT>(); }
template <int MT>
constexpr int n_slots() { return ku_of<MT>() == 256 ? 2 : 3; } /* as many as fit in 227 KB */
template <int MT>
constexpr int smem_bytes() { return kLutBytes + 1024 + n_slots<MT>() * slot_bytes<MT>() + 2 * 8 * n_slots<MT>() + 64; }

__device__ __forceinline__ void mma_bf16_16816(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
                 "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t split_pair(float c)
{
    const uint32_t hi = f32_to_bf16_bits(c);
    const float rest = c - __uint_as_float(hi << 16);
    return hi | (f32_to_bf16_bits(rest) << 16);
}

/* The per-lane codebook replicas, written by the consumer threads: each 16-byte
 * store covers a quarter of one entry's 128-byte row of 32 replicas, so a warp's
 * store fills four whole rows (four wavefronts, no bank conflicts; one thread per
 * entry writing its own row would put all 32 lanes on the same four banks). */
__device__ __forceinline__ void build_pair_lut(uint32_t *lut)
{
    for (int i = (int)threadIdx.x; i < 256 * 8; i += kConsumers * 32) {
        const int e = i >> 3;
        const uint32_t v = split_pair(g_cells[e >> 4][e & 15]);
        reinterpret_cast<uint4 *>(lut + e * 64)[i & 7] = make_uint4(v, v, v, v);
    }
}

struct DecodeArgs {
    const __nv_bfloat16 *x;
    void *y;
    float *ws;          /* partial sums: [row block][part][128][8*MT] */
    int *flags;         /* per row block, part and consumer warp: part published; zero between calls */
    int M, N, K;
    int KU;             /* units per row block (K / 256) */
    int64_t units;      /* row blocks * KU */
    int max_parts;
    GatherArgs ga;
};

/* first unit of CTA c under the even split of `units` over `ctas` */
__device__ __forceinline__ int64_t unit_start(int64_t c, int64_t units, int64_t ctas) { return c * units / ctas; }
/* CTA whose range holds unit u */
__device__ __forceinline__ int64_t cta_of(int64_t u, int64_t units, int64_t ctas)
{
    int64_t c = (u * ctas) / units;
    while (c + 1 < ctas && unit_start(c + 1, units, ctas) <= u)
        ++c;
    while (c > 0 && unit_start(c, units, ctas) > u)
        --c;
    return c;
}

/* Physical row (within its group of 8) behind mma fragment row g.  A half-warp
 * holds fragment rows 0-3 (or 4-7); the map spreads them over rows whose swizzled
 * 16-byte chunks of a 64-k block are all different, so its 8-byte plane loads
 * cover the 32 banks once (the identity map reads 4 chunks twice: 2-way
 * conflicts).  128-byte rows: rows 0,2,4,6 | 1,3,5,7 (chunk ^ (row & 7)); 64-byte
 * rows: rows 0,1,4,5 | 2,3,6,7 (chunk ^ ((row >> 1) & 3), row parity picks the
 * bank half). */
template <int ROWB>
__device__ __forceinline__ int frag_row(int g)
{
    return ROWB == 128 ? (((g & 3) << 1) | (g >> 2)) : ((g & 1) | (((g >> 1) & 1) << 2) | ((g >> 2) << 1));
}

/* Arithmetic of one 64-k block (see tile_block): codes -> codebook -> MMAs -> the
 * block's sums scaled by its absmax and added to acc. */
template <int MT, bool SPLIT>
__device__ __forceinline__ void tile_math(const uint32_t (&E)[2][2], const uint32_t (&O)[2][2], const float (&sc)[2],
                                          const uint4 (&xb)[MT][2], uint32_t lut_base, uint32_t lane4,
                                          float (&acc)[MT][4])
{
    /* two accumulators (even and odd MMA steps) keep the chains independent */
    float part[2][MT][4];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
            part[h][mt][0] = part[h][mt][1] = part[h][mt][2] = part[h][mt][3] = 0.f;
#pragma unroll
    for (int st = 0; st < 4; ++st) {
        const int wd = st >> 1, b0 = (st & 1) * 2;
        uint32_t e[2][4];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            /* address = (code << 8) | (lane << 2): byte b0 or b0+1 of E / O into byte 1 */
            e[r][0] = lds32(lut_base + __byte_perm(E[r][wd], lane4, 0x5504 | (b0 << 4)));
            e[r][1] = lds32(lut_base + __byte_perm(O[r][wd], lane4, 0x5504 | (b0 << 4)));
            e[r][2] = lds32(lut_base + __byte_perm(E[r][wd], lane4, 0x5504 | ((b0 + 1) << 4)));
            e[r][3] = lds32(lut_base + __byte_perm(O[r][wd], lane4, 0x5504 | ((b0 + 1) << 4)));
        }
        const uint32_t ahi[4] = {__byte_perm(e[0][0], e[0][1], 0x5410), __byte_perm(e[1][0], e[1][1], 0x5410),
                                 __byte_perm(e[0][2], e[0][3], 0x5410), __byte_perm(e[1][2], e[1][3], 0x5410)};
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            const uint32_t xw[4] = {xb[mt][wd].x, xb[mt][wd].y, xb[mt][wd].z, xb[mt][wd].w};
            mma_bf16_16816(part[st & 1][mt], ahi, xw[(st & 1) * 2], xw[(st & 1) * 2 + 1]);
        }
        if (SPLIT) {
            const uint32_t alo[4] = {__byte_perm(e[0][0], e[0][1], 0x7632), __byte_perm(e[1][0], e[1][1], 0x7632),
                                     __byte_perm(e[0][2], e[0][3], 0x7632), __byte_perm(e[1][2], e[1][3], 0x7632)};
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                const uint32_t xw[4] = {xb[mt][wd].x, xb[mt][wd].y, xb[mt][wd].z, xb[mt][wd].w};
                mma_bf16_16816(part[st & 1][mt], alo, xw[(st & 1) * 2], xw[(st & 1) * 2 + 1]);
            }
        }
    }
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
        for (int q = 0; q < 4; ++q)
            acc[mt][q] = fmaf(sc[q >> 1], part[0][mt][q] + part[1][mt][q], acc[mt][q]);
    }
}

/* One 64-k absmax block of a 16-row weight tile against the activations:
 * acc[mt] += absmax * (W[rows r0+g, r0+g+8][block] . x[mt*8+g'][block]).
 * `hole`/`plug`: plane tiles with ROWB-byte rows (128: 128B swizzle, 16-byte chunk j
 * of row r at j ^ (r & 7); 64: 64B swizzle, j ^ ((r >> 1) & 3)), 1 KB aligned; the
 * tile's rows start at row `ro` of them (the swizzle phase follows the row's place
 * in the tile, ro + r); the block at byte 32*c of a row; `am`: absmax rows of 16
 * bytes (row ro + r), this block in column am_col; `xbox`: the block's activation
 * rows of 128 B (128B swizzle) whose first row has swizzle phase `xph`.  Swap-AB
 * mma.sync.m16n8k16: weights are the A operand (lane (g, t) holds rows
 * frag_row(g) and frag_row(g)+8),
 * activations the B operand read with the same k map, so the dot product is exact
 * whatever the k order; hi (and lo in precise mode) BF16 halves of the codebook.
 * Lanes whose activation row mt*8+g is >= M (rows the TMA box fills with zeros)
 * take zeros without reading shared memory. */
template <int MT, bool SPLIT, int ROWB>
__device__ __forceinline__ void tile_block(uint32_t hole, uint32_t plug, uint32_t am, uint32_t am_col, uint32_t xbox,
                                           uint32_t xph, int c, int r0, int ro, int g, int t, uint32_t lut_base,
                                           uint32_t lane4, int M, float (&acc)[MT][4])
{
    uint32_t E[2][2], O[2][2];
    float sc[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int row = ro + r0 + frag_row<ROWB>(g) + 8 * r;
        const uint32_t chunk = (uint32_t)(2 * c + (t >> 1)) ^ (uint32_t)(ROWB == 128 ? (row & 7) : ((row >> 1) & 3));
        const uint32_t off = (uint32_t)row * (uint32_t)ROWB + (chunk << 4) + (uint32_t)(t & 1) * 8u;
        const uint2 hw = lds64(hole + off), pw = lds64(plug + off);
        const uint32_t hv[2] = {hw.x, hw.y}, pv[2] = {pw.x, pw.y};
#pragma unroll
        for (int wd = 0; wd < 2; ++wd) {
            E[r][wd] = ((hv[wd] << 4) & 0xF0F0F0F0u) | (pv[wd] & 0x0F0F0F0Fu);
            O[r][wd] = (hv[wd] & 0xF0F0F0F0u) | ((pv[wd] >> 4) & 0x0F0F0F0Fu);
        }
        sc[r] = __uint_as_float(lds32(am + (uint32_t)row * 16u + am_col * 4u));
    }
    /* x fragments: row m = mt*8 + g of the block's rows, 16 consecutive k at 32*t
     * bytes (16-byte chunks 2t and 2t+1, 128B swizzle: chunk ^ ((xph + m) & 7)) */
    uint4 xb[MT][2];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
        const int m = mt * 8 + g;
        const uint32_t rowb = xbox + (uint32_t)m * 128u;
        const uint32_t ph = (xph + (uint32_t)m) & 7u;
        const bool live = m < M;
        xb[mt][0] = lds128_if(rowb + (((uint32_t)(2 * t) ^ ph) << 4), live);
        xb[mt][1] = lds128_if(rowb + (((uint32_t)(2 * t + 1) ^ ph) << 4), live);
    }
    tile_math<MT, SPLIT>(E, O, sc, xb, lut_base, lane4, acc);
}

/* Shared-memory byte offsets, within a ring stage, of one lane's operands of one 64-k
 * block: its two plane rows, their absmax and its activation chunks.  They depend
 * only on the warp, the lane and the block's place in the unit, so the row-owned
 * kernel computes them once, outside its K loop (in the loop their arithmetic cost
 * about half an instruction per weight at M = 1). */
template <int MT>
struct BlockOffs {
    uint32_t pl[2];          /* plane bytes of rows frag_row(g) and frag_row(g) + 8 */
    uint32_t am[2];          /* their absmax */
    uint32_t x0[MT], x1[MT]; /* the lane's two 16-byte activation chunks per row group */
    uint32_t live;           /* bit mt: activation row mt * 8 + g < M */
};

/* Offsets for 64-k block c of rows starting at row ro of 128-byte plane rows (128B
 * swizzle), absmax rows of 16 bytes at am_off (column am_col) and activation rows of
 * 128 bytes at x_off whose first row has swizzle phase xph (as tile_block reads them). */
template <int MT>
__device__ __forceinline__ BlockOffs<MT> block_offs(int c, int r0, int ro, int g, int t, uint32_t am_off,
                                                    uint32_t am_col, uint32_t x_off, uint32_t xph, int M)
{
    BlockOffs<MT> o;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int row = ro + r0 + frag_row<128>(g) + 8 * r;
        const uint32_t chunk = (uint32_t)(2 * c + (t >> 1)) ^ (uint32_t)(row & 7);
        o.pl[r] = (uint32_t)row * 128u + (chunk << 4) + (uint32_t)(t & 1) * 8u;
        o.am[r] = am_off + (uint32_t)row * 16u + am_col * 4u;
    }
    o.live = 0u;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
        const int m = mt * 8 + g;
        const uint32_t ph = (xph + (uint32_t)m) & 7u;
        o.x0[mt] = x_off + (uint32_t)m * 128u + (((uint32_t)(2 * t) ^ ph) << 4);
        o.x1[mt] = x_off + (uint32_t)m * 128u + (((uint32_t)(2 * t + 1) ^ ph) << 4);
        o.live |= (m < M ? 1u : 0u) << mt;
    }
    return o;
}

/* tile_block with the operands at precomputed offsets from the stage base `st`
 * (plug tile at st + pt). */
template <int MT, bool SPLIT>
__device__ __forceinline__ void tile_block_at(uint32_t st, uint32_t pt, const BlockOffs<MT> &o, uint32_t lut_base,
                                              uint32_t lane4, float (&acc)[MT][4])
{
    uint32_t E[2][2], O[2][2];
    float sc[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const uint2 hw = lds64(st + o.pl[r]), pw = lds64(st + pt + o.pl[r]);
        const uint32_t hv[2] = {hw.x, hw.y}, pv[2] = {pw.x, pw.y};
#pragma unroll
        for (int wd = 0; wd < 2; ++wd) {
            E[r][wd] = ((hv[wd] << 4) & 0xF0F0F0F0u) | (pv[wd] & 0x0F0F0F0Fu);
            O[r][wd] = (hv[wd] & 0xF0F0F0F0u) | ((pv[wd] >> 4) & 0x0F0F0F0Fu);
        }
        sc[r] = __uint_as_float(lds32(st + o.am[r]));
    }
    uint4 xb[MT][2];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
        const bool live = (o.live >> mt) & 1u;
        xb[mt][0] = lds128_if(st + o.x0[mt], live);
        xb[mt][1] = lds128_if(st + o.x1[mt], live);
    }
    tile_math<MT, SPLIT>(E, O, sc, xb, lut_base, lane4, acc);
}

template <int MT, bool SPLIT, bool BF16OUT>
__global__ void __launch_bounds__(kThreads, 1)
    htile_decode_kernel(const __grid_constant__ CUtensorMap hmap, const __grid_constant__ CUtensorMap pmap,
                        const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap xmap,
                        const DecodeArgs a)
{
    constexpr int kSlots = n_slots<MT>();
    constexpr int kSlotBytes = slot_bytes<MT>();
    constexpr int kKU = ku_of<MT>(), kPlaneTile = plane_tile<MT>();
    static_assert(smem_bytes<MT>() <= 232448, "shared memory");
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint32_t *lut = reinterpret_cast<uint32_t *>(smem_raw);
    uint8_t *ring = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw + kLutBytes) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(ring + kSlots * kSlotBytes);
    uint64_t *empty = full + kSlots;
    uint32_t *cta_done = reinterpret_cast<uint32_t *>(empty + kSlots); /* gathered calls: warps done */

    /* barriers first, so the producer can start streaming while the consumers
     * build the codebook */
    if (threadIdx.x == 0) {
        for (int s = 0; s < kSlots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumers);
        }
        *cta_done = 0u;
        mbar_init_fence();
    }
    if (threadIdx.x == kConsumers * 32) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(&hmap) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&pmap) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&amap) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&xmap) : "memory");
    }
    __syncthreads();

    const int warp = threadIdx.x >> 5;
    const uint32_t lane = lane_id();
    const int64_t ctas = gridDim.x;
    const int64_t u0 = unit_start(blockIdx.x, a.units, ctas), u1 = unit_start(blockIdx.x + 1, a.units, ctas);

    if (warp == kConsumers) {
        if (lane == 0) {
            auto load_x = [&](int64_t u, int s) {
                const int ku = (int)(u % a.KU);
                uint8_t *slot = ring + s * kSlotBytes;
#pragma unroll
                for (int c = 0; c < kKU / 64; ++c)
                    tma_load_2d(slot + 2 * kPlaneTile + kAmTile + c * (8 * MT * 128), &xmap, &full[s],
                                ku * kKU + c * 64, 0);
            };
            int64_t i = 0;
            bool ok = true;
            for (int64_t u = u0; u < u1; ++u, ++i) {
                const int s = (int)(i % kSlots);
                const uint32_t ph = (uint32_t)(i / kSlots) & 1u;
                if (i >= kSlots && !(ok = mbar_wait_suspend_bounded(&empty[s], ph ^ 1u, &g_decode_error)))
                    break;
                const int rb = (int)(u / a.KU), ku = (int)(u % a.KU);
                uint8_t *slot = ring + s * kSlotBytes;
                mbar_expect_tx(&full[s], kSlotBytes);
                tma_load_2d(slot, &hmap, &full[s], ku * (kKU / 2), rb * kRows);
                tma_load_2d(slot + kPlaneTile, &pmap, &full[s], ku * (kKU / 2), rb * kRows);
                /* absmax box of 4 blocks: the unit's own (k 256) or, for k 128, taken at an
                 * even unit so the x coordinate stays 16-byte aligned */
                tma_load_2d(slot + 2 * kPlaneTile, &amap, &full[s], kKU == 256 ? ku * 4 : (ku >> 1) * 4, rb * kRows);
                if (i >= kSlots) {
                    load_x(u, s);
                } else if (i == kSlots - 1 || u == u1 - 1) {
                    /* The weights do not depend on earlier kernels, the activations may:
                     * under programmatic dependent launch the first slots' weights are
                     * already streaming while the previous kernel finishes (a no-op
                     * otherwise). */
                    asm volatile("griddepcontrol.wait;" ::: "memory");
                    for (int64_t j = 0; j <= i; ++j)
                        load_x(u0 + j, (int)j);
                }
            }
            /* all loads issued: the next kernel in the stream may start launching */
            asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
            if (!ok) {
                const int64_t issued = i;
                for (int64_t j = issued > kSlots ? issued - kSlots : 0; j < issued; ++j)
                    if (!mbar_wait_bounded(&full[(int)(j % kSlots)], (uint32_t)(j / kSlots) & 1u, &g_decode_error))
                        break;
            }
        }
        return;
    }

    /* codebook as BF16 hi/lo pairs, one replica per lane (first 128 B of each 256-B
     * entry row); the consumer warps then meet on named barrier 1 (the producer is
     * not in it) */
    build_pair_lut(lut);
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumers * 32) : "memory");
    /* y, the workspace and its flags are touched only after the previous kernel
     * in the stream is complete (no-op without programmatic dependent launch) */
    asm volatile("griddepcontrol.wait;" ::: "memory");

    /* consumer warp: rows r0 + pg and r0 + pg + 8 of each unit's 128 */
    const int g = (int)(lane >> 2), t = (int)(lane & 3);
    const int r0 = warp * 16, pg = frag_row<kKU / 2>(g);
    const uint32_t lut_base = saddr(lut);
    const uint32_t lane4 = lane * 4u;
    float acc[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
        acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;
    int cur_rb = -1, seg_k0 = 0;

    /* Publish this warp's sums for its 16 rows of row block rb (k units [k0, k1) of
     * the block).  A whole block goes straight to y.  A block split between CTAs
     * has a fixed owner, part 0: the CTA holding the block's first k unit, which
     * reaches it at the end of its range.  Every other part is the first segment of
     * its CTA's range (or the whole range): it stores its sums in the workspace and
     * sets its flag with a release add that nothing waits for.  The owner waits for
     * the flags (bounded; parts never wait on anything, so they complete as soon as
     * their CTAs run), adds the parts to its own sums in k order (results do not
     * depend on timing), resets the flags for the next call and writes y. */
    auto flush = [&](int rb, int k0, int k1) {
        constexpr int MP = 8 * MT;
        auto put_y = [&](int n, int col, float v) {
            if (n < a.N && col < a.M) {
                if (a.ga.world > 0)
                    gather_store<BF16OUT>(a.ga, col, n, v);
                else if (BF16OUT)
                    static_cast<__nv_bfloat16 *>(a.y)[(int64_t)col * a.N + n] = __float2bfloat16_rn(v);
                else
                    static_cast<float *>(a.y)[(int64_t)col * a.N + n] = v;
            }
        };
        if (k0 == 0 && k1 == a.KU) {
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    put_y(rb * kRows + r0 + pg + (q >> 1) * 8, mt * 8 + 2 * t + (q & 1), acc[mt][q]);
            return;
        }
        const int64_t first = cta_of((int64_t)rb * a.KU, a.units, ctas);
        const int part = (int)(blockIdx.x - first);
        const int parts = (int)(cta_of((int64_t)rb * a.KU + a.KU - 1, a.units, ctas) - first + 1);
        const float *wsp = a.ws + ((int64_t)rb * a.max_parts) * kRows * MP;
        int *flg = a.flags + ((int64_t)rb * a.max_parts) * kConsumers + warp;
        if (part != 0) {
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    __stcg(const_cast<float *>(wsp) + ((int64_t)part * kRows + r0 + pg + (q >> 1) * 8) * MP + mt * 8 +
                               2 * t + (q & 1),
                           acc[mt][q]);
            __syncwarp();
            if (lane == 0)
                asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(flg + part * kConsumers) : "memory");
            return;
        }
        /* lane l waits for the flag of part l (and l + 32, ...): the waits overlap */
        bool ok = true;
        for (int pp = (int)lane; pp < parts && ok; pp += 32) {
            if (pp == 0)
                continue;
            int *f = flg + pp * kConsumers;
            const long long t0 = clock64();
            uint32_t v = 0;
            while (true) {
                asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
                if (v)
                    break;
                if (clock64() - t0 > kWaitCycles) {
                    atomicOr(&g_decode_error, kErrTimeout);
                    ok = false;
                    break;
                }
                __nanosleep(64);
            }
            *f = 0; /* consumed: zero for the next call */
        }
        if (!__all_sync(0xFFFFFFFFu, ok))
            return;
        /* the parts' sums in part (k) order; loads issued eight at a time so their
         * L2 latencies overlap */
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int row = r0 + pg + (q >> 1) * 8, col = mt * 8 + 2 * t + (q & 1);
                const float *src = wsp + (int64_t)row * MP + col;
                const int64_t step = (int64_t)kRows * MP;
                float v = acc[mt][q];
                int pp = 1;
                for (; pp + 8 <= parts; pp += 8) {
                    float w8[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        w8[j] = __ldcg(src + (pp + j) * step);
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        v += w8[j];
                }
                for (; pp < parts; ++pp)
                    v += __ldcg(src + pp * step);
                put_y(rb * kRows + row, col, v);
            }
        }
    };

    int64_t i = 0;
    for (int64_t u = u0; u < u1; ++u, ++i) {
        const int rb = (int)(u / a.KU), ku = (int)(u % a.KU);
        if (rb != cur_rb) {
            if (cur_rb >= 0)
                flush(cur_rb, seg_k0, a.KU);
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
                acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;
            cur_rb = rb;
            seg_k0 = ku;
        }
        const int s = (int)(i % kSlots);
        const uint32_t ph = (uint32_t)(i / kSlots) & 1u;
        const bool ok = lane == 0 ? mbar_wait_suspend_bounded(&full[s], ph, &g_decode_error) : true;
        if (!__shfl_sync(0xFFFFFFFFu, ok ? 1 : 0, 0)) {
            cur_rb = -1; /* give up: no partial results are published */
            break;
        }
        const uint32_t slot = saddr(ring + s * kSlotBytes);
        const uint32_t xs = slot + 2 * kPlaneTile + kAmTile;
        const uint32_t am_col = kKU == 256 ? 0u : (uint32_t)(ku & 1) * 2;
#pragma unroll
        for (int c = 0; c < kKU / 64; ++c)
            tile_block<MT, SPLIT, kKU / 2>(slot, slot + kPlaneTile, slot + 2 * kPlaneTile, am_col + c,
                                           xs + (uint32_t)c * (8 * MT * 128), 0u, c, r0, 0, g, t, lut_base, lane4, a.M,
                                           acc);
        __syncwarp();
        if (lane == 0)
            mbar_arrive(&empty[s]);
    }
    if (cur_rb >= 0)
        flush(cur_rb, seg_k0, (int)(u1 - 1 - (int64_t)cur_rb * a.KU) + 1);
    if (a.ga.world > 0)
        gather_complete(a.ga, kConsumers, lane, cta_done, &g_decode_error);
}

/* ---- row-owned decode for wide layers ------------------------------------------
 * When every SM can own at least 16 rows (N >= 16 x SMs), CTA c takes the rows
 * [c*R, (c+1)*R), R = ceil(N / ctas), over the whole K, so no row is split between
 * CTAs: no workspace, no cross-CTA sums, and the per-SM work differs by at most
 * one row.  Its rows go in row blocks of RB <= 112 (7 tiles of 16).  A unit is
 * (row block, UB x 256 k), loaded into one ring stage by four 3-D TMA requests:
 * hole and plug [UB slices][RB rows][128 B] (128B swizzle), absmax
 * [UB][RB][4 blocks] and the activations [4 UB blocks][M rows][64 k] (128B
 * swizzle; only the M rows that exist).  Narrow row blocks take up to four 256-k
 * slices per unit: a TMA request then carries ~14 KB instead of one slice's 3.5 KB
 * (with 28-row blocks, one slice per request streamed 62 MB in ~20 us, four in
 * ~11 us), and the bytes in flight per SM stay near the same whatever RB is.
 * Consumer warp w works on tile w / KH
 * and NB = 4*UB/KH of every unit's 64-k blocks (unrolled, so the blocks' shared
 * loads and MMAs interleave); at the end of a row block the KH partial sums of a
 * tile are added in k order through shared memory (bounded mbarrier handshakes)
 * and written to y. */
constexpr int kRowBlockMax = 112;
constexpr int kRMaxStages = 8;
template <int MT>
constexpr int r_xsub() { return 4 * 8 * MT * 128; } /* activation rows of 256 k: 4 blocks x up to 8 MT rows */
/* ring capacity: 4 (MT 1) or 3 stages of the widest row block and one 256-k slice */
template <int MT>
constexpr int r_ring() { return (MT == 1 ? 4 : 3) * (2 * kRowBlockMax * 128 + 2048 + r_xsub<MT>()); }
/* partial sums exchanged at a row block's end: T * (KH - 1) <= 14 warps x 32 lanes */
template <int MT>
constexpr int r_scratch_floats() { return (MT <= 2 ? 14 : 7) * 32 * 4 * MT; }
/* one unit of a shared tail tile (MT <= 2): hole and plug 16 x 128 B, absmax
 * 16 x 16 B in 1 KB, the unit's activations [4 blocks][M rows][64 k], and the
 * partial sums of 3 of the 4 warps that share it (32 lanes x 4 MT floats each) */
constexpr int kTailWarps = 4;
constexpr int kTailX = 5 * 1024; /* offset of the activation boxes */
template <int MT>
constexpr int r_tail_bytes() { return MT <= 2 ? kTailX + r_xsub<MT>() + 3 * 32 * 4 * MT * 4 : 0; }
template <int MT>
constexpr int r_smem_bytes()
{
    return kLutBytes + 1024 + r_ring<MT>() + r_tail_bytes<MT>() + r_scratch_floats<MT>() * 4 +
           8 * (2 * kRMaxStages + 3) + 64;
}

struct RowArgs {
    void *y;
    int M, N, K;
    int KU; /* units per row (K / (256 UB)) */
    int UB; /* 256-k slices per unit */
    int R;  /* rows per CTA */
    int nb; /* row blocks per CTA */
    int RB; /* rows per row block (the TMA box height) */
    int T;  /* 16-row tiles per row block */
    int KH; /* consumer warps per tile */
    int S;  /* ring stages */
    int pt; /* bytes of a unit's plane tile (UB x RB x 128, 1 KB aligned) */
    int at; /* bytes of its absmax tile (UB x RB x 16, 1 KB aligned) */
    int xt; /* bytes of its activation tile (4 UB x xrows x 128, 1 KB aligned) */
    int stage; /* bytes of a ring stage: 2 pt + at + xt */
    int xrows; /* activation rows loaded: min(M, 8 MT) */
    uint32_t tx; /* TMA bytes per stage */
    GatherArgs ga;
    /* Shared tail: when the 16-row tiles do not divide evenly over the SMs, every
     * CTA owns R = 16 * floor(tiles / SMs) rows and the leftover tiles, from row
     * tail_row0, are cut into 16-row x 256-k units: CTA c < tail_units takes unit
     * c % KU of tile c / KU on kTailWarps otherwise idle warps, stores its partial
     * sum in tail_ws[c], and the last of a tile's KU CTAs (tail_cnt) adds the KU
     * partials in unit order and writes y.  0 tail units: off. */
    int tail_units;
    int tail_row0;
    uint32_t tail_tx;
    float *tail_ws;
    int *tail_cnt;
};

template <int MT, bool SPLIT, bool BF16OUT, int NB>
__global__ void __launch_bounds__(kThreads, 1)
    htile_rows_kernel(const __grid_constant__ CUtensorMap hmap, const __grid_constant__ CUtensorMap pmap,
                      const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap xmap,
                      const __grid_constant__ CUtensorMap hmap16, const __grid_constant__ CUtensorMap pmap16,
                      const __grid_constant__ CUtensorMap amap16, const RowArgs a)
{
    static_assert(r_smem_bytes<MT>() <= 232448, "shared memory");
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint32_t *lut = reinterpret_cast<uint32_t *>(smem_raw);
    uint8_t *ring = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw + kLutBytes) + 1023) & ~uintptr_t(1023));
    uint8_t *tail = ring + r_ring<MT>(); /* 1 KB aligned: the ring is a multiple of 1 KB */
    float *scratch = reinterpret_cast<float *>(tail + r_tail_bytes<MT>());
    uint64_t *full = reinterpret_cast<uint64_t *>(scratch + r_scratch_floats<MT>());
    uint64_t *empty = full + kRMaxStages;
    uint64_t *cmb_full = empty + kRMaxStages; /* a row block's KH-1 partials per tile are in scratch */
    uint64_t *cmb_empty = cmb_full + 1;       /* the tile owners have read them */
    uint64_t *tail_full = cmb_empty + 1;      /* the tail unit's planes, absmax and activations landed */
    uint32_t *cta_done = reinterpret_cast<uint32_t *>(tail_full + 1); /* gathered calls: warps done */
    const int S = a.S, KH = a.KH;
    const int stage_bytes = a.stage;

    const int active = a.T * KH;
    const bool has_tail = MT <= 2 && (int)blockIdx.x < a.tail_units;
    const int tail_tile = (int)blockIdx.x / a.KU, tail_ku = (int)blockIdx.x % a.KU;
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], active);
        }
        mbar_init(cmb_full, KH > 1 ? a.T * (KH - 1) : 1);
        mbar_init(cmb_empty, a.T);
        mbar_init(tail_full, 1);
        *cta_done = 0u;
        mbar_init_fence();
    }
    if (threadIdx.x == kConsumers * 32) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(&hmap) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&pmap) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&amap) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&xmap) : "memory");
    }
    __syncthreads();

    const int warp = threadIdx.x >> 5;
    const uint32_t lane = lane_id();
    const int n_begin = blockIdx.x * a.R, n_end = min(a.N, n_begin + a.R);
    const int units = a.nb * a.KU;

    if (warp == kConsumers) {
        if (lane == 0) {
            /* the unit's activations: blocks [4 UB ku, 4 UB (ku + 1)) of every row */
            auto load_x = [&](int ku, int s) {
                tma_load_3d(ring + s * stage_bytes + 2 * a.pt + a.at, &xmap, &full[s], 0, 0, ku * a.UB * 4);
            };
            /* the tail unit first, so its warps work beside the row blocks (one
             * 256-k slice: the ring's units have UB == 1 whenever a tail is set) */
            if (has_tail) {
                const int n16 = a.tail_row0 + tail_tile * 16;
                mbar_expect_tx(tail_full, a.tail_tx);
                tma_load_2d(tail, &hmap16, tail_full, tail_ku * 128, n16);
                tma_load_2d(tail + 2048, &pmap16, tail_full, tail_ku * 128, n16);
                tma_load_2d(tail + 4096, &amap16, tail_full, tail_ku * 4, n16);
            }
            bool ok = true;
            int i = 0, s = 0, blk = 0, ku = 0;
            uint32_t ph = 0;
            for (; i < units; ++i) {
                if (i >= S && !(ok = mbar_wait_suspend_bounded(&empty[s], ph ^ 1u, &g_decode_error)))
                    break;
                const int nb0 = n_begin + blk * a.RB;
                uint8_t *st = ring + s * stage_bytes;
                mbar_expect_tx(&full[s], a.tx);
                /* slices [UB ku, UB (ku + 1)) of rows [nb0, nb0 + RB): one request per tensor */
                tma_load_3d(st, &hmap, &full[s], 0, nb0, ku * a.UB);
                tma_load_3d(st + a.pt, &pmap, &full[s], 0, nb0, ku * a.UB);
                tma_load_3d(st + 2 * a.pt, &amap, &full[s], 0, nb0, ku * a.UB);
                if (i >= S) {
                    load_x(ku, s);
                } else if (i == S - 1 || i == units - 1) {
                    /* weights stream before the previous kernel is done, activations after
                     * (programmatic dependent launch; a no-op otherwise) */
                    asm volatile("griddepcontrol.wait;" ::: "memory");
                    if (has_tail) /* UB == 1 whenever a tail is set: the map's box is one 256-k slice */
                        tma_load_3d(tail + kTailX, &xmap, tail_full, 0, 0, tail_ku * 4);
                    for (int j = 0; j <= i; ++j)
                        load_x(j % a.KU, j);
                }
                if (++ku == a.KU)
                    ku = 0, ++blk;
                if (++s == S)
                    s = 0, ph ^= 1u;
            }
            asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
            if (!ok) {
                for (int j = i > S ? i - S : 0; j < i; ++j)
                    if (!mbar_wait_bounded(&full[j % S], (uint32_t)(j / S) & 1u, &g_decode_error))
                        break;
                if (has_tail)
                    mbar_wait_bounded(tail_full, 0u, &g_decode_error);
            }
        }
        return;
    }

    build_pair_lut(lut);
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumers * 32) : "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int g = (int)(lane >> 2), t = (int)(lane & 3), pg = frag_row<128>(g);
    const uint32_t lut_base = saddr(lut), lane4 = lane * 4u;
    if (warp >= active) {
        /* tail warp j: 64-k block j of the tail unit; warp 0 of them adds the four
         * in block order, publishes the unit's partial and, as the tile's last
         * unit, adds the tile's KU partials in unit order.  No waits on other CTAs:
         * a failed TMA wait still publishes (zeros), so the count stays whole. */
        if constexpr (MT <= 2) { /* the tail's shared buffer exists for MT <= 2 only */
            const int j = warp - active;
            if (!has_tail || j >= kTailWarps)
                return;
            float acc[MT][4];
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
                acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;
            const bool ok = lane == 0 ? mbar_wait_suspend_bounded(tail_full, 0u, &g_decode_error) : true;
            const uint32_t ts = saddr(tail);
            if (__shfl_sync(0xFFFFFFFFu, ok ? 1 : 0, 0))
                tile_block<MT, SPLIT, 128>(ts, ts + 2048, ts + 4096, (uint32_t)j,
                                           ts + (uint32_t)(kTailX + j * a.xrows * 128), (uint32_t)(j * a.xrows) & 7u, j,
                                           0, 0, g, t, lut_base, lane4, a.M, acc);
            float4 *part = reinterpret_cast<float4 *>(tail + kTailX + r_xsub<MT>());
            if (j > 0) {
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
                    part[((j - 1) * 32 + (int)lane) * MT + mt] = make_float4(acc[mt][0], acc[mt][1], acc[mt][2], acc[mt][3]);
            }
            asm volatile("bar.sync 2, %0;" ::"n"(kTailWarps * 32) : "memory");
            if (j > 0)
                return;
#pragma unroll
            for (int jj = 1; jj < kTailWarps; ++jj)
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    const float4 v = part[((jj - 1) * 32 + (int)lane) * MT + mt];
                    acc[mt][0] += v.x, acc[mt][1] += v.y, acc[mt][2] += v.z, acc[mt][3] += v.w;
                }
            float4 *ws = reinterpret_cast<float4 *>(a.tail_ws);
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
                __stcg(ws + ((int64_t)blockIdx.x * 32 + lane) * MT + mt,
                       make_float4(acc[mt][0], acc[mt][1], acc[mt][2], acc[mt][3]));
            __threadfence();
            __syncwarp();
            int last = 0;
            if (lane == 0)
                last = atomicAdd(a.tail_cnt + tail_tile, 1) == a.KU - 1;
            if (!__shfl_sync(0xFFFFFFFFu, last, 0))
                return;
            __threadfence();
            float sum[MT][4];
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
                sum[mt][0] = sum[mt][1] = sum[mt][2] = sum[mt][3] = 0.f;
            const int64_t u0 = (int64_t)tail_tile * a.KU;
            for (int u = 0; u < a.KU; u += 8) {
                /* eight units' loads in flight at once, added in unit order */
                float4 v[8][MT];
#pragma unroll
                for (int q = 0; q < 8; ++q)
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt)
                        v[q][mt] = u + q < a.KU ? __ldcg(ws + ((u0 + u + q) * 32 + lane) * MT + mt)
                                                : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int q = 0; q < 8; ++q)
                    if (u + q < a.KU) {
#pragma unroll
                        for (int mt = 0; mt < MT; ++mt) {
                            sum[mt][0] += v[q][mt].x, sum[mt][1] += v[q][mt].y;
                            sum[mt][2] += v[q][mt].z, sum[mt][3] += v[q][mt].w;
                        }
                    }
            }
            if (lane == 0)
                a.tail_cnt[tail_tile] = 0; /* every unit has arrived: zero for the next call */
            const int n16 = a.tail_row0 + tail_tile * 16;
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int n = n16 + pg + (q >> 1) * 8, col = mt * 8 + 2 * t + (q & 1);
                    if (n < a.N && col < a.M) {
                        if (BF16OUT)
                            static_cast<__nv_bfloat16 *>(a.y)[(int64_t)col * a.N + n] = __float2bfloat16_rn(sum[mt][q]);
                        else
                            static_cast<float *>(a.y)[(int64_t)col * a.N + n] = sum[mt][q];
                    }
                }
            return;
        }
        return;
    }

    /* warp kh takes the unit's 64-k blocks [kh*NB, (kh+1)*NB) (block b: slice b/4, block b%4) */
    const int tile = warp / KH, kh = warp % KH, b0 = kh * NB, r0 = tile * 16;
    /* block b of a unit: 64-k block c of slice u, whose rows start at row u RB of the
     * plane and absmax tiles; activation block 4 u + c */
    BlockOffs<MT> offs[NB];
#pragma unroll
    for (int j = 0; j < NB; ++j) {
        const int b = b0 + j, c = b & 3, u = b >> 2, xb = b * a.xrows;
        offs[j] = block_offs<MT>(c, r0, u * a.RB, g, t, (uint32_t)(2 * a.pt), (uint32_t)c,
                                 (uint32_t)(2 * a.pt + a.at + xb * 128), (uint32_t)xb & 7u, a.M);
    }
    float acc[MT][4];
    bool alive = true;
    int s = 0;
    uint32_t ph = 0;
    for (int blk = 0; blk < a.nb && alive; ++blk) {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
            acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;
        for (int ku = 0; ku < a.KU; ++ku) {
            bool ok = lane == 0 ? mbar_wait_suspend_bounded(&full[s], ph, &g_decode_error) : true;
            if (!__shfl_sync(0xFFFFFFFFu, ok ? 1 : 0, 0)) {
                alive = false;
                break;
            }
            const uint32_t st = saddr(ring + s * stage_bytes);
#pragma unroll
            for (int j = 0; j < NB; ++j)
                tile_block_at<MT, SPLIT>(st, (uint32_t)a.pt, offs[j], lut_base, lane4, acc);
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&empty[s]);
            if (++s == S)
                s = 0, ph ^= 1u;
        }
        if (!alive)
            break;
        /* add the tile's KH partial sums in k order (kh 0, 1, ...), then y */
        if (KH > 1) {
            if (kh > 0) {
                bool ok = true;
                if (blk > 0 && lane == 0)
                    ok = mbar_wait_suspend_bounded(cmb_empty, (uint32_t)(blk - 1) & 1u, &g_decode_error);
                if (!__shfl_sync(0xFFFFFFFFu, ok ? 1 : 0, 0))
                    break;
                float *dst = scratch + ((tile * (KH - 1) + kh - 1) * 32 + (int)lane) * 4 * MT;
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        dst[mt * 4 + q] = acc[mt][q];
                __syncwarp();
                if (lane == 0)
                    mbar_arrive(cmb_full);
                continue;
            }
            bool ok = lane == 0 ? mbar_wait_suspend_bounded(cmb_full, (uint32_t)blk & 1u, &g_decode_error) : true;
            if (!__shfl_sync(0xFFFFFFFFu, ok ? 1 : 0, 0))
                break;
            for (int kk = 1; kk < KH; ++kk) {
                const float *src = scratch + ((tile * (KH - 1) + kk - 1) * 32 + (int)lane) * 4 * MT;
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        acc[mt][q] += src[mt * 4 + q];
            }
            __syncwarp();
            if (lane == 0)
                mbar_arrive(cmb_empty);
        }
        const int nb0 = n_begin + blk * a.RB;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int row = r0 + pg + (q >> 1) * 8, col = mt * 8 + 2 * t + (q & 1);
                const int n = nb0 + row;
                if (row < a.RB && n < n_end && col < a.M) {
                    if (a.ga.world > 0) {
                        gather_store<BF16OUT>(a.ga, col, n, acc[mt][q]);
                    } else if (BF16OUT) {
                        static_cast<__nv_bfloat16 *>(a.y)[(int64_t)col * a.N + n] = __float2bfloat16_rn(acc[mt][q]);
                    } else {
                        static_cast<float *>(a.y)[(int64_t)col * a.N + n] = acc[mt][q];
                    }
                }
            }
        }
    }
    if (a.ga.world > 0)
        gather_complete(a.ga, active, lane, cta_done, &g_decode_error);
}

/* 3-D map: dims (d0, d1, d2) with byte strides s1, s2 for dims 1 and 2 (any order
 * of sizes), box (b0, b1, b2). */
bool make_map3(CUtensorMap *m, CUtensorMapDataType dt, const void *base, uint64_t d0, uint64_t d1, uint64_t d2,
               uint64_t s1, uint64_t s2, uint32_t b0, uint32_t b1, uint32_t b2, CUtensorMapSwizzle sw)
{
    auto enc = tensor_map_encoder();
    if (!enc)
        return false;
    cuuint64_t dims[3] = {d0, d1, d2};
    cuuint64_t strides[2] = {s1, s2};
    cuuint32_t box[3] = {b0, b1, b2};
    cuuint32_t estr[3] = {1, 1, 1};
    return enc(m, dt, 3, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_map(CUtensorMap *m, CUtensorMapDataType dt, const void *base, uint64_t cols, uint64_t rows,
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

/* Per (device, stream) scratch: partial sums and split-block flags. */
struct Scratch {
    float *ws = nullptr;
    size_t ws_floats = 0;
    int *counters = nullptr;
    size_t n_counters = 0;
};
std::mutex g_scratch_mu;
std::unordered_map<uint64_t, Scratch> g_scratch;

bool get_scratch(cudaStream_t st, size_t ws_floats, size_t n_counters, Scratch &out)
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess)
        return false;
    const uint64_t key = (reinterpret_cast<uint64_t>(st) << 8) ^ (uint64_t)dev;
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    Scratch &S = g_scratch[key];
    if (S.ws_floats < ws_floats) {
        if (S.ws)
            cudaFree(S.ws);
        S.ws = nullptr;
        S.ws_floats = 0;
        if (cudaMalloc(&S.ws, ws_floats * sizeof(float)) != cudaSuccess) {
            cudaGetLastError();
            return false;
        }
        S.ws_floats = ws_floats;
    }
    if (S.n_counters < n_counters) {
        if (S.counters)
            cudaFree(S.counters);
        S.counters = nullptr;
        S.n_counters = 0;
        if (cudaMalloc(&S.counters, n_counters * sizeof(int)) != cudaSuccess ||
            cudaMemset(S.counters, 0, n_counters * sizeof(int)) != cudaSuccess) {
            cudaGetLastError();
            return false;
        }
        S.n_counters = n_counters;
    }
    out = S;
    return true;
}

struct Maps {
    CUtensorMap h, p, am, x;
    CUtensorMap h16, p16, am16; /* 16-row boxes: the row-owned kernel's shared tail */
};

/* Launched with programmatic stream serialisation (PDL): the kernel may start
 * while the previous kernel in the stream drains; it streams weights at once and
 * waits (griddepcontrol.wait) before reading activations or touching y and its
 * workspace.  `pdl` is off for the fixed-scratch entry, whose flags are reset
 * by a memset just before the launch. */
template <int MT, bool SPLIT, bool BF16OUT>
int launch_t(const Maps &m, const DecodeArgs &a, int grid, cudaStream_t st, bool pdl)
{
    auto kern = htile_decode_kernel<MT, SPLIT, BF16OUT>;
    if (!ensure_smem((const void *)kern, smem_bytes<MT>()))
        return kLaunch;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem_bytes<MT>();
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    if (cudaLaunchKernelEx(&cfg, kern, m.h, m.p, m.am, m.x, a) != cudaSuccess) {
        cudaGetLastError();
        return kLaunch;
    }
    return kOk;
}

template <bool SPLIT, bool BF16OUT>
int launch_mt(int MT, const Maps &m, const DecodeArgs &a, int grid, cudaStream_t st, bool pdl)
{
    if (MT == 1)
        return launch_t<1, SPLIT, BF16OUT>(m, a, grid, st, pdl);
    if (MT == 2)
        return launch_t<2, SPLIT, BF16OUT>(m, a, grid, st, pdl);
    return launch_t<4, SPLIT, BF16OUT>(m, a, grid, st, pdl);
}

template <int MT, bool SPLIT, bool BF16OUT, int NB>
int launch_rows_nb(const Maps &m, const RowArgs &a, int grid, cudaStream_t st, bool pdl)
{
    auto kern = htile_rows_kernel<MT, SPLIT, BF16OUT, NB>;
    if (!ensure_smem((const void *)kern, r_smem_bytes<MT>()))
        return kLaunch;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = r_smem_bytes<MT>();
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    if (cudaLaunchKernelEx(&cfg, kern, m.h, m.p, m.am, m.x, m.h16, m.p16, m.am16, a) != cudaSuccess) {
        cudaGetLastError();
        return kLaunch;
    }
    return kOk;
}
template <int MT, bool SPLIT, bool BF16OUT>
int launch_rows_t(const Maps &m, const RowArgs &a, int grid, cudaStream_t st, bool pdl)
{
    const int nb = 4 * a.UB / a.KH;
    if (nb == 2)
        return launch_rows_nb<MT, SPLIT, BF16OUT, 2>(m, a, grid, st, pdl);
    if (nb == 1)
        return launch_rows_nb<MT, SPLIT, BF16OUT, 1>(m, a, grid, st, pdl);
    return kLaunch;
}

constexpr int align1k(int v) { return (v + 1023) & ~1023; }

/* Row block, warp and ring layout of the row-owned kernel for R rows per CTA.
 * Units take as many 256-k slices (UB = 4, 2, 1) as keep >= 3 ring stages, the
 * consumer warps' plan valid and K whole; row blocks of more than 4 tiles take
 * one (their requests are large already, and the shared tail needs UB = 1). */
bool plan_rows(RowArgs &a, int R, int MT)
{
    const int M = a.M, K = a.K;
    a.R = R;
    a.nb = (a.R + kRowBlockMax - 1) / kRowBlockMax;
    a.RB = (a.R + a.nb - 1) / a.nb;
    a.T = (a.RB + 15) / 16;
    a.xrows = std::min(M, 8 * MT);
    const int ring = MT == 1 ? r_ring<1>() : MT == 2 ? r_ring<2>() : r_ring<4>();
    const int scratch_warps = MT <= 2 ? 14 : 7;
    for (int ub = 4; ub >= 1; ub >>= 1) {
        if (ub > 1 && (a.T > 4 || K % (256 * ub) != 0))
            continue;
        /* warps per tile: as many consumer warps as the 16 allow, two blocks per warp
         * and unit where that still fills them (MT 4: one, for registers) */
        const int blocks = 4 * ub;
        int nbk = MT <= 2 ? 2 : 1, kh = blocks / nbk;
        while ((a.T * kh > kConsumers || a.T * (kh - 1) > scratch_warps) && nbk < blocks) {
            nbk *= 2;
            kh = blocks / nbk;
        }
        if (a.T * kh < kConsumers / 2 && nbk > 1 && a.T * kh * 2 <= kConsumers && a.T * (kh * 2 - 1) <= scratch_warps) {
            nbk /= 2;
            kh = blocks / nbk;
        }
        if (a.T * kh > kConsumers || a.T * (kh - 1) > scratch_warps || nbk > 2)
            continue;
        const int pt = align1k(ub * a.RB * 128), at = align1k(ub * a.RB * 16), xt = align1k(4 * ub * a.xrows * 128);
        const int stage = 2 * pt + at + xt;
        const int S = std::min(kRMaxStages, ring / stage);
        if (S < (ub > 1 ? 3 : 2))
            continue;
        a.UB = ub, a.KH = kh, a.pt = pt, a.at = at, a.xt = xt, a.stage = stage, a.S = S;
        a.KU = K / (256 * ub);
        a.tx = (uint32_t)(ub * (2 * a.RB * 128 + a.RB * 16 + 4 * a.xrows * 128));
        return true;
    }
    return false;
}

/* The row-owned kernel for N >= 16 x SMs.  Where the 16-row tiles leave a
 * remainder over the SMs (N = 14336: 896 tiles, 6.05 per SM) and it is small
 * enough for one 256-k unit per CTA, the CTAs own 16 x floor(tiles / SMs) rows
 * and share the leftover tiles unit by unit on idle warps (`tail`: not for
 * gathered calls or the fixed-scratch entry), instead of 16 x ceil rows, which
 * leave most SMs a mostly empty last tile. */
int launch_rows(const uint8_t *hole, const uint8_t *plug, const float *am, const __nv_bfloat16 *x, void *y,
                OutKind yk, int M, int N, int K, HtileMode mode, cudaStream_t st, bool pdl,
                const GatherArgs *gt = nullptr, bool tail = false)
{
    const int MT = M <= 8 ? 1 : (M <= 16 ? 2 : 4);
    const int sms = sm_count();
    RowArgs a{};
    a.y = y, a.M = M, a.N = N, a.K = K;
    if (gt)
        a.ga = *gt;
    int grid = 0;
    const int tiles = (N + 15) / 16, base = tiles / sms, extra = tiles - base * sms;
    if (tail && !gt && MT <= 2 && base >= 1 && extra > 0 && (int64_t)extra * (K / 256) <= sms) {
        RowArgs t = a;
        if (plan_rows(t, base * 16, MT) && t.UB == 1 && t.T * t.KH + kTailWarps <= kConsumers) {
            Scratch S;
            t.tail_units = extra * t.KU;
            if (get_scratch(st, (size_t)t.tail_units * 32 * 4 * MT, (size_t)extra, S)) {
                t.tail_row0 = sms * base * 16;
                t.tail_tx = (uint32_t)(2 * 16 * 128 + 16 * 16 + 4 * t.xrows * 128);
                t.tail_ws = S.ws;
                t.tail_cnt = S.counters;
                a = t;
                grid = sms;
            }
        }
    }
    if (!grid) {
        const int g0 = std::max(1, std::min(sms, tiles));
        if (!plan_rows(a, (N + g0 - 1) / g0, MT))
            return kLaunch;
        grid = (N + a.R - 1) / a.R;
    }
    /* 3-D views (inner bytes, rows, k slices) of the row-major planes, absmax and
     * activations: a box is [slices][rows][inner] in shared memory */
    Maps maps;
    if (!make_map3(&maps.h, CU_TENSOR_MAP_DATA_TYPE_UINT8, hole, 128, (uint64_t)N, (uint64_t)K / 256,
                   (uint64_t)K / 2, 128, 128, (uint32_t)a.RB, (uint32_t)a.UB, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_map3(&maps.p, CU_TENSOR_MAP_DATA_TYPE_UINT8, plug, 128, (uint64_t)N, (uint64_t)K / 256,
                   (uint64_t)K / 2, 128, 128, (uint32_t)a.RB, (uint32_t)a.UB, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_map3(&maps.am, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, am, 4, (uint64_t)N, (uint64_t)K / 256,
                   (uint64_t)K / 64 * 4, 16, 4, (uint32_t)a.RB, (uint32_t)a.UB, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !make_map3(&maps.x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, 64, (uint64_t)M, (uint64_t)K / 64, (uint64_t)K * 2,
                   128, 64, (uint32_t)a.xrows, (uint32_t)(4 * a.UB), CU_TENSOR_MAP_SWIZZLE_128B))
        return kLaunch;
    if (a.tail_units) {
        if (!make_map(&maps.h16, CU_TENSOR_MAP_DATA_TYPE_UINT8, hole, (uint64_t)K / 2, (uint64_t)N, (uint64_t)K / 2,
                      128, 16, CU_TENSOR_MAP_SWIZZLE_128B) ||
            !make_map(&maps.p16, CU_TENSOR_MAP_DATA_TYPE_UINT8, plug, (uint64_t)K / 2, (uint64_t)N, (uint64_t)K / 2,
                      128, 16, CU_TENSOR_MAP_SWIZZLE_128B) ||
            !make_map(&maps.am16, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, am, (uint64_t)K / 64, (uint64_t)N,
                      (uint64_t)K / 64 * 4, 4, 16, CU_TENSOR_MAP_SWIZZLE_NONE))
            return kLaunch;
    } else {
        maps.h16 = maps.h, maps.p16 = maps.p, maps.am16 = maps.am; /* not read */
    }
    const bool bf = yk == kOutBF16, pr = mode == kPrecise;
#define GLINT_ROWS_CASE(mt)                                                                                            \
    if (MT == mt)                                                                                                      \
        return pr ? (bf ? launch_rows_t<mt, true, true>(maps, a, grid, st, pdl)                                         \
                        : launch_rows_t<mt, true, false>(maps, a, grid, st, pdl))                                       \
                  : (bf ? launch_rows_t<mt, false, true>(maps, a, grid, st, pdl)                                        \
                        : launch_rows_t<mt, false, false>(maps, a, grid, st, pdl));
    GLINT_ROWS_CASE(1)
    GLINT_ROWS_CASE(2)
    GLINT_ROWS_CASE(4)
#undef GLINT_ROWS_CASE
    return kLaunch;
}

/* Row-owned decode when every SM can own >= 16 rows and no CTA has more than 2
 * row blocks (beyond that stream-K keeps more warps busy), and for narrower layers
 * (16-row CTAs on fewer SMs) while a CTA's slice stays <= 16 x 8192 weights: up
 * to there it beats stream-K, whose split-K partial sums cost more than the SMs
 * left idle (N = 1024, K = 4096: 8.0 against 11.7 us); for longer K, stream-K. */
bool rows_supported(int N, int K)
{
    const int sms = sm_count();
    return N >= 16 && N <= 2 * kRowBlockMax * sms && (N >= 16 * sms || K <= 8192);
}

} // namespace

bool htile_decode_supported(const uint8_t *hole, const uint8_t *plug, const float *am, const __nv_bfloat16 *x,
                            int M, int N, int K, int bs)
{
    /* K % 256: the absmax rows (K/64 floats) must be a multiple of 16 bytes for TMA */
    return M >= 1 && M <= 32 && bs == 64 && K % 256 == 0 && aligned_to(hole, 16) && aligned_to(plug, 16) &&
           aligned_to(am, 16) && aligned_to(x, 16) && N >= 1 && tensor_map_encoder() != nullptr;
}

/* tensor maps of one call: plane rows of kKU/2 bytes (64B or 128B swizzle) */
bool decode_maps(Maps &maps, const uint8_t *hole, const uint8_t *plug, const float *am, const __nv_bfloat16 *x, int M,
                 int N, int K, int MT)
{
    const int ku = MT <= 2 ? ku_of<1>() : ku_of<4>();
    const CUtensorMapSwizzle sw = ku == 256 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    return make_map(&maps.h, CU_TENSOR_MAP_DATA_TYPE_UINT8, hole, (uint64_t)K / 2, (uint64_t)N, (uint64_t)K / 2,
                    (uint32_t)ku / 2, kRows, sw) &&
           make_map(&maps.p, CU_TENSOR_MAP_DATA_TYPE_UINT8, plug, (uint64_t)K / 2, (uint64_t)N, (uint64_t)K / 2,
                    (uint32_t)ku / 2, kRows, sw) &&
           make_map(&maps.am, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, am, (uint64_t)K / 64, (uint64_t)N, (uint64_t)K / 64 * 4,
                    4, kRows, CU_TENSOR_MAP_SWIZZLE_NONE) &&
           make_map(&maps.x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, 64,
                    (uint32_t)(8 * MT), CU_TENSOR_MAP_SWIZZLE_128B);
}

int decode_launch_impl(const uint8_t *hole, const uint8_t *plug, const float *am, const __nv_bfloat16 *x, void *y,
                       OutKind yk, int M, int N, int K, HtileMode mode, cudaStream_t st, const GatherArgs *gt)
{
    if (rows_supported(N, K))
        return launch_rows(hole, plug, am, x, y, yk, M, N, K, mode, st, true, gt, gt == nullptr);
    const int MT = M <= 8 ? 1 : (M <= 16 ? 2 : 4);
    Maps maps;
    if (!decode_maps(maps, hole, plug, am, x, M, N, K, MT))
        return kLaunch;
    DecodeArgs a{};
    a.x = x;
    a.y = y;
    a.M = M;
    a.N = N;
    a.K = K;
    a.KU = K / (MT <= 2 ? ku_of<1>() : ku_of<4>());
    const int64_t rbs = (N + kRows - 1) / kRows;
    a.units = rbs * a.KU;
    const int grid = (int)std::min<int64_t>(a.units, sm_count());
    /* parts per row block: at most ceil(KU / units_per_cta) + 1 */
    const int64_t per_cta = std::max<int64_t>(1, a.units / grid);
    a.max_parts = (int)std::min<int64_t>(grid, (a.KU + per_cta - 1) / per_cta + 1);
    Scratch S;
    if (!get_scratch(st, (size_t)rbs * a.max_parts * kRows * 8 * MT, (size_t)rbs * a.max_parts * kConsumers, S))
        return kLaunch;
    a.ws = S.ws;
    a.flags = S.counters;
    if (gt)
        a.ga = *gt;
    const bool bf = yk == kOutBF16;
    if (mode == kPrecise)
        return bf ? launch_mt<true, true>(MT, maps, a, grid, st, true) : launch_mt<true, false>(MT, maps, a, grid, st, true);
    return bf ? launch_mt<false, true>(MT, maps, a, grid, st, true) : launch_mt<false, false>(MT, maps, a, grid, st, true);
}

/* ---- fixed-scratch variant ---------------------------------------------------
 * Some callers cannot let a library allocate device memory: a serving process
 * that hands all free HBM to its own cache pool up front, or an integration whose
 * memory is budgeted before the first call and must not see cudaMalloc (which can
 * fail under that budget and synchronises the device).  For them the decode path
 * can run on a fixed scratch area compiled into this file instead of the
 * per-stream workspace above: kNoAllocBytes per device, allocated with the
 * library's device image when it is loaded on a device and held until the
 * process exits.  The first kNoAllocCounterBytes hold the per (row block, part,
 * warp) split-block flags, the rest the split-K partial sums: rb x parts x 256
 * rows x 8 MT floats (rb row blocks, parts as max_parts below), so calls whose
 * sums exceed 4 MiB - 64 KiB return kScratch.  Only the stream-K kernel uses it;
 * row-owned shapes need no scratch. */
constexpr size_t kNoAllocBytes = size_t(4) << 20;   /* 4 MiB per device */
constexpr size_t kNoAllocCounterBytes = 64 << 10;   /* 16384 flags (row blocks x parts x warps) */
constexpr int kNoAllocMaxN = 65536;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

namespace {
/* The array's device address, looked up once per device and context: keyed on the
 * context's process-unique id, so a context destroyed by cudaDeviceReset and
 * created again gets a fresh lookup instead of a dangling address. */
struct NoAllocAddr {
    unsigned long long ctx_id = 0;
    void *addr = nullptr;
};
std::mutex g_noalloc_mu;
NoAllocAddr g_noalloc_addr[64];

using PFN_ctxGetCurrent = CUresult (*)(CUcontext *);
using PFN_ctxGetId = CUresult (*)(CUcontext, unsigned long long *);

/* id of the calling thread's current context (0 when none is current or the driver
 * entry points are unavailable) */
unsigned long long current_ctx_id()
{
    static PFN_ctxGetCurrent get_cur = nullptr;
    static PFN_ctxGetId get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr, *q = nullptr;
        cudaDriverEntryPointQueryResult r1, r2;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &r1) == cudaSuccess &&
            r1 == cudaDriverEntryPointSuccess &&
            cudaGetDriverEntryPoint("cuCtxGetId", &q, cudaEnableDefault, &r2) == cudaSuccess &&
            r2 == cudaDriverEntryPointSuccess) {
            get_cur = reinterpret_cast<PFN_ctxGetCurrent>(p);
            get_id = reinterpret_cast<PFN_ctxGetId>(q);
        } else {
            cudaGetLastError();
        }
    });
    CUcontext c = nullptr;
    unsigned long long id = 0;
    if (!get_cur || !get_id || get_cur(&c) != CUDA_SUCCESS || !c || get_id(c, &id) != CUDA_SUCCESS)
        return 0;
    return id;
}

/* Device address of g_noalloc_scratch on the current device (nullptr on failure). */
void *noalloc_base(int dev)
{
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    NoAllocAddr &e = g_noalloc_addr[dev];
    const unsigned long long id = current_ctx_id();
    if (e.addr && id != 0 && id == e.ctx_id)
        return e.addr;
    /* host code only sees a stand-in for the array: ask the runtime for its device
     * address with this device current (this also creates the context if needed) */
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) {
        cudaGetLastError();
        e = NoAllocAddr{};
        return nullptr;
    }
    e.addr = p;
    e.ctx_id = current_ctx_id();
    return p;
}
} // namespace

int htile_decode_launch(const uint8_t *hole, const uint8_t *plug, const float *am, const __nv_bfloat16 *x, void *y,
                        OutKind yk, int M, int N, int K, HtileMode mode, cudaStream_t st)
{
    return decode_launch_impl(hole, plug, am, x, y, yk, M, N, K, mode, st, nullptr);
}

bool htile_gather_supported(int M, int N) { return M >= 1 && M <= 32 && N >= 1; }

int htile_decode_gather_launch(const uint8_t *hole, const uint8_t *plug, const float *am, const __nv_bfloat16 *x,
                               void *const *y_ranks, uint32_t *const *flag_ranks, int world, int rank,
                               OutKind yk, int M, int N, int K, int ldy, int n0, HtileMode mode, cudaStream_t st)
{
    GatherArgs g;
    if (!htile_gather_supported(M, N) || !make_gather_args(&g, y_ranks, flag_ranks, world, rank, ldy, n0))
        return kUnsupported;
    return decode_launch_impl(hole, plug, am, x, y_ranks[rank], yk, M, N, K, mode, st, &g);
}

namespace {
/* A column shard gathered into every rank's buffer: src [M, cols] (row stride
 * ld_src elements, elem_bytes 2 or 4) goes to columns [n0, n0 + cols) of every
 * rank's y [M, ldy], then the CTA counts in (gather_complete).  One warp per 32
 * consecutive elements of a row; 8 warps per CTA. */
__global__ void __launch_bounds__(256) gather_copy_kernel(const GatherArgs g, const uint8_t *__restrict__ src,
                                                          int elem_bytes, int M, int cols, int ld_src)
{
    __shared__ uint32_t cta_done;
    if (threadIdx.x == 0)
        cta_done = 0;
    __syncthreads();
    const int64_t total = (int64_t)M * cols;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int m = (int)(e / cols), c = (int)(e - (int64_t)m * cols);
        const int64_t si = (int64_t)m * ld_src + c, di = (int64_t)m * g.ldy + g.n0 + c;
        for (int i = 1; i <= g.world; ++i) {
            const int r = (g.rank + i) % g.world;
            if (elem_bytes == 2)
                reinterpret_cast<uint16_t *>(g.yr[r])[di] = reinterpret_cast<const uint16_t *>(src)[si];
            else
                reinterpret_cast<uint32_t *>(g.yr[r])[di] = reinterpret_cast<const uint32_t *>(src)[si];
        }
    }
    gather_complete(g, (int)(blockDim.x >> 5), threadIdx.x & 31u, &cta_done, &g_decode_error);
}
} // namespace

int gather_copy_launch(const void *src, int elem_bytes, int M, int cols, int ld_src, void *const *y_ranks,
                       uint32_t *const *flag_ranks, int world, int rank, int ldy, int n0, cudaStream_t st)
{
    GatherArgs g;
    if ((elem_bytes != 2 && elem_bytes != 4) || !make_gather_args(&g, y_ranks, flag_ranks, world, rank, ldy, n0))
        return kUnsupported;
    const int64_t total = (int64_t)M * cols;
    const int ctas = (int)std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, 2 * sm_count()));
    gather_copy_kernel<<<ctas, 256, 0, st>>>(g, static_cast<const uint8_t *>(src), elem_bytes, M, cols, ld_src);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunch;
}

int htile_decode_launch_noalloc(const uint8_t *hole, const uint8_t *plug, const float *am, const __nv_bfloat16 *x,
                                void *y, OutKind yk, int M, int N, int K, HtileMode mode, cudaStream_t st)
{
    /* the documented limit of this entry point, whichever kernel runs */
    if (N > kNoAllocMaxN)
        return kScratch;
    if (rows_supported(N, K)) /* needs no scratch at all */
        return launch_rows(hole, plug, am, x, y, yk, M, N, K, mode, st, false);
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return kLaunch;
    void *base = noalloc_base(dev);
    if (!base)
        return kLaunch;
    const int MT = M <= 8 ? 1 : (M <= 16 ? 2 : 4);
    DecodeArgs a{};
    a.x = x;
    a.y = y;
    a.M = M;
    a.N = N;
    a.K = K;
    a.KU = K / (MT <= 2 ? ku_of<1>() : ku_of<4>());
    const int64_t rbs = (N + kRows - 1) / kRows;
    a.units = rbs * a.KU;
    const int grid = (int)std::min<int64_t>(a.units, sm_count());
    const int64_t per_cta = std::max<int64_t>(1, a.units / grid);
    a.max_parts = (int)std::min<int64_t>(grid, (a.KU + per_cta - 1) / per_cta + 1);
    const size_t counter_bytes = (size_t)rbs * a.max_parts * kConsumers * sizeof(int);
    const size_t ws_bytes = (size_t)rbs * a.max_parts * kRows * 8 * MT * sizeof(float);
    if (counter_bytes > kNoAllocCounterBytes || ws_bytes > kNoAllocBytes - kNoAllocCounterBytes)
        return kScratch;
    Maps maps;
    if (!decode_maps(maps, hole, plug, am, x, M, N, K, MT))
        return kLaunch;
    /* the array keeps the previous call's contents: the flags must start at 0 */
    a.flags = static_cast<int *>(base);
    a.ws = reinterpret_cast<float *>(static_cast<unsigned char *>(base) + kNoAllocCounterBytes);
    if (cudaMemsetAsync(a.flags, 0, counter_bytes, st) != cudaSuccess)
        return kLaunch;
    const bool bf = yk == kOutBF16;
    if (mode == kPrecise)
        return bf ? launch_mt<true, true>(MT, maps, a, grid, st, false) : launch_mt<true, false>(MT, maps, a, grid, st, false);
    return bf ? launch_mt<false, true>(MT, maps, a, grid, st, false) : launch_mt<false, false>(MT, maps, a, grid, st, false);
}

/* This file's kernel error word (bounded waits that ran out); clear resets it. */
int decode_error_word(bool clear) { return read_error_word(g_decode_error, g_decode_error_taken, clear); }

} // namespace glint
