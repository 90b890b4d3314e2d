/* K-major GLINT: parent-only decode GEMV with an activation-selected plug
 * correction, on sm_100a.
 *
 * Follows the reference's Mojo decoders (Jadon-Fox/glint):
 *   - layout           transpose_plug (mojo/p7_glint_select_decode.mojo:120-135) for
 *                      both planes, transpose_scales (mojo/p7_select_device.mojo:197-208):
 *                      plane_k[c * n/2 + r/2] holds row r of input channel c in
 *                      nibble r & 1; scales_k[(c/64) * n + r] = absmax[r * K/64 + c/64];
 *   - parent GEMV      glint_gemv_km + gemv_km_combine (mojo/p7_glint_gemv_km.mojo:17-95):
 *                      y[r] = sum_c PARENT[h] * scale * x[c], M = 1, hole plane only;
 *   - selection        select_topk's default rule (mojo/p7_select_device.mojo:15-153):
 *                      key = BF16 bits & 0x7FFF, T = the largest key value with at
 *                      least nsel keys >= T, every channel with key >= T kept,
 *                      ascending; nsel = 0 keeps none;
 *   - correction       apply_corr_k (mojo/p7_select_device.mojo:210-238): y[r] +=
 *                      sum over the selected channels, in list order, of
 *                      (delta[h][p] * scale) * x[c], delta = CELLS - PARENT.
 * With every channel selected, parent GEMV + correction is the full GLINT GEMV.
 *
 * The B200 shape of it:
 *   - parent GEMV: a thread owns 8 rows (one 32-bit word of a channel row, so a warp
 *     reads 128 contiguous bytes per channel); the 8 warps of a CTA share 256 rows
 *     and take different 64-channel blocks, so each 64-block is summed in a register
 *     accumulator and scaled once (y += scale * sum(parent * x)); the CTA adds its
 *     warps in order and writes one partial per channel slice; the combine adds the
 *     slices in order.  Lookups go through a per-lane replica of a 256-entry table
 *     of parent PAIRS (one byte = two rows), addressed with one byte permute, so a
 *     warp's 32 lookups never share a bank.  Hole words stream with 16 loads in
 *     flight per thread.  Algorithmic bytes: N*K/2 (hole) + N*K/16 (scales) + 2K + 4N.
 *   - selection: one CTA; the keys go to shared memory once, two histogram passes
 *     (key >> 7, then key & 127 inside the threshold's bucket) find T exactly, then
 *     a block-wide scan writes the kept channels in ascending order.
 *   - correction: the same 8-rows-per-thread mapping over the selected channels,
 *     cut into fixed chunks of the list (partials added in order, so the result
 *     does not depend on scheduling); the scale row is reloaded only when the
 *     channel's 64-block changes; the plug rows may be device memory or pinned host
 *     memory mapped into the device (zero-copy: only the selected channels' plug
 *     bytes cross PCIe).
 * No kernel here waits on another CTA or another kernel, so nothing can hang.
 */
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "glint_internal.h"
#include "ptx.cuh"

namespace glint {

namespace {

static __device__ const float g_parent[16] = GLINT_PARENT_INIT;

/* ---- layout ------------------------------------------------------------------ */
constexpr int kTR = 64;  /* rows per transpose tile */
constexpr int kTC = 128; /* channels per transpose tile (64 bytes of a row) */

/* plane [n, K/2] (row-major nibbles) -> plane_k [K, n/2]; blockIdx.z picks the plane */
__global__ void __launch_bounds__(256) kmajor_planes_kernel(const uint8_t *__restrict__ hole,
                                                            const uint8_t *__restrict__ plug,
                                                            uint8_t *__restrict__ hole_k,
                                                            uint8_t *__restrict__ plug_k, int n, int K)
{
    __shared__ uint8_t t[kTR][kTC / 2 + 4];
    const uint8_t *src = blockIdx.z ? plug : hole;
    uint8_t *dst = blockIdx.z ? plug_k : hole_k;
    const int r0 = (int)blockIdx.y * kTR, c0 = (int)blockIdx.x * kTC;
    const int64_t rb = K / 2, half = n / 2;
    for (int i = threadIdx.x; i < kTR * (kTC / 2); i += 256) {
        const int rr = i / (kTC / 2), bb = i % (kTC / 2);
        const int r = r0 + rr;
        const int64_t byte = c0 / 2 + bb;
        t[rr][bb] = (r < n && byte < rb) ? src[(int64_t)r * rb + byte] : 0;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < kTC * (kTR / 2); i += 256) {
        const int cc = i / (kTR / 2), b = i % (kTR / 2);
        const int c = c0 + cc;
        const int64_t ob = r0 / 2 + b;
        if (c < K && ob < half) {
            const int sh = 4 * (cc & 1);
            const uint32_t lo = (t[2 * b][cc >> 1] >> sh) & 15u, hi = (t[2 * b + 1][cc >> 1] >> sh) & 15u;
            dst[(int64_t)c * half + ob] = (uint8_t)(lo | (hi << 4));
        }
    }
}

/* absmax [n, KB] -> scales_k [KB, n] */
__global__ void __launch_bounds__(256) kmajor_scales_kernel(const float *__restrict__ am, float *__restrict__ sk,
                                                            int n, int KB)
{
    __shared__ float t[32][33];
    const int r0 = (int)blockIdx.y * 32, b0 = (int)blockIdx.x * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    for (int j = ty; j < 32; j += 8) {
        const int r = r0 + j, b = b0 + tx;
        t[j][tx] = (r < n && b < KB) ? am[(int64_t)r * KB + b] : 0.f;
    }
    __syncthreads();
    for (int j = ty; j < 32; j += 8) {
        const int b = b0 + j, r = r0 + tx;
        if (b < KB && r < n)
            sk[(int64_t)b * n + r] = t[tx][j];
    }
}

/* ---- parent-only GEMV -------------------------------------------------------- */
constexpr int kKmThreads = 128;           /* 4 warps on 4 consecutive 256-row groups */
constexpr int kKmRows = kKmThreads * 8;   /* 1024 rows: 512 contiguous bytes of each channel row */
constexpr int kUnroll = 16;               /* channels per load batch (two batches in flight) */
constexpr int kMaxBps = 128;              /* 64-blocks per channel slice at most (x: 32 KB) */
constexpr int kPairBytes = 256 * 32 * 8;  /* pair table: entry e (a plane byte), lane l at e*256 + l*8 */
constexpr int kCorrChunk = 8;             /* correction: list entries per warp */
constexpr int kCorrThreads = 256;         /* correction: 8 warps on the same 256 rows, different list chunks */

__device__ __forceinline__ uint32_t ldg_stream32(const uint32_t *p)
{
    uint32_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}

template <int U>
__device__ __forceinline__ void load_words(uint32_t (&w)[U], const uint32_t *hp, int nw)
{
#pragma unroll
    for (int u = 0; u < U; ++u)
        w[u] = ldg_stream32(hp + (int64_t)u * nw);
}

/* acc[j] += PARENT[nibble j of w[u]] * x[u] over a batch; tb = this lane's table base */
template <int U>
__device__ __forceinline__ void parent_batch(float (&acc)[8], const uint32_t (&w)[U], const float *xb, uint32_t tb)
{
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const float xv = xb[u];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            /* entry (nibble) at nibble * 128 bytes, this lane's copy at lane * 4 */
            const float pv = __uint_as_float(lds32(tb + (((w[u] >> (4 * j)) & 15u) << 7)));
            acc[j] = fmaf(pv, xv, acc[j]);
        }
    }
}

/* part[blockIdx.y][r] (or y when there is one slice) for the 1024 rows of row group
 * blockIdx.x and 64-blocks [b0, b1) of slice blockIdx.y.  A thread owns rows
 * 8 wi .. 8 wi + 7 (one 32-bit word of every channel row); every 64-block's sum is
 * scaled once.  Loads run a batch ahead of the arithmetic. */
__global__ void __launch_bounds__(kKmThreads) gemv_km_kernel(const uint32_t *__restrict__ hole_k,
                                                             const float *__restrict__ sk,
                                                             const __nv_bfloat16 *__restrict__ x,
                                                             float *__restrict__ out, int n, int K, int bps)
{
    __shared__ __align__(16) float tab[16 * 32]; /* PARENT[v] for lane l at v * 32 + l */
    extern __shared__ __align__(16) float xs[];   /* x of the slice, f32 */
    const int lane = (int)(threadIdx.x & 31);
    const int nw = n / 8;
    const int wi = (int)blockIdx.x * kKmThreads + (int)threadIdx.x;
    const int KB = K / 64;
    const int b0 = (int)blockIdx.y * bps, b1 = min(KB, b0 + bps);
    const int nch = (b1 - b0) * 64;
    const bool live = wi < nw;
    const uint32_t *hp = hole_k + (int64_t)b0 * 64 * nw + wi;

    uint32_t wa[kUnroll], wb[kUnroll];
    if (live)
        load_words(wa, hp, nw); /* in flight while the tables fill */
    for (int i = threadIdx.x; i < 16 * 32; i += kKmThreads)
        tab[i] = g_parent[i >> 5];
    for (int i = threadIdx.x; i < nch; i += kKmThreads)
        xs[i] = __bfloat162float(x[(int64_t)b0 * 64 + i]);
    __syncthreads();
    if (!live)
        return;
    const uint32_t tb = smem_u32(tab) + (uint32_t)lane * 4u;
    float y8[8], acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
        y8[j] = 0.f, acc[j] = 0.f;
    float4 s0 = __ldg(reinterpret_cast<const float4 *>(sk + (int64_t)b0 * n + 8 * wi));
    float4 s1 = __ldg(reinterpret_cast<const float4 *>(sk + (int64_t)b0 * n + 8 * wi + 4));
    /* two batches per step: wa holds channels c .. c+15, wb c+16 .. c+31 */
#pragma unroll 1
    for (int c = 0; c < nch; c += 2 * kUnroll) {
        load_words(wb, hp + (int64_t)(c + kUnroll) * nw, nw);
        parent_batch(acc, wa, xs + c, tb);
        if (c + 2 * kUnroll < nch)
            load_words(wa, hp + (int64_t)(c + 2 * kUnroll) * nw, nw);
        parent_batch(acc, wb, xs + c + kUnroll, tb);
        if (((c + 2 * kUnroll) & 63) == 0) {
            /* end of a 64-block: scale its sums, fetch the next block's scales */
            y8[0] = fmaf(s0.x, acc[0], y8[0]);
            y8[1] = fmaf(s0.y, acc[1], y8[1]);
            y8[2] = fmaf(s0.z, acc[2], y8[2]);
            y8[3] = fmaf(s0.w, acc[3], y8[3]);
            y8[4] = fmaf(s1.x, acc[4], y8[4]);
            y8[5] = fmaf(s1.y, acc[5], y8[5]);
            y8[6] = fmaf(s1.z, acc[6], y8[6]);
            y8[7] = fmaf(s1.w, acc[7], y8[7]);
#pragma unroll
            for (int j = 0; j < 8; ++j)
                acc[j] = 0.f;
            const int nb = b0 + (c + 2 * kUnroll) / 64;
            if (nb < b1) {
                s0 = __ldg(reinterpret_cast<const float4 *>(sk + (int64_t)nb * n + 8 * wi));
                s1 = __ldg(reinterpret_cast<const float4 *>(sk + (int64_t)nb * n + 8 * wi + 4));
            }
        }
    }
    float4 *o = reinterpret_cast<float4 *>(out + (int64_t)blockIdx.y * n + 8 * wi);
    o[0] = make_float4(y8[0], y8[1], y8[2], y8[3]);
    o[1] = make_float4(y8[4], y8[5], y8[6], y8[7]);
}

/* ---- parent-only GEMV, streamed (n % 32 == 0) --------------------------------
 * Persistent CTAs, one per SM: a producer warp moves the hole plane through a
 * shared-memory ring with 1-D bulk copies (one 1 KB channel segment = 2048 rows
 * per copy, 16 channels and their 16 x values per stage), so the bytes in flight do
 * not depend on how many warps are resident; 8 consumer warps (a thread per 8 rows)
 * read their words from shared memory and look parents up in pairs.  Work is split
 * stream-K over units (2048-row group g, 16-channel unit q), u = g * K/16 + q: CTA p
 * takes units [p U / P, (p+1) U / P), at most two row groups, and writes one
 * partial per group it touches; the combine adds, for each row, the partials of the
 * CTAs that covered its group, in CTA order. */
constexpr int kSRows = 2048, kSWords = kSRows / 8, kSegBytes = kSRows / 2;
constexpr int kSCh = 16;     /* channels per stage */
constexpr int kSStages = 6;
constexpr int kSCons = 16;   /* consumer warps: two halves of 8, each on half of a stage's channels */
constexpr int kSThreads = (kSCons + 1) * 32;
constexpr int kStageBytes = kSCh * kSegBytes; /* 16 KB */
/* dynamic shared memory: pair table, stage ring (TMA destinations: 128-byte aligned
 * offsets), x values, barriers, the 16 parents; no static shared memory in the
 * kernel, so the dynamic area starts at the base */
constexpr int kSSmem = kPairBytes + kSStages * kStageBytes + kSStages * 32 + 2 * kSStages * 8 + 16 * 4;

__device__ __forceinline__ uint64_t lds64u(uint32_t a)
{
    uint64_t v;
    asm volatile("ld.shared.b64 %0, [%1];" : "=l"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint64_t f2pack(float lo, float hi)
{
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ float2 f2unpack(uint64_t v)
{
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
    return r;
}
/* d = a * b + d on two f32 lanes */
__device__ __forceinline__ void fma2(uint64_t &d, uint64_t a, uint64_t b)
{
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(d) : "l"(a), "l"(b));
}

__device__ int g_km_error = 0;
__device__ int g_km_error_taken = 0;

struct KmStream {
    int n, K, QK;  /* QK = K / 16 units per row group */
    int64_t U;     /* units in all */
    int P;         /* CTAs */
};
__device__ __forceinline__ int64_t km_unit_begin(const KmStream &a, int p) { return (int64_t)p * a.U / a.P; }

__global__ void __launch_bounds__(kSThreads, 1) gemv_km_stream_kernel(const __grid_constant__ CUtensorMap hmap,
                                                                      const float *__restrict__ sk,
                                                                      const __nv_bfloat16 *__restrict__ x,
                                                                      float *__restrict__ part, const KmStream a)
{
    extern __shared__ __align__(16) uint8_t smem[];
    uint8_t *pairs = smem;
    uint8_t *ring = smem + kPairBytes;
    uint8_t *xring = ring + kSStages * kStageBytes;
    uint64_t *full = reinterpret_cast<uint64_t *>(xring + kSStages * 32);
    uint64_t *empty = full + kSStages;
    float *par = reinterpret_cast<float *>(empty + kSStages);
    const int warp = (int)(threadIdx.x >> 5), lane = (int)(threadIdx.x & 31);
    const int p = (int)blockIdx.x;
    const int64_t ub = km_unit_begin(a, p), ue = km_unit_begin(a, p + 1);
    if (threadIdx.x == 0) {
        for (int i = 0; i < kSStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kSCons);
        }
        mbar_init_fence();
    }
    if ((smem_u32(ring) & 127u) != 0u) {
        /* a tensor copy needs a 128-byte aligned destination: report, never issue */
        if (threadIdx.x == 0)
            atomicOr(&g_km_error, 2);
        return;
    }
    if (threadIdx.x < 16)
        par[threadIdx.x] = g_parent[threadIdx.x];
    __syncthreads();
    for (int i = threadIdx.x; i < 256 * 32 / 2; i += kSThreads) {
        const int e = i >> 4;
        const float2 pr = make_float2(par[e & 15], par[e >> 4]);
        reinterpret_cast<float4 *>(pairs)[i] = make_float4(pr.x, pr.y, pr.x, pr.y);
    }
    __syncthreads();
    if (warp == kSCons) {
        /* ---- producer */
        if (lane == 0) {
            int64_t i = 0;
            bool ok = true;
            for (int64_t u = ub; u < ue && ok; ++u, ++i) {
                const int st = (int)(i % kSStages);
                const uint32_t ph = (uint32_t)(i / kSStages) & 1u;
                if (i >= kSStages && !(ok = mbar_wait_suspend_bounded(&empty[st], ph ^ 1u, &g_km_error)))
                    break;
                const int g = (int)(u / a.QK), q = (int)(u - (int64_t)g * a.QK);
                /* one box: 16 channel rows x 256 words (1 KB each; words past n/8 are
                 * zero-filled and count in full), then the 16 x values */
                mbar_expect_tx(&full[st], (uint32_t)(kStageBytes + 32));
                tma_load_2d(ring + st * kStageBytes, &hmap, &full[st], g * kSWords, q * kSCh);
                bulk_g2s(xring + st * 32, x + (int64_t)q * kSCh, 32u, &full[st]);
            }
            if (!ok) {
                /* let the copies already issued land before the CTA exits */
                for (int64_t j = i > kSStages ? i - kSStages : 0; j < i; ++j)
                    if (!mbar_wait_bounded(&full[(int)(j % kSStages)], (uint32_t)(j / kSStages) & 1u, &g_km_error))
                        break;
            }
        }
        return;
    }
    /* ---- consumers: thread t of a half owns rows 8 t .. 8 t + 7 of the current row
     * group; half h takes channels 8 h .. 8 h + 7 of every stage */
    const int h = warp >> 3, t = (int)threadIdx.x & 255;
    const uint32_t pbase = smem_u32(pairs), lane8 = (uint32_t)lane * 8u;
    uint64_t acc[4], y2[4]; /* row pairs (2q, 2q+1) */
#pragma unroll
    for (int q = 0; q < 4; ++q)
        acc[q] = 0ull, y2[q] = 0ull;
    uint64_t sc[4] = {0ull, 0ull, 0ull, 0ull};
    int gcur = -1, bcur = -1, slot = -1;
    auto flush_block = [&]() {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            fma2(y2[q], sc[q], acc[q]);
            acc[q] = 0ull;
        }
    };
    auto write_group = [&]() {
        /* each half writes its own partial of the rows; the combine adds them */
        const float2 a0 = f2unpack(y2[0]), a1 = f2unpack(y2[1]), a2 = f2unpack(y2[2]), a3 = f2unpack(y2[3]);
        float4 *o = reinterpret_cast<float4 *>(part + (((int64_t)p * 2 + slot) * 2 + h) * kSRows + 8 * t);
        o[0] = make_float4(a0.x, a0.y, a1.x, a1.y);
        o[1] = make_float4(a2.x, a2.y, a3.x, a3.y);
#pragma unroll
        for (int q = 0; q < 4; ++q)
            y2[q] = 0ull;
    };
    const int nw = a.n / 8;
    int64_t i = 0;
    bool alive = true;
    for (int64_t u = ub; u < ue; ++u, ++i) {
        const int g = (int)(u / a.QK), q = (int)(u - (int64_t)g * a.QK);
        const int wi = g * kSWords + t;
        if (g != gcur) {
            if (gcur >= 0) {
                flush_block();
                write_group();
            }
            gcur = g, bcur = -1, ++slot;
        }
        if ((q >> 2) != bcur) {
            if (bcur >= 0)
                flush_block();
            bcur = q >> 2;
            if (wi < nw) { /* used at the block's end, four stages later */
                const float *sp = sk + (int64_t)bcur * a.n + 8 * wi;
                const float4 s0 = __ldg(reinterpret_cast<const float4 *>(sp));
                const float4 s1 = __ldg(reinterpret_cast<const float4 *>(sp + 4));
                sc[0] = f2pack(s0.x, s0.y), sc[1] = f2pack(s0.z, s0.w);
                sc[2] = f2pack(s1.x, s1.y), sc[3] = f2pack(s1.z, s1.w);
            }
        }
        const int st = (int)(i % kSStages);
        const uint32_t ph = (uint32_t)(i / kSStages) & 1u;
        bool ok = lane == 0 ? mbar_wait_suspend_bounded(&full[st], ph, &g_km_error) : true;
        ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
        if (!ok) {
            alive = false;
            break;
        }
        const uint32_t sw = smem_u32(ring + st * kStageBytes) + (uint32_t)(h * 8 * kSegBytes) + (uint32_t)t * 4u;
        const uint4 xw = *reinterpret_cast<const uint4 *>(xring + st * 32 + h * 16); /* 8 BF16 x values */
        const uint32_t xs[4] = {xw.x, xw.y, xw.z, xw.w};
        uint32_t w[8];
#pragma unroll
        for (int ch = 0; ch < 8; ++ch)
            w[ch] = lds32(sw + ch * kSegBytes);
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
            const float xv = __uint_as_float(ch & 1 ? (xs[ch >> 1] & 0xFFFF0000u) : (xs[ch >> 1] << 16));
            const uint64_t xx = f2pack(xv, xv);
#pragma unroll
            for (int qq = 0; qq < 4; ++qq)
                fma2(acc[qq], lds64u(pbase + __byte_perm(w[ch], lane8, 0x5504u | (qq << 4))), xx);
        }
        __syncwarp();
        if (lane == 0)
            mbar_arrive(&empty[st]);
    }
    if (gcur >= 0 && alive) {
        flush_block();
        write_group();
    }
}

/* ---- channel selection ------------------------------------------------------- */
constexpr int kSelThreads = 256; /* small enough to share an SM with the parent GEMV */

/* exclusive prefix sum of v over the block's threads in thread order; the block's
 * total goes to *total (every thread calls it) */
__device__ __forceinline__ int block_excl_scan(int v, int *wsum, int *total)
{
    const int lane = (int)(threadIdx.x & 31), warp = (int)(threadIdx.x >> 5);
    int s = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xFFFFFFFFu, s, o);
        if (lane >= o)
            s += t;
    }
    if (lane == 31)
        wsum[warp] = s;
    __syncthreads();
    constexpr int kWarps = kSelThreads / 32;
    if (warp == 0) {
        int ws = lane < kWarps ? wsum[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xFFFFFFFFu, ws, o);
            if (lane >= o)
                ws += t;
        }
        if (lane < kWarps)
            wsum[lane] = ws; /* inclusive over warps */
    }
    __syncthreads();
    const int before = (warp ? wsum[warp - 1] : 0) + s - v;
    *total = wsum[kWarps - 1];
    __syncthreads();
    return before;
}

/* the largest bin index B (of nb, counts hist[]) with sum_{b >= B} hist[b] + base >= need,
 * or -1; run by warp 0 (bins per lane = nb / 32) */
__device__ __forceinline__ int top_bin(const int *hist, int nb, int base, int need, int lane)
{
    const int per = nb / 32;
    /* lane l owns bins [nb - per*(l+1), nb - per*l): lane 0 the top ones */
    int local = 0;
    for (int j = 0; j < per; ++j)
        local += hist[nb - per * (lane + 1) + j];
    int s = local; /* inclusive prefix from the top */
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xFFFFFFFFu, s, o);
        if (lane >= o)
            s += t;
    }
    const bool reach = base + s >= need, prev = base + s - local >= need;
    const unsigned m = __ballot_sync(0xFFFFFFFFu, reach && !prev);
    if (!m)
        return -1;
    const int l = __ffs((int)m) - 1;
    int acc = base + __shfl_sync(0xFFFFFFFFu, s - local, l);
    int found = -1;
    if (lane == l) {
        for (int b = nb - per * l - 1; b >= nb - per * (l + 1); --b) {
            acc += hist[b];
            if (acc >= need) {
                found = b;
                break;
            }
        }
    }
    return __shfl_sync(0xFFFFFFFFu, found, l);
}

__global__ void __launch_bounds__(kSelThreads) select_topk_kernel(const uint16_t *__restrict__ x, int K, int nsel,
                                                                  int *__restrict__ idx, int *__restrict__ cnt)
{
    extern __shared__ __align__(16) uint8_t smem[];
    uint16_t *keys = reinterpret_cast<uint16_t *>(smem);
    __shared__ int hist[256];
    __shared__ int wsum[32];
    __shared__ int s_thr, s_above;
    const int t = (int)threadIdx.x, lane = t & 31;
    for (int i = t; i < K; i += kSelThreads)
        keys[i] = (uint16_t)(x[i] & 0x7FFFu);
    for (int i = t; i < 256; i += kSelThreads)
        hist[i] = 0;
    __syncthreads();
    if (nsel == 0 || nsel > K) {
        /* nothing selected, or every channel (fewer channels than asked for) */
        if (t == 0)
            s_thr = nsel == 0 ? 32768 : 0;
    } else {
        for (int i = t; i < K; i += kSelThreads)
            atomicAdd(&hist[keys[i] >> 7], 1);
        __syncthreads();
        if (t < 32) {
            const int B = top_bin(hist, 256, 0, nsel, lane);
            /* keys in buckets above B */
            int above = 0;
            for (int b = B + 1 + lane; b < 256; b += 32)
                above += hist[b];
            above = __reduce_add_sync(0xFFFFFFFFu, above);
            if (lane == 0)
                s_thr = B, s_above = above;
        }
        __syncthreads();
        const int B = s_thr;
        for (int i = t; i < 128; i += kSelThreads)
            hist[i] = 0;
        __syncthreads();
        for (int i = t; i < K; i += kSelThreads)
            if ((keys[i] >> 7) == B)
                atomicAdd(&hist[keys[i] & 127], 1);
        __syncthreads();
        if (t < 32) {
            const int L = top_bin(hist, 128, s_above, nsel, lane);
            if (lane == 0)
                s_thr = B * 128 + L;
        }
    }
    __syncthreads();
    const int T = s_thr;
    /* ascending compaction over contiguous chunks */
    const int per = (K + kSelThreads - 1) / kSelThreads;
    const int lo = min(K, t * per), hi = min(K, lo + per);
    int mine = 0;
    for (int i = lo; i < hi; ++i)
        mine += keys[i] >= T;
    int total = 0;
    int pos = block_excl_scan(mine, wsum, &total);
    for (int i = lo; i < hi; ++i)
        if (keys[i] >= T)
            idx[pos++] = i;
    if (t == 0)
        *cnt = total;
}

/* ---- plug correction ---------------------------------------------------------- */

/* part[sl][r] = sum over list entries [(sl*8 + warp)*8, +8) of this
 * CTA's warps (in order) of (delta[h][p] * scale) * x[c], for every slice this CTA
 * walks.  Two load rounds per warp: the chunk's channel numbers, then every entry's
 * hole word, plug word and scales. */
__global__ void __launch_bounds__(kCorrThreads) apply_corr_kernel(const uint32_t *__restrict__ hole_k,
                                                                  const uint32_t *plug_k,
                                                                  const float *__restrict__ sk,
                                                                  const __nv_bfloat16 *__restrict__ x,
                                                                  const int *__restrict__ idx,
                                                                  const int *__restrict__ cnt_p,
                                                                  float *__restrict__ part, int n)
{
    __shared__ float dl[256]; /* CELLS - PARENT by code h*16 + p */
    __shared__ __align__(16) float red[8 * 256];
    const int cnt = *cnt_p;
    if ((int)blockIdx.y * 8 * kCorrChunk >= cnt)
        return; /* no slice of the list for this CTA: the combine reads none */
    const int lane = (int)(threadIdx.x & 31), warp = (int)(threadIdx.x >> 5);
    const int nw = n / 8;
    const int wi = (int)blockIdx.x * 32 + lane;
    for (int e = threadIdx.x; e < 256; e += kCorrThreads)
        dl[e] = g_cells[e >> 4][e & 15] - g_parent[e >> 4];
    /* slices blockIdx.y, blockIdx.y + gridDim.y, ... of 64 list entries while the list lasts */
    for (int sl = (int)blockIdx.y; sl * 8 * kCorrChunk < cnt; sl += (int)gridDim.y) {
        const int i0 = sl * 8 * kCorrChunk + warp * kCorrChunk;
        const int m = max(0, min(kCorrChunk, cnt - i0)); /* this warp's entries */
        const bool live = wi < nw && m > 0;
        int c[kCorrChunk];
        uint32_t wh[kCorrChunk], wp[kCorrChunk];
        float4 s0[kCorrChunk], s1[kCorrChunk];
        float xv[kCorrChunk];
        if (live) {
#pragma unroll
            for (int u = 0; u < kCorrChunk; ++u)
                c[u] = u < m ? idx[i0 + u] : 0;
#pragma unroll
            for (int u = 0; u < kCorrChunk; ++u) {
                if (u < m) {
                    wh[u] = hole_k[(int64_t)c[u] * nw + wi];
                    wp[u] = plug_k[(int64_t)c[u] * nw + wi];
                    const float *sp = sk + (int64_t)(c[u] >> 6) * n + 8 * wi;
                    s0[u] = __ldg(reinterpret_cast<const float4 *>(sp));
                    s1[u] = __ldg(reinterpret_cast<const float4 *>(sp + 4));
                    xv[u] = __bfloat162float(x[c[u]]);
                }
            }
        }
        __syncthreads(); /* dl filled; red free from the previous slice */
        float acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
            acc[j] = 0.f;
        if (live) {
#pragma unroll
            for (int u = 0; u < kCorrChunk; ++u) {
                if (u < m) {
                    const float sv[8] = {s0[u].x, s0[u].y, s0[u].z, s0[u].w, s1[u].x, s1[u].y, s1[u].z, s1[u].w};
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const uint32_t code = (((wh[u] >> (4 * j)) & 15u) << 4) | ((wp[u] >> (4 * j)) & 15u);
                        acc[j] = fmaf(dl[code] * sv[j], xv[u], acc[j]);
                    }
                }
            }
        }
        float4 *rw = reinterpret_cast<float4 *>(red + warp * 256 + lane * 8);
        rw[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        rw[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
        __syncthreads();
        const int row = (int)blockIdx.x * 256 + (int)threadIdx.x;
        if (row < n) {
            float v = red[threadIdx.x];
#pragma unroll
            for (int u = 1; u < 8; ++u)
                v += red[u * 256 + threadIdx.x];
            part[(int64_t)sl * n + row] = v;
        }
    }
}

/* The closing sums of a decode step.  For each row r:
 *   g = the GEMV partials of r, added in their fixed order: the slices [s][n]
 *       (gmode 1), or the partials of the CTAs that covered r's row group, in CTA
 *       order (gmode 2); gmode 0 takes y[r] as it is;
 *   y[r] = g + (sum of the first ceil(cnt / 64) correction slices, in order), or g.
 * A CTA takes 32 rows (one per lane) and its 8 warps take every 8th partial, so
 * each row's loads are in flight together; the warps' sums are added in warp order,
 * so the result does not depend on timing. */
struct Combine {
    const float *g;
    int gmode, S;
    KmStream a;
    const float *c;
    const int *cnt;
    float *y;
    int n;
};

__device__ __forceinline__ float ordered_warp_sums(float v, float (*red)[32], int warp, int lane)
{
    red[warp][lane] = v;
    __syncthreads();
    float s = red[0][lane];
#pragma unroll
    for (int w = 1; w < 8; ++w)
        s += red[w][lane];
    __syncthreads();
    return s;
}

__global__ void __launch_bounds__(256) km_combine_kernel(const Combine cb)
{
    __shared__ float red[8][32];
    const int warp = (int)(threadIdx.x >> 5), lane = (int)(threadIdx.x & 31);
    const int r = (int)blockIdx.x * 32 + lane;
    const bool live = r < cb.n;
    float v = 0.f;
    if (cb.gmode == 1) {
        float a = 0.f;
#pragma unroll 4
        for (int q = warp; q < cb.S; q += 8)
            a += live ? cb.g[(int64_t)q * cb.n + r] : 0.f;
        v = ordered_warp_sums(a, red, warp, lane);
    } else if (cb.gmode == 2) {
        const int g = (int)blockIdx.x * 32 / kSRows, lr = (int)blockIdx.x * 32 - g * kSRows + lane;
        const int64_t u0 = (int64_t)g * cb.a.QK, u1 = u0 + cb.a.QK - 1;
        const int pf = (int)(((u0 + 1) * cb.a.P - 1) / cb.a.U), pl = (int)(((u1 + 1) * cb.a.P - 1) / cb.a.U);
        float a = 0.f;
#pragma unroll 4
        for (int q = pf + warp; q <= pl; q += 8) {
            const int slot = km_unit_begin(cb.a, q) / cb.a.QK == g ? 0 : 1;
            const float *pp = cb.g + ((int64_t)q * 2 + slot) * 2 * kSRows + lr;
            a += live ? pp[0] + pp[kSRows] : 0.f; /* the CTA's two halves */
        }
        v = ordered_warp_sums(a, red, warp, lane);
    } else {
        v = live ? cb.y[r] : 0.f;
    }
    if (cb.c) {
        const int cs = (*cb.cnt + 8 * kCorrChunk - 1) / (8 * kCorrChunk);
        if (cs > 0) {
            float a = 0.f;
#pragma unroll 4
            for (int q = warp; q < cs; q += 8)
                a += live ? cb.c[(int64_t)q * cb.n + r] : 0.f;
            v = v + ordered_warp_sums(a, red, warp, lane);
        }
    }
    if (live && warp == 0)
        cb.y[r] = v;
}

/* ---- host side ------------------------------------------------------------------ */
struct KmScratch {
    float *buf = nullptr;
    size_t floats = 0;
};
std::mutex g_km_mu;
std::unordered_map<uint64_t, KmScratch> g_km_scratch;

/* A side stream and two events per (device, stream): the channel selection runs
 * beside the parent GEMV (it needs only x), joined before the correction.  Event
 * records and waits are captured into CUDA graphs as a parallel branch. */
struct KmFork {
    cudaStream_t side = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr;
};
std::unordered_map<uint64_t, KmFork> g_km_fork;

bool km_fork(cudaStream_t st, KmFork *out)
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess)
        return false;
    const uint64_t key = (reinterpret_cast<uint64_t>(st) << 8) ^ (uint64_t)dev;
    std::lock_guard<std::mutex> lk(g_km_mu);
    KmFork &f = g_km_fork[key];
    if (!f.side) {
        if (cudaStreamCreateWithFlags(&f.side, cudaStreamNonBlocking) != cudaSuccess ||
            cudaEventCreateWithFlags(&f.fork, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&f.join, cudaEventDisableTiming) != cudaSuccess) {
            cudaGetLastError();
            f = KmFork{};
            return false;
        }
    }
    *out = f;
    return true;
}

float *km_scratch(cudaStream_t st, size_t floats)
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess)
        return nullptr;
    const uint64_t key = (reinterpret_cast<uint64_t>(st) << 8) ^ (uint64_t)dev;
    std::lock_guard<std::mutex> lk(g_km_mu);
    KmScratch &S = g_km_scratch[key];
    if (S.floats < floats) {
        if (S.buf)
            cudaFree(S.buf);
        S.buf = nullptr, S.floats = 0;
        if (cudaMalloc(&S.buf, floats * sizeof(float)) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        S.floats = floats;
    }
    return S.buf;
}

/* channel slices of the parent GEMV: about 4 CTAs per SM in one wave, at least two
 * 64-blocks per CTA (fewer partial sums to add) */
void km_split(int n, int K, int *slices, int *bps)
{
    const int KB = K / 64, rg = (n + kKmRows - 1) / kKmRows;
    const int target = 4 * sm_count();
    int s = std::max(1, (target + rg - 1) / rg);
    s = std::min(s, std::max(1, KB / 2));
    s = std::max(s, (KB + kMaxBps - 1) / kMaxBps); /* x of a slice fits its shared-memory area */
    *bps = (KB + s - 1) / s;
    *slices = (KB + *bps - 1) / *bps;
}

int km_smem(int bps) { return bps * 64 * 4; }
/* the kernels' dynamic shared memory limits are raised once, to the largest size
 * any call needs */
bool km_smem_limits()
{
    return ensure_smem((const void *)gemv_km_kernel, km_smem(kMaxBps)) &&
           ensure_smem((const void *)select_topk_kernel, kKmMaxK * 2);
}

int corr_slices(int K) { return (K + 8 * kCorrChunk - 1) / (8 * kCorrChunk); }

int combine(const float *g, int gmode, int S, const KmStream *a, const float *c, const int *cnt, float *y, int n,
            cudaStream_t st)
{
    Combine cb{};
    cb.g = g, cb.gmode = gmode, cb.S = S, cb.c = c, cb.cnt = cnt, cb.y = y, cb.n = n;
    if (a)
        cb.a = *a;
    km_combine_kernel<<<(n + 31) / 32, 256, 0, st>>>(cb);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunch;
}

} // namespace

bool km_supported(int n, int K, const void *hole_k, const void *scales_k)
{
    return n >= 8 && n % 8 == 0 && K >= 64 && K % 64 == 0 && K <= kKmMaxK && aligned_to(hole_k, 16) &&
           aligned_to(scales_k, 16);
}

int km_layout_launch(const uint8_t *hole, const uint8_t *plug, const float *am, int n, int K, uint8_t *hole_k,
                     uint8_t *plug_k, float *scales_k, cudaStream_t st)
{
    const dim3 g((K + kTC - 1) / kTC, (n + kTR - 1) / kTR, plug_k ? 2 : 1);
    kmajor_planes_kernel<<<g, 256, 0, st>>>(hole, plug, hole_k, plug_k, n, K);
    const int KB = K / 64;
    kmajor_scales_kernel<<<dim3((KB + 31) / 32, (n + 31) / 32), 256, 0, st>>>(am, scales_k, n, KB);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunch;
}

namespace {
/* the streamed kernel's split, or false when it does not apply (then the per-slice
 * kernel runs): n % 32 (16-byte channel segments), a 16-byte aligned x, and every
 * CTA's units within two row groups */
bool km_stream_split(int n, int K, const void *x, KmStream *a)
{
    if (n % 32 || !aligned_to(x, 16))
        return false;
    a->n = n, a->K = K, a->QK = K / kSCh;
    const int G = (n + kSRows - 1) / kSRows;
    a->U = (int64_t)G * a->QK;
    a->P = (int)std::min<int64_t>(sm_count(), a->U);
    return (a->U + a->P - 1) / a->P <= a->QK;
}

int km_stream_launch(const uint8_t *hole_k, const float *sk, const __nv_bfloat16 *x, const KmStream &a,
                     float *part, cudaStream_t st)
{
    /* the hole plane as uint32 words [K channels][n/8]: boxes of 256 words x 16 channels */
    auto enc = tensor_map_encoder();
    CUtensorMap hmap;
    cuuint64_t dims[2] = {(cuuint64_t)(a.n / 8), (cuuint64_t)a.K};
    cuuint64_t strides[1] = {(cuuint64_t)(a.n / 2)};
    cuuint32_t box[2] = {(cuuint32_t)kSWords, (cuuint32_t)kSCh};
    cuuint32_t estr[2] = {1, 1};
    if (!enc || enc(&hmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint8_t *>(hole_k), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return kLaunch;
    if (!ensure_smem((const void *)gemv_km_stream_kernel, kSSmem))
        return kLaunch;
    gemv_km_stream_kernel<<<a.P, kSThreads, kSSmem, st>>>(hmap, sk, x, part, a);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunch;
}

size_t km_stream_part_floats(const KmStream &a) { return (size_t)a.P * 2 * 2 * kSRows; }

int gemv_km_parts(const uint8_t *hole_k, const float *sk, const __nv_bfloat16 *x, float *y, int n, int K,
                  cudaStream_t st, float **gpart, int *slices)
{
    int s = 1, bps = 1;
    km_split(n, K, &s, &bps);
    const int smem = km_smem(bps);
    if (!km_smem_limits())
        return kLaunch;
    /* the kernel stores 16-byte vectors: an unaligned y is written by the combine */
    const bool direct = s == 1 && aligned_to(y, 16);
    float *out = y;
    if (!direct) {
        out = km_scratch(st, (size_t)s * n + (size_t)corr_slices(K) * n);
        if (!out)
            return kLaunch;
    }
    gemv_km_kernel<<<dim3((n + kKmRows - 1) / kKmRows, s), kKmThreads, smem, st>>>(
        reinterpret_cast<const uint32_t *>(hole_k), sk, x, out, n, K, bps);
    *gpart = direct ? nullptr : out;
    *slices = s;
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunch;
}
} // namespace

int km_gemv_launch(const uint8_t *hole_k, const float *sk, const __nv_bfloat16 *x, float *y, int n, int K,
                   cudaStream_t st)
{
    KmStream a;
    if (km_stream_split(n, K, x, &a)) {
        float *part = km_scratch(st, km_stream_part_floats(a) + (size_t)corr_slices(K) * n);
        if (!part)
            return kLaunch;
        const int rc = km_stream_launch(hole_k, sk, x, a, part, st);
        if (rc != kOk)
            return rc;
        return combine(part, 2, 0, &a, nullptr, nullptr, y, n, st);
    }
    float *gpart = nullptr;
    int s = 1;
    const int rc = gemv_km_parts(hole_k, sk, x, y, n, K, st, &gpart, &s);
    if (rc != kOk || !gpart)
        return rc;
    return combine(gpart, 1, s, nullptr, nullptr, nullptr, y, n, st);
}

int km_select_launch(const __nv_bfloat16 *x, int K, int nsel, int *idx, int *cnt, cudaStream_t st)
{
    const int smem = ((K * 2 + 15) / 16) * 16;
    if (!km_smem_limits())
        return kLaunch;
    select_topk_kernel<<<1, kSelThreads, std::max(smem, 16), st>>>(reinterpret_cast<const uint16_t *>(x), K, nsel,
                                                                    idx, cnt);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunch;
}

namespace {
int corr_parts(const uint8_t *hole_k, const uint8_t *plug_k, const float *sk, const __nv_bfloat16 *x,
               const int *idx, const int *cnt, int n, int K, float *cpart, cudaStream_t st)
{
    /* a small fixed grid whose CTAs walk the list's slices (the count is on the device) */
    const int rg = (n + 255) / 256;
    const int ys = std::min(corr_slices(K), std::max(1, 2 * sm_count() / rg));
    apply_corr_kernel<<<dim3(rg, ys), kCorrThreads, 0, st>>>(
        reinterpret_cast<const uint32_t *>(hole_k), reinterpret_cast<const uint32_t *>(plug_k), sk, x, idx, cnt,
        cpart, n);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunch;
}
} // namespace

int km_corr_launch(const uint8_t *hole_k, const uint8_t *plug_k, const float *sk, const __nv_bfloat16 *x,
                   const int *idx, const int *cnt, float *y, int n, int K, cudaStream_t st)
{
    float *cpart = km_scratch(st, (size_t)corr_slices(K) * n);
    if (!cpart)
        return kLaunch;
    const int rc = corr_parts(hole_k, plug_k, sk, x, idx, cnt, n, K, cpart, st);
    if (rc != kOk)
        return rc;
    return combine(nullptr, 0, 0, nullptr, cpart, cnt, y, n, st);
}

int km_gemv_select_launch(const uint8_t *hole_k, const uint8_t *plug_k, const float *sk, const __nv_bfloat16 *x,
                          float *y, int n, int K, int nsel, int *idx, int *cnt, cudaStream_t st)
{
    KmStream a;
    if (km_stream_split(n, K, x, &a)) {
        const size_t pf = km_stream_part_floats(a);
        float *part = km_scratch(st, pf + (size_t)corr_slices(K) * n);
        KmFork f;
        if (!part || !km_fork(st, &f))
            return kLaunch;
        /* selection on the side stream, beside the parent GEMV */
        if (cudaEventRecord(f.fork, st) != cudaSuccess || cudaStreamWaitEvent(f.side, f.fork, 0) != cudaSuccess)
            return kLaunch;
        int rc = km_select_launch(x, K, nsel, idx, cnt, f.side);
        if (rc != kOk || cudaEventRecord(f.join, f.side) != cudaSuccess)
            return rc != kOk ? rc : kLaunch;
        if ((rc = km_stream_launch(hole_k, sk, x, a, part, st)) != kOk)
            return rc;
        if (cudaStreamWaitEvent(st, f.join, 0) != cudaSuccess)
            return kLaunch;
        if ((rc = corr_parts(hole_k, plug_k, sk, x, idx, cnt, n, K, part + pf, st)) != kOk)
            return rc;
        return combine(part, 2, 0, &a, part + pf, cnt, y, n, st);
    }
    int rc = km_select_launch(x, K, nsel, idx, cnt, st);
    if (rc != kOk)
        return rc;
    int s = 1, bps = 1;
    km_split(n, K, &s, &bps);
    /* scratch: [s][n] GEMV slices (when s > 1), then the correction slices */
    float *base = km_scratch(st, (size_t)(s + corr_slices(K)) * n);
    if (!base)
        return kLaunch;
    const int smem = km_smem(bps);
    if (!km_smem_limits())
        return kLaunch;
    const bool direct = s == 1 && aligned_to(y, 16);
    float *gout = direct ? y : base;
    gemv_km_kernel<<<dim3((n + kKmRows - 1) / kKmRows, s), kKmThreads, smem, st>>>(
        reinterpret_cast<const uint32_t *>(hole_k), sk, x, gout, n, K, bps);
    float *cpart = base + (size_t)s * n;
    rc = corr_parts(hole_k, plug_k, sk, x, idx, cnt, n, K, cpart, st);
    if (rc != kOk)
        return rc;
    return combine(direct ? nullptr : base, direct ? 0 : 1, s, nullptr, cpart, cnt, y, n, st);
}

int km_error_word(bool clear) { return read_error_word(g_km_error, g_km_error_taken, clear); }

} // namespace glint
