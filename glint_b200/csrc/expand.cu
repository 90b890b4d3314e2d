/* GLINT expand for sm_100a: hole/plug planes + absmax -> dense BF16 or f32.
 *
 * Reference behaviour: cuda/glint_encode.cu:103-114 (k_expand, f32 out) and
 * glint_unpin._expand / glint_np.expand + f32_to_bf16_bytes (glint_unpin.py:25-31,
 * glint_np.py:25-31, 84-92): out = GLINT_CELLS[h][p] * absmax[i / bs] as one f32
 * multiply, then for BF16 a round to nearest even with the NaN rule
 * (u >> 16) | 0x40.
 *
 * One persistent CTA per SM: 16 consumer warps and a producer warp that streams
 * each unit of 16384 weights (8 KB of each plane and the unit's absmax) into a
 * 6-slot shared-memory ring with cp.async.bulk, and publishes a small descriptor
 * of the unit (pointers, valid count) beside it.  A consumer lane expands four
 * groups of 8 weights per unit, one 16-byte BF16 store each (512 contiguous
 * bytes per warp store).  The 256-entry f32 codebook sits in shared memory with
 * one replica per lane at a 256-byte entry stride, so each lookup address is one
 * byte permute; the scale multiply runs two weights per f32x2 instruction.
 * Blocksizes that are not a power of two in [8, 1024] and unaligned outputs go
 * through a one-thread-per-weight kernel; ragged last units and unaligned planes
 * are read straight from global memory.
 *
 * NaN absmax: the reference's host expand multiplies on x86, which returns the
 * NaN operand (quietened) unchanged, so the product carries absmax's bits.  The
 * GPU multiply would return its canonical NaN instead; both outputs are
 * produced from absmax's bits here to match the host reference bit for bit.
 */
#include <algorithm>

#include "common.cuh"
#include "glint_internal.h"
#include "ptx.cuh"

namespace glint {

__device__ int g_expand_error = 0;
__device__ int g_expand_error_taken = 0; /* read_error_word's result slot */

namespace {

constexpr int kMaxItems = 32;
constexpr int kConsumerWarps = 16;
constexpr int kGroups = 4;                               /* 8-weight groups per lane per unit */
constexpr int kUnitW = kConsumerWarps * 32 * 8 * kGroups; /* 16384 weights per ring slot */
constexpr int kPlaneBytes = kUnitW / 2;                  /* 8 KB of each plane per unit */
constexpr int kAmMax = kUnitW / 8 * 4;                   /* absmax bytes of a unit at bs = 8 */
constexpr int kSlotBytes = 2 * kPlaneBytes + kAmMax;
constexpr int kSlots = 6;
constexpr int kExpThreads = (kConsumerWarps + 1) * 32;
/* f32 codebook, one replica per lane, entry stride 256 B: a lookup address is one
 * byte permute, (code << 8) | (lane << 2) */
constexpr int kLutBytes = 256 * 256;
constexpr int kMetaBytes = 48;
constexpr int kExpSmem = kLutBytes + kSlots * kSlotBytes + kSlots * kMetaBytes + 2 * 8 * kSlots + 128;

struct ExpandBatch {
    const uint8_t *hole[kMaxItems];
    const uint8_t *plug[kMaxItems];
    const float *absmax[kMaxItems];
    void *out[kMaxItems];
    int64_t n[kMaxItems];
    int64_t unit_end[kMaxItems]; /* inclusive prefix sum of ceil(n / kUnitW) */
    uint32_t direct;             /* bit i: item i's planes are read straight from global */
    int count;
    int bs_log2;
};

/* The producer's description of the unit in a slot (pointers offset to the unit). */
struct UnitMeta {
    const uint8_t *hole;
    const uint8_t *plug;
    const float *absmax;
    void *out;
    int valid;  /* weights in the unit */
    int staged; /* planes and absmax sit in the slot */
    int pad[2];
};
static_assert(sizeof(UnitMeta) == kMetaBytes, "slot descriptor layout");

__device__ __forceinline__ float quiet_nan_of(float s) { return __uint_as_float(__float_as_uint(s) | 0x00400000u); }

__device__ __forceinline__ uint64_t pack2f(float lo, float hi)
{
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void unpack2f(uint64_t v, float &lo, float &hi) { asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v)); }
__device__ __forceinline__ uint64_t mul2f(uint64_t a, uint64_t b)
{
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

/* values of the 8 weights whose nibbles are in H and P (lo nibble first), one f32
 * multiply each, two per instruction */
__device__ __forceinline__ void dequant8(uint32_t lut_base, uint32_t lane4, uint32_t H, uint32_t P, float s, float v[8])
{
    /* byte b of E holds the code of element 2b, byte b of O the code of element 2b+1 */
    const uint32_t E = ((H << 4) & 0xF0F0F0F0u) | (P & 0x0F0F0F0Fu);
    const uint32_t O = (H & 0xF0F0F0F0u) | ((P >> 4) & 0x0F0F0F0Fu);
    const uint64_t s2 = pack2f(s, s);
#pragma unroll
    for (int b = 0; b < 4; ++b) {
        const float c0 = __uint_as_float(lds32(lut_base + __byte_perm(E, lane4, 0x5504 | (b << 4))));
        const float c1 = __uint_as_float(lds32(lut_base + __byte_perm(O, lane4, 0x5504 | (b << 4))));
        unpack2f(mul2f(pack2f(c0, c1), s2), v[2 * b], v[2 * b + 1]);
    }
}

template <bool BF16>
__global__ void __launch_bounds__(kExpThreads, 1) expand_stream_kernel(const __grid_constant__ ExpandBatch b)
{
    extern __shared__ __align__(128) uint8_t smem[];
    float *lut = reinterpret_cast<float *>(smem);
    uint8_t *ring = smem + kLutBytes;
    UnitMeta *meta = reinterpret_cast<UnitMeta *>(ring + kSlots * kSlotBytes);
    uint64_t *full = reinterpret_cast<uint64_t *>(meta + kSlots);
    uint64_t *empty = full + kSlots;

    /* 32 replicas per entry in the first 128 B of its 256-B row; a 16-byte store
     * covers a quarter row, so each warp store fills four whole rows (no bank
     * conflicts) */
    for (int i = (int)threadIdx.x; i < 256 * 8; i += kExpThreads) {
        const float c = (&g_cells[0][0])[i >> 3];
        reinterpret_cast<float4 *>(lut + (i >> 3) * 64)[i & 7] = make_float4(c, c, c, c);
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < kSlots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        mbar_init_fence();
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5;
    const uint32_t lane = lane_id();
    const int64_t total = b.unit_end[b.count - 1];
    const int L2 = b.bs_log2;

    if (warp == kConsumerWarps) {
        if (lane == 0) {
            int it = 0;
            int64_t i = 0;
            bool ok = true;
            for (int64_t u = blockIdx.x; u < total; u += gridDim.x, ++i) {
                const int s = (int)(i % kSlots);
                const uint32_t ph = (uint32_t)(i / kSlots) & 1u;
                if (i >= kSlots && !(ok = mbar_wait_bounded(&empty[s], ph ^ 1u, &g_expand_error)))
                    break;
                while (b.unit_end[it] <= u)
                    ++it;
                const int64_t off = (u - (it ? b.unit_end[it - 1] : 0)) * kUnitW;
                const int64_t left = b.n[it] - off;
                const bool staged = left >= kUnitW && !((b.direct >> it) & 1u);
                UnitMeta &m = meta[s];
                m.hole = b.hole[it] + off / 2;
                m.plug = b.plug[it] + off / 2;
                m.absmax = b.absmax[it] + (off >> L2);
                m.out = static_cast<char *>(b.out[it]) + off * (BF16 ? 2 : 4);
                m.valid = left >= kUnitW ? kUnitW : (int)left;
                m.staged = staged ? 1 : 0;
                if (staged) {
                    const uint32_t am_bytes = (uint32_t)(kUnitW >> L2) * 4u;
                    mbar_expect_tx(&full[s], 2 * kPlaneBytes + am_bytes);
                    bulk_g2s(ring + s * kSlotBytes, m.hole, kPlaneBytes, &full[s]);
                    bulk_g2s(ring + s * kSlotBytes + kPlaneBytes, m.plug, kPlaneBytes, &full[s]);
                    bulk_g2s(ring + s * kSlotBytes + 2 * kPlaneBytes, m.absmax, am_bytes, &full[s]);
                } else {
                    mbar_arrive(&full[s]);
                }
            }
            if (!ok) {
                const int64_t issued = i;
                for (int64_t j = issued > kSlots ? issued - kSlots : 0; j < issued; ++j)
                    if (!mbar_wait_bounded(&full[(int)(j % kSlots)], (uint32_t)(j / kSlots) & 1u, &g_expand_error))
                        break;
            }
        }
        return;
    }

    const uint32_t lut_base = saddr(lut), lane4 = lane * 4u;
    int64_t i = 0;
    for (int64_t u = blockIdx.x; u < total; u += gridDim.x, ++i) {
        const int s = (int)(i % kSlots);
        const uint32_t ph = (uint32_t)(i / kSlots) & 1u;
        const bool ok = lane == 0 ? mbar_wait_bounded(&full[s], ph, &g_expand_error) : true;
        if (!__shfl_sync(0xFFFFFFFFu, ok ? 1 : 0, 0))
            break;
        const UnitMeta m = meta[s];
        const uint32_t slot = saddr(ring + s * kSlotBytes);
        uint32_t H[kGroups], P[kGroups];
        float S[kGroups];
        int valid[kGroups], rel[kGroups];
#pragma unroll
        for (int grp = 0; grp < kGroups; ++grp) {
            rel[grp] = warp * (32 * 8 * kGroups) + grp * 256 + (int)lane * 8;
            const int left = m.valid - rel[grp];
            valid[grp] = left >= 8 ? 8 : (left > 0 ? left : 0);
            if (m.staged) {
                H[grp] = lds32(slot + rel[grp] / 2);
                P[grp] = lds32(slot + kPlaneBytes + rel[grp] / 2);
                S[grp] = __uint_as_float(lds32(slot + 2 * kPlaneBytes + (uint32_t)(rel[grp] >> L2) * 4u));
            } else {
                H[grp] = P[grp] = 0;
                S[grp] = 0.f;
                for (int bb = 0; bb < (valid[grp] + 1) / 2; ++bb) {
                    H[grp] |= (uint32_t)m.hole[rel[grp] / 2 + bb] << (8 * bb);
                    P[grp] |= (uint32_t)m.plug[rel[grp] / 2 + bb] << (8 * bb);
                }
                if (valid[grp] > 0)
                    S[grp] = __ldg(m.absmax + (rel[grp] >> L2));
            }
        }
        __syncwarp();
        if (lane == 0)
            mbar_arrive(&empty[s]); /* the slot's data now lives in registers */
#pragma unroll
        for (int grp = 0; grp < kGroups; ++grp) {
            if (valid[grp] == 0)
                continue;
            float v[8];
            dequant8(lut_base, lane4, H[grp], P[grp], S[grp], v);
            const bool nan_scale = isnan(S[grp]);
            if (BF16) {
                uint32_t o[4];
                if (!nan_scale) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        __nv_bfloat162 h2 = __floats2bfloat162_rn(v[2 * q], v[2 * q + 1]);
                        o[q] = *reinterpret_cast<uint32_t *>(&h2);
                    }
                } else {
                    const uint32_t nb = (__float_as_uint(S[grp]) >> 16) | 0x40u;
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        o[q] = nb | (nb << 16);
                }
                uint16_t *dst = static_cast<uint16_t *>(m.out) + rel[grp];
                if (valid[grp] == 8) {
                    __stcs(reinterpret_cast<uint4 *>(dst), make_uint4(o[0], o[1], o[2], o[3]));
                } else {
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        if (j < valid[grp])
                            dst[j] = (uint16_t)(o[j >> 1] >> (16 * (j & 1)));
                }
            } else {
                if (nan_scale) {
                    const float qn = quiet_nan_of(S[grp]);
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        v[j] = qn;
                }
                float *dst = static_cast<float *>(m.out) + rel[grp];
                if (valid[grp] == 8) {
                    __stcs(reinterpret_cast<float4 *>(dst), make_float4(v[0], v[1], v[2], v[3]));
                    __stcs(reinterpret_cast<float4 *>(dst + 4), make_float4(v[4], v[5], v[6], v[7]));
                } else {
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        if (j < valid[grp])
                            dst[j] = v[j];
                }
            }
        }
    }
}

/* One thread per weight: any blocksize, any alignment. */
template <bool BF16>
__global__ void expand_generic_kernel(const uint8_t *hole, const uint8_t *plug, const float *absmax, int64_t n,
                                      int bs, void *out)
{
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int sh = (int)(i & 1) * 4;
        const uint32_t h = (hole[i >> 1] >> sh) & 15u, p = (plug[i >> 1] >> sh) & 15u;
        const float s = absmax[i / bs];
        const float v = isnan(s) ? quiet_nan_of(s) : g_cells[h][p] * s;
        if (BF16)
            static_cast<uint16_t *>(out)[i] = (uint16_t)f32_to_bf16_bits(v);
        else
            static_cast<float *>(out)[i] = v;
    }
}

template <bool BF16>
int launch_fast(const ExpandBatch &b, cudaStream_t st)
{
    auto kern = expand_stream_kernel<BF16>;
    if (!ensure_smem((const void *)kern, kExpSmem))
        return kLaunch;
    const int64_t total = b.unit_end[b.count - 1];
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(total, (int64_t)sm_count()));
    kern<<<grid, kExpThreads, kExpSmem, st>>>(b);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunch;
}

int log2_if_pow2(int bs)
{
    for (int l = 0; l < 31; ++l)
        if (bs == (1 << l))
            return l;
    return -1;
}

} // namespace

int expand_launch(const ExpandJob *jobs, int count, int bs, OutKind out, cudaStream_t st)
{
    if (bs <= 0)
        return kBadArg;
    const bool bf16 = out == kOutBF16;
    const int l2 = log2_if_pow2(bs);
    ExpandBatch b{};
    b.bs_log2 = l2;
    int rc = kOk;
    auto flush = [&]() -> int {
        if (b.count == 0)
            return kOk;
        int r = bf16 ? launch_fast<true>(b, st) : launch_fast<false>(b, st);
        b = ExpandBatch{};
        b.bs_log2 = l2;
        return r;
    };
    for (int i = 0; i < count && rc == kOk; ++i) {
        const ExpandJob &j = jobs[i];
        if (j.n <= 0)
            continue;
        if (!j.hole || !j.plug || !j.absmax || !j.out)
            return kBadArg;
        /* fast path: a power-of-two blocksize in [8, 1024] (8-weight groups inside one
         * block, absmax index by shift, a unit's absmax a multiple of 16 bytes) and a
         * 16-byte aligned output */
        const bool fast = l2 >= 3 && l2 <= 10 && aligned_to(j.absmax, 4) && aligned_to(j.out, 16);
        if (!fast) {
            const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((j.n + 255) / 256, (int64_t)sm_count() * 8));
            if (bf16)
                expand_generic_kernel<true><<<grid, 256, 0, st>>>(j.hole, j.plug, j.absmax, j.n, bs, j.out);
            else
                expand_generic_kernel<false><<<grid, 256, 0, st>>>(j.hole, j.plug, j.absmax, j.n, bs, j.out);
            rc = cudaGetLastError() == cudaSuccess ? kOk : kLaunch;
            continue;
        }
        const int k = b.count;
        b.hole[k] = j.hole;
        b.plug[k] = j.plug;
        b.absmax[k] = j.absmax;
        b.out[k] = j.out;
        b.n[k] = j.n;
        b.unit_end[k] = (k ? b.unit_end[k - 1] : 0) + (j.n + kUnitW - 1) / kUnitW;
        if (!aligned_to(j.hole, 16) || !aligned_to(j.plug, 16) || !aligned_to(j.absmax, 16))
            b.direct |= 1u << k;
        b.count = k + 1;
        if (b.count == kMaxItems)
            rc = flush();
    }
    if (rc == kOk)
        rc = flush();
    return rc;
}

namespace {

/* Squared dequantisation error of an encoded range, per CTA: the f64 sum over the
 * CTA's elements of ((double)w_i - (double)(CELLS[h_i][p_i] * absmax[i / bs]))^2,
 * the dequantised value being the expand kernels' f32 product.  Element pairs (one
 * plane byte) are dealt out grid-stride, then lanes and warps are added in index
 * order, so a given grid gives the same bits on every call.  The pin tool's rmse
 * (glint_pin.py:66-72 of the reference: glint_np.rmse on glint_np.expand,
 * glint_np.py:93-95) is sqrt(total / n). */
template <bool F32IN>
__global__ void __launch_bounds__(kSqErrThreads) sq_error_kernel(const void *w, const uint8_t *hole,
                                                                 const uint8_t *plug, const float *absmax,
                                                                 int64_t n, int bs, double *partial)
{
    __shared__ float cells[256];
    __shared__ double warp_sum[kSqErrThreads / 32];
    for (int i = threadIdx.x; i < 256; i += kSqErrThreads)
        cells[i] = (&g_cells[0][0])[i];
    __syncthreads();
    double acc = 0.0;
    const int64_t pairs = (n + 1) / 2;
    for (int64_t b = (int64_t)blockIdx.x * kSqErrThreads + threadIdx.x; b < pairs;
         b += (int64_t)gridDim.x * kSqErrThreads) {
        const uint32_t hb = hole[b], pb = plug[b];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int64_t i = 2 * b + e;
            if (i >= n)
                break;
            const uint32_t h = (hb >> (4 * e)) & 15u, p = (pb >> (4 * e)) & 15u;
            const float wf = F32IN ? static_cast<const float *>(w)[i]
                                   : __uint_as_float((uint32_t)static_cast<const uint16_t *>(w)[i] << 16);
            const float q = __fmul_rn(cells[h * 16 + p], absmax[i / bs]);
            const double d = __dsub_rn((double)wf, (double)q);
            acc = __dadd_rn(acc, __dmul_rn(d, d));
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        acc = __dadd_rn(acc, __shfl_down_sync(0xFFFFFFFFu, acc, o));
    if ((threadIdx.x & 31) == 0)
        warp_sum[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        double s = 0.0;
        for (int k = 0; k < kSqErrThreads / 32; ++k)
            s = __dadd_rn(s, warp_sum[k]);
        partial[blockIdx.x] = s;
    }
}

} // namespace

int sq_error_grid(int64_t n)
{
    const int64_t pairs = (n + 1) / 2;
    return (int)std::max<int64_t>(1, std::min<int64_t>((pairs + kSqErrThreads - 1) / kSqErrThreads,
                                                       std::min<int64_t>(kMaxSqErrPartials, 2 * sm_count())));
}

int sq_error_launch(const void *w, bool f32_in, const uint8_t *hole, const uint8_t *plug, const float *absmax,
                    int64_t n, int bs, double *partial, cudaStream_t st)
{
    if (n <= 0 || bs <= 0 || !w || !hole || !plug || !absmax || !partial)
        return kBadArg;
    const int grid = sq_error_grid(n);
    if (f32_in)
        sq_error_kernel<true><<<grid, kSqErrThreads, 0, st>>>(w, hole, plug, absmax, n, bs, partial);
    else
        sq_error_kernel<false><<<grid, kSqErrThreads, 0, st>>>(w, hole, plug, absmax, n, bs, partial);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunch;
}

/* This file's kernel error word (bounded waits that ran out); clear resets it. */
int expand_error_word(bool clear) { return read_error_word(g_expand_error, g_expand_error_taken, clear); }

} // namespace glint
