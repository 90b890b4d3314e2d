/* GLINT encode for sm_100a: BF16 (or f32) weights -> hole/plug planes + absmax.
 *
 * Reference behaviour: cuda/glint_encode.cu:35-102 (k_bf16_to_f32, k_absmax,
 * k_encode_pack) and glint_np.encode_f32 (glint_np.py:63-83).  The reference
 * widens BF16 into an f32 copy, reduces absmax with one 256-thread CTA per
 * 64-weight block, then scans 2 x 16 table entries per weight.  Here one pass
 * reads the input once:
 *
 *   - one persistent CTA per SM: 24 consumer warps (12 for f32 input) and a
 *     producer warp that streams 48 KB units (24576 BF16 weights) into a 3-slot
 *     shared-memory ring, BF16 through 2-D TMA with the 64-byte swizzle (rows of
 *     32 weights; a quarter-warp's 16-byte reads of eight rows cover the 32
 *     banks), f32 with cp.async.bulk, so 144 KB per SM are in flight whatever the
 *     register pressure; full/empty mbarriers hand the slots over;
 *   - a consumer lane owns 32 consecutive weights (four 16-byte shared loads), so
 *     a block of bs weights is bs/32 adjacent lanes and its absmax a shuffle-max
 *     over them.  The maximum is taken with the packed BF16 max of absolute
 *     values that propagates NaN (for f32 input: integer max of |w|'s bits, where
 *     NaN sorts above inf), so the same pass tells whether the block holds a NaN;
 *     such blocks recompute absmax with fmaxf, which skips NaN as the reference's
 *     `a > m` does;
 *   - v = RN(w / s) comes from one correctly rounded reciprocal per block and
 *     Markstein's correction per weight (glint_codec.cuh), evaluated two weights
 *     per instruction with the f32x2 forms; blocks with a NaN, with s == 0 or
 *     with s outside the theorem's range use the IEEE divide (and 0 when s == 0);
 *   - code = base + (v >= thr) from a 513-cell table in shared memory, 16
 *     replicas so the 8-byte lookups of a half-warp hit 16 distinct bank pairs;
 *     the replicas hold thr lowered by one ulp, so the test is v > thr', on the
 *     fast path the sign bit of one subtraction;
 *     on NaN-free blocks v lies in [-1, 1], so the cell is one fma and its
 *     address one multiply-add (the other blocks clamp first);
 *   - codes are byte-permuted into 8 bytes of hole and 8 bytes of plug per lane
 *     (one 8-byte store each), lo nibble first (element 2e in the low nibble of
 *     byte e).
 *
 * Up to 32 tensors share one launch (a unit prefix table in the kernel
 * parameters), so a whole model is encoded in a handful of launches.  Ragged
 * last units and inputs that are not 16-byte aligned are read by the consumers
 * straight from global memory.  Blocksizes that are not a power of two in
 * [16, 512] and planes that are not 8-byte aligned go through the generic
 * two-kernel path, which follows the reference's structure (absmax, then one
 * thread per output byte) with the same arithmetic.
 */
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "glint_internal.h"
#include "ptx.cuh"

namespace glint {

__device__ int g_encode_error = 0;
__device__ int g_encode_error_taken = 0; /* read_error_word's result slot */

namespace {

constexpr int kMaxItems = 32;
constexpr int kEncReplicas = 16;
constexpr int kLutBytes = kNumCells * kEncReplicas * (int)sizeof(uint2); /* 65,664 */
constexpr int kSlotBytes = 48 * 1024;                                   /* one unit of input */
constexpr int kSlots = 3;
constexpr int kWpl = 32;                                                /* weights per consumer lane */



struct EncodeBatch {
    /* BF16 inputs viewed as rows of 32 weights (64 B) for 2-D TMA with the 64-byte
     * swizzle; used for the full units of the items in `tma` */
    CUtensorMap wmap[kMaxItems];
    const void *w[kMaxItems];
    uint8_t *hole[kMaxItems];
    uint8_t *plug[kMaxItems];
    float *absmax[kMaxItems];
    int64_t n[kMaxItems];
    int64_t unit_end[kMaxItems]; /* inclusive prefix sum of ceil(n / unit weights) */
    uint32_t direct;             /* bit i: item i is read straight from global (input not 16-B aligned) */
    uint32_t tma;                /* bit i: item i's full units are staged through wmap[i] */
    int count;
};

/* one unit fills a slot: 24576 BF16 or 12288 f32 weights, 32 per consumer lane */
template <typename In>
constexpr int unit_w() { return kSlotBytes / (int)sizeof(In); }
template <typename In>
constexpr int consumer_warps() { return unit_w<In>() / (32 * kWpl); }
template <typename In>
constexpr int enc_threads() { return (consumer_warps<In>() + 1) * 32; }
constexpr int kMetaBytes = 48;
constexpr int kRingOff = (kLutBytes + 1023) / 1024 * 1024; /* the ring starts on a 1 KB boundary (TMA swizzle) */
constexpr int kEncSmem = kRingOff + kSlots * kSlotBytes + kSlots * kMetaBytes + 2 * 8 * kSlots + 128;
constexpr int kTmaRows = 256; /* rows of 32 BF16 weights per TMA box: 16 KB, 3 boxes per unit */

/* What the producer tells the consumers about the unit in a slot: pointers already
 * offset to the unit's first element, how many weights it holds, and whether its
 * input sits in the slot (or must be read from global memory). */
struct UnitMeta {
    const void *src;
    uint8_t *hole;
    uint8_t *plug;
    float *absmax;
    int valid;
    int staged;
    int swz; /* staged through TMA with the 64-byte swizzle (else a linear bulk copy) */
    int pad;
};
static_assert(sizeof(UnitMeta) == kMetaBytes, "slot descriptor layout");

/* ring position of the next unit: slot s, and the phase parity of its barriers */
__device__ __forceinline__ void next_slot(int &s, uint32_t &ph)
{
    if (++s == kSlots) {
        s = 0;
        ph ^= 1u;
    }
}

/* generic-path lookup (non-replicated table) */
__device__ __forceinline__ uint32_t lut_code(const uint2 *lut, int stride, float v)
{
    uint2 e = lut[cell_of(v) * stride];
    return e.y + (v >= __uint_as_float(e.x) ? 1u : 0u);
}

__device__ __forceinline__ uint64_t pack2(float lo, float hi)
{
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void unpack2(uint64_t v, float &lo, float &hi) { asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v)); }
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b)
{
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c)
{
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

/* 16 weights of one lane as f32, and the lane's |w| bit maximum (NaN above inf) */
struct Lane16 {
    float w[16];
    uint32_t mag; /* max over the lane of |w| as an order-preserving integer */
};
__device__ __forceinline__ uint32_t absmax_bf16x2(uint32_t a, uint32_t b)
{
    uint32_t d; /* per half: max(|a|, |b|) (sign = xor, ignored), NaN if either is NaN */
    asm("max.NaN.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ void from_words(const uint16_t *, const uint32_t (&u)[8], Lane16 &L)
{
    /* BF16 max on |w| with NaN propagation: one instruction per two weights; a NaN
     * comes out as the canonical 0x7FFF, which as f32 bits sorts above inf */
    uint32_t m = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        L.w[2 * i] = __uint_as_float(u[i] << 16);
        L.w[2 * i + 1] = __uint_as_float(u[i] & 0xFFFF0000u);
        m = absmax_bf16x2(m, u[i]);
    }
    L.mag = (absmax_bf16x2(m, m >> 16) & 0x7FFFu) << 16; /* as f32 bits */
}
__device__ __forceinline__ void from_words(const float *, const uint32_t (&u)[16], Lane16 &L)
{
    uint32_t m = 0;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        L.w[i] = __uint_as_float(u[i]);
        m = max(m, u[i] & 0x7FFFFFFFu);
    }
    L.mag = m;
}
template <typename In>
struct Words {
    static constexpr int N = 16 * (int)sizeof(In) / 4;
};
__device__ __forceinline__ void smem_words(const uint16_t *, uint32_t a, uint32_t (&u)[8])
{
    const uint4 q0 = lds128(a), q1 = lds128(a + 16);
    u[0] = q0.x, u[1] = q0.y, u[2] = q0.z, u[3] = q0.w, u[4] = q1.x, u[5] = q1.y, u[6] = q1.z, u[7] = q1.w;
}
__device__ __forceinline__ void smem_words(const float *, uint32_t a, uint32_t (&u)[16])
{
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint4 q = lds128(a + 16 * i);
        u[4 * i] = q.x, u[4 * i + 1] = q.y, u[4 * i + 2] = q.z, u[4 * i + 3] = q.w;
    }
}
__device__ __forceinline__ void global_words(const uint16_t *p, int64_t e0, int valid, uint32_t (&u)[8])
{
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t lo = 2 * i < valid ? (uint32_t)__ldcs(p + e0 + 2 * i) : 0u;
        const uint32_t hi = 2 * i + 1 < valid ? (uint32_t)__ldcs(p + e0 + 2 * i + 1) : 0u;
        u[i] = lo | (hi << 16);
    }
}
__device__ __forceinline__ void global_words(const float *p, int64_t e0, int valid, uint32_t (&u)[16])
{
#pragma unroll
    for (int i = 0; i < 16; ++i)
        u[i] = i < valid ? __float_as_uint(__ldcs(p + e0 + i)) : 0u;
}

/* A = codes of elements 0,2,4,6 of c[o..o+7] as bytes, B = elements 1,3,5,7 ->
 * one hole word and one plug word (lo nibble first). */
__device__ __forceinline__ void pack8(const uint32_t *c, uint32_t &hw, uint32_t &pw)
{
    const uint32_t A = __byte_perm(__byte_perm(c[0], c[2], 0x0040), __byte_perm(c[4], c[6], 0x0040), 0x5410);
    const uint32_t B = __byte_perm(__byte_perm(c[1], c[3], 0x0040), __byte_perm(c[5], c[7], 0x0040), 0x5410);
    hw = ((A >> 4) & 0x0F0F0F0Fu) | (B & 0xF0F0F0F0u);
    pw = (A & 0x0F0F0F0Fu) | ((B << 4) & 0xF0F0F0F0u);
}

/* y = RN(1/s) for a block scale s in the Markstein range.  BF16 input: s is a
 * BF16 value (the |w| maximum of BF16 weights), so y is the table entry of its
 * 7-bit fraction with the exponent moved; f32 input: the correctly rounded
 * reciprocal. */
__device__ __forceinline__ float block_rcp(const uint16_t *, float s, const uint32_t *rcp_tab)
{
    const uint32_t b = __float_as_uint(s);
    return __uint_as_float(rcp_tab[(b >> 16) & 0x7Fu] + (127u << 23) - (b & 0x7F800000u));
}
__device__ __forceinline__ float block_rcp(const float *, float s, const uint32_t *) { return __frcp_rn(s); }

/* Bits of the largest float below the float with bits `b` (b neither +-0 nor
 * NaN: the table's thresholds are nonzero, +inf where a cell has none).  For
 * every non-NaN v, v >= thr exactly when v > prev_below(thr): no float lies
 * between the two. */
__device__ __forceinline__ uint32_t prev_below(uint32_t b) { return (b >> 31) ? b + 1u : b - 1u; }

/* Codes of 16 weights of one block of absmax s; y = RN(1/s) when `fast` (the block
 * is NaN-free and s lies in the Markstein range).  The shared table holds
 * (thr' = prev_below(thr), base) per cell, and code = base + (v > thr').  On the
 * fast path v is finite, so v > thr' is the sign bit of RN(thr' - v): the
 * difference is negative exactly when v > thr', and an exact zero comes out +0
 * (it could be -0 only for thr' = -0, which prev_below never yields), so one
 * subtraction and one shift-add replace the compare and select. */
__device__ __forceinline__ void codes16(const float *w, float s, float y, bool fast, uint32_t lut_c, uint32_t (&c)[16])
{
    if (fast) {
        /* v = RN(w / s) exactly, so v is in [-1, 1] and the cell needs no clamp */
        const uint64_t y2 = pack2(y, y), ns2 = pack2(-s, -s);
        const uint64_t k256 = pack2(256.0f, 256.0f), kadd = pack2(kMagic + 256.0f, kMagic + 256.0f);
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
            const uint64_t w2 = pack2(w[j], w[j + 1]);
            const uint64_t q2 = mul2(w2, y2);
            const uint64_t v2 = fma2(fma2(q2, ns2, w2), y2, q2);
            const uint64_t t2 = fma2(v2, k256, kadd);
            float v0, v1, t0, t1;
            unpack2(v2, v0, v1);
            unpack2(t2, t0, t1);
            const uint2 e0 = lds64(__float_as_uint(t0) * (uint32_t)(kEncReplicas * 8) + lut_c);
            const uint2 e1 = lds64(__float_as_uint(t1) * (uint32_t)(kEncReplicas * 8) + lut_c);
            c[j] = e0.y + (__float_as_uint(__fsub_rn(__uint_as_float(e0.x), v0)) >> 31);
            c[j + 1] = e1.y + (__float_as_uint(__fsub_rn(__uint_as_float(e1.x), v1)) >> 31);
        }
    } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const float v = (s == 0.f) ? 0.f : __fdiv_rn(w[j], s);
            const uint2 e = lds64((cell_of(v) + kMagicBits) * (uint32_t)(kEncReplicas * 8) + lut_c);
            c[j] = e.y + (v > __uint_as_float(e.x) ? 1u : 0u); /* NaN v: base, as v >= thr */
        }
    }
}

/* hole and plug bytes of 16 codes (8 bytes each, as two words) */
__device__ __forceinline__ void pack16(const uint32_t (&c)[16], uint32_t &h0, uint32_t &h1, uint32_t &p0, uint32_t &p1)
{
    pack8(c, h0, p0);
    pack8(c + 8, h1, p1);
}

template <int G>
__device__ __forceinline__ uint32_t group_max_u32(uint32_t v)
{
#pragma unroll
    for (int off = G / 2; off > 0; off >>= 1)
        v = max(v, __shfl_xor_sync(0xFFFFFFFFu, v, off));
    return v;
}

/* the block absmax of one lane group: NaN-ignoring max over the group's weights */
template <int G>
__device__ __forceinline__ float nan_skipping_max(const float *w, int n)
{
    float a = 0.f;
    for (int j = 0; j < n; ++j)
        a = fmaxf(a, fabsf(w[j]));
    const unsigned act = __activemask();
#pragma unroll
    for (int o = G / 2; o > 0; o >>= 1)
        a = fmaxf(a, __shfl_xor_sync(act, a, o));
    return a;
}

template <typename In, int BS_LOG2>
__global__ void __launch_bounds__(enc_threads<In>(), 1) encode_stream_kernel(const __grid_constant__ EncodeBatch b)
{
    constexpr int UW = unit_w<In>();
    constexpr int CW = consumer_warps<In>();
    /* lanes per block for bs >= 32 (a lane's 32 weights share one block); for bs == 16
     * each 16-weight half of a lane is its own block */
    constexpr int G = BS_LOG2 >= 5 ? (1 << BS_LOG2) / kWpl : 1;
    extern __shared__ __align__(128) uint8_t smem[];
    uint2 *lut = reinterpret_cast<uint2 *>(smem);
    uint8_t *ring = smem + kRingOff;
    UnitMeta *meta = reinterpret_cast<UnitMeta *>(ring + kSlots * kSlotBytes);
    uint64_t *full = reinterpret_cast<uint64_t *>(meta + kSlots);
    uint64_t *empty = full + kSlots;

    /* the replicas hold each cell's threshold lowered by one ulp (prev_below), so
     * v >= thr becomes v > thr' (see codes16) */
    for (int i = threadIdx.x; i < kNumCells * kEncReplicas; i += enc_threads<In>()) {
        const uint2 e = g_encode_lut[i / kEncReplicas];
        lut[i] = make_uint2(prev_below(e.x), e.y);
    }
    /* RN(1 / (1 + k/128)), k = 0..127: with BF16 input a block's absmax is itself a
     * BF16 value, 1.k x 2^E with a 7-bit fraction k, and RN(1/s) = RN(1/1.k) x 2^-E
     * exactly (scaling by a power of two rounds nothing) */
    __shared__ uint32_t rcp_tab[128];
    if (threadIdx.x < 128)
        rcp_tab[threadIdx.x] = __float_as_uint(__frcp_rn(1.0f + (float)threadIdx.x * (1.0f / 128.0f)));
    if (threadIdx.x == 0) {
        for (int s = 0; s < kSlots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], CW);
        }
        mbar_init_fence();
    }
    __syncthreads();

    const int warp = threadIdx.x >> 5;
    const uint32_t lane = lane_id();
    const int64_t total = b.unit_end[b.count - 1];

    if (warp == CW) {
        /* producer: publish each unit's descriptor, then one bulk copy per full, aligned unit */
        if (lane == 0) {
            int it = 0, s = 0;
            int64_t i = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int64_t u = blockIdx.x; u < total; u += gridDim.x, ++i, next_slot(s, ph)) {
                if (i >= kSlots && !(ok = mbar_wait_bounded(&empty[s], ph ^ 1u, &g_encode_error)))
                    break;
                while (b.unit_end[it] <= u)
                    ++it;
                const int64_t off = (u - (it ? b.unit_end[it - 1] : 0)) * UW;
                const int64_t left = b.n[it] - off;
                const bool staged = left >= UW && !((b.direct >> it) & 1u);
                UnitMeta &m = meta[s];
                m.src = static_cast<const In *>(b.w[it]) + off;
                m.hole = b.hole[it] + off / 2;
                m.plug = b.plug[it] + off / 2;
                m.absmax = b.absmax[it] + (off >> BS_LOG2);
                m.valid = left >= UW ? UW : (int)left;
                m.staged = staged ? 1 : 0;
                m.swz = staged && sizeof(In) == 2 && ((b.tma >> it) & 1u) ? 1 : 0;
                if (m.swz) {
                    /* three boxes of 256 rows x 64 B, each 16-byte chunk c of row r landing at
                     * chunk c ^ ((r >> 1) & 3): a quarter-warp's 16-byte reads of eight rows
                     * then cover all 32 banks */
                    mbar_expect_tx(&full[s], kSlotBytes);
                    const int row0 = (int)(off / 32);
#pragma unroll
                    for (int bx = 0; bx < kSlotBytes / (kTmaRows * 64); ++bx)
                        tma_load_2d(ring + s * kSlotBytes + bx * kTmaRows * 64, &b.wmap[it], &full[s], 0,
                                    row0 + bx * kTmaRows);
                } else if (staged) {
                    mbar_expect_tx(&full[s], kSlotBytes);
                    bulk_g2s(ring + s * kSlotBytes, m.src, kSlotBytes, &full[s]);
                } else {
                    mbar_arrive(&full[s]);
                }
            }
            /* after a timeout, let the copies already issued land before the CTA exits */
            if (!ok) {
                const int64_t issued = i;
                for (int64_t j = issued > kSlots ? issued - kSlots : 0; j < issued; ++j)
                    if (!mbar_wait_bounded(&full[(int)(j % kSlots)], (uint32_t)(j / kSlots) & 1u, &g_encode_error))
                        break;
            }
        }
        return;
    }

    /* consumers: a lane owns 32 consecutive weights of a unit */
    const uint32_t lut_c = saddr(lut) + (lane & (kEncReplicas - 1)) * 8u - kMagicBits * (uint32_t)(kEncReplicas * 8);
    const int rel = (warp * 32 + (int)lane) * kWpl; /* element offset inside a unit */
    int s = 0;
    uint32_t ph = 0;
    for (int64_t u = blockIdx.x; u < total; u += gridDim.x, next_slot(s, ph)) {
        const bool ok = lane == 0 ? mbar_wait_bounded(&full[s], ph, &g_encode_error) : true;
        if (!__shfl_sync(0xFFFFFFFFu, ok ? 1 : 0, 0))
            break;
        const UnitMeta m = meta[s];
        const int valid = m.valid - rel >= kWpl ? kWpl : (m.valid - rel > 0 ? m.valid - rel : 0);
        const In *src = static_cast<const In *>(m.src);
        uint32_t wa[Words<In>::N], wb[Words<In>::N];
        if (m.swz) {
            /* row rel/32 of the slot, chunk j at j ^ ((row >> 1) & 3) (BF16 only) */
            const uint32_t row = (uint32_t)rel / 32u, sw = (row >> 1) & 3u;
            const uint32_t a = saddr(ring + s * kSlotBytes) + row * 64u;
            uint32_t q[16];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint4 v = lds128(a + (((uint32_t)j ^ sw) << 4));
                q[4 * j] = v.x, q[4 * j + 1] = v.y, q[4 * j + 2] = v.z, q[4 * j + 3] = v.w;
            }
#pragma unroll
            for (int j = 0; j < Words<In>::N; ++j)
                wa[j] = q[j], wb[j] = q[j + Words<In>::N];
        } else if (m.staged) {
            const uint32_t a = saddr(ring + s * kSlotBytes) + rel * (int)sizeof(In);
            smem_words(src, a, wa);
            smem_words(src, a + 16 * (int)sizeof(In), wb);
        } else {
            global_words(src, rel, valid, wa);
            global_words(src, rel + 16, valid - 16, wb);
        }
        __syncwarp();
        if (lane == 0)
            mbar_arrive(&empty[s]); /* the slot's data now lives in registers */

        Lane16 A, B;
        from_words(src, wa, A);
        from_words(src, wb, B);
        uint32_t ca[16], cb[16];
        float sa, sb;
        if (BS_LOG2 >= 5) {
            const uint32_t mag = group_max_u32<G>(max(A.mag, B.mag));
            const bool nan_free = mag <= 0x7F800000u; /* NaN sorts above inf */
            float sc = __uint_as_float(mag);
            if (!nan_free) {
                float both[32];
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    both[j] = A.w[j], both[16 + j] = B.w[j];
                sc = nan_skipping_max<G>(both, 32); /* absmax skips NaN, as the reference's (a > m) does */
            }
            const bool fast = nan_free && sc >= kMarksteinLo && sc <= kMarksteinHi;
            const float y = fast ? block_rcp(src, sc, rcp_tab) : 0.f;
            codes16(A.w, sc, y, fast, lut_c, ca);
            codes16(B.w, sc, y, fast, lut_c, cb);
            sa = sb = sc;
        } else {
            /* bs == 16: two blocks per lane */
            const bool nfa = A.mag <= 0x7F800000u, nfb = B.mag <= 0x7F800000u;
            sa = nfa ? __uint_as_float(A.mag) : nan_skipping_max<1>(A.w, 16);
            sb = nfb ? __uint_as_float(B.mag) : nan_skipping_max<1>(B.w, 16);
            const bool fa = nfa && sa >= kMarksteinLo && sa <= kMarksteinHi;
            const bool fb = nfb && sb >= kMarksteinLo && sb <= kMarksteinHi;
            codes16(A.w, sa, fa ? block_rcp(src, sa, rcp_tab) : 0.f, fa, lut_c, ca);
            codes16(B.w, sb, fb ? block_rcp(src, sb, rcp_tab) : 0.f, fb, lut_c, cb);
        }
        uint32_t h[4], p[4];
        pack16(ca, h[0], h[1], p[0], p[1]);
        pack16(cb, h[2], h[3], p[2], p[3]);
        if (BS_LOG2 >= 5) {
            if (valid > 0 && (lane & (G - 1)) == 0)
                m.absmax[rel >> BS_LOG2] = sa;
        } else {
            if (valid > 0)
                m.absmax[rel >> BS_LOG2] = sa;
            if (valid > 16)
                m.absmax[(rel >> BS_LOG2) + 1] = sb;
        }
        uint8_t *hd = m.hole + (rel >> 1), *pd = m.plug + (rel >> 1);
        if (valid == kWpl) {
            __stcs(reinterpret_cast<uint4 *>(hd), make_uint4(h[0], h[1], h[2], h[3]));
            __stcs(reinterpret_cast<uint4 *>(pd), make_uint4(p[0], p[1], p[2], p[3]));
        } else if (valid > 0) {
            /* ragged end: nibbles past n stay 0 (the odd-n pad nibble) */
#pragma unroll
            for (int bb = 0; bb < 16; ++bb) {
                if (bb < (valid + 1) / 2) {
                    const int e = 2 * bb; /* first element of this byte */
                    const uint32_t keep = (e + 1 < valid) ? 0xFFu : 0x0Fu;
                    hd[bb] = (uint8_t)((h[bb >> 2] >> (8 * (bb & 3))) & keep);
                    pd[bb] = (uint8_t)((p[bb >> 2] >> (8 * (bb & 3))) & keep);
                }
            }
        }
    }
}

/* ---- generic path: any blocksize, any alignment ------------------------------ */

__device__ __forceinline__ float load_one(const uint16_t *p, int64_t i) { return __uint_as_float((uint32_t)p[i] << 16); }
__device__ __forceinline__ float load_one(const float *p, int64_t i) { return p[i]; }

template <typename In>
__global__ void encode_generic_absmax_kernel(const In *w, int64_t n, int bs, float *absmax)
{
    const int64_t nb = (n + bs - 1) / bs;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
    for (int64_t blk = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); blk < nb; blk += warps) {
        float m = 0.f;
        const int64_t b0 = blk * bs;
        for (int64_t i = b0 + lane_id(); i < b0 + bs && i < n; i += 32)
            m = fmaxf(m, fabsf(load_one(w, i)));
        m = group_max<32>(m);
        if (lane_id() == 0)
            absmax[blk] = m;
    }
}

template <typename In>
__global__ void encode_generic_pack_kernel(const In *w, int64_t n, int bs, const float *absmax, uint8_t *hole,
                                           uint8_t *plug)
{
    __shared__ uint2 lut[kNumCells];
    for (int i = threadIdx.x; i < kNumCells; i += blockDim.x)
        lut[i] = g_encode_lut[i];
    __syncthreads();
    const int64_t npack = (n + 1) / 2;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < npack; e += (int64_t)gridDim.x * blockDim.x) {
        uint32_t c[2] = {0, 0};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int64_t i = 2 * e + h;
            if (i < n) {
                const float s = absmax[i / bs];
                const float v = (s == 0.f) ? 0.f : __fdiv_rn(load_one(w, i), s);
                c[h] = lut_code(lut, 1, v);
            }
        }
        hole[e] = (uint8_t)((c[0] >> 4) | ((c[1] >> 4) << 4));
        plug[e] = (uint8_t)((c[0] & 15u) | ((c[1] & 15u) << 4));
    }
}

template <typename In>
int launch_generic(const EncodeJob &j, int bs, cudaStream_t st)
{
    const int64_t nb = (j.n + bs - 1) / bs;
    const int sms = sm_count();
    const int g1 = (int)std::min<int64_t>((nb + 7) / 8, (int64_t)sms * 16);
    encode_generic_absmax_kernel<In><<<std::max(g1, 1), 256, 0, st>>>(static_cast<const In *>(j.w), j.n, bs, j.absmax);
    const int64_t npack = (j.n + 1) / 2;
    const int g2 = (int)std::min<int64_t>((npack + 255) / 256, (int64_t)sms * 8);
    encode_generic_pack_kernel<In><<<std::max(g2, 1), 256, 0, st>>>(static_cast<const In *>(j.w), j.n, bs, j.absmax,
                                                                    j.hole, j.plug);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunch;
}

template <typename In, int BS_LOG2>
int launch_fast_bs(const EncodeBatch &b, cudaStream_t st)
{
    auto kern = encode_stream_kernel<In, BS_LOG2>;
    if (!ensure_smem((const void *)kern, kEncSmem))
        return kLaunch;
    const int64_t total = b.unit_end[b.count - 1];
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(total, (int64_t)sm_count()));
    kern<<<grid, enc_threads<In>(), kEncSmem, st>>>(b);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunch;
}

template <typename In>
int launch_fast(const EncodeBatch &b, int bs_log2, cudaStream_t st)
{
    switch (bs_log2) {
    case 4: return launch_fast_bs<In, 4>(b, st);
    case 5: return launch_fast_bs<In, 5>(b, st);
    case 6: return launch_fast_bs<In, 6>(b, st);
    case 7: return launch_fast_bs<In, 7>(b, st);
    case 8: return launch_fast_bs<In, 8>(b, st);
    case 9: return launch_fast_bs<In, 9>(b, st);
    default: return kBadBlocksize;
    }
}

/* BF16 tensor of n weights as [n / 32 rows][32] for 64-byte-swizzled TMA boxes of
 * 256 rows; false when the driver entry point is missing or the map is refused */
bool bf16_row_map(CUtensorMap *m, const void *w, int64_t n)
{
    auto enc = tensor_map_encoder();
    if (!enc || n < 32)
        return false;
    cuuint64_t dims[2] = {32, (cuuint64_t)(n / 32)};
    cuuint64_t strides[1] = {64};
    cuuint32_t box[2] = {32, kTmaRows};
    cuuint32_t estr[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(w), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int log2_if_pow2(int bs)
{
    for (int l = 0; l < 31; ++l)
        if (bs == (1 << l))
            return l;
    return -1;
}

} // namespace

int encode_launch(const EncodeJob *jobs, int count, int bs, bool f32_in, cudaStream_t st)
{
    if (bs <= 0)
        return kBadArg;
    const int l2 = log2_if_pow2(bs);
    const bool fast_bs = l2 >= 4 && l2 <= 9;
    EncodeBatch b{};
    int rc = kOk;
    auto flush = [&]() -> int {
        if (b.count == 0)
            return kOk;
        int r = f32_in ? launch_fast<float>(b, l2, st) : launch_fast<uint16_t>(b, l2, st);
        b = EncodeBatch{};
        return r;
    };
    for (int i = 0; i < count && rc == kOk; ++i) {
        const EncodeJob &j = jobs[i];
        if (j.n <= 0)
            continue;
        if (!j.w || !j.hole || !j.plug || !j.absmax)
            return kBadArg;
        const bool aligned = aligned_to(j.hole, 16) && aligned_to(j.plug, 16) && aligned_to(j.absmax, 4);
        if (!fast_bs || !aligned) {
            rc = f32_in ? launch_generic<float>(j, bs, st) : launch_generic<uint16_t>(j, bs, st);
            continue;
        }
        const int k = b.count;
        b.w[k] = j.w;
        b.hole[k] = j.hole;
        b.plug[k] = j.plug;
        b.absmax[k] = j.absmax;
        b.n[k] = j.n;
        const int64_t uw = f32_in ? unit_w<float>() : unit_w<uint16_t>();
        b.unit_end[k] = (k ? b.unit_end[k - 1] : 0) + (j.n + uw - 1) / uw;
        if (!aligned_to(j.w, 16))
            b.direct |= 1u << k;
        else if (!f32_in && j.n >= uw && bf16_row_map(&b.wmap[k], j.w, j.n))
            b.tma |= 1u << k;
        b.count = k + 1;
        if (b.count == kMaxItems)
            rc = flush();
    }
    if (rc == kOk)
        rc = flush();
    return rc;
}

/* This file's kernel error word (bounded waits that ran out); clear resets it. */
int encode_error_word(bool clear) { return read_error_word(g_encode_error, g_encode_error_taken, clear); }

} // namespace glint
