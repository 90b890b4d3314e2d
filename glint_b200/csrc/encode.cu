/* GLINT encode for sm_100a: BF16 (or f32) weights -> hole/plug planes + absmax.
 *
 * Reference behaviour: cuda/glint_encode.cu:35-102 (k_bf16_to_f32, k_absmax,
 * k_encode_pack) and glint_np.encode_f32 (glint_np.py:63-83).  The reference
 * widens BF16 into an f32 copy, reduces absmax with one 256-thread CTA per
 * 64-weight block, then scans 2 x 16 table entries per weight.  Here one pass
 * reads the input once:
 *
 *   - persistent CTAs of 8 consumer warps and 1 producer warp; the producer
 *     streams units of 4096 weights (8 KB of BF16) into a 5-slot shared-memory
 *     ring with cp.async.bulk, so ~80 KB per SM are in flight regardless of
 *     register pressure; full/empty mbarriers hand the slots over;
 *   - a consumer lane takes 8 consecutive weights (one 16-byte shared load) of
 *     two 256-weight groups per unit, so a block of bs weights is bs/8 adjacent
 *     lanes and its absmax a shuffle-max over them (fmaxf skips NaN, as the
 *     reference's `a > m` does);
 *   - v = RN(w / s) comes from one correctly rounded reciprocal per block and
 *     Markstein's correction per weight (glint_codec.cuh), IEEE division for
 *     blocks whose scale is out of the theorem's range, and 0 when s == 0;
 *   - code = base + (v >= thr) from a 513-cell table in shared memory, 16
 *     replicas so the 8-byte lookups of a half-warp hit 16 distinct bank pairs;
 *     the cell comes from a saturating fma (which also sends NaN to code 0) and
 *     its address from one multiply-add;
 *   - codes are byte-permuted into one 32-bit hole word and one plug word per 8
 *     weights, lo nibble first (element 2e in the low nibble of byte e).
 *
 * Up to 32 tensors share one launch (a unit prefix table in the kernel
 * parameters), so a whole model is encoded in a handful of launches.  Ragged
 * last units and inputs that are not 16-byte aligned are read by the consumers
 * straight from global memory.  Blocksizes that are not a power of two in
 * [8, 256] and planes that are not 4-byte aligned go through the generic
 * two-kernel path, which follows the reference's structure (absmax, then one
 * thread per output byte) with the same arithmetic.
 */
#include <algorithm>
#include <vector>

#include "common.cuh"
#include "glint_internal.h"
#include "ptx.cuh"

namespace glint {
namespace {

constexpr int kMaxItems = 32;
constexpr int kEncReplicas = 16;
constexpr int kLutBytes = kNumCells * kEncReplicas * (int)sizeof(uint2); /* 65,664 */
constexpr int kUnitW = 4096;                                            /* weights per ring slot */
constexpr int kConsumerWarps = 8;                                       /* 512 weights per warp per unit */
constexpr int kEncThreads = (kConsumerWarps + 1) * 32;                  /* + one producer warp */
constexpr int kRingBytes = 40 * 1024;

__device__ int g_encode_error = 0;

struct EncodeBatch {
    const void *w[kMaxItems];
    uint8_t *hole[kMaxItems];
    uint8_t *plug[kMaxItems];
    float *absmax[kMaxItems];
    int64_t n[kMaxItems];
    int64_t unit_end[kMaxItems]; /* inclusive prefix sum of ceil(n / kUnitW) */
    uint32_t direct;             /* bit i: item i is read straight from global (input not 16-B aligned) */
    int count;
};

template <typename In>
constexpr int slot_bytes() { return kUnitW * (int)sizeof(In); }
template <typename In>
constexpr int ring_slots() { return kRingBytes / slot_bytes<In>(); }
template <typename In>
constexpr int enc_smem() { return kLutBytes + kRingBytes + 2 * 8 * ring_slots<In>() + 128; }

/* generic-path lookup (non-replicated table) */
__device__ __forceinline__ uint32_t lut_code(const uint2 *lut, int stride, float v)
{
    uint2 e = lut[cell_of(v) * stride];
    return e.y + (v >= __uint_as_float(e.x) ? 1u : 0u);
}

/* the 8 weights at element offset `off` of the lane's group, from shared memory or
 * (ragged / unaligned units) from global memory */
__device__ __forceinline__ void group_from_smem(const uint16_t *, uint32_t a, float w[8])
{
    const uint4 q = lds128(a);
    const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        w[2 * i] = __uint_as_float(u[i] << 16);
        w[2 * i + 1] = __uint_as_float(u[i] & 0xFFFF0000u);
    }
}
__device__ __forceinline__ void group_from_smem(const float *, uint32_t a, float w[8])
{
    const uint4 q0 = lds128(a), q1 = lds128(a + 16);
    w[0] = __uint_as_float(q0.x), w[1] = __uint_as_float(q0.y), w[2] = __uint_as_float(q0.z), w[3] = __uint_as_float(q0.w);
    w[4] = __uint_as_float(q1.x), w[5] = __uint_as_float(q1.y), w[6] = __uint_as_float(q1.z), w[7] = __uint_as_float(q1.w);
}
__device__ __forceinline__ float gload(const uint16_t *p, int64_t i) { return __uint_as_float((uint32_t)__ldcs(p + i) << 16); }
__device__ __forceinline__ float gload(const float *p, int64_t i) { return __ldcs(p + i); }

/* Codes of 8 weights of one block (absmax s) -> 8 hole nibbles and 8 plug nibbles. */
__device__ __forceinline__ void encode8(const float w[8], float s, uint32_t lut_c, uint32_t &hw, uint32_t &pw)
{
    uint32_t c[8];
    if (s >= kMarksteinLo && s <= kMarksteinHi) {
        const float y = __frcp_rn(s);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float v = quotient_markstein(w[j], s, y);
            const float t = __fmaf_rn(half_sat(v), 512.0f, kMagic);
            const uint2 e = lds64(__float_as_uint(t) * (uint32_t)(kEncReplicas * 8) + lut_c);
            c[j] = e.y + (v >= __uint_as_float(e.x) ? 1u : 0u);
        }
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float v = (s == 0.f) ? 0.f : __fdiv_rn(w[j], s);
            const float t = __fmaf_rn(half_sat(v), 512.0f, kMagic);
            const uint2 e = lds64(__float_as_uint(t) * (uint32_t)(kEncReplicas * 8) + lut_c);
            c[j] = e.y + (v >= __uint_as_float(e.x) ? 1u : 0u);
        }
    }
    /* A = codes of elements 0,2,4,6 as bytes, B = elements 1,3,5,7 */
    const uint32_t A = __byte_perm(__byte_perm(c[0], c[2], 0x0040), __byte_perm(c[4], c[6], 0x0040), 0x5410);
    const uint32_t B = __byte_perm(__byte_perm(c[1], c[3], 0x0040), __byte_perm(c[5], c[7], 0x0040), 0x5410);
    hw = ((A >> 4) & 0x0F0F0F0Fu) | (B & 0xF0F0F0F0u);
    pw = (A & 0x0F0F0F0Fu) | ((B << 4) & 0xF0F0F0F0u);
}

template <typename In, int BS_LOG2>
__global__ void __launch_bounds__(kEncThreads, 2) encode_stream_kernel(const __grid_constant__ EncodeBatch b)
{
    constexpr int S = ring_slots<In>();
    constexpr int SB = slot_bytes<In>();
    constexpr int G = (1 << BS_LOG2) / 8; /* lanes per block */
    extern __shared__ __align__(128) uint8_t smem[];
    uint2 *lut = reinterpret_cast<uint2 *>(smem);
    uint8_t *ring = smem + kLutBytes;
    uint64_t *full = reinterpret_cast<uint64_t *>(ring + kRingBytes);
    uint64_t *empty = full + S;
    __shared__ int64_t unit_end[kMaxItems];

    for (int i = threadIdx.x; i < kNumCells * kEncReplicas; i += kEncThreads)
        lut[i] = g_encode_lut[i / kEncReplicas];
    if (threadIdx.x < kMaxItems)
        unit_end[threadIdx.x] = threadIdx.x < b.count ? b.unit_end[threadIdx.x] : INT64_MAX;
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        mbar_init_fence();
    }
    __syncthreads();

    const int warp = threadIdx.x >> 5;
    const uint32_t lane = lane_id();
    const int64_t total = unit_end[b.count - 1];

    if (warp == kConsumerWarps) {
        /* producer: one bulk copy per full, aligned unit */
        if (lane == 0) {
            int it = 0;
            int64_t i = 0;
            bool ok = true;
            for (int64_t u = blockIdx.x; u < total; u += gridDim.x, ++i) {
                const int s = (int)(i % S);
                const uint32_t ph = (uint32_t)(i / S) & 1u;
                if (i >= S && !(ok = mbar_wait_bounded(&empty[s], ph ^ 1u, &g_encode_error)))
                    break;
                while (unit_end[it] <= u)
                    ++it;
                const int64_t off = (u - (it ? unit_end[it - 1] : 0)) * kUnitW;
                if (b.n[it] - off >= kUnitW && !((b.direct >> it) & 1u)) {
                    mbar_expect_tx(&full[s], SB);
                    bulk_g2s(ring + s * SB, static_cast<const In *>(b.w[it]) + off, SB, &full[s]);
                } else {
                    mbar_arrive(&full[s]);
                }
            }
            /* after a timeout, let the copies already issued land before the CTA exits */
            if (!ok) {
                const int64_t issued = i;
                for (int64_t j = issued > S ? issued - S : 0; j < issued; ++j)
                    if (!mbar_wait_bounded(&full[(int)(j % S)], (uint32_t)(j / S) & 1u, &g_encode_error))
                        break;
            }
        }
        return;
    }

    /* consumers: a warp owns 512 weights of a unit, as two groups of 256 (8 per lane) */
    const uint32_t lut_c = saddr(lut) + (lane & (kEncReplicas - 1)) * 8u - kMagicBits * (uint32_t)(kEncReplicas * 8);
    int it = 0;
    int64_t i = 0;
    for (int64_t u = blockIdx.x; u < total; u += gridDim.x, ++i) {
        const int s = (int)(i % S);
        const uint32_t ph = (uint32_t)(i / S) & 1u;
        const bool ok = lane == 0 ? mbar_wait_bounded(&full[s], ph, &g_encode_error) : true;
        if (!__shfl_sync(0xFFFFFFFFu, ok ? 1 : 0, 0))
            break;
        while (unit_end[it] <= u)
            ++it;
        const int64_t off = (u - (it ? unit_end[it - 1] : 0)) * kUnitW;
        const int64_t n = b.n[it];
        const bool staged = n - off >= kUnitW && !((b.direct >> it) & 1u);
        const In *src = static_cast<const In *>(b.w[it]);
#pragma unroll
        for (int grp = 0; grp < 2; ++grp) {
            const int rel = warp * 512 + grp * 256 + (int)lane * 8; /* element offset inside the unit */
            const int64_t e0 = off + rel;
            const int valid = n - e0 >= 8 ? 8 : (n - e0 > 0 ? (int)(n - e0) : 0);
            float w[8];
            if (staged) {
                group_from_smem(src, saddr(ring + s * SB) + rel * (int)sizeof(In), w);
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    w[j] = j < valid ? gload(src, e0 + j) : 0.f;
            }
            float a = 0.f;
#pragma unroll
            for (int j = 0; j < 8; ++j)
                a = fmaxf(a, fabsf(w[j]));
            const float sc = group_max<G>(a);
            uint32_t hw, pw;
            encode8(w, sc, lut_c, hw, pw);
            if (valid > 0 && (lane & (G - 1)) == 0)
                b.absmax[it][e0 >> BS_LOG2] = sc;
            if (valid == 8) {
                __stcs(reinterpret_cast<uint32_t *>(b.hole[it] + (e0 >> 1)), hw);
                __stcs(reinterpret_cast<uint32_t *>(b.plug[it] + (e0 >> 1)), pw);
            } else if (valid > 0) {
                /* ragged end: nibbles past n stay 0 (the odd-n pad nibble) */
                const uint32_t keep = 0xFFFFFFFFu >> (32 - 4 * valid);
                hw &= keep;
                pw &= keep;
                for (int bb = 0; bb < (valid + 1) / 2; ++bb) {
                    b.hole[it][(e0 >> 1) + bb] = (uint8_t)(hw >> (8 * bb));
                    b.plug[it][(e0 >> 1) + bb] = (uint8_t)(pw >> (8 * bb));
                }
            }
        }
        __syncwarp();
        if (lane == 0)
            mbar_arrive(&empty[s]);
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
    if (!ensure_smem((const void *)kern, enc_smem<In>()))
        return kLaunch;
    const int64_t total = b.unit_end[b.count - 1];
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(total, (int64_t)sm_count() * 2));
    kern<<<grid, kEncThreads, enc_smem<In>(), st>>>(b);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunch;
}

template <typename In>
int launch_fast(const EncodeBatch &b, int bs_log2, cudaStream_t st)
{
    switch (bs_log2) {
    case 3: return launch_fast_bs<In, 3>(b, st);
    case 4: return launch_fast_bs<In, 4>(b, st);
    case 5: return launch_fast_bs<In, 5>(b, st);
    case 6: return launch_fast_bs<In, 6>(b, st);
    case 7: return launch_fast_bs<In, 7>(b, st);
    case 8: return launch_fast_bs<In, 8>(b, st);
    default: return kBadBlocksize;
    }
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
    const bool fast_bs = l2 >= 3 && l2 <= 8;
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
        const bool aligned = aligned_to(j.hole, 4) && aligned_to(j.plug, 4) && aligned_to(j.absmax, 4);
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
        b.unit_end[k] = (k ? b.unit_end[k - 1] : 0) + (j.n + kUnitW - 1) / kUnitW;
        if (!aligned_to(j.w, 16))
            b.direct |= 1u << k;
        b.count = k + 1;
        if (b.count == kMaxItems)
            rc = flush();
    }
    if (rc == kOk)
        rc = flush();
    return rc;
}

} // namespace glint
