/* GLINT encode for sm_100a: BF16 (or f32) weights -> hole/plug planes + absmax.
 *
 * Reference behaviour: cuda/glint_encode.cu:35-102 (k_bf16_to_f32, k_absmax,
 * k_encode_pack) and glint_np.encode_f32 (glint_np.py:63-83).  The reference
 * widens BF16 into an f32 copy, reduces absmax with one 256-thread CTA per
 * 64-weight block, then scans 2 x 16 table entries per weight.  Here one pass
 * reads the input once:
 *
 *   - a warp owns a chunk of 256 consecutive weights, 8 per lane (one 16-byte
 *     load for BF16), so a block of bs weights is bs/8 adjacent lanes;
 *   - block absmax is a shuffle-max over those lanes (fmaxf skips NaN, as the
 *     reference's `a > m` does);
 *   - v = RN(w / s) comes from one correctly rounded reciprocal per block and
 *     Markstein's correction per weight (glint_codec.cuh), IEEE division for
 *     blocks whose scale is out of the theorem's range, and 0 when s == 0;
 *   - code = base + (v >= thr) from a 513-cell table held in shared memory in 16
 *     replicas, so the 8-byte lookups of a half-warp hit 16 distinct bank pairs;
 *   - the 8 hole and 8 plug nibbles of a lane are one 32-bit store each, lo
 *     nibble first (element 2e in the low nibble of byte e).
 *
 * Up to 32 tensors share one launch (a chunk prefix table in the kernel
 * parameters), so a whole model is encoded in a handful of launches.  Tensors
 * whose blocksize is not a power of two in [8, 256] or whose pointers are not
 * aligned go through the generic two-kernel path, which follows the reference's
 * structure (absmax, then one thread per output byte) with the same arithmetic.
 */
#include <algorithm>
#include <vector>

#include "common.cuh"
#include "glint_internal.h"

namespace glint {
namespace {

constexpr int kEncThreads = 256;
constexpr int kEncReplicas = 16;
constexpr int kMaxItems = 32;
constexpr int kChunk = 256; /* weights per warp chunk: 32 lanes x 8 */
constexpr int kEncSmem = kNumCells * kEncReplicas * (int)sizeof(uint2);

struct EncodeBatch {
    const void *w[kMaxItems];
    uint8_t *hole[kMaxItems];
    uint8_t *plug[kMaxItems];
    float *absmax[kMaxItems];
    int64_t n[kMaxItems];
    int64_t chunk_end[kMaxItems]; /* inclusive prefix sum of ceil(n / 256) */
    int count;
};

__device__ __forceinline__ uint32_t lut_code(const uint2 *lut, int stride, float v)
{
    uint2 e = lut[cell_of(v) * stride];
    return e.y + (v >= __uint_as_float(e.x) ? 1u : 0u);
}

/* 8 consecutive weights of lane-chunk `off` (valid = how many exist). */
__device__ __forceinline__ void load8(const uint16_t *p, int64_t off, int valid, float w[8])
{
    if (valid == 8) {
        uint4 q = __ldcs(reinterpret_cast<const uint4 *>(p + off));
        uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            w[2 * i] = __uint_as_float(u[i] << 16);
            w[2 * i + 1] = __uint_as_float(u[i] & 0xFFFF0000u);
        }
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j)
            w[j] = j < valid ? __uint_as_float((uint32_t)__ldcs(p + off + j) << 16) : 0.f;
    }
}
__device__ __forceinline__ void load8(const float *p, int64_t off, int valid, float w[8])
{
    if (valid == 8) {
        float4 a = __ldcs(reinterpret_cast<const float4 *>(p + off));
        float4 b = __ldcs(reinterpret_cast<const float4 *>(p + off + 4));
        w[0] = a.x, w[1] = a.y, w[2] = a.z, w[3] = a.w;
        w[4] = b.x, w[5] = b.y, w[6] = b.z, w[7] = b.w;
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j)
            w[j] = j < valid ? __ldcs(p + off + j) : 0.f;
    }
}

template <typename In, int BS_LOG2, int U>
__global__ void __launch_bounds__(kEncThreads) encode_fast_kernel(const __grid_constant__ EncodeBatch b)
{
    extern __shared__ uint2 lut_rep[];
    for (int i = threadIdx.x; i < kNumCells * kEncReplicas; i += kEncThreads)
        lut_rep[i] = g_encode_lut[i / kEncReplicas];
    __syncthreads();

    constexpr int G = (1 << BS_LOG2) / 8; /* lanes per block */
    const uint32_t lane = lane_id();
    const uint2 *lut = lut_rep + (lane & (kEncReplicas - 1));
    const int64_t total = b.chunk_end[b.count - 1];
    const int64_t nwarps = (int64_t)gridDim.x * (kEncThreads / 32);

    for (int64_t g0 = ((int64_t)blockIdx.x * (kEncThreads / 32) + (threadIdx.x >> 5)) * U; g0 < total;
         g0 += nwarps * U) {
        float w[U][8];
        int item[U], valid[U];
        int64_t start[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t g = g0 + u;
            item[u] = 0;
            valid[u] = 0;
            start[u] = 0;
            if (g < total) {
                int it = 0;
                while (b.chunk_end[it] <= g)
                    ++it;
                const int64_t first = it ? b.chunk_end[it - 1] : 0;
                const int64_t s0 = (g - first) * kChunk + 8 * (int64_t)lane;
                const int64_t left = b.n[it] - s0;
                item[u] = it;
                start[u] = s0;
                valid[u] = left >= 8 ? 8 : (left > 0 ? (int)left : 0);
            }
            load8(static_cast<const In *>(b.w[item[u]]), start[u], valid[u], w[u]);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if (g0 + u >= total)
                break; /* uniform over the warp */
            const int it = item[u];
            float a = 0.f;
#pragma unroll
            for (int j = 0; j < 8; ++j)
                a = fmaxf(a, fabsf(w[u][j]));
            const float s = group_max<G>(a);
            if (valid[u] > 0 && (lane & (G - 1)) == 0)
                b.absmax[it][start[u] >> BS_LOG2] = s;
            uint32_t hw = 0, pw = 0;
            if (s >= kMarksteinLo && s <= kMarksteinHi) {
                const float y = __frcp_rn(s);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint32_t c = lut_code(lut, kEncReplicas, quotient_markstein(w[u][j], s, y));
                    hw |= (c >> 4) << (4 * j);
                    pw |= (c & 15u) << (4 * j);
                }
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float v = (s == 0.f) ? 0.f : __fdiv_rn(w[u][j], s);
                    const uint32_t c = lut_code(lut, kEncReplicas, v);
                    hw |= (c >> 4) << (4 * j);
                    pw |= (c & 15u) << (4 * j);
                }
            }
            const int64_t byte0 = start[u] >> 1;
            if (valid[u] == 8) {
                __stcs(reinterpret_cast<uint32_t *>(b.hole[it] + byte0), hw);
                __stcs(reinterpret_cast<uint32_t *>(b.plug[it] + byte0), pw);
            } else if (valid[u] > 0) {
                /* ragged end: nibbles past n stay 0 (the odd-n pad nibble) */
                const uint32_t keep = 0xFFFFFFFFu >> (32 - 4 * valid[u]);
                hw &= keep;
                pw &= keep;
                for (int bb = 0; bb < (valid[u] + 1) / 2; ++bb) {
                    b.hole[it][byte0 + bb] = (uint8_t)(hw >> (8 * bb));
                    b.plug[it][byte0 + bb] = (uint8_t)(pw >> (8 * bb));
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

constexpr int kUnroll = 4;

template <typename In, int BS_LOG2>
int launch_fast_bs(const EncodeBatch &b, cudaStream_t st)
{
    auto kern = encode_fast_kernel<In, BS_LOG2, kUnroll>;
    if (!ensure_smem((const void *)kern, kEncSmem))
        return kLaunch;
    const int64_t total = b.chunk_end[b.count - 1];
    const int64_t warps_needed = (total + kUnroll - 1) / kUnroll;
    const int64_t ctas_needed = (warps_needed + (kEncThreads / 32) - 1) / (kEncThreads / 32);
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(ctas_needed, (int64_t)sm_count() * 3));
    kern<<<grid, kEncThreads, kEncSmem, st>>>(b);
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
        const bool aligned = aligned_to(j.w, 16) && aligned_to(j.hole, 4) && aligned_to(j.plug, 4) &&
                             aligned_to(j.absmax, 4);
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
        b.chunk_end[k] = (k ? b.chunk_end[k - 1] : 0) + (j.n + kChunk - 1) / kChunk;
        b.count = k + 1;
        if (b.count == kMaxItems)
            rc = flush();
    }
    if (rc == kOk)
        rc = flush();
    return rc;
}

} // namespace glint
