/* GLINT expand for sm_100a: hole/plug planes + absmax -> dense BF16 or f32.
 *
 * Reference behaviour: cuda/glint_encode.cu:103-114 (k_expand, f32 out) and
 * glint_unpin._expand / glint_np.expand + f32_to_bf16_bytes (glint_unpin.py:25-31,
 * glint_np.py:25-31, 84-92): out = GLINT_CELLS[h][p] * absmax[i / bs] as one f32
 * multiply, then for BF16 a round to nearest even with the NaN rule
 * (u >> 16) | 0x40.
 *
 * A lane expands 8 weights per step: one 32-bit load from each plane and one
 * 16-byte BF16 store (two for f32), so a warp instruction moves 128 contiguous
 * bytes of each plane and 512 contiguous bytes of output.  The 256-entry f32
 * codebook sits in shared memory with one replica per lane (32 KB), so the
 * per-weight lookups never conflict.  Blocksizes that are a multiple of 8 keep
 * a lane's 8 weights inside one block (one absmax load per 8 weights); other
 * blocksizes and unaligned pointers go through a one-thread-per-weight kernel.
 *
 * NaN absmax: the reference's host expand multiplies on x86, which returns the
 * NaN operand (quietened) unchanged, so the product carries absmax's bits.  The
 * GPU multiply would return its canonical NaN instead; both outputs are
 * produced from absmax's bits here to match the host reference bit for bit.
 */
#include <algorithm>

#include "common.cuh"
#include "glint_internal.h"

namespace glint {
namespace {

constexpr int kExpThreads = 256;
constexpr int kMaxItems = 32;
constexpr int kRow = 256; /* weights per warp row: 32 lanes x 8 */
constexpr int kExpSmem = 256 * 32 * (int)sizeof(float);

struct ExpandBatch {
    const uint8_t *hole[kMaxItems];
    const uint8_t *plug[kMaxItems];
    const float *absmax[kMaxItems];
    void *out[kMaxItems];
    int64_t n[kMaxItems];
    int64_t row_end[kMaxItems]; /* inclusive prefix sum of ceil(n / 256) */
    int count;
    uint32_t bs8; /* blocksize / 8 */
};

__device__ __forceinline__ float quiet_nan_of(float s) { return __uint_as_float(__float_as_uint(s) | 0x00400000u); }

/* values of the 8 weights whose nibbles are in H and P (lo nibble first) */
__device__ __forceinline__ void dequant8(const float *cells, uint32_t H, uint32_t P, float s, float v[8])
{
    /* byte b of E holds the code of element 2b, byte b of O the code of element 2b+1 */
    const uint32_t E = ((H << 4) & 0xF0F0F0F0u) | (P & 0x0F0F0F0Fu);
    const uint32_t O = (H & 0xF0F0F0F0u) | ((P >> 4) & 0x0F0F0F0Fu);
#pragma unroll
    for (int b = 0; b < 4; ++b) {
        v[2 * b] = cells[((E >> (8 * b)) & 0xFFu) * 32] * s;
        v[2 * b + 1] = cells[((O >> (8 * b)) & 0xFFu) * 32] * s;
    }
}

template <int U, bool BF16>
__global__ void __launch_bounds__(kExpThreads) expand_fast_kernel(const __grid_constant__ ExpandBatch b)
{
    extern __shared__ float cells_rep[];
    for (int i = threadIdx.x; i < 256 * 32; i += kExpThreads)
        cells_rep[i] = (&g_cells[0][0])[i >> 5];
    __syncthreads();
    const uint32_t lane = lane_id();
    const float *cells = cells_rep + lane;
    const int64_t total = b.row_end[b.count - 1];
    const int64_t nwarps = (int64_t)gridDim.x * (kExpThreads / 32);

    for (int64_t g0 = ((int64_t)blockIdx.x * (kExpThreads / 32) + (threadIdx.x >> 5)) * U; g0 < total;
         g0 += nwarps * U) {
        uint32_t H[U], P[U];
        float S[U];
        int item[U], valid[U];
        int64_t start[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t g = g0 + u;
            item[u] = 0;
            valid[u] = 0;
            start[u] = 0;
            H[u] = P[u] = 0;
            S[u] = 0.f;
            if (g < total) {
                int it = 0;
                while (b.row_end[it] <= g)
                    ++it;
                const int64_t first = it ? b.row_end[it - 1] : 0;
                const int64_t s0 = (g - first) * kRow + 8 * (int64_t)lane;
                const int64_t left = b.n[it] - s0;
                item[u] = it;
                start[u] = s0;
                valid[u] = left >= 8 ? 8 : (left > 0 ? (int)left : 0);
                if (valid[u] == 8) {
                    H[u] = __ldcs(reinterpret_cast<const uint32_t *>(b.hole[it] + (s0 >> 1)));
                    P[u] = __ldcs(reinterpret_cast<const uint32_t *>(b.plug[it] + (s0 >> 1)));
                } else if (valid[u] > 0) {
                    for (int bb = 0; bb < (valid[u] + 1) / 2; ++bb) {
                        H[u] |= (uint32_t)b.hole[it][(s0 >> 1) + bb] << (8 * bb);
                        P[u] |= (uint32_t)b.plug[it][(s0 >> 1) + bb] << (8 * bb);
                    }
                }
                if (valid[u] > 0)
                    S[u] = __ldg(b.absmax[it] + (uint32_t)(s0 >> 3) / b.bs8);
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if (valid[u] == 0)
                continue;
            float v[8];
            dequant8(cells, H[u], P[u], S[u], v);
            const bool nan_scale = isnan(S[u]);
            if (BF16) {
                uint32_t o[4];
                if (!nan_scale) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        __nv_bfloat162 h2 = __floats2bfloat162_rn(v[2 * q], v[2 * q + 1]);
                        o[q] = *reinterpret_cast<uint32_t *>(&h2);
                    }
                } else {
                    const uint32_t nb = (__float_as_uint(S[u]) >> 16) | 0x40u;
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        o[q] = nb | (nb << 16);
                }
                uint16_t *dst = static_cast<uint16_t *>(b.out[item[u]]) + start[u];
                if (valid[u] == 8) {
                    __stcs(reinterpret_cast<uint4 *>(dst), make_uint4(o[0], o[1], o[2], o[3]));
                } else {
                    for (int j = 0; j < valid[u]; ++j)
                        dst[j] = (uint16_t)(o[j >> 1] >> (16 * (j & 1)));
                }
            } else {
                if (nan_scale) {
                    const float qn = quiet_nan_of(S[u]);
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        v[j] = qn;
                }
                float *dst = static_cast<float *>(b.out[item[u]]) + start[u];
                if (valid[u] == 8) {
                    __stcs(reinterpret_cast<float4 *>(dst), make_float4(v[0], v[1], v[2], v[3]));
                    __stcs(reinterpret_cast<float4 *>(dst + 4), make_float4(v[4], v[5], v[6], v[7]));
                } else {
                    for (int j = 0; j < valid[u]; ++j)
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

constexpr int kUnroll = 4;

template <bool BF16>
int launch_fast(const ExpandBatch &b, cudaStream_t st)
{
    auto kern = expand_fast_kernel<kUnroll, BF16>;
    if (!ensure_smem((const void *)kern, kExpSmem))
        return kLaunch;
    const int64_t total = b.row_end[b.count - 1];
    const int64_t warps_needed = (total + kUnroll - 1) / kUnroll;
    const int64_t ctas_needed = (warps_needed + (kExpThreads / 32) - 1) / (kExpThreads / 32);
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(ctas_needed, (int64_t)sm_count() * 6));
    kern<<<grid, kExpThreads, kExpSmem, st>>>(b);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunch;
}

} // namespace

int expand_launch(const ExpandJob *jobs, int count, int bs, OutKind out, cudaStream_t st)
{
    if (bs <= 0)
        return kBadArg;
    const bool bf16 = out == kOutBF16;
    ExpandBatch b{};
    b.bs8 = (uint32_t)(bs / 8);
    int rc = kOk;
    auto flush = [&]() -> int {
        if (b.count == 0)
            return kOk;
        int r = bf16 ? launch_fast<true>(b, st) : launch_fast<false>(b, st);
        const uint32_t keep = b.bs8;
        b = ExpandBatch{};
        b.bs8 = keep;
        return r;
    };
    for (int i = 0; i < count && rc == kOk; ++i) {
        const ExpandJob &j = jobs[i];
        if (j.n <= 0)
            continue;
        if (!j.hole || !j.plug || !j.absmax || !j.out)
            return kBadArg;
        const bool aligned = aligned_to(j.hole, 4) && aligned_to(j.plug, 4) && aligned_to(j.absmax, 4) &&
                             aligned_to(j.out, 16);
        /* fast path: 8-weight steps inside one block, and (i / 8) fits the 32-bit divide */
        const bool fast = (bs % 8 == 0) && aligned && (j.n >> 3) < (int64_t)0xFFFFFFFF;
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
        b.row_end[k] = (k ? b.row_end[k - 1] : 0) + (j.n + kRow - 1) / kRow;
        b.count = k + 1;
        if (b.count == kMaxItems)
            rc = flush();
    }
    if (rc == kOk)
        rc = flush();
    return rc;
}

} // namespace glint
